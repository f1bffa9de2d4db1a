"""Stream order under programmatic dependent launch.

Every kernel of the library may be scheduled while its predecessor on the stream
is still draining.  A chain of dependent kernels (norm -> linear -> SiLU*up ->
linear, each reading what the one before wrote, buffers reused between
iterations) must therefore give exactly the bytes it gives when the host waits
for the device after every call — eagerly, inside a CUDA graph, and with the
weights declared constant (early weight fetch) or not."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _layers(hidden, inter, seed):
    from linkq2_b200.runtime.backends import make_quant_linear
    g = torch.Generator().manual_seed(seed)

    def one(n, k):
        vals = (torch.randint(0, 16, (n, k), generator=g, dtype=torch.uint8).to(torch.int16) - 8).to(torch.int8)
        scale = (torch.rand(n, k // 128, generator=g) * 0.004 + 0.001).half()
        return make_quant_linear("b200", vals, scale, group_size=128, symmetric=True, device="cuda",
                                 dtype=torch.float16)
    return one(2 * inter, hidden), one(hidden, inter)


def _chain(x, w, gate_up, down, inter, rounds, sync):
    from linkq2_b200.kernels.fused import rmsnorm, silu_mul
    outs = []
    h = x
    for _ in range(rounds):
        n = rmsnorm(h, w, 1e-6)
        gu = gate_up(n)
        a = silu_mul(gu[:, :inter], gu[:, inter:])
        h = down(a)
        if sync:
            torch.cuda.synchronize()
        outs.append(h)
    return torch.stack(outs)


@pytest.mark.parametrize("rows", [1, 32])
@pytest.mark.parametrize("constant_weights", [False, True])
def test_dependent_chain_equals_synchronised_execution(rows, constant_weights):
    from linkq2_b200.kernels.gemlite.ops import set_constant_weights
    hidden, inter, rounds = 1024, 3072, 12
    gate_up, down = _layers(hidden, inter, seed=rows)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(rows, hidden, generator=g).half().cuda()
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).half().cuda()
    torch.cuda.synchronize()
    previous = set_constant_weights(constant_weights)
    try:
        expected = _chain(x, w, gate_up, down, inter, rounds, sync=True)
        assert torch.isfinite(expected).all() and expected.abs().max() > 0
        for _ in range(3):
            got = _chain(x, w, gate_up, down, inter, rounds, sync=False)
            torch.cuda.synchronize()
            assert torch.equal(got, expected)
        side = torch.cuda.Stream()
        with torch.cuda.stream(side):
            _chain(x, w, gate_up, down, inter, rounds, sync=False)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                captured = _chain(x, w, gate_up, down, inter, rounds, sync=False)
            for _ in range(3):
                captured.zero_()
                graph.replay()
                torch.cuda.synchronize()
                assert torch.equal(captured, expected)
    finally:
        set_constant_weights(previous)


def test_constant_weights_switch_returns_previous_setting():
    from linkq2_b200.kernels.gemlite.ops import set_constant_weights
    first = set_constant_weights(True)
    assert set_constant_weights(False) is True
    assert set_constant_weights(first) is False
