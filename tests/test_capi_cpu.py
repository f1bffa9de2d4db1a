"""The C-ABI library without a GPU: it loads, exports every symbol the header
declares, and rejects bad arguments before anything is launched."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    from linkq2_b200 import build
    build.build()
    from linkq2_b200 import _lib
    return _lib


def test_every_declared_symbol_is_exported_and_bound(lib):
    header = (ROOT / "include" / "linkq2_b200.h").read_text()
    declared = set(re.findall(r"\b(lq2_[a-z0-9_]+)\s*\(", header))
    assert declared, "no declarations found"
    raw = ctypes.CDLL(str(lib.LIB_PATH))
    for name in declared:
        assert hasattr(raw, name), f"{name} is declared but not exported"
    assert declared == set(lib.SIGNATURES), "ctypes table and header disagree"


def test_header_cites_the_reference_for_every_operator():
    header = (ROOT / "include" / "linkq2_b200.h").read_text()
    for path in ("qslab/kernels/gemlite/ops.py", "qslab/kernels/gemlite/bitpack.py",
                 "qslab/kernels/kv4/store.py", "qslab/kernels/kv4/paged_attention.py",
                 "qslab/kernels/kv4/grouped_attention.py", "qslab/kernels/kv4/layout.py"):
        assert path in header


def test_status_strings_and_version(lib):
    assert lib.lib.lq2_abi_version() >= 1
    assert lib.lib.lq2_status_string(0) == b"ok"
    assert b"align" in lib.lib.lq2_status_string(lib.ERR_ALIGN)


def test_argument_validation_launches_nothing(lib):
    L = lib.lib
    fake = 1 << 20          # an aligned, never dereferenced address
    assert L.lq2_w4_pack(None, 8, fake, 64, 64, None) == lib.ERR_ARG
    assert L.lq2_w4_pack(fake, 8, fake, 64, 60, None) == lib.ERR_SHAPE
    assert L.lq2_w4_pack(fake, 3, fake, 64, 64, None) == lib.ERR_SHAPE
    # N % 32, group not a power of two, group < 32, K % group
    for n, k, group in ((48, 256, 128), (64, 256, 96), (64, 256, 16), (64, 320, 128)):
        assert L.lq2_w4a16_linear(fake, k, fake, fake, None, fake, 1, n, k, group, fake, 1 << 30, None) == lib.ERR_SHAPE
    assert L.lq2_w4a16_linear(fake + 2, 256, fake, fake, None, fake, 1, 64, 256, 128, fake, 1 << 30, None) == lib.ERR_ALIGN
    assert L.lq2_w4a16_linear(fake, 256, fake, fake, None, None, 1, 64, 256, 128, fake, 1 << 30, None) == lib.ERR_ARG
    assert L.lq2_kv4_store(fake, fake, 1024, 1024, fake, fake, fake, fake, fake, 4, 8, 128, 48, 1024, None) == lib.ERR_SHAPE
    assert L.lq2_kv4_store(fake, fake, 1024, 1024, fake, fake, fake, fake, fake, 0, 8, 128, 64, 1024, None) == lib.OK
    # verify_m * HQ/HKV > 64, D not in {64, 128}, page % 16
    assert L.lq2_kv4_attention(fake, 4096, fake, fake, fake, fake, fake, fake, fake, 1, 32, 32, 8, 128, 256, 4, 64,
                               1024, fake, 1 << 30, None) == lib.ERR_SHAPE
    assert L.lq2_kv4_attention_workspace_bytes(1, 1, 32, 8, 96, 256, 4) == 0
    assert L.lq2_kv4_attention_workspace_bytes(1, 1, 32, 8, 128, 250, 4) == 0
    assert L.lq2_kv4_attention(fake, 4096, fake, fake, fake, fake, fake, fake, fake, 2, 1, 32, 8, 128, 256, 4, 64,
                               1024, fake, 16, None) == lib.ERR_WORKSPACE
    assert L.lq2_kv4_materialize(fake, fake, fake, fake, fake, fake, fake, 0, 8, 128, 64, 1024, None) == lib.OK
    assert L.lq2_kv4_materialize(fake, fake, fake, fake, fake, fake + 2, fake, 3, 8, 128, 64, 1024, None) == lib.ERR_ALIGN


def test_split_and_workspace_sizes_depend_on_shapes_only(lib):
    L = lib.lib
    a = L.lq2_kv4_attention_splits(1, 1, 32, 8, 128, 256, 128)
    assert a == L.lq2_kv4_attention_splits(1, 1, 32, 8, 128, 256, 128) and a >= 1
    assert L.lq2_kv4_attention_splits(64, 1, 32, 8, 128, 256, 128) >= 1
    assert L.lq2_kv4_attention_workspace_bytes(8, 16, 32, 8, 128, 256, 16) > 0
    assert L.lq2_w4a16_workspace_bytes(1, 4096, 4096) == L.lq2_w4a16_workspace_bytes(1, 4096, 4096)
    assert L.lq2_w4a16_workspace_bytes(0, 4096, 4096) == 0


def test_python_wrappers_refuse_cpu_tensors(lib):
    import torch
    from linkq2_b200.kernels.gemlite.ops import linear
    meta = (4, 128, 15, 8, 1, 1, 0, 1, 0, 3, True, 104)
    with pytest.raises(RuntimeError):
        linear(torch.zeros(1, 256, dtype=torch.float16), torch.zeros(32, 64, dtype=torch.int32),
               torch.zeros(2, 64, dtype=torch.float16), torch.tensor(8, dtype=torch.int32), meta)
    with pytest.raises(TypeError):
        linear(torch.zeros(1, 256), torch.zeros(32, 64, dtype=torch.int32),
               torch.zeros(2, 64, dtype=torch.float16), torch.tensor(8, dtype=torch.int32), meta)
