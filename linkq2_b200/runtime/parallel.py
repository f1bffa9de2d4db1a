"""Tensor parallelism for the Qwen3 layers: one process per GPU, NCCL (or gloo
on CPU) through ``torch.distributed``.

The reference is single-GPU (``qslab/runtime/model/qwen3.py:1-5``); this module
is the split the hot path gains here.  q/k/v/gate/up projections are split over
output columns, o/down over input rows with a sum all-reduce of the ``[M,
hidden]`` activations, KV heads are sharded with the q heads of their group, so
attention itself needs no communication.  Sharding is applied to the
checkpoint's *logical* tensors (``values [N, K]`` and per-group metadata)
before packing, so the on-disk layout is untouched.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


class PeerLeft(RuntimeError):
    """A rank of the tensor-parallel group has announced that it is leaving."""


def _store():
    from torch.distributed.distributed_c10d import _get_default_store
    return _get_default_store()


class PeerExchange:
    """The exchange buffers of ``lq2_allreduce_fp16``: this rank's buffer (allocated
    by the library, shared through CUDA IPC) and the mapped buffers of its peers.

    Built collectively by ``create``; if any rank cannot allocate, export or map a
    buffer (no peer access, IPC unavailable), every rank gets ``None`` and the
    all-reduce stays on NCCL."""

    def __init__(self, rank, world, max_bytes, own, table, pointers):
        self.rank, self.world, self.max_bytes = rank, world, max_bytes
        self._own, self.table, self._pointers = own, table, pointers

    @classmethod
    def create(cls, rank: int, world: int, device, max_bytes: int, group=None) -> "PeerExchange | None":
        import ctypes
        from linkq2_b200 import _lib
        lib = _lib.lib
        pointers, own, ok = [None] * world, ctypes.c_void_p(), True
        handle = ctypes.create_string_buffer(64)
        with torch.cuda.device(device):
            size = lib.lq2_allreduce_buffer_bytes(world, max_bytes)
            ok = size > 0 and lib.lq2_allreduce_buffer_create(size, ctypes.byref(own), handle) == _lib.OK
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle.raw) if ok else None, group=group)
            ok = ok and all(h is not None for h in handles)
            if ok:
                for peer in range(world):
                    if peer == rank:
                        pointers[peer] = own.value
                        continue
                    mapped = ctypes.c_void_p()
                    if lib.lq2_allreduce_buffer_open(handles[peer], ctypes.byref(mapped)) != _lib.OK:
                        ok = False
                        break
                    pointers[peer] = mapped.value
            agreed = [None] * world
            dist.all_gather_object(agreed, bool(ok), group=group)
            if not all(agreed):
                # unmap everywhere first, free afterwards: an exported buffer must outlive
                # every mapping of it in the other processes
                for peer, ptr in enumerate(pointers):
                    if ptr and peer != rank:
                        lib.lq2_allreduce_buffer_close(ptr, 0)
                dist.barrier(group=group)
                if own.value:
                    lib.lq2_allreduce_buffer_close(own.value, 1)
                return None
        table = (ctypes.c_void_p * world)(*pointers)
        exchange = cls(rank, world, max_bytes, own.value, table, pointers)
        exchange.group = group
        return exchange

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        from linkq2_b200 import _lib
        with torch.cuda.device(x.device):
            status = _lib.lib.lq2_allreduce_fp16(x.data_ptr(), x.data_ptr(), x.numel(), self.table, self.rank,
                                                 self.world, self.max_bytes,
                                                 torch.cuda.current_stream().cuda_stream)
        _lib.check(status, "lq2_allreduce_fp16")
        _lib.count()
        return x

    def accepts(self, x: torch.Tensor) -> bool:
        nbytes = x.numel() * x.element_size()
        return (x.dtype == torch.float16 and x.is_cuda and x.is_contiguous() and 0 < nbytes <= self.max_bytes
                and nbytes % 16 == 0 and x.data_ptr() % 16 == 0)

    def timeouts(self) -> int:
        from linkq2_b200 import _lib
        return int(_lib.lib.lq2_allreduce_timeouts())

    def set_poll_limit(self, polls: int) -> int:
        """Polls a thread of the exchange kernels spends waiting for its peers before it gives
        up (``lq2_allreduce_set_poll_limit``; <= 0: the default).  Returns the previous limit."""
        from linkq2_b200 import _lib
        return int(_lib.lib.lq2_allreduce_set_poll_limit(int(polls)))

    def check(self) -> None:
        """Raise if any wait of an exchange kernel on this device has run out: the outputs of
        that launch were invalid (synchronises the device)."""
        n = self.timeouts()
        if n:
            raise RuntimeError(f"tensor-parallel exchange: {n} abandoned waits on rank {self.rank}; "
                               "a peer did not deliver its part and the results are invalid")

    def close(self):
        """Collective.  Two phases with a barrier between them: every rank unmaps its peers'
        buffers, and only when all have done so does each rank free its own (freeing an
        exported allocation that another process still has mapped is undefined)."""
        from linkq2_b200 import _lib
        for peer, ptr in enumerate(self._pointers):
            if ptr and peer != self.rank:
                _lib.lib.lq2_allreduce_buffer_close(ptr, 0)
        self._pointers = []
        if dist.is_available() and dist.is_initialized():
            dist.barrier(group=getattr(self, "group", None))
        if self._own:
            _lib.lib.lq2_allreduce_buffer_close(self._own, 1)
        self._own = None


@dataclass
class TensorParallel:
    rank: int = 0
    size: int = 1
    group: object | None = None
    exchange: PeerExchange | None = None
    push_enabled: bool = True        # LQ2_PEER_PUSH=0: the norm kernel sends the partial sums itself

    def leave(self) -> None:
        """Announce on the process group's store that this rank stops taking part.  Call it
        between steps, with none of this rank's kernels or collectives in flight; the others
        see it in ``guard()`` before their next launch."""
        if self.size > 1 and dist.is_initialized():
            _store().set(f"lq2/left/{self.rank}", b"1")

    def guard(self) -> None:
        """Raise ``PeerLeft`` if a rank has announced its departure.  The runner calls this on
        the host before it issues a step: an exchange kernel launched without its peer would
        only end when its poll budget runs out, with invalid results.  One non-blocking store
        query per peer."""
        if self.size == 1 or not dist.is_initialized():
            return
        store = _store()
        gone = [r for r in range(self.size) if r != self.rank and store.check([f"lq2/left/{r}"])]
        if gone:
            raise PeerLeft(f"rank(s) {gone} left the tensor-parallel group; rank {self.rank} stops before its next step")

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        """Sum over the ranks, in place.  Small fp16 activations go through the
        library's peer-memory kernel, everything else through NCCL / gloo."""
        if self.size > 1:
            if self.exchange is not None and self.exchange.accepts(x):
                return self.exchange.all_reduce(x)
            dist.all_reduce(x, op=dist.ReduceOp.SUM, group=self.group)
        return x

    def reduce_or_defer(self, x: torch.Tensor):
        """``(tensor, deferred)``: a partial sum that the next residual RMSNorm can
        reduce itself (``rmsnorm_allreduce``) is handed on unreduced with ``deferred``
        set; otherwise it is all-reduced here.  The decision depends on shape and
        dtype only, so all ranks take it alike."""
        if self.size > 1 and self.exchange is not None and self.exchange.accepts(x):
            return x, True
        return self.all_reduce(x), False

    def project_reduce_or_defer(self, layer, x: torch.Tensor):
        """``reduce_or_defer(layer(x))`` for a row-split projection, with one more outcome:
        ``deferred == 2`` when the projection kernel itself has pushed its partial sum to the
        peers, so that the following norm only gathers.  Shape-only decision."""
        if self.size > 1 and self.exchange is not None and self.push_enabled:
            from linkq2_b200.kernels.gemlite.ops import can_push
            rows = x.numel() // x.shape[-1]
            if (hasattr(layer, "forward_push") and getattr(layer, "input_scale", None) is None
                    and not getattr(layer, "gate_up_silu", False) and can_push(rows, layer.out_features, self.exchange)):
                return layer.forward_push(x, self.exchange), 2
        y, deferred = self.reduce_or_defer(layer(x))
        return y, int(deferred)

    def check_geometry(self, hidden, intermediate, num_heads, num_kv_heads, group_size):
        t = self.size
        if num_heads % t or num_kv_heads % t:
            raise ValueError(f"tensor-parallel size {t} must divide {num_heads} query and "
                             f"{num_kv_heads} KV heads")
        if intermediate % t or (intermediate // t) % group_size:
            raise ValueError(f"intermediate size {intermediate} / {t} must be a multiple of the "
                             f"quantization group {group_size}")


_TP = TensorParallel()


def get_tp() -> TensorParallel:
    return _TP


def set_tp(tp: TensorParallel) -> None:
    global _TP
    _TP = tp


def init_from_env(backend: str | None = None, peer_exchange_bytes: int = 4 << 20,
                  timeout_s: float | None = None) -> TensorParallel:
    """Join the process group described by RANK / WORLD_SIZE / MASTER_* and make
    the whole world one tensor-parallel group.  On NCCL, all-reduces of fp16
    activations of up to ``peer_exchange_bytes`` (decode and verify steps) use the
    library's own kernel over peer memory when the GPUs can map each other's
    memory; ``LQ2_PEER_ALLREDUCE=0`` keeps everything on NCCL.  ``timeout_s`` is the process
    group's collective timeout: a library collective whose peer never joins ends with an error
    after that long instead of blocking."""
    import os
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1:
        set_tp(TensorParallel())
        return get_tp()
    if not dist.is_initialized():
        backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        kwargs = {}
        if timeout_s is not None:
            import datetime
            kwargs["timeout"] = datetime.timedelta(seconds=timeout_s)
        if backend == "nccl":
            kwargs["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend=backend, **kwargs)
    tp = TensorParallel(dist.get_rank(), dist.get_world_size(), None)
    if (dist.get_backend() == "nccl" and tp.size <= 8 and peer_exchange_bytes > 0
            and os.environ.get("LQ2_PEER_ALLREDUCE", "1") != "0"):
        device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        tp.exchange = PeerExchange.create(tp.rank, tp.size, device, peer_exchange_bytes)
        tp.push_enabled = os.environ.get("LQ2_PEER_PUSH", "1") != "0"
    set_tp(tp)
    return get_tp()


def shutdown():
    """Orderly end of a multi-rank run: every rank reaches this point, then the
    process group is destroyed.  Captured CUDA graphs that contain collectives must
    have been released before (``ModelRunner.shutdown``)."""
    if dist.is_available() and dist.is_initialized():
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        dist.barrier()
        if get_tp().exchange is not None:
            get_tp().exchange.close()
            dist.barrier()
        dist.destroy_process_group()
    set_tp(TensorParallel())


# ---- sharding of logical quantized tensors ---------------------------------
COLUMN, ROW = "column", "row"


def shard_quantized(data: dict, kind: str, tp: TensorParallel, group_size: int) -> dict:
    """Slice one projection's logical tensors for this rank.

    ``data``: ``values [N, K]``, ``scale [N, K/G]``, ``zero_point [N, K/G] | None``,
    ``input_scale [K] | None``.  ``column`` keeps rows ``[r*N/t, (r+1)*N/t)`` of
    every tensor (output channels); ``row`` keeps input channels
    ``[r*K/t, (r+1)*K/t)``, i.e. whole quantization groups, and the matching
    slice of ``input_scale``.
    """
    if tp.size == 1:
        return data
    n, k = data["values"].shape
    t, r = tp.size, tp.rank
    out = dict(data)
    if kind == COLUMN:
        if n % t:
            raise ValueError(f"cannot split {n} output channels over {t} ranks")
        sl = slice(r * n // t, (r + 1) * n // t)
        out["values"] = data["values"][sl].contiguous()
        out["scale"] = data["scale"][sl].contiguous()
        if data.get("zero_point") is not None:
            out["zero_point"] = data["zero_point"][sl].contiguous()
    elif kind == ROW:
        if k % t or (k // t) % group_size:
            raise ValueError(f"cannot split {k} input channels over {t} ranks in groups of {group_size}")
        ks = slice(r * k // t, (r + 1) * k // t)
        gs = slice(r * k // t // group_size, (r + 1) * k // t // group_size)
        out["values"] = data["values"][:, ks].contiguous()
        out["scale"] = data["scale"][:, gs].contiguous()
        if data.get("zero_point") is not None:
            out["zero_point"] = data["zero_point"][:, gs].contiguous()
        if data.get("input_scale") is not None:
            out["input_scale"] = data["input_scale"][ks].contiguous()
    else:
        raise ValueError(kind)
    return out


def shard_dense(weight: torch.Tensor, kind: str, tp: TensorParallel) -> torch.Tensor:
    """Same split for an unquantized ``[N, K]`` weight."""
    if tp.size == 1:
        return weight
    n, k = weight.shape
    t, r = tp.size, tp.rank
    if kind == COLUMN:
        return weight[r * n // t:(r + 1) * n // t].contiguous()
    return weight[:, r * k // t:(r + 1) * k // t].contiguous()
