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


@dataclass
class TensorParallel:
    rank: int = 0
    size: int = 1
    group: object | None = None

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            dist.all_reduce(x, op=dist.ReduceOp.SUM, group=self.group)
        return x

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


def init_from_env(backend: str | None = None) -> TensorParallel:
    """Join the process group described by RANK / WORLD_SIZE / MASTER_* and make
    the whole world one tensor-parallel group."""
    import os
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1:
        set_tp(TensorParallel())
        return get_tp()
    if not dist.is_initialized():
        backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        kwargs = {}
        if backend == "nccl":
            kwargs["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend=backend, **kwargs)
    set_tp(TensorParallel(dist.get_rank(), dist.get_world_size(), None))
    return get_tp()


def shutdown():
    """Orderly end of a multi-rank run: every rank reaches this point, then the
    process group is destroyed.  Captured CUDA graphs that contain collectives must
    have been released before (``ModelRunner.shutdown``)."""
    if dist.is_available() and dist.is_initialized():
        if torch.cuda.is_available():
            torch.cuda.synchronize()
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
