"""ctypes binding of ``liblinkq2_b200.so`` (the C ABI in ``include/linkq2_b200.h``).

The library is the only compute path of this package: importing this module
raises when the shared object is missing instead of falling back to anything
else.  Build it with ``python -m linkq2_b200.build``.
"""
from __future__ import annotations

import ctypes
from ctypes import c_char_p, c_float, c_int, c_int64, c_size_t, c_uint, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "liblinkq2_b200.so"

OK = 0
ERR_ARG, ERR_SHAPE, ERR_ALIGN, ERR_WORKSPACE, ERR_CUDA, ERR_LIMIT = 1, 2, 3, 4, 5, 6

# name -> (restype, argtypes); mirrors include/linkq2_b200.h one to one
SIGNATURES = {
    "lq2_status_string": (c_char_p, [c_int]),
    "lq2_abi_version": (c_int, []),
    "lq2_w4_pack": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_void_p]),
    "lq2_w4a16_set_constant_weights": (c_int, [c_int]),
    "lq2_allreduce_buffer_bytes": (c_size_t, [c_int, c_size_t]),
    "lq2_allreduce_buffer_create": (c_int, [c_size_t, c_void_p, c_void_p]),
    "lq2_allreduce_buffer_open": (c_int, [c_void_p, c_void_p]),
    "lq2_allreduce_buffer_close": (c_int, [c_void_p, c_int]),
    "lq2_allreduce_fp16": (c_int, [c_void_p, c_void_p, c_int64, c_void_p, c_int, c_int, c_size_t, c_void_p]),
    "lq2_rmsnorm_allreduce": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                      c_float, c_void_p, c_int, c_int, c_size_t, c_void_p]),
    "lq2_rmsnorm_allreduce_pushed": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                             c_float, c_void_p, c_int, c_int, c_size_t, c_void_p]),
    "lq2_w4a16_linear_push": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                      c_int, c_void_p, c_int, c_int, c_size_t, c_void_p]),
    "lq2_allreduce_timeouts": (c_uint, []),
    "lq2_allreduce_set_poll_limit": (ctypes.c_longlong, [ctypes.c_longlong]),
    "lq2_w4a16_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "lq2_w4a16_linear": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                 c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lq2_w4a16_gate_up_silu": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                       c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lq2_kv4_store": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                              c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int64, c_void_p]),
    "lq2_kv4_store_f32": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int64, c_void_p]),
    "lq2_kv4_attention_splits": (c_int, [c_int] * 7),
    "lq2_kv4_attention_workspace_bytes": (c_size_t, [c_int] * 7),
    "lq2_kv4_attention": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                  c_int, c_int64, c_void_p, c_size_t, c_void_p]),
    "lq2_kv4_attention_prefix": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                         c_int, c_int, c_int64, c_void_p, c_size_t, c_void_p]),
    "lq2_chunk_attention": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_void_p,
                                    c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "lq2_kv4_attention_static": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                         c_int, c_int, c_int64, c_void_p]),
    "lq2_kv4_attention_static_max_bytes": (c_size_t, []),
    "lq2_rmsnorm": (c_int, [c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p]),
    "lq2_silu_mul": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int, c_int, c_void_p]),
    "lq2_pre_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int64,
                                  c_float, c_void_p]),
    "lq2_stage_decode": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                 c_int, c_void_p]),
    "lq2_kv4_materialize": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_int, c_int, c_int, c_int, c_int64, c_void_p]),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: the CUDA library has not been built. "
            "Run `python -m linkq2_b200.build` (needs nvcc); there is no fallback path.")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)           # AttributeError if the symbol is not exported
        fn.restype, fn.argtypes = restype, argtypes
    return lib


lib = _load()

# Number of kernels of this library enqueued by this process (a launch captured
# into a CUDA graph counts once at capture and once more per replay, which the
# graph runner adds through ``count``).
launches = 0


def count(n: int = 1) -> None:
    global launches
    launches += n


class LinkQ2Error(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {lib.lq2_status_string(status).decode()} (status {status})")


def check(status: int, where: str) -> None:
    """Map a non-zero status to the exception type the reference would raise:
    shape problems are ``ValueError`` (``runtime/backends/gemlite.py:17-18``)."""
    if status == OK:
        return
    if status == ERR_SHAPE:
        raise ValueError(f"{where}: {lib.lq2_status_string(status).decode()}")
    raise LinkQ2Error(status, where)
