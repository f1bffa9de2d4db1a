"""KV4 cache operators with the signatures of ``qslab.kernels.kv4``
(``qslab/kernels/kv4/__init__.py:2-6``)."""
from .ops import materialize_kv, paged_attention_decode, store_kv_quant

__all__ = ["materialize_kv", "paged_attention_decode", "store_kv_quant"]
