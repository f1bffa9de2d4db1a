"""Construction of online quantized Linear implementations
(``qslab/runtime/backends/__init__.py:3-10``).  ``'gemlite'`` is accepted as an
alias so that a configuration written for the reference selects these kernels."""
from .base import QuantLinear

QUANT_BACKENDS = ('b200', 'gemlite')


def make_quant_linear(backend, values, scale, **kwargs):
    if backend not in QUANT_BACKENDS:
        raise ValueError(f'unknown quantization backend: {backend}')
    from .b200 import B200Linear
    return B200Linear.from_quantized(values, scale, **kwargs)


__all__ = ["QUANT_BACKENDS", "QuantLinear", "make_quant_linear"]
