"""pytest plugin that performs, at run time, the rebinding a maintainer of the reference
would commit to use this library (a backend registration and three rebound names), so that the
reference's own, unmodified tests exercise the sm_100a kernels:

  * ``qslab.runtime.backends``: ``'b200'`` joins ``QUANT_BACKENDS`` and
    ``make_quant_linear`` builds a ``B200Linear`` for it.  The reference's tests and its
    ``Config`` default ask for ``'gemlite'`` by name; with ``LINKQ2_DROPIN_GEMLITE=1`` that
    name is served by ``B200Linear`` too, which is what lets those tests run unchanged.
  * ``qslab.kernels.kv4``: ``store_kv_quant``, ``paged_attention_decode`` and
    ``materialize_kv`` are bound to ``linkq2_b200.kernels.kv4`` before any test module or
    ``qslab.runtime.model.attention`` imports them by name.

    python -m pytest -p baseline.dropin_plugin baseline/_ref/reference_tests/kernels ...

Without ``LINKQ2_DROPIN=1`` the plugin only installs the ``accelerate`` stand-in and the
reference runs on its own Triton kernels.  ``LINKQ2_HF_COMPAT=1`` additionally presents a
``transformers`` 5.x model config under the 4.57 attribute names the reference reads
(``hf_compat``); the reference pins 4.57.6 and the image has 5.5.
"""
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
for p in (str(HERE / "_ref"), str(HERE.parent)):
    if p not in sys.path:
        sys.path.insert(0, p)


def rebind(serve_gemlite: bool = False) -> None:
    import qslab.kernels.kv4 as ref_kv4
    import qslab.runtime.backends as ref_backends
    from linkq2_b200.kernels import kv4 as ours
    from linkq2_b200.runtime.backends.b200 import B200Linear

    ref_kv4.store_kv_quant = ours.store_kv_quant
    ref_kv4.paged_attention_decode = ours.paged_attention_decode
    ref_kv4.materialize_kv = ours.materialize_kv
    attention = sys.modules.get("qslab.runtime.model.attention")
    if attention is not None:                   # already imported: rebind its copies of the names
        attention.store_kv_quant = ours.store_kv_quant
        attention.paged_attention_decode = ours.paged_attention_decode
        attention.materialize_kv = ours.materialize_kv

    # a backend committed inside qslab would derive from qslab's QuantLinear; from outside,
    # B200Linear joins that ABC as a registered subclass (same three methods, same buffers)
    from qslab.runtime.backends.base import QuantLinear as RefQuantLinear
    RefQuantLinear.register(B200Linear)

    stock = ref_backends.make_quant_linear
    ref_backends.QUANT_BACKENDS = ("gemlite", "b200")

    def make_quant_linear(backend, values, scale, **kwargs):
        if backend == "b200" or (serve_gemlite and backend == "gemlite"):
            return B200Linear.from_quantized(values, scale, **kwargs)
        return stock(backend, values, scale, **kwargs)

    ref_backends.make_quant_linear = make_quant_linear
    quantization = sys.modules.get("qslab.runtime.quantization")
    if quantization is not None:
        quantization.make_quant_linear = make_quant_linear


def hf_compat() -> None:
    """``transformers`` 5 keeps RoPE settings in ``config.rope_parameters`` and aliases
    ``rope_scaling`` to that dict, which the reference (written against 4.57.6) takes for an
    unknown scaling request (``qslab/runtime/model/rotary.py:66-72``; it reads ``rope_theta``
    and ``rope_scaling`` at ``qslab/runtime/model/qwen3.py:78-79``).  Configs loaded by the
    reference's ``Config`` get the 4.57 view back: ``rope_theta`` a float, ``rope_scaling``
    ``None`` for the default RoPE type."""
    import qslab.runtime.config as ref_config
    stock = ref_config.AutoConfig.from_pretrained

    def view(cfg):
        params = getattr(cfg, "rope_parameters", None)
        if not isinstance(params, dict) or "rope_theta" in cfg.__dict__:
            return cfg
        scaling = None if params.get("rope_type", "default") == "default" else \
            {k: v for k, v in params.items() if k != "rope_theta"}
        cfg.__class__ = type("Compat" + type(cfg).__name__, (type(cfg),), {
            "rope_theta": property(lambda self: float(self.rope_parameters["rope_theta"])),
            "rope_scaling": property(lambda self: scaling)})
        return cfg

    class _AutoConfig:
        @staticmethod
        def from_pretrained(*args, **kwargs):
            return view(stock(*args, **kwargs))

    ref_config.AutoConfig = _AutoConfig


def pytest_configure(config):
    from baseline import accelerate_stub
    accelerate_stub.install()
    if os.environ.get("LINKQ2_HF_COMPAT") == "1":
        hf_compat()
    if os.environ.get("LINKQ2_DROPIN") == "1":
        rebind(serve_gemlite=os.environ.get("LINKQ2_DROPIN_GEMLITE") == "1")
