"""Stand-in for the two ``accelerate`` functions the LinkQ2 reference imports
(``qslab/runtime/execute/model_runner.py:4``, ``qslab/runtime/quantization.py:5``); the
package itself is not in this image.  ``install()`` registers it as ``accelerate`` /
``accelerate.utils`` unless the real package is importable.  Import ``transformers``
first: its optional-dependency probe must not find a version-less ``accelerate``."""
from __future__ import annotations

import sys
import types
from contextlib import contextmanager

import torch
from torch import nn


@contextmanager
def init_empty_weights(include_buffers: bool = False):
    """Parameters registered inside the block live on the meta device (buffers are left
    where they are created unless ``include_buffers``)."""
    reg_param, reg_buf = nn.Module.register_parameter, nn.Module.register_buffer

    def register_parameter(module, name, param):
        reg_param(module, name, param)
        if param is not None:
            old = module._parameters[name]
            new = nn.Parameter(old.detach().to("meta"), requires_grad=old.requires_grad)
            new.__dict__.update(old.__dict__)
            module._parameters[name] = new

    def register_buffer(module, name, tensor, persistent=True):
        reg_buf(module, name, tensor, persistent=persistent)
        if tensor is not None:
            module._buffers[name] = module._buffers[name].to("meta")

    nn.Module.register_parameter = register_parameter
    if include_buffers:
        nn.Module.register_buffer = register_buffer
    try:
        yield
    finally:
        nn.Module.register_parameter, nn.Module.register_buffer = reg_param, reg_buf


def set_module_tensor_to_device(module, tensor_name, device, value=None, dtype=None, **_):
    """Replace parameter or buffer ``tensor_name`` (dotted path) by ``value`` on ``device``."""
    if "." in tensor_name:
        parent, tensor_name = tensor_name.rsplit(".", 1)
        module = module.get_submodule(parent)
    if value is None:
        raise ValueError("this stand-in only loads given values")
    cast = dtype if (dtype is not None and value.is_floating_point()) else None
    new = value.to(device=device, dtype=cast)
    if tensor_name in module._buffers:
        module._buffers[tensor_name] = new
        return
    old = module._parameters.get(tensor_name)
    param = nn.Parameter(new, requires_grad=False)
    if old is not None:
        param.__dict__.update(old.__dict__)
    module._parameters[tensor_name] = param


def install() -> bool:
    """True when the stand-in was registered, False when the real package exists."""
    import importlib.util
    if "accelerate" in sys.modules:
        return False
    try:
        if importlib.util.find_spec("accelerate") is not None:
            return False
    except (ImportError, ValueError):
        pass
    import transformers  # noqa: F401  (before the version-less module appears)
    pkg = types.ModuleType("accelerate")
    utils = types.ModuleType("accelerate.utils")
    pkg.init_empty_weights = init_empty_weights
    utils.set_module_tensor_to_device = set_module_tensor_to_device
    pkg.utils = utils
    pkg.__path__ = []
    sys.modules["accelerate"], sys.modules["accelerate.utils"] = pkg, utils
    return True
