"""gdsllm_b200: a B200-native (sm_100a) rebuild of GdsLLM's decode hot path,
fused dequantize + GEMV over GGUF Q4_0 / Q8_0 and affine-Q4 weights.

* ``gdsllm_b200.ext()`` returns the ``gds_io_ext`` module: the same Python op
  API as the reference's ``gdsllm.runtime.gds_io_ext``.
* ``gdsllm_b200.install_as_reference_module()`` registers it under the
  reference's import name so that GdsLLM's llama.py / qwen_moe.py /
  schedulers use these kernels unchanged.
* ``gdsllm_b200.capi`` calls the C ABI (include/gdsq.h) on torch tensors.
"""
from __future__ import annotations

import sys

from ._native import GdsqError, check, ext, lib

__all__ = ["ext", "lib", "check", "GdsqError", "install_as_reference_module"]


def install_as_reference_module(name: str = "gdsllm.runtime.gds_io_ext"):
    """Makes ``from gdsllm.runtime import gds_io_ext`` resolve to this build.

    GdsLLM imports the extension lazily inside its functions
    (gdsllm/runtime/llama.py:115,133; qwen_moe.py:30,47;
    torch_bridge.py:115), so registering the module before the first call is
    enough.  Returns the module.
    """
    mod = ext()
    sys.modules[name] = mod
    parent_name, _, attr = name.rpartition(".")
    parent = sys.modules.get(parent_name)
    if parent is not None:
        setattr(parent, attr, mod)
    return mod
