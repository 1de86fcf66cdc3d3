"""TEST INFRASTRUCTURE ONLY.  A stand-in for the reference's ``gds_io_ext``
module whose compute ops run GdsLLM's own CUDA kernels (compiled unchanged
into oracle/_ref by oracle/build.py, called through oracle.reference_kernels)
with the reference binding's semantics (gdsllm/runtime/gds_bindings.cpp:
255-512): the same op names and arguments, the same output shapes, the
``dequant_gguf`` / ``dequant_affine_q4`` scratch-view rule, batch-1 fused
GEMVs that check ``x.numel() == in_dim``.

Loads (``load_file``, ``load_file_region``, ``load_expert``, ``load_tensor``)
read the file with plain host I/O and copy it to the GPU: the GPU pool has no
GPUDirect Storage stack, so the reference's cuFile path cannot run there.
Register it under ``gdsllm.runtime.gds_io_ext`` (``install``) to run the
reference's Python callers (llama.py, scheduler.py, qwen_moe.py) unchanged
on the reference kernels, for comparison with this build's module.
"""
from __future__ import annotations

import sys

import numpy as np
import torch

from . import reference_kernels as refk

_DTYPES = {"float16": torch.float16, "half": torch.float16, "float32": torch.float32, "float": torch.float32,
           "bfloat16": torch.bfloat16, "int8": torch.int8, "int32": torch.int32, "int": torch.int32}


class GdsBufferHandle:
    """A CUDA byte buffer (4 KB-rounded, as gds_io.cu allocates)."""

    def __init__(self, size_bytes: int, device_id: int):
        self._size = int(size_bytes)
        self._t = torch.zeros((self._size + 4095) // 4096 * 4096, dtype=torch.uint8,
                              device=torch.device("cuda", device_id))

    @property
    def size(self) -> int:
        return self._size

    @property
    def device_id(self) -> int:
        return self._t.device.index

    @property
    def registered(self) -> bool:
        return False

    def bytes(self, offset: int, nbytes: int) -> torch.Tensor:
        if offset < 0 or offset + nbytes > self._t.numel():
            raise RuntimeError(f"offset {offset} + {nbytes} bytes outside the buffer")
        return self._t[offset:offset + nbytes]


def init() -> None:
    pass


def shutdown() -> None:
    pass


def is_driver_open() -> bool:
    return False


def _read(h: GdsBufferHandle, path: str, size: int, file_offset: int, buf_offset: int, what: str) -> None:
    data = np.fromfile(path, dtype=np.uint8, count=size, offset=file_offset)
    if data.size < size:
        raise RuntimeError(f"{what}: expected {size} bytes, got {data.size}")
    h.bytes(buf_offset, size).copy_(torch.from_numpy(data))


def load_file(filepath: str, size_bytes: int, device_id: int = 0) -> GdsBufferHandle:
    h = GdsBufferHandle(size_bytes, device_id)
    _read(h, filepath, size_bytes, 0, 0, "py_load_file")
    return h


def load_file_region(filepath: str, size_bytes: int, file_offset: int, device_id: int = 0) -> GdsBufferHandle:
    h = GdsBufferHandle(size_bytes, device_id)
    _read(h, filepath, size_bytes, file_offset, 0, "py_load_file_region")
    return h


def load_expert(filepath, w_file_offset, w_size, s_file_offset, s_size, b_file_offset, b_size, device_id=0):
    h = GdsBufferHandle(w_size + s_size + b_size, device_id)
    _read(h, filepath, w_size, w_file_offset, 0, "py_load_expert")
    _read(h, filepath, s_size, s_file_offset, w_size, "py_load_expert")
    _read(h, filepath, b_size, b_file_offset, w_size + s_size, "py_load_expert")
    return h, 0, w_size, w_size + s_size


def view_tensor(handle: GdsBufferHandle, shape, dtype: str, offset: int) -> torch.Tensor:
    dt = _DTYPES[dtype]
    n = int(np.prod(shape)) if len(shape) else 1
    nbytes = n * torch.empty(0, dtype=dt).element_size()
    return handle.bytes(offset, nbytes).view(dt).view(list(shape))


def load_tensor(filepath, shape, dtype="float16", file_offset=0, size_bytes=0, device_id=0):
    h = load_file_region(filepath, size_bytes, file_offset, device_id)
    t = view_tensor(h, shape, dtype, 0)
    t._gds_handle = h  # keeps the buffer alive with the view
    return t


def _output(output, shape, numel, device, what):
    if output is None:
        return torch.empty(list(shape), dtype=torch.float16, device=device)
    if output.numel() < numel:
        raise RuntimeError(f"{what}: scratch buffer too small ({output.numel()} < {numel})")
    return output.flatten()[:numel].view(list(shape))


def dequant_gguf(handle, shape, gguf_type, offset, output=None):
    numel = int(np.prod(shape))
    if numel % 32:
        raise RuntimeError("py_dequant_gguf: total elements must be a multiple of 32 (block size)")
    bb = {"q4_0": 18, "q8_0": 34}.get(gguf_type)
    if bb is None:
        raise RuntimeError(f"py_dequant_gguf: unsupported type '{gguf_type}'")
    out = _output(output, shape, numel, handle._t.device, "py_dequant_gguf")
    raw = handle.bytes(offset, numel // 32 * bb)
    (refk.dequant_q4_0 if gguf_type == "q4_0" else refk.dequant_q8_0)(raw, out)
    return out


def fused_dequant_gemv(handle, x, weight_shape, gguf_type, offset):
    n, k = int(weight_shape[0]), int(weight_shape[1])
    if k % 32:
        raise RuntimeError("py_fused_dequant_gemv: in_dim must be a multiple of 32")
    if x.numel() != k:
        raise RuntimeError(f"py_fused_dequant_gemv: x has {x.numel()} elements, expected in_dim={k}")
    bb = {"q4_0": 18, "q8_0": 34}.get(gguf_type)
    if bb is None:
        raise RuntimeError(f"py_fused_dequant_gemv: unsupported type '{gguf_type}'")
    raw = handle.bytes(offset, n * (k // 32) * bb)
    xc = x.contiguous()
    out = torch.empty(1, n, dtype=torch.float16, device=handle._t.device)
    (refk.gemv_q4_0 if gguf_type == "q4_0" else refk.gemv_q8_0)(raw, xc, n, k, out)
    return out


def _affine_parts(handle, n, k, weight_offset, scale_offset, bias_offset, group_size):
    words = handle.bytes(weight_offset, n * k // 2).view(torch.int32)
    scales = handle.bytes(scale_offset, n * (k // group_size) * 2).view(torch.float16)
    biases = handle.bytes(bias_offset, n * (k // group_size) * 2).view(torch.float16)
    return words, scales, biases


def dequant_affine_q4(handle, weight_shape, weight_offset, scale_offset, bias_offset, group_size, output=None):
    k = int(weight_shape[-1])
    numel = int(np.prod(weight_shape))
    out = _output(output, weight_shape, numel, handle._t.device, "py_dequant_affine_q4")
    w, s, b = _affine_parts(handle, numel // k, k, weight_offset, scale_offset, bias_offset, group_size)
    refk.dequant_affine_q4(w, s, b, k, group_size, out)
    return out


def fused_affine_q4_gemv(handle, x, weight_shape, weight_offset, scale_offset, bias_offset, group_size):
    n, k = int(weight_shape[0]), int(weight_shape[1])
    if x.numel() != k:
        raise RuntimeError(f"py_fused_affine_q4_gemv: x has {x.numel()} elements, expected in_dim={k}")
    w, s, b = _affine_parts(handle, n, k, weight_offset, scale_offset, bias_offset, group_size)
    out = torch.empty(1, n, dtype=torch.float16, device=handle._t.device)
    refk.gemv_affine_q4(w, s, b, x.contiguous(), n, k, group_size, out)
    return out


def install(name: str = "gdsllm.runtime.gds_io_ext"):
    """Registers this module under the reference's import name."""
    mod = sys.modules[__name__]
    sys.modules[name] = mod
    parent_name, _, attr = name.rpartition(".")
    parent = sys.modules.get(parent_name)
    if parent is not None:
        setattr(parent, attr, mod)
    return mod
