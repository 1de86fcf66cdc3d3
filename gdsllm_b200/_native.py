"""Loads the in-tree native libraries.  There is no fallback: if the CUDA
library or the binding is missing, importing them raises."""
from __future__ import annotations

import ctypes
import importlib.util
import sys

from .build import EXT_PATH, LIB_PATH

_lib = None
_ext = None

_C_SIGNATURES = {
    "gdsq_version": (ctypes.c_int, []),
    "gdsq_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "gdsq_last_error": (ctypes.c_char_p, []),
    "gdsq_device_error": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "gdsq_set_pdl": (ctypes.c_int, [ctypes.c_int]),
    "gdsq_set_peer_wait_limit_ns": (ctypes.c_ulonglong, [ctypes.c_ulonglong]),
    "gdsq_dequant_q4_0": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]),
    "gdsq_dequant_q8_0": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]),
    "gdsq_dequant_rows_gguf": (ctypes.c_int, [ctypes.c_int, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int,
                                              ctypes.c_void_p, ctypes.c_longlong, ctypes.c_void_p, ctypes.c_void_p]),
    "gdsq_dequant_affine_q4": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_void_p]),
    "gdsq_fused_q4_0_gemv": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "gdsq_fused_q8_0_gemv": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "gdsq_fused_affine_q4_gemv": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                 ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                                 ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_void_p]),
    "gdsq_moe_affine_q4_gate_up": (ctypes.c_int, [ctypes.c_void_p] * 15 + [ctypes.c_int] * 8
                                   + [ctypes.c_void_p]),
    "gdsq_moe_affine_q4_down": (ctypes.c_int, [ctypes.c_void_p] * 11 + [ctypes.c_int] * 9
                                + [ctypes.c_void_p]),
    "gdsq_fused_gemv_group": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                                             ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_void_p),
                                             ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "gdsq_moe_affine_q4_noalloc": (ctypes.c_int, [ctypes.c_void_p] * 23 + [ctypes.c_int] * 9 + [ctypes.c_void_p]),
    "gdsq_allreduce_sum_f16": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                              ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "gdsq_allreduce_sum_words": (ctypes.c_int, [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                                ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "gdsq_fused_gemv_allreduce": (ctypes.c_int, [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                                 ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                                                 ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_int, ctypes.c_void_p]),
    "gdsq_moe_route": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                      ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.c_void_p, ctypes.c_void_p]),
    "gdsq_add_rmsnorm_f16": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                            ctypes.c_void_p]),
    "gdsq_rope_kv_f16": (ctypes.c_int, [ctypes.c_void_p] * 8 + [ctypes.c_int] * 4 + [ctypes.c_void_p]),
    "gdsq_attention_decode_f16": (ctypes.c_int, [ctypes.c_void_p] * 5 + [ctypes.c_int] * 4 +
                                  [ctypes.c_float, ctypes.c_void_p]),
    "gdsq_attention_decode_rope_f16": (ctypes.c_int, [ctypes.c_void_p] * 8 + [ctypes.c_int] * 4 +
                                       [ctypes.c_float, ctypes.c_void_p]),
    "gdsq_allreduce_sum_words_residual": (ctypes.c_int, [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                                         ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                                                         ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                         ctypes.c_void_p, ctypes.c_void_p]),
    "gdsq_moe_affine_q4_down_residual": (ctypes.c_int, [ctypes.c_void_p] * 6 + [ctypes.c_void_p] * 5 +
                                         [ctypes.c_int] * 9 + [ctypes.c_void_p, ctypes.c_void_p]),
    "gdsq_moe_router": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_int] + [ctypes.c_void_p] * 6),
    "gdsq_silu_mul_f16": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong,
                                         ctypes.c_void_p]),
    "gdsq_argmax_f16": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p]),
}


def _missing(path) -> ImportError:
    return ImportError(
        f"gdsllm_b200 native code not found at {path}; build it with "
        "`python -m gdsllm_b200.build` (there is no CPU fallback)")


def lib() -> ctypes.CDLL:
    """The C-ABI library (include/gdsq.h) with argument types declared."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise _missing(LIB_PATH)
        handle = ctypes.CDLL(str(LIB_PATH), mode=ctypes.RTLD_GLOBAL)
        for name, (restype, argtypes) in _C_SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


def ext():
    """The gds_io_ext torch binding (same op API as gdsllm.runtime.gds_io_ext)."""
    global _ext
    if _ext is None:
        import torch  # noqa: F401  (loads libtorch / libcudart before the binding)

        lib()  # libgdsq.so must be resident: the binding links against it
        if not EXT_PATH.exists():
            raise _missing(EXT_PATH)
        spec = importlib.util.spec_from_file_location("gds_io_ext", EXT_PATH)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        sys.modules.setdefault("gdsllm_b200.gds_io_ext", mod)
        _ext = mod
    return _ext


class GdsqError(RuntimeError):
    pass


def check(status: int, what: str = "gdsq") -> None:
    """Raises GdsqError for a non-zero status from a C-ABI call."""
    if status != 0:
        l = lib()
        detail = l.gdsq_last_error().decode()
        raise GdsqError(f"{what}: {l.gdsq_status_string(status).decode()} ({detail})")
