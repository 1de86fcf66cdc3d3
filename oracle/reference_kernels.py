"""TEST INFRASTRUCTURE ONLY.  ctypes access to GdsLLM's own CUDA kernels,
compiled unchanged from the reference tree into oracle/_ref/libref_kernels.so
by oracle/build.py (see ref_shim.cu).  Used by GPU parity tests, the golden
vector recorder and the reference leg of bench.py.  Batch 1 only, as in the
reference."""
from __future__ import annotations

import ctypes

from .build import REF_LIB

_lib = None


def available() -> bool:
    return REF_LIB.exists()


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not REF_LIB.exists():
            raise FileNotFoundError(f"{REF_LIB} is not built (python oracle/build.py, needs the reference tree)")
        l = ctypes.CDLL(str(REF_LIB))
        vp, i, u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64
        sig = {
            "ref_fused_q4_0_gemv": [vp, vp, vp, i, i, vp],
            "ref_fused_q8_0_gemv": [vp, vp, vp, i, i, vp],
            "ref_fused_affine_q4_gemv": [vp, vp, vp, vp, vp, i, i, i, vp],
            "ref_dequant_q4_0": [vp, vp, u64, vp],
            "ref_dequant_q8_0": [vp, vp, u64, vp],
            "ref_dequant_affine_q4": [vp, vp, vp, vp, u64, i, i, vp],
        }
        for name, args in sig.items():
            fn = getattr(l, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        _lib = l
    return _lib


def _check(err: int, what: str) -> None:
    if err != 0:
        raise RuntimeError(f"reference kernel {what}: cudaError {err}")


def _stream(t):
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream


def gemv_q4_0(w, x, n, k, out):
    _check(lib().ref_fused_q4_0_gemv(w.data_ptr(), x.data_ptr(), out.data_ptr(), n, k, _stream(x)), "q4_0 gemv")
    return out


def gemv_q8_0(w, x, n, k, out):
    _check(lib().ref_fused_q8_0_gemv(w.data_ptr(), x.data_ptr(), out.data_ptr(), n, k, _stream(x)), "q8_0 gemv")
    return out


def gemv_affine_q4(words, scales, biases, x, n, k, group, out):
    _check(lib().ref_fused_affine_q4_gemv(words.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                                          x.data_ptr(), out.data_ptr(), n, k, group, _stream(x)),
           "affine gemv")
    return out


def dequant_q4_0(raw, out):
    _check(lib().ref_dequant_q4_0(raw.data_ptr(), out.data_ptr(), raw.numel() // 18, _stream(raw)), "q4_0 dequant")
    return out


def dequant_q8_0(raw, out):
    _check(lib().ref_dequant_q8_0(raw.data_ptr(), out.data_ptr(), raw.numel() // 34, _stream(raw)), "q8_0 dequant")
    return out


def dequant_affine_q4(words, scales, biases, in_dim, group, out):
    _check(lib().ref_dequant_affine_q4(words.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                                       out.data_ptr(), words.numel() * 8, in_dim, group, _stream(words)),
           "affine dequant")
    return out
