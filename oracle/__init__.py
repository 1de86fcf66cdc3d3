"""TEST INFRASTRUCTURE ONLY — the parity oracle for gdsllm_b200.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs use this package, and only as the checker (or as the timed CPU path of
the reference), never as a product code path.

Contents
* C restatement of GdsLLM's dequantization formulas (gdsq_oracle.c, with
  file:line citations there), loaded with ctypes:
  ``dequant_q4_0``, ``dequant_q8_0``, ``dequant_affine_q4``.
* An independent numpy restatement of the same formulas (``np_dequant_*``),
  used to cross-check the C code.
* The reference's CPU GEMV path: dequantize with the formula, then
  ``torch.matmul`` in fp32 and round to fp16 (``gemv_cpu``), plus an fp64
  version used as the exact value (``gemv_exact``).
* ``error_bound``: the GEMV tolerance 2e-3 * ||x||_2 * max|W| per batch row.

Parity is pinned by tests/golden/ fixtures: the third-party ``gguf`` 0.19.0
package's Q4_0 / Q8_0 dequantizer, and outputs of the reference's own CUDA
kernels (oracle/_ref, compiled unchanged from the reference tree) recorded on
a B200.
"""
from __future__ import annotations

import ctypes

import numpy as np

from .build import ORACLE_LIB, build_oracle

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_LIB.exists():
            build_oracle()
        l = ctypes.CDLL(str(ORACLE_LIB))
        vp, u64 = ctypes.c_void_p, ctypes.c_uint64
        l.gdsq_oracle_dequant_q4_0.argtypes = [vp, vp, u64]
        l.gdsq_oracle_dequant_q8_0.argtypes = [vp, vp, u64]
        l.gdsq_oracle_dequant_affine_q4.argtypes = [vp, vp, vp, vp, u64, ctypes.c_int]
        l.gdsq_oracle_halves_to_floats.argtypes = [vp, vp, u64]
        l.gdsq_oracle_floats_to_halves.argtypes = [vp, vp, u64]
        l.gdsq_oracle_num_threads.restype = ctypes.c_int
        for n in ("gdsq_oracle_dequant_q4_0", "gdsq_oracle_dequant_q8_0",
                  "gdsq_oracle_dequant_affine_q4", "gdsq_oracle_halves_to_floats",
                  "gdsq_oracle_floats_to_halves"):
            getattr(l, n).restype = None
        _lib = l
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def num_threads() -> int:
    return lib().gdsq_oracle_num_threads()


# ---- C restatement ---------------------------------------------------------

def dequant_q4_0(raw: np.ndarray) -> np.ndarray:
    """raw: uint8 bytes of n Q4_0 blocks (18 B each) -> float16[n*32]."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    assert raw.size % 18 == 0
    n = raw.size // 18
    out = np.empty(n * 32, dtype=np.float16)
    lib().gdsq_oracle_dequant_q4_0(_ptr(raw), _ptr(out), n)
    return out


def dequant_q8_0(raw: np.ndarray) -> np.ndarray:
    """raw: uint8 bytes of n Q8_0 blocks (34 B each) -> float16[n*32]."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    assert raw.size % 34 == 0
    n = raw.size // 34
    out = np.empty(n * 32, dtype=np.float16)
    lib().gdsq_oracle_dequant_q8_0(_ptr(raw), _ptr(out), n)
    return out


def dequant_affine_q4(words: np.ndarray, scales: np.ndarray, biases: np.ndarray,
                      group_size: int) -> np.ndarray:
    """words: uint32 [..., K/8]; scales, biases: float16 [..., K/group] -> float16 [..., K]."""
    w = np.ascontiguousarray(words).view(np.uint32)
    s = np.ascontiguousarray(scales, dtype=np.float16)
    b = np.ascontiguousarray(biases, dtype=np.float16)
    n = w.size * 8
    assert s.size * group_size == n and b.size == s.size
    out = np.empty(n, dtype=np.float16)
    lib().gdsq_oracle_dequant_affine_q4(_ptr(w), _ptr(s), _ptr(b), _ptr(out), n, group_size)
    return out.reshape(*w.shape[:-1], w.shape[-1] * 8)


def halves_to_floats(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h).view(np.uint16).reshape(-1)
    f = np.empty(h.size, dtype=np.float32)
    lib().gdsq_oracle_halves_to_floats(_ptr(h), _ptr(f), h.size)
    return f


def floats_to_halves(f: np.ndarray) -> np.ndarray:
    f = np.ascontiguousarray(f, dtype=np.float32).reshape(-1)
    h = np.empty(f.size, dtype=np.uint16)
    lib().gdsq_oracle_floats_to_halves(_ptr(f), _ptr(h), f.size)
    return h.view(np.float16)


# ---- numpy restatement (independent cross-check) ----------------------------

def np_dequant_q4_0(raw: np.ndarray) -> np.ndarray:
    blk = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1, 18)
    d = blk[:, :2].copy().view(np.float16).astype(np.float32)          # [n,1]
    qs = blk[:, 2:]
    lo = (qs & 0x0F).astype(np.int32) - 8
    hi = (qs >> 4).astype(np.int32) - 8
    q = np.concatenate([lo, hi], axis=1).astype(np.float32)           # [n,32]
    return (d * q).astype(np.float16).reshape(-1)


def np_dequant_q8_0(raw: np.ndarray) -> np.ndarray:
    blk = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1, 34)
    d = blk[:, :2].copy().view(np.float16).astype(np.float32)
    qs = blk[:, 2:].copy().view(np.int8).astype(np.float32)
    return (d * qs).astype(np.float16).reshape(-1)


def np_dequant_affine_q4(words: np.ndarray, scales: np.ndarray, biases: np.ndarray,
                         group_size: int) -> np.ndarray:
    w = np.ascontiguousarray(words).view(np.uint32).reshape(-1)
    shifts = np.arange(8, dtype=np.uint32) * 4
    nib = ((w[:, None] >> shifts) & 0xF).reshape(-1).astype(np.float64)
    s = np.repeat(np.asarray(scales, np.float16).reshape(-1).astype(np.float64), group_size)
    b = np.repeat(np.asarray(biases, np.float16).reshape(-1).astype(np.float64), group_size)
    # The product of an fp16 scale and a 4-bit integer is exact in fp64, so
    # the fp64 sum rounded once to fp32 equals fmaf(nibble, scale, bias).
    return (nib * s + b).astype(np.float32).astype(np.float16)


# ---- GEMV ------------------------------------------------------------------

def gemv_cpu(w_f16: np.ndarray, x_f16: np.ndarray):
    """The reference's CPU path: dequantized fp16 weights, torch.matmul in
    fp32, fp16 output.  w: [N,K], x: [B,K] -> [B,N] float16."""
    import torch
    w = torch.from_numpy(np.ascontiguousarray(w_f16)).float()
    x = torch.from_numpy(np.ascontiguousarray(x_f16).reshape(-1, w.shape[1])).float()
    return torch.matmul(x, w.t()).half().numpy()


def gemv_exact(w_f16: np.ndarray, x_f16: np.ndarray) -> np.ndarray:
    """fp64 accumulation of the same product (the 'true' value)."""
    w = np.asarray(w_f16, np.float64)
    x = np.asarray(x_f16, np.float64).reshape(-1, w.shape[1])
    return x @ w.T


def error_bound(w_f16: np.ndarray, x_f16: np.ndarray) -> np.ndarray:
    """Per batch row: 2e-3 * ||x||_2 * max|W| (the GEMV parity bar)."""
    w = np.asarray(w_f16, np.float64)
    x = np.asarray(x_f16, np.float64).reshape(-1, w.shape[1])
    return 2e-3 * np.linalg.norm(x, axis=1) * np.abs(w).max()
