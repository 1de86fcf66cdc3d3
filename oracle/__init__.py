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


# ---- MoE expert gather -----------------------------------------------------
# gdsllm/runtime/qwen_moe.py:453-474 (routed experts, decode branch) and
# :497-513 (shared expert).  Expert stacks are (words uint32 [E, rows, cols/8],
# scales f16 [E, rows, cols/g], biases f16) numpy arrays.

def silu_f16(v16: np.ndarray) -> np.ndarray:
    """F.silu on a float16 tensor, the op the reference calls (v / (1 + exp(-v))
    in fp32, rounded to fp16).  Computed by torch on the CPU: the fp32 exp is
    not correctly rounded, and 3 of the 63488 finite halves round to the
    neighbouring fp16 value under numpy's exp."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(v16, np.float16))
    return torch.nn.functional.silu(t).numpy()


def expert_f16(stack, e: int, group: int) -> np.ndarray:
    """Dequantized fp16 matrix of expert e of a stack (C restatement)."""
    w, s, b = stack
    return dequant_affine_q4(np.ascontiguousarray(w[e]), np.ascontiguousarray(s[e]),
                             np.ascontiguousarray(b[e]), group)


def moe_gate_up_exact(x: np.ndarray, ids: np.ndarray, gate, up, group: int,
                      e_first: int = 0):
    """h[t][k] = fp16(silu(fp16(gate x)) * fp16(up x)) with the GEMVs summed in
    fp64 and rounded once (qwen_moe.py:467-469).  Also returns the exact
    fp64 gate and up outputs.  Slots whose expert is outside the stack are
    left as NaN."""
    ntok, top_k = ids.shape
    inter = gate[0].shape[1]
    h = np.full((ntok, top_k, inter), np.nan, np.float16)
    g_ex = np.full((ntok, top_k, inter), np.nan)
    u_ex = np.full((ntok, top_k, inter), np.nan)
    cache = {}
    for t in range(ntok):
        for k in range(top_k):
            z = int(ids[t, k]) - e_first
            if z < 0 or z >= gate[0].shape[0]:
                continue
            if z not in cache:
                cache[z] = (expert_f16(gate, z, group), expert_f16(up, z, group))
            gw, uw = cache[z]
            g = gemv_exact(gw, x[t])[0]
            u = gemv_exact(uw, x[t])[0]
            g_ex[t, k], u_ex[t, k] = g, u
            s = silu_f16(g.astype(np.float16)).astype(np.float32)
            h[t, k] = (s * u.astype(np.float16).astype(np.float32)).astype(np.float16)
    return h, g_ex, u_ex


def moe_down_exact(h: np.ndarray, ids: np.ndarray, route_w: np.ndarray, down, group: int,
                   e_first: int = 0):
    """y[t] = sum over resident slots of w[t][k] * (down_e h[t][k]) in fp64,
    with the bar sum_k |w| * 2e-3 * ||h[t][k]||_2 * max|down_e|."""
    ntok, top_k = ids.shape
    hidden = down[0].shape[1]
    y = np.zeros((ntok, hidden))
    bar = np.zeros(ntok)
    cache = {}
    for t in range(ntok):
        for k in range(top_k):
            z = int(ids[t, k]) - e_first
            if z < 0 or z >= down[0].shape[0]:
                continue
            if z not in cache:
                cache[z] = expert_f16(down, z, group)
            dw = cache[z]
            w = float(np.float16(route_w[t, k]))
            y[t] += w * gemv_exact(dw, h[t, k])[0]
            bar[t] += abs(w) * error_bound(dw, h[t, k])[0]
    return y, bar


def moe_decode_reference(x: np.ndarray, ids: np.ndarray, route_w: np.ndarray, gate, up, down,
                         group: int) -> np.ndarray:
    """moe_mlp_selective's decode arithmetic, one token at a time: fp16 GEMV
    outputs (fp32 accumulation, gemv_cpu), SiLU * up in fp16, and the
    expert_output += w * down_out update in fp16 per slot
    (qwen_moe.py:466-474)."""
    ntok, top_k = ids.shape
    hidden = down[0].shape[1]
    out = np.zeros((ntok, hidden), np.float16)
    for t in range(ntok):
        acc = np.zeros(hidden, np.float16)
        for k in range(top_k):
            e = int(ids[t, k])
            g = gemv_cpu(expert_f16(gate, e, group), x[t])[0]
            u = gemv_cpu(expert_f16(up, e, group), x[t])[0]
            hh = (silu_f16(g).astype(np.float32) * u.astype(np.float32)).astype(np.float16)
            d = gemv_cpu(expert_f16(down, e, group), hh)[0]
            w = np.float16(route_w[t, k])
            prod = (np.float32(w) * d.astype(np.float32)).astype(np.float16)
            acc = (acc.astype(np.float32) + prod.astype(np.float32)).astype(np.float16)
        out[t] = acc
    return out


def moe_mlp_reference(x: np.ndarray, ids: np.ndarray, route_w: np.ndarray, gate, up, down,
                      group: int, shared=None, shared_gate_w: np.ndarray | None = None) -> np.ndarray:
    """moe_mlp_selective's decode result (qwen_moe.py:453-516): the routed sum
    of moe_decode_reference, plus the shared expert (fp16 GEMVs, SiLU * up,
    down) scaled by sigmoid(F.linear(x, shared_gate_w)) in fp16, added in fp16
    and clamped to +-65504.  shared = (gate, up, down) stacks of one expert."""
    import torch
    routed = moe_decode_reference(x, ids, route_w, gate, up, down, group)
    if shared is None:
        return np.clip(routed.astype(np.float32), -65504.0, 65504.0).astype(np.float16)
    sg, su, sd = shared
    out = np.zeros_like(routed)
    for t in range(x.shape[0]):
        g = gemv_cpu(expert_f16(sg, 0, group), x[t])[0]
        u = gemv_cpu(expert_f16(su, 0, group), x[t])[0]
        hh = (silu_f16(g).astype(np.float32) * u.astype(np.float32)).astype(np.float16)
        d = gemv_cpu(expert_f16(sd, 0, group), hh)[0]
        xt = torch.from_numpy(np.ascontiguousarray(x[t], np.float16)).view(1, 1, -1)
        sw = torch.sigmoid(torch.nn.functional.linear(xt, torch.from_numpy(shared_gate_w))).numpy()
        sw = sw.reshape(-1)[0]
        so = (np.float32(sw) * d.astype(np.float32)).astype(np.float16)
        r = (routed[t].astype(np.float32) + so.astype(np.float32)).astype(np.float16)
        out[t] = np.clip(r.astype(np.float32), -65504.0, 65504.0).astype(np.float16)
    return out
