"""Thin torch-tensor front end to the C ABI (include/gdsq.h), via ctypes.

Every function launches on the current CUDA stream of the tensors' device
and raises ``GdsqError`` for a non-OK status.  Outputs are allocated unless
``out`` is given (then they are written in place and returned).
"""
from __future__ import annotations

import ctypes

import torch

from ._native import check, lib


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _out(out, shape, like):
    if out is None:
        return torch.empty(shape, dtype=torch.float16, device=like.device)
    return out


def set_pdl(enable: bool) -> None:
    check(lib().gdsq_set_pdl(1 if enable else 0), "gdsq_set_pdl")


def device_error(device: int = 0, clear: bool = True) -> int:
    bits = ctypes.c_int(0)
    check(lib().gdsq_device_error(device, 1 if clear else 0, ctypes.byref(bits)), "gdsq_device_error")
    return bits.value


def dequant_q4_0(raw: torch.Tensor, num_blocks: int | None = None, out=None) -> torch.Tensor:
    n = raw.numel() // 18 if num_blocks is None else num_blocks
    out = _out(out, (n * 32,), raw)
    check(lib().gdsq_dequant_q4_0(_p(raw), _p(out), n, _stream(raw)), "gdsq_dequant_q4_0")
    return out


def dequant_q8_0(raw: torch.Tensor, num_blocks: int | None = None, out=None) -> torch.Tensor:
    n = raw.numel() // 34 if num_blocks is None else num_blocks
    out = _out(out, (n * 32,), raw)
    check(lib().gdsq_dequant_q8_0(_p(raw), _p(out), n, _stream(raw)), "gdsq_dequant_q8_0")
    return out


def dequant_affine_q4(words, scales, biases, in_dim: int, group: int, out=None) -> torch.Tensor:
    n = words.numel() * 8
    out = _out(out, (n,), words)
    check(lib().gdsq_dequant_affine_q4(_p(words), _p(scales), _p(biases), _p(out), n, in_dim, group,
                                       _stream(words)), "gdsq_dequant_affine_q4")
    return out


def gemv_q4_0(w: torch.Tensor, x: torch.Tensor, n: int, k: int, out=None) -> torch.Tensor:
    b = x.numel() // k
    out = _out(out, (b, n), x)
    check(lib().gdsq_fused_q4_0_gemv(_p(w), _p(x), _p(out), n, k, b, _stream(x)), "gdsq_fused_q4_0_gemv")
    return out


def gemv_q8_0(w: torch.Tensor, x: torch.Tensor, n: int, k: int, out=None) -> torch.Tensor:
    b = x.numel() // k
    out = _out(out, (b, n), x)
    check(lib().gdsq_fused_q8_0_gemv(_p(w), _p(x), _p(out), n, k, b, _stream(x)), "gdsq_fused_q8_0_gemv")
    return out


def gemv_affine_q4(words, scales, biases, x: torch.Tensor, n: int, k: int, group: int,
                   out=None) -> torch.Tensor:
    b = x.numel() // k
    out = _out(out, (b, n), x)
    check(lib().gdsq_fused_affine_q4_gemv(_p(words), _p(scales), _p(biases), _p(x), _p(out), n, k,
                                          group, b, _stream(x)), "gdsq_fused_affine_q4_gemv")
    return out


def gemv_group(fmt: str, weights, x: torch.Tensor, out_dims, k: int, outs=None):
    """Several GGUF matrices sharing x (and K) in one launch:
    [y_m [B, out_dims[m]]] = W_m . x."""
    b = x.numel() // k
    count = len(weights)
    if outs is None:
        outs = [torch.empty(b, n, dtype=torch.float16, device=x.device) for n in out_dims]
    wa = (ctypes.c_void_p * count)(*[w.data_ptr() for w in weights])
    ya = (ctypes.c_void_p * count)(*[y.data_ptr() for y in outs])
    na = (ctypes.c_int * count)(*out_dims)
    check(lib().gdsq_fused_gemv_group(0 if fmt == "q4_0" else 1, count, wa, na, ya, _p(x), k, b, _stream(x)),
          "gdsq_fused_gemv_group")
    return outs


MOE_OUT_F32 = 1      # GDSQ_MOE_OUT_F32
MOE_ACCUMULATE = 2   # GDSQ_MOE_ACCUMULATE
MOE_CLAMP = 4        # GDSQ_MOE_CLAMP


def _shared_ptrs(shared, n):
    if shared is None:
        return [None] * n
    return [t.data_ptr() for m in shared for t in m]


def moe_gate_up(gate, up, x: torch.Tensor, ids: torch.Tensor, group: int, expert_first: int = 0,
                expert_total: int | None = None, out=None, shared=None) -> torch.Tensor:
    """h [ntok, top_k (+1 with shared), inter] = fp16(silu(gate_e x) * up_e x).
    gate / up: (words int32 [E, inter, hidden/8], scales, biases); ids int32
    [ntok, top_k]; shared = (shared gate stack, shared up stack) with E = 1."""
    gw, gs, gb = gate
    uw, us, ub = up
    e, inter, hidden = gw.shape[0], gw.shape[1], gw.shape[2] * 8
    ntok, top_k = ids.shape
    total = expert_first + e if expert_total is None else expert_total
    if out is None:
        out = torch.empty((ntok, top_k + (shared is not None), inter), dtype=torch.float16, device=x.device)
    check(lib().gdsq_moe_affine_q4_gate_up(_p(gw), _p(gs), _p(gb), _p(uw), _p(us), _p(ub), *_shared_ptrs(shared, 6),
                                           _p(x), _p(ids), _p(out), ntok, top_k, inter, hidden, group, expert_first,
                                           e, total, _stream(x)), "gdsq_moe_affine_q4_gate_up")
    return out


def moe_down(down, h: torch.Tensor, ids: torch.Tensor, route: torch.Tensor, group: int,
             expert_first: int = 0, expert_total: int | None = None, out=None, flags: int = 0,
             shared=None, shared_weights=None) -> torch.Tensor:
    """y [ntok, hidden] = sum_k route[:, k] * down_e h[:, k] (+ shared_weights *
    shared_down h[:, top_k]) in fp32.  down: (words int32 [E, hidden, inter/8],
    scales, biases); route fp16 [ntok, top_k]; shared = the shared down stack."""
    dw, ds, db = down
    e, hidden, inter = dw.shape[0], dw.shape[1], dw.shape[2] * 8
    ntok, top_k = ids.shape
    total = expert_first + e if expert_total is None else expert_total
    if out is None:
        dt = torch.float32 if flags & MOE_OUT_F32 else torch.float16
        out = torch.empty((ntok, hidden), dtype=dt, device=h.device)
    sh = [None] * 3 if shared is None else [t.data_ptr() for t in shared]
    check(lib().gdsq_moe_affine_q4_down(_p(dw), _p(ds), _p(db), *sh, _p(h), _p(ids), _p(route),
                                        _p(shared_weights), _p(out), ntok, top_k, hidden, inter, group,
                                        expert_first, e, total, flags, _stream(h)), "gdsq_moe_affine_q4_down")
    return out


def moe_route(logits: torch.Tensor, top_k: int, x: torch.Tensor | None = None,
              shared_gate: torch.Tensor | None = None):
    """(ids int32 [ntok, k], weights fp16 [ntok, k], shared weight fp16 [ntok] or
    None) from router logits fp16 [ntok, E] -- moe_route's top-k / softmax
    tail, plus sigmoid(x . shared_gate)."""
    ntok, e = logits.shape
    ids = torch.empty(ntok, top_k, dtype=torch.int32, device=logits.device)
    w = torch.empty(ntok, top_k, dtype=torch.float16, device=logits.device)
    sw = None if shared_gate is None else torch.empty(ntok, dtype=torch.float16, device=logits.device)
    hidden = 0 if x is None else x.shape[-1]
    check(lib().gdsq_moe_route(_p(logits), ntok, e, top_k, _p(x), _p(shared_gate), hidden, _p(ids), _p(w), _p(sw),
                               _stream(logits)), "gdsq_moe_route")
    return ids, w, sw


# ---- decode step (batch 1, position in device memory) ----------------------

def add_rmsnorm(h: torch.Tensor, weight: torch.Tensor, eps: float, delta: torch.Tensor | None = None,
                h_out: torch.Tensor | None = None, out=None) -> torch.Tensor:
    """h_out = h + delta (when delta is given; h_out defaults to h, in place),
    then rms_norm(h_out) * weight (llama.py:17-23) into `out`."""
    hidden = weight.numel()
    rows = h.numel() // hidden
    out = _out(out, h.shape, h)
    if delta is not None and h_out is None:
        h_out = h
    check(lib().gdsq_add_rmsnorm_f16(_p(h), _p(delta), _p(h_out), _p(weight), _p(out), rows, hidden, float(eps),
                                     _stream(h)), "gdsq_add_rmsnorm_f16")
    return out


def rope_kv(q, k, v, q_out, freqs: torch.Tensor, pos: torch.Tensor, k_cache, v_cache, num_heads: int,
            num_kv_heads: int, head_dim: int, max_seq: int) -> torch.Tensor:
    """RoPE of q into q_out and of k into k_cache[:, *pos], v into
    v_cache[:, *pos]; freqs is view_as_real(freqs_cis) (fp32 pairs)."""
    check(lib().gdsq_rope_kv_f16(_p(q), _p(k), _p(v), _p(q_out), _p(freqs), _p(pos), _p(k_cache), _p(v_cache),
                                 num_heads, num_kv_heads, head_dim, max_seq, _stream(q)), "gdsq_rope_kv_f16")
    return q_out


def attention_scale(head_dim: int) -> float:
    """The fp32 factor torch multiplies by for `scores / head_dim ** 0.5`."""
    import numpy as np
    return float(np.float32(1.0) / np.float32(head_dim ** 0.5))


def attention_decode(q, k_cache, v_cache, pos: torch.Tensor, num_heads: int, num_kv_heads: int, head_dim: int,
                     max_seq: int, out=None) -> torch.Tensor:
    out = _out(out, (num_heads * head_dim,), q)
    check(lib().gdsq_attention_decode_f16(_p(q), _p(k_cache), _p(v_cache), _p(pos), _p(out), num_heads,
                                          num_kv_heads, head_dim, max_seq, attention_scale(head_dim), _stream(q)),
          "gdsq_attention_decode_f16")
    return out


def attention_decode_rope(q, k, v, freqs: torch.Tensor, pos: torch.Tensor, k_cache, v_cache, num_heads: int,
                          num_kv_heads: int, head_dim: int, max_seq: int, out=None) -> torch.Tensor:
    """attention_decode with the RoPE of q and k and the cache write of k
    and v at *pos folded in (q, k, v before RoPE)."""
    out = _out(out, (num_heads * head_dim,), q)
    check(lib().gdsq_attention_decode_rope_f16(_p(q), _p(k), _p(v), _p(freqs), _p(pos), _p(k_cache), _p(v_cache),
                                               _p(out), num_heads, num_kv_heads, head_dim, max_seq,
                                               attention_scale(head_dim), _stream(q)),
          "gdsq_attention_decode_rope_f16")
    return out


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out=None) -> torch.Tensor:
    out = _out(out, gate.shape, gate)
    check(lib().gdsq_silu_mul_f16(_p(gate), _p(up), _p(out), gate.numel(), _stream(gate)), "gdsq_silu_mul_f16")
    return out


def argmax(logits: torch.Tensor, token: torch.Tensor, pos: torch.Tensor | None = None) -> torch.Tensor:
    """token[0] = first index of the largest logit; pos[0] += 1 if given."""
    check(lib().gdsq_argmax_f16(_p(logits), logits.numel(), _p(token), _p(pos), _stream(logits)), "gdsq_argmax_f16")
    return token


def dequant_rows(fmt: str, table: torch.Tensor, rows: int, cols: int, ids: torch.Tensor, out=None) -> torch.Tensor:
    """fp16 [len(ids), cols]: the GGUF table rows `ids` (int64, on the device),
    dequantized; an id outside [0, rows) gives a zero row and device error
    bit 4."""
    out = _out(out, (ids.numel(), cols), table)
    check(lib().gdsq_dequant_rows_gguf(0 if fmt == "q4_0" else 1, _p(table), rows, cols, _p(ids), ids.numel(),
                                       _p(out), _stream(table)), "gdsq_dequant_rows_gguf")
    return out

