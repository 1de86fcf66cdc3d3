"""Drop-in replacements for the reference scheduler's embedding and lm_head
helpers, which dequantize the whole vocabulary table on every call.

GdsLLM's ``_embed_tokens`` and ``_lm_head_proj`` (gdsllm/runtime/
scheduler.py:22-69; the MoE scheduler's copies at qwen_moe_scheduler.py:
28-53) turn a GGUF table into a full fp16 matrix before ``F.embedding`` /
``F.linear``: for LLaMA-7B's 32000 x 4096 Q8_0 lm_head that is 139 MB read,
262 MB written and 262 MB read again per decode token.  The functions here
keep the same signatures and results:

* ``embed_tokens``: a GGUF table goes through ``gds_io_ext.embedding_gguf``,
  which dequantizes only the looked-up rows (the same bits as dequant +
  F.embedding); INT8 and fp16 tables behave exactly as the reference.
* ``lm_head_proj``: a GGUF head with at most 16 positions (decode) goes
  through the fused dequant-GEMV (``fused_dequant_gemv`` on [B, K] inputs,
  fp32 accumulation); prefill and other weight types take the reference's
  path.

``install(module)`` puts them into a scheduler module (the reference's
``gdsllm.runtime.scheduler`` or ``qwen_moe_scheduler``), which then calls
them unchanged.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ._native import ext

_MAX_FUSED_ROWS = 16  # the fused GEMV's batch limit


def _is_gguf(w) -> bool:
    return isinstance(w, dict) and "gguf_type" in w


def _is_affine(w) -> bool:
    return isinstance(w, dict) and w.get("quant_type") == "affine_q4"


def _affine_dequant(w, scratch):
    return ext().dequant_affine_q4(w["buffer"], list(w["shape"]), w["weight_offset"], w["scale_offset"],
                                   w["bias_offset"], w["group_size"], scratch)


def embed_tokens(token_ids, tensors, scratch=None):
    """Same contract as gdsllm/runtime/scheduler.py:_embed_tokens (and, for
    affine-Q4 tables, qwen_moe_scheduler.py:_embed_tokens, whose full-table
    dequantization it keeps)."""
    w = tensors["model.embed_tokens.weight"]
    if _is_affine(w):
        return F.embedding(token_ids, _affine_dequant(w, scratch))
    if _is_gguf(w):
        ids = token_ids.to(device=torch.device("cuda", w["buffer"].device_id), dtype=torch.long)
        return ext().embedding_gguf(w["buffer"], ids, list(w["shape"]), w["gguf_type"], w["offset"])
    if w.dtype == torch.int8:
        scale = tensors["model.embed_tokens.scale"]
        rows = F.embedding(token_ids, w)
        return (rows.float() * scale).half()
    return F.embedding(token_ids, w)


def lm_head_proj(h, tensors, key="lm_head.weight", scratch=None):
    """Same contract as gdsllm/runtime/scheduler.py:_lm_head_proj (and
    qwen_moe_scheduler.py:_lm_head_proj for affine-Q4 heads)."""
    w = tensors[key]
    if _is_affine(w):
        n, k = int(w["shape"][0]), int(w["shape"][1])
        rows = h.numel() // k
        if h.shape[-1] == k and 1 <= rows <= _MAX_FUSED_ROWS and h.dtype == torch.float16:
            y = ext().fused_affine_q4_gemv(w["buffer"], h.reshape(rows, k), [n, k], w["weight_offset"],
                                           w["scale_offset"], w["bias_offset"], w["group_size"])
            return y.view(*h.shape[:-1], n)
        return F.linear(h, _affine_dequant(w, scratch))
    if _is_gguf(w):
        n, k = int(w["shape"][0]), int(w["shape"][1])
        rows = h.numel() // k
        if h.shape[-1] == k and 1 <= rows <= _MAX_FUSED_ROWS and h.dtype == torch.float16:
            y = ext().fused_dequant_gemv(w["buffer"], h.reshape(rows, k), [n, k], w["gguf_type"], w["offset"])
            return y.view(*h.shape[:-1], n)
        wd = ext().dequant_gguf(w["buffer"], list(w["shape"]), w["gguf_type"], w["offset"], scratch)
        return F.linear(h, wd)
    if w.dtype == torch.int8:
        scale = tensors[key.rsplit(".weight", 1)[0] + ".scale"]
        if w.shape[0] * w.shape[1] * 4 > 512 * 1024 * 1024:
            chunks = []
            for i in range(0, w.shape[0], 16384):
                chunks.append(F.linear(h, (w[i:i + 16384].float() * scale).half()))
            return torch.cat(chunks, dim=-1)
        return F.linear(h, (w.float() * scale).half())
    return F.linear(h, w)


def install(module) -> None:
    """Replaces ``module._embed_tokens`` and ``module._lm_head_proj`` (when
    present) with the functions above."""
    if hasattr(module, "_embed_tokens"):
        module._embed_tokens = embed_tokens
    if hasattr(module, "_lm_head_proj"):
        module._lm_head_proj = lm_head_proj
