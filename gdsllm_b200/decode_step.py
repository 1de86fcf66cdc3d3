"""One greedy LLaMA decode position as a single CUDA graph.

GdsLLM's decode loop runs ``CachedScheduler.forward`` once per token
(gdsllm/runtime/scheduler.py:304-386).  That is about a thousand eager torch
launches per token, a host-side KV position (kv_cache.py:57-67), the layer
cache's VRAM bookkeeping (scheduler.py:353,372 -> torch_bridge.py:546,567) and
a full dequantization of the lm_head table (scheduler.py:46-69).  At batch 1
the GPU waits on the host for most of the token.

``GraphDecodeStep`` keeps the scheduler's model (the layer dicts, norms,
embedding, lm_head and ``freqs_cis``) and the reference ``KVCache``
tensors, but holds the input token and the position in device memory, so one
token is a fixed sequence of launches.  The sequence is captured once and
replayed per token:

    embedding row gather (fp16 table: index_select; GGUF: dequant of the row)
    per layer:
        add_rmsnorm   (residual add of the previous MLP output + input norm)
        q/k/v         one grouped fused dequant-GEMV launch
        attention     RoPE of q and k and the K/V write at the position folded
                      in; positions split over a thread-block cluster
        o             fused dequant-GEMV
        add_rmsnorm   (residual add of the attention output + post norm)
        gate/up       one grouped fused dequant-GEMV launch
        silu_mul
        down          fused dequant-GEMV
    add_rmsnorm (last residual + final norm), lm_head fused GEMV,
    argmax -> next token in device memory, position + 1,
    and a copy of the token to pinned host memory.

Each op follows the arithmetic of the torch code it replaces
(gdsllm/runtime/llama.py:17-23, 83-105, 228-293).  Attention over the
positions [0, pos] is the same softmax as the reference's over its
``[:end]`` slice.  The GEMVs accumulate in fp32 like the reference's
kernels.  Results agree with ``CachedScheduler.forward`` within the GEMV
error bars, with the same greedy tokens (tests/test_decode_step_gpu.py).

The kernels launch with programmatic dependent launch, so each one's
prologue (for a GEMV, its weight stream) overlaps its predecessor's tail.
That is also why the RMSNorm and SiLU*up stay kernels of their own: a
one-CTA kernel between two GEMVs runs while the next GEMV's CTAs already
stream their weights, whereas folding it into that GEMV's activation staging
puts it on every CTA's path (measured 3 % slower per token for the norm,
no gain for SiLU*up, on config 1).
"""
from __future__ import annotations

import torch

from . import capi
from ._native import ext

_GGUF_BLOCK_BYTES = {"q4_0": 18, "q8_0": 34}


def _gguf_matrix(entry, what: str):
    """(format, raw bytes on the device, out_dim, in_dim) of a Q4_0 / Q8_0
    weight entry as torch_bridge._make_tensor_entry builds it
    (gdsllm/runtime/torch_bridge.py:125-146)."""
    if not (isinstance(entry, dict) and entry.get("gguf_type") in _GGUF_BLOCK_BYTES):
        raise ValueError(f"GraphDecodeStep: {what} must be a Q4_0 or Q8_0 weight, got "
                         f"{entry.get('gguf_type') or entry.get('quant_type') if isinstance(entry, dict) else type(entry).__name__}")
    n, k = (int(d) for d in entry["shape"])
    nbytes = n * (k // 32) * _GGUF_BLOCK_BYTES[entry["gguf_type"]]
    raw = ext().view_tensor(entry["buffer"], [nbytes], "int8", int(entry["offset"]))
    return entry["gguf_type"], raw, n, k


def _gemv(fmt, w, x, n, k, out):
    (capi.gemv_q4_0 if fmt == "q4_0" else capi.gemv_q8_0)(w, x, n, k, out=out)


class _Layer:
    """One layer's weights: raw GGUF matrices and fp16 norm vectors."""

    def __init__(self, tensors: dict, index: int):
        get = lambda name: _gguf_matrix(tensors[name], f"layer {index} {name}")  # noqa: E731
        self.q, self.k, self.v = (get(f"self_attn.{p}_proj.weight") for p in "qkv")
        self.o = get("self_attn.o_proj.weight")
        self.gate = get("mlp.gate_proj.weight")
        self.up = get("mlp.up_proj.weight")
        self.down = get("mlp.down_proj.weight")
        self.in_norm = tensors["input_layernorm.weight"]
        self.post_norm = tensors["post_attention_layernorm.weight"]
        for t in (self.in_norm, self.post_norm):
            if not (isinstance(t, torch.Tensor) and t.dtype == torch.float16):
                raise ValueError(f"GraphDecodeStep: layer {index} norms must be fp16 tensors")


class GraphDecodeStep:
    """A greedy decode position of a LLaMA model whose weights are resident:
    ``layers`` are the per-layer tensor dicts that ``transformer_block``
    receives (Q4_0 / Q8_0 projections, fp16 norms), ``embed`` the
    embed_tokens dict (fp16 or GGUF table), ``final_norm`` the fp16 norm
    weight, ``lm_head`` the GGUF head entry, ``freqs_cis`` the scheduler's
    complex RoPE table, and ``kv_cache`` the reference ``KVCache`` (batch 1).

    ``reset(token, pos)`` sets the input token and its position.  Each
    ``step()`` replays the captured graph: it writes that token's K/V at the
    position, leaves the argmax of its logits as the next input token, and
    advances the position.  ``logits`` holds the last step's logits."""

    def __init__(self, layers, embed: dict, final_norm: torch.Tensor, lm_head: dict, freqs_cis: torch.Tensor,
                 kv_cache, num_heads: int, num_kv_heads: int, rms_norm_eps: float, fused: bool = True):
        self.layers = [_Layer(t, i) for i, t in enumerate(layers)]
        if not self.layers:
            raise ValueError("GraphDecodeStep: no layers")
        first = self.layers[0]
        self.hidden = first.q[3]
        self.num_heads, self.num_kv_heads = int(num_heads), int(num_kv_heads)
        self.head_dim = self.hidden // self.num_heads  # as llama.attention derives it
        self.q_rows, self.kv_rows, self.ffn = first.q[2], first.k[2], first.gate[2]
        self.eps = float(rms_norm_eps)
        kc, vc = kv_cache.k_cache, kv_cache.v_cache
        if (kc.dim() != 5 or kc.shape[0] != len(self.layers) or kc.shape[1] != 1 or
                kc.shape[2] != self.num_kv_heads or kc.shape[4] != self.head_dim or kc.dtype != torch.float16 or
                not kc.is_contiguous() or vc.shape != kc.shape or not vc.is_contiguous()):
            raise ValueError(f"GraphDecodeStep: KV cache {tuple(kc.shape)} does not match {len(self.layers)} layers, "
                             f"batch 1, {self.num_kv_heads} KV heads of {self.head_dim}")
        self.kv = kv_cache
        self.max_seq = int(kc.shape[3])
        self.device = kc.device
        self.freqs = torch.view_as_real(freqs_cis[: self.max_seq]).contiguous()
        w = embed["model.embed_tokens.weight"]
        if isinstance(w, torch.Tensor):
            if w.dtype != torch.float16:
                raise ValueError("GraphDecodeStep: the embedding table must be fp16, Q4_0 or Q8_0")
            self.embed = ("f16", w, int(w.shape[0]), int(w.shape[1]))
        else:
            self.embed = _gguf_matrix(w, "model.embed_tokens.weight")
        self.final_norm = final_norm
        self.lm = _gguf_matrix(lm_head, "lm_head")
        self.vocab = self.lm[2]
        dev = self.device
        f16 = dict(dtype=torch.float16, device=dev)
        self.token = torch.zeros(1, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int64, device=dev)
        self.host_token = torch.zeros(1, dtype=torch.int64, pin_memory=True)
        self.h = torch.empty(self.hidden, **f16)
        self.x = torch.empty(self.hidden, **f16)
        self.qkv = torch.empty(self.q_rows + 2 * self.kv_rows, **f16)
        self.q_rot = torch.empty(self.q_rows, **f16)
        self.attn = torch.empty(self.num_heads * self.head_dim, **f16)
        self.o = torch.empty(self.hidden, **f16)
        self.gu = torch.empty(2 * self.ffn, **f16)
        self.act = torch.empty(self.ffn, **f16)
        self.d = torch.empty(self.hidden, **f16)
        self.logits = torch.empty(self.vocab, **f16)
        self.graph = None
        self.fused = bool(fused) and self.head_dim in (64, 128)

    @classmethod
    def from_scheduler(cls, sched, kv_cache, fused: bool = True) -> "GraphDecodeStep":
        """From an entered ``CachedScheduler`` (gdsllm/runtime/scheduler.py):
        every layer is taken from its layer cache and stays referenced here,
        so the buffers the graph reads stay allocated."""
        w = sched.weights
        layers = [sched.cache.get_layer(i) for i in range(w.num_layers)]
        embed = sched.cache.get_special("embed_tokens")
        norm = sched.cache.get_special("final_norm")["model.norm.weight"]
        if w.special.get("lm_head") is not None:
            head = sched.cache.get_special("lm_head")["lm_head.weight"]
        else:
            head = embed["model.embed_tokens.weight"]
        c = sched.config
        return cls(layers, embed, norm, head, sched.freqs_cis, kv_cache, c["num_heads"], c["num_kv_heads"],
                   c["rms_norm_eps"], fused=fused)

    # -- the token's launches ------------------------------------------------

    def _embed(self):
        kind, table, rows, cols = self.embed
        row = self.h.view(1, self.hidden)
        if kind == "f16":
            torch.index_select(table, 0, self.token, out=row)
        else:
            capi.dequant_rows(kind, table, rows, cols, self.token, out=row)

    def _record(self):
        nq, nk, ffn = self.q_rows, self.kv_rows, self.ffn
        q, k, v = self.qkv[:nq], self.qkv[nq:nq + nk], self.qkv[nq + nk:]
        gate, up = self.gu[:ffn], self.gu[ffn:]
        self._embed()
        for i, lay in enumerate(self.layers):
            capi.add_rmsnorm(self.h, lay.in_norm, self.eps, delta=self.d if i else None, out=self.x)
            self._project([lay.q, lay.k, lay.v], self.x, [q, k, v])
            kc, vc = self.kv.k_cache[i, 0], self.kv.v_cache[i, 0]
            if self.fused:  # RoPE and the cache write inside the attention kernel
                capi.attention_decode_rope(q, k, v, self.freqs, self.pos, kc, vc, self.num_heads, self.num_kv_heads,
                                           self.head_dim, self.max_seq, out=self.attn)
            else:
                capi.rope_kv(q, k, v, self.q_rot, self.freqs, self.pos, kc, vc, self.num_heads, self.num_kv_heads,
                             self.head_dim, self.max_seq)
                capi.attention_decode(self.q_rot, kc, vc, self.pos, self.num_heads, self.num_kv_heads,
                                      self.head_dim, self.max_seq, out=self.attn)
            _gemv(lay.o[0], lay.o[1], self.attn, lay.o[2], lay.o[3], self.o)
            capi.add_rmsnorm(self.h, lay.post_norm, self.eps, delta=self.o, out=self.x)
            self._project([lay.gate, lay.up], self.x, [gate, up])
            capi.silu_mul(gate, up, out=self.act)
            _gemv(lay.down[0], lay.down[1], self.act, lay.down[2], lay.down[3], self.d)
        capi.add_rmsnorm(self.h, self.final_norm, self.eps, delta=self.d, out=self.x)
        _gemv(self.lm[0], self.lm[1], self.x, self.lm[2], self.lm[3], self.logits)
        capi.argmax(self.logits, self.token, self.pos)
        self.host_token.copy_(self.token, non_blocking=True)

    def _project(self, mats, x, outs):
        if self._groupable(mats):
            capi.gemv_group(mats[0][0], [m[1] for m in mats], x, [m[2] for m in mats], mats[0][3], outs=outs)
        else:
            for m, y in zip(mats, outs):
                _gemv(m[0], m[1], x, m[2], m[3], y)

    @staticmethod
    def _groupable(mats) -> bool:
        """One launch serves matrices of one format and one K."""
        return len({m[0] for m in mats}) == 1 and len({m[3] for m in mats}) == 1

    def launches_per_step(self) -> int:
        """Kernels of one token (the pinned copy of the token is not one)."""
        n = 1 + 3  # embedding; final norm, lm_head, argmax
        for lay in self.layers:
            n += 6 + (0 if self.fused else 1)  # two norms, (rope_kv), attention, o, silu_mul, down
            n += 1 if self._groupable([lay.q, lay.k, lay.v]) else 3
            n += 1 if self._groupable([lay.gate, lay.up]) else 2
        return n

    # -- capture and replay ----------------------------------------------------

    def reset(self, token: int, pos: int) -> None:
        """The next step consumes `token` at position `pos`."""
        if not 0 <= pos < self.max_seq:
            raise ValueError(f"position {pos} outside the KV cache [0, {self.max_seq})")
        self.token.fill_(int(token))
        self.pos.fill_(int(pos))

    def capture(self) -> None:
        """Runs the token once eagerly (plans, tensor maps and shared-memory
        limits are set up on first use) and captures it as a CUDA graph.  The
        token and position are restored afterwards, so the next ``step()``
        repeats the eager position with the same result.  Programmatic
        dependent launch is switched on library-wide."""
        capi.set_pdl(True)
        saved_token, saved_pos = self.token.clone(), self.pos.clone()
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._record()
            self.token.copy_(saved_token)
            self.pos.copy_(saved_pos)
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._record()
        self.graph = graph

    def step(self, sync: bool = True):
        """One token.  With ``sync`` the host waits for it and returns the
        greedy token id (read from pinned memory the graph copied it to);
        without, the replay is only queued and None is returned."""
        if self.graph is None:
            self.capture()
        self.graph.replay()
        if not sync:
            return None
        torch.cuda.current_stream(self.device).synchronize()
        return int(self.host_token[0])

    def position(self) -> int:
        """The position the next step writes (synchronises)."""
        return int(self.pos.item())
