"""Seeded synthetic weights and activations in the reference's packed layouts.

Distributions follow the benchmark configurations:
* Q4_0: nibbles uniform over 0..15 (so each packed byte is uniform over
  0..255), d = fp16(|N(0, 0.02)| / 4).
* Q8_0: int8 uniform over -127..127, d as for Q4_0.
* affine Q4: nibbles uniform over 0..15 (each uint32 word uniform),
  scale = fp16(|N(0, 0.01)|), bias = fp16(N(0, 0.01)), group size 128.
* activations: fp16 N(0, 1).

Layouts (byte-identical to what gdsllm/tools/convert_gguf.py:164-169 and
convert_qwen_moe.py:205-253 write):
* Q4_0: [N][K/32] blocks of 18 bytes = fp16 d (little-endian) + 16 qs bytes.
* Q8_0: [N][K/32] blocks of 34 bytes = fp16 d + 32 int8.
* affine: uint32 [N][K/8] (stored here as int32), fp16 scales/biases [N][K/g].
"""
from __future__ import annotations

import torch


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def q4_0_weight(n: int, k: int, seed: int = 0, device="cpu") -> torch.Tensor:
    """Packed Q4_0 bytes, uint8 [n, k/32*18]."""
    assert k % 32 == 0
    g = _gen(seed, device)
    nb = k // 32
    d = (torch.randn(n, nb, generator=g, device=device) * 0.02).abs().div_(4).half()
    qs = torch.randint(0, 256, (n, nb, 16), generator=g, device=device, dtype=torch.uint8)
    blocks = torch.cat([d.view(torch.uint8).view(n, nb, 2), qs], dim=2)
    return blocks.reshape(n, nb * 18).contiguous()


def q8_0_weight(n: int, k: int, seed: int = 0, device="cpu") -> torch.Tensor:
    """Packed Q8_0 bytes, uint8 [n, k/32*34]."""
    assert k % 32 == 0
    g = _gen(seed, device)
    nb = k // 32
    d = (torch.randn(n, nb, generator=g, device=device) * 0.02).abs().div_(4).half()
    qs = torch.randint(-127, 128, (n, nb, 32), generator=g, device=device, dtype=torch.int8)
    blocks = torch.cat([d.view(torch.uint8).view(n, nb, 2), qs.view(torch.uint8)], dim=2)
    return blocks.reshape(n, nb * 34).contiguous()


def affine_q4_weight(n: int, k: int, group: int = 128, seed: int = 0, device="cpu",
                     lead: tuple = ()):
    """(words int32 [*lead, n, k/8], scales fp16 [*lead, n, k/group], biases fp16)."""
    assert k % group == 0 and group % 8 == 0
    g = _gen(seed, device)
    shape = (*lead, n)
    words = torch.randint(-(2 ** 31), 2 ** 31, (*shape, k // 8), generator=g, device=device,
                          dtype=torch.int64).to(torch.int32)
    scales = (torch.randn(*shape, k // group, generator=g, device=device) * 0.01).abs().half()
    biases = (torch.randn(*shape, k // group, generator=g, device=device) * 0.01).half()
    return words.contiguous(), scales.contiguous(), biases.contiguous()


def activations(b: int, k: int, seed: int = 1, device="cpu") -> torch.Tensor:
    """fp16 N(0,1) [b, k]."""
    g = _gen(seed, device)
    return torch.randn(b, k, generator=g, device=device).half()


LLAMA_LAYER_TENSORS = ("input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
                       "self_attn.v_proj.weight", "self_attn.o_proj.weight", "post_attention_layernorm.weight",
                       "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")


def _tensor_bytes(kind: str, rows: int, cols: int, seed: int, device) -> tuple:
    """(uint8 host bytes, dtype string, quant string or None) of one tensor."""
    if kind == "q4_0":
        return q4_0_weight(rows, cols, seed=seed, device=device).cpu().reshape(-1), "gguf_q4_0", "q4_0"
    if kind == "q8_0":
        return q8_0_weight(rows, cols, seed=seed, device=device).cpu().reshape(-1), "gguf_q8_0", "q8_0"
    g = _gen(seed, device)
    t = (torch.randn(rows, cols, generator=g, device=device) * 0.02).half()
    return t.cpu().reshape(-1).view(torch.uint8), "float16", None


def write_llama_model_dir(path, *, layers: int, hidden: int, heads: int, kv_heads: int, ffn: int, vocab: int,
                          max_seq_len: int, body: str = "q4_0", lm_head: str = "q8_0", embed: str = "q4_0",
                          rms_norm_eps: float = 1e-5, rope_theta: float = 10000.0, norm_jitter: float = 0.0,
                          seed: int = 0, device="cpu") -> dict:
    """Writes a synthetic LLaMA model directory in the layout GdsLLM's GGUF
    converter produces (gdsllm/tools/convert_gguf.py:378-431, 520-560): one
    file per layer with the nine tensors in converter order, each 4 KB
    aligned, plus embed_tokens.bin, final_norm.bin, lm_head.bin and
    metadata.json.  Block-quantized tensors keep GGUF blocks verbatim
    ([rows][cols/32] blocks), norms are fp16 (ones, or 1 + U(-j, j) with
    norm_jitter j), fp16 tensors are N(0, 0.02).  Returns the metadata."""
    import json
    import os

    os.makedirs(path, exist_ok=True)
    head_dim = hidden // heads
    align = 4096

    def write(f, data: torch.Tensor, name, shape, dtype, quant):
        off = f.tell()
        raw = data.numpy().tobytes()
        f.write(raw)
        padded = (len(raw) + align - 1) // align * align
        f.write(b"\0" * (padded - len(raw)))
        meta = {"name": name, "shape": list(shape), "dtype": dtype, "offset": off, "size_bytes": len(raw),
                "padded_size": padded, "quant": quant}
        if quant in ("q4_0", "q8_0"):
            meta["block_size"] = 32
        return meta

    def norm(seed_):
        if norm_jitter <= 0:
            return torch.ones(hidden, dtype=torch.float16).view(torch.uint8)
        g = torch.Generator().manual_seed(seed_)
        return (1 + (torch.rand(hidden, generator=g) * 2 - 1) * norm_jitter).half().view(torch.uint8)

    def special(fname, name, kind, rows, cols, seed_):
        with open(os.path.join(path, fname), "wb") as f:
            if kind == "norm":
                meta = write(f, norm(seed_), name, [cols], "float16", None)
            else:
                data, dtype, quant = _tensor_bytes(kind, rows, cols, seed_, device)
                meta = write(f, data, name, [rows, cols], dtype, quant)
            return {"path": fname, "size_bytes": f.tell(), "tensors": [meta]}

    shapes = {"self_attn.q_proj.weight": (hidden, hidden), "self_attn.k_proj.weight": (kv_heads * head_dim, hidden),
              "self_attn.v_proj.weight": (kv_heads * head_dim, hidden), "self_attn.o_proj.weight": (hidden, hidden),
              "mlp.gate_proj.weight": (ffn, hidden), "mlp.up_proj.weight": (ffn, hidden),
              "mlp.down_proj.weight": (hidden, ffn)}
    layer_metas = []
    for li in range(layers):
        fname = f"layer_{li:03d}.bin"
        tensors = []
        with open(os.path.join(path, fname), "wb") as f:
            for ti, name in enumerate(LLAMA_LAYER_TENSORS):
                s = seed * 100003 + li * 16 + ti
                if name.endswith("layernorm.weight"):
                    tensors.append(write(f, norm(s), name, [hidden], "float16", None))
                else:
                    data, dtype, quant = _tensor_bytes(body, *shapes[name], s, device)
                    tensors.append(write(f, data, name, list(shapes[name]), dtype, quant))
            layer_metas.append({"index": li, "path": fname, "size_bytes": f.tell(), "tensors": tensors})
    meta = {
        "model": "llama", "dtype": body, "quantization": body, "alignment": align,
        "vocab_size": vocab, "hidden_size": hidden, "intermediate_size": ffn, "num_layers": layers,
        "num_heads": heads, "num_kv_heads": kv_heads, "rms_norm_eps": rms_norm_eps, "rope_theta": rope_theta,
        "max_seq_len": max_seq_len, "head_dim": head_dim, "lm_head_tied": False,
        "files": {
            "embed_tokens": special("embed_tokens.bin", "model.embed_tokens.weight", embed, vocab, hidden,
                                    seed * 100003 + 99991),
            "final_norm": special("final_norm.bin", "model.norm.weight", "norm", 1, hidden, seed * 100003 + 99992),
            "lm_head": special("lm_head.bin", "lm_head.weight", lm_head, vocab, hidden, seed * 100003 + 99993),
            "layers": layer_metas,
        },
    }
    with open(os.path.join(path, "metadata.json"), "w") as f:
        json.dump(meta, f, indent=1)
    return meta


def write_moe_layer_dir(path, *, experts: int, hidden: int, inter: int, group: int = 128, seed: int = 0,
                        device="cpu") -> dict:
    """Writes a synthetic one-layer Qwen-MoE model directory with the MoE
    tensors in the layout of GdsLLM's converter (gdsllm/tools/
    convert_qwen_moe.py:205-253): affine-Q4 tensors as packed uint32 words,
    fp16 scales and fp16 biases, each region 4 KB aligned, with the weight
    entry carrying the scale/bias offsets; routed experts stacked 3-D
    [experts][rows][cols/8] under mlp.switch_mlp.*; an fp16 router
    (mlp.gate.weight, N(0, 1/hidden)), the shared expert and its fp16 gate.
    Returns the metadata."""
    import json
    import os

    os.makedirs(path, exist_ok=True)
    align = 4096
    tensors = []

    def write(f, data: torch.Tensor):
        off = f.tell()
        raw = data.contiguous().cpu().numpy().tobytes()
        f.write(raw)
        padded = (len(raw) + align - 1) // align * align
        f.write(b"\0" * (padded - len(raw)))
        return off, len(raw), padded

    def affine(f, prefix, rows, cols, seed_, lead=()):
        words, scales, biases = affine_q4_weight(rows, cols, group=group, seed=seed_, device=device, lead=lead)
        w_off, w_size, w_pad = write(f, words)
        s_off, s_size, s_pad = write(f, scales)
        b_off, b_size, b_pad = write(f, biases)
        tensors.append({"name": f"{prefix}.weight", "shape": [*lead, rows, cols], "dtype": "uint32",
                        "offset": w_off, "size_bytes": w_size, "padded_size": w_pad, "quant": "affine_q4",
                        "group_size": group, "scale_shape": list(scales.shape), "scale_offset": s_off,
                        "scale_size_bytes": s_size, "scale_padded_size": s_pad, "bias_shape": list(biases.shape),
                        "bias_offset": b_off, "bias_size_bytes": b_size, "bias_padded_size": b_pad})
        tensors.append({"name": f"{prefix}.scales", "shape": list(scales.shape), "dtype": "float16",
                        "offset": s_off, "size_bytes": s_size, "padded_size": s_pad, "quant": None})
        tensors.append({"name": f"{prefix}.biases", "shape": list(biases.shape), "dtype": "float16",
                        "offset": b_off, "size_bytes": b_size, "padded_size": b_pad, "quant": None})

    def fp16(f, name, t):
        off, size, pad = write(f, t.half())
        tensors.append({"name": name, "shape": list(t.shape), "dtype": "float16", "offset": off, "size_bytes": size,
                        "padded_size": pad, "quant": None})

    g = torch.Generator().manual_seed(seed)
    fname = "layer_000.bin"
    with open(os.path.join(path, fname), "wb") as f:
        fp16(f, "mlp.gate.weight", torch.randn(experts, hidden, generator=g) / hidden ** 0.5)
        affine(f, "mlp.shared_expert.gate_proj", inter, hidden, seed * 64 + 1)
        affine(f, "mlp.shared_expert.up_proj", inter, hidden, seed * 64 + 2)
        affine(f, "mlp.shared_expert.down_proj", hidden, inter, seed * 64 + 3)
        fp16(f, "mlp.shared_expert_gate.weight", torch.randn(1, hidden, generator=g) / hidden ** 0.5)
        affine(f, "mlp.switch_mlp.gate_proj", inter, hidden, seed * 64 + 4, lead=(experts,))
        affine(f, "mlp.switch_mlp.up_proj", inter, hidden, seed * 64 + 5, lead=(experts,))
        affine(f, "mlp.switch_mlp.down_proj", hidden, inter, seed * 64 + 6, lead=(experts,))
        size = f.tell()
    meta = {"model": "qwen3_5_moe", "quantization": "affine_q4", "alignment": align, "hidden_size": hidden,
            "moe_intermediate_size": inter, "num_experts": experts, "group_size": group, "num_layers": 1,
            "files": {"layers": [{"index": 0, "path": fname, "size_bytes": size, "layer_type": "full_attention",
                                  "tensors": tensors}]}}
    with open(os.path.join(path, "metadata.json"), "w") as f:
        json.dump(meta, f, indent=1)
    return meta


def pack_affine_buffer(words: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                       align: int = 4096):
    """Lays out weight | scales | biases in one uint8 buffer the way the
    reference's layer files do (each region 4 KB aligned).  Returns
    (buffer, weight_offset, scale_offset, bias_offset)."""
    def nbytes(t):
        return t.numel() * t.element_size()

    def up(v):
        return (v + align - 1) // align * align

    w_off = 0
    s_off = up(nbytes(words))
    b_off = s_off + up(nbytes(scales))
    total = b_off + up(nbytes(biases))
    buf = torch.zeros(total, dtype=torch.uint8, device=words.device)
    buf[w_off:w_off + nbytes(words)] = words.reshape(-1).view(torch.uint8)
    buf[s_off:s_off + nbytes(scales)] = scales.reshape(-1).view(torch.uint8)
    buf[b_off:b_off + nbytes(biases)] = biases.reshape(-1).view(torch.uint8)
    return buf, w_off, s_off, b_off
