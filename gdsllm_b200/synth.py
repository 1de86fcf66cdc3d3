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
