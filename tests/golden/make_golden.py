"""Generates the committed golden vectors under tests/golden/.

gguf_blocks.npz — third-party pin for the GGUF formats.
  Seeded Q4_0 and Q8_0 blocks (with the synthetic distributions plus hand-made
  edge blocks: zero, negative-zero, subnormal, largest and non-finite scales,
  extreme quants) and the fp32 output of ``gguf.dequantize`` from the ``gguf``
  Python package 0.19.0 (the GGUF format's published dequantizer; GdsLLM's
  converter depends on it, gdsllm/tools/convert_gguf.py:25).  gguf returns
  the exact fp32 product d*q; GdsLLM's kernels round it to fp16 with
  round-to-nearest-even (gdsllm/runtime/gguf_dequant.cu:56,105-106), so the
  pin is fp16(gguf) == oracle, bit for bit.

Run from the repository root: ``python tests/golden/make_golden.py``.
The reference-kernel fixtures (ref_kernels.npz) come from
tests/golden/make_ref_golden.py, which needs a GPU.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _edge_scales():
    # fp16 bit patterns for d
    return np.array([0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0xBC00, 0x7BFF, 0xFBFF,
                     0x7C00, 0xFC00, 0x7E00, 0x2E66, 0x1400], dtype=np.uint16)


def q4_0_blocks(rng: np.random.Generator, n_random: int) -> np.ndarray:
    d = (np.abs(rng.normal(0, 0.02, n_random)) / 4).astype(np.float16).view(np.uint16)
    qs = rng.integers(0, 256, (n_random, 16), dtype=np.uint8)
    edges_d = _edge_scales()
    patterns = [np.zeros(16, np.uint8), np.full(16, 0xFF, np.uint8), np.full(16, 0x88, np.uint8),
                np.arange(16, dtype=np.uint8) * 17, np.full(16, 0x0F, np.uint8),
                np.full(16, 0xF0, np.uint8)]
    ed, eq = [], []
    for dv in edges_d:
        for p in patterns:
            ed.append(dv)
            eq.append(p)
    d = np.concatenate([d, np.array(ed, np.uint16)])
    qs = np.concatenate([qs, np.stack(eq)])
    blocks = np.concatenate([d.reshape(-1, 1).view(np.uint8).reshape(-1, 2), qs], axis=1)
    return np.ascontiguousarray(blocks, dtype=np.uint8)


def q8_0_blocks(rng: np.random.Generator, n_random: int) -> np.ndarray:
    d = (np.abs(rng.normal(0, 0.02, n_random)) / 4).astype(np.float16).view(np.uint16)
    qs = rng.integers(-127, 128, (n_random, 32), dtype=np.int8)
    edges_d = _edge_scales()
    patterns = [np.zeros(32, np.int8), np.full(32, 127, np.int8), np.full(32, -127, np.int8),
                np.full(32, -128, np.int8), np.arange(-16, 16, dtype=np.int8),
                np.array([(-1) ** i * 127 for i in range(32)], np.int8)]
    ed, eq = [], []
    for dv in edges_d:
        for p in patterns:
            ed.append(dv)
            eq.append(p)
    d = np.concatenate([d, np.array(ed, np.uint16)])
    qs = np.concatenate([qs, np.stack(eq)])
    blocks = np.concatenate([d.reshape(-1, 1).view(np.uint8).reshape(-1, 2), qs.view(np.uint8)],
                            axis=1)
    return np.ascontiguousarray(blocks, dtype=np.uint8)


def main() -> None:
    import gguf
    from gguf import GGMLQuantizationType as T
    from gguf import dequantize

    rng = np.random.default_rng(20240601)
    q4 = q4_0_blocks(rng, 512)
    q8 = q8_0_blocks(rng, 512)
    with np.errstate(all="ignore"):
        q4_out = dequantize(q4.reshape(-1), T.Q4_0).reshape(-1).astype(np.float32)
        q8_out = dequantize(q8.reshape(-1), T.Q8_0).reshape(-1).astype(np.float32)
    np.savez_compressed(HERE / "gguf_blocks.npz", q4_0_blocks=q4, q4_0_gguf_f32=q4_out,
                        q8_0_blocks=q8, q8_0_gguf_f32=q8_out,
                        gguf_version=np.array(getattr(gguf, "__version__", "0.19.0")))
    print("wrote", HERE / "gguf_blocks.npz", q4.shape, q8.shape)


if __name__ == "__main__":
    main()
