"""Tensor-parallel splits of the block-quantized projections (one process
per GPU, NCCL all-reduce over NVLink).

Megatron-style placement for a LLaMA block:
* column split (output rows) of q, k, v, gate, up: rank r owns rows
  ``[r * N / ws, (r + 1) * N / ws)`` of the packed matrix -- a contiguous slice
  of whole rows, so no re-packing; its output slice feeds the next
  row-split projection directly (attention heads and the SwiGLU product are
  per-rank);
* row split (input columns) of o and down: rank r owns columns
  ``[r * K / ws, (r + 1) * K / ws)``, whole quantization blocks only
  (``K / ws`` a multiple of 32, or of the affine group), re-packed into a
  contiguous ``[N][K / ws]`` matrix once at load time; every rank produces a
  partial ``[N]`` output and one all-reduce sums them.

The reference runs one GPU only; these splits and the all-reduce are the
whole of its multi-GPU path here.  The GEMV itself is the C-ABI kernel.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

BLOCK_BYTES = {"q4_0": 18, "q8_0": 34}


def row_range(n: int, rank: int, world: int):
    if n % world:
        raise ValueError(f"{n} rows do not split evenly over {world} ranks")
    per = n // world
    return rank * per, per


def split_rows(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Column-parallel shard: whole rows of a row-major packed matrix."""
    first, per = row_range(w.shape[0], rank, world)
    return w[first:first + per].contiguous()


def split_k_gguf(w: torch.Tensor, k: int, fmt: str, rank: int, world: int) -> torch.Tensor:
    """Row-parallel shard of a GGUF matrix [N][K/32 * block] (uint8): the
    blocks covering columns [r*K/ws, (r+1)*K/ws), re-packed contiguously."""
    if k % (32 * world):
        raise ValueError(f"K={k} does not split into whole 32-column blocks over {world} ranks")
    bb = BLOCK_BYTES[fmt]
    nb = k // 32 // world
    n = w.shape[0]
    blocks = w.reshape(n, k // 32, bb)
    return blocks[:, rank * nb:(rank + 1) * nb].reshape(n, nb * bb).contiguous()


def split_k_affine(words: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, k: int, group: int,
                   rank: int, world: int):
    """Row-parallel shard of an affine-Q4 matrix: words [N][K/8] and the
    per-group scales/biases [N][K/group] of columns [r*K/ws, (r+1)*K/ws)."""
    if k % (group * world):
        raise ValueError(f"K={k} does not split into whole groups of {group} over {world} ranks")
    kw = k // world
    w = words[:, rank * kw // 8:(rank + 1) * kw // 8].contiguous()
    g0, g1 = rank * kw // group, (rank + 1) * kw // group
    return w, scales[:, g0:g1].contiguous(), biases[:, g0:g1].contiguous()


def default_gemv(fmt: str) -> Callable:
    """(weight tensors, x [B, K], n, k) -> y [B, n] fp16 through the C ABI."""
    from . import capi

    if fmt == "q4_0":
        return lambda w, x, n, k, out=None: capi.gemv_q4_0(w[0], x, n, k, out=out)
    if fmt == "q8_0":
        return lambda w, x, n, k, out=None: capi.gemv_q8_0(w[0], x, n, k, out=out)
    raise ValueError(fmt)


class ColumnParallelGemv:
    """y_local [B, N/ws] = W[rows of this rank] . x (no communication)."""

    def __init__(self, weight, n: int, k: int, fmt: str = "q4_0", rank: int = 0, world: int = 1,
                 gemv: Optional[Callable] = None):
        self.n_local = n // world
        self.k = k
        self.weight = weight
        self.gemv = gemv or default_gemv(fmt)

    def __call__(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self.gemv(self.weight, x, self.n_local, self.k, out)


class RowParallelGemv:
    """y [B, N] = sum over ranks of W[:, cols of rank] . x_local.

    ``exchange``: None -> NCCL all-reduce after the GEMV; a
    ``p2p.PeerRowGemv`` -> the sum happens inside the GEMV's epilogue over
    NVLink peer memory (batch 1, GGUF formats)."""

    def __init__(self, weight, n: int, k: int, fmt: str = "q4_0", rank: int = 0, world: int = 1,
                 group: Optional[dist.ProcessGroup] = None, gemv: Optional[Callable] = None, exchange=None):
        self.n = n
        self.k_local = k // world
        self.weight = weight
        self.fmt = fmt
        self.world = world
        self.group = group
        self.gemv = gemv or default_gemv(fmt)
        self.exchange = exchange

    def __call__(self, x_local: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.world > 1 and self.exchange is not None and x_local.numel() == self.k_local:
            w = self.weight[0] if isinstance(self.weight, (tuple, list)) else self.weight
            return self.exchange(self.fmt, w, x_local, self.n, self.k_local, out)
        y = self.gemv(self.weight, x_local, self.n, self.k_local, out)
        if self.world > 1:
            dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        return y
