"""Expert-parallel placement of the MoE experts (one process per GPU).

Experts ``[r * E / ws, (r + 1) * E / ws)`` live on rank r (the same contiguous
placement as ``e // (E / ws)``).  Every rank holds the replicated router and
computes the same routing from the same hidden state, so no ids are
exchanged; each rank runs the fused expert-gather kernels over its own
experts only (slots routed elsewhere are skipped on the device) and adds the
shared expert on rank 0; one all-reduce of the fp32 partial sums [B, hidden]
per layer combines them.  The reference has no expert parallelism: this is
the only exchange the path needs.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import moe


def expert_range(rank: int, world: int, num_experts: int):
    """(first, count) of the experts resident on ``rank``."""
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split evenly over {world} ranks")
    per = num_experts // world
    return rank * per, per


def local_stack(full: moe.Stack, rank: int, world: int) -> moe.Stack:
    """This rank's slice of a stacked expert tensor triple (contiguous copy)."""
    first, count = expert_range(rank, world, full[0].shape[0])
    return tuple(t[first:first + count].contiguous() for t in full)


class ExpertParallelMoE:
    """One MoE MLP split over the ranks of ``group``.

    ``layer`` holds this rank's experts (``expert_first``/``expert_total`` set
    accordingly).  ``partial`` computes the rank's fp32 partial sum; it is
    ``moe.moe_partial`` (the CUDA kernels) unless a test substitutes a
    checker.  ``allreduce`` sums the partial in place over the ranks, e.g. a
    ``p2p.PeerWordAllReduce`` over NVLink peer memory; None uses NCCL.
    """

    def __init__(self, layer: moe.MoeLayer, group: Optional[dist.ProcessGroup] = None,
                 top_k: int = 10, partial: Optional[Callable] = None, router: Optional[Callable] = None,
                 allreduce: Optional[Callable] = None):
        self.layer = layer
        self.group = group
        self.top_k = top_k
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        first, count = expert_range(self.rank, self.world, layer.total)
        if (first, count) != (layer.expert_first, layer.num_local):
            raise ValueError(f"rank {self.rank} holds experts [{layer.expert_first}, "
                             f"{layer.expert_first + layer.num_local}), expected [{first}, {first + count})")
        self.partial = partial or moe.moe_partial
        # default: the fused router kernel (deterministic, so every rank routes alike)
        self.router = router or (lambda x2d, _w, k, _sg: moe.route_fused(x2d, self.layer, k))
        self.allreduce = allreduce  # in-place sum of the fp32 partial; None -> NCCL

    def forward(self, x: torch.Tensor, out32: Optional[torch.Tensor] = None,
                add_residual: bool = False) -> torch.Tensor:
        """The layer's output, or x + output (the caller's residual add in
        the same fp16 roundings) with ``add_residual``."""
        x2d = x.reshape(-1, x.shape[-1])
        sg = self.layer.shared_gate if self.layer.shared is not None else None
        ids, weights, sw = self.router(x2d, self.layer.router, self.top_k, sg)
        y32 = self.partial(x2d, ids, weights, self.layer, out=out32, include_shared=self.rank == 0,
                           shared_weights=sw)
        if self.allreduce is not None and getattr(self.allreduce, "finishes_fp16", False):
            y = torch.empty(y32.shape, dtype=x.dtype, device=y32.device)
            # sum, clamp, fp16 (and the residual add) in the exchange kernel
            self.allreduce(y32, out=y, residual=x2d.contiguous() if add_residual else None)
            return y.view(x.shape)
        if self.allreduce is not None:
            self.allreduce(y32)
        else:
            dist.all_reduce(y32, op=dist.ReduceOp.SUM, group=self.group)
        y = moe.finish(y32, x)
        return x + y if add_residual else y

    __call__ = forward
