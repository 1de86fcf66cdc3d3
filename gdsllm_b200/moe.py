"""MoE decode layer on the fused expert-gather kernels.

Mirrors the reference's decode path of one Qwen-MoE MLP
(gdsllm/runtime/qwen_moe.py:386-516):

* ``route``: ``moe_route`` -- router logits ``F.linear(x, W_r)``, top-k, softmax
  of the top-k logits in fp32, cast back to x's dtype (qwen_moe.py:407-413).
  Expert ids stay on the device (the reference reads them back with
  ``.unique().tolist()`` and ``.item()``).
* ``moe_partial``: the routed experts resident in this process (all of them
  on one GPU, a contiguous range under expert parallelism) through
  ``gds_io_ext.fused_moe_affine_q4``, plus optionally the shared expert scaled
  by ``sigmoid(F.linear(x, W_sg))`` (qwen_moe.py:497-510), summed in fp32.
* ``moe_mlp_decode``: the full single-GPU layer output, clamped to the fp16
  range as qwen_moe.py:513-514 does.

There is no CPU path: the routed/shared expert math runs only in the CUDA
extension.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional, Tuple

import torch
import torch.nn.functional as F

Stack = Tuple[torch.Tensor, torch.Tensor, torch.Tensor]  # (words int32, scales fp16, biases fp16)


@dataclass
class MoeLayer:
    """Weights of one MoE MLP as resident on this device.

    gate / up: words [E, inter, hidden/8], scales/biases [E, inter, hidden/group];
    down: words [E, hidden, inter/8], scales/biases [E, hidden, inter/group];
    holding experts ``expert_first .. expert_first + E - 1`` of
    ``expert_total``.  ``shared`` = (gate, up, down) stacks of one expert;
    ``shared_gate`` fp16 [1, hidden]; ``router`` fp16 [expert_total, hidden].
    """
    router: torch.Tensor
    gate: Stack
    up: Stack
    down: Stack
    group: int = 128
    expert_first: int = 0
    expert_total: Optional[int] = None
    shared: Optional[Tuple[Stack, Stack, Stack]] = None
    shared_gate: Optional[torch.Tensor] = None
    _router: Optional["FusedRouter"] = field(default=None, repr=False, compare=False)

    @property
    def num_local(self) -> int:
        return self.gate[0].shape[0]

    @property
    def total(self) -> int:
        return self.expert_total if self.expert_total is not None else self.expert_first + self.num_local


def route_torch(x2d: torch.Tensor, router: torch.Tensor, top_k: int,
                shared_gate: Optional[torch.Tensor] = None):
    """moe_route as the reference writes it in torch (qwen_moe.py:407-413),
    plus the shared expert's sigmoid gate (qwen_moe.py:505-509):
    (ids int32 [B, k], weights fp16 [B, k], shared weight fp16 [B] or None)."""
    logits = F.linear(x2d, router)
    top_logits, ids = torch.topk(logits, top_k, dim=-1)
    weights = F.softmax(top_logits.float(), dim=-1).type_as(x2d)
    sw = None
    if shared_gate is not None:
        sw = torch.sigmoid(F.linear(x2d, shared_gate.view(1, -1))).view(-1)
    return ids.to(torch.int32), weights, sw


def route(x2d: torch.Tensor, router: torch.Tensor, top_k: int, shared_gate: Optional[torch.Tensor] = None):
    """Same outputs as route_torch: the router logits from the same F.linear,
    then top-k, softmax and the shared gate in one kernel (gdsq_moe_route)."""
    logits = F.linear(x2d, router)
    g = None if shared_gate is None else shared_gate.reshape(-1).contiguous()
    return _ext().moe_route(logits, top_k, x2d if g is not None else None, g)


ROUTER_MAX_EXPERTS, ROUTER_MAX_TOP_K = 512, 32
# The kernel takes up to 16 tokens; from 5 on, cuBLAS's F.linear + the route
# kernel is faster (config 4 at 8 tokens: 435 vs 346 tok/s), so route_fused
# uses the fused kernel for at most 4.
ROUTER_MAX_TOKENS = 4


class FusedRouter:
    """The router GEMV and the routing in one launch (gdsq_moe_router): no
    F.linear.  The logits are this build's fused fp16 GEMV of x and the
    router (fp32 sums of the fp16 products, rounded once, as F.linear
    rounds its output), so a near-tie at the top-k boundary can resolve
    differently from cuBLAS's logits; the selection is the exact top-k of
    ``self.logits``.  One instance per call sequence on a stream (it owns
    the kernel's completion counter)."""

    def __init__(self, router: torch.Tensor, shared_gate: Optional[torch.Tensor] = None):
        self.router = router.contiguous()
        self.shared_gate = None if shared_gate is None else shared_gate.reshape(-1).contiguous()
        self.experts, self.hidden = self.router.shape
        self.counter = torch.zeros(1, dtype=torch.int32, device=router.device)
        self.logits = None

    @staticmethod
    def fits(router: torch.Tensor, top_k: int, tokens: int) -> bool:
        return (router.shape[0] <= ROUTER_MAX_EXPERTS and top_k <= ROUTER_MAX_TOP_K and
                1 <= tokens <= ROUTER_MAX_TOKENS and router.shape[1] % 512 == 0)

    def __call__(self, x2d: torch.Tensor, top_k: int):
        from . import capi
        b = x2d.shape[0]
        x2d = x2d.contiguous()
        if self.logits is None or self.logits.shape[0] < b:
            self.logits = torch.empty(b, self.experts + 1, dtype=torch.float16, device=x2d.device)
        ids = torch.empty(b, top_k, dtype=torch.int32, device=x2d.device)
        w = torch.empty(b, top_k, dtype=torch.float16, device=x2d.device)
        sw = None if self.shared_gate is None else torch.empty(b, dtype=torch.float16, device=x2d.device)
        capi.check(capi.lib().gdsq_moe_router(
            x2d.data_ptr(), b, self.hidden, self.router.data_ptr(), self.experts,
            None if self.shared_gate is None else self.shared_gate.data_ptr(), top_k, self.logits.data_ptr(),
            ids.data_ptr(), w.data_ptr(), None if sw is None else sw.data_ptr(), self.counter.data_ptr(),
            torch.cuda.current_stream(x2d.device).cuda_stream), "gdsq_moe_router")
        return ids, w, sw


def route_fused(x2d: torch.Tensor, layer: "MoeLayer", top_k: int):
    """``route`` through the layer's FusedRouter when its shapes fit (else
    ``route``): (ids, weights, shared weight or None)."""
    sg = layer.shared_gate if layer.shared is not None else None
    if not FusedRouter.fits(layer.router, top_k, x2d.shape[0]):
        return route(x2d, layer.router, top_k, sg)
    if layer._router is None:
        layer._router = FusedRouter(layer.router, sg)
    return layer._router(x2d, top_k)


def _ext():
    from ._native import ext
    return ext()


def _shared_list(layer: "MoeLayer"):
    return [t for stack in layer.shared for t in stack]


def moe_partial(x2d: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, layer: MoeLayer,
                out: Optional[torch.Tensor] = None, include_shared: bool = True,
                shared_weights: Optional[torch.Tensor] = None, out_fp32: bool = True,
                clamp: bool = False, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[B, hidden]: sum over this device's resident routed experts, plus the
    shared expert (weighted by ``shared_weights``) when ``include_shared`` --
    one gate/up launch and one down launch.  fp32 by default (partial sums
    for an all-reduce); ``out_fp32=False, clamp=True`` gives the final fp16."""
    b, hidden = x2d.shape
    if out is None:
        out = torch.empty(b, hidden, dtype=torch.float32 if out_fp32 else torch.float16, device=x2d.device)
    use_shared = include_shared and layer.shared is not None
    if use_shared and shared_weights is None:
        shared_weights = torch.sigmoid(F.linear(x2d, layer.shared_gate)).view(-1)
    _ext().fused_moe_affine_q4(x2d, ids, weights, layer.gate, layer.up, layer.down, group_size=layer.group,
                               expert_first=layer.expert_first, expert_total=layer.total, out=out,
                               out_fp32=out_fp32, shared=_shared_list(layer) if use_shared else None,
                               shared_weights=shared_weights if use_shared else None, clamp=clamp,
                               residual=residual)
    return out


def finish(y32: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """fp32 layer sum -> fp16 in x's shape, clamped like qwen_moe.py:514."""
    return y32.clamp(min=-65504.0, max=65504.0).to(like.dtype).view(like.shape)


def moe_mlp_decode(x: torch.Tensor, layer: MoeLayer, top_k: int = 10, add_residual: bool = False) -> torch.Tensor:
    """One MoE MLP on one GPU: x (B, S, hidden) or (B, hidden) fp16.  Three
    launches: router + route (one kernel, ``route_fused``), gate/up, down
    (clamped fp16).
    ``add_residual`` returns x + moe(x) (the caller's residual add, in the
    same fp16 roundings) from the down launch itself."""
    x2d = x.reshape(-1, x.shape[-1])
    ids, weights, sw = route_fused(x2d, layer, top_k)
    y = moe_partial(x2d, ids, weights, layer, shared_weights=sw, out_fp32=False, clamp=True,
                    residual=x2d.contiguous() if add_residual else None)
    return y.view(x.shape)
