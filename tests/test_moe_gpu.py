"""GPU parity of the fused MoE expert gather (gdsq_moe_affine_q4_gate_up /
_down through the C ABI, and gds_io_ext.fused_moe_affine_q4) against the CPU
oracle's restatement of moe_mlp_selective's decode branch
(gdsllm/runtime/qwen_moe.py:453-474).

Bars (stated here, applied below):
* h (stage 0): |h - h_ref| <= 1.1 |u| (bar_g + ulp(g)) + 1.1 |silu(g)| (bar_u + ulp(u)) + 2 ulp(h_ref),
  h_ref from fp64 gate/up GEMVs rounded once, bar_* the GEMV bar
  2e-3 * ||x||_2 * max|W| of that expert;
* y (stage 1, on the kernel's own h): |y - y_exact| <= sum_k |w_k| 2e-3 ||h_k||_2 max|W_down,k|
  + 1 ulp(y);
* end to end against the fp16 reference sequence: the stage-1 bar plus the
  stage-0 bar carried through down (sum_k |w_k| ||W_down,k row||_2 ||tol_h,k||_2)
  plus top_k fp16 ulps of the reference's running fp16 sum.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from gdsllm_b200 import synth

pytestmark = pytest.mark.gpu


def _ulp16(v):
    a = np.abs(np.asarray(v, np.float64))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -14)))
    return 2.0 ** (e - 10)


def _stacks(experts, hidden, inter, group, seed, device):
    gate = synth.affine_q4_weight(inter, hidden, group=group, seed=seed, lead=(experts,))
    up = synth.affine_q4_weight(inter, hidden, group=group, seed=seed + 1, lead=(experts,))
    down = synth.affine_q4_weight(hidden, inter, group=group, seed=seed + 2, lead=(experts,))
    cpu = tuple(tuple(t.numpy() for t in m) for m in (gate, up, down))
    dev = tuple(tuple(t.to(device) for t in m) for m in (gate, up, down))
    return cpu, dev


def _routing(ntok, top_k, experts, seed):
    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(experts, generator=g)[:top_k] for _ in range(ntok)]).to(torch.int32)
    logits = torch.randn(ntok, top_k, generator=g)
    w = torch.softmax(logits, dim=-1).half()
    return ids, w


def _h_tolerance(cpu, ids, x, g_ex, u_ex, group):
    gate, up, _ = cpu
    ntok, top_k = ids.shape
    tol = np.zeros_like(g_ex)
    for t in range(ntok):
        for k in range(top_k):
            e = int(ids[t, k])
            bg = oracle.error_bound(oracle.expert_f16(gate, e, group), x[t])[0]
            bu = oracle.error_bound(oracle.expert_f16(up, e, group), x[t])[0]
            g, u = g_ex[t, k], u_ex[t, k]
            s = np.abs(oracle.silu_f16(g.astype(np.float16)).astype(np.float64))
            tol[t, k] = 1.1 * np.abs(u) * (bg + _ulp16(g)) + 1.1 * s * (bu + _ulp16(u))
    return tol


def _check_h(h_gpu, cpu, ids, x, group):
    h_ref, g_ex, u_ex = oracle.moe_gate_up_exact(x, ids, cpu[0], cpu[1], group)
    h = h_gpu.float().cpu().numpy().astype(np.float64)
    tol = _h_tolerance(cpu, ids, x, g_ex, u_ex, group) + 2 * _ulp16(h_ref.astype(np.float64))
    err = np.abs(h - h_ref.astype(np.float64))
    assert np.isfinite(h).all(), "non-finite h"
    bad = err > tol
    assert not bad.any(), f"h: {bad.sum()} entries over the bar; worst {(err / tol).max():.3f}"
    return h_ref, tol


def _check_y(y_gpu, h_used, cpu, ids, w, group, e_first=0, extra=None):
    y_ex, bar = oracle.moe_down_exact(h_used, ids, w, cpu[2], group, e_first)
    y = y_gpu.float().cpu().numpy().astype(np.float64).reshape(y_ex.shape)
    tol = bar[:, None] + _ulp16(y_ex)
    if extra is not None:
        tol = tol + extra
    err = np.abs(y - y_ex)
    assert np.isfinite(y).all(), "non-finite y"
    assert (err <= tol).all(), f"y: worst err/bar {(err / tol).max():.3f}"
    return (err / tol).max()


SHAPES = [
    # experts, hidden, inter, group, ntok, top_k
    (8, 1024, 512, 128, 1, 4),
    (8, 1024, 512, 64, 3, 4),
    (16, 4096, 1024, 128, 1, 10),
    (16, 4096, 1024, 128, 8, 10),
    (6, 2048, 768, 32, 2, 6),
]


@pytest.mark.parametrize("experts,hidden,inter,group,ntok,top_k", SHAPES)
def test_moe_stages_parity(gdsq, cuda, experts, hidden, inter, group, ntok, top_k):
    cpu, dev = _stacks(experts, hidden, inter, group, seed=hidden + inter + ntok, device=cuda)
    ids, w = _routing(ntok, top_k, experts, seed=ntok)
    x = synth.activations(ntok, hidden, seed=3)
    h = gdsq.moe_gate_up(dev[0], dev[1], x.to(cuda), ids.to(cuda), group)
    y = gdsq.moe_down(dev[2], h, ids.to(cuda), w.to(cuda), group)
    torch.cuda.synchronize()
    assert gdsq.device_error(0) == 0
    _check_h(h, cpu, ids.numpy(), x.numpy(), group)
    _check_y(y, h.cpu().numpy(), cpu, ids.numpy(), w.numpy(), group)


@pytest.mark.parametrize("ntok", [1, 2])
def test_moe_matches_reference_decode_sequence(ext, cuda, ntok):
    """The whole routed-expert MLP against the reference's fp16 arithmetic."""
    experts, hidden, inter, group, top_k = 16, 4096, 1024, 128, 10
    cpu, dev = _stacks(experts, hidden, inter, group, seed=77, device=cuda)
    ids, w = _routing(ntok, top_k, experts, seed=5 + ntok)
    x = synth.activations(ntok, hidden, seed=11)
    y = ext.fused_moe_affine_q4(x.to(cuda), ids.to(cuda).long(), w.to(cuda), dev[0], dev[1], dev[2],
                                group_size=group)
    torch.cuda.synchronize()
    ref = oracle.moe_decode_reference(x.numpy(), ids.numpy(), w.numpy(), *cpu, group)
    h_ref, g_ex, u_ex = oracle.moe_gate_up_exact(x.numpy(), ids.numpy(), cpu[0], cpu[1], group)
    tol_h = _h_tolerance(cpu, ids.numpy(), x.numpy(), g_ex, u_ex, group) + 2 * _ulp16(h_ref.astype(np.float64))
    _, bar = oracle.moe_down_exact(h_ref, ids.numpy(), w.numpy(), cpu[2], group)
    carried = np.zeros((ntok, hidden))
    for t in range(ntok):
        for k in range(top_k):
            dw = oracle.expert_f16(cpu[2], int(ids[t, k]), group).astype(np.float64)
            carried[t] += abs(float(w[t, k])) * np.linalg.norm(dw, axis=1) * np.linalg.norm(tol_h[t, k])
    ref64 = ref.astype(np.float64)
    tol = bar[:, None] + carried + (top_k + 1) * _ulp16(ref64)
    got = y.float().cpu().numpy().astype(np.float64)
    err = np.abs(got - ref64)
    assert np.isfinite(got).all()
    assert (err <= tol).all(), f"worst err/bar {(err / tol).max():.3f}"


def test_moe_expert_parallel_partials(gdsq, cuda):
    """Experts split over 4 'ranks': each rank's fp32 partial covers only its
    resident experts, h entries of other ranks' slots stay untouched, and the
    partials add up to the single-rank result."""
    experts, hidden, inter, group, ntok, top_k, ws = 16, 2048, 512, 128, 3, 8, 4
    cpu, dev = _stacks(experts, hidden, inter, group, seed=5, device=cuda)
    ids, w = _routing(ntok, top_k, experts, seed=9)
    x = synth.activations(ntok, hidden, seed=4).to(cuda)
    idc, wc = ids.to(cuda), w.to(cuda)
    full = gdsq.moe_down(dev[2], gdsq.moe_gate_up(dev[0], dev[1], x, idc, group), idc, wc, group,
                         flags=gdsq.MOE_OUT_F32)
    per = experts // ws
    total = torch.zeros_like(full)
    for r in range(ws):
        sl = slice(r * per, (r + 1) * per)
        loc = [tuple(t[sl].contiguous() for t in m) for m in dev]
        h = torch.full((ntok, top_k, inter), 7.0, dtype=torch.float16, device=cuda)
        gdsq.moe_gate_up(loc[0], loc[1], x, idc, group, expert_first=r * per, expert_total=experts, out=h)
        part = gdsq.moe_down(loc[2], h, idc, wc, group, expert_first=r * per, expert_total=experts,
                             flags=gdsq.MOE_OUT_F32)
        resident = ((ids >= r * per) & (ids < (r + 1) * per)).to(cuda)
        assert bool((h[~resident] == 7.0).all()), "h of a non-resident slot was written"
        total += part
    torch.cuda.synchronize()
    assert gdsq.device_error(0) == 0
    scale = full.abs().max().item()
    assert torch.allclose(total, full, rtol=1e-5, atol=1e-5 * scale), (total - full).abs().max().item()


def test_moe_accumulate_and_fp16_output(gdsq, cuda):
    experts, hidden, inter, group, ntok, top_k = 4, 1024, 256, 128, 2, 2
    cpu, dev = _stacks(experts, hidden, inter, group, seed=21, device=cuda)
    ids, w = _routing(ntok, top_k, experts, seed=2)
    x = synth.activations(ntok, hidden, seed=6).to(cuda)
    idc, wc = ids.to(cuda), w.to(cuda)
    h = gdsq.moe_gate_up(dev[0], dev[1], x, idc, group)
    y32 = gdsq.moe_down(dev[2], h, idc, wc, group, flags=gdsq.MOE_OUT_F32)
    base = torch.randn(ntok, hidden, device=cuda)
    acc = base.clone()
    gdsq.moe_down(dev[2], h, idc, wc, group, out=acc, flags=gdsq.MOE_OUT_F32 | gdsq.MOE_ACCUMULATE)
    y16 = gdsq.moe_down(dev[2], h, idc, wc, group)
    torch.cuda.synchronize()
    assert torch.allclose(acc, base + y32, rtol=1e-6, atol=1e-6)
    assert torch.equal(y16, y32.half())


def test_moe_generic_path(gdsq, cuda):
    """Shapes off the TMA path (hidden not a multiple of 256) take the
    warp-per-row kernels; same bars."""
    experts, hidden, inter, group, ntok, top_k = 5, 960, 192, 64, 2, 3
    cpu, dev = _stacks(experts, hidden, inter, group, seed=31, device=cuda)
    ids, w = _routing(ntok, top_k, experts, seed=8)
    x = synth.activations(ntok, hidden, seed=12)
    h = gdsq.moe_gate_up(dev[0], dev[1], x.to(cuda), ids.to(cuda), group)
    y = gdsq.moe_down(dev[2], h, ids.to(cuda), w.to(cuda), group)
    torch.cuda.synchronize()
    _check_h(h, cpu, ids.numpy(), x.numpy(), group)
    _check_y(y, h.cpu().numpy(), cpu, ids.numpy(), w.numpy(), group)


def test_moe_bad_expert_id_sets_error_bit(gdsq, cuda):
    """An id outside 0..E-1 is skipped by the kernels and reported through the
    device error word (bit 4); the other slots are still computed."""
    experts, hidden, inter, group = 4, 1024, 256, 128
    cpu, dev = _stacks(experts, hidden, inter, group, seed=41, device=cuda)
    ids = torch.tensor([[1, experts + 3]], dtype=torch.int32)
    w = torch.tensor([[0.75, 0.25]], dtype=torch.float16)
    x = synth.activations(1, hidden, seed=1)
    gdsq.device_error(0, clear=True)
    h = gdsq.moe_gate_up(dev[0], dev[1], x.to(cuda), ids.to(cuda), group)
    y = gdsq.moe_down(dev[2], h, ids.to(cuda), w.to(cuda), group)
    torch.cuda.synchronize()
    assert gdsq.device_error(0, clear=True) & 4
    good = torch.tensor([[1]], dtype=torch.int32)
    _check_y(y, h.cpu().numpy()[:, :1], cpu, good.numpy(), w.numpy()[:, :1], group)


def test_moe_host_validation(gdsq, cuda):
    from gdsllm_b200 import GdsqError
    cpu, dev = _stacks(2, 512, 256, 128, seed=1, device=cuda)
    x = synth.activations(1, 512).to(cuda)
    ids = torch.zeros(1, 65, dtype=torch.int32, device=cuda)
    with pytest.raises(GdsqError, match="top_k"):
        gdsq.moe_gate_up(dev[0], dev[1], x, ids, 128)
    ids = torch.zeros(1, 2, dtype=torch.int32, device=cuda)
    with pytest.raises(GdsqError, match="resident experts"):
        gdsq.moe_gate_up(dev[0], dev[1], x, ids, 128, expert_first=1, expert_total=2)
    with pytest.raises(GdsqError, match="group_size"):
        gdsq.moe_gate_up(dev[0], dev[1], x, ids, 96)


def test_fused_moe_binding_shapes(ext, cuda):
    """The binding takes the reference's routing tensors as they come out of
    moe_route ((B, S, k) int64 ids, fp16 weights) and returns x's shape."""
    experts, hidden, inter, group = 8, 1024, 512, 128
    cpu, dev = _stacks(experts, hidden, inter, group, seed=51, device=cuda)
    ids, w = _routing(1, 4, experts, seed=1)
    x = synth.activations(1, hidden, seed=2).view(1, 1, hidden).to(cuda)
    y = ext.fused_moe_affine_q4(x, ids.view(1, 1, 4).long().to(cuda), w.view(1, 1, 4).to(cuda),
                                dev[0], dev[1], dev[2], group_size=group)
    assert y.shape == (1, 1, hidden) and y.dtype == torch.float16
    with pytest.raises(RuntimeError, match="accumulate"):
        ext.fused_moe_affine_q4(x, ids.to(cuda), w.to(cuda), dev[0], dev[1], dev[2], accumulate=True)
    with pytest.raises(RuntimeError, match="weight shape"):
        ext.fused_moe_affine_q4(x, ids.to(cuda), w.to(cuda), dev[0], dev[0], dev[0])


def test_moe_layer_decode_matches_reference_layer(cuda):
    """gdsllm_b200.moe.moe_mlp_decode (routing, routed experts, shared expert,
    clamp) against oracle.moe_mlp_reference on the same routing."""
    from gdsllm_b200 import moe
    experts, hidden, inter, group, top_k = 16, 4096, 1024, 128, 10
    cpu, dev = _stacks(experts, hidden, inter, group, seed=91, device=cuda)
    scpu, sdev = _stacks(1, hidden, inter, group, seed=95, device=cuda)
    g = torch.Generator().manual_seed(4)
    router = (torch.randn(experts, hidden, generator=g) / hidden ** 0.5).half()
    sgate = (torch.randn(1, hidden, generator=g) / hidden ** 0.5).half()
    layer = moe.MoeLayer(router=router.to(cuda), gate=dev[0], up=dev[1], down=dev[2], group=group,
                         shared=sdev, shared_gate=sgate.to(cuda))
    x = synth.activations(1, hidden, seed=6).view(1, 1, hidden)
    y = moe.moe_mlp_decode(x.to(cuda), layer, top_k)
    ids, w, _ = moe.route_fused(x.view(1, hidden).to(cuda), layer, top_k)  # the routing moe_mlp_decode used
    torch.cuda.synchronize()
    ref = oracle.moe_mlp_reference(x.view(1, hidden).numpy(), ids.cpu().numpy(), w.cpu().numpy(), *cpu, group,
                                   shared=scpu, shared_gate_w=sgate.numpy())
    # bar: the routed bar of the decode-sequence test plus the shared expert's
    # own GEMV bar (one more expert, weight sigmoid <= 1)
    idn = np.concatenate([ids.cpu().numpy(), np.zeros((1, 1), np.int32)], axis=1)
    got = y.view(1, hidden).float().cpu().numpy().astype(np.float64)
    h_ref, _, _ = oracle.moe_gate_up_exact(x.view(1, hidden).numpy(), ids.cpu().numpy(), cpu[0], cpu[1], group)
    _, bar = oracle.moe_down_exact(h_ref, ids.cpu().numpy(), w.cpu().numpy(), cpu[2], group)
    hs, _, _ = oracle.moe_gate_up_exact(x.view(1, hidden).numpy(), np.zeros((1, 1), np.int32), scpu[0], scpu[1], group)
    _, sbar = oracle.moe_down_exact(hs, np.zeros((1, 1), np.int32), np.ones((1, 1), np.float16), scpu[2], group)
    scale = np.abs(ref.astype(np.float64)).max()
    tol = 3 * (bar + sbar)[:, None] + (top_k + 3) * _ulp16(ref.astype(np.float64)) + 2e-3 * scale
    err = np.abs(got - ref.astype(np.float64))
    assert np.isfinite(got).all()
    assert (err <= tol).all(), f"worst err/bar {(err / tol).max():.3f}"
    assert idn.shape == (1, top_k + 1)
    # the residual add inside the down launch: the bits of x + moe(x) in fp16
    xd = x.to(cuda)
    xr = moe.moe_mlp_decode(xd, layer, top_k, add_residual=True)
    assert torch.equal(xr, xd + y)
    with pytest.raises(RuntimeError, match="residual"):
        moe.moe_partial(xd.view(1, hidden), ids, w, layer, out_fp32=True, residual=xd.view(1, hidden))


@pytest.mark.parametrize("ntok,top_k", [(1, 10), (8, 10), (3, 4)])
def test_moe_shared_expert_slot(gdsq, cuda, ntok, top_k):
    """The shared expert as slot top_k of the same two launches equals the
    routed sum plus sigmoid-weighted shared expert (qwen_moe.py:497-510)."""
    experts, hidden, inter, group = 16, 2048, 512, 128
    cpu, dev = _stacks(experts, hidden, inter, group, seed=61 + ntok, device=cuda)
    scpu, sdev = _stacks(1, hidden, inter, group, seed=71, device=cuda)
    ids, w = _routing(ntok, top_k, experts, seed=ntok)
    sw = torch.rand(ntok, generator=torch.Generator().manual_seed(2)).half()
    x = synth.activations(ntok, hidden, seed=9)
    h = gdsq.moe_gate_up(dev[0], dev[1], x.to(cuda), ids.to(cuda), group, shared=(sdev[0], sdev[1]))
    y = gdsq.moe_down(dev[2], h, ids.to(cuda), w.to(cuda), group, flags=gdsq.MOE_OUT_F32, shared=sdev[2],
                      shared_weights=sw.to(cuda))
    torch.cuda.synchronize()
    assert h.shape == (ntok, top_k + 1, inter)
    _check_h(h[:, :top_k], cpu, ids.numpy(), x.numpy(), group)
    zero = np.zeros((ntok, 1), np.int32)
    _check_h(h[:, top_k:], scpu, zero, x.numpy(), group)
    hn = h.cpu().numpy()
    y_r, bar_r = oracle.moe_down_exact(hn[:, :top_k], ids.numpy(), w.numpy(), cpu[2], group)
    y_s, bar_s = oracle.moe_down_exact(hn[:, top_k:], zero, sw.numpy().reshape(-1, 1), scpu[2], group)
    got = y.cpu().numpy().astype(np.float64)
    err = np.abs(got - (y_r + y_s))
    tol = (bar_r + bar_s)[:, None] + 1e-6 * np.abs(y_r + y_s).max()
    assert (err <= tol).all(), f"worst err/bar {(err / tol).max():.3f}"


def test_moe_clamp_flag(gdsq, cuda):
    experts, hidden, inter, group = 2, 1024, 256, 128
    cpu, dev = _stacks(experts, hidden, inter, group, seed=5, device=cuda)
    ids = torch.tensor([[0, 1]], dtype=torch.int32)
    w = torch.tensor([[30000.0, 30000.0]], dtype=torch.float16)   # drives |y| past the fp16 range
    x = (synth.activations(1, hidden, seed=3) * 8).half()
    h = gdsq.moe_gate_up(dev[0], dev[1], x.to(cuda), ids.to(cuda), group)
    y_inf = gdsq.moe_down(dev[2], h, ids.to(cuda), w.to(cuda), group)
    y_cl = gdsq.moe_down(dev[2], h, ids.to(cuda), w.to(cuda), group, flags=gdsq.MOE_CLAMP)
    torch.cuda.synchronize()
    assert torch.isinf(y_inf).any(), "test input does not overflow fp16"
    assert torch.isfinite(y_cl).all() and y_cl.abs().max().item() == 65504.0


@pytest.mark.parametrize("ntok,experts,top_k", [(1, 512, 10), (8, 512, 10), (5, 64, 7), (4, 512, 32), (3, 33, 1),
                                                (2, 128, 40), (3, 1000, 12)])
def test_moe_route_kernel_matches_torch_topk(gdsq, cuda, ntok, experts, top_k):
    """Top-k set exactly as torch.topk on the same fp16 logits (ties at the
    boundary excepted, there any equal logit is a valid pick), softmax weights
    and the shared gate within fp16 rounding."""
    import torch.nn.functional as F
    hidden = 4096
    g = torch.Generator(device=cuda).manual_seed(ntok + experts)
    router = (torch.randn(experts, hidden, generator=g, device=cuda) / hidden ** 0.5).half()
    sgate = (torch.randn(hidden, generator=g, device=cuda) / hidden ** 0.5).half()
    x = torch.randn(ntok, hidden, generator=g, device=cuda).half()
    logits = F.linear(x, router)
    ids, w, sw = gdsq.moe_route(logits, top_k, x, sgate)
    tv, ti = torch.topk(logits, top_k, dim=-1)
    tw = F.softmax(tv.float(), dim=-1).half()
    tsw = torch.sigmoid(F.linear(x, sgate.view(1, -1))).view(-1)
    torch.cuda.synchronize()
    lg = logits.float().cpu()
    for t in range(ntok):
        mine, ref = set(ids[t].tolist()), set(ti[t].tolist())
        chosen = lg[t, ids[t].long().cpu()]
        rest = torch.ones(experts, dtype=torch.bool)
        rest[ids[t].long().cpu()] = False
        assert lg[t][rest].max() <= chosen.min(), "not a top-k set"
        if mine != ref:  # only an exact tie at the boundary may differ
            boundary = tv[t, -1].float().item()
            assert all(abs(lg[t, e].item() - boundary) == 0 for e in mine ^ ref), (t, mine ^ ref)
        # weights follow the ids' order: compare through the logits they belong to
        assert torch.equal(lg[t, ids[t].long().cpu()], tv[t].float().cpu()), "order differs from torch.topk"
    assert (w.float() - tw.float()).abs().max().item() <= 2 * 2 ** -11
    assert (sw.float() - tsw.float()).abs().max().item() <= 2 * 2 ** -11


@pytest.mark.parametrize("ntok,experts,top_k,shared", [(1, 512, 10, True), (8, 512, 10, True), (16, 64, 7, False),
                                                       (3, 33, 1, True)])
def test_fused_router_matches_linear_and_route(gdsq, cuda, ntok, experts, top_k, shared):
    """gdsq_moe_router: logits within an fp16 ulp of the fp64 product (fp32
    sums, one rounding), and exactly the ids, weights and
    shared gate that gdsq_moe_route gives on those logits; twice in a row
    (the completion counter resets itself)."""
    from gdsllm_b200 import moe
    hidden = 4096
    g = torch.Generator().manual_seed(ntok * 100 + experts)
    router = (torch.randn(experts, hidden, generator=g) / hidden ** 0.5).half().to(cuda)
    sgate = (torch.randn(hidden, generator=g) / hidden ** 0.5).half().to(cuda) if shared else None
    x = synth.activations(ntok, hidden, seed=ntok + 5).to(cuda)
    fr = moe.FusedRouter(router, sgate)  # called directly: every token count the kernel takes (<= 16)
    for _ in range(2):
        ids, w, sw = fr(x, top_k)
        lg = fr.logits[:ntok]
        # against the fp64 product: one fp16 rounding of an fp32 sum (cuBLAS's
        # F.linear may reduce in lower precision, so it is not the yardstick)
        exact = x.double() @ router.double().T
        err = (lg[:, :experts].double() - exact).abs()
        assert (err <= exact.abs() * 2 ** -10 + 2 ** -24 * 4096).all(), err.max().item()
        if shared:
            ex_g = x.double() @ sgate.double()
            assert ((lg[:, experts].double() - ex_g).abs() <= ex_g.abs() * 2 ** -10 + 2 ** -14).all()
        ids2, w2, sw2 = gdsq_route_on(lg[:, :experts].contiguous(), top_k, x if shared else None, sgate)
        assert torch.equal(ids, ids2) and torch.equal(w, w2)
        if shared:
            # the fused kernel's gate is sigmoid of its own fp16 logit of x . g
            expect = torch.sigmoid(lg[:, experts].float()).half()
            assert (sw.float() - expect.float()).abs().max().item() <= 2 ** -10
    torch.cuda.synchronize()
    assert int(fr.counter.item()) == 0
    assert capi_device_error() == 0


def gdsq_route_on(logits, top_k, x, g):
    from gdsllm_b200 import moe
    return moe._ext().moe_route(logits, top_k, x, g)


def capi_device_error():
    from gdsllm_b200 import capi
    return capi.device_error(0)
