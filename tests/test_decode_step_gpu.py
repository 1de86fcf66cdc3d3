"""The graph-captured decode step (gdsllm_b200.decode_step) and its kernels.

Each decode kernel is checked against the torch code it replaces, restated
here in plain torch exactly as GdsLLM writes it (gdsllm/runtime/llama.py:
rms_norm 17-23, apply_rotary_emb 83-105, attention 228-242, mlp 248-252;
kv_cache.py:44-67).  Then the whole step, captured as a CUDA graph, is run
against GdsLLM's own CachedScheduler (the reference package in baseline/_ref,
unchanged) on a synthetic model: the same greedy tokens, and logits within
the bar the decode GEMVs allow.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch
import torch.nn.functional as F

from gdsllm_b200 import capi

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
REF_PKG = ROOT / "baseline" / "_ref"


def ulps(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|a - b| in fp16 units in the last place of b (finite values)."""
    a, b = a.float(), b.float()
    e = torch.floor(torch.log2(b.abs().clamp_min(2.0 ** -14)))
    return (a - b).abs() / torch.exp2(e - 10)


# ---- torch restatements of the reference's decode ops -----------------------

def rms_norm_ref(x, weight, eps):
    dt = x.dtype
    x = x.float()
    norm = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return (x * norm).to(dt) * weight


def rope_ref(xq, xk, freqs_cis):
    xq_c = torch.view_as_complex(xq.float().reshape(*xq.shape[:-1], -1, 2))
    xk_c = torch.view_as_complex(xk.float().reshape(*xk.shape[:-1], -1, 2))
    f = freqs_cis.unsqueeze(0).unsqueeze(2)
    return (torch.view_as_real(xq_c * f).flatten(-2).type_as(xq),
            torch.view_as_real(xk_c * f).flatten(-2).type_as(xk))


def attention_ref(xq, keys, values, n_rep):
    """xq [1, nh, 1, d], keys/values [1, nkv, L, d] fp16."""
    keys = keys[:, :, None].expand(-1, -1, n_rep, -1, -1).reshape(1, -1, *keys.shape[2:])
    values = values[:, :, None].expand(-1, -1, n_rep, -1, -1).reshape(1, -1, *values.shape[2:])
    scores = torch.matmul(xq, keys.transpose(-2, -1)) / (xq.shape[-1] ** 0.5)
    scores = F.softmax(scores.float(), dim=-1).type_as(xq)
    return torch.matmul(scores, values)


def freqs_cis_ref(head_dim, seq_len, theta=10000.0, device=None):
    freqs = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))
    t = torch.arange(seq_len, device=device)
    freqs = torch.outer(t, freqs)
    return torch.polar(torch.ones_like(freqs), freqs)


# ---- kernels ----------------------------------------------------------------

@pytest.mark.parametrize("hidden", [512, 4096, 8192])
def test_add_rmsnorm_matches_reference_formula(cuda, hidden):
    g = torch.Generator().manual_seed(hidden)
    h = torch.randn(hidden, generator=g).half().to(cuda)
    d = torch.randn(hidden, generator=g).half().to(cuda)
    w = (1 + 0.2 * torch.randn(hidden, generator=g)).half().to(cuda)
    # first layer: no residual
    x = capi.add_rmsnorm(h, w, 1e-5)
    ref = rms_norm_ref(h.view(1, 1, -1), w, 1e-5).view(-1)
    assert ulps(x, ref).max().item() <= 1
    assert (x != ref).float().mean().item() < 0.01
    # residual add in place, then the norm
    h2 = h.clone()
    x2 = capi.add_rmsnorm(h2, w, 1e-5, delta=d)
    s = h + d
    assert torch.equal(h2, s), "the residual add is one fp16 rounding of the exact sum"
    ref2 = rms_norm_ref(s.view(1, 1, -1), w, 1e-5).view(-1)
    assert ulps(x2, ref2).max().item() <= 1


@pytest.mark.parametrize("nh,nkv,hd", [(32, 32, 128), (8, 2, 64), (64, 8, 128)])
def test_rope_kv_matches_reference(cuda, nh, nkv, hd):
    max_seq = 96
    g = torch.Generator().manual_seed(nh * 7 + nkv)
    q = torch.randn(nh * hd, generator=g).half().to(cuda)
    k = torch.randn(nkv * hd, generator=g).half().to(cuda)
    v = torch.randn(nkv * hd, generator=g).half().to(cuda)
    fc = freqs_cis_ref(hd, max_seq, device=cuda)
    freqs = torch.view_as_real(fc).contiguous()
    kc = torch.randn(nkv, max_seq, hd, generator=g).half().to(cuda)
    vc = torch.randn(nkv, max_seq, hd, generator=g).half().to(cuda)
    for p in (0, 1, 57, max_seq - 1):
        kc0, vc0 = kc.clone(), vc.clone()
        pos = torch.tensor([p], dtype=torch.int64, device=cuda)
        q_out = torch.empty_like(q)
        capi.rope_kv(q, k, v, q_out, freqs, pos, kc, vc, nh, nkv, hd, max_seq)
        rq, rk = rope_ref(q.view(1, 1, nh, hd), k.view(1, 1, nkv, hd), fc[p:p + 1])
        assert ulps(q_out.view(-1), rq.reshape(-1)).max().item() <= 1
        assert ulps(kc[:, p].reshape(-1), rk.reshape(-1)).max().item() <= 1
        assert torch.equal(vc[:, p].reshape(-1), v)
        others = torch.ones(max_seq, dtype=torch.bool, device=cuda)
        others[p] = False
        assert torch.equal(kc[:, others], kc0[:, others]) and torch.equal(vc[:, others], vc0[:, others])
    torch.cuda.synchronize()
    assert capi.device_error(0) == 0


@pytest.mark.parametrize("nh,nkv,hd,max_seq", [(32, 32, 128, 640), (8, 2, 64, 200), (64, 8, 128, 1024),
                                              (4, 4, 64, 3)])
def test_attention_decode_matches_reference(cuda, nh, nkv, hd, max_seq):
    g = torch.Generator().manual_seed(nh + max_seq)
    q = torch.randn(nh * hd, generator=g).half().to(cuda)
    kc = torch.randn(nkv, max_seq, hd, generator=g).half().to(cuda)
    vc = torch.randn(nkv, max_seq, hd, generator=g).half().to(cuda)
    for p in sorted({0, 1, max_seq // 2, max_seq - 1}):
        pos = torch.tensor([p], dtype=torch.int64, device=cuda)
        out = capi.attention_decode(q, kc, vc, pos, nh, nkv, hd, max_seq)
        ref = attention_ref(q.view(1, nh, 1, hd), kc[None, :, : p + 1], vc[None, :, : p + 1], nh // nkv).view(-1)
        # fp64 of the same math: both may differ from it by their own roundings
        qd, kd, vd = q.double().view(nh, hd), kc.double(), vc.double()
        kvh = torch.arange(nh, device=cuda) // (nh // nkv)
        sc = torch.einsum("hd,hld->hl", qd, kd[kvh, : p + 1]) / hd ** 0.5
        exact = torch.einsum("hl,hld->hd", torch.softmax(sc, -1), vd[kvh, : p + 1]).reshape(-1)
        err_ours = (out.double() - exact).abs().max().item()
        err_ref = (ref.double() - exact).abs().max().item()
        assert err_ours <= 2 * err_ref + 2e-3, f"pos {p}: error {err_ours:.2e} vs reference {err_ref:.2e}"
        assert (out.float() - ref.float()).abs().max().item() <= 4e-3 + 4e-3 * ref.float().abs().max().item()
    torch.cuda.synchronize()
    assert capi.device_error(0) == 0


@pytest.mark.parametrize("nh,nkv,hd,max_seq", [(32, 32, 128, 640), (8, 2, 64, 200), (64, 8, 128, 1024)])
def test_attention_with_rope_folded_in(cuda, nh, nkv, hd, max_seq):
    """gdsq_attention_decode_rope_f16 = rope_kv then attention_decode: the
    same cache rows (bit for bit) and outputs within the attention bar."""
    g = torch.Generator().manual_seed(nh * 3 + max_seq)
    q = torch.randn(nh * hd, generator=g).half().to(cuda)
    k = torch.randn(nkv * hd, generator=g).half().to(cuda)
    v = torch.randn(nkv * hd, generator=g).half().to(cuda)
    freqs = torch.view_as_real(freqs_cis_ref(hd, max_seq, device=cuda)).contiguous()
    kc = torch.randn(nkv, max_seq, hd, generator=g).half().to(cuda)
    vc = torch.randn(nkv, max_seq, hd, generator=g).half().to(cuda)
    for p in sorted({0, 1, max_seq // 3, max_seq - 1}):
        pos = torch.tensor([p], dtype=torch.int64, device=cuda)
        kc1, vc1 = kc.clone(), vc.clone()
        q_rot = torch.empty_like(q)
        capi.rope_kv(q, k, v, q_rot, freqs, pos, kc1, vc1, nh, nkv, hd, max_seq)
        ref = capi.attention_decode(q_rot, kc1, vc1, pos, nh, nkv, hd, max_seq)
        kc2, vc2 = kc.clone(), vc.clone()
        out = capi.attention_decode_rope(q, k, v, freqs, pos, kc2, vc2, nh, nkv, hd, max_seq)
        assert torch.equal(kc1, kc2) and torch.equal(vc1, vc2), f"pos {p}: cache rows differ"
        torch.testing.assert_close(out.float(), ref.float(), atol=4e-3, rtol=4e-3)
    torch.cuda.synchronize()
    assert capi.device_error(0) == 0


def test_attention_position_outside_cache_sets_error(cuda):
    q = torch.zeros(4 * 64, dtype=torch.float16, device=cuda)
    kc = torch.zeros(4, 8, 64, dtype=torch.float16, device=cuda)
    out = torch.full((4 * 64,), 7.0, dtype=torch.float16, device=cuda)
    capi.device_error(0)
    capi.attention_decode(q, kc, kc, torch.tensor([8], dtype=torch.int64, device=cuda), 4, 4, 64, 8, out=out)
    torch.cuda.synchronize()
    assert capi.device_error(0) & 4
    assert (out == 7.0).all(), "nothing is written for a bad position"


@pytest.mark.parametrize("n", [11008, 28672, 1000, 13])
def test_silu_mul_matches_reference(cuda, n):
    g = torch.Generator().manual_seed(n)
    gate = (3 * torch.randn(n, generator=g)).half().to(cuda)
    up = torch.randn(n, generator=g).half().to(cuda)
    out = capi.silu_mul(gate, up)
    ref = F.silu(gate) * up
    assert ulps(out, ref).max().item() <= 1
    assert (out != ref).float().mean().item() < 1e-3


def test_argmax_first_index_and_position(cuda):
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(32000, generator=g).half().to(cuda)
    tok = torch.zeros(1, dtype=torch.int64, device=cuda)
    pos = torch.tensor([41], dtype=torch.int64, device=cuda)
    capi.argmax(logits, tok, pos)
    assert int(tok) == int(torch.argmax(logits)) and int(pos) == 42
    logits[[123, 31999, 7777]] = 20.0  # ties: the first index wins
    capi.argmax(logits, tok)
    assert int(tok) == 123 and int(pos) == 42
    logits.fill_(float("-inf"))
    capi.argmax(logits, tok)
    assert int(tok) == 0


# ---- the whole step against GdsLLM's CachedScheduler --------------------------

@pytest.fixture(scope="module")
def reference():
    if not (REF_PKG / "gdsllm" / "runtime" / "scheduler.py").exists():
        pytest.skip("the reference package is not installed in baseline/_ref (python oracle/build.py)")
    if str(REF_PKG) not in sys.path:
        sys.path.insert(0, str(REF_PKG))
    from gdsllm.runtime import kv_cache, scheduler
    import gdsllm_b200
    gdsllm_b200.install_as_reference_module()
    return scheduler, kv_cache


@pytest.mark.parametrize("cfg,body,lm_head,embed", [
    (dict(layers=2, hidden=512, heads=4, kv_heads=2, ffn=1536, vocab=2048, max_seq_len=64), "q4_0", "q8_0", "f16"),
    (dict(layers=3, hidden=512, heads=8, kv_heads=8, ffn=1024, vocab=1000, max_seq_len=40), "q8_0", "q4_0", "q4_0"),
])
@pytest.mark.parametrize("fused", [True, False])
def test_graph_step_matches_cached_scheduler(reference, tmp_path, cuda, cfg, body, lm_head, embed, fused):
    """Prefill through CachedScheduler.forward, then 12 greedy tokens twice:
    by CachedScheduler.forward per token (the reference loop) and by replays
    of the captured GraphDecodeStep on a second KV cache prefilled the same
    way.  Same tokens; logits within the decode GEMV bar of the callers'
    test (the two paths use the same fused GEMVs, grouped differently)."""
    from gdsllm_b200 import synth
    from gdsllm_b200.decode_step import GraphDecodeStep
    sched_mod, kv_mod = reference
    synth.write_llama_model_dir(tmp_path / "m", body=body, lm_head=lm_head, embed=embed, norm_jitter=0.2, seed=11,
                                **cfg)
    prompt = torch.randint(0, cfg["vocab"], (1, 9), generator=torch.Generator().manual_seed(2))
    steps = 12
    with torch.inference_mode(), sched_mod.CachedScheduler(str(tmp_path / "m"), device="cuda:0") as sched:
        c = sched.config
        kvs = [kv_mod.KVCache(c["num_layers"], c["num_kv_heads"], c["head_dim"], c["max_seq_len"], device=cuda)
               for _ in range(2)]
        first = []
        for kv in kvs:
            logits = sched.forward(prompt.to(cuda), kv_cache=kv, start_pos=0)
            first.append(int(logits[0, -1].argmax()))
        assert first[0] == first[1]
        ref_tokens, ref_logits = [], []
        tok, pos = first[0], prompt.shape[1]
        for _ in range(steps):
            logits = sched.forward(torch.tensor([[tok]], device=cuda), kv_cache=kvs[0], start_pos=pos)
            ref_logits.append(logits[0, -1].float().clone())
            tok = int(logits[0, -1].argmax())
            ref_tokens.append(tok)
            pos += 1
        step = GraphDecodeStep.from_scheduler(sched, kvs[1], fused=fused)
        assert step.fused == fused
        step.reset(first[1], prompt.shape[1])
        step.capture()
        tokens, got = [], []
        for _ in range(steps):
            tokens.append(step.step())
            got.append(step.logits.float().clone())
        assert step.position() == prompt.shape[1] + steps
    torch.cuda.synchronize()
    assert capi.device_error(0) == 0
    for i, (a, b) in enumerate(zip(got, ref_logits)):
        scale = b.abs().max().item()
        err = (a - b).abs().max().item()
        assert err <= 2e-2 * scale + 1e-2, f"step {i}: max |logit diff| {err} (scale {scale})"
    for i, (a, b) in enumerate(zip(tokens, ref_tokens)):
        if a != b:  # only a near-tie at the top may flip
            top = torch.topk(ref_logits[i], 2).values
            assert (top[0] - top[1]).abs().item() <= 2e-2 * top[0].abs().item() + 1e-2, f"token {i}: {a} vs {b}"
            break
    # the graph wrote the same K/V rows the scheduler did, within the bar
    k0, k1 = kvs[0].k_cache.float(), kvs[1].k_cache.float()
    assert (k0 - k1).abs().max().item() <= 2e-2 * k0.abs().max().item() + 1e-2


def test_graph_step_launch_count_and_rejects(cuda, tmp_path, reference):
    """The number of kernels per token, and the inputs the step refuses."""
    from gdsllm_b200 import synth
    from gdsllm_b200.decode_step import GraphDecodeStep
    sched_mod, kv_mod = reference
    cfg = dict(layers=2, hidden=512, heads=4, kv_heads=2, ffn=1536, vocab=2048, max_seq_len=32)
    synth.write_llama_model_dir(tmp_path / "m", body="q4_0", lm_head="q8_0", embed="f16", seed=1, **cfg)
    with torch.inference_mode(), sched_mod.CachedScheduler(str(tmp_path / "m"), device="cuda:0") as sched:
        c = sched.config
        kv = kv_mod.KVCache(c["num_layers"], c["num_kv_heads"], c["head_dim"], c["max_seq_len"], device=cuda)
        step = GraphDecodeStep.from_scheduler(sched, kv, fused=False)
        assert step.launches_per_step() == 1 + 2 * 9 + 3
        assert GraphDecodeStep.from_scheduler(sched, kv).launches_per_step() == 1 + 2 * 8 + 3
        with pytest.raises(ValueError, match="outside the KV cache"):
            step.reset(0, 32)
        bad = kv_mod.KVCache(c["num_layers"] + 1, c["num_kv_heads"], c["head_dim"], c["max_seq_len"], device=cuda)
        with pytest.raises(ValueError, match="does not match"):
            GraphDecodeStep.from_scheduler(sched, bad)
