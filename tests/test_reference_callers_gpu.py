"""The drop-in claim, tested on the reference's own Python callers.

GdsLLM's llama.py, scheduler.py (CachedScheduler) and qwen_moe.py are run
unchanged, from the reference package installed into baseline/_ref, on a
synthetic model directory written in the converter's layout.  Each run goes
once through this build's gds_io_ext (install_as_reference_module) and once
through a stand-in module that runs GdsLLM's own CUDA kernels compiled
unchanged (oracle/ref_module.py, oracle/_ref); the results must agree:

* prefill (dequant_gguf + F.linear in the callers): identical bits, since
  the dequantized weights are bit-exact and the rest is the same torch code;
* decode (fused GEMVs): logits within the GEMV bar carried through the
  layers, and the same greedy tokens;
* MoE decode (moe_route + moe_mlp_selective with experts from load_experts):
  within the GEMV bars.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
REF_PKG = ROOT / "baseline" / "_ref"


@pytest.fixture(scope="module")
def reference():
    if not (REF_PKG / "gdsllm" / "runtime" / "scheduler.py").exists():
        pytest.skip("the reference package is not installed in baseline/_ref (python oracle/build.py)")
    from oracle import reference_kernels as refk
    if not refk.available():
        pytest.skip("oracle/_ref (the reference kernels) is not built")
    if str(REF_PKG) not in sys.path:
        sys.path.insert(0, str(REF_PKG))
    import gdsllm.runtime  # noqa: F401  (the package only; its extension is never imported)
    from gdsllm.runtime import kv_cache, qwen_moe, scheduler, torch_bridge
    return {"scheduler": scheduler, "kv_cache": kv_cache, "qwen_moe": qwen_moe, "torch_bridge": torch_bridge}


def _use(module: str):
    if module == "ours":
        import gdsllm_b200
        return gdsllm_b200.install_as_reference_module()
    from oracle import ref_module
    return ref_module.install()


CFG = dict(layers=2, hidden=512, heads=4, kv_heads=2, ffn=1536, vocab=2048, max_seq_len=64)


def _generate(reference, model_dir, module, prompt, steps, cuda):
    _use(module)
    sched_mod, kv_mod = reference["scheduler"], reference["kv_cache"]
    logits_seq = []
    with sched_mod.CachedScheduler(str(model_dir), device="cuda:0") as sched:
        c = sched.config
        kv = kv_mod.KVCache(c["num_layers"], c["num_kv_heads"], c["head_dim"], c["max_seq_len"], device=cuda)
        logits = sched.forward(prompt.view(1, -1), kv_cache=kv, start_pos=0)
        prefill = logits[0, -1].float().clone()
        tok = logits[0, -1].argmax()
        tokens = [int(tok)]
        pos = prompt.numel()
        for _ in range(steps):
            logits = sched.forward(tok.view(1, 1), kv_cache=kv, start_pos=pos)
            logits_seq.append(logits[0, -1].float().clone())
            tok = logits[0, -1].argmax()
            tokens.append(int(tok))
            pos += 1
    torch.cuda.synchronize()
    return prefill, logits_seq, tokens


@pytest.mark.parametrize("body,lm_head,embed", [("q4_0", "q8_0", "q4_0"), ("q8_0", "q4_0", "f16")])
def test_cached_scheduler_runs_unchanged(reference, tmp_path, cuda, body, lm_head, embed):
    from gdsllm_b200 import synth
    synth.write_llama_model_dir(tmp_path / "m", body=body, lm_head=lm_head, embed=embed, norm_jitter=0.2, seed=3,
                                **CFG)
    prompt = torch.randint(0, CFG["vocab"], (12,), generator=torch.Generator().manual_seed(5)).to(cuda)
    p_ours, d_ours, t_ours = _generate(reference, tmp_path / "m", "ours", prompt, 8, cuda)
    p_ref, d_ref, t_ref = _generate(reference, tmp_path / "m", "reference", prompt, 8, cuda)
    # prefill: bit-exact dequant + the same torch ops
    assert torch.equal(p_ours, p_ref), "prefill logits differ"
    # decode: fp32 GEMV sums in another order, fp16 outputs; two layers deep
    for i, (a, b) in enumerate(zip(d_ours, d_ref)):
        scale = b.abs().max().item()
        err = (a - b).abs().max().item()
        assert err <= 2e-2 * scale + 1e-2, f"decode step {i}: max |logit diff| {err} (scale {scale})"
    for i, (a, b) in enumerate(zip(t_ours, t_ref)):
        if a != b:  # only a near-tie at the top may flip; the two candidates' logits must be within the bar
            top = torch.topk(d_ref[i - 1], 2).values
            assert (top[0] - top[1]).abs().item() <= 2e-2 * top[0].abs().item() + 1e-2, f"token {i}: {a} vs {b}"
            break


def test_transformer_block_decode_matches(reference, tmp_path, cuda):
    """llama.transformer_block on one decode position, both modules, the same
    layer tensors from ModelWeights.load_layer."""
    from gdsllm_b200 import synth
    synth.write_llama_model_dir(tmp_path / "m", norm_jitter=0.2, seed=4, **CFG)
    llama = sys.modules["gdsllm.runtime.llama"]
    tb = reference["torch_bridge"]
    outs = []
    for module in ("ours", "reference"):
        _use(module)
        mw = tb.ModelWeights(str(tmp_path / "m"))
        mw.init_gds()
        tensors, handle = mw.load_layer(0)
        freqs = llama.precompute_freqs_cis(CFG["hidden"] // CFG["heads"], CFG["max_seq_len"], device=cuda)
        x = torch.randn(1, 1, CFG["hidden"], generator=torch.Generator().manual_seed(9)).half().to(cuda)
        with torch.inference_mode():
            y = llama.transformer_block(x, tensors, freqs[3:4], None, CFG["heads"], CFG["kv_heads"])
        torch.cuda.synchronize()
        outs.append(y.float())
        mw.shutdown_gds()
        del tensors, handle
    scale = outs[1].abs().max().item()
    assert (outs[0] - outs[1]).abs().max().item() <= 1e-2 * scale + 1e-3


def test_moe_mlp_selective_matches(reference, tmp_path, cuda):
    """qwen_moe.moe_route + moe_mlp_selective (the decode branch, one
    fused GEMV per expert projection) with experts from
    ModelWeights.load_experts, through both modules: the same routing and
    the same MLP output within the GEMV bars."""
    from gdsllm_b200 import synth
    E, H, I = 32, 2048, 512
    synth.write_moe_layer_dir(tmp_path / "moe", experts=E, hidden=H, inter=I, seed=2)
    qm, tb = reference["qwen_moe"], reference["torch_bridge"]
    x = torch.randn(1, 1, H, generator=torch.Generator().manual_seed(11)).half().to(cuda)
    res = {}
    for module in ("ours", "reference"):
        _use(module)
        mw = tb.ModelWeights(str(tmp_path / "moe"))
        mw.init_gds()
        weights, handles = mw.load_layer_partial(0)
        with torch.inference_mode():
            idx, w, uniq = qm.moe_route(x, weights, 10)
            experts, eh = mw.load_experts(0, uniq)
            y = qm.moe_mlp_selective(x, weights, experts, idx, w, 10)
        torch.cuda.synchronize()
        res[module] = (idx.clone(), y.float())
        mw.shutdown_gds()
        del weights, handles, experts, eh
    assert torch.equal(res["ours"][0], res["reference"][0]), "routing differs"
    scale = res["reference"][1].abs().max().item()
    assert (res["ours"][1] - res["reference"][1]).abs().max().item() <= 1e-2 * scale + 1e-3


@pytest.mark.parametrize("body,lm_head,embed", [("q4_0", "q8_0", "q4_0"), ("q4_0", "q4_0", "q8_0")])
def test_scheduler_ops_replace_the_full_table_paths(reference, tmp_path, cuda, body, lm_head, embed):
    """gdsllm_b200.scheduler_ops installed into the reference scheduler: the
    embedding (row gather, bit-exact) and the lm_head (fused GEMV at decode
    and for prompts of up to 16 positions) give the unpatched scheduler's
    tokens, with logits within the GEMV bar."""
    from gdsllm_b200 import scheduler_ops, synth
    synth.write_llama_model_dir(tmp_path / "m", body=body, lm_head=lm_head, embed=embed, norm_jitter=0.2, seed=7,
                                **CFG)
    prompt = torch.randint(0, CFG["vocab"], (10,), generator=torch.Generator().manual_seed(6)).to(cuda)
    sched_mod = reference["scheduler"]
    saved = (sched_mod._embed_tokens, sched_mod._lm_head_proj)
    try:
        p_ref, d_ref, t_ref = _generate(reference, tmp_path / "m", "ours", prompt, 6, cuda)
        scheduler_ops.install(sched_mod)
        p_new, d_new, t_new = _generate(reference, tmp_path / "m", "ours", prompt, 6, cuda)
    finally:
        sched_mod._embed_tokens, sched_mod._lm_head_proj = saved
    for a, b in zip([p_new] + d_new, [p_ref] + d_ref):
        scale = b.abs().max().item()
        assert (a - b).abs().max().item() <= 2e-2 * scale + 1e-2
    assert t_new == t_ref


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_embedding_gguf_is_dequant_then_gather(cuda, fmt):
    import torch.nn.functional as F
    import gdsllm_b200
    from gdsllm_b200 import capi, synth
    ext = gdsllm_b200.ext()
    V, H = 1000, 512
    w = (synth.q4_0_weight if fmt == "q4_0" else synth.q8_0_weight)(V, H, seed=3).to(cuda)
    h = ext.handle_from_tensor(w.reshape(-1))
    ids = torch.tensor([[0, 5, 999, 5], [17, 998, 1, 0]], dtype=torch.long, device=cuda)
    full = ext.dequant_gguf(h, [V, H], fmt, 0)
    got = ext.embedding_gguf(h, ids, [V, H], fmt, 0)
    torch.cuda.synchronize()
    assert got.shape == (2, 4, H)
    assert torch.equal(got, F.embedding(ids, full))
    bad = ext.embedding_gguf(h, torch.tensor([3, V], dtype=torch.long, device=cuda), [V, H], fmt, 0)
    torch.cuda.synchronize()
    assert torch.equal(bad[0], full[3]) and (bad[1] == 0).all()
    assert capi.device_error(0, clear=True) & 4
