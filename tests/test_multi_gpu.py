"""Expert-parallel MoE and tensor-parallel GEMV on 2 and 4 GPUs over NCCL and
over NVLink peer memory, each rank's CUDA kernels + the exchange, against the
single-GPU result computed on every rank.  Each case is skipped unless that
many GPUs are visible (a box with one GPU cannot run NCCL ranks)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    from gdsllm_b200 import capi, ep, moe, synth, tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        res = {}
        # ---- expert parallel MoE layer ----
        experts, hidden, inter, group = 32, 2048, 512, 128

        def st(rows, cols, seed, e):
            return tuple(t.to(dev) for t in synth.affine_q4_weight(rows, cols, group=group, seed=seed, lead=(e,)))

        gate, up, down = st(inter, hidden, 1, experts), st(inter, hidden, 2, experts), st(hidden, inter, 3, experts)
        shared = (st(inter, hidden, 4, 1), st(inter, hidden, 5, 1), st(hidden, inter, 6, 1))
        g = torch.Generator().manual_seed(7)
        router = (torch.randn(experts, hidden, generator=g) / hidden ** 0.5).half().to(dev)
        sgate = (torch.randn(1, hidden, generator=g) / hidden ** 0.5).half().to(dev)
        first, count = ep.expert_range(rank, world, experts)
        local = moe.MoeLayer(router=router, gate=ep.local_stack(gate, rank, world), up=ep.local_stack(up, rank, world),
                             down=ep.local_stack(down, rank, world), group=group, expert_first=first,
                             expert_total=experts, shared=shared, shared_gate=sgate)
        x = synth.activations(8, hidden, seed=8).to(dev)
        y_ep = ep.ExpertParallelMoE(local, top_k=10)(x)
        full = moe.MoeLayer(router=router, gate=gate, up=up, down=down, group=group, shared=shared, shared_gate=sgate)
        y_one = moe.moe_mlp_decode(x, full, 10)
        res["ep"] = (y_ep.float() - y_one.float()).abs().max().item()
        res["ep_scale"] = y_one.float().abs().max().item()
        # the same layer with the partials summed over peer memory (rank-order
        # fp32 sums; two ranks add a + b exactly as NCCL does)
        from gdsllm_b200.p2p import PeerWordAllReduce
        words = PeerWordAllReduce(8 * hidden)
        y_ep_words = ep.ExpertParallelMoE(local, top_k=10, allreduce=words)(x)
        res["ep_words_equal"] = torch.equal(y_ep_words, y_ep)
        res["ep_words_diff"] = (y_ep_words.float() - y_ep.float()).abs().max().item()
        # the residual add inside the exchange kernel: x + layer(x) in fp16
        y_res = ep.ExpertParallelMoE(local, top_k=10, allreduce=words)(x, add_residual=True)
        res["ep_residual_equal"] = torch.equal(y_res, x + y_ep_words)
        worst_w = 0.0
        for it, (nel, dt) in enumerate([(8 * hidden, torch.float32), (1000, torch.float32), (4096, torch.float16),
                                        (8 * hidden, torch.float32), (7, torch.float16)]):
            t = torch.randn(nel, generator=torch.Generator().manual_seed(200 + 10 * it + rank)).to(dt).to(dev)
            ref = t.clone().float()   # .float() of an fp32 tensor is the tensor itself
            dist.all_reduce(ref)
            out = words(t.clone())
            worst_w = max(worst_w, ((out.float() - ref).abs() / (ref.abs() + 1)).max().item())
        # fp32 partials in, the clamped fp16 sum out (moe.finish in the same kernel)
        t = (3e4 * torch.randn(8 * hidden, generator=torch.Generator().manual_seed(250 + rank))).to(dev)
        ref = t.clone()
        dist.all_reduce(ref)
        out16 = torch.empty(8 * hidden, dtype=torch.float16, device=dev)
        words(t, out=out16)
        ref16 = ref.clamp(min=-65504.0, max=65504.0).half()
        res["words_f16_equal"] = torch.equal(out16, ref16)
        res["words_f16_diff"] = ((out16.float() - ref16.float()).abs() / (ref16.float().abs() + 1)).max().item()
        gin = torch.empty(8 * hidden, dtype=torch.float32, device=dev)
        s0 = torch.cuda.Stream()
        s0.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s0):
            words(gin.zero_())
        torch.cuda.current_stream().wait_stream(s0)
        g = torch.cuda.CUDAGraph()
        gout = torch.empty_like(gin)
        with torch.cuda.graph(g):
            words(gin, out=gout)
        for it in range(4):
            gin.copy_(torch.randn(8 * hidden, generator=torch.Generator().manual_seed(300 + it + 10 * rank)).to(dev))
            g.replay()
            ref = gin.clone()
            dist.all_reduce(ref)
            torch.cuda.synchronize()
            worst_w = max(worst_w, ((gout - ref).abs() / (ref.abs() + 1)).max().item())
        del g
        res["words"] = worst_w
        res["words_err"] = capi.device_error(rank, clear=True)
        words.close()
        # ---- tensor parallel Q4_0: column split then row split + all-reduce ----
        n, k = 4096, 8192
        w = synth.q4_0_weight(n, k, seed=11).to(dev)
        xv = synth.activations(1, k, seed=12).to(dev)
        col = tp.ColumnParallelGemv(tp.split_rows(w, rank, world), n, k, "q4_0", rank, world)
        y_col = col(xv)
        parts = [torch.empty_like(y_col) for _ in range(world)]
        dist.all_gather(parts, y_col)
        y_full = capi.gemv_q4_0(w, xv, n, k)
        res["col"] = (torch.cat(parts, dim=1).float() - y_full.float()).abs().max().item()
        res["col_scale"] = y_full.float().abs().max().item()
        wt = synth.q4_0_weight(k, n, seed=13).to(dev)  # [8192, 4096]: K = 4096 split
        xk = synth.activations(1, n, seed=14).to(dev)
        row = tp.RowParallelGemv(tp.split_k_gguf(wt, n, "q4_0", rank, world), k, n, "q4_0", rank, world)
        kl = n // world
        y_row = row(xk[:, rank * kl:(rank + 1) * kl].contiguous())
        y_ref = capi.gemv_q4_0(wt, xk, k, n)
        res["row"] = (y_row.float() - y_ref.float()).abs().max().item()
        res["row_scale"] = y_ref.float().abs().max().item()
        # ---- one-shot all-reduce over peer memory vs NCCL ----
        from gdsllm_b200.p2p import PeerAllReduce
        ar = PeerAllReduce(32768)
        worst = 0.0
        for it, n in enumerate([8192, 1024, 24576, 8192, 8192]):
            t = synth.activations(1, n, seed=100 * it + rank).to(dev).view(-1)
            ref = t.float()  # fp32 sum: NCCL's fp16 sum of more than 2 ranks rounds once per step
            dist.all_reduce(ref)
            out = ar(t.clone())
            worst = max(worst, ((out.float() - ref.float()).abs() / (ref.float().abs() + 1)).max().item())
        # inside a CUDA graph, replayed with new inputs (device-side epochs)
        gin = torch.empty(8192, dtype=torch.float16, device=dev)
        gout = torch.empty_like(gin)
        s0 = torch.cuda.Stream()
        s0.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s0):
            ar(gin.copy_(synth.activations(1, 8192, seed=1).view(-1).to(dev)), out=gout)
        torch.cuda.current_stream().wait_stream(s0)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ar(gin, out=gout)
        for it in range(5):
            gin.copy_(synth.activations(1, 8192, seed=50 + it + 10 * rank).view(-1).to(dev))
            g.replay()
            ref = gin.float()
            dist.all_reduce(ref)
            torch.cuda.synchronize()
            worst = max(worst, ((gout.float() - ref.float()).abs() / (ref.float().abs() + 1)).max().item())
        del g
        # back-to-back calls with programmatic dependent launch on, a GEMV
        # (itself a dependent launch) between consecutive calls: each call's
        # epoch must be read only after its predecessor completed
        capi.set_pdl(True)
        wq = synth.q4_0_weight(8192, 4096, seed=70).to(dev)
        xs_in = [synth.activations(1, 4096, seed=71 + 3 * i + 97 * rank).to(dev) for i in range(12)]
        ys = [torch.empty(1, 8192, dtype=torch.float16, device=dev) for _ in range(12)]
        outs = [torch.empty(8192, dtype=torch.float16, device=dev) for _ in range(12)]
        for rep in range(3):
            for i in range(12):
                capi.gemv_q4_0(wq, xs_in[i], 8192, 4096, out=ys[i])
                ar(ys[i].view(-1), out=outs[i])
            torch.cuda.synchronize()
            for i in range(12):
                ref = ys[i].view(-1).float()
                dist.all_reduce(ref)
                worst = max(worst, ((outs[i].float() - ref.float()).abs() / (ref.float().abs() + 1)).max().item())
        capi.set_pdl(False)
        res["p2p"] = worst
        res["p2p_err"] = capi.device_error(rank, clear=True)
        torch.cuda.synchronize()
        ar.close()
        # ---- row split with the all-reduce inside the GEMV epilogue ----
        from gdsllm_b200.p2p import PeerRowGemv
        fused = PeerRowGemv(k)
        worst_f, worst_n, agree = 0.0, 0.0, True
        cases = [("q4_0", synth.q4_0_weight, capi.gemv_q4_0, k, n), ("q8_0", synth.q8_0_weight, capi.gemv_q8_0, k, n),
                 ("q4_0", synth.q4_0_weight, capi.gemv_q4_0, 4096, 14336),
                 ("q4_0", synth.q4_0_weight, capi.gemv_q4_0, 1000, 2048)]
        for ci, (fmt, make, full_gemv, nn, kk) in enumerate(cases):
            wf = make(nn, kk, seed=20 + ci).to(dev)
            kl = kk // world
            wl = tp.split_k_gguf(wf, kk, fmt, rank, world)
            layer = tp.RowParallelGemv((wl,), nn, kk, fmt, rank, world, exchange=fused)
            layer_nccl = tp.RowParallelGemv((wl,), nn, kk, fmt, rank, world)
            for rep in range(3):  # epochs advance per row group
                xf = synth.activations(1, kk, seed=30 + 7 * ci + rep).to(dev)
                xl = xf[:, rank * kl:(rank + 1) * kl].contiguous()
                y_f = layer(xl)
                y_n = layer_nccl(xl)
                y_1 = full_gemv(wf, xf, nn, kk)
                scale = y_1.float().abs().max().item()
                worst_f = max(worst_f, (y_f.float() - y_1.float()).abs().max().item() / (scale + 1))
                # NCCL adds the fp16 partials in fp16 (one rounding per step beyond two ranks)
                worst_n = max(worst_n, (y_f.float() - y_n.float()).abs().max().item() / (scale + 1))
                both = [torch.empty_like(y_f) for _ in range(world)]
                dist.all_gather(both, y_f)
                agree = agree and all(torch.equal(both[0], b) for b in both)
        # captured in a CUDA graph and replayed with new activations
        wf = synth.q4_0_weight(k, n, seed=40).to(dev)
        wl = tp.split_k_gguf(wf, n, "q4_0", rank, world)
        kl = n // world
        gx = torch.empty(1, kl, dtype=torch.float16, device=dev)
        gy = torch.empty(1, k, dtype=torch.float16, device=dev)
        s0 = torch.cuda.Stream()
        s0.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s0):
            fused("q4_0", wl, gx.zero_(), k, kl, out=gy)
        torch.cuda.current_stream().wait_stream(s0)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fused("q4_0", wl, gx, k, kl, out=gy)
        for it in range(4):
            xf = synth.activations(1, n, seed=60 + it).to(dev)
            gx.copy_(xf[:, rank * kl:(rank + 1) * kl])
            g.replay()
            y_1 = capi.gemv_q4_0(wf, xf, k, n)
            torch.cuda.synchronize()
            worst_f = max(worst_f, (gy.float() - y_1.float()).abs().max().item() / (y_1.float().abs().max().item() + 1))
        del g
        res["fused"] = worst_f
        res["fused_nccl"] = worst_n
        res["fused_agree"] = agree
        res["fused_err"] = capi.device_error(rank, clear=True)
        torch.cuda.synchronize()
        fused.close()
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_and_tensor_parallel_on_gpus(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, res in out.items():
        # EP: fp32 partial sums reordered across ranks, one fp16 rounding
        assert res["ep"] <= 2e-3 * res["ep_scale"] + 1e-3, (rank, res)
        # column split: the same rows; a shard may take another K split, so
        # the fp32 summation order (not the math) can differ
        assert res["col"] <= 2e-3 * res["col_scale"] + 1e-3, (rank, res)
        # row split: two fp16 partials added (one extra rounding each)
        assert res["row"] <= 4e-3 * res["row_scale"] + 2e-3, (rank, res)
        # peer all-reduce: its fp16 result vs the fp32 sum, relative to the value
        assert res["p2p"] <= 2e-3, (rank, res)
        assert res["p2p_err"] == 0, (rank, res)
        # two ranks: NCCL adds a + b as the word all-reduce does (same bits);
        # more ranks: NCCL's order may differ, one fp16 rounding apart
        assert res["ep_words_equal"] or (world > 2 and res["ep_words_diff"] <= 2e-3 * res["ep_scale"] + 1e-3), (rank, res)
        assert res["words_f16_equal"] or (world > 2 and res["words_f16_diff"] <= 2e-3), (rank, res)
        assert res["ep_residual_equal"], (rank, res)
        assert res["words"] <= 1e-3, (rank, res)   # fp32 rank-order sum vs NCCL (fp16 inputs summed in fp32)
        assert res["words_err"] == 0, (rank, res)
        # fused row split: fp32 partials summed in rank order then one fp16
        # rounding, against the full single-GPU GEMV and the NCCL path
        assert res["fused"] <= 4e-3, (rank, res)
        assert res["fused_nccl"] <= 2e-3 * world, (rank, res)
        assert res["fused_agree"], (rank, res)   # every rank holds the same bits
        assert res["fused_err"] == 0, (rank, res)
