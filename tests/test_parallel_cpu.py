"""Host logic of the multi-GPU paths on CPU: expert-parallel placement and
tensor-parallel splits, run as world_size-2 gloo process groups.  The per-rank
compute is the CPU oracle here (the product path calls the CUDA kernels),
so these tests check placement, slicing, which rank adds the shared expert,
and the all-reduce composition against the single-process oracle."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from gdsllm_b200 import ep, moe, synth, tp

HIDDEN, INTER, EXPERTS, GROUP, TOP_K, NTOK = 256, 128, 8, 32, 3, 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _stacks(experts, seed):
    def st(rows, cols, sd):
        return synth.affine_q4_weight(rows, cols, group=GROUP, seed=sd, lead=(experts,))
    return st(INTER, HIDDEN, seed), st(INTER, HIDDEN, seed + 1), st(HIDDEN, INTER, seed + 2)


def _np(stack):
    return tuple(t.numpy() for t in stack)


def oracle_partial(x2d, ids, weights, layer, out=None, include_shared=True, shared_weights=None):
    """CPU stand-in for moe.moe_partial (fp64 oracle sums, returned as fp32)."""
    x = x2d.numpy()
    idn = ids.numpy()
    wn = weights.numpy()
    h, _, _ = oracle.moe_gate_up_exact(x, idn, _np(layer.gate), _np(layer.up), layer.group, layer.expert_first)
    y, _ = oracle.moe_down_exact(h, idn, wn, _np(layer.down), layer.group, layer.expert_first)
    if include_shared and layer.shared is not None:
        sw = (shared_weights if shared_weights is not None
              else torch.sigmoid(torch.nn.functional.linear(x2d, layer.shared_gate)).view(-1)).view(-1, 1).numpy()
        sid = np.zeros((x.shape[0], 1), np.int32)
        sg, su, sd = (_np(s) for s in layer.shared)
        hs, _, _ = oracle.moe_gate_up_exact(x, sid, sg, su, layer.group)
        ys, _ = oracle.moe_down_exact(hs, sid, sw, sd, layer.group)
        y = y + ys
    t = torch.from_numpy(y.astype(np.float32))
    if out is not None:
        out.copy_(t)
        return out
    return t


def _full_layer():
    gate, up, down = _stacks(EXPERTS, 1)
    shared = _stacks(1, 10)
    g = torch.Generator().manual_seed(3)
    router = (torch.randn(EXPERTS, HIDDEN, generator=g) / HIDDEN ** 0.5).half()
    sgate = (torch.randn(1, HIDDEN, generator=g) / HIDDEN ** 0.5).half()
    return moe.MoeLayer(router=router, gate=gate, up=up, down=down, group=GROUP, shared=shared,
                        shared_gate=sgate)


def _ep_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = _full_layer()
        first, count = ep.expert_range(rank, world, EXPERTS)
        local = moe.MoeLayer(router=full.router, gate=ep.local_stack(full.gate, rank, world),
                             up=ep.local_stack(full.up, rank, world), down=ep.local_stack(full.down, rank, world),
                             group=GROUP, expert_first=first, expert_total=EXPERTS, shared=full.shared,
                             shared_gate=full.shared_gate)
        layer = ep.ExpertParallelMoE(local, top_k=TOP_K, partial=oracle_partial, router=moe.route_torch)
        x = synth.activations(NTOK, HIDDEN, seed=5)
        y = layer(x)
        # an injected in-place sum (the peer-memory all-reduce on GPUs) replaces the default
        calls = []

        def summed(t):
            calls.append((tuple(t.shape), t.dtype))
            dist.all_reduce(t)
            return t

        y2 = ep.ExpertParallelMoE(local, top_k=TOP_K, partial=oracle_partial, router=moe.route_torch,
                                  allreduce=summed)(x)
        assert calls == [((NTOK, HIDDEN), torch.float32)], calls
        assert torch.equal(y, y2)
        q.put((rank, y.numpy()))
    finally:
        dist.destroy_process_group()


def _tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, k = 96, 512
        w = synth.q4_0_weight(n, k, seed=7)
        x = synth.activations(1, k, seed=8)

        def gemv(wt, xx, nn, kk, out=None):  # oracle GEMV in fp32 (CPU stand-in for the kernel)
            w16 = oracle.dequant_q4_0(wt.numpy()).reshape(nn, kk)
            return torch.from_numpy((xx.float().numpy() @ w16.astype(np.float32).T).astype(np.float32))

        row = tp.RowParallelGemv(tp.split_k_gguf(w, k, "q4_0", rank, world), n, k, "q4_0", rank, world,
                                 gemv=lambda wt, xx, nn, kk, out=None: gemv(wt, xx, nn, kk))
        first = rank * (k // world)
        y_row = row(x[:, first:first + k // world].contiguous())
        col = tp.ColumnParallelGemv(tp.split_rows(w, rank, world), n, k, "q4_0", rank, world,
                                    gemv=lambda wt, xx, nn, kk, out=None: gemv(wt, xx, nn, kk))
        y_col = col(x)
        q.put((rank, y_row.numpy(), y_col.numpy()))
    finally:
        dist.destroy_process_group()


def _run(worker, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(out, key=lambda t: t[0])


def test_expert_range_covers_all_experts_once():
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            first, count = ep.expert_range(r, world, 512)
            seen += list(range(first, first + count))
        assert seen == list(range(512))
    with pytest.raises(ValueError):
        ep.expert_range(0, 3, 512)


def test_split_k_gguf_is_a_column_slice_of_the_dequantized_matrix():
    n, k, world = 8, 1024, 4
    for fmt, make, deq in (("q4_0", synth.q4_0_weight, oracle.dequant_q4_0),
                           ("q8_0", synth.q8_0_weight, oracle.dequant_q8_0)):
        w = make(n, k, seed=2)
        full = deq(w.numpy()).reshape(n, k)
        for r in range(world):
            part = deq(tp.split_k_gguf(w, k, fmt, r, world).numpy()).reshape(n, k // world)
            assert np.array_equal(part.view(np.uint16), full[:, r * k // world:(r + 1) * k // world].view(np.uint16))
    with pytest.raises(ValueError):
        tp.split_k_gguf(synth.q4_0_weight(2, 96), 96, "q4_0", 0, 2)


def test_split_k_affine_is_a_column_slice():
    n, k, g, world = 4, 1024, 128, 2
    words, s, b = synth.affine_q4_weight(n, k, group=g, seed=4)
    full = oracle.dequant_affine_q4(words.numpy(), s.numpy(), b.numpy(), g).reshape(n, k)
    for r in range(world):
        w2, s2, b2 = tp.split_k_affine(words, s, b, k, g, r, world)
        part = oracle.dequant_affine_q4(w2.numpy(), s2.numpy(), b2.numpy(), g).reshape(n, k // world)
        assert np.array_equal(part.view(np.uint16), full[:, r * k // world:(r + 1) * k // world].view(np.uint16))


def test_split_rows_is_a_row_slice():
    w = synth.q4_0_weight(12, 64, seed=1)
    parts = [tp.split_rows(w, r, 3) for r in range(3)]
    assert torch.equal(torch.cat(parts), w)


def test_expert_parallel_two_ranks_matches_single_process():
    out = _run(_ep_worker)
    full = _full_layer()
    x = synth.activations(NTOK, HIDDEN, seed=5)
    ids, weights, sw = moe.route_torch(x, full.router, TOP_K, full.shared_gate)
    ref = moe.finish(oracle_partial(x, ids, weights, full, shared_weights=sw), x).numpy()
    for rank, y in out:
        np.testing.assert_allclose(y.astype(np.float32), ref.astype(np.float32), rtol=2e-3, atol=1e-4,
                                   err_msg=f"rank {rank}")
    assert np.array_equal(out[0][1], out[1][1]), "ranks disagree after the all-reduce"


def test_tensor_parallel_two_ranks_matches_full_product():
    out = _run(_tp_worker)
    n, k = 96, 512
    w = synth.q4_0_weight(n, k, seed=7)
    x = synth.activations(1, k, seed=8)
    exact = oracle.gemv_exact(oracle.dequant_q4_0(w.numpy()).reshape(n, k), x.numpy())
    cols = np.concatenate([o[2] for o in out], axis=1)
    np.testing.assert_allclose(cols, exact, rtol=1e-5, atol=1e-4)
    for rank, y_row, _ in out:
        np.testing.assert_allclose(y_row, exact, rtol=1e-5, atol=1e-4, err_msg=f"rank {rank}")


def _tp_exchange_worker(rank, world, port, q):
    """Row split with an injected exchange (the shape of p2p.PeerRowGemv):
    batch-1 inputs go to the exchange, batch > 1 to the GEMV + all-reduce."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, k = 64, 512
        w = synth.q4_0_weight(n, k, seed=21)
        kl = k // world
        shard = tp.split_k_gguf(w, k, "q4_0", rank, world)

        def local(wt, xx, nn, kk):
            w16 = oracle.dequant_q4_0(wt.numpy()).reshape(nn, kk)
            return torch.from_numpy((xx.float().numpy() @ w16.astype(np.float32).T).astype(np.float32))

        calls = []

        def exchange(fmt, wt, x_local, nn, kk, out=None):  # CPU stand-in for the fused kernel
            calls.append((fmt, tuple(x_local.shape), nn, kk))
            y = local(wt, x_local, nn, kk)
            dist.all_reduce(y)
            return y

        row = tp.RowParallelGemv((shard,), n, k, "q4_0", rank, world, exchange=exchange,
                                 gemv=lambda wt, xx, nn, kk, out=None: local(wt[0], xx, nn, kk))
        x1 = synth.activations(1, k, seed=22)
        x2 = synth.activations(2, k, seed=23)
        y1 = row(x1[:, rank * kl:(rank + 1) * kl].contiguous())
        y2 = row(x2[:, rank * kl:(rank + 1) * kl].contiguous())
        q.put((rank, y1.numpy(), y2.numpy(), calls))
    finally:
        dist.destroy_process_group()


def test_row_parallel_routes_batch_one_to_the_exchange():
    out = _run(_tp_exchange_worker)
    n, k = 64, 512
    w16 = oracle.dequant_q4_0(synth.q4_0_weight(n, k, seed=21).numpy()).reshape(n, k)
    e1 = oracle.gemv_exact(w16, synth.activations(1, k, seed=22).numpy())
    e2 = oracle.gemv_exact(w16, synth.activations(2, k, seed=23).numpy())
    for rank, y1, y2, calls in out:
        assert calls == [("q4_0", (1, k // 2), n, k // 2)], calls   # batch 2 took the all-reduce path
        np.testing.assert_allclose(y1, e1, rtol=1e-5, atol=1e-4, err_msg=f"rank {rank}")
        np.testing.assert_allclose(y2, e2, rtol=1e-5, atol=1e-4, err_msg=f"rank {rank}")
