"""gdsq_moe_affine_q4_noalloc: the MoE gate/up + down pair with its
intermediate in the library's static device array instead of a caller
buffer.  It must give exactly the two-call results, reject requests larger
than the array before touching CUDA, and keep working when called again
(the array is reused, its address is looked up once per device)."""
from __future__ import annotations

import pytest
import torch

from gdsllm_b200 import capi, synth
from gdsllm_b200._native import lib

NOALLOC_MAX_H = 2 << 20  # fp16 elements of the static array


def _ptr(t):
    return None if t is None else t.data_ptr()


def _noalloc(gate, up, down, shared, x, ids, w, sw, y, inter, hidden, group, flags=0, stream=None,
             ntok=None, top_k=None):
    sg, su, sd = shared if shared is not None else ((None,) * 3,) * 3
    ntok = ids.shape[0] if ntok is None else ntok
    top_k = ids.shape[1] if top_k is None else top_k
    e = gate[0].shape[0] if gate[0] is not None else 1
    args = [*[_ptr(t) for t in (*gate, *up, *down, *sg, *su, *sd)], _ptr(x), _ptr(ids), _ptr(w), _ptr(sw), _ptr(y),
            ntok, top_k, hidden, inter, group, 0, e, e, flags, stream]
    return lib().gdsq_moe_affine_q4_noalloc(*args)


def test_noalloc_rejects_oversize_before_any_cuda_call():
    """Runs without a GPU: the size check comes first."""
    args = [16] * 23 + [4096, 64, 4096, 1024, 128, 0, 512, 512, 0, None]   # 4096 x 64 x 1024 > 2 Mi
    st = lib().gdsq_moe_affine_q4_noalloc(*args)
    assert st == 1  # GDSQ_ERR_INVALID_VALUE
    msg = lib().gdsq_last_error().decode()
    assert "static scratch" in msg and str(NOALLOC_MAX_H) in msg, msg


@pytest.mark.parametrize("missing", [15, 16, 17, 21])
def test_noalloc_rejects_partial_shared_expert(missing):
    """Runs without a GPU: shared gate/up given but a shared down tensor or the
    shared weights missing would make the two stages disagree on the slots
    per token, so the call is rejected before any CUDA call."""
    args = [16] * 23 + [1, 10, 4096, 1024, 128, 0, 512, 512, 0, None]
    args[missing] = None  # 15-17: shared down weight/scales/biases, 21: shared_weights
    st = lib().gdsq_moe_affine_q4_noalloc(*args)
    assert st == 1  # GDSQ_ERR_INVALID_VALUE
    assert "all given or all null" in lib().gdsq_last_error().decode()


@pytest.mark.gpu
@pytest.mark.parametrize("ntok,top_k,with_shared", [(1, 10, True), (8, 10, False), (3, 4, True)])
def test_noalloc_matches_two_call_form(cuda, ntok, top_k, with_shared):
    experts, hidden, inter, group = 16, 2048, 512, 128

    def st(rows, cols, seed, e):
        return tuple(t.to(cuda) for t in synth.affine_q4_weight(rows, cols, group=group, seed=seed, lead=(e,)))

    gate, up, down = st(inter, hidden, 1, experts), st(inter, hidden, 2, experts), st(hidden, inter, 3, experts)
    shared = (st(inter, hidden, 4, 1), st(inter, hidden, 5, 1), st(hidden, inter, 6, 1)) if with_shared else None
    g = torch.Generator().manual_seed(ntok)
    ids = torch.stack([torch.randperm(experts, generator=g)[:top_k] for _ in range(ntok)]).to(torch.int32).to(cuda)
    w = torch.softmax(torch.randn(ntok, top_k, generator=g), -1).half().to(cuda)
    sw = torch.rand(ntok, generator=g).half().to(cuda) if with_shared else None
    x = synth.activations(ntok, hidden, seed=9).to(cuda)
    h = capi.moe_gate_up(gate, up, x, ids, group, shared=shared[:2] if shared else None)
    ref = capi.moe_down(down, h, ids, w, group, flags=capi.MOE_OUT_F32, shared=shared[2] if shared else None,
                        shared_weights=sw)
    for _ in range(2):  # the second call reuses the array (and the cached address)
        y = torch.full((ntok, hidden), float("nan"), dtype=torch.float32, device=cuda)
        stream = torch.cuda.current_stream().cuda_stream
        assert _noalloc(gate, up, down, shared, x, ids, w, sw, y, inter, hidden, group, flags=capi.MOE_OUT_F32,
                        stream=stream) == 0, lib().gdsq_last_error()
        torch.cuda.synchronize()
        assert torch.equal(y, ref)
    assert capi.device_error(0, clear=True) == 0


@pytest.mark.gpu
def test_noalloc_consecutive_calls_on_one_stream(cuda):
    """Two layers back to back on one stream: the second call's gate/up runs
    only after the first call's down has read the array (stream order)."""
    experts, hidden, inter, group, top_k = 8, 1024, 256, 128, 4

    def st(rows, cols, seed):
        return tuple(t.to(cuda) for t in synth.affine_q4_weight(rows, cols, group=group, seed=seed, lead=(experts,)))

    layers = [(st(inter, hidden, 10 * i), st(inter, hidden, 10 * i + 1), st(hidden, inter, 10 * i + 2))
              for i in range(2)]
    ids = torch.tensor([[0, 3, 5, 7], [1, 2, 4, 6]], dtype=torch.int32, device=cuda)
    w = torch.full((2, top_k), 0.25, dtype=torch.float16, device=cuda)
    x = synth.activations(2, hidden, seed=2).to(cuda)
    stream = torch.cuda.current_stream().cuda_stream
    outs, refs = [], []
    for gate, up, down in layers:
        y = torch.empty(2, hidden, dtype=torch.float16, device=cuda)
        assert _noalloc(gate, up, down, None, x, ids, w, None, y, inter, hidden, group, stream=stream) == 0
        outs.append(y)
        refs.append(capi.moe_down(down, capi.moe_gate_up(gate, up, x, ids, group), ids, w, group))
    torch.cuda.synchronize()
    for y, r in zip(outs, refs):
        assert torch.equal(y, r)
