"""The bounded waits for another GPU, exercised on one GPU without any fault.

Each exchange kernel waits (on the device) for words that the other ranks'
copies of the same launch store into this rank's buffer.  Here "rank 1" is a
local buffer that nobody writes, so the wait runs out: with the bound
lowered to 1 ms (gdsq_set_peer_wait_limit_ns) the call must come back
quickly, set device error bit 1, leave its output unwritten, and leave the
context usable for the next call.  No kernel spins without a bound, and
nothing here traps or faults.
"""
from __future__ import annotations

import ctypes
import time

import pytest
import torch

from gdsllm_b200 import capi, synth
from gdsllm_b200._native import lib

pytestmark = pytest.mark.gpu

LIMIT_NS = 1_000_000  # 1 ms


def _ptrs(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _with_limit(fn):
    l = lib()
    prev = l.gdsq_set_peer_wait_limit_ns(LIMIT_NS)
    try:
        t0 = time.perf_counter()
        st = fn()
        torch.cuda.synchronize()
        return st, time.perf_counter() - t0
    finally:
        l.gdsq_set_peer_wait_limit_ns(prev)


def test_word_allreduce_wait_runs_out(cuda):
    l = lib()
    n = 3000
    stream = torch.cuda.current_stream().cuda_stream
    bufs = [torch.zeros(2 * 2 * n, dtype=torch.int64, device=cuda) for _ in range(2)]  # [2 slots][world][n]
    epochs = torch.zeros(32, dtype=torch.int32, device=cuda)
    x = torch.randn(n, device=cuda)
    out = torch.full((n,), 123.0, device=cuda)
    assert capi.device_error(0, clear=True) == 0
    st, secs = _with_limit(lambda: l.gdsq_allreduce_sum_words(1, x.data_ptr(), out.data_ptr(), n, _ptrs(bufs),
                                                               epochs.data_ptr(), n, 0, 2, stream))
    assert st == 0, l.gdsq_last_error()
    assert capi.device_error(0, clear=True) & 1, "the expired wait must set device error bit 1"
    assert torch.all(out == 123.0), "no output may be written after an expired wait"
    assert secs < 0.5, f"the call took {secs:.3f} s; the 1 ms bound was not applied"
    # the context is usable: a normal one-rank call right after
    own = torch.zeros(2 * n, dtype=torch.int64, device=cuda)
    ep1 = torch.zeros(32, dtype=torch.int32, device=cuda)
    out1 = torch.empty_like(x)
    assert l.gdsq_allreduce_sum_words(1, x.data_ptr(), out1.data_ptr(), n, _ptrs([own]), ep1.data_ptr(), n, 0, 1,
                                      stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(out1, x)
    assert capi.device_error(0, clear=True) == 0


def test_oneshot_allreduce_wait_runs_out(cuda):
    l = lib()
    n = 4096
    stream = torch.cuda.current_stream().cuda_stream
    bufs = [torch.zeros(2 * n, dtype=torch.float16, device=cuda) for _ in range(2)]
    flags = [torch.zeros(32 * 8, dtype=torch.int32, device=cuda) for _ in range(2)]
    x = torch.randn(n, device=cuda).half()
    out = torch.full((n,), 7.0, dtype=torch.float16, device=cuda)
    st, secs = _with_limit(lambda: l.gdsq_allreduce_sum_f16(x.data_ptr(), out.data_ptr(), n, _ptrs(bufs),
                                                             _ptrs(flags), n, 0, 2, stream))
    assert st == 0, l.gdsq_last_error()
    assert capi.device_error(0, clear=True) & 1
    assert torch.all(out == 7.0)
    assert secs < 0.5
    y = capi.gemv_q4_0(synth.q4_0_weight(64, 256, seed=1).to(cuda), synth.activations(1, 256).to(cuda), 64, 256)
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
    assert capi.device_error(0, clear=True) == 0


@pytest.mark.parametrize("fmt", [0, 1])
def test_row_split_gemv_finishers_wait_runs_out(cuda, fmt):
    l = lib()
    n, k = 4096, 2048
    stream = torch.cuda.current_stream().cuda_stream
    w = (synth.q4_0_weight if fmt == 0 else synth.q8_0_weight)(n, k, seed=3).to(cuda)
    x = synth.activations(1, k, seed=4).to(cuda)
    y = torch.full((n,), 5.0, dtype=torch.float16, device=cuda)
    bufs = [torch.zeros(2 * 2 * n, dtype=torch.int64, device=cuda) for _ in range(2)]
    flags = [torch.zeros(64, dtype=torch.int32, device=cuda) for _ in range(2)]
    st, secs = _with_limit(lambda: l.gdsq_fused_gemv_allreduce(fmt, w.data_ptr(), x.data_ptr(), y.data_ptr(), n, k,
                                                                _ptrs(bufs), _ptrs(flags), n, 0, 2, stream))
    assert st == 0, l.gdsq_last_error()
    assert capi.device_error(0, clear=True) & 1
    assert torch.all(y == 5.0)
    assert secs < 0.5
    y1 = (capi.gemv_q4_0 if fmt == 0 else capi.gemv_q8_0)(w, x, n, k)
    torch.cuda.synchronize()
    assert torch.isfinite(y1.float()).all()
    assert capi.device_error(0, clear=True) == 0
