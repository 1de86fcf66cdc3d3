"""The reference-facing op API (module gds_io_ext) on a GPU, used the way
GdsLLM's callers use it: handles plus byte offsets, meta dicts as built by
torch_bridge._make_tensor_entry (gdsllm/runtime/torch_bridge.py:125-146),
``x.view(-1)`` inputs (llama.py:136-141, qwen_moe.py:48-55) and a shared
fp16 scratch for prefill dequant (llama.py:106-119, scheduler.py:72-90)."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import oracle
from gdsllm_b200 import synth
from tests.conftest import assert_f16_bitexact

pytestmark = pytest.mark.gpu
TOL = 2e-3


def within_bar(y, w16, x):
    xn = x.float().cpu().numpy().reshape(-1, w16.shape[1]).astype(np.float64)
    exact = xn @ w16.astype(np.float64).T
    bound = TOL * np.linalg.norm(xn, axis=1) * np.abs(w16.astype(np.float64)).max()
    err = np.abs(y.float().cpu().numpy().reshape(exact.shape) - exact).max(axis=1)
    assert (err <= bound).all(), (err, bound)


def layer_buffer(cuda):
    """Two Q4_0 tensors and one Q8_0 tensor at 4 KB-aligned offsets in one handle."""
    a = synth.q4_0_weight(256, 1024, seed=1)
    b = synth.q4_0_weight(512, 256, seed=2)
    c = synth.q8_0_weight(64, 512, seed=3)
    offs, cur, parts = [], 0, []
    for t in (a, b, c):
        offs.append(cur)
        pad = (-t.numel()) % 4096
        parts += [t.reshape(-1), torch.zeros(pad, dtype=torch.uint8)]
        cur += t.numel() + pad
    return torch.cat(parts).to(cuda), offs, (a, b, c)


def test_fused_dequant_gemv_as_llama_calls_it(ext, cuda):
    buf, offs, (a, b, c) = layer_buffer(cuda)
    h = ext.handle_from_tensor(buf)
    assert h.device_id == 0 and h.size == buf.numel()
    metas = [{"buffer": h, "shape": [256, 1024], "gguf_type": "q4_0", "offset": offs[0]},
             {"buffer": h, "shape": [512, 256], "gguf_type": "q4_0", "offset": offs[1]},
             {"buffer": h, "shape": [64, 512], "gguf_type": "q8_0", "offset": offs[2]}]
    refs = [oracle.dequant_q4_0(a.numpy()).reshape(256, 1024),
            oracle.dequant_q4_0(b.numpy()).reshape(512, 256),
            oracle.dequant_q8_0(c.numpy()).reshape(64, 512)]
    for meta, w16 in zip(metas, refs):
        x = synth.activations(1, meta["shape"][1], seed=4).to(cuda).view(1, 1, -1)
        out = ext.fused_dequant_gemv(meta["buffer"], x.view(-1), meta["shape"], meta["gguf_type"],
                                     meta["offset"])
        assert out.shape == (1, meta["shape"][0]) and out.dtype == torch.float16
        within_bar(out, w16, x)
        # prefill path: dequant into a shared scratch, then F.linear
        scratch = torch.empty(512 * 1024, dtype=torch.float16, device=cuda)
        wd = ext.dequant_gguf(meta["buffer"], meta["shape"], meta["gguf_type"], meta["offset"], scratch)
        assert wd.shape == tuple(meta["shape"])
        assert wd.data_ptr() == scratch.data_ptr()
        assert_f16_bitexact(wd.cpu().numpy(), w16, "dequant_gguf")
        wd2 = ext.dequant_gguf(meta["buffer"], meta["shape"], meta["gguf_type"], meta["offset"])
        assert_f16_bitexact(wd2.cpu().numpy(), w16, "dequant_gguf (alloc)")


def test_batched_input_returns_batch_rows(ext, cuda):
    buf, offs, (a, _, _) = layer_buffer(cuda)
    h = ext.handle_from_tensor(buf)
    x = synth.activations(5, 1024, seed=6).to(cuda)
    out = ext.fused_dequant_gemv(h, x, [256, 1024], "q4_0", offs[0])
    assert out.shape == (5, 256)
    within_bar(out, oracle.dequant_q4_0(a.numpy()).reshape(256, 1024), x)


def test_affine_ops_as_qwen_moe_calls_them(ext, cuda):
    words, s, b = synth.affine_q4_weight(1024, 4096, seed=7)
    buf, wo, so, bo = synth.pack_affine_buffer(words, s, b)
    h = ext.handle_from_tensor(buf.to(cuda))
    meta = {"buffer": h, "shape": [1024, 4096], "quant_type": "affine_q4", "weight_offset": wo,
            "scale_offset": so, "bias_offset": bo, "group_size": 128}
    w16 = oracle.dequant_affine_q4(words.numpy(), s.numpy(), b.numpy(), 128).reshape(1024, 4096)
    x = synth.activations(1, 4096, seed=8).to(cuda).view(1, 1, -1)
    out = ext.fused_affine_q4_gemv(meta["buffer"], x.view(-1), meta["shape"], meta["weight_offset"],
                                   meta["scale_offset"], meta["bias_offset"], meta["group_size"])
    assert out.shape == (1, 1024)
    within_bar(out, w16, x)
    wd = ext.dequant_affine_q4(meta["buffer"], meta["shape"], meta["weight_offset"],
                               meta["scale_offset"], meta["bias_offset"], meta["group_size"], None)
    assert_f16_bitexact(wd.cpu().numpy(), w16, "dequant_affine_q4")
    # 3-D expert tensor shape (router / per-expert slices use >= 2 dims)
    wd3 = ext.dequant_affine_q4(h, [2, 512, 4096], wo, so, bo, 128)
    assert wd3.shape == (2, 512, 4096)
    assert_f16_bitexact(wd3.cpu().numpy().reshape(1024, 4096), w16, "3-D shape")


@pytest.mark.parametrize("bad", [
    dict(shape=[16, 48], gguf_type="q4_0", offset=0),        # in_dim % 32
    dict(shape=[16, 64], gguf_type="q5_k", offset=0),        # unknown type
    dict(shape=[16, 64, 1], gguf_type="q4_0", offset=0),     # not 2-D
    dict(shape=[16, 64], gguf_type="q4_0", offset=1 << 30),  # outside the buffer
])
def test_fused_gemv_errors_raise(ext, cuda, bad):
    h = ext.handle_from_tensor(torch.zeros(8192, dtype=torch.uint8, device=cuda))
    x = torch.zeros(bad["shape"][-1] if len(bad["shape"]) == 2 else 64, dtype=torch.float16, device=cuda)
    with pytest.raises(RuntimeError):
        ext.fused_dequant_gemv(h, x, bad["shape"], bad["gguf_type"], bad["offset"])


def test_wrong_input_size_and_small_scratch_raise(ext, cuda):
    h = ext.handle_from_tensor(torch.zeros(8192, dtype=torch.uint8, device=cuda))
    with pytest.raises(RuntimeError, match="in_dim"):
        ext.fused_dequant_gemv(h, torch.zeros(100, dtype=torch.float16, device=cuda), [16, 64], "q4_0", 0)
    with pytest.raises(RuntimeError, match="too small"):
        ext.dequant_gguf(h, [16, 64], "q4_0", 0, torch.empty(10, dtype=torch.float16, device=cuda))
    with pytest.raises(RuntimeError, match="multiple of 32"):
        ext.dequant_gguf(h, [3, 5], "q4_0", 0)


def test_load_ops_read_files(ext, cuda, tmp_path):
    ext.init()
    data = np.random.default_rng(0).integers(0, 256, 3 * 4096 + 100, dtype=np.uint8)
    path = tmp_path / "layer_000.bin"
    data.tofile(path)
    h = ext.load_file(str(path), data.size)
    assert h.size >= data.size
    v = ext.view_tensor(h, [data.size], "int8", 0)
    assert np.array_equal(v.cpu().numpy().view(np.uint8), data)
    r = ext.load_file_region(str(path), 4096, 4096)
    assert np.array_equal(ext.view_tensor(r, [4096], "int8", 0).cpu().numpy().view(np.uint8),
                          data[4096:8192])
    eh, wo, so, bo = ext.load_expert(str(path), 0, 4096, 4096, 100, 8192, 28)
    got = ext.view_tensor(eh, [4096 + 100 + 28], "int8", 0).cpu().numpy().view(np.uint8)
    assert np.array_equal(got, np.concatenate([data[:4096], data[4096:4196], data[8192:8220]]))
    assert (wo, so, bo) == (0, 4096, 4196)
    t = ext.load_tensor(str(path), [1024], "float16", 4096, 2048)
    assert np.array_equal(t.cpu().numpy().view(np.uint8), data[4096:6144])
    with pytest.raises(RuntimeError):
        ext.load_file(str(path), data.size + 10)  # short read
    with pytest.raises(RuntimeError, match="exceeds buffer size"):
        ext.view_tensor(r, [4096], "float16", 0)  # 8192 bytes of a 4096-byte region
    with pytest.raises(RuntimeError, match="exceeds buffer size"):
        ext.view_tensor(r, [16], "int8", r.size - 8)
    ext.shutdown()


def test_load_file_async_and_prefetch(ext, cuda, tmp_path):
    """load_file_async reads through two pinned staging buffers with one
    cudaMemcpyAsync per chunk on a loader stream while the caller's stream
    keeps running; wait() returns the same bytes load_file reads.  A
    prefetch_file()d region is what the next load_file / load_file_region of
    that region returns."""
    from gdsllm_b200 import capi, synth
    rng = np.random.default_rng(1)
    data = rng.integers(0, 256, (40 << 20) + 123, dtype=np.uint8)  # 5+ chunks, ragged tail
    path = tmp_path / "layer_007.bin"
    data.tofile(path)
    ext.init()
    pending = [ext.load_file_async(str(path), data.size),
               ext.load_file_async(str(path), 10_000_000, 12345),
               ext.load_file_async(str(path), 4096, data.size - 4096)]
    w = synth.q4_0_weight(4096, 4096, seed=1).to(cuda)   # the caller's stream stays busy meanwhile
    x = synth.activations(1, 4096, seed=2).to(cuda)
    for _ in range(20):
        capi.gemv_q4_0(w, x, 4096, 4096)
    handles = [p.wait() for p in reversed(pending)][::-1]
    assert all(p.ready for p in pending)
    got = [ext.view_tensor(h, [n], "int8", 0).cpu().numpy().view(np.uint8)
           for h, n in zip(handles, [data.size, 10_000_000, 4096])]
    assert np.array_equal(got[0], data)
    assert np.array_equal(got[1], data[12345:12345 + 10_000_000])
    assert np.array_equal(got[2], data[-4096:])
    with pytest.raises(RuntimeError, match="expected"):
        ext.load_file_async(str(path), data.size + 10).wait()  # short read
    ext.prefetch_file(str(path), data.size)
    ext.prefetch_file(str(path), 8192, 4096)
    h = ext.load_file(str(path), data.size)
    r = ext.load_file_region(str(path), 8192, 4096)
    assert np.array_equal(ext.view_tensor(h, [data.size], "int8", 0).cpu().numpy().view(np.uint8), data)
    assert np.array_equal(ext.view_tensor(r, [8192], "int8", 0).cpu().numpy().view(np.uint8), data[4096:12288])
    ext.shutdown()
