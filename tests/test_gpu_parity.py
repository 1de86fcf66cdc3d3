"""GPU parity of the gdsq kernels, called through the C ABI (ctypes), against
the CPU oracle and against GdsLLM's own CUDA kernels on the same inputs.

Bars (stated here, applied below):
* dequantized fp16 weights: bit-exact;
* GEMV: |y - y_exact| <= 2e-3 * ||x||_2 * max|W| per batch row, where y_exact
  is the fp64 product of the oracle's dequantized weights and x.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from gdsllm_b200 import synth
from oracle import reference_kernels as refk
from tests.conftest import assert_f16_bitexact

pytestmark = pytest.mark.gpu

TOL = 2e-3  # the GEMV bar: TOL * ||x||_2 * max|W|


def _check_gemv(y_gpu: torch.Tensor, w_f16: np.ndarray, x: torch.Tensor, what: str):
    xn = x.cpu().numpy().reshape(-1, w_f16.shape[1])
    y = y_gpu.float().cpu().numpy().reshape(xn.shape[0], -1).astype(np.float64)
    exact = oracle.gemv_exact(w_f16, xn)
    bound = TOL * np.linalg.norm(xn.astype(np.float64), axis=1) * np.abs(w_f16.astype(np.float64)).max()
    err = np.abs(y - exact).max(axis=1)
    assert np.isfinite(y).all(), f"{what}: non-finite output"
    assert (err <= bound).all(), f"{what}: max err {err} > bound {bound}"
    return err / bound


# ---- dequantization: bit-exact ---------------------------------------------

@pytest.mark.parametrize("n,k", [(1, 32), (3, 96), (64, 4096), (11008, 4096), (32000, 4096)])
def test_dequant_q4_0_bitexact(gdsq, cuda, n, k):
    w = synth.q4_0_weight(n, k, seed=n + k)
    out = gdsq.dequant_q4_0(w.to(cuda))
    assert_f16_bitexact(out.cpu().numpy(), oracle.dequant_q4_0(w.numpy()), "q4_0")


@pytest.mark.parametrize("n,k", [(1, 32), (3, 96), (64, 4096), (32000, 4096)])
def test_dequant_q8_0_bitexact(gdsq, cuda, n, k):
    w = synth.q8_0_weight(n, k, seed=n + k)
    out = gdsq.dequant_q8_0(w.to(cuda))
    assert_f16_bitexact(out.cpu().numpy(), oracle.dequant_q8_0(w.numpy()), "q8_0")


@pytest.mark.parametrize("n,k,g", [(1, 128, 128), (5, 64, 8), (16, 256, 32), (1024, 4096, 128),
                                   (4096, 1024, 128), (7, 1536, 512)])
def test_dequant_affine_bitexact(gdsq, cuda, n, k, g):
    words, s, b = synth.affine_q4_weight(n, k, group=g, seed=n)
    out = gdsq.dequant_affine_q4(words.to(cuda), s.to(cuda), b.to(cuda), k, g)
    expected = oracle.dequant_affine_q4(words.numpy(), s.numpy(), b.numpy(), g).reshape(-1)
    assert_f16_bitexact(out.cpu().numpy(), expected, "affine")


def test_dequant_edge_blocks_match_gguf_golden(gdsq, cuda):
    from pathlib import Path
    z = np.load(Path(__file__).parent / "golden" / "gguf_blocks.npz")
    for fmt, fn in (("q4_0", gdsq.dequant_q4_0), ("q8_0", gdsq.dequant_q8_0)):
        raw = torch.from_numpy(z[f"{fmt}_blocks"].reshape(-1).copy()).to(cuda)
        with np.errstate(all="ignore"):
            expected = z[f"{fmt}_gguf_f32"].astype(np.float16)
        assert_f16_bitexact(fn(raw).cpu().numpy(), expected, fmt)


def test_dequant_unaligned_output_uses_scalar_stores(gdsq, cuda):
    w = synth.q4_0_weight(5, 64, seed=3).to(cuda)
    big = torch.zeros(5 * 64 + 1, dtype=torch.float16, device=cuda)
    out = big[1:]  # 2-byte aligned, not 16
    gdsq.dequant_q4_0(w, out=out)
    assert_f16_bitexact(out.cpu().numpy(), oracle.dequant_q4_0(w.cpu().numpy()), "q4_0 unaligned")
    assert big[0].item() == 0


# ---- fused GEMV: within the bar ---------------------------------------------

GEMV_SHAPES = [(11008, 4096), (4096, 11008), (4096, 4096), (1, 256), (33, 512), (100, 768),
               (37, 96), (5, 32)]


@pytest.mark.parametrize("n,k", GEMV_SHAPES)
@pytest.mark.parametrize("batch", [1, 3])
def test_gemv_q4_0(gdsq, cuda, n, k, batch):
    w = synth.q4_0_weight(n, k, seed=7)
    x = synth.activations(batch, k, seed=8).to(cuda)
    y = gdsq.gemv_q4_0(w.to(cuda), x, n, k)
    torch.cuda.synchronize()
    _check_gemv(y, oracle.dequant_q4_0(w.numpy()).reshape(n, k), x, f"q4_0 {n}x{k} b{batch}")


@pytest.mark.parametrize("n,k", [(32000, 4096), (4096, 4096), (33, 512), (37, 96)])
@pytest.mark.parametrize("batch", [1, 4])
def test_gemv_q8_0(gdsq, cuda, n, k, batch):
    w = synth.q8_0_weight(n, k, seed=9)
    x = synth.activations(batch, k, seed=10).to(cuda)
    y = gdsq.gemv_q8_0(w.to(cuda), x, n, k)
    torch.cuda.synchronize()
    _check_gemv(y, oracle.dequant_q8_0(w.numpy()).reshape(n, k), x, f"q8_0 {n}x{k} b{batch}")


@pytest.mark.parametrize("n,k,g", [(1024, 4096, 128), (4096, 1024, 128), (4096, 4096, 128),
                                   (65, 512, 32), (65, 512, 64), (40, 1024, 256), (9, 96, 8),
                                   (12, 1024, 512)])
@pytest.mark.parametrize("batch", [1, 2])
def test_gemv_affine(gdsq, cuda, n, k, g, batch):
    words, s, b = synth.affine_q4_weight(n, k, group=g, seed=n)
    x = synth.activations(batch, k, seed=2).to(cuda)
    y = gdsq.gemv_affine_q4(words.to(cuda), s.to(cuda), b.to(cuda), x, n, k, g)
    torch.cuda.synchronize()
    w16 = oracle.dequant_affine_q4(words.numpy(), s.numpy(), b.numpy(), g).reshape(n, k)
    _check_gemv(y, w16, x, f"affine {n}x{k} g{g} b{batch}")


@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 8, 13, 16])
def test_gemv_every_batch_size(gdsq, cuda, batch):
    n, k = 300, 2048
    w = synth.q4_0_weight(n, k, seed=batch)
    x = synth.activations(batch, k, seed=batch + 100).to(cuda)
    y = gdsq.gemv_q4_0(w.to(cuda), x, n, k)
    torch.cuda.synchronize()
    _check_gemv(y, oracle.dequant_q4_0(w.numpy()).reshape(n, k), x, f"q4_0 b{batch}")
    w8 = synth.q8_0_weight(n, k, seed=batch)
    y8 = gdsq.gemv_q8_0(w8.to(cuda), x, n, k)
    words, s, b = synth.affine_q4_weight(n, k, seed=batch)
    ya = gdsq.gemv_affine_q4(words.to(cuda), s.to(cuda), b.to(cuda), x, n, k, 128)
    torch.cuda.synchronize()
    _check_gemv(y8, oracle.dequant_q8_0(w8.numpy()).reshape(n, k), x, f"q8_0 b{batch}")
    _check_gemv(ya, oracle.dequant_affine_q4(words.numpy(), s.numpy(), b.numpy(), 128).reshape(n, k),
                x, f"affine b{batch}")


def test_gemv_misaligned_weight_takes_generic_path(gdsq, cuda):
    n, k = 64, 512
    w = synth.q4_0_weight(n, k, seed=4)
    buf = torch.zeros(w.numel() + 2, dtype=torch.uint8, device=cuda)
    buf[2:] = w.reshape(-1).to(cuda)   # 2-byte aligned, not 16
    x = synth.activations(1, k, seed=5).to(cuda)
    y = gdsq.gemv_q4_0(buf[2:], x, n, k)
    torch.cuda.synchronize()
    _check_gemv(y, oracle.dequant_q4_0(w.numpy()).reshape(n, k), x, "q4_0 misaligned")


def test_gemv_zero_in_dim_gives_zeros(gdsq, cuda):
    y = torch.full((2, 7), 5.0, dtype=torch.float16, device=cuda)
    dummy = torch.zeros(16, dtype=torch.uint8, device=cuda)
    x = torch.zeros(2, 16, dtype=torch.float16, device=cuda)
    from gdsllm_b200._native import check, lib
    check(lib().gdsq_fused_q4_0_gemv(dummy.data_ptr(), x.data_ptr(), y.data_ptr(), 7, 0, 2,
                                     torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert (y == 0).all()


def test_no_device_error_after_parity_runs(gdsq, cuda):
    assert gdsq.device_error(0, clear=True) == 0


# ---- against the reference's own kernels -------------------------------------

needs_ref = pytest.mark.skipif(not refk.available(), reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("n,k", [(11008, 4096), (4096, 4096), (96, 1024)])
def test_q4_0_against_reference_kernels(gdsq, cuda, n, k):
    w = synth.q4_0_weight(n, k, seed=21).to(cuda)
    x = synth.activations(1, k, seed=22).to(cuda)
    d_ours = gdsq.dequant_q4_0(w)
    d_ref = refk.dequant_q4_0(w, torch.empty_like(d_ours))
    y_ours = gdsq.gemv_q4_0(w, x, n, k)
    y_ref = refk.gemv_q4_0(w, x, n, k, torch.empty_like(y_ours))
    torch.cuda.synchronize()
    assert_f16_bitexact(d_ours.cpu().numpy(), d_ref.cpu().numpy(), "q4_0 dequant vs reference")
    w16 = d_ref.cpu().numpy().reshape(n, k)
    _check_gemv(y_ours, w16, x, "ours")
    _check_gemv(y_ref, w16, x, "reference")


@needs_ref
@pytest.mark.parametrize("n,k", [(32000, 4096), (96, 1024)])
def test_q8_0_against_reference_kernels(gdsq, cuda, n, k):
    w = synth.q8_0_weight(n, k, seed=23).to(cuda)
    x = synth.activations(1, k, seed=24).to(cuda)
    d_ours = gdsq.dequant_q8_0(w)
    d_ref = refk.dequant_q8_0(w, torch.empty_like(d_ours))
    y_ours = gdsq.gemv_q8_0(w, x, n, k)
    y_ref = refk.gemv_q8_0(w, x, n, k, torch.empty_like(y_ours))
    torch.cuda.synchronize()
    assert_f16_bitexact(d_ours.cpu().numpy(), d_ref.cpu().numpy(), "q8_0 dequant vs reference")
    w16 = d_ref.cpu().numpy().reshape(n, k)
    _check_gemv(y_ours, w16, x, "ours")
    _check_gemv(y_ref, w16, x, "reference")


@needs_ref
@pytest.mark.parametrize("n,k,g", [(1024, 4096, 128), (4096, 1024, 128), (64, 512, 32)])
def test_affine_against_reference_kernels(gdsq, cuda, n, k, g):
    words, s, b = (t.to(cuda) for t in synth.affine_q4_weight(n, k, group=g, seed=25))
    x = synth.activations(1, k, seed=26).to(cuda)
    d_ours = gdsq.dequant_affine_q4(words, s, b, k, g)
    d_ref = refk.dequant_affine_q4(words, s, b, k, g, torch.empty_like(d_ours))
    y_ours = gdsq.gemv_affine_q4(words, s, b, x, n, k, g)
    y_ref = refk.gemv_affine_q4(words, s, b, x, n, k, g, torch.empty_like(y_ours))
    torch.cuda.synchronize()
    assert_f16_bitexact(d_ours.cpu().numpy(), d_ref.cpu().numpy(), "affine dequant vs reference")
    w16 = d_ref.cpu().numpy().reshape(n, k)
    _check_gemv(y_ours, w16, x, "ours")
    _check_gemv(y_ref, w16, x, "reference")


ERR_RATIO = 1.25  # our RMS and max error may exceed the reference kernel's by this factor at most


def _errors(y: torch.Tensor, exact: np.ndarray):
    e = y.float().cpu().numpy().reshape(-1).astype(np.float64) - exact.reshape(-1)
    return float(np.sqrt(np.mean(e * e))), float(np.abs(e).max())


@needs_ref
@pytest.mark.parametrize("fmt,n,k", [("q4_0", 11008, 4096), ("q4_0", 4096, 11008), ("q4_0", 4096, 4096),
                                     ("q8_0", 4096, 4096), ("q8_0", 11008, 4096), ("q8_0", 4096, 11008),
                                     ("q8_0", 32000, 4096), ("affine", 4096, 4096), ("affine", 11008, 4096),
                                     ("affine", 4096, 11008), ("affine", 32000, 4096)])
def test_error_no_larger_than_reference_kernels(gdsq, cuda, fmt, n, k):
    """Arithmetic parity with the reference (config 0 and the config-2 shapes,
    batch 1, the configs' value distributions, seed 0): against the fp64
    product of the dequantized weights, the RMS and the max error of our
    output are at most ERR_RATIO times those of GdsLLM's own kernel on the
    same buffers.  Both accumulate in fp32 and round once to fp16, so the
    final rounding dominates both errors."""
    x = synth.activations(1, k, seed=0).to(cuda)
    if fmt == "affine":
        words, s, b = (t.to(cuda) for t in synth.affine_q4_weight(n, k, group=128, seed=0))
        y_ours = gdsq.gemv_affine_q4(words, s, b, x, n, k, 128)
        y_ref = refk.gemv_affine_q4(words, s, b, x, n, k, 128, torch.empty_like(y_ours))
        w16 = oracle.dequant_affine_q4(words.cpu().numpy(), s.cpu().numpy(), b.cpu().numpy(), 128)
    else:
        make, deq = (synth.q4_0_weight, oracle.dequant_q4_0) if fmt == "q4_0" else (synth.q8_0_weight,
                                                                                   oracle.dequant_q8_0)
        w = make(n, k, seed=0).to(cuda)
        ours, ref = (gdsq.gemv_q4_0, refk.gemv_q4_0) if fmt == "q4_0" else (gdsq.gemv_q8_0, refk.gemv_q8_0)
        y_ours = ours(w, x, n, k)
        y_ref = ref(w, x, n, k, torch.empty_like(y_ours))
        w16 = deq(w.cpu().numpy())
    torch.cuda.synchronize()
    exact = oracle.gemv_exact(w16.reshape(n, k), x.cpu().numpy())
    rms_o, max_o = _errors(y_ours, exact)
    rms_r, max_r = _errors(y_ref, exact)
    assert rms_o <= ERR_RATIO * rms_r, f"{fmt} {n}x{k}: RMS error {rms_o:.3e} vs reference {rms_r:.3e}"
    assert max_o <= ERR_RATIO * max_r, f"{fmt} {n}x{k}: max error {max_o:.3e} vs reference {max_r:.3e}"


# ---- tensor-core batched GEMV (default for batch >= 2) ----------------------

def _weights(fmt, n, k, g, seed):
    if fmt == "q4_0":
        w = synth.q4_0_weight(n, k, seed=seed)
        return (w,), oracle.dequant_q4_0(w.numpy()).reshape(n, k)
    if fmt == "q8_0":
        w = synth.q8_0_weight(n, k, seed=seed)
        return (w,), oracle.dequant_q8_0(w.numpy()).reshape(n, k)
    words, s, b = synth.affine_q4_weight(n, k, group=g, seed=seed)
    return (words, s, b), oracle.dequant_affine_q4(words.numpy(), s.numpy(), b.numpy(), g).reshape(n, k)


def _run(gdsq, fmt, ws, x, n, k, g):
    ws = [t.to(x.device) for t in ws]
    if fmt == "q4_0":
        return gdsq.gemv_q4_0(ws[0], x, n, k)
    if fmt == "q8_0":
        return gdsq.gemv_q8_0(ws[0], x, n, k)
    return gdsq.gemv_affine_q4(ws[0], ws[1], ws[2], x, n, k, g)


@pytest.mark.parametrize("fmt,g", [("q4_0", 0), ("q8_0", 0), ("affine", 128), ("affine", 32), ("affine", 256)])
@pytest.mark.parametrize("n,k", [(4096, 4096), (11008, 4096), (4096, 11008), (300, 1024), (129, 512)])
@pytest.mark.parametrize("batch", [1, 2, 5, 8, 16])
def test_gemv_tensor_core_batched(gdsq, cuda, fmt, g, n, k, batch, monkeypatch):
    """The tcgen05 batched kernel (forced on for batch 1 as well) meets the
    GEMV bar for every format, odd row counts and every batch tile."""
    monkeypatch.setenv("GDSQ_GEMV_TCB", "1")
    ws, w16 = _weights(fmt, n, k, g, seed=n + batch)
    x = synth.activations(batch, k, seed=k + batch).to(cuda)
    y = _run(gdsq, fmt, ws, x, n, k, g)
    torch.cuda.synchronize()
    _check_gemv(y, w16, x, f"tcb {fmt} g{g} {n}x{k} b{batch}")


@pytest.mark.parametrize("plan", ["1:3", "1:5", "2:3", "2:4", "4:3", "8:3"])
@pytest.mark.parametrize("fmt,g", [("q4_0", 0), ("q8_0", 0), ("affine", 64)])
def test_gemv_tensor_core_launch_plans(gdsq, cuda, fmt, g, plan, monkeypatch):
    """Every cluster split and ring depth of the tensor-core kernel, including
    K slices of uneven length and several row tiles per cluster."""
    monkeypatch.setenv("GDSQ_GEMV_TCB", "1")
    monkeypatch.setenv("GDSQ_GEMV_PLAN", plan)
    n, k, batch = 1000, 2560, 6
    ws, w16 = _weights(fmt, n, k, g, seed=3)
    x = synth.activations(batch, k, seed=4).to(cuda)
    y = _run(gdsq, fmt, ws, x, n, k, g)
    torch.cuda.synchronize()
    _check_gemv(y, w16, x, f"tcb plan {plan} {fmt}")
    assert gdsq.device_error(0, clear=True) == 0


def test_gemv_batched_paths_agree(gdsq, cuda, monkeypatch):
    """Tensor-core and CUDA-core batched results are both within the bar of
    the exact product (and so within twice the bar of each other)."""
    n, k, batch = 4096, 4096, 8
    ws, w16 = _weights("q4_0", n, k, 0, seed=12)
    x = synth.activations(batch, k, seed=13).to(cuda)
    monkeypatch.setenv("GDSQ_GEMV_TCB", "0")
    y_cc = _run(gdsq, "q4_0", ws, x, n, k, 0)
    monkeypatch.setenv("GDSQ_GEMV_TCB", "1")
    y_tc = _run(gdsq, "q4_0", ws, x, n, k, 0)
    torch.cuda.synchronize()
    _check_gemv(y_cc, w16, x, "cuda cores")
    _check_gemv(y_tc, w16, x, "tensor cores")


# ---- grouped launch: matrices sharing x (q/k/v, gate/up) ---------------------

@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
@pytest.mark.parametrize("dims,k", [((4096, 4096, 4096), 4096), ((4096, 1024, 1024), 8192), ((11008, 11008), 4096),
                                    ((100, 33, 300, 64), 1024), ((96, 40), 96)])
@pytest.mark.parametrize("batch", [1, 3, 8])
def test_gemv_group(gdsq, cuda, fmt, dims, k, batch):
    """Each output of one grouped launch meets the GEMV bar of its own matrix
    (K = 96 and batch 8 run as one launch per matrix)."""
    make, deq = (synth.q4_0_weight, oracle.dequant_q4_0) if fmt == "q4_0" else (synth.q8_0_weight, oracle.dequant_q8_0)
    ws = [make(n, k, seed=11 * i + n) for i, n in enumerate(dims)]
    x = synth.activations(batch, k, seed=len(dims) + batch).to(cuda)
    ys = gdsq.gemv_group(fmt, [w.to(cuda) for w in ws], x, list(dims), k)
    torch.cuda.synchronize()
    for i, (w, y) in enumerate(zip(ws, ys)):
        _check_gemv(y, deq(w.numpy()).reshape(dims[i], k), x, f"group {fmt} m{i} {dims[i]}x{k} b{batch}")
    assert gdsq.device_error(0, clear=True) == 0


def test_gemv_group_validation(gdsq, cuda):
    from gdsllm_b200 import GdsqError
    w = synth.q4_0_weight(64, 256).to(cuda)
    x = synth.activations(1, 256).to(cuda)
    with pytest.raises(GdsqError, match="count"):
        gdsq.gemv_group("q4_0", [w] * 5, x, [64] * 5, 256)


@pytest.mark.parametrize("plan", ["1:2:1", "2:1:1", "4:2:1", "8:1:1", "8:2:1"])
@pytest.mark.parametrize("fmt,batch", [("q4_0", 1), ("q8_0", 3), ("q4_0", 4)])
def test_gemv_cuda_core_launch_plans(gdsq, cuda, plan, fmt, batch, monkeypatch):
    """Every cluster split of the CUDA-core kernel, with many row groups per
    cluster (32000 rows), so the cluster's partial-sum buffers are reused
    and released item after item."""
    monkeypatch.setenv("GDSQ_GEMV_TCB", "0")
    monkeypatch.setenv("GDSQ_GEMV_PLAN", plan)
    n, k = 32000, 4096
    ws, w16 = _weights(fmt, n, k, 0, seed=17)
    x = synth.activations(batch, k, seed=18).to(cuda)
    y = _run(gdsq, fmt, ws, x, n, k, 0)
    torch.cuda.synchronize()
    _check_gemv(y, w16, x, f"cuda-core plan {plan} {fmt} b{batch}")
    assert gdsq.device_error(0, clear=True) == 0
