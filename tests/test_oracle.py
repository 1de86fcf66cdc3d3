"""CPU tests of the parity oracle itself: the C restatement against an
independent numpy restatement, against the third-party gguf 0.19.0
dequantizer (committed golden vectors), against numpy's fp16 rounding, and
against the reference's own CUDA kernels (golden vectors recorded on a B200,
when present)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle
from gdsllm_b200 import synth
from tests.conftest import assert_f16_bitexact

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_half_conversions_match_numpy_on_every_half():
    allh = np.arange(65536, dtype=np.uint16)
    got = oracle.halves_to_floats(allh)
    ref = allh.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(got[~nan], ref[~nan])
    assert np.isnan(got[nan]).all()


def test_float_to_half_matches_numpy_rne():
    rng = np.random.default_rng(0)
    f = np.concatenate([
        rng.standard_normal(200_000).astype(np.float32) * np.float32(3000),
        rng.standard_normal(50_000).astype(np.float32) * np.float32(1e-5),   # subnormal range
        np.array([65504, 65519.99, 65520, 65536, 1e-8, 2 ** -25, 2 ** -24 * 1.5, 2 ** -24 * 2.5,
                  2 ** -14, -0.0, 0.0, np.inf, -np.inf], np.float32),
        # exact ties between fp16 neighbours
        (np.arange(1, 2000, dtype=np.float32) + np.float32(0.5)) * np.float32(2 ** -10),
    ])
    with np.errstate(over="ignore"):
        ref = f.astype(np.float16)
    assert_f16_bitexact(oracle.floats_to_halves(f), ref, "f32->f16")


@pytest.mark.parametrize("n,k", [(1, 32), (7, 64), (64, 512), (33, 4096)])
def test_c_and_numpy_restatements_agree(n, k):
    w = synth.q4_0_weight(n, k, seed=n).numpy()
    assert_f16_bitexact(oracle.dequant_q4_0(w), oracle.np_dequant_q4_0(w), "q4_0")
    w8 = synth.q8_0_weight(n, k, seed=n).numpy()
    assert_f16_bitexact(oracle.dequant_q8_0(w8), oracle.np_dequant_q8_0(w8), "q8_0")
    for g in (32, 128):
        if k % g:
            continue
        words, s, b = (t.numpy() for t in synth.affine_q4_weight(n, k, group=g, seed=n))
        assert_f16_bitexact(oracle.dequant_affine_q4(words, s, b, g),
                            oracle.np_dequant_affine_q4(words, s, b, g), f"affine g={g}")


def test_oracle_matches_gguf_golden_vectors():
    z = np.load(GOLDEN / "gguf_blocks.npz")
    assert str(z["gguf_version"]) == "0.19.0"
    for fmt, fn in (("q4_0", oracle.dequant_q4_0), ("q8_0", oracle.dequant_q8_0)):
        with np.errstate(all="ignore"):
            expected = z[f"{fmt}_gguf_f32"].astype(np.float16)
        assert_f16_bitexact(fn(z[f"{fmt}_blocks"]), expected, f"{fmt} vs gguf")


def test_affine_is_one_fp32_rounding_then_fp16():
    # nibble*scale is exact in fp32 (4-bit x 11-bit significands), so the
    # value is rounded once, when the bias is added, then rounded to fp16.
    # Edge cases: tiny scales against large biases, subnormal scales, overflow.
    rng = np.random.default_rng(5)
    s = np.concatenate([rng.normal(0, 0.01, 64), [2 ** -24, 2 ** -14, 1e-3, 60000.0, -3.0, 0.0]])
    b = np.concatenate([rng.normal(0, 0.01, 64), [2048.0, -2047.0, 1000.0, 65504.0, 0.5, -0.0]])
    s = s.astype(np.float16)
    b = b.astype(np.float16)
    words = rng.integers(0, 2 ** 32, (s.size, 128 // 8), dtype=np.uint64).astype(np.uint32)
    got = oracle.dequant_affine_q4(words, s, b, 128).reshape(-1)
    nib = ((words.reshape(-1)[:, None] >> (np.arange(8, dtype=np.uint32) * 4)) & 0xF).reshape(-1)
    exact = nib.astype(np.float64) * np.repeat(s.astype(np.float64), 128) + \
        np.repeat(b.astype(np.float64), 128)
    with np.errstate(over="ignore"):
        expected = exact.astype(np.float32).astype(np.float16)
    assert_f16_bitexact(got, expected, "affine rounding")


def test_reference_kernel_golden_vectors():
    """Oracle vs outputs of GdsLLM's own CUDA kernels, recorded on a B200 by
    tests/golden/make_ref_golden.py."""
    path = GOLDEN / "ref_kernels.npz"
    if not path.exists():
        pytest.skip("reference-kernel fixtures not recorded yet")
    z = np.load(path)
    assert_f16_bitexact(oracle.dequant_q4_0(z["q4_0_w"]), z["q4_0_dequant"], "ref q4_0 dequant")
    assert_f16_bitexact(oracle.dequant_q8_0(z["q8_0_w"]), z["q8_0_dequant"], "ref q8_0 dequant")
    g = int(z["affine_group"])
    assert_f16_bitexact(oracle.dequant_affine_q4(z["affine_words"], z["affine_scales"],
                                                 z["affine_biases"], g).reshape(-1),
                        z["affine_dequant"], "ref affine dequant")
    for fmt in ("q4_0", "q8_0", "affine"):
        w = z[f"{fmt}_dequant"].reshape(z[f"{fmt}_shape"])
        x = z[f"{fmt}_x"]
        exact = oracle.gemv_exact(w, x)
        bound = oracle.error_bound(w, x)[:, None]
        err = np.abs(z[f"{fmt}_gemv"].astype(np.float64) - exact)
        assert (err <= bound).all(), f"{fmt}: reference kernel outside the bar?"


def test_gemv_cpu_path_is_within_the_bar():
    w = oracle.dequant_q4_0(synth.q4_0_weight(256, 1024).numpy()).reshape(256, 1024)
    x = synth.activations(3, 1024).numpy()
    y = oracle.gemv_cpu(w, x)
    err = np.abs(y.astype(np.float64) - oracle.gemv_exact(w, x))
    assert (err <= oracle.error_bound(w, x)[:, None]).all()


def test_moe_oracle_matches_reference_decode_code():
    """oracle.moe_mlp_reference reproduces, bit for bit, GdsLLM's own
    moe_mlp_selective decode arithmetic (recorded by make_moe_golden.py with
    the fused GEMV replaced by the oracle's CPU GEMV)."""
    z = np.load(GOLDEN / "moe_decode.npz")
    g = int(z["group"])

    def st(name):
        return (z[f"{name}_w"], z[f"{name}_s"], z[f"{name}_b"])

    y = oracle.moe_mlp_reference(z["x"], z["ids"], z["route_w"], st("gate"), st("up"), st("down"), g,
                                 shared=(st("sgate"), st("sup"), st("sdown")),
                                 shared_gate_w=z["shared_gate_w"])
    assert_f16_bitexact(y, z["y"], "moe decode")


def test_moe_exact_forms_agree_with_reference_sequence():
    """The fp64 stage forms used as GPU bars stay within their own bars of
    the reference's fp16 sequence (a check of the bars, on the fixture)."""
    z = np.load(GOLDEN / "moe_decode.npz")
    g = int(z["group"])
    gate, up, down = [(z[f"{n}_w"], z[f"{n}_s"], z[f"{n}_b"]) for n in ("gate", "up", "down")]
    h, _, _ = oracle.moe_gate_up_exact(z["x"], z["ids"], gate, up, g)
    y, bar = oracle.moe_down_exact(h, z["ids"], z["route_w"], down, g)
    ref = oracle.moe_decode_reference(z["x"], z["ids"], z["route_w"], gate, up, down, g)
    err = np.abs(y - ref.astype(np.float64))
    assert (err <= 4 * bar[:, None] + 16 * 2.0 ** -10 * np.abs(ref.astype(np.float64)) + 1e-6).all()
