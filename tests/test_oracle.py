"""Pins the CPU oracle (our restatement) against the golden vectors that the
reference's own kernels produced (tests/golden/make_golden.py).  CPU only."""
import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden

INT4_CASES = sorted(os.path.basename(p) for p in glob.glob(os.path.join(GOLDEN, "int4_gemv_*.npz")))


@pytest.mark.parametrize("name", INT4_CASES)
def test_int4_gemv_restatement_matches_reference_bitexact(oracle_mod, name):
    g = golden(name)
    K, N, gs = int(g["K"]), int(g["N"]), int(g["gs"])
    Z = g["Z"] if "Z" in g else None
    C = oracle_mod.matmul_int4_grouped(g["A"], g["B"], g["S"], Z, K, N, gs)
    assert np.array_equal(C.ravel().view(np.uint16), g["C"].view(np.uint16))


@pytest.mark.parametrize("name", INT4_CASES)
def test_int4_packer_pinned(oracle_mod, name):
    g = golden(name)
    if "W" not in g:
        pytest.skip("no weights stored for this case")
    B, S, Z = oracle_mod.quantize_int4_grouped(g["W"], int(g["gs"]), bool(g["sym"]))
    assert np.array_equal(B, g["B"])
    assert np.array_equal(S.view(np.uint16), g["S"].view(np.uint16))
    if Z is not None:
        assert np.array_equal(Z, g["Z"])


def test_int4_quant_params_match_reference_calibration(oracle_mod):
    """Scale / zero point of a group equal python/armcc/calibration.py:37-50's."""
    g = golden("int4_quant_params.npz")
    mins, maxs = g["min"], g["max"]
    n = len(mins)
    K = 8
    W = np.zeros((K, n), np.float32)
    for j in range(n):
        W[:, j] = np.linspace(mins[j], maxs[j], K, dtype=np.float32)
        W[0, j], W[-1, j] = mins[j], maxs[j]
    B, S, Z = oracle_mod.quantize_int4_grouped(W, K, False)
    want_s = g["scale"].astype(np.float32).astype(np.float16)
    assert np.array_equal(S[0].view(np.uint16), want_s.view(np.uint16))
    assert np.array_equal(Z[0].astype(np.int32), g["zp"])


def test_int4_dequant_equals_reference_weight_formula(oracle_mod):
    g = golden("int4_gemv_k130_n48_g32_partial.npz")
    K, N, gs = int(g["K"]), int(g["N"]), int(g["gs"])
    W = oracle_mod.dequant_int4_grouped(g["B"], g["S"], g["Z"], K, N, gs)
    # C = A @ W computed in the reference's order must reproduce the golden output
    A = g["A"].astype(np.float32)
    acc = np.zeros(N, np.float32)
    for k in range(0, K, 2):
        acc = (acc + A[k] * W[k]).astype(np.float32)
        if k + 1 < K:
            acc = (acc + A[k + 1] * W[k + 1]).astype(np.float32)
    assert np.array_equal(acc.astype(np.float16).view(np.uint16), g["C"].view(np.uint16))


def test_fp16_gemv_restatement(oracle_mod):
    g = golden("fp16_gemv.npz")
    K, N = g["B"].shape
    C = oracle_mod.matmul_f16w(g["A"], g["B"], None, 1, K, N).ravel()
    assert np.array_equal(C.view(np.uint16), g["C_scalar"].view(np.uint16))
    assert np.array_equal(C.view(np.uint16), g["C_neon"].view(np.uint16))
    # bias: the NEON path rounds to fp16 before adding; ours adds in fp32 first
    Cb = oracle_mod.matmul_f16w(g["A"], g["B"], g["bias"], 1, K, N).ravel().astype(np.float32)
    np.testing.assert_allclose(Cb, g["C_neon_bias"].astype(np.float32), rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("name", ["attn_fp16_gqa_causal.npz", "attn_fp16_mha_noncausal.npz",
                                  "attn_fp16_gqa7_causal.npz"])
def test_attention_fp16_restatement_bitexact(oracle_mod, name):
    g = golden(name)
    O = oracle_mod.flash_attention(g["Q"], g["K"], g["V"], causal=bool(g["causal"]))
    assert np.array_equal(O.view(np.uint16), g["O"].view(np.uint16))


def test_attention_f32_head_restatement_bitexact(oracle_mod):
    g = golden("attn_f32_head.npz")
    O = oracle_mod.flash_attention(g["Q"], g["K"], g["V"], causal=True, scale=float(g["scale"]))
    assert np.array_equal(O, g["O"])


def test_block_ops_restatement(oracle_mod):
    g = golden("block_ops.npz")
    x, w = g["x"], g["w"]
    assert np.array_equal(oracle_mod.rmsnorm_f16(x, w).view(np.uint16), g["rmsnorm_scalar"].view(np.uint16))
    assert np.array_equal(oracle_mod.silu_f16(x).view(np.uint16), g["silu_scalar"].view(np.uint16))
    assert np.array_equal(oracle_mod.softmax_f16(x).view(np.uint16), g["softmax_scalar"].view(np.uint16))
    assert np.array_equal(oracle_mod.rope_f16(x[:64].copy(), 37, 500000.0).view(np.uint16),
                          g["rope_scalar"].view(np.uint16))
    # the NEON branches sum in a different order (vaddvq_f32) -- equal within fp16 rounding
    for op in ("rmsnorm", "silu", "softmax"):
        np.testing.assert_allclose(g[f"{op}_neon"].astype(np.float32), g[f"{op}_scalar"].astype(np.float32),
                                   rtol=2e-3, atol=1e-3)


def test_int8_channel_known_answer(oracle_mod):
    rng = np.random.default_rng(3)
    M, K, N = 3, 37, 20
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    s = rng.random(N).astype(np.float32)
    C = oracle_mod.gemm_int8_channel(A, B, s, M, K, N, 0.5)
    acc = A.astype(np.int64) @ B.astype(np.int64)
    want = (acc.astype(np.float32) * np.float32(0.5)) * s
    assert np.array_equal(C, want.astype(np.float32))


def test_bf16_helpers_roundtrip(oracle_mod):
    x = np.array([1.0, -2.5, 3.14159, 1e-3, 65504.0], np.float32)
    b = oracle_mod.f32_to_bf16_bits(x)
    y = oracle_mod.bf16_bits_to_f32(b)
    np.testing.assert_allclose(y, x, rtol=4e-3)


def test_int8_channel_matches_reference_golden(oracle_mod):
    """The restated INT8 per-channel kernel against the reference's own
    OpenCL-C gemm_int8_m1 (opencl_kernels.h:36-52) run as host C: bit for bit."""
    g = golden("int8_channel.npz")
    for name in g["cases"]:
        A, B, s, C = (g[f"{name}_{k}"] for k in ("A", "B", "s", "C"))
        K, N = B.shape
        got = oracle_mod.gemm_int8_channel(A[None, :], B, s, 1, K, N, float(g[f"{name}_scale_A"]))
        assert np.array_equal(got[0].view(np.uint32), C.view(np.uint32)), name
