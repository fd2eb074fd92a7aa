"""Generate the golden vectors under tests/golden/ from the REFERENCE itself.

Run in a checkout where the reference is present (it is not needed later):

    make -C oracle ref REF=<reference checkout>
    python tests/golden/make_golden.py --reference <reference checkout>

Every expected output here comes from the reference's own code:
  * INT4 GEMV, fp16 GEMV, attention and block ops: the reference's CPU kernels
    (compiler/kernels/cpu/matmul_neon.h, flash_attention.h) compiled unmodified
    into oracle/_ref/libsg_ref.so -- NEON branches through oracle/neon_shim
    (the INT4 loop exists only there, matmul_neon.h:114-142) and the scalar
    branches;
  * INT8 per-channel GEMV: the reference's OpenCL-C kernel gemm_int8_m1
    (compiler/kernels/gpu/opencl_kernels.h:36-52), cut out of its string
    literal and compiled as host C into the same library (oracle/ref_opencl.c);
  * INT4 quantisation parameters: python/armcc/calibration.py's
    CalibrationStats.computeQuantParams (imported from the reference).
Inputs are seeded numpy draws (default_rng(seed)); the INT4 weight bytes are
produced by our packer, which the reference does not have -- the packer is
pinned separately against computeQuantParams (int4_quant_params.npz).
"""
from __future__ import annotations

import argparse
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402


def p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def gen_int4_gemv(R):
    cases = [
        # name, K, N, gs, symmetric
        ("k256_n64_g32", 256, 64, 32, False),
        ("k130_n48_g32_partial", 130, 48, 32, False),
        ("k127_n33_g16_sym_oddk", 127, 33, 16, True),
        ("k64_n16_gdefault", 64, 16, 0, False),
        ("k96_n20_g7_oddgroup", 96, 20, 7, False),
        ("k512_n128_g64", 512, 128, 64, False),
    ]
    out = {}
    for i, (name, K, N, gs, sym) in enumerate(cases):
        rng = np.random.default_rng(1000 + i)
        W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
        B, S, Z = oracle.quantize_int4_grouped(W, gs, sym)
        A = rng.integers(-128, 128, K, dtype=np.int8)
        C = np.zeros(N, np.float16)
        R.sgref_neon_matmul_int4_grouped(p(A), p(B), p(S), p(Z), p(C), K, N, gs)
        d = dict(K=K, N=N, gs=gs, sym=int(sym), A=A, B=B, S=S, C=C)
        if K * N <= 16384:
            d["W"] = W  # small cases also pin the packer's bytes
        if Z is not None:
            d["Z"] = Z
        np.savez_compressed(os.path.join(HERE, f"int4_gemv_{name}.npz"), **d)
        out[name] = C
    return out


def gen_quant_params(reference):
    sys.path.insert(0, os.path.join(reference, "python"))
    from armcc.calibration import CalibrationStats

    rng = np.random.default_rng(7)
    mins, maxs, scales, zps = [], [], [], []
    for _ in range(400):
        a, b = sorted(rng.standard_normal(2).astype(np.float32) * rng.choice([0.001, 0.02, 1.0, 30.0]))
        if rng.random() < 0.1:
            b = a  # degenerate range -> defaults
        st = CalibrationStats("t", float(a), float(b), 0.0, 1.0)
        st.computeQuantParams()
        mins.append(a)
        maxs.append(b)
        scales.append(st.scale_int4)
        zps.append(st.zero_point_int4)
    np.savez_compressed(os.path.join(HERE, "int4_quant_params.npz"), min=np.array(mins, np.float32),
                        max=np.array(maxs, np.float32), scale=np.array(scales, np.float64),
                        zp=np.array(zps, np.int32))


def gen_fp16_gemv(R):
    rng = np.random.default_rng(21)
    K, N = 96, 40
    A = rng.standard_normal(K).astype(np.float16)
    B = (rng.standard_normal((K, N)) * 0.1).astype(np.float16)
    bias = rng.standard_normal(N).astype(np.float16)
    C_neon = np.zeros(N, np.float16)
    C_scalar = np.zeros(N, np.float16)
    C_neon_bias = np.zeros(N, np.float16)
    R.sgref_neon_matmul_fp16_m1(p(A), p(B), None, p(C_neon), K, N)
    R.sgref_scalar_matmul_fp16_m1(p(A), p(B), None, p(C_scalar), K, N)
    R.sgref_neon_matmul_fp16_m1(p(A), p(B), p(bias), p(C_neon_bias), K, N)
    np.savez_compressed(os.path.join(HERE, "fp16_gemv.npz"), A=A, B=B, bias=bias, C_neon=C_neon,
                        C_scalar=C_scalar, C_neon_bias=C_neon_bias)


def gen_attention(R):
    # fp16 driver (flash_attention_fp16): causal GQA and non-causal MHA
    for seed, (name, (Bn, H, Hkv, S, D, causal)) in enumerate({
        "gqa_causal": (1, 4, 2, 33, 16, 1),
        "mha_noncausal": (2, 2, 2, 17, 8, 0),
        "gqa7_causal": (1, 7, 1, 24, 32, 1),
    }.items()):
        rng = np.random.default_rng(300 + seed)
        Q = rng.standard_normal((Bn, H, S, D)).astype(np.float16)
        K = rng.standard_normal((Bn, Hkv, S, D)).astype(np.float16)
        V = rng.standard_normal((Bn, Hkv, S, D)).astype(np.float16)
        O = np.zeros_like(Q)
        R.sgref_neon_flash_attention_fp16(p(Q), p(K), p(V), p(O), Bn, S, H, Hkv, D, 0.0, causal)
        np.savez_compressed(os.path.join(HERE, f"attn_fp16_{name}.npz"), Q=Q, K=K, V=V, O=O,
                            causal=causal)
    # fp32 per-query kernel (flash_attn_head) on a config-1-like shape, scaled down
    rng = np.random.default_rng(5)
    H, S, D = 3, 40, 64
    Q = rng.standard_normal((1, H, S, D)).astype(np.float32)
    K = rng.standard_normal((1, H, S, D)).astype(np.float32)
    V = rng.standard_normal((1, H, S, D)).astype(np.float32)
    O = np.zeros_like(Q)
    for h in range(H):
        for s in range(S):
            q = np.ascontiguousarray(Q[0, h, s])
            k = np.ascontiguousarray(K[0, h])
            v = np.ascontiguousarray(V[0, h])
            o = np.zeros(D, np.float32)
            R.sgref_neon_flash_attn_head(p(q), p(k), p(v), p(o), S, D, 1.0 / 8.0, 1, s)
            O[0, h, s] = o
    np.savez_compressed(os.path.join(HERE, "attn_f32_head.npz"), Q=Q, K=K, V=V, O=O, scale=1.0 / 8.0)


def gen_int8_channel(R):
    cases = [
        # name, K, N, scale_A
        ("k37_n20", 37, 20, 0.5),
        ("k256_n64", 256, 64, 0.02),
        ("k1000_n40", 1000, 40, 1.0),
        ("k2048_n24", 2048, 24, 0.0078125),
    ]
    d = {}
    for i, (name, K, N, scale_A) in enumerate(cases):
        rng = np.random.default_rng(500 + i)
        A = rng.integers(-128, 128, K, dtype=np.int8)
        B = rng.integers(-128, 128, (K, N), dtype=np.int8)
        if i == 3:  # extremes: every product at its largest magnitude in some columns
            A[:] = -128
            B[:, :8] = -128
            B[:, 8:16] = 127
        s = (rng.random(N) * 0.01).astype(np.float32)
        C = np.zeros(N, np.float32)
        R.sgref_cl_gemm_int8_m1(p(A), p(B), p(s), p(C), K, N, scale_A)
        d.update({f"{name}_A": A, f"{name}_B": B, f"{name}_s": s, f"{name}_C": C,
                  f"{name}_scale_A": np.float32(scale_A)})
    d["cases"] = np.array([c[0] for c in cases])
    np.savez_compressed(os.path.join(HERE, "int8_channel.npz"), **d)


def gen_block_ops(R):
    rng = np.random.default_rng(33)
    n = 100
    x = rng.standard_normal(n).astype(np.float16)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float16)
    d = {"x": x, "w": w}
    for pre in ("neon", "scalar"):
        y = np.zeros(n, np.float16)
        getattr(R, f"sgref_{pre}_rmsnorm")(p(x), p(w), p(y), n, 1e-5)
        d[f"rmsnorm_{pre}"] = y
        y = np.zeros(n, np.float16)
        getattr(R, f"sgref_{pre}_silu")(p(x), p(y), n)
        d[f"silu_{pre}"] = y
        y = np.zeros(n, np.float16)
        getattr(R, f"sgref_{pre}_softmax")(p(x), p(y), n)
        d[f"softmax_{pre}"] = y
        xr = x[:64].copy()
        getattr(R, f"sgref_{pre}_rope")(p(xr), 64, 37, 500000.0)
        d[f"rope_{pre}"] = xr
    np.savez_compressed(os.path.join(HERE, "block_ops.npz"), **d)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SG_REFERENCE_DIR"),
                    help="the reference checkout (default: $SG_REFERENCE_DIR)")
    ap.add_argument("--only", action="append", default=[],
                    help="generate only these sets (int4_gemv, quant_params, fp16_gemv, attention, block_ops, "
                         "int8_channel); repeatable; default all")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or SG_REFERENCE_DIR")
    oracle.build(ref=True, refdir=args.reference)
    R = oracle.ref()
    gens = {"int4_gemv": lambda: gen_int4_gemv(R), "quant_params": lambda: gen_quant_params(args.reference),
            "fp16_gemv": lambda: gen_fp16_gemv(R), "attention": lambda: gen_attention(R),
            "block_ops": lambda: gen_block_ops(R), "int8_channel": lambda: gen_int8_channel(R)}
    for name in args.only or gens:
        gens[name]()
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
