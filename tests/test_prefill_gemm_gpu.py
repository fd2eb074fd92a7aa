"""Parity of the tcgen05 prefill GEMM (many activation rows) with the oracle,
through the C ABI: INT4 group-quantized weights in the reference layout
(matmul_neon.h:113-147 applied to every row) and INT8 per-channel weights with
float activations.

Tolerance for floating outputs: |got - want| <= 2e-3 + 1e-2 |want|."""
import numpy as np
import pytest
import torch

from test_linear_gpu import DEV, _mm, bf16_tensor, close, t, w4_problem

pytestmark = pytest.mark.gpu


def _acts(oracle_mod, rng, M, K, adt):
    x32 = rng.standard_normal((M, K)).astype(np.float32)
    if adt == "f32":
        return x32, t(x32), {}
    if adt == "f16":
        xo = x32.astype(np.float16)
        return xo, t(xo), {}
    if adt == "bf16":
        return oracle_mod.f32_to_bf16_bits(x32), bf16_tensor(x32), {"a_bf16": True}
    xo = rng.integers(-128, 128, (M, K), dtype=np.int8)
    return xo, t(xo), {}


TDT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


@pytest.fixture(params=[(0, 2), (128, 1), (128, 2), (192, 1), (192, 2), (256, 2)],
                ids=["auto", "bt128_par1", "bt128_par2", "bt192_par1", "bt192_par2", "bt256_par2"])
def token_tile(sg, request):
    """Token tile of the GEMM (0 = automatic) and the number of dequant warp
    groups working on alternate k steps."""
    bt, par = request.param
    sg.set_tuning("gemm_tc.bt", bt)
    sg.set_tuning("gemm_tc.par", par)
    yield request.param
    sg.set_tuning("gemm_tc.bt", 0)
    sg.set_tuning("gemm_tc.par", 2)


@pytest.mark.parametrize("M,K,N,gs,sym,adt,cdt", [
    (64, 256, 128, 64, True, "bf16", "bf16"),
    (130, 2048, 1040, 32, False, "f32", "f32"),     # ragged rows and columns
    (200, 130, 256, 16, False, "f16", "f16"),       # K not a multiple of the 64-k step, groups of 16
    (96, 1000, 384, 128, False, "i8", "f16"),       # reference int8 activations, last group partial
    (257, 512, 640, 256, True, "bf16", "f32"),
])
def test_int4_prefill_vs_oracle(sg, oracle_mod, token_tile, M, K, N, gs, sym, adt, cdt):
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=M + K, sym=sym)
    rng = np.random.default_rng(N)
    xo, xt, kw = _acts(oracle_mod, rng, M, K, adt)
    bias = (0.1 * rng.standard_normal(N)).astype(np.float16)
    scale_A = 0.05 if adt == "i8" else 1.0
    want = oracle_mod.matmul_int4_grouped(xo, B, S, Z, K, N, gs, M=M, bias=bias, c_dt=oracle_mod.DT_F32,
                                          scale_A=scale_A, **kw)
    C = sg.matmul_int4_grouped(xt, t(B), t(S), None if Z is None else t(Z), K, N, gs, out_dtype=TDT[cdt],
                               bias=t(bias), scale_A=scale_A)
    close(C.float().cpu().numpy(), want)


def test_int4_prefill_agrees_with_row_kernel(sg, oracle_mod):
    """The tensor-core GEMM and the CUDA-core row kernel on one problem."""
    M, K, N, gs = 160, 1024, 768, 32
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=7)
    x = t(np.random.default_rng(8).standard_normal((M, K)).astype(np.float32))
    args = (x, t(B), t(S), t(Z), K, N, gs)
    a = sg.matmul_int4_grouped(*args, out_dtype=torch.float32)
    sg.set_tuning("w4_gemv.path", 1)
    try:
        b = sg.matmul_int4_grouped(*args, out_dtype=torch.float32)
    finally:
        sg.set_tuning("w4_gemv.path", 0)
    close(a.cpu().numpy(), b.cpu().numpy())
    assert torch.equal(a, sg.matmul_int4_grouped(*args, out_dtype=torch.float32))  # deterministic


@pytest.mark.parametrize("M,K,N,adt", [
    (64, 512, 256, "bf16"),
    (300, 1000, 1040, "f32"),
    (129, 96, 128, "f16"),
])
def test_int8_prefill_vs_oracle(sg, oracle_mod, token_tile, M, K, N, adt):
    rng = np.random.default_rng(M)
    xo, xt, kw = _acts(oracle_mod, rng, M, K, adt)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    s = (rng.random(N) * 1e-3).astype(np.float32)
    want = oracle_mod.gemm_w8_channel(xo, B, s, M, K, N, **kw)
    C = torch.zeros((M, N), dtype=torch.float32, device=DEV)
    _mm(sg, "sg_matmul_int8_channel", xt, t(B), C, M, K, N, scales=t(s))
    close(C.cpu().numpy(), want)


def _row_subset(M, seed):
    rng = np.random.default_rng(seed)
    return np.unique(np.concatenate([[0, 1, 127, 128, M - 1], rng.integers(0, M, 11)]))


def test_prefill_benchmark_shape_int4(sg, oracle_mod):
    """[2048, 2048] bf16 activations x INT4 symmetric groups of 64 [2048, 8192], bf16 out:
    16 rows checked against the oracle, all rows finite."""
    M, K, N, gs = 2048, 2048, 8192, 64
    B, S, _ = w4_problem(oracle_mod, K, N, gs, seed=31, sym=True)
    x32 = np.random.default_rng(32).standard_normal((M, K)).astype(np.float32)
    C = sg.matmul_int4_grouped(bf16_tensor(x32), t(B), t(S), None, K, N, gs, out_dtype=torch.bfloat16)
    rows = _row_subset(M, 33)
    xo = oracle_mod.f32_to_bf16_bits(x32[rows])
    want = oracle_mod.matmul_int4_grouped(xo, B, S, None, K, N, gs, M=len(rows), c_dt=oracle_mod.DT_F32,
                                          a_bf16=True)
    got = C.float().cpu().numpy()
    assert np.isfinite(got).all()
    close(got[rows], want)


def test_prefill_benchmark_shape_int8(sg, oracle_mod):
    M, K, N = 2048, 2048, 8192
    rng = np.random.default_rng(41)
    x32 = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    s = (rng.random(N) * 1e-3).astype(np.float32)
    C = torch.zeros((M, N), dtype=torch.bfloat16, device=DEV)
    _mm(sg, "sg_matmul_int8_channel", bf16_tensor(x32), t(B), C, M, K, N, scales=t(s))
    rows = _row_subset(M, 42)
    want = oracle_mod.gemm_w8_channel(oracle_mod.f32_to_bf16_bits(x32[rows]), B, s, len(rows), K, N, a_bf16=True)
    close(C.float().cpu().numpy()[rows], want)


def test_prefill_caller_workspace_keeps_gemv_tickets(sg, oracle_mod):
    """One caller workspace shared by the prefill GEMM (which converts fp32
    activations into it) and the single-row GEMV (which keeps zeroed counters
    at its start)."""
    K, N, gs = 1024, 2048, 32
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=51)
    rng = np.random.default_rng(52)
    xm = t(rng.standard_normal((192, K)).astype(np.float32))
    x1 = t(rng.standard_normal((1, K)).astype(np.float32))
    wargs = (t(B), t(S), t(Z), K, N, gs)
    need = max(sg.matmul_int4_grouped_workspace_size(xm, *wargs, out_dtype=torch.float32),
               sg.matmul_int4_grouped_workspace_size(x1, *wargs, out_dtype=torch.float32))
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    ref_m = sg.matmul_int4_grouped(xm, *wargs, out_dtype=torch.float32)
    ref_1 = sg.matmul_int4_grouped(x1, *wargs, out_dtype=torch.float32)
    for _ in range(2):
        assert torch.equal(sg.matmul_int4_grouped(xm, *wargs, out_dtype=torch.float32, workspace=ws), ref_m)
        assert torch.equal(sg.matmul_int4_grouped(x1, *wargs, out_dtype=torch.float32, workspace=ws), ref_1)


def test_prefill_no_device_error(sg):
    from silicongraph_b200 import _lib
    _lib.check(_lib.load().sg_device_error_check(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("cdt", [torch.bfloat16, torch.float16])
def test_prefill_store_paths_identical(sg, oracle_mod, cdt):
    """The TMA-store epilogue and the direct-store epilogue write the same bits,
    also into a C with padded rows (ldc > N) and ragged M / N edges."""
    import ctypes
    from silicongraph_b200 import _lib
    M, K, N, gs = 200, 512, 400, 32
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=61)
    x = t(np.random.default_rng(62).standard_normal((M, K)).astype(np.float32)).to(torch.bfloat16)
    outs = []
    for tma in (1, 0):
        sg.set_tuning("gemm_tc.tma_store", tma)
        try:
            Cpad = torch.full((M, N + 24), 7.0, dtype=cdt, device=DEV)
            p = sg.matmul_params(x, t(B), Cpad, M=M, K=K, N=N, scales=t(S), zeros=t(Z), group_size=gs)
            p.ldc = N + 24
            _lib.check(_lib.load().sg_matmul_int4_grouped(ctypes.byref(p), torch.cuda.current_stream().cuda_stream))
            outs.append(Cpad)
        finally:
            sg.set_tuning("gemm_tc.tma_store", 1)
    assert torch.equal(outs[0], outs[1])
    assert (outs[0][:, N:] == 7.0).all()  # the padding columns are untouched
    want = oracle_mod.matmul_int4_grouped(oracle_mod.f32_to_bf16_bits(x.float().cpu().numpy()), B, S, Z, K, N, gs,
                                          M=M, c_dt=oracle_mod.DT_F32, a_bf16=True)
    close(outs[0][:, :N].float().cpu().numpy(), want)


@pytest.mark.parametrize("M,K,N,gs,zeros,cdt", [
    (256, 2048, 2048, 32, True, torch.float32),      # one round of 16 tiles: every tile split in two k halves
    (200, 1024, 1000, 64, False, torch.bfloat16),    # ragged rows and columns in the split tiles
    (1300, 1024, 4096, 128, True, torch.float16),    # 6 x 32 = 192 tiles: 44 of them split after one whole round
])
def test_prefill_split_last_round(sg, oracle_mod, M, K, N, gs, zeros, cdt):
    """The last, partial round of tiles split into two k halves on two SMs
    (fp32 partial sums in the scratch, the second half to finish adds them):
    within tolerance of the oracle on every row and of the unsplit GEMM, and
    the same bits on every run."""
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=M + N, sym=not zeros)
    x32 = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
    args = (t(x32), t(B), t(S), None if Z is None else t(Z), K, N, gs)
    split = sg.matmul_int4_grouped(*args, out_dtype=cdt)
    assert torch.equal(split, sg.matmul_int4_grouped(*args, out_dtype=cdt))
    sg.set_tuning("gemm_tc.split", 0)
    try:
        whole = sg.matmul_int4_grouped(*args, out_dtype=cdt)
    finally:
        sg.set_tuning("gemm_tc.split", 1)
    want = oracle_mod.matmul_int4_grouped(x32, B, S, Z, K, N, gs, M=M, c_dt=oracle_mod.DT_F32)
    close(split.float().cpu().numpy(), want)
    close(whole.float().cpu().numpy(), want)
    close(split.float().cpu().numpy(), whole.float().cpu().numpy())


@pytest.fixture
def cta_pairs(sg):
    """Tiles of 256 weight columns x 256 tokens on clusters of two CTAs
    (tcgen05 cta_group::2), forced for every shape."""
    sg.set_tuning("gemm_tc.bt", 256)
    sg.set_tuning("gemm_tc.pair", 2)
    yield
    sg.set_tuning("gemm_tc.pair", 0)
    sg.set_tuning("gemm_tc.bt", 0)


@pytest.mark.parametrize("M,K,N,gs,zeros,adt,cdt", [
    (300, 512, 1000, 32, True, "f32", torch.float32),     # ragged rows and a ragged last column pair
    (256, 2048, 384, 64, False, "bf16", torch.bfloat16),  # the second CTA of the last pair: 128 columns
    (520, 1024, 2048, 16, False, "f16", torch.float16),   # groups of 16; last token tile 8 rows
    (96, 1000, 640, 128, True, "i8", torch.float16),      # int8 activations, partial last group
])
def test_int4_prefill_cta_pairs_vs_oracle(sg, oracle_mod, cta_pairs, M, K, N, gs, zeros, adt, cdt):
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=M + 3 * N, sym=not zeros)
    rng = np.random.default_rng(K + N)
    xo, xt, kw = _acts(oracle_mod, rng, M, K, adt)
    bias = (0.1 * rng.standard_normal(N)).astype(np.float16)
    scale_A = 0.05 if adt == "i8" else 1.0
    want = oracle_mod.matmul_int4_grouped(xo, B, S, Z, K, N, gs, M=M, bias=bias, c_dt=oracle_mod.DT_F32,
                                          scale_A=scale_A, **kw)
    args = (xt, t(B), t(S), None if Z is None else t(Z), K, N, gs)
    C = sg.matmul_int4_grouped(*args, out_dtype=cdt, bias=t(bias), scale_A=scale_A)
    close(C.float().cpu().numpy(), want)
    assert torch.equal(C, sg.matmul_int4_grouped(*args, out_dtype=cdt, bias=t(bias), scale_A=scale_A))


@pytest.mark.parametrize("M,K,N,adt", [(300, 1000, 1040, "f32"), (512, 512, 512, "bf16")])
def test_int8_prefill_cta_pairs_vs_oracle(sg, oracle_mod, cta_pairs, M, K, N, adt):
    rng = np.random.default_rng(M + 1)
    xo, xt, kw = _acts(oracle_mod, rng, M, K, adt)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    s = (rng.random(N) * 1e-3).astype(np.float32)
    want = oracle_mod.gemm_w8_channel(xo, B, s, M, K, N, **kw)
    C = torch.zeros((M, N), dtype=torch.float32, device=DEV)
    _mm(sg, "sg_matmul_int8_channel", xt, t(B), C, M, K, N, scales=t(s))
    close(C.cpu().numpy(), want)


def test_prefill_benchmark_shape_cta_pairs(sg, oracle_mod):
    """[2048, 2048] bf16 x INT4 symmetric g64 [2048, 8192] on CTA pairs: within
    tolerance of the oracle on sampled rows and of the one-CTA kernel on all."""
    M, K, N, gs = 2048, 2048, 8192, 64
    B, S, _ = w4_problem(oracle_mod, K, N, gs, seed=31, sym=True)
    x32 = np.random.default_rng(32).standard_normal((M, K)).astype(np.float32)
    args = (bf16_tensor(x32), t(B), t(S), None, K, N, gs)
    sg.set_tuning("gemm_tc.pair", 1)
    try:
        C = sg.matmul_int4_grouped(*args, out_dtype=torch.bfloat16)
    finally:
        sg.set_tuning("gemm_tc.pair", 0)
    one = sg.matmul_int4_grouped(*args, out_dtype=torch.bfloat16)
    rows = _row_subset(M, 34)
    xo = oracle_mod.f32_to_bf16_bits(x32[rows])
    want = oracle_mod.matmul_int4_grouped(xo, B, S, None, K, N, gs, M=len(rows), c_dt=oracle_mod.DT_F32,
                                          a_bf16=True)
    got = C.float().cpu().numpy()
    close(got[rows], want)
    close(got, one.float().cpu().numpy())
