"""Parity of the CUDA linear kernels with the oracle and the reference goldens,
called through the C ABI (silicongraph_b200.kernels -> libsg_b200.so).

Tolerance for floating outputs: |got - want| <= 2e-3 + 1e-2 |want|.
Integer work (packing, unpacking, int8 x int8) is compared bit for bit."""
import glob
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, golden

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-3
DEV = "cuda"


def close(got, want, rtol=RTOL, atol=ATOL):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    err = np.abs(got - want)
    bad = err > atol + rtol * np.abs(want)
    assert not bad.any(), f"{bad.sum()} / {bad.size} outside tolerance; max err {err.max():.3e}"


def t(a, dtype=None):
    x = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        x = x.to(dtype)
    return x.to(DEV)


def bf16_tensor(a32):
    return torch.from_numpy(np.ascontiguousarray(a32, np.float32)).to(torch.bfloat16).to(DEV)


def w4_problem(oracle, K, N, gs, seed=0, sym=False):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    B, S, Z = oracle.quantize_int4_grouped(W, gs, sym)
    return B, S, Z


INT4_CASES = sorted(os.path.basename(p) for p in glob.glob(os.path.join(GOLDEN, "int4_gemv_*.npz")))


@pytest.mark.parametrize("name", INT4_CASES)
def test_int4_gemv_matches_reference_golden(sg, name):
    g = golden(name)
    K, N, gs = int(g["K"]), int(g["N"]), int(g["gs"])
    Z = t(g["Z"]) if "Z" in g else None
    C = sg.matmul_int4_grouped(t(g["A"]).view(1, K), t(g["B"]), t(g["S"]), Z, K, N, gs)
    close(C.cpu().numpy().ravel(), g["C"])


@pytest.mark.parametrize("K,N,gs", [(127, 33, 16), (96, 20, 7), (130, 40, 32), (64, 24, 0)])
def test_int4_generic_path_bitexact(sg, oracle_mod, K, N, gs):
    """Shapes outside the fast path run the reference's loop order exactly."""
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=K)
    rng = np.random.default_rng(1)
    A = rng.standard_normal((2, K)).astype(np.float32)
    want = oracle_mod.matmul_int4_grouped(A, B, S, Z, K, N, gs, M=2, c_dt=oracle_mod.DT_F32)
    C = sg.matmul_int4_grouped(t(A), t(B), t(S), t(Z), K, N, gs, out_dtype=torch.float32)
    assert np.array_equal(C.cpu().numpy(), want)


@pytest.fixture(params=[0, 1], ids=["auto", "cudacore"])
def w4_path(sg, request):
    """Run under the automatic path choice (tensor-core kernel for one row) and
    with the CUDA-core kernel forced."""
    sg.set_tuning("w4_gemv.path", request.param)
    yield request.param
    sg.set_tuning("w4_gemv.path", 0)


@pytest.mark.parametrize("K,N,gs,sym", [
    (4096, 14336, 32, False),   # the INT4 GEMV benchmark shape (x fp32 [1, 4096])
    (2048, 8192, 64, True),
    (4096, 512, 128, False),
    (272, 48, 16, False),       # single split
    (4000, 1024, 32, False),    # partial last group
    (18944, 3584, 128, False),  # Qwen-7B down projection
    (2048, 1040, 32, False),    # N not a multiple of the 512-column tile
    (96, 16, 32, False),        # tiny K: one partial chunk
    (2048, 128256 // 8, 32, False),  # a TP-8 shard of a Llama-3 lm_head
])
def test_int4_fast_path_fp32_activation(sg, oracle_mod, w4_path, K, N, gs, sym):
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=N, sym=sym)
    x = np.random.default_rng(K).standard_normal((1, K)).astype(np.float32)
    want = oracle_mod.matmul_int4_grouped(x, B, S, Z, K, N, gs, c_dt=oracle_mod.DT_F32)
    C = sg.matmul_int4_grouped(t(x), t(B), t(S), t(Z) if Z is not None else None, K, N, gs,
                               out_dtype=torch.float32)
    close(C.cpu().numpy(), want)


def outlier_activations(K, amp, seed, rows=1, group=32):
    """x ~ N(0,1) with one value of magnitude amp..1.5 amp, random sign, in
    every group of `group` k: the heavy-tailed activations real decoders feed
    their linears."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, K)).astype(np.float32)
    for r in range(rows):
        for g0 in range(0, K, group):
            n = min(group, K - g0)
            x[r, g0 + int(rng.integers(0, n))] = np.float32(amp * (1.0 + 0.5 * rng.random())
                                                              * np.sign(rng.standard_normal()))
    return x


@pytest.mark.parametrize("amp", [100.0, 1000.0])
@pytest.mark.parametrize("K,N,gs", [(4096, 14336, 32), (18944, 3584, 128), (2048, 3072, 32)])
def test_int4_fast_path_outlier_activations(sg, oracle_mod, w4_path, K, N, gs, amp):
    """One large activation per 32 k through the fp32-activation GEMV,
    against the oracle at the same elementwise bar."""
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=N + 1)
    x = outlier_activations(K, amp, seed=K + int(amp))
    want = oracle_mod.matmul_int4_grouped(x, B, S, Z, K, N, gs, c_dt=oracle_mod.DT_F32)
    C = sg.matmul_int4_grouped(t(x), t(B), t(S), t(Z), K, N, gs, out_dtype=torch.float32)
    close(C.cpu().numpy(), want)


@pytest.mark.parametrize("adt", ["f16", "bf16", "i8"])
def test_int4_single_row_dtypes_bias(sg, oracle_mod, w4_path, adt):
    K, N, gs = 3072, 2560, 64
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=21)
    rng = np.random.default_rng(22)
    x32 = rng.standard_normal((1, K)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(N)).astype(np.float16)
    if adt == "f16":
        xo = x32.astype(np.float16)
        xt, kw = t(xo), {}
    elif adt == "bf16":
        xo, xt, kw = oracle_mod.f32_to_bf16_bits(x32), bf16_tensor(x32), {"a_bf16": True}
    else:
        xo = rng.integers(-128, 128, (1, K), dtype=np.int8)
        xt, kw = t(xo), {}
    scale_A = 0.03 if adt == "i8" else 1.0
    want = oracle_mod.matmul_int4_grouped(xo, B, S, Z, K, N, gs, bias=bias, c_dt=oracle_mod.DT_F32,
                                          scale_A=scale_A, **kw)
    C = sg.matmul_int4_grouped(xt, t(B), t(S), t(Z), K, N, gs, out_dtype=torch.float32, bias=t(bias),
                               scale_A=scale_A)
    close(C.cpu().numpy(), want)


def test_int4_paths_agree_on_reference_golden(sg):
    """The reference's own output (int8 activations, fp16 out) from every path."""
    g = golden("int4_gemv_k512_n128_g64.npz")
    K, N, gs = int(g["K"]), int(g["N"]), int(g["gs"])
    try:
        for path in (0, 1, 2):
            sg.set_tuning("w4_gemv.path", path)
            C = sg.matmul_int4_grouped(t(g["A"]).view(1, K), t(g["B"]), t(g["S"]), t(g["Z"]), K, N, gs)
            close(C.cpu().numpy().ravel(), g["C"])
    finally:
        sg.set_tuning("w4_gemv.path", 0)


def test_no_device_error_recorded(sg):
    from silicongraph_b200 import _lib
    _lib.check(_lib.load().sg_device_error_check(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8])
@pytest.mark.parametrize("adt", ["f32", "f16", "bf16", "i8"])
def test_int4_rows_and_dtypes(sg, oracle_mod, M, adt):
    K, N, gs = 1024, 1536, 32
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=11)
    rng = np.random.default_rng(M)
    x32 = rng.standard_normal((M, K)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(N)).astype(np.float16)
    if adt == "f32":
        xo, xt, kw = x32, t(x32), {}
    elif adt == "f16":
        xo = x32.astype(np.float16)
        xt, kw = t(xo), {}
    elif adt == "bf16":
        xo = oracle_mod.f32_to_bf16_bits(x32)
        xt, kw = bf16_tensor(x32), {"a_bf16": True}
    else:
        xo = rng.integers(-128, 128, (M, K), dtype=np.int8)
        xt, kw = t(xo), {}
    scale_A = 0.05 if adt == "i8" else 1.0
    for cdt, tdt in ((oracle_mod.DT_F32, torch.float32), (oracle_mod.DT_F16, torch.float16)):
        want = oracle_mod.matmul_int4_grouped(xo, B, S, Z, K, N, gs, M=M, bias=bias, c_dt=cdt,
                                              scale_A=scale_A, **kw)
        C = sg.matmul_int4_grouped(xt, t(B), t(S), t(Z), K, N, gs, out_dtype=tdt, bias=t(bias),
                                   scale_A=scale_A)
        close(C.float().cpu().numpy(), want.astype(np.float32))


def test_int4_bf16_output(sg, oracle_mod):
    K, N, gs = 512, 1024, 64
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=5)
    x = np.random.default_rng(9).standard_normal((1, K)).astype(np.float32)
    want = oracle_mod.matmul_int4_grouped(x, B, S, Z, K, N, gs, c_dt=oracle_mod.DT_F32)
    C = sg.matmul_int4_grouped(t(x), t(B), t(S), t(Z), K, N, gs, out_dtype=torch.bfloat16)
    close(C.float().cpu().numpy(), want, rtol=1e-2, atol=1e-2)


def test_int4_deterministic_and_k0(sg, oracle_mod):
    K, N, gs = 4096, 2048, 32
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=2)
    x = t(np.random.default_rng(0).standard_normal((1, K)).astype(np.float32))
    a = sg.matmul_int4_grouped(x, t(B), t(S), t(Z), K, N, gs, out_dtype=torch.float32)
    b = sg.matmul_int4_grouped(x, t(B), t(S), t(Z), K, N, gs, out_dtype=torch.float32)
    assert torch.equal(a, b)
    # K == 0: the reference writes zeros (acc never updated)
    C = torch.full((1, 16), 7.0, dtype=torch.float16, device=DEV)
    sg.matmul_int4_grouped(x[:, :0], t(B), t(S), t(Z), 0, 16, gs, C=C)
    assert (C == 0).all()


def test_int4_caller_workspace(sg, oracle_mod):
    from silicongraph_b200._lib import SgError
    K, N, gs = 4096, 4096, 32
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=3)
    x = t(np.random.default_rng(4).standard_normal((1, K)).astype(np.float32))
    args = (x, t(B), t(S), t(Z), K, N, gs)
    sg.set_tuning("w4_gemv_mma.cluster", 0)  # the stream-K split, whose partials need scratch
    try:
        need = sg.matmul_int4_grouped_workspace_size(*args, out_dtype=torch.float32)
        assert need > 0
        ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
        a = sg.matmul_int4_grouped(*args, out_dtype=torch.float32, workspace=ws)
        b = sg.matmul_int4_grouped(*args, out_dtype=torch.float32)
        assert torch.equal(a, b)
        a2 = sg.matmul_int4_grouped(*args, out_dtype=torch.float32, workspace=ws)  # tickets were reset
        assert torch.equal(a, a2)
        with pytest.raises(SgError):
            sg.matmul_int4_grouped(*args, out_dtype=torch.float32, workspace=ws[: need // 2])
    finally:
        sg.set_tuning("w4_gemv_mma.cluster", 1)


@pytest.mark.parametrize("gpw", [1, 2, 4, 8])
def test_int4_split_granularity_invariant(sg, oracle_mod, gpw):
    K, N, gs = 4096, 14336, 32
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=7)
    x = np.random.default_rng(8).standard_normal((1, K)).astype(np.float32)
    want = oracle_mod.matmul_int4_grouped(x, B, S, Z, K, N, gs, c_dt=oracle_mod.DT_F32)
    try:
        sg.set_tuning("w4_gemv.path", 1)
        sg.set_tuning("w4_gemv.groups_per_warp", gpw)
        C = sg.matmul_int4_grouped(t(x), t(B), t(S), t(Z), K, N, gs, out_dtype=torch.float32)
    finally:
        sg.set_tuning("w4_gemv.groups_per_warp", 0)
        sg.set_tuning("w4_gemv.path", 0)
    close(C.cpu().numpy(), want)


# ------------------------------------------------------------------ packer
@pytest.mark.parametrize("K,N,gs,sym", [(256, 64, 32, False), (127, 33, 16, True), (96, 20, 7, False),
                                        (4096, 1024, 32, False), (130, 48, 0, False)])
def test_device_packer_bitexact(sg, oracle_mod, K, N, gs, sym):
    import ctypes
    from silicongraph_b200 import _lib
    rng = np.random.default_rng(K + N)
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    W[: min(K, 5), 0] = 0.0  # a degenerate-ish column start
    B0, S0, Z0 = oracle_mod.quantize_int4_grouped(W, gs, sym)
    Wd = t(W)
    B = torch.zeros(B0.shape, dtype=torch.uint8, device=DEV)
    S = torch.zeros(S0.shape, dtype=torch.float16, device=DEV)
    Z = torch.zeros(S0.shape, dtype=torch.int8, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.load().sg_quantize_int4_grouped(Wd.data_ptr(), K, N, gs, int(sym), B.data_ptr(),
                                                     S.data_ptr(), None if sym else Z.data_ptr(), st))
    assert np.array_equal(B.cpu().numpy(), B0)
    assert np.array_equal(S.cpu().numpy().view(np.uint16), S0.view(np.uint16))
    if not sym:
        assert np.array_equal(Z.cpu().numpy(), Z0)
    # unpack
    Wq = torch.zeros((K, N), dtype=torch.float32, device=DEV)
    _lib.check(_lib.load().sg_dequantize_int4_grouped(B.data_ptr(), S.data_ptr(),
                                                       None if sym else Z.data_ptr(), K, N, gs,
                                                       Wq.data_ptr(), st))
    want = oracle_mod.dequant_int4_grouped(B0, S0, Z0, K, N, gs)
    assert np.array_equal(Wq.cpu().numpy(), want)
    del ctypes


# ------------------------------------------------------------------ int8 / fp16
def _mm(sg, fn, A, B, C, M, K, N, scales=None, bias=None, scale_A=1.0):
    import ctypes
    from silicongraph_b200 import _lib
    p = sg.matmul_params(A, B, C, M=M, K=K, N=N, scales=scales, bias=bias, scale_A=scale_A)
    _lib.check(getattr(_lib.load(), fn)(ctypes.byref(p), torch.cuda.current_stream().cuda_stream))
    return C


@pytest.mark.parametrize("M,K,N", [(1, 2048, 8192), (1, 37, 20), (3, 1000, 512), (1, 4096, 14336)])
def test_int8_channel_int8_activations_bitexact(sg, oracle_mod, M, K, N):
    rng = np.random.default_rng(K)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    s = (rng.random(N) * 0.01).astype(np.float32)
    want = oracle_mod.gemm_int8_channel(A, B, s, M, K, N, 0.02)
    C = torch.zeros((M, N), dtype=torch.float32, device=DEV)
    _mm(sg, "sg_matmul_int8_channel", t(A), t(B), C, M, K, N, scales=t(s), scale_A=0.02)
    assert np.array_equal(C.cpu().numpy(), want)


@pytest.mark.parametrize("M", [1, 2])
def test_int8_channel_matches_reference_golden(sg, M):
    """Bit for bit against the reference's own OpenCL-C gemm_int8_m1
    (opencl_kernels.h:36-52) run as host C; M = 2 repeats the row so that the
    multi-row kernel is held to the same reference output."""
    g = golden("int8_channel.npz")
    for name in g["cases"]:
        A, B, s, want = (g[f"{name}_{k}"] for k in ("A", "B", "s", "C"))
        K, N = B.shape
        C = torch.zeros((M, N), dtype=torch.float32, device=DEV)
        _mm(sg, "sg_matmul_int8_channel", t(np.repeat(A[None, :], M, 0)), t(B), C, M, K, N, scales=t(s),
            scale_A=float(g[f"{name}_scale_A"]))
        got = C.cpu().numpy()
        for m in range(M):
            assert np.array_equal(got[m].view(np.uint32), want.view(np.uint32)), (name, m)


@pytest.mark.parametrize("M,K,N,adt", [(1, 2048, 8192, "bf16"), (2, 1024, 1024, "f32"), (1, 100, 48, "f16")])
def test_int8_channel_float_activations(sg, oracle_mod, M, K, N, adt):
    rng = np.random.default_rng(N)
    x32 = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    s = (rng.random(N) * 1e-3).astype(np.float32)
    if adt == "bf16":
        xo, xt, kw = oracle_mod.f32_to_bf16_bits(x32), bf16_tensor(x32), {"a_bf16": True}
    elif adt == "f16":
        xo = x32.astype(np.float16)
        xt, kw = t(xo), {}
    else:
        xo, xt, kw = x32, t(x32), {}
    want = oracle_mod.gemm_w8_channel(xo, B, s, M, K, N, **kw)
    C = torch.zeros((M, N), dtype=torch.float32, device=DEV)
    _mm(sg, "sg_matmul_int8_channel", xt, t(B), C, M, K, N, scales=t(s))
    close(C.cpu().numpy(), want)


@pytest.mark.parametrize("amp", [100.0, 1000.0])
@pytest.mark.parametrize("M,K,N", [(1, 4096, 14336), (2, 2048, 1024)])
def test_int8_channel_outlier_activations(sg, oracle_mod, M, K, N, amp):
    """INT8 weights, fp32 activations with one large value per 32 k."""
    rng = np.random.default_rng(K + int(amp))
    x = outlier_activations(K, amp, seed=N + int(amp), rows=M)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    s = (rng.random(N) * 1e-3).astype(np.float32)
    want = oracle_mod.gemm_w8_channel(x, B, s, M, K, N)
    C = torch.zeros((M, N), dtype=torch.float32, device=DEV)
    _mm(sg, "sg_matmul_int8_channel", t(x), t(B), C, M, K, N, scales=t(s))
    close(C.cpu().numpy(), want)


def test_fp16_gemv_matches_reference_golden(sg):
    g = golden("fp16_gemv.npz")
    K, N = g["B"].shape
    C = torch.zeros((1, N), dtype=torch.float16, device=DEV)
    _mm(sg, "sg_matmul_fp16", t(g["A"]).view(1, K), t(g["B"]), C, 1, K, N)
    close(C.cpu().numpy().ravel(), g["C_neon"])
    _mm(sg, "sg_matmul_fp16", t(g["A"]).view(1, K), t(g["B"]), C, 1, K, N, bias=t(g["bias"]))
    close(C.cpu().numpy().ravel(), g["C_neon_bias"])


@pytest.mark.parametrize("M,K,N", [(1, 2048, 8192), (2, 333, 64), (1, 64, 40)])
def test_fp16_gemv_vs_oracle(sg, oracle_mod, M, K, N):
    rng = np.random.default_rng(M * K)
    A = rng.standard_normal((M, K)).astype(np.float16)
    B = (0.02 * rng.standard_normal((K, N))).astype(np.float16)
    want = oracle_mod.matmul_f16w(A, B, None, M, K, N, c_dt=oracle_mod.DT_F32)
    C = torch.zeros((M, N), dtype=torch.float32, device=DEV)
    _mm(sg, "sg_matmul_fp16", t(A), t(B), C, M, K, N)
    close(C.cpu().numpy(), want)


@pytest.mark.parametrize("cluster", [2, 1, 0, "one-block-per-sm"])
@pytest.mark.parametrize("K,N,gs", [
    (4096, 14336, 32),        # benchmark shape
    (2048, 8192, 64),
    (2048, 128256 // 8, 32),
    (2048, 3072, 32),         # decoder q|k|v projection: 6 tiles shared by many blocks
    (8192, 2048, 32),         # decoder down projection
    (128, 512 * 200, 32),     # ranges longer than K: activation staged by row, 2 tiles per block
    (64, 512 * 300, 64),      # one chunk per tile: ranges over 3 tiles
])
def test_int4_cluster_and_stream_k_splits(sg, oracle_mod, cluster, K, N, gs):
    """Tile-aligned cluster split (partials reduced in distributed shared memory;
    one 16-warp or two 8-warp blocks per SM) and the stream-K split (partials
    of shared tiles reduced through scratch)
    give the oracle's result, repeatably; the static-weight launch (weights
    requested before the dependency wait) gives the same bits."""
    from silicongraph_b200 import _lib
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=N + 1)
    x = np.random.default_rng(K + 1).standard_normal((1, K)).astype(np.float32)
    want = oracle_mod.matmul_int4_grouped(x, B, S, Z, K, N, gs, c_dt=oracle_mod.DT_F32)
    try:
        if cluster == "one-block-per-sm":  # no two-blocks-per-SM cluster shapes
            sg.set_tuning("w4_gemv_mma.pair", 0)
            cluster = 1
        sg.set_tuning("w4_gemv_mma.cluster", cluster)
        args = (t(x), t(B), t(S), t(Z), K, N, gs)
        C = sg.matmul_int4_grouped(*args, out_dtype=torch.float32)
        C2 = sg.matmul_int4_grouped(*args, out_dtype=torch.float32)
        C3 = sg.matmul_int4_grouped(*args, out_dtype=torch.float32, flags=_lib.SG_MM_STATIC_WEIGHTS)
    finally:
        sg.set_tuning("w4_gemv_mma.cluster", 1)
        sg.set_tuning("w4_gemv_mma.pair", 1)
    close(C.cpu().numpy(), want)
    assert torch.equal(C, C2)
    assert torch.equal(C, C3)


@pytest.mark.parametrize("M,K,N,gs,sym", [
    (16, 2048, 3072, 32, False),   # batch-16 decode, q|k|v shape
    (13, 8192, 2048, 32, False),   # odd row count, long K (clusters of K splits)
    (7, 1024, 4096, 128, True),    # symmetric, group 128
    (2, 2048, 8192, 32, False),    # 64 tiles
    (9, 130, 48, 32, False),       # ragged K and a partial tile
])
def test_int4_few_rows_kernel(sg, oracle_mod, M, K, N, gs, sym):
    """2..16 activation rows on the fp16-dequant mma.sync kernel: the oracle's
    result within tolerance, repeatable bit for bit, with and without the
    static-weight launch."""
    from silicongraph_b200 import _lib
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=M * 7 + K, sym=sym)
    x = np.random.default_rng(M + N).standard_normal((M, K)).astype(np.float32)
    xh = x.astype(np.float16)
    want = oracle_mod.matmul_int4_grouped(xh, B, S, Z, K, N, gs, M=M, c_dt=oracle_mod.DT_F32)
    args = (t(xh), t(B), t(S), None if Z is None else t(Z), K, N, gs)
    C = sg.matmul_int4_grouped(*args, out_dtype=torch.float32)
    C2 = sg.matmul_int4_grouped(*args, out_dtype=torch.float32, flags=_lib.SG_MM_STATIC_WEIGHTS)
    close(C.cpu().numpy(), want)
    assert torch.equal(C, C2)


@pytest.mark.parametrize("xdt", ["f32", "bf16"])
def test_int4_few_rows_activation_types(sg, oracle_mod, xdt):
    """fp32 and bf16 activation rows on the few-rows kernel (staged as fp16,
    8 values per load): the oracle's result on the same activations within
    tolerance."""
    M, K, N, gs = 6, 2048, 1024, 32
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=21)
    x = np.random.default_rng(5).standard_normal((M, K)).astype(np.float32)
    if xdt == "bf16":
        xt = bf16_tensor(x)
        x = xt.float().cpu().numpy()
    else:
        xt = t(x)
    want = oracle_mod.matmul_int4_grouped(x, B, S, Z, K, N, gs, M=M, c_dt=oracle_mod.DT_F32)
    C = sg.matmul_int4_grouped(xt, t(B), t(S), t(Z), K, N, gs, out_dtype=torch.float32)
    close(C.cpu().numpy(), want)


@pytest.mark.parametrize("M,K,N,sym", [
    (5, 1024, 40960, False),   # 320 tiles: persistent blocks take two or three tiles each
    (16, 2048, 20480, True),   # 160 tiles: one tile per block, no K split
])
def test_int4_few_rows_persistent(sg, oracle_mod, M, K, N, sym):
    """Wide outputs on the few-rows kernel: persistent blocks without a K
    split; the oracle's result within tolerance and repeatable bit for bit."""
    gs = 32
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=M + 3, sym=sym)
    x = np.random.default_rng(N).standard_normal((M, K)).astype(np.float32).astype(np.float16)
    want = oracle_mod.matmul_int4_grouped(x, B, S, Z, K, N, gs, M=M, c_dt=oracle_mod.DT_F32)
    args = (t(x), t(B), t(S), None if Z is None else t(Z), K, N, gs)
    C = sg.matmul_int4_grouped(*args, out_dtype=torch.float32)
    C2 = sg.matmul_int4_grouped(*args, out_dtype=torch.float32)
    close(C.cpu().numpy(), want)
    assert torch.equal(C, C2)


@pytest.mark.parametrize("M,dt", [(1, torch.float16), (2, torch.float16), (5, torch.float16), (16, torch.float16),
                                  (1, torch.bfloat16), (4, torch.bfloat16)])
def test_int4_swiglu_fused_matches_two_kernels(sg, oracle_mod, M, dt):
    """SG_MM_A_SWIGLU: the down projection staging silu(gate) * up itself gives
    the same bits as sg_swiglu_rows followed by the plain GEMM."""
    from silicongraph_b200 import _lib
    K, N, gs = 2048, 1024, 32
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=M + 40)
    gu = torch.from_numpy(np.random.default_rng(M).standard_normal((M, 2 * K)).astype(np.float32) * 2).to(dt).to(DEV)
    act = sg.swiglu_rows(gu, K)
    want = sg.matmul_int4_grouped(act, t(B), t(S), t(Z), K, N, gs, out_dtype=torch.float32)
    got = sg.matmul_int4_grouped(gu, t(B), t(S), t(Z), K, N, gs, out_dtype=torch.float32,
                                 flags=_lib.SG_MM_A_SWIGLU)
    assert torch.equal(got, want)


def test_int4_swiglu_fused_refuses_many_rows(sg, oracle_mod):
    """The fused SwiGLU exists on the few-row kernels only; a prefill-sized call
    is refused with SG_ERR_UNSUPPORTED instead of computing something else."""
    from silicongraph_b200 import _lib
    K, N, gs = 256, 256, 32
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=3)
    gu = torch.zeros((64, 2 * K), dtype=torch.float16, device=DEV)
    with pytest.raises(Exception, match="SG_MM_A_SWIGLU"):
        sg.matmul_int4_grouped(gu, t(B), t(S), t(Z), K, N, gs, flags=_lib.SG_MM_A_SWIGLU)


@pytest.mark.parametrize("M,K,N,gs", [(17, 2048, 3072, 32), (24, 3584, 4608, 128), (32, 1024, 40960, 32),
                                      (32, 2368, 3584, 128)])
def test_int4_two_pass_rows(sg, oracle_mod, M, K, N, gs):
    """17..32 activation rows run as two passes of the few-row kernel (the
    second over rows 16..M-1): the oracle's result within tolerance."""
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=M + K)
    x = np.random.default_rng(M * 3).standard_normal((M, K)).astype(np.float32).astype(np.float16)
    want = oracle_mod.matmul_int4_grouped(x, B, S, Z, K, N, gs, M=M, c_dt=oracle_mod.DT_F32)
    C = sg.matmul_int4_grouped(t(x), t(B), t(S), t(Z), K, N, gs, out_dtype=torch.float32)
    close(C.cpu().numpy(), want)


# ------------------------------------------------------------------ fused norm / residual add
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("K,N,gs", [(2048, 3072, 32), (3584, 4608, 128), (2048, 128256 // 8, 32)])
def test_fused_rmsnorm_gemv_equals_two_kernels(sg, oracle_mod, dt, K, N, gs):
    """SG_MM_A_RMSNORM: the GEMV of RMSNorm(h) equals sg_rmsnorm then the GEMV,
    bit for bit (both form the row's sum of squares the same way)."""
    from silicongraph_b200._lib import SG_MM_A_RMSNORM
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=K + N)
    g = torch.Generator(device="cuda")
    g.manual_seed(K)
    h = (torch.randn(1, K, generator=g, device="cuda") * 3).to(dt)
    w = (1 + 0.1 * torch.randn(K, generator=g, device="cuda")).to(dt)
    xn = sg.rmsnorm(h, w, eps=1e-5)
    want = sg.matmul_int4_grouped(xn, t(B), t(S), t(Z), K, N, gs, out_dtype=dt)
    import ctypes
    from silicongraph_b200 import _lib
    got = torch.empty_like(want)
    p = sg.matmul_params(h, t(B), got, M=1, K=K, N=N, scales=t(S), zeros=t(Z), group_size=gs,
                         flags=SG_MM_A_RMSNORM, norm_weight=w, norm_eps=1e-5)
    _lib.check(_lib.load().sg_matmul_int4_grouped(ctypes.byref(p), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_accumulating_gemv_equals_residual_add(sg, oracle_mod, dt):
    """SG_MM_C_ACCUMULATE: C = round(C + round(y)) equals the GEMV followed by
    sg_rmsnorm's residual update, bit for bit."""
    import ctypes
    from silicongraph_b200 import _lib
    from silicongraph_b200._lib import SG_MM_C_ACCUMULATE
    K, N, gs = 8192, 2048, 32
    B, S, Z = w4_problem(oracle_mod, K, N, gs, seed=3)
    x = torch.randn(1, K, device="cuda").to(dt)
    resid0 = (torch.randn(1, N, device="cuda") * 4).to(dt)
    y = sg.matmul_int4_grouped(x, t(B), t(S), t(Z), K, N, gs, out_dtype=dt)
    want = resid0.clone()
    sg.rmsnorm(y, torch.ones(N, dtype=dt, device="cuda"), residual=want)  # want = round(resid0 + y)
    got = resid0.clone()
    p = sg.matmul_params(x, t(B), got, M=1, K=K, N=N, scales=t(S), zeros=t(Z), group_size=gs,
                         flags=SG_MM_C_ACCUMULATE)
    _lib.check(_lib.load().sg_matmul_int4_grouped(ctypes.byref(p), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert torch.equal(got, want)
