"""One process driving two GPUs in turn: the per-device state of the linear
kernels (shared-memory opt-ins, occupancy caches, error words, scratch) must
serve a second device as it serves the first.  Device 0 runs first, then device
1, each against the oracle at the elementwise bar |got - want| <= 2e-3 +
1e-2 |want|.  Skipped with fewer than two GPUs."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-3


def close(got, want):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    err = np.abs(got - want)
    bad = err > ATOL + RTOL * np.abs(want)
    assert not bad.any(), f"{bad.sum()} / {bad.size} outside tolerance; max err {err.max():.3e}"


def _run_three(sg, oracle, dev):
    from silicongraph_b200 import _lib
    d = f"cuda:{dev}"

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(d)

    rng = np.random.default_rng(dev + 11)
    K, N, gs = 2048, 3072, 32
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    B, S, Z = oracle.quantize_int4_grouped(W, gs, False)

    # Few-row INT4 GEMM, 8 fp16 rows.
    x8 = rng.standard_normal((8, K)).astype(np.float16)
    want8 = oracle.matmul_int4_grouped(x8, B, S, Z, K, N, gs, M=8, c_dt=oracle.DT_F32)
    C8 = sg.matmul_int4_grouped(t(x8), t(B), t(S), t(Z), K, N, gs, out_dtype=torch.float32)

    # One-row INT4 GEMV, fp32 activations.
    x1 = rng.standard_normal((1, K)).astype(np.float32)
    want1 = oracle.matmul_int4_grouped(x1, B, S, Z, K, N, gs, c_dt=oracle.DT_F32)
    C1 = sg.matmul_int4_grouped(t(x1), t(B), t(S), t(Z), K, N, gs, out_dtype=torch.float32)

    # INT8 per-channel GEMV, fp32 activations.
    K8, N8 = 4096, 4096
    xa = rng.standard_normal((1, K8)).astype(np.float32)
    W8 = rng.integers(-128, 128, (K8, N8), dtype=np.int8)
    s8 = (rng.random(N8) * 1e-3).astype(np.float32)
    want_i8 = oracle.gemm_w8_channel(xa, W8, s8, 1, K8, N8)
    Ci8 = torch.zeros((1, N8), dtype=torch.float32, device=d)
    p = sg.matmul_params(t(xa), t(W8), Ci8, M=1, K=K8, N=N8, scales=t(s8))
    _lib.check(_lib.load().sg_matmul_int8_channel(ctypes.byref(p), torch.cuda.current_stream(dev).cuda_stream))

    torch.cuda.synchronize(dev)
    close(C8.cpu().numpy(), want8)
    close(C1.cpu().numpy(), want1)
    close(Ci8.cpu().numpy(), want_i8)
    assert _lib.load().sg_device_error_check(torch.cuda.current_stream(dev).cuda_stream) == 0


def test_linear_kernels_on_two_devices_in_one_process(sg, oracle_mod):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    for dev in (0, 1):
        with torch.cuda.device(dev):
            _run_three(sg, oracle_mod, dev)
