"""The allocation-free INT4 GEMV entry point, sg_matmul_int4_grouped_noalloc.

It serves callers that may not allocate device memory once running (a runtime
that sizes all memory when a session is admitted, or a host framework whose
pool owns the device).  Its scratch is a fixed 2 MiB array inside the library,
so these tests check, through the C ABI, that it gives the same results as
sg_matmul_int4_grouped on two calls in a row (the array keeps the previous
call's contents) and that a problem needing more scratch is refused.

Kept in a file of its own that pytest collects last; it must pass both alone
in a fresh process and after the other tests."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-3


def _problem(oracle_mod, K, N, gs, seed):
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    B, S, Z = oracle_mod.quantize_int4_grouped(W, gs)
    dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    return dev(B), dev(S), dev(Z)


def _call(lib, fn, x, B, S, Z, K, N, gs, M=1):
    from silicongraph_b200 import kernels
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    p = kernels.matmul_params(x, B, y, M=M, K=K, N=N, scales=S, zeros=Z, group_size=gs)
    st = getattr(lib, fn)(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
    return st, y


@pytest.mark.parametrize("K,N,gs,M", [(4096, 14336, 32, 1), (2048, 3072, 64, 1), (1024, 2048, 32, 3)])
def test_noalloc_matches_allocating_entry_point_twice(sg, oracle_mod, K, N, gs, M):
    from silicongraph_b200 import _lib
    lib = _lib.load()
    B, S, Z = _problem(oracle_mod, K, N, gs, seed=K + N)
    for call in range(2):  # second call sees the first call's leftover scratch
        x = torch.from_numpy(np.random.default_rng(call).standard_normal((M, K)).astype(np.float32)).cuda()
        st_ref, want = _call(lib, "sg_matmul_int4_grouped", x, B, S, Z, K, N, gs, M)
        assert st_ref == 0, _lib.last_error()
        st, got = _call(lib, "sg_matmul_int4_grouped_noalloc", x, B, S, Z, K, N, gs, M)
        assert st == 0, _lib.last_error()
        # a timed-out wait inside the allocation-free kernels is reported here
        assert lib.sg_device_error_check(torch.cuda.current_stream().cuda_stream) == 0, _lib.last_error()
        torch.cuda.synchronize()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        err = np.abs(g - w)
        assert np.all(err <= ATOL + RTOL * np.abs(w)), f"call {call}: max err {err.max():.3e}"


def test_noalloc_rejects_scratch_beyond_its_maximum(sg, oracle_mod):
    """A prefill-sized call with fp32 activations (512 x 4096: a 4 MiB fp16
    copy for the tensor-core GEMM) needs more than the 2 MiB array: refused
    with a message, output untouched."""
    from silicongraph_b200 import _lib
    lib = _lib.load()
    M, K, N, gs = 512, 4096, 512, 32
    B, S, Z = _problem(oracle_mod, K, N, gs, seed=5)
    x = torch.randn(M, K, device="cuda")
    from silicongraph_b200 import kernels
    y = torch.full((M, N), 7.0, dtype=torch.float32, device="cuda")
    p = kernels.matmul_params(x, B, y, M=M, K=K, N=N, scales=S, zeros=Z, group_size=gs)
    need = lib.sg_matmul_int4_grouped_workspace_size(ctypes.byref(p))
    assert need > (2 << 20)
    st = lib.sg_matmul_int4_grouped_noalloc(ctypes.byref(p), torch.cuda.current_stream().cuda_stream)
    assert st == _lib.SG_ERR_INVALID
    assert b"maximum" in lib.sg_last_error()
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())
