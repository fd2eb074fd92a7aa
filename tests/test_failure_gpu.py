"""Failure detection without a GPU fault, on one GPU.

* A bounded device wait runs out: the peer all-reduce (sg_tp_allreduce_f16)
  is launched as rank 0 of a two-rank group whose regions both live on this
  GPU, and rank 1 never runs, so its flag is never raised.  With the wait
  shortened to 20 ms the kernel gives up, leaves the vector unreduced,
  records the timeout in the device error word, and sg_device_error_check
  reports it; the GPU keeps working.
* sg_session_abort: an aborted session refuses every later call with the
  reason and can still be destroyed."""
import ctypes
import time

import numpy as np
import pytest
import torch

from silicongraph_b200 import armpack

pytestmark = pytest.mark.gpu


def test_peer_allreduce_wait_runs_out_and_is_reported(sg):
    from silicongraph_b200 import _lib
    lib = _lib.load()
    lib.sg_tp_allreduce_region_bytes.restype = ctypes.c_size_t
    lib.sg_tp_allreduce_region_bytes.argtypes = [ctypes.c_int32, ctypes.c_int32]
    lib.sg_tp_allreduce_f16.restype = ctypes.c_int32
    lib.sg_tp_allreduce_f16.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                        ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32, ctypes.c_void_p]
    st = torch.cuda.current_stream().cuda_stream
    assert lib.sg_device_error_check(st) == 0
    max_n, n = 4096, 2048
    rb = lib.sg_tp_allreduce_region_bytes(2, max_n)
    regions = [torch.zeros(rb, dtype=torch.uint8, device="cuda") for _ in range(2)]
    data = torch.randn(n, device="cuda").half()
    before = data.clone()
    arr = (ctypes.c_void_p * 2)(regions[0].data_ptr(), regions[1].data_ptr())
    sg.set_tuning("tp_allreduce.wait_ms", 20)
    try:
        t0 = time.perf_counter()
        _lib.check(lib.sg_tp_allreduce_f16(data.data_ptr(), n, 0, 2, arr, max_n, st))
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        sg.set_tuning("tp_allreduce.wait_ms", 0)  # back to 2 s
    assert elapsed < 1.0, f"the 20 ms wait took {elapsed:.3f} s"
    assert lib.sg_device_error_check(st) == _lib.SG_ERR_RUNTIME
    assert b"timed out" in lib.sg_last_error()
    assert torch.equal(data, before)                 # left unreduced
    assert lib.sg_device_error_check(st) == 0        # read and cleared
    # the GPU still answers: a library kernel against the oracle
    K, N, gs = 256, 512, 32
    rng = np.random.default_rng(0)
    import oracle
    B, S, Z = oracle.quantize_int4_grouped((rng.standard_normal((K, N)) * 0.02).astype(np.float32), gs)
    x = rng.standard_normal((1, K)).astype(np.float32)
    want = oracle.matmul_int4_grouped(x, B, S, Z, K, N, gs, c_dt=oracle.DT_F32)
    t = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    got = sg.matmul_int4_grouped(t(x), t(B), t(S), t(Z), K, N, gs, out_dtype=torch.float32).cpu().numpy()
    assert np.all(np.abs(got - want) <= 2e-3 + 1e-2 * np.abs(want))


def test_aborted_session_refuses_with_the_reason(sg, tmp_path):
    from silicongraph_b200 import sdk
    cfg = armpack.llama_config(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000,
                               rope_theta=500000.0, max_pos=4096)
    t = armpack.cuda_tensors(cfg, armpack.random_llama_weights(cfg, seed=1), group_size=32)
    path = armpack.write_package(str(tmp_path / "m.armpack"), cfg, t, max_context=256, max_prefill_chunk=64)
    with sdk.Package(path) as pkg:
        with pkg.select().session() as s:
            s.prefill(np.arange(10, dtype=np.int32))
            s.decode()
            s.abort("the operator stopped it")
            with pytest.raises(sdk.ArmError) as e:
                s.decode()
            assert e.value.status == -5 and "the operator stopped it" in str(e.value)
            with pytest.raises(sdk.ArmError):
                s.prefill(np.arange(4, dtype=np.int32))
