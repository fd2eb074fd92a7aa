"""C-ABI checks that need no GPU: the native library loads, exports every
function include/*.h declares, and fails loudly (no CPU fallback) when no
CUDA device is present."""
import ctypes
import glob
import os
import re

import pytest

from conftest import ROOT

HEADERS = sorted(glob.glob(os.path.join(ROOT, "include", "*.h")))


def declared_functions():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        for m in re.finditer(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(([^;{}]*)\)\s*;", src):
            name = m.group(1)
            if name in ("if", "while", "for", "return", "sizeof"):
                continue
            # skip typedef'd function pointer parameters such as (*output_cb)
            if name.startswith("(") or name in ("output_cb",):
                continue
            names.add(name)
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from silicongraph_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        from silicongraph_b200 import build
        build.build()
    return _lib.load()


def test_headers_exist():
    assert any(h.endswith("sg_kernels.h") for h in HEADERS)


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_library_is_sm100a_only():
    from silicongraph_b200 import build
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.ARCH)


def test_version(lib):
    assert lib.sg_version() == (0 << 16) | (1 << 8) | 0


def test_null_params_rejected(lib):
    from silicongraph_b200._lib import SG_ERR_INVALID
    assert lib.sg_matmul_int4_grouped(None, None) == SG_ERR_INVALID
    assert b"NULL" in lib.sg_last_error()


def test_unknown_tuning_key(lib):
    from silicongraph_b200._lib import SG_ERR_NOT_FOUND
    assert lib.sg_set_tuning(b"no.such.key", 1) == SG_ERR_NOT_FOUND


def test_no_cpu_fallback_without_device(lib):
    """Without a CUDA device a compute call must fail with SG_ERR_RUNTIME."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from silicongraph_b200._lib import SG_ERR_RUNTIME, SgMatMulParams
    assert lib.sg_device_count() == 0
    buf = (ctypes.c_uint8 * 4096)()
    p = SgMatMulParams()
    p.A = p.B = p.C = p.scales_B = ctypes.addressof(buf)
    p.M, p.K, p.N, p.group_size = 1, 32, 16, 32
    assert lib.sg_matmul_int4_grouped(ctypes.byref(p), None) == SG_ERR_RUNTIME
    assert b"no CUDA device" in lib.sg_last_error()


def test_flag_values_match_header():
    """The Python binding's SG_MM_* flag values are the header's."""
    from silicongraph_b200 import _lib
    src = open(os.path.join(ROOT, "include", "sg_kernels.h")).read()
    for name in ("SG_MM_STATIC_WEIGHTS", "SG_MM_A_SWIGLU", "SG_MM_A_RMSNORM", "SG_MM_C_ACCUMULATE"):
        m = re.search(rf"#define {name} (\d+)u", src)
        assert m, name
        assert int(m.group(1)) == getattr(_lib, name)


@pytest.mark.parametrize("key,value", [
    ("w4_rows.enable", 1), ("w4_rows.stages", 0), ("w4_rows.producer_sleep", 1), ("w4_rows.max_tiles", 1 << 30),
    ("w4_gemv_mma.strips", 0), ("w4_gemv_mma.variant", 0), ("attn.decode_kernel", 4), ("sdk.fuse_swiglu", 1),
    ("w4_rows.two_pass_rows", 32), ("tp_allreduce.wait_ms", 0), ("sdk.fuse_norm", 1), ("sdk.fuse_rope", 1),
    ("sdk.decode_step_kernel", 0), ("w8_gemv_mma.enable", 1), ("attn_tc.pair", 1),
    ("gemm_tc.split", 1), ("gemm_tc.pair", 0), ("gemm_tc.bt", 0), ("gemm_tc.par", 2),
])
def test_tuning_keys_known(lib, key, value):
    """Every tuning knob the kernels and the SDK read is reachable through
    sg_set_tuning (host-only; the values set are the defaults)."""
    from silicongraph_b200._lib import SG_OK
    assert lib.sg_set_tuning(key.encode(), value) == SG_OK


def test_documented_tuning_keys_accepted():
    """Every key that include/sg_kernels.h documents for sg_set_tuning is one
    the library accepts.  Set in a child process, so the values do not leak
    into the other tests of this session."""
    import subprocess
    import sys
    src = open(os.path.join(ROOT, "include", "sg_kernels.h")).read()
    block = src[src.index("Override a launch heuristic"):src.index("int32_t sg_set_tuning")]
    keys = sorted(set(re.findall(r'^ \*\s+"([a-z0-9_.]+)"', block, re.M) + re.findall(r', "([a-z0-9_.]+)"', block)))
    assert len(keys) >= 15, keys
    code = ("import sys; from silicongraph_b200 import _lib; lib = _lib.load(); "
            "bad = [k for k in sys.argv[1:] if lib.sg_set_tuning(k.encode(), 0) != 0]; "
            "print(bad); sys.exit(1 if bad else 0)")
    r = subprocess.run([sys.executable, "-c", code, *keys], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr


def test_swiglu_flag_argument_checks(lib):
    """SG_MM_A_SWIGLU is refused for int8 / fp32 activations and for an lda
    shorter than the gate | up row, before any device work."""
    from silicongraph_b200._lib import SG_DT_F32, SG_ERR_INVALID, SG_MM_A_SWIGLU, SgMatMulParams
    buf = (ctypes.c_uint8 * 4096)()
    p = SgMatMulParams()
    p.A = p.B = p.C = p.scales_B = ctypes.addressof(buf)
    p.M, p.K, p.N, p.group_size = 1, 64, 16, 32
    p.flags = SG_MM_A_SWIGLU
    p.a_dtype = SG_DT_F32
    assert lib.sg_matmul_int4_grouped(ctypes.byref(p), None) == SG_ERR_INVALID
    assert b"SG_MM_A_SWIGLU" in lib.sg_last_error()
    p.a_dtype = 2  # fp16
    p.lda = 64     # < 2K
    assert lib.sg_matmul_int4_grouped(ctypes.byref(p), None) == SG_ERR_INVALID
    assert b"lda" in lib.sg_last_error()


def test_fused_norm_flag_argument_checks(lib):
    """SG_MM_A_RMSNORM needs a 16-bit A, a norm weight and K % 8 == 0 (checked
    before any device work); SG_MM_C_ACCUMULATE needs a 16-bit C."""
    from silicongraph_b200._lib import (SG_DT_F32, SG_ERR_INVALID, SG_MM_A_RMSNORM, SG_MM_C_ACCUMULATE,
                                        SgMatMulParams)
    buf = (ctypes.c_uint8 * 8192)()
    base = (ctypes.addressof(buf) + 255) // 256 * 256
    p = SgMatMulParams()
    p.A = p.B = p.C = p.scales_B = base
    p.M, p.K, p.N, p.group_size = 1, 64, 16, 32
    p.a_dtype, p.c_dtype = 2, 2
    p.flags = SG_MM_A_RMSNORM
    assert lib.sg_matmul_int4_grouped(ctypes.byref(p), None) == SG_ERR_INVALID  # no norm weight
    assert b"SG_MM_A_RMSNORM" in lib.sg_last_error()
    p.norm_weight = base
    p.K = 60                                                                   # not a multiple of 8
    assert lib.sg_matmul_int4_grouped(ctypes.byref(p), None) == SG_ERR_INVALID
    p.K, p.flags, p.c_dtype = 64, SG_MM_C_ACCUMULATE, SG_DT_F32
    assert lib.sg_matmul_int4_grouped(ctypes.byref(p), None) == SG_ERR_INVALID
    assert b"SG_MM_C_ACCUMULATE" in lib.sg_last_error()
