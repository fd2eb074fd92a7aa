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
