"""ORACLE -- test infrastructure, not product code.

ctypes/numpy front-end for two CPU libraries built by ``oracle/Makefile``:

* ``_build/libsg_oracle.so`` -- our C++ restatement of the reference's
  quantized-block arithmetic (``oracle/sg_oracle.cpp``; each function cites
  the reference file:line it restates);
* ``_ref/libsg_ref.so`` -- the reference's own CPU kernels
  (``compiler/kernels/cpu/matmul_neon.h``, ``flash_attention.h``) compiled
  unmodified from its headers, with the NEON branches enabled through
  ``oracle/neon_shim`` (``ref_neon_*``) and with the scalar branches
  (``ref_scalar_*``).  Present only where it was built.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this package, and only as the checker / CPU baseline.  The product
package ``silicongraph_b200`` never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(_HERE, "_build", "libsg_oracle.so")
REF_SO = os.path.join(_HERE, "_ref", "libsg_ref.so")

# dtype codes shared with include/sg_kernels.h (SgDType)
DT_DEFAULT, DT_F32, DT_F16, DT_BF16, DT_I8 = 0, 1, 2, 3, 4

_P = ctypes.c_void_p
_I = ctypes.c_int32
_F = ctypes.c_float

_lib = None
_ref = None


def build(ref: bool | None = None, refdir: str | None = None) -> None:
    """Compile the restatement, and the reference's own kernels when a
    reference checkout is named (``refdir``, else the ``SG_REFERENCE_DIR``
    environment variable) and present, or when ``ref`` is True (then a missing
    checkout is an error)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    refdir = refdir or os.environ.get("SG_REFERENCE_DIR")
    present = bool(refdir) and os.path.isdir(os.path.join(refdir, "compiler", "kernels", "cpu"))
    if ref and not present:
        raise FileNotFoundError("the reference checkout is needed: pass refdir or set SG_REFERENCE_DIR")
    if present and ref is not False:
        subprocess.run(["make", "-s", "-C", _HERE, "ref", f"REF={refdir}"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build(ref=False)
        L = ctypes.CDLL(ORACLE_SO)
        L.orc_matmul_int4_grouped.argtypes = [_P, _I, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F]
        L.orc_dequant_int4_grouped.argtypes = [_P, _P, _P, _P, _I, _I, _I]
        L.orc_quantize_int4_grouped.argtypes = [_P, _I, _I, _I, _I, _P, _P, _P]
        L.orc_gemm_int8_channel.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _F]
        L.orc_gemm_w8_channel.argtypes = [_P, _I, _P, _P, _P, _I, _I, _I, _I, _I, _I]
        L.orc_matmul_f16w.argtypes = [_P, _I, _P, _P, _P, _I, _I, _I, _I, _I, _I]
        L.orc_flash_attention.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _I, _I]
        L.orc_rmsnorm_f16.argtypes = [_P, _P, _P, _I, _F]
        L.orc_silu_f16.argtypes = [_P, _P, _I]
        L.orc_softmax_f16.argtypes = [_P, _P, _I]
        L.orc_rope_f16.argtypes = [_P, _I, _I, _F]
        L.orc_rmsnorm_f32.argtypes = [_P, _P, _P, _I, _F]
        L.orc_silu_f32.argtypes = [_P, _P, _I]
        L.orc_rope_f32.argtypes = [_P, _I, _I, _F]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> ctypes.CDLL:
    """The reference's own kernels (raises if they were not built)."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(f"{REF_SO} not built (make -C oracle ref)")
        R = ctypes.CDLL(REF_SO)
        for pre in ("sgref_neon_", "sgref_scalar_"):
            getattr(R, pre + "matmul_int4_grouped").argtypes = [_P, _P, _P, _P, _P, _I, _I, _I]
            getattr(R, pre + "matmul_fp16_m1").argtypes = [_P, _P, _P, _P, _I, _I]
            getattr(R, pre + "rmsnorm").argtypes = [_P, _P, _P, _I, _F]
            getattr(R, pre + "silu").argtypes = [_P, _P, _I]
            getattr(R, pre + "softmax").argtypes = [_P, _P, _I]
            getattr(R, pre + "rope").argtypes = [_P, _I, _I, _F]
            getattr(R, pre + "flash_attn_head").argtypes = [_P, _P, _P, _P, _I, _I, _F, _I, _I]
            getattr(R, pre + "flash_attention_fp16").argtypes = [_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _I]
        # the OpenCL-C gemm_int8_m1 kernel run as host C (ref_opencl.c)
        R.sgref_cl_gemm_int8_m1.argtypes = [_P, _P, _P, _P, _I, _I, _F]
        _ref = R
    return _ref


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


_ACT_DT = {np.dtype(np.float32): DT_F32, np.dtype(np.float16): DT_F16, np.dtype(np.int8): DT_I8}


def _act_code(a: np.ndarray, bf16: bool) -> int:
    if bf16:
        assert a.dtype == np.uint16
        return DT_BF16
    return _ACT_DT[a.dtype]


def _out_array(shape, c_dt: int) -> np.ndarray:
    if c_dt == DT_F32:
        return np.zeros(shape, np.float32)
    if c_dt == DT_BF16:
        return np.zeros(shape, np.uint16)
    return np.zeros(shape, np.float16)


# ----------------------------------------------------------------------------- INT4
def quantize_int4_grouped(W_kn: np.ndarray, group_size: int, symmetric: bool = False):
    """Pack a [K, N] fp32 weight into the reference INT4 layout.

    Returns (B u8 [ceil(K/2), N], scales f16 [ceil(K/gs), N], zeros i8 [ceil(K/gs), N] or None)."""
    W = np.ascontiguousarray(W_kn, dtype=np.float32)
    K, N = W.shape
    gs = group_size if group_size > 0 else 128
    G = (K + gs - 1) // gs
    B = np.zeros(((K + 1) // 2, N), np.uint8)
    S = np.zeros((G, N), np.float16)
    Z = None if symmetric else np.zeros((G, N), np.int8)
    lib().orc_quantize_int4_grouped(_p(W), K, N, group_size, int(symmetric), _p(B), _p(S), _p(Z))
    return B, S, Z


def dequant_int4_grouped(B, scales, zeros, K: int, N: int, group_size: int) -> np.ndarray:
    W = np.zeros((K, N), np.float32)
    lib().orc_dequant_int4_grouped(_p(B), _p(scales), _p(zeros), _p(W), K, N, group_size)
    return W


def matmul_int4_grouped(A, B, scales, zeros, K: int, N: int, group_size: int, *, M: int = 1,
                        bias=None, c_dt: int = DT_DEFAULT, scale_A: float = 1.0,
                        a_bf16: bool = False) -> np.ndarray:
    """Restated matmul_int4_grouped_neon; A may be int8 (reference), f32, f16 or bf16 (u16 bits)."""
    A = np.ascontiguousarray(A)
    a_dt = _act_code(A, a_bf16)
    C = _out_array((M, N), c_dt)
    lib().orc_matmul_int4_grouped(_p(A), a_dt, _p(B), _p(scales), _p(zeros), _p(bias), _p(C), c_dt,
                                  M, K, N, K, N, group_size, scale_A)
    return C


# ----------------------------------------------------------------------------- INT8 / fp16
def gemm_int8_channel(A_i8, B_i8, scales_f32, M: int, K: int, N: int, scale_A: float) -> np.ndarray:
    C = np.zeros((M, N), np.float32)
    lib().orc_gemm_int8_channel(_p(np.ascontiguousarray(A_i8)), _p(B_i8), _p(scales_f32), _p(C),
                                M, K, N, K, N, scale_A)
    return C


def gemm_w8_channel(A, B_i8, scales_f32, M: int, K: int, N: int, *, c_dt: int = DT_F32,
                    a_bf16: bool = False) -> np.ndarray:
    A = np.ascontiguousarray(A)
    C = _out_array((M, N), c_dt)
    lib().orc_gemm_w8_channel(_p(A), _act_code(A, a_bf16), _p(B_i8), _p(scales_f32), _p(C), c_dt,
                              M, K, N, K, N)
    return C


def matmul_f16w(A, B_f16, bias, M: int, K: int, N: int, *, c_dt: int = DT_DEFAULT,
                a_bf16: bool = False) -> np.ndarray:
    A = np.ascontiguousarray(A)
    C = _out_array((M, N), c_dt)
    lib().orc_matmul_f16w(_p(A), _act_code(A, a_bf16), _p(B_f16), _p(bias), _p(C), c_dt, M, K, N, K, N)
    return C


# ----------------------------------------------------------------------------- attention
def flash_attention(Q, K, V, *, causal: bool = True, scale: float = 0.0, q_pos0: int = 0,
                    io_dt: int | None = None) -> np.ndarray:
    """Q [B,H,Sq,D], K/V [B,Hkv,Skv,D]; f32 / f16 arrays, or bf16 as uint16 with io_dt=DT_BF16."""
    Q, K, V = (np.ascontiguousarray(t) for t in (Q, K, V))
    if io_dt is None:
        io_dt = DT_F32 if Q.dtype == np.float32 else DT_F16
    Bn, H, Sq, D = Q.shape
    Hkv, Skv = K.shape[1], K.shape[2]
    O = np.zeros_like(Q)
    lib().orc_flash_attention(_p(Q), _p(K), _p(V), _p(O), io_dt, Bn, H, Hkv, Sq, Skv, D, scale,
                              int(causal), q_pos0)
    return O


# ----------------------------------------------------------------------------- block ops
def rmsnorm_f16(x, w, eps=1e-5):
    y = np.zeros_like(x)
    lib().orc_rmsnorm_f16(_p(x), _p(w), _p(y), x.size, eps)
    return y


def silu_f16(x):
    y = np.zeros_like(x)
    lib().orc_silu_f16(_p(x), _p(y), x.size)
    return y


def softmax_f16(x):
    y = np.zeros_like(x)
    lib().orc_softmax_f16(_p(x), _p(y), x.size)
    return y


def rope_f16(x, position: int, base: float = 10000.0):
    y = x.copy()
    lib().orc_rope_f16(_p(y), y.size, position, base)
    return y


def rmsnorm_f32(x, w, eps=1e-5):
    y = np.zeros_like(x)
    lib().orc_rmsnorm_f32(_p(x), _p(w), _p(y), x.size, eps)
    return y


def silu_f32(x):
    y = np.zeros_like(x)
    lib().orc_silu_f32(_p(x), _p(y), x.size)
    return y


def rope_f32(x, position: int, base: float = 10000.0):
    y = x.copy()
    lib().orc_rope_f32(_p(y), y.size, position, base)
    return y


# ----------------------------------------------------------------------------- helpers
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16, returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
