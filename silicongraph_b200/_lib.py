"""ctypes binding of the native library (``lib/libsg_b200.so``).

The structures mirror ``include/sg_kernels.h`` field for field.  There is no
fallback: if the library is missing or no CUDA device is usable, calls raise.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "lib", "libsg_b200.so")

SG_OK = 0
SG_ERR_NOT_FOUND = -1
SG_ERR_INVALID = -2
SG_ERR_OOM = -3
SG_ERR_UNSUPPORTED = -4
SG_ERR_RUNTIME = -5

SG_DT_DEFAULT, SG_DT_F32, SG_DT_F16, SG_DT_BF16, SG_DT_I8 = 0, 1, 2, 3, 4


class SgError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"status {status}: {msg}")
        self.status = status


class SgMatMulParams(ctypes.Structure):
    """Mirror of armcc::kernels::cpu::MatMulParams (matmul_neon.h:32-43) plus extensions."""
    _fields_ = [
        ("A", ctypes.c_void_p),
        ("B", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("C", ctypes.c_void_p),
        ("M", ctypes.c_int32),
        ("K", ctypes.c_int32),
        ("N", ctypes.c_int32),
        ("lda", ctypes.c_int32),
        ("ldb", ctypes.c_int32),
        ("ldc", ctypes.c_int32),
        ("scale_A", ctypes.c_float),
        ("scales_B", ctypes.c_void_p),
        ("zeros_B", ctypes.c_void_p),
        ("group_size", ctypes.c_int32),
        ("a_dtype", ctypes.c_int32),
        ("c_dtype", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("flags", ctypes.c_uint32),
        ("norm_weight", ctypes.c_void_p),
        ("norm_eps", ctypes.c_float),
    ]


SG_MM_STATIC_WEIGHTS = 1
SG_MM_A_SWIGLU = 2
SG_MM_A_RMSNORM = 4
SG_MM_C_ACCUMULATE = 8


class SgKvPages(ctypes.Structure):
    """Paged KV cache descriptor (include/sg_kernels.h SgKvPages)."""
    _fields_ = [
        ("table", ctypes.c_void_p),
        ("page_size", ctypes.c_int32),
        ("num_pages", ctypes.c_int32),
        ("page_stride", ctypes.c_int64),
        ("table_batch_stride", ctypes.c_int64),
        ("table_page_stride", ctypes.c_int64),
    ]


class SgFlashAttentionParams(ctypes.Structure):
    """Mirror of armcc::kernels::cpu::FlashAttentionParams (flash_attention.h:25-42) plus extensions."""
    _fields_ = [
        ("Q", ctypes.c_void_p),
        ("K", ctypes.c_void_p),
        ("V", ctypes.c_void_p),
        ("O", ctypes.c_void_p),
        ("mask", ctypes.c_void_p),
        ("B", ctypes.c_int32),
        ("S", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("causal", ctypes.c_int32),
        ("streaming", ctypes.c_int32),
        ("chunk_size", ctypes.c_int32),
        ("io_dtype", ctypes.c_int32),
        ("S_kv", ctypes.c_int32),
        ("q_pos0", ctypes.c_int32),
        ("kv_batch_stride", ctypes.c_int64),
        ("kv_head_stride", ctypes.c_int64),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("q_pos_device", ctypes.c_void_p),
        ("kv_pages", ctypes.POINTER(SgKvPages)),
    ]


_lib = None

# name -> (restype, argtypes)
_P = ctypes.c_void_p
_SIGS = {
    "sg_last_error": (ctypes.c_char_p, []),
    "sg_version": (ctypes.c_int32, []),
    "sg_device_count": (ctypes.c_int32, []),
    "sg_set_tuning": (ctypes.c_int32, [ctypes.c_char_p, ctypes.c_int32]),
    "sg_device_error_check": (ctypes.c_int32, [_P]),
    "sg_matmul_int4_grouped": (ctypes.c_int32, [ctypes.POINTER(SgMatMulParams), _P]),
    "sg_matmul_int4_grouped_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(SgMatMulParams)]),
    "sg_matmul_int4_grouped_noalloc": (ctypes.c_int32, [ctypes.POINTER(SgMatMulParams), _P]),
    "sg_matmul_int8_channel": (ctypes.c_int32, [ctypes.POINTER(SgMatMulParams), _P]),
    "sg_matmul_int8_channel_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(SgMatMulParams)]),
    "sg_matmul_fp16": (ctypes.c_int32, [ctypes.POINTER(SgMatMulParams), _P]),
    "sg_matmul_fp16_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(SgMatMulParams)]),
    "sg_flash_attention": (ctypes.c_int32, [ctypes.POINTER(SgFlashAttentionParams), _P]),
    "sg_flash_attention_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(SgFlashAttentionParams)]),
    "sg_flash_decode": (ctypes.c_int32, [ctypes.POINTER(SgFlashAttentionParams), _P]),
    "sg_flash_decode_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(SgFlashAttentionParams)]),
    "sg_quantize_int4_grouped": (ctypes.c_int32, [_P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.c_int32, _P, _P, _P, _P]),
    "sg_dequantize_int4_grouped": (ctypes.c_int32, [_P, _P, _P, ctypes.c_int32, ctypes.c_int32,
                                                    ctypes.c_int32, _P, _P]),
    "sg_rmsnorm": (ctypes.c_int32, [_P, _P, _P, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_float,
                                    ctypes.c_int32, _P]),
    "sg_silu": (ctypes.c_int32, [_P, _P, ctypes.c_int64, ctypes.c_int32, _P]),
    "sg_silu_mul": (ctypes.c_int32, [_P, _P, _P, ctypes.c_int64, ctypes.c_int32, _P]),
    "sg_swiglu_rows": (ctypes.c_int32, [_P, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _P]),
    "sg_softmax": (ctypes.c_int32, [_P, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _P]),
    "sg_rope": (ctypes.c_int32, [_P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _P, ctypes.c_int32,
                                 ctypes.c_float, ctypes.c_int32, _P]),
    "sg_embedding": (ctypes.c_int32, [_P, _P, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                      ctypes.c_int32, _P]),
    "sg_argmax": (ctypes.c_int32, [_P, ctypes.c_int32, ctypes.c_int32, _P, _P]),
    "sg_qkv_rope_append_batched": (ctypes.c_int32, [_P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                                    ctypes.c_int32, ctypes.c_int32, _P, ctypes.c_int32,
                                                    ctypes.c_float, _P, _P, _P, ctypes.c_int64, ctypes.c_int64,
                                                    ctypes.c_int32, _P]),
    "sg_qkv_rope_append_paged": (ctypes.c_int32, [_P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                                  ctypes.c_int32, ctypes.c_int32, _P, ctypes.c_int32,
                                                  ctypes.c_float, _P, _P, _P, ctypes.POINTER(SgKvPages),
                                                  ctypes.c_int32, _P]),
}


def load() -> ctypes.CDLL:
    """Load the native library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"native library missing: {LIB_PATH} "
                               "(run `python -m silicongraph_b200.build`); there is no CPU fallback")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return (load().sg_last_error() or b"").decode(errors="replace")


def check(status: int) -> None:
    if status != SG_OK:
        raise SgError(status, last_error())
