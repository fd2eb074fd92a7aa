"""Host-side mirror of the reference kernel table, over the C ABI.

The reference calls ``matmul_int4_grouped_neon(const MatMulParams&)`` and
``flash_attention_fp16(const FlashAttentionParams&)`` directly
(compiler/kernels/cpu/matmul_neon.h:9,113; flash_attention.h:95).  These
functions take the same parameters -- as torch CUDA tensors, which supply
device memory and the current stream -- fill the C structs of
``include/sg_kernels.h`` and call the native library.  Nothing here computes
on the CPU; a missing library or device raises.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import (SG_DT_BF16, SG_DT_DEFAULT, SG_DT_F16, SG_DT_F32, SG_DT_I8, SgFlashAttentionParams,
                   SgMatMulParams, check)

_TORCH_DT = {
    torch.float32: SG_DT_F32,
    torch.float16: SG_DT_F16,
    torch.bfloat16: SG_DT_BF16,
    torch.int8: SG_DT_I8,
}


def dtype_code(t: torch.dtype) -> int:
    return _TORCH_DT[t]


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("tensor must live on a CUDA device")
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def matmul_params(A, B, C, *, M: int, K: int, N: int, scales=None, zeros=None, bias=None,
                  group_size: int = 0, scale_A: float = 1.0, lda: int = 0, ldc: int = 0,
                  workspace: torch.Tensor | None = None, flags: int = 0, norm_weight=None,
                  norm_eps: float = 1e-5) -> SgMatMulParams:
    p = SgMatMulParams()
    p.flags = flags
    p.norm_weight = _ptr(norm_weight)
    p.norm_eps = norm_eps
    p.A = _ptr(A)
    p.B = _ptr(B)
    p.bias = _ptr(bias)
    p.C = _ptr(C)
    p.M, p.K, p.N = M, K, N
    p.lda, p.ldb, p.ldc = lda, 0, ldc
    p.scale_A = scale_A
    p.scales_B = _ptr(scales)
    p.zeros_B = _ptr(zeros)
    p.group_size = group_size
    p.a_dtype = dtype_code(A.dtype) if A is not None else SG_DT_DEFAULT
    p.c_dtype = dtype_code(C.dtype)
    if workspace is not None:
        p.workspace = _ptr(workspace)
        p.workspace_bytes = workspace.numel() * workspace.element_size()
    return p


def matmul_int4_grouped(A: torch.Tensor, B: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor | None,
                        K: int, N: int, group_size: int, *, out_dtype=torch.float16, bias=None,
                        scale_A: float = 1.0, C: torch.Tensor | None = None, stream=None,
                        workspace=None, flags: int = 0) -> torch.Tensor:
    """C[M, N] = A[M, K] @ dequant(B) -- the reference INT4 layout (matmul_neon.h:113-143)."""
    M = A.shape[0] if A.dim() == 2 else 1
    if C is None:
        C = torch.empty((M, N), dtype=out_dtype, device=A.device)
    p = matmul_params(A, B, C, M=M, K=K, N=N, scales=scales, zeros=zeros, bias=bias,
                      group_size=group_size, scale_A=scale_A, workspace=workspace, flags=flags)
    check(_lib.load().sg_matmul_int4_grouped(ctypes.byref(p), _stream(stream)))
    return C


def matmul_int4_grouped_workspace_size(A, B, scales, zeros, K, N, group_size, out_dtype=torch.float16) -> int:
    M = A.shape[0] if A.dim() == 2 else 1
    C = torch.empty((M, N), dtype=out_dtype, device=A.device)
    p = matmul_params(A, B, C, M=M, K=K, N=N, scales=scales, zeros=zeros, group_size=group_size)
    return int(_lib.load().sg_matmul_int4_grouped_workspace_size(ctypes.byref(p)))


def swiglu_rows(gate_up: torch.Tensor, ffn: int, stream=None) -> torch.Tensor:
    """[rows, 2 ffn] gate | up -> [rows, ffn] silu(gate) * up, each product rounded
    as the decoder writes it (ops_swiglu)."""
    rows = gate_up.shape[0]
    y = torch.empty((rows, ffn), dtype=gate_up.dtype, device=gate_up.device)
    check(_lib.load().sg_swiglu_rows(_ptr(gate_up), _ptr(y), rows, ffn, dtype_code(gate_up.dtype), _stream(stream)))
    return y


def set_tuning(key: str, value: int) -> None:
    check(_lib.load().sg_set_tuning(key.encode(), int(value)))


def flash_attention(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, *, causal: bool = True, scale: float = 0.0,
                    q_pos0: int = 0, decode: bool = False, O: torch.Tensor | None = None, stream=None,
                    kv_len: int | None = None, workspace=None, q_pos_device: torch.Tensor | None = None
                    ) -> torch.Tensor:
    """Q [B,H,Sq,D], K/V [B,Hkv,Smax,D] (only the first kv_len rows are used) --
    flash_attention_fp16 (flash_attention.h:95-144) on the GPU.  With q_pos_device
    (an int32 device scalar) the position of query 0 is read on the device and the
    keys used are min(kv_len, position + Sq), as a captured decode step does."""
    from ._lib import SgFlashAttentionParams
    Bn, H, Sq, D = Q.shape
    Hkv, Smax = K.shape[1], K.shape[2]
    if O is None:
        O = torch.empty_like(Q)
    p = SgFlashAttentionParams()
    p.Q, p.K, p.V, p.O = _ptr(Q), _ptr(K), _ptr(V), _ptr(O)
    p.B, p.S, p.num_heads, p.num_kv_heads, p.head_dim = Bn, Sq, H, Hkv, D
    p.scale = scale
    p.causal = int(causal)
    p.io_dtype = dtype_code(Q.dtype)
    p.S_kv = kv_len if kv_len is not None else Smax
    p.q_pos0 = q_pos0
    p.kv_head_stride = K.stride(1)
    p.kv_batch_stride = K.stride(0)
    if q_pos_device is not None:
        p.q_pos_device = _ptr(q_pos_device)
    if workspace is not None:
        p.workspace = _ptr(workspace)
        p.workspace_bytes = workspace.numel() * workspace.element_size()
    fn = _lib.load().sg_flash_decode if decode else _lib.load().sg_flash_attention
    check(fn(ctypes.byref(p), _stream(stream)))
    return O


# ----------------------------------------------------------------------------- block ops
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5, residual: torch.Tensor | None = None,
            out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """rmsnorm_fp16_neon (matmul_neon.h:154-190) per row of x [rows, n]; with a
    residual: residual += x (rounded to the I/O type) and that is normalised."""
    n = x.shape[-1]
    rows = x.numel() // n if n else 0
    y = torch.empty_like(x) if out is None else out
    check(_lib.load().sg_rmsnorm(_ptr(x), _ptr(residual), _ptr(w), _ptr(y), rows, n, eps, dtype_code(x.dtype),
                                 _stream(stream)))
    return y


def silu(x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    y = torch.empty_like(x) if out is None else out
    check(_lib.load().sg_silu(_ptr(x), _ptr(y), x.numel(), dtype_code(x.dtype), _stream(stream)))
    return y


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    y = torch.empty_like(gate) if out is None else out
    check(_lib.load().sg_silu_mul(_ptr(gate), _ptr(up), _ptr(y), gate.numel(), dtype_code(gate.dtype),
                                  _stream(stream)))
    return y


def softmax(x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    n = x.shape[-1]
    y = torch.empty_like(x) if out is None else out
    check(_lib.load().sg_softmax(_ptr(x), _ptr(y), x.numel() // n, n, dtype_code(x.dtype), _stream(stream)))
    return y


def rope(x: torch.Tensor, pos0: int = 0, positions: torch.Tensor | None = None, base: float = 10000.0,
         stream=None) -> torch.Tensor:
    """In place on x [tokens, heads, head_dim] (rope_apply_neon, matmul_neon.h:262-275)."""
    t, h, d = x.shape
    check(_lib.load().sg_rope(_ptr(x), t, h, d, _ptr(positions), pos0, base, dtype_code(x.dtype), _stream(stream)))
    return x


def embedding(table: torch.Tensor, ids: torch.Tensor, stream=None) -> torch.Tensor:
    vocab, hidden = table.shape
    out = torch.empty((ids.numel(), hidden), dtype=table.dtype, device=table.device)
    check(_lib.load().sg_embedding(_ptr(table), _ptr(ids), _ptr(out), ids.numel(), hidden, vocab,
                                   dtype_code(table.dtype), _stream(stream)))
    return out


def argmax(logits: torch.Tensor, stream=None) -> torch.Tensor:
    n = logits.shape[-1]
    rows = logits.numel() // n
    out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    check(_lib.load().sg_argmax(_ptr(logits), rows, n, _ptr(out), _stream(stream)))
    return out
