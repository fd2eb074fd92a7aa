"""Attention on the GPU through the C ABI against the reference goldens
(flash_attention_fp16 / flash_attn_head compiled from the reference) and the
oracle restatement.  Tolerance |got - want| <= 2e-3 + 1e-2 |want|."""
import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-2, 2e-3


def close(got, want, rtol=RTOL, atol=ATOL):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    err = np.abs(got - want)
    bad = err > atol + rtol * np.abs(want)
    assert not bad.any(), f"{bad.sum()} / {bad.size} outside tolerance; max err {err.max():.3e}"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("name", ["attn_fp16_gqa_causal.npz", "attn_fp16_mha_noncausal.npz",
                                  "attn_fp16_gqa7_causal.npz"])
@pytest.mark.parametrize("decode", [False, True])
def test_attention_matches_reference_golden(sg, name, decode):
    g = golden(name)
    O = sg.flash_attention(dev(g["Q"]), dev(g["K"]), dev(g["V"]), causal=bool(g["causal"]), decode=decode)
    close(O.float().cpu().numpy(), g["O"].astype(np.float32))


def test_attention_f32_matches_reference_head_kernel(sg):
    g = golden("attn_f32_head.npz")
    O = sg.flash_attention(dev(g["Q"]), dev(g["K"]), dev(g["V"]), causal=True, scale=float(g["scale"]))
    close(O.cpu().numpy(), g["O"])


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("B,H,Hkv,S,D,causal", [
    (1, 32, 32, 512, 64, True),     # the flash-attention benchmark shape (config 1)
    (2, 8, 2, 77, 64, True),
    (1, 28, 4, 96, 128, True),      # Qwen-7B head layout
    (1, 4, 1, 33, 32, False),
    (1, 2, 2, 5, 16, True),
])
def test_attention_vs_oracle(sg, oracle_mod, dtype, B, H, Hkv, S, D, causal):
    rng = np.random.default_rng(S + D)
    q = rng.standard_normal((B, H, S, D)).astype(np.float32)
    k = rng.standard_normal((B, Hkv, S, D)).astype(np.float32)
    v = rng.standard_normal((B, Hkv, S, D)).astype(np.float32)
    if dtype == "f32":
        want = oracle_mod.flash_attention(q, k, v, causal=causal)
        got = sg.flash_attention(dev(q), dev(k), dev(v), causal=causal).cpu().numpy()
    elif dtype == "f16":
        # the oracle in fp32 on the same fp16 input values: one rounding of the output, not two
        q, k, v = (a.astype(np.float16) for a in (q, k, v))
        want = oracle_mod.flash_attention(*(a.astype(np.float32) for a in (q, k, v)), causal=causal)
        got = sg.flash_attention(dev(q), dev(k), dev(v), causal=causal).float().cpu().numpy()
    else:
        qb, kb, vb = (oracle_mod.bf16_bits_to_f32(oracle_mod.f32_to_bf16_bits(a)) for a in (q, k, v))
        want = oracle_mod.flash_attention(qb, kb, vb, causal=causal)
        t = lambda a: torch.from_numpy(a).cuda().to(torch.bfloat16)  # noqa: E731
        got = sg.flash_attention(t(q), t(k), t(v), causal=causal).float().cpu().numpy()
    close(got, want)


@pytest.mark.parametrize("kernel", [4, 3, 1, 2, 0],
                         ids=["warp-split", "tensor-core-cluster", "cluster", "key-parallel", "generic"])
@pytest.mark.parametrize("Skv,Sq,H,Hkv,D", [(768, 1, 32, 8, 64), (4096, 1, 28, 4, 128), (1000, 3, 8, 8, 64),
                                            (64, 1, 4, 2, 32), (8192, 1, 28, 4, 128), (37, 2, 16, 2, 64),
                                            (300, 4, 28, 4, 128)])
def test_decode_against_kv_cache(sg, oracle_mod, kernel, Skv, Sq, H, Hkv, D):
    """Queries at the end of a strided KV cache (capacity > S_kv), split-K, with
    each decode kernel: the cluster of key splits merged in distributed shared
    memory (scores and P V on tensor cores, or on CUDA cores), the
    key-parallel kernel plus a combine kernel, the generic one."""
    rng = np.random.default_rng(Skv)
    cap = Skv + 37
    q = rng.standard_normal((2, H, Sq, D)).astype(np.float16)
    kc = rng.standard_normal((2, Hkv, cap, D)).astype(np.float16)
    vc = rng.standard_normal((2, Hkv, cap, D)).astype(np.float16)
    want = oracle_mod.flash_attention(q, np.ascontiguousarray(kc[:, :, :Skv]), np.ascontiguousarray(vc[:, :, :Skv]),
                                      causal=True, q_pos0=Skv - Sq).astype(np.float32)
    try:
        sg.set_tuning("attn.decode_kernel", kernel)
        got = sg.flash_attention(dev(q), dev(kc), dev(vc), causal=True, q_pos0=-1, decode=True, kv_len=Skv)
        got2 = sg.flash_attention(dev(q), dev(kc), dev(vc), causal=True, q_pos0=-1, decode=True, kv_len=Skv)
    finally:
        sg.set_tuning("attn.decode_kernel", 4)
    close(got.float().cpu().numpy(), want)
    assert torch.equal(got, got2)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_decode_cluster_kernel_io_types(sg, oracle_mod, dtype, D):
    """fp32 caches (CUDA-core cluster kernel at head_dim 64, key-parallel at 128)
    and bf16 caches (tensor-core cluster kernel, fp16 inside)."""
    rng = np.random.default_rng(7)
    Skv, Sq, H, Hkv = 700, 1, 32, 8
    q = rng.standard_normal((1, H, Sq, D)).astype(np.float32)
    kc = rng.standard_normal((1, Hkv, Skv, D)).astype(np.float32)
    vc = rng.standard_normal((1, Hkv, Skv, D)).astype(np.float32)
    if dtype == "f32":
        want = oracle_mod.flash_attention(q, kc, vc, causal=True, q_pos0=Skv - Sq)
        t = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    else:
        q, kc, vc = (oracle_mod.bf16_bits_to_f32(oracle_mod.f32_to_bf16_bits(a)) for a in (q, kc, vc))
        want = oracle_mod.flash_attention(q, kc, vc, causal=True, q_pos0=Skv - Sq)
        t = lambda a: torch.from_numpy(a).cuda().to(torch.bfloat16)  # noqa: E731
    got = sg.flash_attention(t(q), t(kc), t(vc), causal=True, q_pos0=-1, decode=True)
    close(got.float().cpu().numpy(), want)


def test_attention_rejects_bad_heads(sg):
    from silicongraph_b200._lib import SgError
    q = torch.zeros(1, 7, 4, 16, dtype=torch.float16, device="cuda")
    k = torch.zeros(1, 2, 4, 16, dtype=torch.float16, device="cuda")
    with pytest.raises(SgError):
        sg.flash_attention(q, k, k)


def test_library_scratch_shared_safely_between_kernels(sg, oracle_mod):
    """Split-scratch users interleaved on one stream (INT4 GEMV at two shapes,
    split-K decode attention, INT8 GEMV) must not corrupt each other's ticket
    counters."""
    rng = np.random.default_rng(0)

    def w4(K, N, gs, seed):
        W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
        B, S, Z = oracle_mod.quantize_int4_grouped(W, gs)
        x = rng.standard_normal((1, K)).astype(np.float32)
        want = oracle_mod.matmul_int4_grouped(x, B, S, Z, K, N, gs, c_dt=oracle_mod.DT_F32)
        return (dev(x), dev(B), dev(S), dev(Z), K, N, gs), want

    small, want_s = w4(1024, 2048, 32, 1)
    large, want_l = w4(2048, 65536, 32, 2)
    q = rng.standard_normal((1, 8, 1, 64)).astype(np.float16)
    kc = rng.standard_normal((1, 2, 900, 64)).astype(np.float16)
    want_a = oracle_mod.flash_attention(q, kc, kc, causal=True, q_pos0=899).astype(np.float32)
    sg.set_tuning("w4_gemv_mma.cluster", 0)  # force the scratch-reduced split
    try:
        for _ in range(3):
            a = sg.matmul_int4_grouped(*small[:4], *small[4:], out_dtype=torch.float32)
            o = sg.flash_attention(dev(q), dev(kc), dev(kc), causal=True, q_pos0=-1, decode=True)
            b = sg.matmul_int4_grouped(*large[:4], *large[4:], out_dtype=torch.float32)
            a2 = sg.matmul_int4_grouped(*small[:4], *small[4:], out_dtype=torch.float32)
            close(a.cpu().numpy(), want_s)
            close(a2.cpu().numpy(), want_s)
            close(b.cpu().numpy(), want_l)
            close(o.float().cpu().numpy(), want_a)
    finally:
        sg.set_tuning("w4_gemv_mma.cluster", 1)


@pytest.mark.parametrize("kernel", [4, 3, 1, 2, 0])
@pytest.mark.parametrize("B,pos", [(1, 0), (1, 63), (1, 600), (1, 1500), (16, 600), (4, 2046)])
def test_decode_position_on_device(sg, oracle_mod, kernel, B, pos):
    """A captured decode step launches for the cache's capacity and reads the
    position from device memory: the live keys are spread over the splits at run
    time.  Every kernel matches the oracle on the live prefix at short, long and
    tile-boundary positions, with one and with many sequences."""
    rng = np.random.default_rng(pos + B)
    cap, H, Hkv, D = 2048, 32, 8, 64
    q = rng.standard_normal((B, H, 1, D)).astype(np.float16)
    kc = rng.standard_normal((B, Hkv, cap, D)).astype(np.float16)
    vc = rng.standard_normal((B, Hkv, cap, D)).astype(np.float16)
    n = pos + 1
    want = oracle_mod.flash_attention(q, np.ascontiguousarray(kc[:, :, :n]), np.ascontiguousarray(vc[:, :, :n]),
                                      causal=True, q_pos0=pos).astype(np.float32)
    p = torch.tensor([pos], dtype=torch.int32, device="cuda")
    try:
        sg.set_tuning("attn.decode_kernel", kernel)
        got = sg.flash_attention(dev(q), dev(kc), dev(vc), causal=True, decode=True, kv_len=cap, q_pos_device=p)
    finally:
        sg.set_tuning("attn.decode_kernel", 4)
    close(got.float().cpu().numpy(), want)


@pytest.mark.parametrize("D,H,Hkv", [(64, 32, 8), (128, 28, 4)])
def test_decode_warp_split_bf16(sg, oracle_mod, D, H, Hkv):
    """bf16 KV caches on the warp-split kernel (fp16 inside), GQA 4 and 7."""
    rng = np.random.default_rng(D)
    Skv = 1000
    q = rng.standard_normal((2, H, 1, D)).astype(np.float32)
    kc = rng.standard_normal((2, Hkv, Skv, D)).astype(np.float32)
    vc = rng.standard_normal((2, Hkv, Skv, D)).astype(np.float32)
    q, kc, vc = (oracle_mod.bf16_bits_to_f32(oracle_mod.f32_to_bf16_bits(a)) for a in (q, kc, vc))
    want = oracle_mod.flash_attention(q, kc, vc, causal=True, q_pos0=Skv - 1)
    t = lambda a: torch.from_numpy(a).cuda().to(torch.bfloat16)  # noqa: E731
    try:
        sg.set_tuning("attn.decode_kernel", 4)
        got = sg.flash_attention(t(q), t(kc), t(vc), causal=True, q_pos0=-1, decode=True)
    finally:
        sg.set_tuning("attn.decode_kernel", 4)
    close(got.float().cpu().numpy(), want)


@pytest.mark.parametrize("qs,ks,vs", [(1.0, 1.0, 1.0), (300.0, 1e-3, 1e5), (1e-20, 1e20, 1e-30)],
                         ids=["unit", "beyond-fp16-range", "extreme-exponents"])
def test_f32_attention_on_tensor_cores(sg, oracle_mod, qs, ks, vs):
    """fp32 I/O at the config-1 shape [1, 32, 512, 64] runs on the tcgen05
    kernel through fp16 copies scaled per tensor by powers of two (exact), so
    values far outside fp16's range give the same result as the fp32 oracle
    within the bar; compared with the CUDA-core fp32 path as well."""
    B, H, S, D = 1, 32, 512, 64
    rng = np.random.default_rng(int(qs * 7) % 1000 + 3)
    q = (rng.standard_normal((B, H, S, D)) * qs).astype(np.float32)
    k = (rng.standard_normal((B, H, S, D)) * ks).astype(np.float32)
    v = (rng.standard_normal((B, H, S, D)) * vs).astype(np.float32)
    want = oracle_mod.flash_attention(q, k, v, causal=True)
    got = sg.flash_attention(dev(q), dev(k), dev(v), causal=True).cpu().numpy()
    close(got / vs, want / vs)
    sg.set_tuning("attn_tc.enable", 0)
    try:
        cc = sg.flash_attention(dev(q), dev(k), dev(v), causal=True).cpu().numpy()
    finally:
        sg.set_tuning("attn_tc.enable", 1)
    close(got / vs, cc / vs)
