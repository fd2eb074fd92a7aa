"""The tcgen05 flash-attention kernel (fp16 / bf16, head_dim 64 or 128, at least
256 queries) through sg_flash_attention, against the oracle restatement of
flash_attention_fp16 (flash_attention.h:95-144).

Tolerance |got - want| <= 2e-3 + 1e-2 |want| (north-star bar for 16-bit outputs)."""
import numpy as np
import pytest
import torch

from test_attention_gpu import close, dev

pytestmark = pytest.mark.gpu


def _qkv(rng, B, H, Hkv, Sq, Skv, D, dtype):
    q = rng.standard_normal((B, H, Sq, D)).astype(np.float32)
    k = rng.standard_normal((B, Hkv, Skv, D)).astype(np.float32)
    v = rng.standard_normal((B, Hkv, Skv, D)).astype(np.float32)
    return q, k, v


def _to(a, dtype, oracle_mod):
    """(array for the oracle, torch tensor on the GPU, oracle io_dt)"""
    if dtype == "f16":
        h = a.astype(np.float16)
        return h, dev(h), oracle_mod.DT_F16
    bits = oracle_mod.f32_to_bf16_bits(a)
    t = torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).cuda()
    return bits, t, oracle_mod.DT_BF16


def _f32(a, io, oracle_mod):
    return oracle_mod.bf16_bits_to_f32(a) if io == oracle_mod.DT_BF16 else np.asarray(a, np.float32)


def _oracle(oracle_mod, qo, ko, vo, io, causal, q_pos0):
    """The oracle in fp32 on the same 16-bit input values: the comparison then
    sees one rounding of the output, not two."""
    q, k, v = (np.ascontiguousarray(_f32(a, io, oracle_mod)) for a in (qo, ko, vo))
    return oracle_mod.flash_attention(q, k, v, causal=causal, q_pos0=q_pos0)


@pytest.mark.parametrize("B,H,Hkv,Sq,Skv,D,causal,dtype,q_pos0", [
    (1, 4, 2, 256, 256, 64, True, "f16", 0),
    (1, 8, 8, 384, 384, 128, True, "bf16", 0),
    (2, 4, 1, 300, 300, 64, False, "f16", 0),       # ragged length, no mask
    (1, 2, 2, 256, 512, 128, True, "bf16", 256),    # chunked prefill: queries at positions 256..511
    (1, 7, 1, 257, 257, 128, True, "f16", 0),       # GQA group of 7, ragged
    (1, 28, 4, 512, 512, 128, True, "bf16", 0),     # Qwen-7B head layout
])
def test_tc_attention_vs_oracle(sg, oracle_mod, B, H, Hkv, Sq, Skv, D, causal, dtype, q_pos0):
    rng = np.random.default_rng(Sq + D + H)
    q, k, v = _qkv(rng, B, H, Hkv, Sq, Skv, D, dtype)
    (qo, qt, io), (ko, kt, _), (vo, vt, _) = (_to(a, dtype, oracle_mod) for a in (q, k, v))
    want = _oracle(oracle_mod, qo, ko, vo, io, causal, q_pos0)
    got = sg.flash_attention(qt, kt, vt, causal=causal, q_pos0=q_pos0).float().cpu().numpy()
    close(got, want)


def test_tc_attention_matches_cuda_core_path(sg, oracle_mod):
    rng = np.random.default_rng(3)
    q, k, v = _qkv(rng, 1, 8, 2, 640, 640, 128, "bf16")
    (_, qt, _), (_, kt, _), (_, vt, _) = (_to(a, "bf16", oracle_mod) for a in (q, k, v))
    a = sg.flash_attention(qt, kt, vt, causal=True)
    sg.set_tuning("attn_tc.enable", 0)
    try:
        b = sg.flash_attention(qt, kt, vt, causal=True)
    finally:
        sg.set_tuning("attn_tc.enable", 1)
    close(a.float().cpu().numpy(), b.float().cpu().numpy())
    assert torch.equal(a, sg.flash_attention(qt, kt, vt, causal=True))  # deterministic


def test_tc_attention_strided_kv_cache(sg, oracle_mod):
    """K / V live in a larger cache [B, Hkv, 1024, D]: 640 valid keys, 256 new queries at 384."""
    rng = np.random.default_rng(5)
    B, H, Hkv, D, Smax, Skv, Sq, pos0 = 1, 4, 2, 64, 1024, 640, 256, 384
    q = rng.standard_normal((B, H, Sq, D)).astype(np.float16)
    kc = rng.standard_normal((B, Hkv, Smax, D)).astype(np.float16)
    vc = rng.standard_normal((B, Hkv, Smax, D)).astype(np.float16)
    want = _oracle(oracle_mod, q, kc[:, :, :Skv], vc[:, :, :Skv], oracle_mod.DT_F16, True, pos0)
    got = sg.flash_attention(dev(q), dev(kc), dev(vc), causal=True, q_pos0=pos0, kv_len=Skv)
    close(got.float().cpu().numpy(), want)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_tc_attention_long_sequence(sg, oracle_mod, dtype):
    """S = 4096: (1) V constant along the keys gives O = V for every query (the
    softmax weights sum to one); (2) sampled rows against the oracle."""
    rng = np.random.default_rng(11)
    B, H, Hkv, S, D = 1, 4, 2, 4096, 128
    q, k, v = _qkv(rng, B, H, Hkv, S, S, D, dtype)
    c = rng.standard_normal((B, Hkv, 1, D)).astype(np.float32)
    vconst = np.broadcast_to(c, v.shape).copy()
    (qo, qt, io), (ko, kt, _), (vo, vt, _) = (_to(a, dtype, oracle_mod) for a in (q, k, v))
    _, vct, _ = _to(vconst, dtype, oracle_mod)
    got_c = sg.flash_attention(qt, kt, vct, causal=True).float().cpu().numpy()
    cexp = np.repeat(vct.float().cpu().numpy()[:, :, :1], H // Hkv, axis=1)  # [B, H, 1, D]
    close(got_c, np.broadcast_to(cexp, got_c.shape))
    got = sg.flash_attention(qt, kt, vt, causal=True).float().cpu().numpy()
    assert np.isfinite(got).all()
    for row in (0, 1, 127, 128, 2047, 4095):
        want = _oracle(oracle_mod, np.ascontiguousarray(qo[:, :, row:row + 1]), ko, vo, io, True, row)
        close(got[:, :, row:row + 1], want)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_tc_attention_config5_layer(sg, oracle_mod, dtype):
    """The Qwen2.5-7B prefill layer of the configuration itself: 28 query / 4
    KV heads (GQA 7), S = 8192, head_dim 128, causal.  Every head's rows at
    sampled positions across all 64 query tiles (tile starts and ends, and
    the last row) against the oracle, and every output finite."""
    rng = np.random.default_rng(5)
    B, H, Hkv, S, D = 1, 28, 4, 8192, 128
    q, k, v = _qkv(rng, B, H, Hkv, S, S, D, dtype)
    (qo, qt, io), (ko, kt, _), (vo, vt, _) = (_to(a, dtype, oracle_mod) for a in (q, k, v))
    got = sg.flash_attention(qt, kt, vt, causal=True).float().cpu().numpy()
    assert np.isfinite(got).all()
    for row in (0, 127, 128, 1000, 4095, 4096, 6143, 8064, 8191):
        want = _oracle(oracle_mod, np.ascontiguousarray(qo[:, :, row:row + 1]), ko[:, :, :row + 1],
                       vo[:, :, :row + 1], io, True, row)
        close(got[:, :, row:row + 1], want)
