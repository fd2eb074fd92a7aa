"""Block ops on the GPU (rmsnorm, silu, SwiGLU, softmax, rope, embedding,
argmax) through the C ABI, against the reference's own kernels (golden vectors
from matmul_neon.h:154-275 compiled here) and the oracle.

Tolerance for 16-bit outputs: the reference's own NEON-vs-scalar spread
(rtol 2e-3, atol 1e-3, about one fp16 ulp); fp32: 1e-5 relative."""
import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def close16(got, want, rtol=2e-3, atol=1e-3):
    np.testing.assert_allclose(np.asarray(got, np.float32), np.asarray(want, np.float32), rtol=rtol, atol=atol)


def test_block_ops_match_reference_golden(sg):
    g = golden("block_ops.npz")
    x, w = g["x"], g["w"]
    close16(sg.rmsnorm(dev(x).view(1, -1), dev(w)).cpu().numpy().ravel(), g["rmsnorm_scalar"])
    close16(sg.silu(dev(x)).cpu().numpy(), g["silu_scalar"])
    close16(sg.softmax(dev(x).view(1, -1)).cpu().numpy().ravel(), g["softmax_scalar"])
    r = dev(x[:64].copy()).view(1, 1, 64)
    close16(sg.rope(r, pos0=37, base=500000.0).cpu().numpy().ravel(), g["rope_scalar"])


@pytest.mark.parametrize("rows,n", [(1, 2048), (7, 3584), (16, 100)])
def test_rmsnorm_vs_oracle(sg, oracle_mod, rows, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal((rows, n)).astype(np.float16)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float16)
    want = np.stack([oracle_mod.rmsnorm_f16(x[r], w) for r in range(rows)])
    close16(sg.rmsnorm(dev(x), dev(w)).cpu().numpy(), want)
    # fused residual: residual <- round(x + residual), y = rmsnorm(residual)
    res = rng.standard_normal((rows, n)).astype(np.float16)
    h = (x.astype(np.float32) + res.astype(np.float32)).astype(np.float16)
    want_r = np.stack([oracle_mod.rmsnorm_f16(h[r], w) for r in range(rows)])
    rt = dev(res)
    y = sg.rmsnorm(dev(x), dev(w), residual=rt)
    assert np.array_equal(rt.cpu().numpy().view(np.uint16), h.view(np.uint16))
    close16(y.cpu().numpy(), want_r)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rmsnorm_other_dtypes(sg, oracle_mod, dtype):
    rng = np.random.default_rng(3)
    x32 = rng.standard_normal((4, 2048)).astype(np.float32)
    w32 = (1 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
    xt, wt = dev(x32).to(dtype), dev(w32).to(dtype)
    xo, wo = xt.float().cpu().numpy(), wt.float().cpu().numpy()
    want = np.stack([oracle_mod.rmsnorm_f32(xo[r], wo) for r in range(4)])
    got = sg.rmsnorm(xt, wt).float().cpu().numpy()
    tol = dict(rtol=1e-5, atol=1e-6) if dtype == torch.float32 else dict(rtol=1e-2, atol=2e-3)
    np.testing.assert_allclose(got, want, **tol)


def test_silu_and_swiglu(sg, oracle_mod):
    rng = np.random.default_rng(5)
    g_ = (3 * rng.standard_normal(8192 * 3)).astype(np.float16)
    u = rng.standard_normal(8192 * 3).astype(np.float16)
    s = oracle_mod.silu_f16(g_)
    close16(sg.silu(dev(g_)).cpu().numpy(), s)
    want = (s.astype(np.float32) * u.astype(np.float32)).astype(np.float16)
    close16(sg.silu_mul(dev(g_), dev(u)).cpu().numpy(), want)


@pytest.mark.parametrize("n", [1000, 128256])
def test_softmax_vs_oracle(sg, oracle_mod, n):
    rng = np.random.default_rng(n)
    x = (2 * rng.standard_normal((2, n))).astype(np.float16)
    want = np.stack([oracle_mod.softmax_f16(x[r]) for r in range(2)])
    got = sg.softmax(dev(x)).cpu().numpy()
    close16(got, want, rtol=2e-3, atol=1e-6)


@pytest.mark.parametrize("D,base,pos0", [(64, 500000.0, 0), (128, 1000000.0, 8000), (64, 10000.0, 3)])
def test_rope_vs_oracle(sg, oracle_mod, D, base, pos0):
    rng = np.random.default_rng(D + pos0)
    T, H = 5, 3
    x = rng.standard_normal((T, H, D)).astype(np.float16)
    want = x.copy()
    for t in range(T):
        for h in range(H):
            want[t, h] = oracle_mod.rope_f16(want[t, h].copy(), pos0 + t, base)
    got = sg.rope(dev(x), pos0=pos0, base=base).cpu().numpy()
    close16(got, want)
    # explicit per-token positions give the same result
    pos = torch.arange(pos0, pos0 + T, dtype=torch.int32, device="cuda")
    got2 = sg.rope(dev(x), positions=pos, base=base).cpu().numpy()
    assert np.array_equal(got.view(np.uint16), got2.view(np.uint16))


def test_embedding_and_argmax(sg):
    rng = np.random.default_rng(9)
    table = rng.standard_normal((1000, 2048)).astype(np.float16)
    ids = np.array([0, 999, 5, 5, 123], np.int32)
    got = sg.embedding(dev(table), dev(ids)).cpu().numpy()
    assert np.array_equal(got.view(np.uint16), table[ids].view(np.uint16))
    logits = rng.standard_normal((3, 128256)).astype(np.float32)
    logits[1, 777] = logits[1, 12345] = 50.0   # tie: the first index wins
    logits[2, :] = -np.inf
    logits[2, 4] = np.nan                      # NaN never wins
    out = sg.argmax(dev(logits)).cpu().numpy()
    assert out[0] == int(np.argmax(logits[0]))
    assert out[1] == 777
    assert out[2] == 0
