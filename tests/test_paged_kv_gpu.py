"""The paged KV cache (the reference's planPagedLayout,
compiler/lib/memory/kv_cache_layout.cpp:65-102: a pool of pages
[page][K|V][kv_head][16][head_dim] and a page table) on the GPU.

Paging changes where a key lives, not what is computed, so every kernel that
reads or writes the cache must give bit for bit the results of the flat
layout: the KV append (sg_qkv_rope_append_paged), every decode-attention
kernel (sg_flash_decode) and the tensor-core and CUDA-core prefill attention
(sg_flash_attention), with the pages of each sequence scattered over the pool
by a random permutation; then whole sessions, paged against flat, logits
equal bit for bit; and a session whose pool is too small refuses with
ARMCC_ERR_OOM before launching anything."""
import ctypes

import numpy as np
import pytest
import torch

from silicongraph_b200 import armpack

pytestmark = pytest.mark.gpu
PAGE = 16


class Pool:
    """K / V [B, Hkv, S, D] copied into a pool of pages in random order, plus
    spare pages, and the table that finds them (table [B][logical page])."""

    def __init__(self, K, V, spare=5, seed=0):
        B, Hkv, S, D = K.shape
        self.lpages = (S + PAGE - 1) // PAGE
        self.npages = B * self.lpages + spare
        rng = np.random.default_rng(seed)
        perm = rng.permutation(self.npages)[:B * self.lpages].reshape(B, self.lpages)
        self.pool = torch.zeros((self.npages, 2, Hkv, PAGE, D), dtype=K.dtype, device=K.device)
        for b in range(B):
            for lp in range(self.lpages):
                n = min(PAGE, S - lp * PAGE)
                self.pool[perm[b, lp], 0, :, :n] = K[b, :, lp * PAGE:lp * PAGE + n]
                self.pool[perm[b, lp], 1, :, :n] = V[b, :, lp * PAGE:lp * PAGE + n]
        self.table = torch.from_numpy(perm.astype(np.int32)).cuda()
        from silicongraph_b200._lib import SgKvPages
        self.desc = SgKvPages()
        self.desc.table = self.table.data_ptr()
        self.desc.page_size = PAGE
        self.desc.num_pages = self.npages
        self.desc.page_stride = 2 * Hkv * PAGE * D
        self.desc.table_batch_stride = self.lpages
        self.desc.table_page_stride = 1
        self.k0 = self.pool[0, 0]  # K half of page 0
        self.v0 = self.pool[0, 1]

    def to_flat(self, B, S):
        """The pool's contents back in the flat layout (for the append check)."""
        Hkv, D = self.pool.shape[2], self.pool.shape[4]
        K = torch.zeros((B, Hkv, self.lpages * PAGE, D), dtype=self.pool.dtype, device=self.pool.device)
        V = torch.zeros_like(K)
        t = self.table.cpu().numpy()
        for b in range(B):
            for lp in range(self.lpages):
                K[b, :, lp * PAGE:(lp + 1) * PAGE] = self.pool[t[b, lp], 0]
                V[b, :, lp * PAGE:(lp + 1) * PAGE] = self.pool[t[b, lp], 1]
        return K[:, :, :S], V[:, :, :S]


def attention(Q, K, V, Skv, q_pos0, decode, pool=None, Hkv=None):
    from silicongraph_b200 import _lib
    from silicongraph_b200._lib import SgFlashAttentionParams
    from silicongraph_b200.kernels import dtype_code
    B, H, Sq, D = Q.shape
    O = torch.empty_like(Q)
    p = SgFlashAttentionParams()
    p.Q, p.O = Q.data_ptr(), O.data_ptr()
    p.B, p.S, p.num_heads, p.head_dim = B, Sq, H, D
    p.causal = 1
    p.io_dtype = dtype_code(Q.dtype)
    p.S_kv = Skv
    p.q_pos0 = q_pos0
    if pool is None:
        p.K, p.V = K.data_ptr(), V.data_ptr()
        p.num_kv_heads = K.shape[1]
        p.kv_head_stride, p.kv_batch_stride = K.stride(1), K.stride(0)
    else:
        p.K, p.V = pool.k0.data_ptr(), pool.v0.data_ptr()
        p.num_kv_heads = Hkv
        p.kv_pages = ctypes.pointer(pool.desc)
    lib = _lib.load()
    fn = lib.sg_flash_decode if decode else lib.sg_flash_attention
    _lib.check(fn(ctypes.byref(p), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return O


def _qkv(B, H, Hkv, Sq, Skv, D, dt, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, device="cuda").to(dt)  # noqa: E731
    return r(B, H, Sq, D), r(B, Hkv, Skv, D), r(B, Hkv, Skv, D)


@pytest.mark.parametrize("kernel", [4, 3, 1, 2, 0], ids=["warp", "tile", "cluster", "keypar", "generic"])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("B,H,Hkv,Skv,D", [(1, 32, 8, 771, 64), (3, 28, 4, 300, 128), (2, 8, 8, 40, 64)])
def test_decode_paged_equals_flat(sg, kernel, dt, B, H, Hkv, Skv, D):
    Q, K, V = _qkv(B, H, Hkv, 1, Skv, D, dt, seed=Skv + D)
    pool = Pool(K, V, seed=B)
    sg.set_tuning("attn.decode_kernel", kernel)
    try:
        want = attention(Q, K, V, Skv, Skv - 1, True)
        got = attention(Q, None, None, Skv, Skv - 1, True, pool, Hkv)
    finally:
        sg.set_tuning("attn.decode_kernel", 4)
    assert torch.equal(got, want)


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("B,H,Hkv,Sq,Skv,D", [
    (1, 28, 4, 512, 512, 128),    # tensor-core prefill (fp16 / bf16), one chunk
    (2, 32, 8, 256, 700, 64),     # a later chunk attending to earlier ones, ragged tail page
    (1, 8, 2, 37, 90, 64),        # CUDA-core prefill (few queries)
])
def test_prefill_paged_equals_flat(sg, dt, B, H, Hkv, Sq, Skv, D):
    Q, K, V = _qkv(B, H, Hkv, Sq, Skv, D, dt, seed=Sq + Skv)
    pool = Pool(K, V, seed=Sq)
    want = attention(Q, K, V, Skv, Skv - Sq, False)
    got = attention(Q, None, None, Skv, Skv - Sq, False, pool, Hkv)
    assert torch.equal(got, want)


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_append_paged_equals_flat(sg, dt):
    """sg_qkv_rope_append_paged writes the same rows the flat append writes,
    at pages found through the table (positions 5 .. 5+T-1 of 2 sequences)."""
    from silicongraph_b200 import _lib
    lib = _lib.load()
    B, Ts, H, Hkv, D, pos0 = 2, 21, 8, 2, 64, 5
    S = pos0 + Ts
    qkv = torch.randn(B * Ts, (H + 2 * Hkv) * D, device="cuda").to(dt)
    q_flat = torch.empty(B, H, Ts, D, dtype=dt, device="cuda")
    Kf = torch.zeros(B, Hkv, S, D, dtype=dt, device="cuda")
    Vf = torch.zeros_like(Kf)
    st = torch.cuda.current_stream().cuda_stream
    code = 2 if dt == torch.float16 else 3
    _lib.check(lib.sg_qkv_rope_append_batched(qkv.data_ptr(), B, Ts, H, Hkv, D, None, pos0, 500000.0,
                                              q_flat.data_ptr(), Kf.data_ptr(), Vf.data_ptr(), S * D, Hkv * S * D,
                                              code, st))
    pool = Pool(torch.zeros_like(Kf), torch.zeros_like(Vf), seed=7)
    q_paged = torch.empty_like(q_flat)
    _lib.check(lib.sg_qkv_rope_append_paged(qkv.data_ptr(), B, Ts, H, Hkv, D, None, pos0, 500000.0,
                                            q_paged.data_ptr(), pool.k0.data_ptr(), pool.v0.data_ptr(),
                                            ctypes.byref(pool.desc), code, st))
    torch.cuda.synchronize()
    Kp, Vp = pool.to_flat(B, S)
    assert torch.equal(q_paged, q_flat)
    assert torch.equal(Kp[:, :, pos0:], Kf[:, :, pos0:]) and torch.equal(Vp[:, :, pos0:], Vf[:, :, pos0:])


def test_bad_page_id_is_reported_not_dereferenced(sg):
    """A table entry outside the pool reads page 0 and sets the device error
    word; the call itself succeeds and the GPU stays usable."""
    from silicongraph_b200 import _lib
    Q, K, V = _qkv(1, 8, 2, 1, 64, 64, torch.float16, seed=3)
    pool = Pool(K, V, seed=1)
    pool.table[0, 2] = pool.npages + 1000  # no such page
    attention(Q, None, None, 64, 63, True, pool, 2)
    assert _lib.load().sg_device_error_check(torch.cuda.current_stream().cuda_stream) == _lib.SG_ERR_RUNTIME
    assert b"device-side error 4" in _lib.load().sg_last_error()
    pool.table[0, 2] = 0
    attention(Q, None, None, 64, 63, True, pool, 2)
    assert _lib.load().sg_device_error_check(torch.cuda.current_stream().cuda_stream) == 0


# ------------------------------------------------------------------ sessions
SMALL = armpack.llama_config(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000,
                             rope_theta=500000.0, max_pos=8192)


def _package(tmp_path, ctx, chunk=64):
    w = armpack.random_llama_weights(SMALL, seed=1)
    t = armpack.cuda_tensors(SMALL, w, group_size=32)
    return armpack.write_package(str(tmp_path / f"m{ctx}.armpack"), SMALL, t, max_context=ctx,
                                 max_prefill_chunk=chunk)


@pytest.mark.parametrize("batch", [1, 3])
def test_paged_session_equals_flat_session(sg, tmp_path, batch):
    from silicongraph_b200 import sdk
    path = _package(tmp_path, 1024)
    V = SMALL["vocab_size"]
    prompts = np.random.default_rng(batch).integers(0, V, (batch, 150)).astype(np.int32)  # three chunks
    runs = []
    for pool_tokens in (None, batch * 200):
        with sdk.Package(path) as pkg:
            with pkg.select().session(batch=batch, kv_pool_tokens=pool_tokens) as s:
                if batch == 1:
                    s.prefill(prompts[0])
                else:
                    s.batch_prefill(prompts)
                logits, toks = [s.last_logits()], []
                for _ in range(6):
                    toks.append(s.decode().next_token_id if batch == 1 else s.batch_decode().tolist())
                    logits.append(s.last_logits())
                info = s.kv_pages
        runs.append((toks, logits, info))
    (t_flat, l_flat, i_flat), (t_paged, l_paged, i_paged) = runs
    assert i_flat is None
    pool, used = i_paged
    assert pool == (batch * 200 + 15) // 16 * SMALL["num_layers"]
    assert used == batch * SMALL["num_layers"] * ((150 + 6 + 15) // 16)
    assert t_paged == t_flat
    for a, b in zip(l_paged, l_flat):
        assert np.array_equal(a, b)


def test_paged_pool_refuses_when_full_and_reset_returns_pages(sg, tmp_path):
    from silicongraph_b200 import sdk
    path = _package(tmp_path, 1024)
    with sdk.Package(path) as pkg:
        with pkg.select().session(kv_pool_tokens=64) as s:  # 4 pages of 16 tokens per layer
            s.prefill(np.arange(60, dtype=np.int32))
            for _ in range(5):
                s.decode()                                  # the prompt's token, then positions 60 .. 63
            with pytest.raises(sdk.ArmError) as e:
                s.decode()                                  # position 64 needs a fifth page
            assert e.value.status == -3 and "pool" in str(e.value)
            s.reset()
            assert s.kv_pages[1] == 0
            s.prefill(np.arange(30, dtype=np.int32))
            assert s.kv_pages[1] == 2 * SMALL["num_layers"]


def test_long_context_graph_pages_by_default(sg, tmp_path):
    """The reference's rule (kv_cache_layout.cpp:107-130): contexts above 4096
    tokens are paged."""
    from silicongraph_b200 import sdk
    with sdk.Package(_package(tmp_path, 8192)) as pkg:
        with pkg.select().session() as s:
            s.prefill(np.arange(20, dtype=np.int32))
            pool, used = s.kv_pages
            assert pool == 8192 // 16 * SMALL["num_layers"] and used == 2 * SMALL["num_layers"]
    with sdk.Package(_package(tmp_path, 4096)) as pkg:
        with pkg.select().session() as s:
            assert s.kv_pages is None


@pytest.mark.parametrize("paged", [False, True], ids=["flat", "paged"])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("H,Hkv,D,K", [(32, 8, 64, 2048), (28, 4, 128, 3584)])
def test_qkv_gemv_rope_append_equals_two_calls(sg, oracle_mod, dt, H, Hkv, D, K, paged):
    """sg_qkv_gemv_rope_append (the q|k|v GEMV with the rope and the KV append
    in its epilogue) writes the same q and cache rows, bit for bit, as the GEMV
    followed by sg_qkv_rope_append."""
    from silicongraph_b200 import _lib
    from silicongraph_b200._lib import SgKvPages
    lib = _lib.load()
    lib.sg_qkv_gemv_rope_append.restype = ctypes.c_int32
    N, gs, pos = (H + 2 * Hkv) * D, 32, 37
    rng = np.random.default_rng(H + D)
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    B, S, Z = (torch.from_numpy(a).cuda() for a in oracle_mod.quantize_int4_grouped(W, gs))
    x = torch.randn(1, K, device="cuda").to(dt)
    st = torch.cuda.current_stream().cuda_stream
    code = 2 if dt == torch.float16 else 3
    # two calls: GEMV, then rope + append into a flat cache of 64 positions
    qkv = sg.matmul_int4_grouped(x, B, S, Z, K, N, gs, out_dtype=dt)
    q_want = torch.empty(H, D, dtype=dt, device="cuda")
    Kw = torch.zeros(1, Hkv, 64, D, dtype=dt, device="cuda")
    Vw = torch.zeros_like(Kw)
    _lib.check(lib.sg_qkv_rope_append_batched(qkv.data_ptr(), 1, 1, H, Hkv, D, None, pos, 500000.0,
                                              q_want.data_ptr(), Kw.data_ptr(), Vw.data_ptr(), 64 * D, Hkv * 64 * D,
                                              code, st))

    class SgRopeAppend(ctypes.Structure):
        _fields_ = [("heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                    ("positions", ctypes.c_void_p), ("pos0", ctypes.c_int32), ("base", ctypes.c_float),
                    ("q_out", ctypes.c_void_p), ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
                    ("kv_head_stride", ctypes.c_int64), ("kv_pages", ctypes.POINTER(SgKvPages))]

    q_got = torch.empty_like(q_want)
    r = SgRopeAppend(heads=H, kv_heads=Hkv, head_dim=D, positions=None, pos0=pos, base=500000.0,
                     q_out=q_got.data_ptr())
    pos_dev = torch.tensor([pos], dtype=torch.int32, device="cuda")
    r.positions = pos_dev.data_ptr()                      # the position read on the device
    if paged:
        pool = Pool(torch.zeros_like(Kw), torch.zeros_like(Vw), seed=3)
        r.k_cache, r.v_cache = pool.k0.data_ptr(), pool.v0.data_ptr()
        r.kv_pages = ctypes.pointer(pool.desc)
    else:
        Kg, Vg = torch.zeros_like(Kw), torch.zeros_like(Vw)
        r.k_cache, r.v_cache, r.kv_head_stride = Kg.data_ptr(), Vg.data_ptr(), 64 * D
    C = torch.empty_like(qkv)
    p = sg.matmul_params(x, B, C, M=1, K=K, N=N, scales=S, zeros=Z, group_size=gs)
    _lib.check(lib.sg_qkv_gemv_rope_append(ctypes.byref(p), ctypes.byref(r), st))
    torch.cuda.synchronize()
    if paged:
        Kg, Vg = pool.to_flat(1, 64)
    assert torch.equal(q_got, q_want)
    assert torch.equal(Kg[:, :, pos], Kw[:, :, pos]) and torch.equal(Vg[:, :, pos], Vw[:, :, pos])
