"""End to end through the armcc SDK on the GPU: a random-init Llama-style INT4
package, prefill + greedy decode, against the decoder composition oracle
(oracle/decoder.py: the reference's kernel semantics with fp16 values at op
boundaries).  Logits within |got - want| <= 2e-3 + 1e-2 |want|; greedy tokens
equal wherever the oracle's top two logits differ by more than that."""
import numpy as np
import pytest

from silicongraph_b200 import armpack

pytestmark = pytest.mark.gpu

SMALL = armpack.llama_config(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000,
                             rope_theta=500000.0, max_pos=4096)
RTOL, ATOL = 1e-2, 2e-3


def close(got, want):
    err = np.abs(got - want)
    bad = err > ATOL + RTOL * np.abs(want)
    assert not bad.any(), f"{bad.sum()} / {bad.size} logits outside tolerance; max err {err.max():.3e}"


def check_token(tok, logits_ref):
    top = np.sort(logits_ref)[-2:]
    if top[1] - top[0] > ATOL + RTOL * abs(top[1]):
        assert tok == int(np.argmax(logits_ref))


def _package(tmp_path, chunk, ctx=1024, seed=1):
    w = armpack.random_llama_weights(SMALL, seed=seed)
    t = armpack.cuda_tensors(SMALL, w, group_size=32)
    path = armpack.write_package(str(tmp_path / f"m{chunk}.armpack"), SMALL, t, max_context=ctx,
                                 max_prefill_chunk=chunk)
    return path, t


@pytest.mark.parametrize("prompt_len,chunk", [
    (37, 128),     # short prompt: CUDA-core attention
    (300, 512),    # one 300-token chunk: tensor-core GEMM and tensor-core attention
    (300, 128),    # chunked prefill: three chunks attending to the earlier ones
])
def test_session_matches_decoder_oracle(sg, oracle_mod, tmp_path, prompt_len, chunk):
    from oracle.decoder import DecoderOracle
    from silicongraph_b200 import sdk
    path, t = _package(tmp_path, chunk)
    rng = np.random.default_rng(prompt_len)
    prompt = rng.integers(0, SMALL["vocab_size"], prompt_len).astype(np.int32)
    ref = DecoderOracle(SMALL, t, group_size=32)
    with sdk.Package(path) as pkg:
        g = pkg.select(context_length=prompt_len + 8)
        with g.session() as s:
            s.prefill(prompt)
            assert s.position == prompt_len
            want = ref.forward(prompt)
            close(s.last_logits(SMALL["vocab_size"]), want)
            tok = s.decode().next_token_id
            check_token(tok, want)
            for step in range(4):
                want = ref.forward([tok])
                r = s.decode()
                close(s.last_logits(SMALL["vocab_size"]), want)
                check_token(r.next_token_id, want)
                assert r.tokens_generated == step + 2
                tok = r.next_token_id
            assert s.position == prompt_len + 4


def test_generate_run_and_reset(sg, tmp_path):
    from silicongraph_b200 import sdk
    path, _ = _package(tmp_path, 128)
    prompt = np.arange(20, dtype=np.int32) * 7 % SMALL["vocab_size"]
    with sdk.Package(path) as pkg:
        g = pkg.select()
        with g.session() as s:
            a = s.generate(prompt, 6)
            s.reset()
            b = s.generate(prompt, 6)
            assert a == b and len(a) == 6
            assert s.position == 20 + 5
        r = g.run(prompt)
        assert r.status == 0 and r.next_token_id == a[0]


def test_session_errors(sg, tmp_path):
    from silicongraph_b200 import sdk
    path, _ = _package(tmp_path, 64, ctx=96)
    with sdk.Package(path) as pkg:
        with pkg.select().session() as s:
            with pytest.raises(sdk.ArmError):
                s.decode()                                   # nothing prefilled
            with pytest.raises(sdk.ArmError):
                s.prefill([0, 5, SMALL["vocab_size"]])       # token outside the vocabulary
            with pytest.raises(sdk.ArmError) as e:
                s.prefill(np.zeros(97, np.int32))            # longer than the context
            assert e.value.status == -3
            s.prefill(np.zeros(95, np.int32))
            s.decode()                                       # the token predicted by the prompt
            s.decode()                                       # fills position 96
            with pytest.raises(sdk.ArmError) as e:
                s.decode()
            assert e.value.status == -3


def test_decode_graph_matches_eager(sg, tmp_path, monkeypatch):
    """Decode steps replayed from the captured CUDA graph give the same tokens
    and logits as eager launches."""
    from silicongraph_b200 import sdk
    path, _ = _package(tmp_path, 128)
    prompt = (np.arange(40, dtype=np.int32) * 13) % SMALL["vocab_size"]
    runs = []
    for flag in ("1", "0"):
        monkeypatch.setenv("SG_DECODE_GRAPH", flag)
        with sdk.Package(path) as pkg:
            with pkg.select().session() as s:
                s.prefill(prompt)
                toks, logits = [], []
                for _ in range(6):
                    toks.append(s.decode().next_token_id)
                    logits.append(s.last_logits(SMALL["vocab_size"]))
                runs.append((toks, np.stack(logits)))
    assert runs[0][0] == runs[1][0]
    assert np.array_equal(runs[0][1], runs[1][1])


def test_batched_session_matches_each_sequence(sg, oracle_mod, tmp_path):
    """Three sequences prefilled and decoded in lockstep through one session
    (sg_session_create_ex / sg_batch_prefill / sg_batch_decode): each
    sequence's logits and tokens match the oracle run on that sequence alone."""
    from oracle.decoder import DecoderOracle
    from silicongraph_b200 import sdk
    path, t = _package(tmp_path, 64)
    B, n, steps, V = 3, 70, 3, SMALL["vocab_size"]  # 70 tokens: two prefill chunks of up to 64
    prompts = np.random.default_rng(17).integers(0, V, (B, n)).astype(np.int32)
    with sdk.Package(path) as pkg:
        with pkg.select().session(batch=B) as s:
            assert s.batch == B
            with pytest.raises(sdk.ArmError):
                s.prefill(prompts[0])  # the single-sequence calls refuse a batched session
            s.batch_prefill(prompts)
            logits = [s.last_logits().reshape(B, V)]
            toks = [s.batch_decode()]
            for _ in range(steps):
                toks.append(s.batch_decode())
                logits.append(s.last_logits().reshape(B, V))
            assert s.position == n + steps
    for b in range(B):
        ref = DecoderOracle(SMALL, t, group_size=32)
        want = ref.forward(prompts[b])
        close(logits[0][b], want)
        check_token(int(toks[0][b]), want)
        for i in range(steps):
            want = ref.forward([int(toks[i][b])])
            close(logits[i + 1][b], want)
            check_token(int(toks[i + 1][b]), want)


def test_select_graph_refuses_before_allocation(sg, tmp_path):
    """armpack_select_graph sizes a graph's session exactly (the slab the
    session then allocates) and refuses when it exceeds 95 % of the budget:
    the device's free memory, capped by ArmDeviceState.ram_mb."""
    from silicongraph_b200 import sdk
    path, _ = _package(tmp_path, 128)
    with sdk.Package(path) as pkg:
        g = pkg.select(64)
        need = g.session_bytes()
        manifest_peak = g.peak_memory_bytes
        with g.session():
            assert g.peak_memory_bytes == max(manifest_peak, need)   # the slab is what was planned
        budget_mb = (need * 100 // 95) // (1 << 20)                  # just under what 95 % needs
        with pytest.raises(sdk.ArmError) as e:
            pkg.select(64, ram_mb=max(1, budget_mb))
        assert "95%" in str(e.value)
        assert pkg.select(64, ram_mb=budget_mb + 2) is not None


def test_fused_norm_decode_equals_unfused(sg, tmp_path):
    """One-row decode steps with the norms and residual adds fused into the
    projections (and the rope + KV append into the q|k|v projection) give the
    same tokens and logits, bit for bit, as the steps with separate kernels
    (sdk.fuse_norm / sdk.fuse_rope 0); the per-op step (sdk.decode_step_kernel
    0), which these switches select between."""
    from silicongraph_b200 import sdk
    path, _ = _package(tmp_path, 128)
    prompt = (np.arange(33, dtype=np.int32) * 11) % SMALL["vocab_size"]
    runs = []
    sg.set_tuning("sdk.decode_step_kernel", 0)
    try:
        for fuse, rope in ((1, 1), (1, 0), (0, 0)):
            sg.set_tuning("sdk.fuse_norm", fuse)
            sg.set_tuning("sdk.fuse_rope", rope)
            with sdk.Package(path) as pkg:
                with pkg.select().session() as s:
                    s.prefill(prompt)
                    toks, logits = [], []
                    for _ in range(6):
                        toks.append(s.decode().next_token_id)
                        logits.append(s.last_logits(SMALL["vocab_size"]))
            runs.append((toks, np.stack(logits)))
    finally:
        sg.set_tuning("sdk.fuse_norm", 1)
        sg.set_tuning("sdk.fuse_rope", 1)
    for other in runs[1:]:
        assert runs[0][0] == other[0]
        assert np.array_equal(runs[0][1], other[1])
