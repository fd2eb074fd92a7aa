"""End to end at the full Llama-3.2-1B shape (16 layers, hidden 2048, 32 query /
8 KV heads, head_dim 64, SwiGLU 8192, vocab 128256, RoPE theta 500000, INT4
group-32 weights, random N(0, 0.02) init) through the armcc SDK on the GPU,
against the decoder composition oracle (oracle/decoder.py: the reference's
kernel semantics, matmul_neon.h:113-147 / flash_attention.h:95-144 /
matmul_neon.h:154-275, fp16 values at op boundaries).

Logits after the prompt and after each of four greedy steps within
|got - want| <= 2e-3 + 1e-2 |want| over the whole vocabulary; greedy tokens
equal wherever the oracle's top two logits differ by more than that.  Batch 1,
and two sequences of a batch-16 session."""
import numpy as np
import pytest

from silicongraph_b200 import armpack

pytestmark = pytest.mark.gpu

LLAMA_1B = armpack.llama_config(layers=16, hidden=2048, heads=32, kv_heads=8, head_dim=64, ffn=8192,
                                vocab=128256, rope_theta=500000.0, max_pos=4096)
RTOL, ATOL = 1e-2, 2e-3
STEPS = 4


def close(got, want, what):
    err = np.abs(got - want)
    bad = err > ATOL + RTOL * np.abs(want)
    assert not bad.any(), f"{what}: {bad.sum()} / {bad.size} logits outside tolerance; max err {err.max():.3e}"


def check_token(tok, logits_ref):
    top = np.sort(logits_ref)[-2:]
    if top[1] - top[0] > ATOL + RTOL * abs(top[1]):
        assert tok == int(np.argmax(logits_ref))


@pytest.fixture(scope="module")
def llama1b(sg, tmp_path_factory):
    t = armpack.random_cuda_tensors_on_device(LLAMA_1B, seed=3, group_size=32)
    path = str(tmp_path_factory.mktemp("llama1b") / "llama1b_int4")
    armpack.write_package(path, LLAMA_1B, t, group_size=32, max_context=256, max_prefill_chunk=64, as_zip=False,
                          model_id="synthetic/llama-3.2-1b-shape")
    return path, t


def test_llama1b_batch1_matches_decoder_oracle(llama1b, oracle_mod):
    from oracle.decoder import DecoderOracle
    from silicongraph_b200 import sdk
    path, t = llama1b
    V = LLAMA_1B["vocab_size"]
    prompt = np.random.default_rng(24).integers(0, V, 24).astype(np.int32)
    ref = DecoderOracle(LLAMA_1B, t, group_size=32)
    with sdk.Package(path) as pkg:
        with pkg.select(context_length=64).session() as s:
            s.prefill(prompt)
            want = ref.forward(prompt)
            close(s.last_logits(V), want, "prompt")
            r = s.decode()
            check_token(r.next_token_id, want)
            tok = r.next_token_id
            for step in range(STEPS):
                want = ref.forward([tok])
                r = s.decode()
                close(s.last_logits(V), want, f"step {step}")
                check_token(r.next_token_id, want)
                tok = r.next_token_id


def test_llama1b_batch16_matches_decoder_oracle(llama1b, oracle_mod):
    """Sixteen sequences in lockstep; sequences 0 and 11 are followed by the oracle."""
    from oracle.decoder import DecoderOracle
    from silicongraph_b200 import sdk
    path, t = llama1b
    B, n, V = 16, 20, LLAMA_1B["vocab_size"]
    prompts = np.random.default_rng(16).integers(0, V, (B, n)).astype(np.int32)
    with sdk.Package(path) as pkg:
        with pkg.select(context_length=64).session(batch=B) as s:
            s.batch_prefill(prompts)
            logits = [s.last_logits().reshape(B, V)]
            toks = [s.batch_decode()]
            for _ in range(STEPS):
                toks.append(s.batch_decode())
                logits.append(s.last_logits().reshape(B, V))
    for b in (0, 11):
        ref = DecoderOracle(LLAMA_1B, t, group_size=32)
        want = ref.forward(prompts[b])
        close(logits[0][b], want, f"sequence {b} prompt")
        check_token(int(toks[0][b]), want)
        for i in range(STEPS):
            want = ref.forward([int(toks[i][b])])
            close(logits[i + 1][b], want, f"sequence {b} step {i}")
            check_token(int(toks[i + 1][b]), want)
