"""End to end at the full Llama-3.2-1B shape (16 layers, hidden 2048, 32 query /
8 KV heads, head_dim 64, SwiGLU 8192, vocab 128256, RoPE theta 500000, INT4
group-32 weights, random N(0, 0.02) init) through the armcc SDK on the GPU,
against the decoder composition oracle (oracle/decoder.py: the reference's
kernel semantics, matmul_neon.h:113-147 / flash_attention.h:95-144 /
matmul_neon.h:154-275, fp16 values at op boundaries).  Batch 1, and two
sequences of a batch-16 session; the logits after the prompt and after each of
four greedy steps (batch 1: the persistent decode-step kernel, decode_step.cu).

The yardstick is the reference's own rounding noise.  With fp16 values between
ops, the reference's logits at this width and depth sit about 3e-3 (relative
L2) from the same kernels run in fp32: they miss an elementwise
2e-3 + 1e-2 |y| bar against exact arithmetic on about 6 % of the vocabulary
(and already on some logits with one layer), so no implementation that sums in
another order can meet that bar against them.  Each check therefore measures
the reference's fp16-vs-fp32 distance on the same tokens (the oracle in both
precisions) and requires the GPU's logits to be
  * within 2x that distance of the fp16 reference and of the fp32 one
    (relative L2; measured 1.3x and about 1x),
  * elementwise within 2e-3 + 1e-2 |y| + 10 sigma of the fp16 reference,
    sigma the RMS of the reference's own fp16-vs-fp32 difference,
and the greedy token equal to the reference's wherever its top two logits
differ by more than that elementwise bound.  The strict 2e-3 + 1e-2 |y| bar
holds per kernel at these shapes (tests/test_linear_gpu.py and the attention
tests) and end to end on the small model (tests/test_sdk_gpu.py)."""
import numpy as np
import pytest

from silicongraph_b200 import armpack

pytestmark = pytest.mark.gpu

LLAMA_1B = armpack.llama_config(layers=16, hidden=2048, heads=32, kv_heads=8, head_dim=64, ffn=8192,
                                vocab=128256, rope_theta=500000.0, max_pos=4096)
RTOL, ATOL = 1e-2, 2e-3
STEPS = 4


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(np.asarray(b, np.float64)))


def check(got, want16, want32, what):
    """Returns the elementwise bound used (for the greedy-token check)."""
    noise = rel_l2(want16, want32)
    sigma = float(np.sqrt(np.mean((want16.astype(np.float64) - want32) ** 2)))
    d16, d32 = rel_l2(got, want16), rel_l2(got, want32)
    assert d16 <= 2.0 * noise, f"{what}: GPU vs fp16 reference {d16:.2e}, reference's own noise {noise:.2e}"
    assert d32 <= 2.0 * noise, f"{what}: GPU vs fp32 {d32:.2e}, reference's own noise {noise:.2e}"
    bound = ATOL + RTOL * np.abs(want16) + 10.0 * sigma
    err = np.abs(got - want16)
    bad = err > bound
    assert not bad.any(), f"{what}: {bad.sum()} / {bad.size} logits beyond the bound; max err {err.max():.3e}"
    return ATOL + 10.0 * sigma


def check_token(tok, logits_ref, slack):
    top = np.sort(logits_ref)[-2:]
    if top[1] - top[0] > slack + RTOL * abs(top[1]):
        assert tok == int(np.argmax(logits_ref))


@pytest.fixture(scope="module")
def llama1b(sg, tmp_path_factory):
    t = armpack.random_cuda_tensors_on_device(LLAMA_1B, seed=3, group_size=32)
    path = str(tmp_path_factory.mktemp("llama1b") / "llama1b_int4")
    armpack.write_package(path, LLAMA_1B, t, group_size=32, max_context=256, max_prefill_chunk=64, as_zip=False,
                          model_id="synthetic/llama-3.2-1b-shape")
    return path, t


def test_llama1b_batch1_matches_decoder_oracle(sg, llama1b, oracle_mod):
    from oracle.decoder import DecoderOracle
    from silicongraph_b200 import sdk
    path, t = llama1b
    V = LLAMA_1B["vocab_size"]
    prompt = np.random.default_rng(24).integers(0, V, 24).astype(np.int32)
    r16 = DecoderOracle(LLAMA_1B, t, group_size=32)
    r32 = DecoderOracle(LLAMA_1B, t, group_size=32, precision="f32")
    sg.set_tuning("sdk.decode_step_kernel", 1)
    with sdk.Package(path) as pkg:
        with pkg.select(context_length=64).session() as s:
            s.prefill(prompt)
            want = r16.forward(prompt)
            slack = check(s.last_logits(V), want, r32.forward(prompt), "prompt")
            r = s.decode()
            check_token(r.next_token_id, want, slack)
            tok = r.next_token_id
            for step in range(STEPS):
                want = r16.forward([tok])
                r = s.decode()
                slack = check(s.last_logits(V), want, r32.forward([tok]), f"step {step}")
                check_token(r.next_token_id, want, slack)
                tok = r.next_token_id
            on, why = s.step_kernel
    sg.set_tuning("sdk.decode_step_kernel", 0)
    assert on, why  # the steps ran as the persistent decode-step kernel


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
        r16 = DecoderOracle(LLAMA_1B, t, group_size=32)
        r32 = DecoderOracle(LLAMA_1B, t, group_size=32, precision="f32")
        want = r16.forward(prompts[b])
        slack = check(logits[0][b], want, r32.forward(prompts[b]), f"sequence {b} prompt")
        check_token(int(toks[0][b]), want, slack)
        for i in range(STEPS):
            tok = int(toks[i][b])
            want = r16.forward([tok])
            slack = check(logits[i + 1][b], want, r32.forward([tok]), f"sequence {b} step {i}")
            check_token(int(toks[i + 1][b]), want, slack)
