"""Independent check of the decoder composition oracle against Hugging Face's
own LlamaForCausalLM (transformers), the model the reference's ingestion path
exports and its prompt script runs on the host (scripts/run_prompt.py:186-225).

A small random-init Llama-style model is packed to the "cuda" profile (INT4
group 32); the HF model, built from a config with no download, gets the same
weights dequantised back to fp32 (and the fp16-rounded embedding and norm
weights the package holds) and runs in fp32 eager attention.  The oracle keeps
fp16 values at every op boundary, as the reference's fp16 kernels do, so the two
differ by fp16 rounding only (4e-4 at most here): logits within the same
2e-3 + 1e-2 |y| bar as the kernels, and the same greedy continuation.  An
interleaved RoPE pairing in the oracle fails this on 150 of 512 logits, a
wrong GQA mapping (h % Hkv) on 504.  This pins
what the oracle's own kernel tests cannot: the block order, the RoPE pairing
(rotate-half, i with i + D/2), the GQA head mapping and the SwiGLU order."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
transformers = pytest.importorskip("transformers")

from silicongraph_b200 import armpack  # noqa: E402

CFG = armpack.llama_config(layers=2, hidden=128, heads=4, kv_heads=2, head_dim=32, ffn=256, vocab=512,
                           rope_theta=500000.0, max_pos=512)
GS = 32


def _hf_model(cfg, t):
    import oracle
    from transformers import LlamaConfig, LlamaForCausalLM
    H, Hq, Hkv, D, F, V = (cfg[k] for k in ("hidden_size", "num_heads", "num_kv_heads", "head_dim",
                                           "intermediate_size", "vocab_size"))
    hc = LlamaConfig(vocab_size=V, hidden_size=H, intermediate_size=F, num_hidden_layers=cfg["num_layers"],
                     num_attention_heads=Hq, num_key_value_heads=Hkv, head_dim=D, rms_norm_eps=cfg["rms_norm_eps"],
                     max_position_embeddings=cfg["max_position_embeddings"], tie_word_embeddings=False,
                     attention_bias=False, mlp_bias=False, hidden_act="silu",
                     rope_parameters={"rope_type": "default", "rope_theta": cfg["rope_theta"]})
    hc._attn_implementation = "eager"
    model = LlamaForCausalLM(hc).float().eval()

    def deq(name):  # [K, N] -> HF [N, K]
        B, S, Z = t[name + ".qweight"], t[name + ".scales"], t.get(name + ".zeros")
        K = 2 * B.shape[0]
        return oracle.dequant_int4_grouped(B, S, Z, K, B.shape[1], GS).T

    sd = {"model.embed_tokens.weight": t["embed_tokens"].astype(np.float32),
          "model.norm.weight": t["final_norm"].astype(np.float32), "lm_head.weight": deq("lm_head")}
    for i in range(cfg["num_layers"]):
        p, q = f"model.layers.{i}.", f"layers.{i}."
        qkv = deq(q + "qkv")
        sd[p + "self_attn.q_proj.weight"] = qkv[:Hq * D]
        sd[p + "self_attn.k_proj.weight"] = qkv[Hq * D:(Hq + Hkv) * D]
        sd[p + "self_attn.v_proj.weight"] = qkv[(Hq + Hkv) * D:]
        sd[p + "self_attn.o_proj.weight"] = deq(q + "o")
        gu = deq(q + "gate_up")
        sd[p + "mlp.gate_proj.weight"] = gu[:F]
        sd[p + "mlp.up_proj.weight"] = gu[F:]
        sd[p + "mlp.down_proj.weight"] = deq(q + "down")
        sd[p + "input_layernorm.weight"] = t[q + "input_norm"].astype(np.float32)
        sd[p + "post_attention_layernorm.weight"] = t[q + "post_norm"].astype(np.float32)
    missing, unexpected = model.load_state_dict({k: torch.from_numpy(np.ascontiguousarray(v, np.float32))
                                                 for k, v in sd.items()}, strict=False)
    assert not unexpected and all("rotary" in m for m in missing), (missing, unexpected)
    return model


def test_decoder_oracle_matches_hf_llama(oracle_mod):
    from oracle.decoder import DecoderOracle
    t = armpack.cuda_tensors(CFG, armpack.random_llama_weights(CFG, seed=4), group_size=GS)
    model = _hf_model(CFG, t)
    prompt = np.random.default_rng(8).integers(0, CFG["vocab_size"], 23)
    ref = DecoderOracle(CFG, t, group_size=GS)
    toks = [int(x) for x in prompt]
    for step in range(5):
        ids = prompt if step == 0 else [toks[-1]]
        got = ref.forward(ids)
        with torch.no_grad():
            want = model(torch.tensor([toks])).logits[0, -1].double().numpy()
        err = np.abs(got - want)
        assert np.all(err <= 2e-3 + 1e-2 * np.abs(want)), f"step {step}: max err {err.max():.3e}"
        assert int(np.argmax(got)) == int(np.argmax(want))
        toks.append(int(np.argmax(want)))


def test_fp32_decoder_oracle_matches_hf_llama_closely(oracle_mod):
    """The oracle's fp32 mode (the same restated kernels with no fp16 rounding
    between ops) against fp32 HF: only summation order differs, so the bar
    is 1e-4 absolute; any structural mismatch is orders of magnitude larger."""
    from oracle.decoder import DecoderOracle
    t = armpack.cuda_tensors(CFG, armpack.random_llama_weights(CFG, seed=5), group_size=GS)
    model = _hf_model(CFG, t)
    prompt = [int(x) for x in np.random.default_rng(9).integers(0, CFG["vocab_size"], 19)]
    ref = DecoderOracle(CFG, t, group_size=GS, precision="f32")
    toks = list(prompt)
    for step in range(4):
        got = ref.forward(prompt if step == 0 else [toks[-1]])
        with torch.no_grad():
            want = model(torch.tensor([toks])).logits[0, -1].double().numpy()
        err = np.abs(got - want)
        assert err.max() <= 1e-4, f"step {step}: max err {err.max():.3e}"
        toks.append(int(np.argmax(want)))
