"""Writes .armpack packages with a "cuda" graph entry that libsg_b200's SDK
runs (armpack_load / armpack_select_graph / armgraph_create_session).

Container and manifest follow the reference's package writer
(compiler/lib/package/package_generator.cpp:104-211, 618-695: a ZIP holding
manifest.json with "arch", "graphs", "kernels", "weights", plus graph files and
weight files, weights stored uncompressed).  The reference never writes
quantized bytes (its exporter dumps raw fp16 without an index,
python/armcc/graph_exporter.py:528-538), so the "cuda" profile adds:
  graphs/<id>.json                     "sg-cuda-decoder": model hyperparameters,
                                       quantization, weight file and index
  weights/weights_int4_g<gs>.bin       4096-aligned tensors (stored)
  weights/weights_int4_g<gs>.index.json  name -> offset, bytes, dtype, shape
Linears use the reference's INT4 layout (compiler/kernels/cpu/matmul_neon.h:
113-147): qweight u8 [ceil(K/2), N] (low nibble = even k), scales fp16
[ceil(K/gs), N], zeros int8 [ceil(K/gs), N] in [-8, 7], with the zero-point
convention of python/armcc/calibration.py:37-50 applied per (group, column).
Hugging Face nn.Linear weights are [N_out, K_in] and are transposed to [K, N];
q/k/v and gate/up are concatenated along N.
"""
from __future__ import annotations

import io
import json
import os
import tempfile
import time
import zipfile

import numpy as np

ALIGN = 4096
GRAPH_FORMAT = "sg-cuda-decoder"


# ----------------------------------------------------------------------------- quantization
def quantize_int4_grouped(w_kn: np.ndarray, group_size: int, symmetric: bool = False):
    """[K, N] fp32 -> (qweight u8 [ceil(K/2), N], scales f16 [G, N], zeros i8 [G, N] or None).

    Asymmetric: scale = (max - min) / 15, zero = round(-8 - min / scale)
    clamped to [-8, 7] (calibration.py:37-50; Python round = half to even);
    symmetric: scale = absmax / 7, no zeros.  q = clamp(rint(w / scale) + zero,
    -8, 7), stored as q + 8.  Scales are computed in double and rounded to fp16;
    the division uses the fp16 scale in fp32."""
    W = np.ascontiguousarray(w_kn, dtype=np.float32)
    K, N = W.shape
    gs = group_size if group_size > 0 else 128
    G = (K + gs - 1) // gs
    pad = G * gs - K
    Wp = np.pad(W, ((0, pad), (0, 0))) if pad else W
    Wg = Wp.reshape(G, gs, N)
    valid = np.ones((G, gs, 1), bool)
    if pad:
        valid[-1, gs - pad:, 0] = False
    big = np.float32(np.inf)
    mn = np.where(valid, Wg, big).min(axis=1)           # [G, N]
    mx = np.where(valid, Wg, -big).max(axis=1)
    amax = np.where(valid, np.abs(Wg), 0).max(axis=1)
    if symmetric:
        sd = np.where(amax > 0, amax.astype(np.float64) / 7.0, 1.0)
        zp = np.zeros((G, N), np.int32)
    else:
        rng = mx.astype(np.float64) - mn.astype(np.float64)
        sd = np.where(rng > 0, rng / 15.0, 1.0)
        with np.errstate(divide="ignore", invalid="ignore"):
            zp = np.where(rng > 0, np.rint(-8.0 - mn.astype(np.float64) / sd), 0.0)
        zp = np.clip(zp, -8, 7).astype(np.int32)
    s16 = sd.astype(np.float32).astype(np.float16)
    s32 = s16.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.where(s32[:, None, :] > 0, np.rint(Wg / s32[:, None, :]), np.float32(0))
    q = np.clip(r + zp[:, None, :].astype(np.float32), -8, 7).astype(np.int8).reshape(G * gs, N)[:K]
    nib = (q.astype(np.int16) + 8).astype(np.uint8) & 0x0F
    if K % 2:
        nib = np.concatenate([nib, np.zeros((1, N), np.uint8)], axis=0)
    B = (nib[0::2] | (nib[1::2] << 4)).astype(np.uint8)
    return B, s16, (None if symmetric else zp.astype(np.int8))


# ----------------------------------------------------------------------------- model description
def llama_config(layers=16, hidden=2048, heads=32, kv_heads=8, head_dim=64, ffn=8192, vocab=128256,
                 rope_theta=500000.0, rms_eps=1e-5, max_pos=131072):
    """Llama-style decoder hyperparameters (defaults: Llama-3.2-1B shape)."""
    return dict(num_layers=layers, hidden_size=hidden, num_heads=heads, num_kv_heads=kv_heads, head_dim=head_dim,
                intermediate_size=ffn, vocab_size=vocab, rope_theta=rope_theta, rms_norm_eps=rms_eps,
                max_position_embeddings=max_pos)


def random_llama_weights(cfg: dict, seed: int = 0, std: float = 0.02, dtype=np.float32) -> dict:
    """Hugging Face-named weights, N(0, std) for matrices and 1 + N(0, std) for norms."""
    rng = np.random.default_rng(seed)
    H, V, F = cfg["hidden_size"], cfg["vocab_size"], cfg["intermediate_size"]
    Hq, Hkv, D = cfg["num_heads"], cfg["num_kv_heads"], cfg["head_dim"]

    def mat(n_out, k_in):
        return (rng.standard_normal((n_out, k_in), dtype=np.float32) * std).astype(dtype)

    def norm(n):
        return (1.0 + rng.standard_normal(n, dtype=np.float32) * std).astype(dtype)

    w = {"model.embed_tokens.weight": mat(V, H)}
    for i in range(cfg["num_layers"]):
        p = f"model.layers.{i}."
        w[p + "input_layernorm.weight"] = norm(H)
        w[p + "self_attn.q_proj.weight"] = mat(Hq * D, H)
        w[p + "self_attn.k_proj.weight"] = mat(Hkv * D, H)
        w[p + "self_attn.v_proj.weight"] = mat(Hkv * D, H)
        w[p + "self_attn.o_proj.weight"] = mat(H, Hq * D)
        w[p + "post_attention_layernorm.weight"] = norm(H)
        w[p + "mlp.gate_proj.weight"] = mat(F, H)
        w[p + "mlp.up_proj.weight"] = mat(F, H)
        w[p + "mlp.down_proj.weight"] = mat(H, F)
    w["model.norm.weight"] = norm(H)
    w["lm_head.weight"] = mat(V, H)
    return w


def cuda_tensors(cfg: dict, weights: dict, group_size: int = 32, symmetric: bool = False,
                 quantize=quantize_int4_grouped):
    """HF-named weights -> the "cuda" profile's tensors (name -> array), in file order."""
    out = {}
    f16 = lambda a: np.ascontiguousarray(a, dtype=np.float16)  # noqa: E731

    def linear(name, *hf_mats):
        w_kn = np.concatenate([np.asarray(m, np.float32).T for m in hf_mats], axis=1)
        B, S, Z = quantize(w_kn, group_size, symmetric)
        out[name + ".qweight"] = B
        out[name + ".scales"] = S
        if Z is not None:
            out[name + ".zeros"] = Z

    out["embed_tokens"] = f16(weights["model.embed_tokens.weight"])
    for i in range(cfg["num_layers"]):
        p, q = f"model.layers.{i}.", f"layers.{i}."
        out[q + "input_norm"] = f16(weights[p + "input_layernorm.weight"])
        out[q + "post_norm"] = f16(weights[p + "post_attention_layernorm.weight"])
        linear(q + "qkv", weights[p + "self_attn.q_proj.weight"], weights[p + "self_attn.k_proj.weight"],
               weights[p + "self_attn.v_proj.weight"])
        linear(q + "o", weights[p + "self_attn.o_proj.weight"])
        linear(q + "gate_up", weights[p + "mlp.gate_proj.weight"], weights[p + "mlp.up_proj.weight"])
        linear(q + "down", weights[p + "mlp.down_proj.weight"])
    out["final_norm"] = f16(weights["model.norm.weight"])
    lm = weights.get("lm_head.weight", weights["model.embed_tokens.weight"])  # tied embeddings
    linear("lm_head", lm)
    return out


# ----------------------------------------------------------------------------- writer
def write_package(path: str, cfg: dict, tensors: dict, *, model_id: str = "synthetic/llama-style",
                  group_size: int = 32, symmetric: bool = False, max_context=4096,
                  max_prefill_chunk: int = 512, as_zip: bool = True, graph_conditions=None) -> str:
    """Writes a package (ZIP file, or a directory with the same layout) with
    execution_backend "cuda" graph entries sharing one weight file: one graph
    per context length in `max_context` (an int or a list).  graph_conditions
    (a list of dicts, one per graph) overrides manifest fields of the entries,
    e.g. thermal_state / latency_mode / estimated_tpot_ms.  Returns `path`."""
    contexts = [max_context] if isinstance(max_context, int) else list(max_context)
    conds = list(graph_conditions) if graph_conditions else [{} for _ in contexts]
    assert len(conds) == len(contexts)
    wid = f"weights_int4_g{group_size}"
    wpath, ipath = f"weights/{wid}.bin", f"weights/{wid}.index.json"
    index, offset = {}, 0
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr)
        offset = (offset + ALIGN - 1) // ALIGN * ALIGN
        index[name] = {"offset": offset, "bytes": int(arr.nbytes), "dtype": arr.dtype.name,
                       "shape": list(arr.shape)}
        offset += arr.nbytes
    total = (offset + ALIGN - 1) // ALIGN * ALIGN
    H, L = cfg["hidden_size"], cfg["num_layers"]
    kv_per_token = 2 * L * cfg["num_kv_heads"] * cfg["head_dim"] * 2
    graphs, entries = {}, []
    for gi, (ctx, cond) in enumerate(zip(contexts, conds)):
        gid = f"cuda_int4_g{group_size}_ctx{ctx}" + (f"_{gi}" if len(contexts) > 1 else "")
        gpath = f"graphs/{gid}.json"
        graphs[gpath] = {
            "format": GRAPH_FORMAT, "version": 1,
            "model": {"family": "llama_style", **{k: cfg[k] for k in (
                "num_layers", "hidden_size", "num_heads", "num_kv_heads", "head_dim", "intermediate_size",
                "vocab_size", "rope_theta", "rms_norm_eps")}},
            "quant": {"scheme": "int4_grouped", "group_size": group_size, "zero_point": not symmetric,
                      "lm_head": "int4"},
            "weights": wid, "tensor_index": ipath,
            "max_context": ctx, "max_prefill_chunk": max_prefill_chunk,
        }
        entries.append({
            "index": gi, "id": gid, "path": gpath, "soc_name": "nvidia_b200", "quant_dtype": f"int4_g{group_size}",
            "memory_budget_mb": 0, "context_length": ctx, "thermal_state": "nominal",
            "latency_mode": "interactive", "execution_backend": "cuda", "estimated_ttft_ms": 0.0,
            "estimated_tpot_ms": 0.0, "peak_memory_bytes": total + kv_per_token * ctx,
            "weight_bytes": total, "activation_bytes": 0, "kv_cache_bytes": kv_per_token * ctx,
            "kv_bytes_per_token": kv_per_token, "kernel_ids": [], **cond})
    manifest = {
        "armpack_version": "1.0", "compiler_version": "sg-b200-0.1.0", "model_id": model_id,
        "model_family": "llama_style", "created_at": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
        "arch": {"num_layers": L, "hidden_size": H, "num_heads": cfg["num_heads"],
                 "num_kv_heads": cfg["num_kv_heads"], "vocab_size": cfg["vocab_size"],
                 "max_position_embeddings": cfg.get("max_position_embeddings", max(contexts))},
        "graphs": entries,
        "kernels": [],
        "weights": [{"id": wid, "path": wpath, "dtype": "int4", "size_bytes": total, "mmap_safe": True,
                     "page_alignment": ALIGN}],
        "tokenizer_path": "tokenizer/", "selector_wasm_path": "selector.wasm",
        "runtime_config_path": "runtime_config.json", "memory_maps_path": "memory_maps/",
    }
    runtime_config = {"temperature": 1.0, "top_p": 0.9, "top_k": 50, "max_new_tokens": 512,
                      "bos_token_id": 1, "eos_token_id": 2, "pad_token_id": 0}

    def weight_bytes(fh):
        pos = 0
        for name, arr in tensors.items():
            off = index[name]["offset"]
            if off > pos:
                fh.write(b"\0" * (off - pos))
                pos = off
            b = np.ascontiguousarray(arr).tobytes()
            fh.write(b)
            pos += len(b)
        if total > pos:
            fh.write(b"\0" * (total - pos))

    texts = {"manifest.json": json.dumps(manifest, indent=2),
             **{gp: json.dumps(g, indent=2) for gp, g in graphs.items()},
             ipath: json.dumps({"tensors": index}), "runtime_config.json": json.dumps(runtime_config, indent=2)}
    if not as_zip:
        os.makedirs(os.path.join(path, "weights"), exist_ok=True)
        os.makedirs(os.path.join(path, "graphs"), exist_ok=True)
        for name, text in texts.items():
            with open(os.path.join(path, name), "w") as fh:
                fh.write(text)
        with open(os.path.join(path, wpath), "wb") as fh:
            weight_bytes(fh)
        return path
    with tempfile.TemporaryDirectory() as td:
        tmpw = os.path.join(td, "w.bin")
        with open(tmpw, "wb") as fh:
            weight_bytes(fh)
        with zipfile.ZipFile(path, "w", compression=zipfile.ZIP_DEFLATED, allowZip64=True) as zf:
            for name, text in texts.items():
                zf.writestr(name, text)
            zf.write(tmpw, wpath, compress_type=zipfile.ZIP_STORED)
    return path


def pack_random_llama(path: str, cfg: dict | None = None, seed: int = 0, **kw) -> tuple[str, dict, dict]:
    """Random-init Llama-style model -> package.  Returns (path, cfg, cuda tensors)."""
    cfg = cfg or llama_config()
    w = random_llama_weights(cfg, seed)
    gs, sym = kw.get("group_size", 32), kw.get("symmetric", False)
    t = cuda_tensors(cfg, w, group_size=gs, symmetric=sym)
    write_package(path, cfg, t, **kw)
    return path, cfg, t


def random_cuda_tensors_on_device(cfg: dict, seed: int = 0, group_size: int = 32, std: float = 0.02) -> dict:
    """The "cuda" profile's tensors of a random-init Llama-style model, drawn
    on the current CUDA device (N(0, std) matrices, 1 + N(0, std) norms) and
    packed there by the library's own INT4 packer (sg_quantize_int4_grouped,
    the same convention as quantize_int4_grouped); returned as host arrays in
    file order.  For models too large to draw and quantise on the host in
    reasonable time (the Llama-3.2-1B and Qwen2.5-7B shapes)."""
    import torch

    from . import _lib
    lib = _lib.load()
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    H, V, F = cfg["hidden_size"], cfg["vocab_size"], cfg["intermediate_size"]
    Hq, Hkv, D = cfg["num_heads"], cfg["num_kv_heads"], cfg["head_dim"]
    gs = group_size
    stream = torch.cuda.current_stream().cuda_stream

    def randn(*shape):
        return torch.randn(*shape, generator=g, device="cuda", dtype=torch.float32) * std

    def quant(K, N):
        w = randn(K, N)
        G = (K + gs - 1) // gs
        B = torch.empty(((K + 1) // 2, N), dtype=torch.uint8, device="cuda")
        S = torch.empty((G, N), dtype=torch.float16, device="cuda")
        Z = torch.empty((G, N), dtype=torch.int8, device="cuda")
        _lib.check(lib.sg_quantize_int4_grouped(w.data_ptr(), K, N, gs, 0, B.data_ptr(), S.data_ptr(),
                                                Z.data_ptr(), stream))
        return B.cpu().numpy(), S.cpu().numpy(), Z.cpu().numpy()

    t = {"embed_tokens": randn(V, H).half().cpu().numpy()}
    for i in range(cfg["num_layers"]):
        q = f"layers.{i}."
        t[q + "input_norm"] = (1 + randn(H)).half().cpu().numpy()
        t[q + "post_norm"] = (1 + randn(H)).half().cpu().numpy()
        for name, K, N in (("qkv", H, (Hq + 2 * Hkv) * D), ("o", Hq * D, H), ("gate_up", H, 2 * F), ("down", F, H)):
            B, S, Z = quant(K, N)
            t[q + name + ".qweight"], t[q + name + ".scales"], t[q + name + ".zeros"] = B, S, Z
    t["final_norm"] = (1 + randn(H)).half().cpu().numpy()
    t["lm_head.qweight"], t["lm_head.scales"], t["lm_head.zeros"] = quant(H, V)
    return t
