"""Test infrastructure: the decoder composition oracle.

A CPU composition of the reference's own kernel semantics, restated in this
directory (matmul_int4_grouped_neon, rmsnorm / silu / rope, flash_attention_fp16),
over the tensors of a "cuda" package (silicongraph_b200.armpack): the same
Llama-style block order as the GPU session, with fp16 values at every op
boundary, as the reference's fp16 kernels produce them.  With precision="f32"
the same restated kernels run on fp32 values with no rounding between ops: the
exact-arithmetic yardstick against which the fp16 compositions' own rounding
noise is measured.  Only tests/ and bench.py's CPU baseline use it.  Parity pinned through the kernels it
composes (each checked against the reference's own outputs in
tests/test_oracle.py)."""
from __future__ import annotations

import numpy as np

from . import (DT_F16, DT_F32, flash_attention, matmul_int4_grouped, rmsnorm_f16, rmsnorm_f32, rope_f16, rope_f32,
               silu_f16, silu_f32)


def _f16(a):
    return np.asarray(a, np.float32).astype(np.float16)


class DecoderOracle:
    def __init__(self, cfg: dict, tensors: dict, group_size: int, precision: str = "f16"):
        assert precision in ("f16", "f32")
        self.c, self.t, self.gs = cfg, tensors, group_size
        self.f32 = precision == "f32"
        self.act = np.float32 if self.f32 else np.float16
        c = cfg
        self.H, self.Hq, self.Hkv, self.D = c["hidden_size"], c["num_heads"], c["num_kv_heads"], c["head_dim"]
        self.F, self.V, self.L = c["intermediate_size"], c["vocab_size"], c["num_layers"]
        self.eps, self.theta = float(c["rms_norm_eps"]), float(c["rope_theta"])
        self.k_cache = [np.zeros((self.Hkv, 0, self.D), self.act) for _ in range(self.L)]
        self.v_cache = [np.zeros((self.Hkv, 0, self.D), self.act) for _ in range(self.L)]
        self.pos = 0

    def _linear(self, name, x, c_dt=DT_F16):
        B = self.t[name + ".qweight"]
        S = self.t[name + ".scales"]
        Z = self.t.get(name + ".zeros")
        K = x.shape[1]
        N = B.shape[1]
        if self.f32:
            c_dt = DT_F32
        return matmul_int4_grouped(np.ascontiguousarray(x, self.act), B, S, Z, K, N, self.gs, M=x.shape[0],
                                   c_dt=c_dt)

    def _round(self, a):
        return np.asarray(a, np.float32) if self.f32 else _f16(a)

    def _add_norm(self, x, resid, w):
        h = self._round(x.astype(np.float32) + resid.astype(np.float32))
        if self.f32:
            w32 = np.asarray(w, np.float32)
            y = np.stack([rmsnorm_f32(np.ascontiguousarray(h[r]), w32, self.eps) for r in range(h.shape[0])])
        else:
            y = np.stack([rmsnorm_f16(h[r], w, self.eps) for r in range(h.shape[0])])
        return h, y

    def forward(self, ids) -> np.ndarray:
        """Processes tokens `ids` at the next positions; returns the fp32 logits of the last one."""
        ids = np.asarray(ids, np.int64)
        T, H, Hq, Hkv, D = len(ids), self.H, self.Hq, self.Hkv, self.D
        x = self.t["embed_tokens"][ids].astype(self.act)
        resid = np.zeros((T, H), self.act)
        rope = rope_f32 if self.f32 else rope_f16
        for layer in range(self.L):
            p = f"layers.{layer}."
            resid, xn = self._add_norm(x, resid, self.t[p + "input_norm"])
            qkv = self._linear(p + "qkv", xn)
            q = qkv[:, :Hq * D].reshape(T, Hq, D).copy()
            k = qkv[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D).copy()
            v = qkv[:, (Hq + Hkv) * D:].reshape(T, Hkv, D).copy()
            for t in range(T):
                for h in range(Hq):
                    q[t, h] = rope(q[t, h].copy(), self.pos + t, self.theta)
                for h in range(Hkv):
                    k[t, h] = rope(k[t, h].copy(), self.pos + t, self.theta)
            self.k_cache[layer] = np.concatenate([self.k_cache[layer], k.transpose(1, 0, 2)], axis=1)
            self.v_cache[layer] = np.concatenate([self.v_cache[layer], v.transpose(1, 0, 2)], axis=1)
            Q = np.ascontiguousarray(q.transpose(1, 0, 2)[None])          # [1, Hq, T, D]
            Kc = np.ascontiguousarray(self.k_cache[layer][None])           # [1, Hkv, S, D]
            Vc = np.ascontiguousarray(self.v_cache[layer][None])
            O = flash_attention(Q, Kc, Vc, causal=True, q_pos0=self.pos)   # [1, Hq, T, D]
            attn = np.ascontiguousarray(O[0].transpose(1, 0, 2).reshape(T, Hq * D))
            o = self._linear(p + "o", attn)
            resid, xn = self._add_norm(o, resid, self.t[p + "post_norm"])
            gu = self._linear(p + "gate_up", xn)
            g, u = gu[:, :self.F], gu[:, self.F:]
            if self.f32:
                act = silu_f32(np.ascontiguousarray(g)) * u
            else:
                act = _f16(silu_f16(np.ascontiguousarray(g)).astype(np.float32) * u.astype(np.float32))
            x = self._linear(p + "down", act)
        _, xn = self._add_norm(x[-1:], resid[-1:], self.t["final_norm"])
        self.pos += T
        return self._linear("lm_head", xn, c_dt=DT_F32)[0]

    def generate(self, prompt, n_new: int):
        """Greedy: returns (tokens, logits of each step)."""
        logits = [self.forward(prompt)]
        toks = [int(np.argmax(logits[-1]))]
        for _ in range(n_new - 1):
            logits.append(self.forward([toks[-1]]))
            toks.append(int(np.argmax(logits[-1])))
        return toks, logits
