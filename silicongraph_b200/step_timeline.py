"""Phase timeline of the persistent decode-step kernel (decode_step.cu).

Builds a random-init Llama-style INT4 model (the Llama-3.2-1B shape by
default), prefills a prompt, runs decode steps through the kernel with its
timeline on (sg_session_step_trace) and prints, per phase kind, the median
over layers of: the slowest CTA's time from the previous grid barrier's
release to its arrival at the next one, the spread of arrivals, and the
release latency (last arrival to the first / last release); then, for a few
phases, where the time went inside them (activation staging, waiting for
weight chunks, the chunks themselves).

  python -m silicongraph_b200.step_timeline [--layers 16 --prompt 512 --steps 3]

Steps run eagerly (SG_DECODE_GRAPH=0): a captured graph keeps the timeline
pointer it was captured with."""
from __future__ import annotations

import argparse
import os
import tempfile

import numpy as np

PHASES = ["q|k|v", "attention", "o", "gate|up", "down"]


def run(layers=16, hidden=2048, heads=32, kv_heads=8, head_dim=64, ffn=8192, vocab=128256, prompt=512, steps=3,
        seed=11):
    os.environ["SG_DECODE_GRAPH"] = "0"
    import torch

    from silicongraph_b200 import armpack, kernels, sdk
    torch.cuda.set_device(0)
    kernels.set_tuning("sdk.decode_step_kernel", 1)
    cfg = armpack.llama_config(layers=layers, hidden=hidden, heads=heads, kv_heads=kv_heads, head_dim=head_dim,
                               ffn=ffn, vocab=vocab)
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "model")
        t = armpack.random_cuda_tensors_on_device(cfg, seed=seed, group_size=32)
        armpack.write_package(path, cfg, t, group_size=32, max_context=prompt + steps + 16, as_zip=False)
        ids = np.random.default_rng(seed).integers(0, vocab, prompt).astype(np.int32)
        with sdk.Package(path) as pkg:
            with pkg.select(context_length=prompt + steps + 8).session() as s:
                s.prefill(ids)
                s.decode()
                s.decode()
                on, why = s.step_kernel
                if not on:
                    raise SystemExit(f"the decode-step kernel is not in use: {why}")
                s.step_trace(True)
                for _ in range(steps):
                    s.decode()
                tr = s.step_trace(False)
    kernels.set_tuning("sdk.decode_step_kernel", 0)
    return tr, layers


def report(tr, layers):
    nbar = 5 * layers
    start = tr[:, 0]
    base = start.min()
    arr = tr[:, 1:1 + 2 * nbar:2]
    rel = tr[:, 2:2 + 2 * nbar:2]
    end = tr[:, 1 + 2 * nbar]
    print(f"kernel: {(end.max() - base) / 1e3:.1f} us from the first CTA's start to the last CTA's end")
    rows = {}
    prev = start
    for k in range(nbar + 1):
        a = arr[:, k] if k < nbar else end
        slowest = (a - prev).max() / 1e3
        if k < nbar:
            spread = (a.max() - a.min()) / 1e3
            lat = ((rel[:, k].min() - a.max()) / 1e3, (rel[:, k].max() - a.max()) / 1e3)
            prev = rel[:, k]
        else:
            spread, lat = 0.0, (0.0, 0.0)
        name = PHASES[k % 5] if k < nbar else "LM head + pick"
        rows.setdefault(name, []).append((slowest, spread, lat[0], lat[1]))
    print(f"{'phase':16s} {'n':>3s} {'slowest CTA us':>15s} {'arrival spread':>15s} {'release us':>14s}")
    total = 0.0
    for name, v in rows.items():
        v = np.array(v)
        med = np.median(v, axis=0)
        total += v[:, 0].sum() + v[:, 3].sum()
        print(f"{name:16s} {len(v):3d} {med[0]:15.2f} {med[1]:15.2f} {med[2]:6.2f}..{med[3]:6.2f}")
    print(f"sum of slowest-CTA phase times and release latencies: {total:.1f} us")
    print("inside phases of layer 1 (medians over CTAs with work; us):")
    for ph in (5, 7, 8, 9, nbar):
        stage = tr[:, 200 + ph]
        have = stage > 0
        if not have.any():
            continue
        pstart = rel[:, ph - 1]
        a = arr[:, ph] if ph < nbar else end
        name = PHASES[ph % 5] if ph < nbar else "LM head"
        print(f"  {name:10s} staging {np.median((stage - pstart)[have]) / 1e3:6.2f}  "
              f"warp 0 waiting for weight chunks {np.median(tr[have, 300 + ph]) / 1e3:6.2f}  "
              f"staged -> arrival {np.median((a - stage)[have]) / 1e3:6.2f}")
    print(f"producer: waited {np.median(tr[:, 400]) / 1e3:.1f} us for free ring slots (median over CTAs)")


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--layers", type=int, default=16)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--steps", type=int, default=3)
    args = ap.parse_args()
    tr, layers = run(layers=args.layers, prompt=args.prompt, steps=args.steps)
    report(tr, layers)


if __name__ == "__main__":
    main()
