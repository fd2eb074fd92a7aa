"""Tensor parallelism on the CPU: the shard plan that sg_session_create_tp cuts
the weights by (sg_tp_shard, host code of libsg_b200), and the arithmetic of
the sharded decoder layer restated with the oracle over two gloo ranks: the
column-split projections, the row-split projections summed by an all-reduce,
and the greedy token picked from the ranks' (max, log-sum-exp, index)
triples after an all-gather."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from silicongraph_b200 import armpack

LLAMA_1B = armpack.llama_config(layers=16, hidden=2048, heads=32, kv_heads=8, head_dim=64, ffn=8192, vocab=128256,
                                rope_theta=500000.0)
QWEN_7B = armpack.llama_config(layers=28, hidden=3584, heads=28, kv_heads=4, head_dim=128, ffn=18944, vocab=152064,
                               rope_theta=1000000.0)
SMALL = armpack.llama_config(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1008,
                             rope_theta=500000.0)


@pytest.mark.parametrize("cfg,gs", [(LLAMA_1B, 32), (QWEN_7B, 128), (SMALL, 32)], ids=["llama1b", "qwen7b", "small"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_partition_the_model(cfg, gs, world):
    from silicongraph_b200 import sdk
    H, Hkv, D = cfg["num_heads"], cfg["num_kv_heads"], cfg["head_dim"]
    F, V, G = cfg["intermediate_size"], cfg["vocab_size"], H // Hkv
    if world > 2 * Hkv or (F // gs) < world:
        pytest.skip("shape does not split this far")
    shards = [sdk.tp_shard(cfg, r, world, gs) for r in range(world)]
    # query heads, FFN columns and vocabulary columns: consecutive, disjoint, complete
    for lo, hi, total, unit in (("q_head0", "q_head1", H, 1), ("ffn0", "ffn1", F, gs), ("vocab0", "vocab1", V, 16)):
        assert shards[0][lo] == 0 and shards[-1][hi] == total
        for a, b in zip(shards, shards[1:]):
            assert a[hi] == b[lo]
        for s in shards:
            assert s[hi] > s[lo] and s[lo] % unit == 0
    for r, s in enumerate(shards):
        # every query head of the rank reads a kv head the rank holds
        assert all(s["kv_head0"] <= h // G < s["kv_head1"] for h in range(s["q_head0"], s["q_head1"]))
        # the output projection's rows start and end on quantisation groups
        assert (s["q_head0"] * D) % gs == 0 and (s["q_head1"] * D) % gs == 0
        if world <= Hkv:
            assert s["kv_head1"] - s["kv_head0"] == Hkv // world and s["kv_head0"] == r * Hkv // world
        else:
            assert s["kv_head1"] - s["kv_head0"] == 1 and s["kv_head0"] == r // (world // Hkv)


def test_unsplittable_shapes_are_refused():
    from silicongraph_b200 import sdk
    bad = dict(SMALL, num_heads=6, num_kv_heads=3)
    with pytest.raises(sdk.ArmError) as e:
        sdk.tp_shard(bad, 0, 2, 32)
    assert e.value.status == -4
    with pytest.raises(sdk.ArmError):
        sdk.tp_shard(dict(SMALL, vocab_size=1000), 0, 2, 32)  # vocabulary not on 16 columns
    with pytest.raises(sdk.ArmError):
        sdk.tp_shard(SMALL, 2, 2, 32)                          # rank outside the group


# ----------------------------------------------------------------------------- two gloo ranks
def _layer_tensors(oracle, cfg, gs, seed=3):
    rng = np.random.default_rng(seed)
    H, D, Hq, Hkv, F, V = (cfg["hidden_size"], cfg["head_dim"], cfg["num_heads"], cfg["num_kv_heads"],
                           cfg["intermediate_size"], cfg["vocab_size"])
    t = {}
    for name, K, N in (("qkv", H, (Hq + 2 * Hkv) * D), ("o", Hq * D, H), ("gate_up", H, 2 * F), ("down", F, H),
                       ("lm_head", H, V)):
        W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
        t[name] = (K, N) + tuple(oracle.quantize_int4_grouped(W, gs))
    return t


def _cols(q, ranges):
    B, S, Z = q
    pick = lambda a: np.ascontiguousarray(np.concatenate([a[:, c0:c1] for c0, c1 in ranges], axis=1))  # noqa: E731
    return pick(B), pick(S), pick(Z)


def _rows(q, r0, r1, gs):
    B, S, Z = q
    return (np.ascontiguousarray(B[r0 // 2:r1 // 2]), np.ascontiguousarray(S[r0 // gs:r1 // gs]),
            np.ascontiguousarray(Z[r0 // gs:r1 // gs]))


def _rank_main(rank, world, port, cfg, gs, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle
        from silicongraph_b200 import sdk
        oracle.lib()
        F32 = oracle.DT_F32
        mm = lambda x, q, K, N: oracle.matmul_int4_grouped(x, *q, K, N, gs, M=x.shape[0], c_dt=F32)  # noqa: E731
        H, D, Hq, Hkv, F, V = (cfg["hidden_size"], cfg["head_dim"], cfg["num_heads"], cfg["num_kv_heads"],
                               cfg["intermediate_size"], cfg["vocab_size"])
        t = _layer_tensors(oracle, cfg, gs)
        s = sdk.tp_shard(cfg, rank, world, gs)
        rng = np.random.default_rng(11)
        x = rng.standard_normal((3, H)).astype(np.float32)
        got = {}
        # column split: q|k|v of the rank's heads, gate|up of its FFN columns, its vocabulary columns
        q0, q1, k0, k1 = s["q_head0"], s["q_head1"], s["kv_head0"], s["kv_head1"]
        cq = [(q0 * D, q1 * D), ((Hq + k0) * D, (Hq + k1) * D), ((Hq + Hkv + k0) * D, (Hq + Hkv + k1) * D)]
        K, N = t["qkv"][:2]
        local = mm(x, _cols(t["qkv"][2:], cq), K, sum(b - a for a, b in cq))
        full = mm(x, t["qkv"][2:], K, N)
        got["qkv_cols"] = float(np.abs(local - np.concatenate([full[:, a:b] for a, b in cq], 1)).max())
        # row split + all-reduce: output projection (rows of the rank's heads), down (its FFN rows)
        for name, r0, r1, xin_dim in (("o", q0 * D, q1 * D, Hq * D), ("down", s["ffn0"], s["ffn1"], F)):
            K, N = t[name][:2]
            xin = rng.standard_normal((3, xin_dim)).astype(np.float32)
            part = mm(np.ascontiguousarray(xin[:, r0:r1]), _rows(t[name][2:], r0, r1, gs), r1 - r0, N)
            tot = torch.from_numpy(part.copy())
            dist.all_reduce(tot)
            want = mm(xin, t[name][2:], K, N)
            got[name] = float((np.abs(tot.numpy() - want) / (1e-3 + np.abs(want))).max())
        # vocabulary split: local argmax / log-prob, all-gather of the triples, global pick
        K, N = t["lm_head"][:2]
        xl = rng.standard_normal((1, H)).astype(np.float32)
        logits = mm(xl, _cols(t["lm_head"][2:], [(s["vocab0"], s["vocab1"])]), K, s["vocab1"] - s["vocab0"])[0]
        i = int(np.argmax(logits))
        m = float(logits[i])
        lse = m + float(np.log(np.exp(logits.astype(np.float64) - m).sum()))
        mine = torch.tensor([m, lse, float(s["vocab0"] + i)], dtype=torch.float64)
        allt = [torch.zeros(3, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(allt, mine)
        trip = torch.stack(allt).numpy()
        best = int(np.argmax(trip[:, 0]))  # first rank among equal maxima
        Lmax = trip[:, 1].max()
        gl = Lmax + np.log(np.exp(trip[:, 1] - Lmax).sum())
        full_logits = mm(xl, t["lm_head"][2:], K, N)[0].astype(np.float64)
        want_lse = full_logits.max() + np.log(np.exp(full_logits - full_logits.max()).sum())
        got["token_ok"] = int(trip[best, 2]) == int(np.argmax(full_logits))
        got["logprob_err"] = float(abs((trip[best, 0] - gl) - (full_logits.max() - want_lse)))
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.array([got], dtype=object), allow_pickle=True)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cfg,gs", [(SMALL, 32), (dict(SMALL, num_heads=8, num_kv_heads=2, hidden_size=512), 64)],
                         ids=["small", "gqa4"])
def test_sharded_layer_matches_whole_layer_on_two_gloo_ranks(tmp_path, cfg, gs):
    import socket
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    mp.start_processes(_rank_main, args=(2, port, cfg, gs, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        got = np.load(tmp_path / f"rank{r}.npy", allow_pickle=True)[0]
        assert got["qkv_cols"] == 0.0           # a column shard is exactly the whole kernel's columns
        assert got["o"] < 1e-3 and got["down"] < 1e-3  # row shards sum to the whole (fp32 order only)
        assert got["token_ok"] and got["logprob_err"] < 1e-5
