"""A tensor-parallel session over two GPUs (sg_session_create_tp): each rank
holds its shard of every linear; the row-split projections are summed by the
peer-memory all-reduce (decode) or NCCL (prefill, or everywhere with
SG_TP_P2P=0), and NCCL picks the greedy token across the vocabulary shards.  The gathered logits
and the tokens must match the decoder composition oracle like a one-GPU
session does (|got - want| <= 2e-3 + 1e-2 |want|), and every rank must emit
the same tokens.  Skipped with fewer than two GPUs."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from silicongraph_b200 import armpack

pytestmark = pytest.mark.gpu

SMALL = armpack.llama_config(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1008,
                             rope_theta=500000.0, max_pos=4096)
# eight ranks need a query head each
SMALL8 = armpack.llama_config(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=64, ffn=1024, vocab=1008,
                              rope_theta=500000.0, max_pos=4096)
RTOL, ATOL = 1e-2, 2e-3
STEPS = 4


def _worker(rank, world, uid, path, prompt, batch, p2p, out_dir):
    os.environ["SG_DEVICE"] = str(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["SG_TP_P2P"] = "1" if p2p else "0"
    torch.cuda.set_device(rank)
    from silicongraph_b200 import sdk
    with sdk.Package(path) as pkg:
        g = pkg.select(context_length=prompt.shape[1] + STEPS + 4)
        with g.session(tp=(rank, world, uid), batch=batch) as s:
            lo, hi = s.vocab_range
            if batch == 1:
                s.prefill(prompt[0])
                logits = [s.last_logits()]
                toks = [[s.decode().next_token_id]]  # predicted by the prompt
                for _ in range(STEPS):
                    toks.append([s.decode().next_token_id])
                    logits.append(s.last_logits())
            else:
                s.batch_prefill(prompt)
                logits = [s.last_logits()]
                toks = [s.batch_decode()]
                for _ in range(STEPS):
                    toks.append(s.batch_decode())
                    logits.append(s.last_logits())
    # logits [steps + 1, batch, shard], toks [steps + 1, batch]
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), logits=np.stack(logits).reshape(STEPS + 1, batch, hi - lo),
             toks=np.array(toks), lo=lo, hi=hi)


@pytest.mark.parametrize("world,batch,p2p", [(2, 1, True), (2, 2, True), (2, 2, False), (4, 1, True), (4, 2, False),
                                             (8, 1, True)],
                         ids=["peer-allreduce", "batch2-peer-allreduce", "batch2-nccl", "world4-peer-allreduce",
                              "world4-batch2-nccl", "world8-peer-allreduce"])
def test_tp_session_matches_decoder_oracle(sg, oracle_mod, tmp_path, world, batch, p2p):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from oracle.decoder import DecoderOracle
    from silicongraph_b200 import sdk
    cfg = SMALL8 if world > 4 else SMALL
    w = armpack.random_llama_weights(cfg, seed=4)
    t = armpack.cuda_tensors(cfg, w, group_size=32)
    path = armpack.write_package(str(tmp_path / "tp.armpack"), cfg, t, max_context=256, max_prefill_chunk=64)
    prompt = np.random.default_rng(9).integers(0, cfg["vocab_size"], (batch, 90)).astype(np.int32)  # 2 chunks
    uid = sdk.tp_unique_id()
    mp.start_processes(_worker, args=(world, uid, path, prompt, batch, p2p, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    ranks = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    assert [int(r["lo"]) for r in ranks] == sorted(int(r["lo"]) for r in ranks)
    assert int(ranks[-1]["hi"]) == cfg["vocab_size"]
    for r in ranks[1:]:
        assert np.array_equal(r["toks"], ranks[0]["toks"])  # every rank emits the same tokens
    logits = np.concatenate([r["logits"] for r in ranks], axis=2)  # [steps + 1, batch, vocab]
    toks = ranks[0]["toks"]

    def close(got, want):
        err = np.abs(got - want)
        bad = err > ATOL + RTOL * np.abs(want)
        assert not bad.any(), f"{bad.sum()} / {bad.size} logits outside tolerance; max err {err.max():.3e}"

    def check_token(tok, want):
        top = np.sort(want)[-2:]
        if top[1] - top[0] > ATOL + RTOL * abs(top[1]):
            assert tok == int(np.argmax(want))

    for b in range(batch):
        ref = DecoderOracle(cfg, t, group_size=32)
        want = ref.forward(prompt[b])
        close(logits[0, b], want)
        check_token(int(toks[0][b]), want)
        for i in range(STEPS):
            want = ref.forward([int(toks[i][b])])
            close(logits[i + 1, b], want)
            check_token(int(toks[i + 1][b]), want)



# ------------------------------------------------------------------ failure handling on two GPUs
def _leave_worker(rank, world, uid, path, out_dir):
    """After two steps rank 1 announces on the host (a marker file) that it
    leaves; rank 0 learns it before its next launch, aborts its session and
    gets a clean refusal.  Both ranks then leave in order (markers), so no rank
    frees memory the other still maps, and no collective is in flight when a
    rank goes."""
    import time
    os.environ["SG_DEVICE"] = str(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["SG_TP_P2P"] = "1"
    torch.cuda.set_device(rank)
    from silicongraph_b200 import sdk
    marker = lambda name: os.path.join(out_dir, name)  # noqa: E731

    def wait_for(name, limit=120.0):
        t0 = time.time()
        while not os.path.exists(marker(name)):
            if time.time() - t0 > limit:
                raise TimeoutError(name)
            time.sleep(0.01)

    result = {}
    with sdk.Package(path) as pkg:
        with pkg.select(context_length=64).session(tp=(rank, world, uid)) as s:
            s.prefill(np.arange(20, dtype=np.int32) % SMALL["vocab_size"])
            s.decode()
            s.decode()
            if rank == 1:
                open(marker("leaving"), "w").close()
                wait_for("rank0_done")            # rank 0 has aborted and closed its mappings
                s.abort("leaving")
            else:
                t0 = time.time()
                wait_for("leaving")               # learned on the host, before the next launch
                s.abort("rank 1 left")
                try:
                    s.decode()
                    result["status"] = 0
                except sdk.ArmError as e:
                    result["status"], result["msg"] = e.status, str(e)
                result["seconds"] = time.time() - t0
                open(marker("rank0_done"), "w").close()
                wait_for("rank1_done")
        if rank == 1:
            open(marker("rank1_done"), "w").close()
    np.save(os.path.join(out_dir, f"leave{rank}.npy"), np.array([result], dtype=object), allow_pickle=True)


def test_tp_rank_leaving_between_steps(sg, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from silicongraph_b200 import sdk
    t = armpack.cuda_tensors(SMALL, armpack.random_llama_weights(SMALL, seed=4), group_size=32)
    path = armpack.write_package(str(tmp_path / "tp.armpack"), SMALL, t, max_context=256, max_prefill_chunk=64)
    mp.start_processes(_leave_worker, args=(2, sdk.tp_unique_id(), path, str(tmp_path)), nprocs=2,
                       join=True, start_method="spawn")
    r0 = np.load(tmp_path / "leave0.npy", allow_pickle=True)[0]
    assert r0["status"] == -5, r0
    assert "rank 1 left" in r0["msg"] and r0["seconds"] < 10
