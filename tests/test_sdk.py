"""The armcc SDK surface on the CPU: packages written by silicongraph_b200.armpack
load through libsg_b200's armpack_load (ZIP and directory form), the packer's
INT4 bytes equal the oracle's, and the calls that need a GPU fail cleanly."""
import json
import os
import zipfile

import numpy as np
import pytest

from silicongraph_b200 import armpack

SMALL = armpack.llama_config(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000,
                             rope_theta=500000.0, max_pos=4096)


@pytest.mark.parametrize("K,N,gs,sym", [(256, 64, 32, False), (130, 48, 32, False), (127, 33, 16, True),
                                        (512, 40, 128, False), (96, 20, 64, True)])
def test_packer_quantizer_matches_oracle(oracle_mod, K, N, gs, sym):
    rng = np.random.default_rng(K + N)
    W = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    W[:, 0] = 0.0            # constant column: scale falls back to 1, zero to 0
    B, S, Z = armpack.quantize_int4_grouped(W, gs, sym)
    B0, S0, Z0 = oracle_mod.quantize_int4_grouped(W, gs, sym)
    assert np.array_equal(B, B0)
    assert np.array_equal(S.view(np.uint16), S0.view(np.uint16))
    assert (Z is None and Z0 is None) or np.array_equal(Z, Z0)


@pytest.fixture(scope="module")
def small_packages(tmp_path_factory):
    d = tmp_path_factory.mktemp("pkg")
    w = armpack.random_llama_weights(SMALL, seed=1)
    t = armpack.cuda_tensors(SMALL, w, group_size=32)
    z = armpack.write_package(str(d / "small.armpack"), SMALL, t, max_context=1024, max_prefill_chunk=128)
    dd = armpack.write_package(str(d / "small_dir"), SMALL, t, max_context=1024, max_prefill_chunk=128, as_zip=False)
    return z, dd, t


def test_package_layout(small_packages):
    z, _, t = small_packages
    with zipfile.ZipFile(z) as zf:
        names = set(zf.namelist())
        m = json.loads(zf.read("manifest.json"))
        info = {i.filename: i for i in zf.infolist()}
    assert {"manifest.json", "weights/weights_int4_g32.bin", "weights/weights_int4_g32.index.json"} <= names
    assert info["weights/weights_int4_g32.bin"].compress_type == zipfile.ZIP_STORED
    assert m["graphs"][0]["execution_backend"] == "cuda"
    assert m["arch"]["num_layers"] == 2 and m["arch"]["vocab_size"] == 1000
    for name in ("layers.0.qkv.qweight", "layers.1.gate_up.scales", "lm_head.zeros"):
        assert name in t
    assert t["layers.0.qkv.qweight"].shape == (128, (4 + 2 * 2) * 64)


@pytest.mark.parametrize("form", ["zip", "dir"])
def test_armpack_load_and_inspect(small_packages, form):
    from silicongraph_b200 import sdk
    path = small_packages[0] if form == "zip" else small_packages[1]
    with sdk.Package(path) as pkg:
        assert pkg.num_graphs() == 1
        info = pkg.info()
        assert info["num_layers"] == 2 and info["hidden_size"] == 256 and info["vocab_size"] == 1000
        assert info["model_family"] == "llama_style" and info["num_weight_files"] == 1
        g = pkg.graph(0)
        assert "cuda" in g.description and "int4_g32" in g.description
        assert g.peak_memory_bytes > 0
        with pytest.raises(sdk.ArmError):
            pkg.graph(5)


def test_gpu_calls_fail_cleanly_without_a_device(small_packages):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from silicongraph_b200 import sdk
    with sdk.Package(small_packages[0]) as pkg:
        with pytest.raises(sdk.ArmError, match="no CUDA device"):
            pkg.select()
        with pytest.raises(sdk.ArmError):
            pkg.graph(0).session()


def test_malformed_packages(tmp_path):
    from silicongraph_b200 import sdk
    with pytest.raises(sdk.ArmError, match="not found"):
        sdk.Package(str(tmp_path / "missing.armpack"))
    bad = tmp_path / "bad.armpack"
    bad.write_bytes(b"not a zip at all, just bytes" * 10)
    with pytest.raises(sdk.ArmError, match="ZIP"):
        sdk.Package(str(bad))
    nojson = tmp_path / "nojson.armpack"
    with zipfile.ZipFile(nojson, "w") as zf:
        zf.writestr("manifest.json", "{ this is not json")
    with pytest.raises(sdk.ArmError, match="manifest.json"):
        sdk.Package(str(nojson))
    # a package with only a CPU graph loads, lists the graph, and has nothing to select
    cpu = tmp_path / "cpu.armpack"
    with zipfile.ZipFile(cpu, "w") as zf:
        zf.writestr("manifest.json", json.dumps({"model_id": "m", "arch": {}, "graphs": [
            {"index": 0, "id": "neon", "path": "graphs/neon.json", "execution_backend": "cpu"}],
            "kernels": [], "weights": []}))
    with sdk.Package(str(cpu)) as pkg:
        assert pkg.num_graphs() == 1
        assert "cpu" in pkg.graph(0).description
        with pytest.raises(sdk.ArmError):
            pkg.graph(0).session()


# ------------------------------------------------------------------ memory-aware selection
def _multi_graph_package(tmp_path, contexts, conditions=None):
    from silicongraph_b200 import armpack
    cfg = armpack.llama_config(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=1000,
                               rope_theta=500000.0, max_pos=65536)
    t = armpack.cuda_tensors(cfg, armpack.random_llama_weights(cfg, seed=2), group_size=32)
    return armpack.write_package(str(tmp_path / "multi.armpack"), cfg, t, max_context=contexts,
                                 max_prefill_chunk=128, graph_conditions=conditions)


def test_select_prefers_fitting_context_and_refuses_before_allocation(tmp_path):
    """graph_selector.cpp:34-94 with device memory as the budget: the graph
    with a long-enough context wins, a graph over 95 % of the budget is
    rejected (:45-51), and with nothing fitting the call refuses with the
    reason instead of allocating."""
    from silicongraph_b200 import sdk
    path = _multi_graph_package(tmp_path, [1024, 4096, 16384])
    with sdk.Package(path) as pkg:
        need = [pkg.graph(i).session_bytes() for i in range(3)]
        assert need[0] < need[1] < need[2]               # the KV cache grows with the context
        big = 100 * need[2]
        assert "ctx4096" in pkg.select(2000, device_bytes_available=big).description
        assert "ctx16384" in pkg.select(10000, device_bytes_available=big).description
        # the 4096-token graph exactly over 95 %: the shorter one is taken despite its context
        just_under = need[1] * 100 // 95 + 200
        assert "ctx4096" in pkg.select(2000, device_bytes_available=just_under).description
        assert "ctx1024" in pkg.select(2000, device_bytes_available=need[1]).description
        with pytest.raises(sdk.ArmError) as e:
            pkg.select(2000, device_bytes_available=need[0])   # nothing fits in 95 %
        assert "95%" in str(e.value) and "needs" in str(e.value)


def test_select_penalises_thermal_and_latency_mismatch(tmp_path):
    from silicongraph_b200 import sdk
    conds = [{"thermal_state": "hot", "latency_mode": "interactive"},
             {"thermal_state": "nominal", "latency_mode": "background"},
             {"thermal_state": "nominal", "latency_mode": "interactive"}]
    path = _multi_graph_package(tmp_path, [4096, 4096, 4096], conds)
    with sdk.Package(path) as pkg:
        big = 100 * pkg.graph(0).session_bytes()
        assert pkg.select(4096, device_bytes_available=big).description.startswith("cuda_int4_g32_ctx4096_2")
        # a hot device prefers the graph built for it (10 per thermal step outweighs nothing else)
        assert pkg.select(4096, thermal=2, device_bytes_available=big).description.startswith(
            "cuda_int4_g32_ctx4096_0")
        assert pkg.select(4096, latency=2, device_bytes_available=big).description.startswith(
            "cuda_int4_g32_ctx4096_1")
