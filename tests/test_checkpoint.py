"""The NVFP4 checkpoint reader (checkpoint.py) on the CPU: the contract's
inventory restated from the geometry against the reference's published
inventory digest, the safetensors container, the directory validation
(docs/laguna-weight-contract.md:35-127 of the reference) and the [gate32,
up32] interleave (LagunaRuntimeModel.swift:10605-10625)."""
import importlib
import json
import os

import numpy as np
import pytest
import torch

from conftest import PKG, ROOT

ck = importlib.import_module(PKG + ".checkpoint")
INV_GOLDEN = os.path.join(ROOT, "tests", "golden", "laguna_inventory_golden.json")


def test_inventory_matches_the_reference_digest():
    """expected_inventory for Laguna XS 2.1 gives the 912 tensors, dtype
    counts and (name, dtype, shape) digest of the reference's inventory."""
    gold = json.load(open(INV_GOLDEN))
    g = ck.LagunaGeometry.from_config(ck.laguna_xs_2_1_config())
    inv = ck.expected_inventory(g)
    assert len(inv) == gold["tensor_count"] == 912
    counts = {}
    for _, d, _ in inv:
        counts[d] = counts.get(d, 0) + 1
    assert counts == gold["dtype_counts"]
    assert ck.canonical_inventory_sha256(inv) == gold["sha256_name_dtype_shape"]
    assert g.sparse_layers() == list(range(1, 40)) and g.moe.num_sparse_layers == 39


def test_canonical_hash_reproduces_the_fixture_with_shards():
    """With shard names, the canonical form reproduces the fixture's own
    published digest (read from the reference tree when it is present)."""
    path = "/root/reference/fixtures/poolside_laguna_xs_2_1_nvfp4_tensor_inventory.json"
    if not os.path.exists(path):
        pytest.skip("reference tree not present")
    inv = json.load(open(path))
    names = [s["name"] for s in inv["shards"]]
    rows = [(n, d, tuple(s), names[i - 1]) for n, d, s, i in inv["tensors"]]
    assert ck.canonical_inventory_sha256(rows) == json.load(open(INV_GOLDEN))[
        "canonical_sha256_with_shards"]


def tiny_config(shared=True):
    q = dict(ck.NVFP4_QUANT)
    return {"hidden_size": 256, "vocab_size": 64, "num_hidden_layers": 3, "head_dim": 16,
            "num_key_value_heads": 2, "num_attention_heads": 4,
            "num_attention_heads_per_layer": [4, 8, 8],
            "mlp_layer_types": ["dense", "sparse", "sparse"], "intermediate_size": 128,
            "moe_intermediate_size": 128, "shared_expert_intermediate_size": 128 if shared else 0,
            "num_experts": 8, "num_experts_per_tok": 2, "moe_routed_scaling_factor": 2.5,
            "norm_topk_prob": True, "rms_norm_eps": 1e-6, "quantization": q,
            "quantization_config": dict(q)}


def random_tensor(dtype, shape, rng):
    n = int(np.prod(shape)) if shape else 1
    if dtype == "BF16":
        return torch.from_numpy(rng.integers(0, 1 << 16, n, dtype=np.uint16).reshape(shape)
                                ).view(torch.bfloat16)
    if dtype == "F32":
        return torch.from_numpy(rng.standard_normal(n).astype(np.float32).reshape(shape))
    if dtype == "U32":
        return torch.from_numpy(rng.integers(0, 1 << 32, n, dtype=np.uint32).reshape(shape))
    return torch.from_numpy(rng.integers(0, 256, n, dtype=np.uint8).reshape(shape))


def write_checkpoint(d, cfg, n_shards=2, seed=0, tamper=None):
    """A complete checkpoint directory for cfg with random contents; returns
    the tensors by name.  tamper(tensors, assignment) may edit either first."""
    rng = np.random.default_rng(seed)
    inv = ck.expected_inventory(ck.LagunaGeometry.from_config(cfg))
    tensors = {n: random_tensor(dt, s, rng) for n, dt, s in inv}
    names = sorted(tensors)
    shard = lambda i: f"model-{i + 1:05d}-of-{n_shards:05d}.safetensors"
    assign = {n: shard(i * n_shards // len(names)) for i, n in enumerate(names)}
    if tamper:
        tamper(tensors, assign)
    os.makedirs(d, exist_ok=True)
    json.dump(cfg, open(os.path.join(d, "config.json"), "w"))
    json.dump({"metadata": {}, "weight_map": assign},
              open(os.path.join(d, ck.INDEX_NAME), "w"))
    for s in sorted(set(assign.values())):
        ck.write_safetensors(os.path.join(d, s),
                             {n: t for n, t in tensors.items() if assign[n] == s},
                             metadata={"format": "mlx"})
    return tensors


def test_safetensors_round_trip(tmp_path):
    rng = np.random.default_rng(1)
    ts = {"a": random_tensor("BF16", (3, 5), rng), "b": random_tensor("U32", (2, 7), rng),
          "c": random_tensor("U8", (9,), rng), "d": random_tensor("F32", (4, 1, 2), rng),
          "e": torch.zeros(0, 4, dtype=torch.uint8)}
    p = str(tmp_path / "x.safetensors")
    ck.write_safetensors(p, ts, metadata={"k": "v"})
    f = ck.SafetensorsFile(p)
    assert f.metadata == {"k": "v"} and sorted(f.names()) == sorted(ts)
    for n, t in ts.items():
        got = f.tensor(n)
        assert got.dtype == t.dtype and got.shape == t.shape
        assert torch.equal(got.view(torch.uint8) if got.numel() else got,
                           t.view(torch.uint8) if t.numel() else t)
    # the header is read as the format defines it: little-endian length + JSON
    raw = open(p, "rb").read()
    n = int.from_bytes(raw[:8], "little")
    hdr = json.loads(raw[8:8 + n])
    b, e = hdr["b"]["data_offsets"]
    assert np.array_equal(np.frombuffer(raw[8 + n + b:8 + n + e], dtype="<u4").reshape(2, 7),
                          ts["b"].numpy())


def test_bad_container_is_rejected(tmp_path):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(b"\x05\x00")
    with pytest.raises(ck.CheckpointError, match="shorter"):
        ck.SafetensorsFile(str(p))
    hdr = json.dumps({"t": {"dtype": "U8", "shape": [4], "data_offsets": [0, 8]}}).encode()
    p.write_bytes(len(hdr).to_bytes(8, "little") + hdr + b"\0" * 8)
    with pytest.raises(ck.CheckpointError, match="data_offsets"):
        ck.SafetensorsFile(str(p))
    hdr = json.dumps({"t": {"dtype": "Q7", "shape": [1], "data_offsets": [0, 1]}}).encode()
    p.write_bytes(len(hdr).to_bytes(8, "little") + hdr + b"\0")
    with pytest.raises(ck.CheckpointError, match="dtype"):
        ck.SafetensorsFile(str(p))


def test_checkpoint_opens_validates_and_loads_a_sparse_layer(tmp_path):
    cfg = tiny_config()
    ts = write_checkpoint(str(tmp_path), cfg, n_shards=3)
    c = ck.LagunaCheckpoint(str(tmp_path))
    c.check_inventory()
    assert c.geometry.sparse_layers() == [1, 2]
    raw = c.sparse_layer(2)
    p = "model.layers.2.mlp"
    for proj in ("gate", "up", "down"):
        for kind, suf in (("w", "weight"), ("s", "scales")):
            assert torch.equal(raw["routed"][f"{proj}_{kind}"],
                               ts[f"{p}.switch_mlp.{proj}_proj.{suf}"])
            assert torch.equal(raw["shared"][f"{proj}_{kind}"],
                               ts[f"{p}.shared_expert.{proj}_proj.{suf}"])
    assert raw["routed"]["gate_w"].dtype == torch.uint32
    assert raw["routed"]["gate_w"].shape == (8, 128, 32)
    assert raw["routed"]["down_s"].shape == (8, 256, 8)
    assert torch.equal(raw["router_w"].view(torch.int16),
                       ts[f"{p}.gate.weight"].view(torch.int16))
    assert torch.equal(raw["router_b"], ts[f"{p}.gate.e_score_correction_bias"])
    assert torch.equal(raw["norm_w"].view(torch.int16),
                       ts["model.layers.2.post_attention_layernorm.weight"].view(torch.int16))
    with pytest.raises(ck.CheckpointError, match="dense"):
        c.sparse_layer(0)
    assert len(c.inventory()) == len(ts)


def test_checkpoint_without_shared_expert(tmp_path):
    cfg = tiny_config(shared=False)
    write_checkpoint(str(tmp_path), cfg)
    c = ck.LagunaCheckpoint(str(tmp_path))
    c.check_inventory()
    assert c.sparse_layer(1)["shared"] is None


@pytest.mark.parametrize("case", ["quant_missing", "quant_differs", "quant_other",
                                  "shard_missing", "shard_extra", "wrong_shard",
                                  "wrong_shape", "wrong_dtype", "biases", "missing_tensor"])
def test_contract_violations_are_rejected(tmp_path, case):
    cfg = tiny_config()
    d = str(tmp_path)
    tamper = None
    if case == "quant_missing":
        del cfg["quantization_config"]
    elif case == "quant_differs":
        cfg["quantization_config"] = {"group_size": 32, "bits": 4, "mode": "nvfp4"}
    elif case == "quant_other":
        cfg["quantization"] = cfg["quantization_config"] = {"group_size": 16, "bits": 4,
                                                            "mode": "mxfp4"}
    elif case == "wrong_shape":
        def tamper(t, a):
            t["model.layers.1.mlp.switch_mlp.up_proj.scales"] = torch.zeros(8, 128, 8,
                                                                            dtype=torch.uint8)
    elif case == "wrong_dtype":
        def tamper(t, a):
            t["model.layers.1.mlp.gate.e_score_correction_bias"] = torch.zeros(
                8, dtype=torch.bfloat16)
    elif case == "biases":
        def tamper(t, a):
            n = "model.layers.1.mlp.switch_mlp.up_proj.biases"
            t[n] = torch.zeros(8, 128, 16, dtype=torch.bfloat16)
            a[n] = a["model.layers.1.mlp.switch_mlp.up_proj.scales"]
    elif case == "missing_tensor":
        def tamper(t, a):
            n = "model.layers.2.mlp.shared_expert.down_proj.scales"
            del t[n], a[n]
    write_checkpoint(d, cfg, n_shards=2, tamper=tamper)
    if case == "shard_missing":
        os.remove(os.path.join(d, "model-00002-of-00002.safetensors"))
    elif case == "shard_extra":
        ck.write_safetensors(os.path.join(d, "model-00009-of-00009.safetensors"),
                             {"x": torch.zeros(1, dtype=torch.uint8)})
    elif case == "wrong_shard":
        idx = json.load(open(os.path.join(d, ck.INDEX_NAME)))
        n = "model.layers.1.mlp.gate.weight"
        other = [s for s in set(idx["weight_map"].values()) if s != idx["weight_map"][n]][0]
        idx["weight_map"][n] = other
        json.dump(idx, open(os.path.join(d, ck.INDEX_NAME), "w"))
    with pytest.raises(ck.CheckpointError):
        ck.LagunaCheckpoint(d).check_inventory()


def test_rotary_tables_are_excluded(tmp_path):
    def tamper(t, a):
        n = "model.layers.0.self_attn.rotary_emb.inv_freq"
        t[n] = torch.zeros(8, dtype=torch.float32)
        a[n] = a["model.layers.0.input_layernorm.weight"]
    write_checkpoint(str(tmp_path), tiny_config(), tamper=tamper)
    c = ck.LagunaCheckpoint(str(tmp_path))
    c.check_inventory()
    assert not any("inv_freq" in n for n, *_ in c.inventory())


def test_gate_up_interleave_layout_and_inverse():
    """Fused rows 64 t .. 64 t + 31 are gate rows 32 t .., the next 32 the same
    up rows; split_gate_up inverts it, for codes and scale bytes alike."""
    rng = np.random.default_rng(3)
    E, I, D = 3, 128, 16
    gate = torch.from_numpy(rng.integers(0, 1 << 32, (E, I, D), dtype=np.uint32))
    up = torch.from_numpy(rng.integers(0, 1 << 32, (E, I, D), dtype=np.uint32))
    f = ck.interleave_gate_up(gate, up)
    assert f.shape == (E, 2 * I, D)
    for t in range(I // 32):
        assert torch.equal(f[:, 64 * t:64 * t + 32], gate[:, 32 * t:32 * t + 32])
        assert torch.equal(f[:, 64 * t + 32:64 * t + 64], up[:, 32 * t:32 * t + 32])
    g2, u2 = ck.split_gate_up(f)
    assert torch.equal(g2, gate) and torch.equal(u2, up)
    s = torch.from_numpy(rng.integers(0, 256, (E, I, D // 2), dtype=np.uint8))
    assert torch.equal(ck.split_gate_up(ck.interleave_gate_up(s, s.flip(0)))[1], s.flip(0))
    with pytest.raises(ValueError):
        ck.interleave_gate_up(gate[:, :100], up[:, :100])
