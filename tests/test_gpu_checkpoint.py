"""A sparse layer read from a checkpoint directory feeds the kernels as
stored: written out through the safetensors writer, read back by
LagunaCheckpoint, the block gives the same bits as the block built from the
tensors in memory, at decode (GEMV engine) and at T = 24 (grouped FP4 path),
and the routed stack runs on the loaded layers."""
import importlib

import pytest
import torch

from conftest import PKG
from test_checkpoint import tiny_config, write_checkpoint

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ck = importlib.import_module(PKG + ".checkpoint")


def test_loaded_layers_run_and_match(nv, tmp_path):
    lag = importlib.import_module(PKG + ".laguna")
    cfg = tiny_config()
    cfg.update(hidden_size=1024, moe_intermediate_size=512, shared_expert_intermediate_size=512,
               num_experts=16, num_experts_per_tok=4)
    mcfg = lag.LagunaMoEConfig(hidden=1024, inter=512, n_experts=16, top_k=4, shared_inter=512)
    made = {n: lag.random_sparse_layer(nv, seed=700 + n, device=DEV, cfg=mcfg) for n in (1, 2)}

    def tamper(t, a):
        for n, (_, raw) in made.items():
            p = f"model.layers.{n}.mlp"
            for stem, bank in (("switch_mlp", raw["routed"]), ("shared_expert", raw["shared"])):
                for proj in ("gate", "up", "down"):
                    t[f"{p}.{stem}.{proj}_proj.weight"] = bank[f"{proj}_w"].cpu()
                    t[f"{p}.{stem}.{proj}_proj.scales"] = bank[f"{proj}_s"].cpu()
            t[f"{p}.gate.weight"] = raw["router_w"].cpu()
            t[f"{p}.gate.e_score_correction_bias"] = raw["router_b"].cpu()
            t[f"model.layers.{n}.post_attention_layernorm.weight"] = raw["norm_w"].cpu()

    write_checkpoint(str(tmp_path), cfg, n_shards=2, tamper=tamper)
    c = ck.LagunaCheckpoint(str(tmp_path))
    c.check_inventory()
    g = torch.Generator(device=DEV).manual_seed(9)
    loaded = {}
    for n in (1, 2):
        blk, raw = c.sparse_block(nv, n, device=DEV)
        loaded[n] = (blk, raw)
        for T in (1, 24):
            x = torch.randn(T, 1024, generator=g, device=DEV).to(torch.bfloat16)
            want = made[n][0](x)
            got = blk(x)
            assert torch.equal(got, want), (n, T)
    chain = nv.MoEDecodeChain([loaded[n][0] for n in (1, 2)], None, T=1, route=True,
                              residual=True, norms=[loaded[n][1]["norm_w"] for n in (1, 2)],
                              device=DEV)
    ref = nv.MoEDecodeChain([made[n][0] for n in (1, 2)], None, T=1, route=True, residual=True,
                            norms=[made[n][1]["norm_w"] for n in (1, 2)], device=DEV)
    assert chain.stack_fp4 and ref.stack_fp4
    h = torch.randn(1, 1024, generator=g, device=DEV).to(torch.bfloat16)
    assert torch.equal(chain(h.cpu()), ref(h.cpu()))
    nv.device_status()
