"""Laguna XS 2.1 sparse-layer geometry and seeded random-init NVFP4 layers.

Geometry from the reference's fixtures/poolside_laguna_xs_2_1_nvfp4_config.json
(hidden_size :61, moe_intermediate_size :153, moe_routed_scaling_factor :154,
norm_topk_prob :155, num_experts :199, num_experts_per_tok :200,
num_hidden_layers :201, quantization :204-213, rms_norm_eps :214,
shared_expert_intermediate_size :233).  Layer 0 is dense BF16; layers 1..39 carry the sparse MoE block.

The real checkpoint is not available, so layers are random-init: bf16 weights
~ N(0, std) quantized to NVFP4 by this library's quantizer (bit-identical to
the reference's quantizer), router weight bf16 ~ N(0, std), router bias f32
~ N(0, bias_std).  Stored layouts follow the checkpoint's tensor inventory:
switch_mlp.{gate,up}_proj [E, I, H/8] u32 + [E, I, H/16] u8, down_proj
[E, H, I/8] + [E, H, I/16], shared_expert likewise without E.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class LagunaMoEConfig:
    hidden: int = 2048
    inter: int = 512
    n_experts: int = 256
    top_k: int = 8
    shared_inter: int = 512
    routed_scaling: float = 2.5
    norm_topk_prob: bool = True
    num_layers: int = 40
    num_sparse_layers: int = 39
    rms_norm_eps: float = 1e-6

    def routed_bytes_per_expert(self) -> int:
        """Packed codes + scales of one expert's gate, up and down projections."""
        per_row = lambda K: K // 2 + K // 16
        return 2 * self.inter * per_row(self.hidden) + self.hidden * per_row(self.inter)

    def shared_bytes(self) -> int:
        per_row = lambda K: K // 2 + K // 16
        return 2 * self.shared_inter * per_row(self.hidden) + self.hidden * per_row(
            self.shared_inter)

    def router_bytes(self) -> int:
        return self.n_experts * self.hidden * 2


LAGUNA_XS_2_1 = LagunaMoEConfig()


def _quantized_bank(nv, shape, std, gen, device, chunk_rows=1 << 20):
    """N(0, std) bf16 weights of `shape` [..., K] quantized in row chunks."""
    K = shape[-1]
    rows = 1
    for d in shape[:-1]:
        rows *= d
    wq = torch.empty(rows, K // 8, dtype=torch.uint32, device=device)
    sq = torch.empty(rows, K // 16, dtype=torch.uint8, device=device)
    step = max(1, chunk_rows // K * 16)
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        w = (torch.randn(r1 - r0, K, generator=gen, device=device) * std).to(torch.bfloat16)
        q, s = nv.quantize(w)
        wq[r0:r1] = q
        sq[r0:r1] = s
    return wq.reshape(*shape[:-1], K // 8), sq.reshape(*shape[:-1], K // 16)


def random_sparse_layer(nv, seed: int, device="cuda:0", cfg: LagunaMoEConfig = LAGUNA_XS_2_1,
                        std: float = 0.02, bias_std: float = 1e-3, n_experts: int | None = None,
                        with_shared: bool = True):
    """Return (SparseMoeBlock, raw dict of banks) for one random-init sparse layer."""
    gen = torch.Generator(device=device).manual_seed(seed)
    E = n_experts or cfg.n_experts
    H, I, Is = cfg.hidden, cfg.inter, cfg.shared_inter
    routed = {}
    routed["gate_w"], routed["gate_s"] = _quantized_bank(nv, (E, I, H), std, gen, device)
    routed["up_w"], routed["up_s"] = _quantized_bank(nv, (E, I, H), std, gen, device)
    routed["down_w"], routed["down_s"] = _quantized_bank(nv, (E, H, I), std, gen, device)
    shared = None
    if with_shared:
        shared = {}
        shared["gate_w"], shared["gate_s"] = _quantized_bank(nv, (Is, H), std, gen, device)
        shared["up_w"], shared["up_s"] = _quantized_bank(nv, (Is, H), std, gen, device)
        shared["down_w"], shared["down_s"] = _quantized_bank(nv, (H, Is), std, gen, device)
    router_w = (torch.randn(E, H, generator=gen, device=device) * std).to(torch.bfloat16)
    router_b = torch.randn(E, generator=gen, device=device) * bias_std
    # the decoder layer's post_attention_layernorm weight in front of the block
    norm_w = (1.0 + 0.1 * torch.randn(H, generator=gen, device=device)).to(torch.bfloat16)
    block = nv.SparseMoeBlock(routed, shared, router_w, router_b, top_k=cfg.top_k,
                              routed_scaling=cfg.routed_scaling,
                              norm_topk_prob=cfg.norm_topk_prob)
    return block, dict(routed=routed, shared=shared, router_w=router_w, router_b=router_b,
                       norm_w=norm_w)


def random_routing(T: int, cfg: LagunaMoEConfig, seed: int, device="cuda:0"):
    """BASELINE config[1] routing: k distinct uniform experts per token, weights =
    softmax of N(0,1) logits."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    inds = torch.stack([torch.randperm(cfg.n_experts, generator=g)[:cfg.top_k]
                        for _ in range(T)]).to(torch.int32)
    w = torch.softmax(torch.randn(T, cfg.top_k, generator=g), dim=-1)
    return inds.to(device), w.to(device)
