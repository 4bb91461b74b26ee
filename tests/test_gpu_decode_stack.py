"""GPU parity of the persistent decode stack (moe_decode_stack_forward): the
whole serial decode over L sparse layers in one cooperative launch.  It runs
the same GEMV engine and staging as the per-layer bulk-copy kernels but sums
partial products in another order, so a single layer must be within the
BASELINE tolerance of the fp32 oracle, an L-layer chain within L times the
relative-L2 bound of the per-layer chains (every layer rounds its output to
bf16 in both), and replays are bit-for-bit repeatable."""
import importlib

import numpy as np
import pytest
import torch

from conftest import PKG, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def u32_np(t):
    return t.contiguous().view(torch.int32).cpu().numpy().view(np.uint32)


def layers(nv, n, n_experts=32, with_shared=True, seed=300):
    lag = importlib.import_module(PKG + ".laguna")
    cfg = lag.LagunaMoEConfig(n_experts=n_experts)
    made = [lag.random_sparse_layer(nv, seed=seed + l, device=DEV, cfg=cfg, n_experts=n_experts,
                                    with_shared=with_shared) for l in range(n)]
    routing = [lag.random_routing(1, cfg, seed=seed + 100 + l, device=DEV) for l in range(n)]
    return [m[0] for m in made], [m[1] for m in made], routing


def chain_tol(n_layers):
    """Relative-L2 bound for two serial chains that each round every layer's
    output to bf16 (the single-op BASELINE bound, compounding with depth)."""
    return 5e-3 * max(1, n_layers)


def seeded_x(seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(1, 2048, generator=g, device=DEV).to(torch.bfloat16)


def layer_by_layer(blocks, routing, x):
    y = x
    for l, b in enumerate(blocks):
        y = b(y, inds=routing[l][0], weights=routing[l][1])
    return y


@pytest.mark.parametrize("with_shared,n", [(True, 2), (False, 2), (True, 5)])
def test_stack_matches_bulk_copy_layer_loop(nv, with_shared, n):
    blocks, _, routing = layers(nv, n, with_shared=with_shared)
    chain = nv.MoEDecodeChain(blocks, routing, T=1, device=DEV).capture()
    assert chain.stack and chain.launches_per_step() == 1
    x = seeded_x(n + 10 * with_shared)
    with nv.launch_flags(bulk_copy=True):
        want = layer_by_layer(blocks, routing, x)
    first = None
    for _ in range(3):  # replays are repeatable
        chain.x0.copy_(x)
        out = chain.replay()
        torch.cuda.synchronize()
        if first is None:
            first = out.clone()
        assert torch.equal(out, first)
    assert_close(first.float().cpu().numpy(), want.float().cpu().numpy(), max_abs=float("inf"),
                 rel_l2=chain_tol(n), what="stack vs loop")
    nv.device_status()
    yh = chain(x.cpu().pin_memory())
    assert torch.equal(yh, first.cpu())


def test_stack_matches_default_kernels_and_oracle(nv, orc):
    blocks, raw, routing = layers(nv, 3, n_experts=256, seed=900)
    chain = nv.MoEDecodeChain(blocks, routing, T=1, device=DEV).capture()
    assert chain.stack
    x = seeded_x(3)
    chain.x0.copy_(x)
    out = chain.replay()
    torch.cuda.synchronize()
    want = layer_by_layer(blocks, routing, x)  # per-thread-load kernels
    assert_close(out.float().cpu().numpy(), want.float().cpu().numpy(), max_abs=float("inf"),
                 rel_l2=chain_tol(3), what="stack vs default")
    # Layer 0 against the fp32 oracle (used experts only).
    one = nv.MoEDecodeChain(blocks[:1], routing[:1], T=1, device=DEV).capture()
    assert one.stack
    one.x0.copy_(x)
    y0 = one.replay()
    torch.cuda.synchronize()
    inds = routing[0][0].cpu().numpy().astype(np.int64)
    used = np.unique(inds)
    remap = {e: i for i, e in enumerate(used)}
    ids = torch.from_numpy(used).to(DEV)
    r = raw[0]
    routed = {k: (u32_np(v.view(torch.int32)[ids]) if v.dtype == torch.uint32 else
                  v[ids].cpu().numpy()) for k, v in r["routed"].items()}
    shared = {k: (u32_np(v) if v.dtype == torch.uint32 else v.cpu().numpy())
              for k, v in r["shared"].items()}
    ci = np.vectorize(remap.get)(inds).astype(np.uint32)
    o = orc.port.moe_block_f32(x.float().cpu().numpy(), ci, routing[0][1].float().cpu().numpy(),
                               routed, shared, scaling=2.5)
    assert_close(y0.float().cpu().numpy(), o, what="stack layer vs oracle")


def test_stack_many_layers(nv):
    blocks, _, routing = layers(nv, 3, seed=500)
    # 39 layers (the model's sparse count) cycling 3 distinct weight sets.
    stack_blocks = [blocks[l % 3] for l in range(39)]
    stack_routing = [routing[l % 3] for l in range(39)]
    chain = nv.MoEDecodeChain(stack_blocks, stack_routing, T=1, device=DEV).capture()
    assert chain.stack
    x = seeded_x(39)
    chain.x0.copy_(x)
    out = chain.replay()
    torch.cuda.synchronize()
    with nv.launch_flags(bulk_copy=True):
        want = layer_by_layer(stack_blocks, stack_routing, x)
    assert_close(out.float().cpu().numpy(), want.float().cpu().numpy(), max_abs=float("inf"),
                 rel_l2=chain_tol(39), what="39-layer stack")


def test_stack_out_of_range_expert_is_reported(nv):
    blocks, _, routing = layers(nv, 2, seed=700)
    bad = [(routing[0][0].clone(), routing[0][1]), routing[1]]
    bad[0][0][0, 3] = 999  # 32 experts
    chain = nv.MoEDecodeChain(blocks, bad, T=1, device=DEV).capture()
    assert chain.stack
    chain.replay()
    with pytest.raises(nv.DeviceIndexError):
        nv.device_status()
    nv.device_status()  # the latch was cleared
