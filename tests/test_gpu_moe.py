"""GPU parity of the fused MoE block (BASELINE configs [1] and [2]) against the
fp32 oracle block, at Laguna XS 2.1's full geometry (H=2048, I=512, E=256,
top-8, shared expert 512, scaling 2.5)."""
import importlib

import numpy as np
import pytest
import torch

from conftest import PKG, assert_close, check_routing

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def u32_np(t):
    return t.contiguous().view(torch.int32).cpu().numpy().view(np.uint32)


@pytest.fixture(scope="module")
def layer(nv):
    lag = importlib.import_module(PKG + ".laguna")
    block, raw = lag.random_sparse_layer(nv, seed=1234, device=DEV)
    return lag, block, raw


def oracle_block(orc, raw, x, inds, wts, residual=None, with_shared=True):
    """Oracle on the experts actually used (remapped to a compact bank)."""
    inds_np = inds.cpu().numpy().astype(np.int64)
    used = np.unique(inds_np)
    remap = {e: i for i, e in enumerate(used)}
    ids = torch.from_numpy(used).to(DEV)
    r = raw["routed"]
    routed = {k: (u32_np(v.view(torch.int32)[ids]) if v.dtype == torch.uint32
                  else v[ids].cpu().numpy()) for k, v in r.items()}
    shared = None
    if with_shared:
        shared = {k: (u32_np(v) if v.dtype == torch.uint32 else v.cpu().numpy())
                  for k, v in raw["shared"].items()}
    ci = np.vectorize(remap.get)(inds_np).astype(np.uint32)
    res = None if residual is None else residual.float().cpu().numpy()
    return orc.port.moe_block_f32(x.float().cpu().numpy(), ci, wts.float().cpu().numpy(),
                                  routed, shared, scaling=2.5, residual=res)


@pytest.mark.parametrize("bulk", [False, True])
@pytest.mark.parametrize("T", [1, 2, 8])
def test_routed_layer_given_routing_config1(nv, orc, layer, T, bulk):
    lag, block, raw = layer
    inds, wts = lag.random_routing(T, lag.LAGUNA_XS_2_1, seed=T)
    g = torch.Generator(device=DEV).manual_seed(T)
    x = torch.randn(T, 2048, generator=g, device=DEV).to(torch.bfloat16)
    with nv.launch_flags(bulk_copy=bulk):
        y = block(x, inds=inds, weights=wts)
    want = oracle_block(orc, raw, x, inds, wts)
    assert_close(y.float().cpu().numpy(), want, what=f"block T={T}")


@pytest.mark.parametrize("bulk", [False, True])
@pytest.mark.parametrize("T", [1, 3, 8, 11])
def test_full_block_with_router_config2(nv, orc, layer, T, bulk):
    lag, block, raw = layer
    g = torch.Generator(device=DEV).manual_seed(100 + T)
    x = torch.randn(T, 2048, generator=g, device=DEV).to(torch.bfloat16)
    res = torch.randn(T, 2048, generator=g, device=DEV).to(torch.bfloat16)
    with nv.launch_flags(bulk_copy=bulk):
        y, inds, wts = block(x, residual=res, return_routing=True)
    # The routing the block used is the router's (checked against the oracle router).
    ri, rw = nv.moe_router_topk(x, raw["router_w"], raw["router_b"], 8)
    assert torch.equal(inds, ri) and torch.equal(wts, rw)
    check_routing(orc, x.view(torch.int16).cpu().numpy().view(np.uint16),
                  raw["router_w"].view(torch.int16).cpu().numpy().view(np.uint16),
                  raw["router_b"].cpu().numpy(), u32_np(inds), wts.cpu().numpy(), 8)
    want = oracle_block(orc, raw, x, inds, wts, residual=res)
    assert_close(y.float().cpu().numpy(), want, what=f"block+router T={T}")


def test_block_without_shared_expert(nv, orc, layer):
    lag, _, raw = layer
    block = nv.SparseMoeBlock(raw["routed"], None, raw["router_w"], raw["router_b"])
    inds, wts = lag.random_routing(2, lag.LAGUNA_XS_2_1, seed=77)
    x = torch.randn(2, 2048, device=DEV).to(torch.bfloat16)
    y = block(x, inds=inds, weights=wts)
    want = oracle_block(orc, raw, x, inds, wts, with_shared=False)
    assert_close(y.float().cpu().numpy(), want, what="no shared")


def test_block_matches_composed_library_ops(nv, layer):
    """The fused kernels equal the op-by-op composition through gather_qmm
    (SwitchGLU.callAsFunction, SwitchLayers.swift:532-580)."""
    lag, block, raw = layer
    r, s = raw["routed"], raw["shared"]
    inds, wts = lag.random_routing(3, lag.LAGUNA_XS_2_1, seed=5)
    x = torch.randn(3, 2048, device=DEV).to(torch.float32)
    y = block(x, inds=inds, weights=wts)
    xe = x.reshape(3, 1, 1, 2048)
    gate = nv.gather_qmm(xe, r["gate_w"], r["gate_s"], rhs_indices=inds.reshape(3, 8))
    up = nv.gather_qmm(xe, r["up_w"], r["up_s"], rhs_indices=inds.reshape(3, 8))
    act = torch.nn.functional.silu(gate) * up
    down = nv.gather_qmm(act, r["down_w"], r["down_s"], rhs_indices=inds.reshape(3, 8))
    routed = (down.squeeze(-2) * wts.unsqueeze(-1)).sum(-2) * 2.5
    sg = nv.quantized_matmul(x, s["gate_w"], s["gate_s"])
    su = nv.quantized_matmul(x, s["up_w"], s["up_s"])
    shared = nv.quantized_matmul(torch.nn.functional.silu(sg) * su, s["down_w"], s["down_s"])
    assert_close(y.cpu().numpy(), (routed + shared).cpu().numpy(), what="fused vs composed")


def test_out_of_range_routing_is_latched(nv, layer):
    lag, block, raw = layer
    nv.device_status()
    inds = torch.tensor([[0, 1, 2, 3, 4, 5, 6, 300]], dtype=torch.int32, device=DEV)
    wts = torch.full((1, 8), 0.125, device=DEV)
    block(torch.ones(1, 2048, device=DEV, dtype=torch.bfloat16), inds=inds, weights=wts)
    with pytest.raises(nv.DeviceIndexError):
        nv.device_status()


@pytest.mark.parametrize("route", [False, True])
@pytest.mark.parametrize("pdl", [False, True])
def test_decode_chain_graph_matches_layer_by_layer(nv, route, pdl):
    """The CUDA-graph chain (with and without programmatic dependent launch)
    equals running the layers one call at a time, bit for bit."""
    lag = importlib.import_module(PKG + ".laguna")
    cfg = lag.LagunaMoEConfig(n_experts=32)
    blocks = [lag.random_sparse_layer(nv, seed=50 + l, device=DEV, cfg=cfg, n_experts=32)[0]
              for l in range(4)]
    routing = [lag.random_routing(2, cfg, seed=60 + l, device=DEV) for l in range(4)]
    # Cover both kernel families (bulk-copy fed with PDL, per-thread loads
    # without); the layer-by-layer reference uses the same family.
    with nv.launch_flags(bulk_copy=pdl):
        chain = nv.MoEDecodeChain(blocks, None if route else routing, T=2, route=route,
                                  device=DEV).capture(pdl=pdl)
        x = torch.randn(2, 2048, device=DEV).to(torch.bfloat16)
        want = x
        for l, b in enumerate(blocks):
            if route:
                want = b(want)
            else:
                want = b(want, inds=routing[l][0], weights=routing[l][1])
        for _ in range(3):  # replays are repeatable
            chain.x0.copy_(x)
            out = chain.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, want)
        yh = chain(x.cpu().pin_memory())
        assert torch.equal(yh, want.cpu())
