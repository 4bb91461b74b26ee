"""GPU parity of the routed decode stack (moe_decode_stack_routed_forward): the
serial decode over L sparse layers with every layer's router inside one
cooperative launch (BASELINE config[2] at one sequence: router top-8, routed
experts, shared expert, summed into the residual), by default with each
layer's RMSNorm in front of its block, the decoder layer's MoE half
(Laguna.swift:242-246).

Checked layer by layer against the CPU oracle: a stack of n layers returns
h_n, and every launch computes each layer the same way whatever follows it,
so the prefixes n = 1 .. L give every intermediate residual stream.  For each
layer l, on the GPU's own h_l, with x_l = the oracle's RMSNorm of h_l:
  * the routing the stack wrote must be the oracle router's on x_l
    (Laguna.swift:165-180) up to logits that round to a neighbouring bf16
    value (the stack sums logits and the norm's squares in another order than
    the oracle: an expert may differ only where its choice lies within one
    such rounding step of the k-th choice, and weights agree to that step);
  * h_{l+1} must equal the oracle's f32 block on x_l (with the GPU's routing)
    plus h_l within the BASELINE bound (max-abs 2e-2, relative-L2 5e-3).
"""
import ctypes
import importlib

import numpy as np
import pytest
import torch

from conftest import PKG, assert_close, assert_close_bf16_out, check_routing

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def u32_np(t):
    return t.contiguous().view(torch.int32).cpu().numpy().view(np.uint32)


def bf16_bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def make_layers(nv, n, n_experts=256, with_shared=True, seed=700, hidden=2048, inter=512,
                top_k=8):
    lag = importlib.import_module(PKG + ".laguna")
    cfg = lag.LagunaMoEConfig(n_experts=n_experts, hidden=hidden, inter=inter,
                              shared_inter=inter, top_k=top_k)
    made = [lag.random_sparse_layer(nv, seed=seed + l, device=DEV, cfg=cfg, n_experts=n_experts,
                                    with_shared=with_shared) for l in range(n)]
    return [m[0] for m in made], [m[1] for m in made]


EPS = 1e-6


def routed_stack(nv, blocks, x, residual=True, norms=None):
    """One call of the routed stack over `blocks`; returns (y, [(inds, wts)])."""
    lib = nv._lib.lib()
    n = len(blocks)
    Desc = nv._lib.MoeLayerDesc
    descs = (Desc * n)(*[b.desc for b in blocks])
    k = blocks[0].top_k
    inds = [torch.full((k,), 0xFFFF, dtype=torch.int32, device=DEV) for _ in range(n)]
    wts = [torch.zeros(k, dtype=torch.float32, device=DEV) for _ in range(n)]
    ip = (ctypes.c_void_p * n)(*[t.data_ptr() for t in inds])
    wp = (ctypes.c_void_p * n)(*[t.data_ptr() for t in wts])
    npp = None if norms is None else ctypes.cast(
        (ctypes.c_void_p * n)(*[w.data_ptr() for w in norms[:n]]), ctypes.c_void_p)
    ws = torch.zeros(lib.moe_decode_stack_workspace_size(descs, n), dtype=torch.uint8, device=DEV)
    y = torch.empty_like(x)
    stream = torch.cuda.current_stream().cuda_stream
    nv._lib.check(lib.moe_decode_stack_routed_forward(
        y.data_ptr(), x.data_ptr(), 0, n, descs, int(residual), npp, EPS,
        ctypes.cast(ip, ctypes.c_void_p), ctypes.cast(wp, ctypes.c_void_p), ws.data_ptr(),
        ws.numel(), stream))
    torch.cuda.synchronize()
    return y, list(zip(inds, wts))


def check_layer_routing(orc, x_bits, raw, inds, wts, k):
    """GPU routing vs the oracle router on the same x (one token, bf16 bits)."""
    gi, gw = u32_np(inds), wts.cpu().numpy()
    check_routing(orc, x_bits, bf16_bits(raw["router_w"]), raw["router_b"].cpu().numpy(),
                  gi.reshape(1, k), gw.reshape(1, k), k)
    return gi, gw


def banks_np(raw_part):
    return {n: (v.contiguous().view(torch.int32).cpu().numpy().view(np.uint32)
                if v.dtype in (torch.uint32, torch.int32) else v.cpu().numpy())
            for n, v in raw_part.items()}


def check_stack(nv, orc, blocks, raws, x0, residual=True, norm=True):
    L = len(blocks)
    k = blocks[0].top_k
    norms = [r["norm_w"] for r in raws] if norm else None
    y_full, routing = routed_stack(nv, blocks, x0, residual, norms)
    hs = [x0]
    for n in range(1, L):
        hs.append(routed_stack(nv, blocks[:n], x0, residual, norms)[0])
    hs.append(y_full)
    for l in range(L):
        inds, wts = routing[l]
        h_bits = bf16_bits(hs[l])
        x_bits = (orc.port.rms_norm_bf16(h_bits, bf16_bits(raws[l]["norm_w"]), EPS) if norm
                  else h_bits)
        gi, gw = check_layer_routing(orc, x_bits, raws[l], inds, wts, k)
        xl = orc.f32_from_bf16_bits(x_bits)
        hl = hs[l].float().cpu().numpy()
        want = orc.port.moe_block_f32(xl, gi.reshape(1, k), gw.reshape(1, k),
                                      banks_np(raws[l]["routed"]),
                                      banks_np(raws[l]["shared"]) if raws[l]["shared"] else None,
                                      scaling=2.5, residual=hl if residual else None)
        assert_close_bf16_out(hs[l + 1].float().cpu().numpy(), want, what=f"layer {l}")
    nv.device_status()  # raises on a latched index error or expired wait
    return y_full, routing


def test_routed_stack_layers_vs_oracle(nv, orc):
    """Laguna shapes (256 experts, top-8, shared expert), 6 decoder-layer MoE
    halves (RMSNorm, router, block, residual)."""
    blocks, raws = make_layers(nv, 6)
    g = torch.Generator(device=DEV).manual_seed(1)
    x0 = torch.randn(1, 2048, generator=g, device=DEV).to(torch.bfloat16)
    y, routing = check_stack(nv, orc, blocks, raws, x0)
    # the same bits again, routing included
    y2, routing2 = routed_stack(nv, blocks, x0, norms=[r["norm_w"] for r in raws])
    assert torch.equal(y, y2)
    for (a, b), (c, d) in zip(routing, routing2):
        assert torch.equal(a, c) and torch.equal(b, d)


def test_routed_stack_39_layers_vs_oracle(nv, orc):
    """The full Laguna stack: 39 sparse layers (two launches of 20 + 19 with the
    shared expert), every layer checked; the norm keeps each layer's input at
    unit scale, so the check is on live activations at every depth."""
    blocks, raws = make_layers(nv, 39, seed=2000)
    assert nv._lib.lib().moe_decode_stack_routed_launches(
        (nv._lib.MoeLayerDesc * 39)(*[b.desc for b in blocks]), 39) == 2
    g = torch.Generator(device=DEV).manual_seed(5)
    x0 = torch.randn(1, 2048, generator=g, device=DEV).to(torch.bfloat16)
    y, _ = check_stack(nv, orc, blocks, raws, x0)
    assert float(y.float().abs().max()) > 1.0


def test_routed_stack_across_launches_plain(nv, orc):
    """24 layers without the norm or the residual (x_{l+1} = block_l(x_l)): two
    launches (20 + 4), the second starting from the first's output."""
    blocks, raws = make_layers(nv, 24, n_experts=64, seed=900)
    g = torch.Generator(device=DEV).manual_seed(2)
    x0 = torch.randn(1, 2048, generator=g, device=DEV).to(torch.bfloat16)
    check_stack(nv, orc, blocks, raws, x0, residual=False, norm=False)


@pytest.mark.parametrize("hidden,inter,shared,top_k", [(1024, 512, False, 8),
                                                       (2048, 1024, True, 3)])
def test_routed_stack_other_shapes(nv, orc, hidden, inter, shared, top_k):
    """Shapes the routed stack's CTA pairs take besides Laguna's: hidden 1024
    (4 row tiles per CTA of a pair), inter 1024 (16 I blocks per segment)."""
    blocks, raws = make_layers(nv, 3, n_experts=128, with_shared=shared, seed=1100,
                               hidden=hidden, inter=inter, top_k=top_k)
    g = torch.Generator(device=DEV).manual_seed(3)
    x0 = torch.randn(1, hidden, generator=g, device=DEV).to(torch.bfloat16)
    check_stack(nv, orc, blocks, raws, x0)


def test_rms_norm_vs_oracle(nv, orc):
    """nvfp4_rms_norm against the oracle's RMSNorm (mlx/fast.cpp:90-108): the
    sums of squares differ in order only, so outputs agree to one bf16 step
    and almost all bits are equal; in place gives the same result."""
    g = torch.Generator(device=DEV).manual_seed(6)
    x = (torch.randn(8, 2048, generator=g, device=DEV) * 3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(2048, generator=g, device=DEV)).to(torch.bfloat16)
    y = nv.rms_norm(x, w, EPS)
    want = orc.port.rms_norm_bf16(bf16_bits(x), bf16_bits(w), EPS)
    got = bf16_bits(y)
    assert (got == want).mean() > 0.99
    gf, wf = orc.f32_from_bf16_bits(got), orc.f32_from_bf16_bits(want)
    assert np.all(np.abs(gf - wf) <= np.abs(wf) * 2.0 ** -7 + 1e-30)
    x2 = x.clone()
    nv.rms_norm(x2, w, EPS, out=x2)
    assert torch.equal(x2, y)
    y32 = nv.rms_norm(x.float(), w.float(), EPS)
    r = torch.rsqrt((x.float() ** 2).mean(-1, keepdim=True) + EPS)
    assert torch.allclose(y32, x.float() * r * w.float(), rtol=1e-5, atol=1e-6)


def test_routed_chain_matches_stack(nv):
    """MoEDecodeChain(route=True) runs the routed stack and, with stack=False,
    the per-layer router + block kernels; both follow the same layer
    semantics, so their outputs agree within the chained tolerance."""
    blocks, raws = make_layers(nv, 4, n_experts=64, seed=1300)
    norms = [r["norm_w"] for r in raws]
    g = torch.Generator(device=DEV).manual_seed(4)
    x0 = torch.randn(1, 2048, generator=g, device=DEV).to(torch.bfloat16)
    chain = nv.MoEDecodeChain(blocks, None, T=1, route=True, residual=True, norms=norms,
                              device=DEV).capture()
    assert chain.stack and chain.stack_fp4 and chain.launches_per_step() == 1
    chain.x0.copy_(x0)
    y = chain.replay().clone()
    per = nv.MoEDecodeChain(blocks, None, T=1, route=True, residual=True, norms=norms,
                            device=DEV, stack=False).capture()
    assert not per.stack and per.launches_per_step() == 16
    per.x0.copy_(x0)
    y_per = per.replay().clone()
    torch.cuda.synchronize()
    same = [set(u32_np(a[0]).ravel().tolist()) == set(u32_np(b[0]).ravel().tolist())
            for a, b in zip(chain.routing, per.routing)]
    if all(same):
        assert_close(y.float().cpu().numpy(), y_per.float().cpu().numpy(), rel_l2=5e-3 * 4,
                     max_abs=8e-2, what="stack vs per-layer")
    # the end-to-end call (pinned host in and out) gives the replay's result
    xh = x0.cpu().pin_memory()
    yh = chain(xh)
    assert torch.equal(yh, y.cpu())


def test_routed_stack_rejects(nv):
    """Shapes without a routed stack are refused with NVFP4_ERR_UNSUPPORTED."""
    blocks, _ = make_layers(nv, 1, n_experts=64, seed=1500)
    lib = nv._lib.lib()
    d = nv._lib.MoeLayerDesc.from_buffer_copy(blocks[0].desc)
    d.router_w = None
    descs = (nv._lib.MoeLayerDesc * 1)(d)
    x = torch.zeros(1, 2048, dtype=torch.bfloat16, device=DEV)
    ws = torch.zeros(lib.moe_decode_stack_workspace_size(descs, 1), dtype=torch.uint8, device=DEV)
    st = lib.moe_decode_stack_routed_forward(x.data_ptr(), x.data_ptr(), 0, 1, descs, 1, None,
                                             EPS, None, None, ws.data_ptr(), ws.numel(),
                                             torch.cuda.current_stream().cuda_stream)
    assert st == 1  # NVFP4_ERR_INVALID: no router weight
    with nv.launch_flags(exact_decode=True):
        assert lib.moe_decode_stack_routed_launches(
            (nv._lib.MoeLayerDesc * 1)(blocks[0].desc), 1) == 0
    # inter 1024 with top-8 and a shared expert: 9 x 16 I blocks do not fit
    # the grid as CTA pairs (the per-layer calls run it)
    wide, _ = make_layers(nv, 1, n_experts=64, seed=1600, inter=1024)
    assert lib.moe_decode_stack_routed_launches((nv._lib.MoeLayerDesc * 1)(wide[0].desc), 1) == 0
