"""GPU parity of the persistent decode stack (moe_decode_stack_forward): the
whole serial decode over L sparse layers in one cooperative launch.  Two
stacks: the default on the block-scaled FP4 tensor cores (activations as four
NVFP4 terms, tcgen05 kind::mxf4nvf4) and, with the exact_decode launch flag,
the mma.sync stack (the per-layer kernels' GEMV engine, partial products summed
in another order).  Either way a single layer must be within the BASELINE
tolerance of the fp32 oracle, an L-layer chain within L times the relative-L2
bound of the per-layer chains (every layer rounds its output to bf16 in both),
and replays are bit-for-bit repeatable."""
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


def make_chain(nv, blocks, routing, exact, dtype=torch.bfloat16):
    """A captured decode chain; exact selects the mma.sync stack."""
    with nv.launch_flags(exact_decode=exact):
        return nv.MoEDecodeChain(blocks, routing, T=1, dtype=dtype, device=DEV).capture()


@pytest.fixture(params=[False, True], ids=["fp4", "exact"])
def exact(request):
    return request.param


def layer_by_layer(blocks, routing, x):
    y = x
    for l, b in enumerate(blocks):
        y = b(y, inds=routing[l][0], weights=routing[l][1])
    return y


@pytest.mark.parametrize("with_shared,n", [(True, 2), (False, 2), (True, 5)])
def test_stack_matches_bulk_copy_layer_loop(nv, with_shared, n, exact):
    blocks, _, routing = layers(nv, n, with_shared=with_shared)
    chain = make_chain(nv, blocks, routing, exact)
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


def test_stack_matches_default_kernels_and_oracle(nv, orc, exact):
    blocks, raw, routing = layers(nv, 3, n_experts=256, seed=900)
    chain = make_chain(nv, blocks, routing, exact)
    assert chain.stack
    x = seeded_x(3)
    chain.x0.copy_(x)
    out = chain.replay()
    torch.cuda.synchronize()
    want = layer_by_layer(blocks, routing, x)  # per-thread-load kernels
    assert_close(out.float().cpu().numpy(), want.float().cpu().numpy(), max_abs=float("inf"),
                 rel_l2=chain_tol(3), what="stack vs default")
    # Layer 0 against the fp32 oracle (used experts only).
    one = make_chain(nv, blocks[:1], routing[:1], exact)
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


def oracle_layer(orc, raw, inds, wts, x):
    """The fp32 oracle block on x (float32 [1, H]) with the given routing (used
    experts only)."""
    inds = inds.cpu().numpy().astype(np.int64).reshape(1, -1)
    used = np.unique(inds)
    remap = {e: i for i, e in enumerate(used)}
    ids = torch.from_numpy(used).to(DEV)
    routed = {k: (u32_np(v.view(torch.int32)[ids]) if v.dtype == torch.uint32 else
                  v[ids].cpu().numpy()) for k, v in raw["routed"].items()}
    shared = None if raw["shared"] is None else {
        k: (u32_np(v) if v.dtype == torch.uint32 else v.cpu().numpy())
        for k, v in raw["shared"].items()}
    ci = np.vectorize(remap.get)(inds).astype(np.uint32)
    return orc.port.moe_block_f32(x, ci, wts.float().cpu().numpy().reshape(1, -1), routed,
                                  shared, scaling=2.5)


def test_stack_many_layers(nv, orc, exact):
    """39 layers (the model's sparse count, 3 distinct weight sets cycled),
    every layer checked against the fp32 oracle at the BASELINE bound: a stack
    of n layers returns x_n, and each launch computes a layer the same way
    whatever follows it, so the prefixes n = 1 .. 39 give every layer's input
    (bit-identical to the full stack's: the 39-layer prefix equals the full
    run).  Without a norm between the blocks the activations shrink layer by
    layer (the block is quadratic in its input) until, a few layers in, the
    SwiGLU activations fall below ~1e-30, where the stack stages a row as
    zeros (its term factors are clamped there): layers whose oracle output is
    below 1e-20 are checked for absolute agreement only.  The routed
    stack's test runs the same depth with RMSNorm and a live residual
    stream."""
    blocks, raw, routing = layers(nv, 3, seed=500)
    stack_blocks = [blocks[l % 3] for l in range(39)]
    stack_routing = [routing[l % 3] for l in range(39)]
    chain = make_chain(nv, stack_blocks, stack_routing, exact)
    assert chain.stack
    # with the shared expert the FP4 stack takes 20 layers per launch
    assert chain.launches_per_step() == (1 if exact else 2)
    x = seeded_x(39)
    chain.x0.copy_(x)
    full = chain.replay().clone()
    torch.cuda.synchronize()
    xs = [x]
    for n in range(1, 40):
        c = make_chain(nv, stack_blocks[:n], stack_routing[:n], exact)
        c.x0.copy_(x)
        xs.append(c.replay().clone())
        torch.cuda.synchronize()
    assert torch.equal(xs[39], full)
    live = 0
    for l in range(39):
        xl = xs[l].float().cpu().numpy()
        if l < 2:
            assert np.abs(xl).max() > 1e-3  # live activations in the first layers
        want = oracle_layer(orc, raw[l % 3], *stack_routing[l], xl)
        if np.abs(want).max() > 1e-20:
            assert_close(xs[l + 1].float().cpu().numpy(), want, what=f"layer {l}")
            live += 1
        else:
            assert_close(xs[l + 1].float().cpu().numpy(), want, rel_l2=float("inf"),
                         what=f"layer {l} (decayed)")
    assert live >= 3
    nv.device_status()


def test_stack_out_of_range_expert_is_reported(nv, exact):
    blocks, _, routing = layers(nv, 2, seed=700)
    bad = [(routing[0][0].clone(), routing[0][1]), routing[1]]
    bad[0][0][0, 3] = 999  # 32 experts
    chain = make_chain(nv, blocks, bad, exact)
    assert chain.stack
    chain.replay()
    with pytest.raises(nv.DeviceIndexError):
        nv.device_status()
    nv.device_status()  # the latch was cleared


@pytest.mark.parametrize("with_shared,n,launches", [(False, 42, 2), (True, 21, 2), (False, 40, 1)])
def test_fp4_stack_split_over_launches(nv, with_shared, n, launches):
    """More layers than one launch's tensor maps hold (40, 20 with a shared
    expert): the FP4 stack continues in a further launch from the previous
    one's per-segment partial sums.  Bit-identical to the same layers run as
    consecutive single-launch stacks.  (A long chain of SwiGLU layers without a
    residual is quadratic per layer, so it is compared with itself, not with
    another arithmetic.)"""
    blocks, _, routing = layers(nv, 3, with_shared=with_shared, seed=1300)
    sb = [blocks[l % 3] for l in range(n)]
    sr = [routing[l % 3] for l in range(n)]
    chain = make_chain(nv, sb, sr, False)
    assert chain.stack and chain.launches_per_step() == launches
    per = 20 if with_shared else 40
    x = seeded_x(n)
    chain.x0.copy_(x)
    out = chain.replay().clone()
    y = x
    # (no device synchronisation between the chains: each call is ordered
    # after the caller's stream, so two stacks never share the GPU)
    for a in range(0, n, per):
        part = make_chain(nv, sb[a:a + per], sr[a:a + per], False)
        assert part.launches_per_step() == 1
        part.x0.copy_(y)
        y = part.replay().clone()
    nv.device_status()
    assert torch.equal(out, y)


def test_stacks_tiny_input(nv, exact):
    """A row below 2^-100 (bf16 subnormals included) gives zeros, not NaN."""
    blocks, _, routing = layers(nv, 2, seed=1700)
    chain = make_chain(nv, blocks, routing, exact)
    chain.x0.copy_((seeded_x(3).float() * 1e-38).to(torch.bfloat16))
    out = chain.replay()
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert float(out.float().abs().max()) < 1e-30


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_fp4_stack_other_dtypes(nv, dtype):
    blocks, _, routing = layers(nv, 2, with_shared=True, seed=1500)
    chain = make_chain(nv, blocks, routing, False, dtype=dtype)
    assert chain.stack
    x = seeded_x(7).to(dtype)
    chain.x0.copy_(x)
    out = chain.replay()
    torch.cuda.synchronize()
    want = layer_by_layer(blocks, routing, x)
    assert out.dtype == dtype
    assert_close(out.float().cpu().numpy(), want.float().cpu().numpy(), max_abs=float("inf"),
                 rel_l2=chain_tol(2), what=f"FP4 stack, {dtype}")


@pytest.mark.parametrize("H,I,with_shared", [(2048, 1024, True), (1024, 512, True),
                                             (1024, 1024, False)])
def test_fp4_stack_other_shapes(nv, H, I, with_shared):
    """Layer shapes other than Laguna's that the FP4 stack takes (one K part of
    x per gate/up item at I = 1024, a half-width hidden size): the same layers
    through the per-layer kernels agree within the chain bound."""
    lag = importlib.import_module(PKG + ".laguna")
    cfg = lag.LagunaMoEConfig(hidden=H, inter=I, shared_inter=I, n_experts=32)
    n = 2
    blocks = [lag.random_sparse_layer(nv, seed=1900 + l, device=DEV, cfg=cfg, n_experts=32,
                                      with_shared=with_shared)[0] for l in range(n)]
    routing = [lag.random_routing(1, cfg, seed=2000 + l, device=DEV) for l in range(n)]
    chain = make_chain(nv, blocks, routing, False)
    assert chain.stack and chain.stack_fp4
    g = torch.Generator(device=DEV).manual_seed(H + I)
    x = torch.randn(1, H, generator=g, device=DEV).to(torch.bfloat16)
    chain.x0.copy_(x)
    out = chain.replay().clone()
    torch.cuda.synchronize()
    nv.device_status()
    want = layer_by_layer(blocks, routing, x)
    assert_close(out.float().cpu().numpy(), want.float().cpu().numpy(), max_abs=float("inf"),
                 rel_l2=chain_tol(n), what=f"FP4 stack H={H} I={I}")
    assert float(want.float().abs().max()) > 0


def test_stacks_nonfinite_input(nv, exact):
    """A non-finite activation gives a non-finite layer output, as the
    reference's products do (the FP4 stack writes NaN term factors for a run
    holding one)."""
    blocks, _, routing = layers(nv, 2, seed=2100)
    chain = make_chain(nv, blocks, routing, exact)
    x = seeded_x(11)
    x[0, 700] = float("inf")
    chain.x0.copy_(x)
    out = chain.replay()
    torch.cuda.synchronize()
    nv.device_status()  # raises on an expired bounded wait (or an index error)
    # inf in the token's x reaches every expert's gate/up sums, so every
    # activation and every output element is non-finite
    assert not bool(torch.isfinite(out.float()).any())
