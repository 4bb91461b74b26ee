"""The bounded waits of the block-scaled FP4 decode stacks give up, report
their site and leave the context usable.

With the test-only launch flag NVFP4_LAUNCH_TEST_EXPIRE the last layer's
segment-0 gate/up items never make their release, so the down items of that
segment wait on a counter that nothing increments; every wait is ~1 ms under
the flag.  The launch must return, nvfp4_device_status() must report
NVFP4_ERR_DEVICE_TIMEOUT naming a wait of the last layer (site 1000 *
(last layer + 1) + 40..59: the down item's counter wait, or its MMA warp's
wait for the act terms, whichever gave up first), and the next call without
the flag must give the normal result.  No GPU
fault, trap or endless wait is involved: the waits are bounded and the
kernel drains its copies and tensor-core work before it exits.
"""
import ctypes
import importlib

import pytest
import torch

from conftest import PKG, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def make_layers(nv, n, seed):
    lag = importlib.import_module(PKG + ".laguna")
    cfg = lag.LagunaMoEConfig(n_experts=64)
    made = [lag.random_sparse_layer(nv, seed=seed + l, device=DEV, cfg=cfg, n_experts=64)
            for l in range(n)]
    routing = [lag.random_routing(1, cfg, seed=seed + 50 + l, device=DEV) for l in range(n)]
    return [m[0] for m in made], [m[1] for m in made], routing


def call_with_expiry(nv, chain):
    lib = nv._lib.lib()
    old = lib.nvfp4_set_launch_flags(nv._lib.NVFP4_LAUNCH_TEST_EXPIRE)
    try:
        st = chain._stack_call(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    finally:
        lib.nvfp4_set_launch_flags(old)
    assert st == 0  # the launch itself is valid; the waits run out on the device
    with pytest.raises(nv.DeviceTimeoutError, match=r"kernel site 30[45][0-9]"):
        nv.device_status()


def test_given_routing_stack_wait_expires_and_recovers(nv):
    blocks, _, routing = make_layers(nv, 3, seed=5100)
    chain = nv.MoEDecodeChain(blocks, routing, T=1, device=DEV)
    assert chain.stack and chain.stack_fp4
    x = torch.randn(1, 2048, device=DEV).to(torch.bfloat16)
    chain.x0.copy_(x)
    call_with_expiry(nv, chain)
    # the next call, without the flag, is correct
    nv._lib.check(chain._stack_call(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    nv.device_status()
    want = x
    for l, b in enumerate(blocks):
        want = b(want, inds=routing[l][0], weights=routing[l][1])
    assert_close(chain.bufs[0].float().cpu().numpy(), want.float().cpu().numpy(),
                 max_abs=float("inf"), rel_l2=1.5e-2, what="after expiry")


def test_routed_stack_wait_expires_and_recovers(nv):
    blocks, raws, _ = make_layers(nv, 3, seed=5200)
    norms = [r["norm_w"] for r in raws]
    chain = nv.MoEDecodeChain(blocks, None, T=1, route=True, residual=True, norms=norms,
                              device=DEV)
    assert chain.stack and chain.stack_fp4
    x = torch.randn(1, 2048, device=DEV).to(torch.bfloat16)
    chain.x0.copy_(x)
    sp = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    nv._lib.check(chain._stack_call(sp))
    torch.cuda.synchronize()
    good = chain.bufs[0].clone()
    call_with_expiry(nv, chain)
    nv._lib.check(chain._stack_call(sp))
    torch.cuda.synchronize()
    nv.device_status()
    assert torch.equal(chain.bufs[0], good)  # the same bits as before the expiry
