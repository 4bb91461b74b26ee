"""moe_block_forward_noalloc: the MoE block for callers that cannot allocate
device memory (hosts that only pass tensor pointers through an operator
interface, or that must keep a fixed device-memory footprint).  It uses the
library's static device scratch instead of a caller workspace.

Checked through the C ABI against moe_block_forward (caller workspace), on two
calls in a row, within the output tolerance the other block tests use.  The
file is named to be collected last; it passes alone in a fresh process too.
"""
import ctypes
import importlib

import pytest
import torch

from conftest import PKG, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def layer(nv):
    lag = importlib.import_module(PKG + ".laguna")
    block, raw = lag.random_sparse_layer(nv, seed=4321, device=DEV, n_experts=64)
    return lag, block, raw


def _noalloc(nv, block, x, residual=None, inds=None, wts=None):
    T = x.shape[0]
    y = torch.empty_like(x)
    inds_out = torch.empty(T, block.top_k, dtype=torch.int32, device=DEV)
    wts_out = torch.empty(T, block.top_k, dtype=torch.float32, device=DEV)
    L = nv._lib.lib()
    st = L.moe_block_forward_noalloc(
        y.data_ptr(), x.data_ptr(), None if residual is None else residual.data_ptr(),
        nv._dtype_code(x, "noalloc"), T, ctypes.byref(block.desc),
        None if inds is None else inds.data_ptr(), None if wts is None else wts.data_ptr(),
        inds_out.data_ptr(), wts_out.data_ptr(),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    nv._lib.check(st)
    return y, inds_out, wts_out


@pytest.mark.parametrize("T", [1, 8])
def test_noalloc_matches_workspace_entry_point_twice(nv, layer, T):
    lag, block, raw = layer
    g = torch.Generator(device=DEV).manual_seed(T)
    x = torch.randn(T, 2048, generator=g, device=DEV).to(torch.bfloat16)
    res = torch.randn(T, 2048, generator=g, device=DEV).to(torch.bfloat16)
    want, winds, wwts = block(x, residual=res, return_routing=True)
    for _ in range(2):  # the static scratch keeps the previous call's contents
        got, inds, wts = _noalloc(nv, block, x, residual=res)
        torch.cuda.synchronize()
        assert torch.equal(inds.view(torch.uint32), winds)
        assert_close(wts.cpu().numpy(), wwts.cpu().numpy(), max_abs=1e-6, rel_l2=1e-6)
        assert_close(got.float().cpu().numpy(), want.float().cpu().numpy(), what=f"noalloc T={T}")


def test_noalloc_with_given_routing(nv, layer):
    lag, block, raw = layer
    inds, wts = lag.random_routing(3, lag.LagunaMoEConfig(n_experts=64), seed=9, device=DEV)
    x = torch.randn(3, 2048, device=DEV).to(torch.bfloat16)
    want = block(x, inds=inds, weights=wts)
    for _ in range(2):
        got, _, _ = _noalloc(nv, block, x, inds=inds, wts=wts)
        torch.cuda.synchronize()
        assert_close(got.float().cpu().numpy(), want.float().cpu().numpy(), what="given routing")


def test_noalloc_rejects_sizes_beyond_its_scratch(nv, layer):
    lag, block, raw = layer
    x = torch.zeros(64, 2048, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="static scratch"):
        _noalloc(nv, block, x)


def test_noalloc_at_its_documented_limit(nv):
    """The documented limit at Laguna XS 2.1 sizes: T = 8 tokens with all 256
    experts (the router's partial logits are then the largest user of the
    scratch), the shared expert and a residual, twice in a row; T = 9 is
    refused."""
    lag = importlib.import_module(PKG + ".laguna")
    block, raw = lag.random_sparse_layer(nv, seed=8765, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(88)
    x = torch.randn(8, 2048, generator=g, device=DEV).to(torch.bfloat16)
    res = torch.randn(8, 2048, generator=g, device=DEV).to(torch.bfloat16)
    want, winds, _ = block(x, residual=res, return_routing=True)
    for _ in range(2):
        got, inds, _ = _noalloc(nv, block, x, residual=res)
        torch.cuda.synchronize()
        assert torch.equal(inds.view(torch.uint32), winds)
        assert_close(got.float().cpu().numpy(), want.float().cpu().numpy(),
                     what="noalloc T=8 E=256")
    with pytest.raises(ValueError, match="static scratch"):
        _noalloc(nv, block, torch.zeros(9, 2048, device=DEV, dtype=torch.bfloat16))
