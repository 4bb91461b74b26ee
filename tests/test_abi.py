"""The C-ABI library loads without a GPU, exports every symbol include/*.h
declares, and rejects invalid arguments on the host before touching CUDA."""
import ctypes
import glob
import importlib
import os
import re

import pytest

from conftest import PKG, ROOT


def declared_symbols():
    names = []
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        names += re.findall(r"NVFP4MOE_API\s+[\w\s\*]+?\b(\w+)\s*\(", src)
    return sorted(set(names))


def test_header_declares_the_boundary():
    names = declared_symbols()
    for n in ("nvfp4_gather_qmm", "nvfp4_quantized_matmul", "nvfp4_quantize", "nvfp4_dequantize",
              "moe_router_topk", "moe_block_forward", "nvfp4_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol(nv):
    L = ctypes.CDLL(nv.library_path())
    for n in declared_symbols():
        assert hasattr(L, n), n


def test_python_binding_covers_every_declared_symbol(nv):
    lib_mod = importlib.import_module(PKG + "._lib")
    assert set(declared_symbols()) == set(lib_mod.SIGNATURES)


def _last(L):
    return L.nvfp4_last_error().decode()


def test_invalid_group_shape_rejected_on_host(nv):
    L = nv._lib.lib()
    # K = 40 is not a multiple of the group size 16.
    st = L.nvfp4_gather_qmm(None, None, 0, None, None, None, None, 1, 1, 1, 1, 8, 40, 0, None)
    assert st == nv._lib.NVFP4_ERR_INVALID
    assert "[gather_qmm]" in _last(L) and "group size 16" in _last(L)


def test_bad_dtype_rejected(nv):
    L = nv._lib.lib()
    assert L.nvfp4_quantized_matmul(None, None, 7, None, None, 1, 16, 16, None) == 1
    assert "floating" in _last(L)


def test_empty_problem_is_a_no_op(nv):
    L = nv._lib.lib()
    assert L.nvfp4_gather_qmm(None, None, 0, None, None, None, None, 0, 0, 1, 1, 16, 32, 0,
                              None) == 0


def test_workspace_too_small_rejected(nv):
    L = nv._lib.lib()
    st = L.moe_router_topk(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 0,
                           ctypes.c_void_p(16), None, 4, 2048, 256, 8, 1, ctypes.c_void_p(16), 8,
                           None)
    assert st == nv._lib.NVFP4_ERR_WORKSPACE
    assert L.moe_router_workspace_size(4, 2048, 256) > 8


def test_error_handler_called(nv):
    L = nv._lib.lib()
    seen = []
    CB = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.c_void_p)
    cb = CB(lambda msg, data: seen.append(msg.decode()))
    L.nvfp4_set_error_handler(ctypes.cast(cb, ctypes.c_void_p), None)
    try:
        L.nvfp4_dequantize(None, 9, None, None, 1, 16, None)
    finally:
        L.nvfp4_set_error_handler(None, None)
    assert seen and "[dequantize]" in seen[0]


def test_moe_block_rejects_unaligned_shapes(nv):
    d = nv.MoeLayerDesc()
    d.hidden, d.inter, d.n_experts, d.top_k = 2000, 512, 256, 8
    L = nv._lib.lib()
    st = L.moe_block_forward(ctypes.c_void_p(16), ctypes.c_void_p(16), None, 0, 1,
                             ctypes.byref(d), None, None, None, None, None, 0, None)
    assert st == nv._lib.NVFP4_ERR_UNSUPPORTED


def test_host_mirror_errors_match_reference_kinds(nv):
    import torch
    w = torch.zeros(4, 32)
    with pytest.raises(ValueError, match="group size 16"):
        nv.quantize(w, group_size=64)
    with pytest.raises(ValueError, match="bits to be 4"):
        nv.quantize(w, bits=3)
    with pytest.raises(NotImplementedError):
        nv.quantize(w, mode="affine")
    with pytest.raises(ValueError, match="Biases must be null"):
        nv.gather_qmm(w, w, w, biases=w, rhs_indices=torch.zeros(1, dtype=torch.int32))
    with pytest.raises(ValueError, match="CUDA device"):
        nv.quantize(w)  # no CPU path


def test_decode_stack_rejects_unsupported_shapes(nv):
    d = (nv.MoeLayerDesc * 2)()
    for i in range(2):
        d[i].hidden, d[i].inter, d[i].n_experts, d[i].top_k = 2048, 512, 256, 8
    d[1].inter = 256  # layers must share one shape
    L = nv._lib.lib()
    ptrs = (ctypes.c_void_p * 2)(16, 16)
    st = L.moe_decode_stack_forward(ctypes.c_void_p(16), ctypes.c_void_p(16), 0, 2, d,
                                    ctypes.cast(ptrs, ctypes.c_void_p),
                                    ctypes.cast(ptrs, ctypes.c_void_p), None, 0, None)
    assert st in (nv._lib.NVFP4_ERR_UNSUPPORTED, nv._lib.NVFP4_ERR_INVALID)
    st = L.moe_decode_stack_forward(ctypes.c_void_p(16), ctypes.c_void_p(16), 0, 65, d,
                                    ctypes.cast(ptrs, ctypes.c_void_p),
                                    ctypes.cast(ptrs, ctypes.c_void_p), None, 0, None)
    assert st == nv._lib.NVFP4_ERR_UNSUPPORTED


@pytest.mark.parametrize("field,value", [("shared_inter", 256), ("inter", 1024),
                                         ("n_experts", 128), ("top_k", 4)])
def test_stacks_reject_layers_of_another_shape(nv, field, value):
    """Every layer of a decode stack must have layer 0's shape, the shared
    expert's width included (its tensor maps and work split come from layer
    0): a later layer that differs is refused on the host."""
    L = nv._lib.lib()
    D = nv._lib.MoeLayerDesc
    a = D()
    a.hidden, a.inter, a.n_experts, a.top_k, a.shared_inter = 2048, 512, 256, 8, 512
    a.routed_scaling, a.norm_topk_prob = 2.5, 1
    b = D.from_buffer_copy(a)
    setattr(b, field, value)
    descs = (D * 2)(a, b)
    assert L.moe_decode_stack_forward(None, None, 0, 2, descs, None, None, None, 0,
                                      None) == nv._lib.NVFP4_ERR_UNSUPPORTED
    assert "share one shape" in _last(L)
    assert L.moe_decode_stack_routed_forward(None, None, 0, 2, descs, 1, None, 1e-6, None, None,
                                             None, 0, None) == nv._lib.NVFP4_ERR_UNSUPPORTED
    assert "[moe_decode_stack_routed]" in _last(L)


def _laguna_desc(nv):
    d = nv._lib.MoeLayerDesc()
    d.hidden, d.inter, d.n_experts, d.top_k, d.shared_inter = 2048, 512, 256, 8, 512
    d.routed_scaling, d.norm_topk_prob = 2.5, 1
    return d


def test_long_batches_leave_the_fp4_gemms(nv):
    """The FP4 prefill GEMMs hold the tile list (E + T k / 32 + T / 32 entries)
    in shared memory; past ~13.8k tokens at Laguna sizes the block's workspace
    no longer carries the FP4 term buffers (the exact path takes the batch)."""
    L = nv._lib.lib()
    d = _laguna_desc(nv)
    fits, over = 13824, 13840
    w_fits = L.moe_block_workspace_size(ctypes.byref(d), fits)
    w_over = L.moe_block_workspace_size(ctypes.byref(d), over)
    # the four term rows per slot (codes, scales, factors of x and act) drop out
    assert w_over < w_fits - 9 * fits * 4 * (1024 + 256)


def test_ep_partial_refuses_a_tile_list_that_does_not_fit(nv):
    """moe_ep_partial_forward has no exact path: a batch whose FP4 tile list
    does not fit is refused on the host with NVFP4_ERR_UNSUPPORTED."""
    L = nv._lib.lib()
    d = _laguna_desc(nv)
    p = ctypes.c_void_p(256)
    T = 16384
    st = L.moe_ep_partial_forward(p, p, 2048, 0, T, ctypes.byref(d), p, p, 0, 0, T, p, 1 << 40,
                                  None)
    assert st == nv._lib.NVFP4_ERR_UNSUPPORTED
    assert "[moe_ep_partial]" in _last(L) and "tile" in _last(L)


@pytest.mark.parametrize("epr,k,shared", [(32, 8, True), (256, 8, True), (64, 16, False)])
def test_ep_chunk_rule_stays_inside_the_fp4_limit(nv, epr, k, shared):
    """ep.py's row-range rule (MAX_TILES entries) never asks the library for a
    batch its FP4 GEMMs would refuse: the largest range the rule allows is
    below the size at which the workspace stops carrying the FP4 buffers."""
    ep = importlib.import_module(PKG + ".ep")
    L = nv._lib.lib()
    d = _laguna_desc(nv)
    d.n_experts, d.top_k = epr, k
    d.shared_inter = 512 if shared else 0

    def ws(T):
        return L.moe_ep_partial_workspace_size(ctypes.byref(d), T)

    # Past the limit the layout is the exact path's, whose size per token is
    # the asymptote below; the FP4 term buffers add >= 4 terms x H/2 bytes of
    # codes per slot on top, so "FP4 included" is a per-token size well above it.
    big = 1 << 18
    exact_per_token = ws(big) / big
    slots = k + (1 if shared else 0)
    margin = slots * 4 * (2048 // 2) / 2

    def has_fp4(T):
        return ws(T) / T > exact_per_token + margin

    lo, hi = 16, big  # a prefill-sized batch (below 2 tokens there is no prefill layout)
    assert has_fp4(lo) and not has_fp4(hi)
    while hi - lo > 1:
        mid = (lo + hi) // 2
        if has_fp4(mid):
            lo = mid
        else:
            hi = mid
    limit = lo  # largest T whose layout still carries the FP4 buffers

    class Ops:
        MAX_TILES = ep.CudaGatherEPOps.MAX_TILES

        class local:
            desc = d

    o = Ops()
    o.epr, o.top_k = epr, k
    c_max = 1
    while True:  # the largest single range the rule accepts
        t = epr + -(-(c_max + 1) * k // 32) + (-(-(c_max + 1) // 32) if shared else 0)
        if t > o.MAX_TILES:
            break
        c_max += 1
    assert ep.CudaGatherEPOps.chunk_tokens(o, c_max) == c_max
    assert c_max <= limit
