"""GPU parity of the tensor-core (tcgen05) prefill path: the dense
quantized_matmul for M > 8 rows (BASELINE config[0] at M=512) and the
sorted-expert MoE block for T > 8 tokens (config[3] at T=512), against the
fp32 oracle on sampled rows / tokens and against the independent decode-path
kernels on every token.  The block runs both ways: the default block-scaled
FP4 path (activations as four NVFP4 terms) and the exact 16-bit path."""
import importlib

import numpy as np
import pytest
import torch

from conftest import PKG, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def u32_np(t):
    return t.contiguous().view(torch.int32).cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("M,N,K", [(9, 256, 256), (32, 512, 2048), (65, 2048, 512),
                                   (512, 4096, 2048), (100, 130, 192)])
def test_dense_qmm_tensor_core_vs_oracle(nv, orc, M, N, K):
    g = torch.Generator(device=DEV).manual_seed(M + N + K)
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    wq, sq = nv.quantize(w)
    x = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
    y = nv.quantized_matmul(x, wq, sq)
    rows = np.unique(np.linspace(0, M - 1, min(M, 24)).astype(int))
    want = orc.port.qmm_f32(x[rows].float().cpu().numpy(), u32_np(wq), sq.cpu().numpy())
    assert_close(y[rows].float().cpu().numpy(), want, what=f"qmm M={M} N={N} K={K}")


def test_dense_qmm_tensor_core_matches_gemv_path(nv):
    """Rows computed by the tcgen05 GEMM equal (within tolerance) the same rows
    through the decode GEMV (8 rows at a time)."""
    g = torch.Generator(device=DEV).manual_seed(1)
    w = (torch.randn(1024, 2048, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    wq, sq = nv.quantize(w)
    x = torch.randn(128, 2048, generator=g, device=DEV).to(torch.bfloat16)
    y = nv.quantized_matmul(x, wq, sq)
    y8 = torch.cat([nv.quantized_matmul(x[i:i + 8], wq, sq) for i in range(0, 128, 8)])
    assert_close(y.float().cpu().numpy(), y8.float().cpu().numpy(), what="gemm vs gemv")


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_dense_qmm_tensor_core_dtypes(nv, orc, dtype):
    g = torch.Generator(device=DEV).manual_seed(2)
    w = (torch.randn(256, 512, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    wq, sq = nv.quantize(w)
    x = torch.randn(40, 512, generator=g, device=DEV).to(dtype)
    y = nv.quantized_matmul(x, wq, sq)
    assert y.dtype == dtype
    want = orc.port.qmm_f32(x.float().cpu().numpy(), u32_np(wq), sq.cpu().numpy())
    assert_close(y.float().cpu().numpy(), want, what=str(dtype))


@pytest.fixture(scope="module")
def layer(nv):
    lag = importlib.import_module(PKG + ".laguna")
    block, raw = lag.random_sparse_layer(nv, seed=777, device=DEV)
    return lag, block, raw


def oracle_tokens(orc, raw, x, inds, wts, tokens, residual=None):
    inds_np = inds.cpu().numpy().astype(np.int64)[tokens]
    used = np.unique(inds_np)
    remap = {e: i for i, e in enumerate(used)}
    ids = torch.from_numpy(used).to(DEV)
    routed = {k: (u32_np(v.view(torch.int32)[ids]) if v.dtype == torch.uint32
                  else v[ids].cpu().numpy()) for k, v in raw["routed"].items()}
    shared = {k: (u32_np(v) if v.dtype == torch.uint32 else v.cpu().numpy())
              for k, v in raw["shared"].items()}
    ci = np.vectorize(remap.get)(inds_np).astype(np.uint32)
    res = None if residual is None else residual.float().cpu().numpy()[tokens]
    return orc.port.moe_block_f32(x.float().cpu().numpy()[tokens], ci,
                                  wts.float().cpu().numpy()[tokens], routed, shared,
                                  scaling=2.5, residual=res)


@pytest.mark.parametrize("exact", [False, True])
@pytest.mark.parametrize("T", [9, 64, 512])
def test_prefill_block_vs_oracle_and_decode_path(nv, orc, layer, T, exact):
    lag, block, raw = layer
    g = torch.Generator(device=DEV).manual_seed(T)
    x = torch.randn(T, 2048, generator=g, device=DEV).to(torch.bfloat16)
    res = torch.randn(T, 2048, generator=g, device=DEV).to(torch.bfloat16)
    with nv.launch_flags(exact_prefill=exact):
        y, inds, wts = block(x, residual=res, return_routing=True)
    nv.device_status()
    assert torch.isfinite(y.float()).all()
    # Oracle on sampled tokens (tokens are independent).
    tokens = np.unique(np.linspace(0, T - 1, min(T, 12)).astype(int))
    want = oracle_tokens(orc, raw, x, inds, wts, tokens, residual=res)
    assert_close(y.float().cpu().numpy()[tokens], want, what=f"prefill T={T} vs oracle")
    # Every token against the decode-path kernels, 8 tokens per call, same routing.
    # Both results are rounded to bf16, so two outputs may sit one bf16 ulp apart
    # (0.031 at |y| in [4, 8)): max-abs 4e-2, relative-L2 at the usual 5e-3.
    parts = [block(x[i:i + 8], residual=res[i:i + 8], inds=inds[i:i + 8].view(torch.int32),
                   weights=wts[i:i + 8]) for i in range(0, T, 8)]
    assert_close(y.float().cpu().numpy(), torch.cat(parts).float().cpu().numpy(),
                 max_abs=4e-2, what=f"prefill T={T} vs decode path")


@pytest.mark.parametrize("exact", [False, True])
def test_prefill_given_routing_with_skew(nv, orc, layer, exact):
    """Heavily skewed routing: one expert takes every token (many tiles per expert)."""
    lag, block, raw = layer
    T = 200
    inds = torch.stack([torch.tensor([5, 9, 17, 33, 64, 100, 200, 255]) for _ in range(T)])
    inds[:, 0] = 3  # expert 3 gets all 200 tokens
    wts = torch.softmax(torch.randn(T, 8), dim=-1)
    inds, wts = inds.to(torch.int32).to(DEV), wts.to(DEV)
    x = torch.randn(T, 2048, device=DEV).to(torch.bfloat16)
    with nv.launch_flags(exact_prefill=exact):
        y = block(x, inds=inds, weights=wts)
    tokens = np.array([0, 31, 32, 63, 64, 127, 128, 199])
    want = oracle_tokens(orc, raw, x, inds, wts, tokens)
    assert_close(y.float().cpu().numpy()[tokens], want, what="skewed routing")


def test_prefill_fp4_terms_close_to_exact_path(nv, layer):
    """The four-term FP4 path against the exact 16-bit path on the same
    routing: both round to bf16, so they differ by bf16 rounding flips only
    (relative-L2 well under 1e-3, the terms themselves ~5e-5)."""
    lag, block, raw = layer
    g = torch.Generator(device=DEV).manual_seed(4)
    x = torch.randn(512, 2048, generator=g, device=DEV).to(torch.bfloat16)
    y0, inds, wts = block(x, return_routing=True)
    with nv.launch_flags(exact_prefill=True):
        y1 = block(x, inds=inds.view(torch.int32), weights=wts)
    nv.device_status()
    assert_close(y0.float().cpu().numpy(), y1.float().cpu().numpy(), max_abs=4e-2, rel_l2=1e-3,
                 what="fp4 terms vs exact")


def test_long_prompt_takes_the_exact_path(nv, orc, layer):
    """T = 14336 at Laguna sizes: the FP4 GEMMs' tile list (E + T*k/32 + T/32
    entries) no longer fits in shared memory, so the block runs on the exact
    path -- the same bits as the exact path on the two halves (tokens are
    independent), and within tolerance of the oracle on sampled tokens."""
    lag, block, raw = layer
    T, h = 14336, 7168
    g = torch.Generator(device=DEV).manual_seed(14)
    x = torch.randn(T, 2048, generator=g, device=DEV).to(torch.bfloat16)
    res = torch.randn(T, 2048, generator=g, device=DEV).to(torch.bfloat16)
    y, inds, wts = block(x, residual=res, return_routing=True)
    with nv.launch_flags(exact_prefill=True):
        halves = [block(x[i:i + h], residual=res[i:i + h]) for i in (0, h)]
    nv.device_status()
    assert torch.equal(y, torch.cat(halves))
    tokens = np.array([0, 4097, 9000, T - 1])
    want = oracle_tokens(orc, raw, x, inds, wts, tokens, residual=res)
    assert_close(y.float().cpu().numpy()[tokens], want, what="T=14336 vs oracle")


@pytest.mark.parametrize("exact", [False, True])
def test_prefill_non_finite_rows_propagate(nv, layer, exact):
    """A token whose activations hold NaN or inf gives a non-finite output row,
    as in the reference; the other tokens are unaffected."""
    lag, block, raw = layer
    g = torch.Generator(device=DEV).manual_seed(8)
    x = torch.randn(40, 2048, generator=g, device=DEV).to(torch.bfloat16)
    y0, inds, wts = block(x, return_routing=True)
    x[3, 100] = float("nan")
    x[7, 5] = float("inf")
    with nv.launch_flags(exact_prefill=exact):
        y = block(x, inds=inds.view(torch.int32), weights=wts)
    nv.device_status()
    bad = ~torch.isfinite(y.float()).all(dim=1)
    assert bad[3] and bad[7]
    keep = [i for i in range(40) if i not in (3, 7)]
    assert torch.isfinite(y[keep].float()).all()
    assert_close(y[keep].float().cpu().numpy(), y0[keep].float().cpu().numpy(), max_abs=4e-2,
                 what="finite rows unchanged")
