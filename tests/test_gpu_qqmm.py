"""GPU parity of the NVFP4 x NVFP4 matmul (qqmm / QQMatmul, mode "nvfp4").

Bars: the activation quantisation is bit-exact against the oracle (which is
pinned bit-exactly to the reference's fp_quantize_dequantize); the matmul is
within max-abs 2e-2 / relative-L2 5e-3 of the fp32-accumulated oracle, and,
with f32 activations (f32 output, no output rounding), within relative-L2
1e-5: every product is exact, only the f32 summation order differs.
"""
import numpy as np
import pytest
import torch

from conftest import assert_close, close_report

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def to_dev_u32(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(DEV).view(torch.uint32)


def u32_np(t):
    return t.view(torch.int32).cpu().numpy().view(np.uint32)


def weights(orc, N, K, seed):
    rng = np.random.default_rng(seed)
    w = orc.bf16_bits_from_f32((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    return orc.port.quantize(w)


def edge_rows(K, dtype):
    """Rows with every special group the quantiser distinguishes."""
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((10, K)) * rng.choice([1e-6, 1e-3, 1, 30, 1e4], (10, 1))).astype(
        np.float32)
    x[0, :16] = 0.0
    x[1, :16] = [6, 3, 0.25, -0.25, 0.75, -0.75, 1.25, -1.25, 1.75, 2.5, -3.5, 5, -5, 0.5, -0.5, 0]
    x[2, :16] = -0.0
    x[3, 16:32] = 1e-30  # scale encodes to 0
    if dtype == torch.float32:
        x[4, :16] = np.nan  # all-NaN group: MLX scale byte 0xFE
        x[5, :16] = [np.nan] * 8 + [1.0] * 8
        x[6, :16] = np.inf
        x[7, 32:48] = -np.inf
    t = torch.from_numpy(x).to(DEV).to(dtype)
    return t


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_quantize_activations_bit_exact(nv, orc, dtype):
    x = edge_rows(512, dtype)
    xq, s = nv.quantize_activations(x)
    oq, os_ = orc.port.quantize_x(x.float().cpu().numpy())
    assert np.array_equal(u32_np(xq), oq)
    assert np.array_equal(s.cpu().numpy(), os_)


def test_quantize_activations_golden_xhat(nv, golden):
    x = torch.from_numpy(golden["qqmm_fq_in"]).to(DEV)
    xq, s = nv.quantize_activations(x)
    xhat = nv.dequantize(xq, s, dtype=torch.float32).cpu().numpy()
    assert np.array_equal(xhat.view(np.uint32), golden["qqmm_fq_out"].view(np.uint32))


def test_qqmm_golden(nv, orc, golden):
    wq, sq = to_dev_u32(golden["qqmm_wq"]), torch.from_numpy(golden["qqmm_sq"]).to(DEV)
    x = torch.from_numpy(golden["qqmm_x_f32"]).to(DEV)
    y = nv.qqmm(x, wq, sq).cpu().numpy()
    ma, rl = close_report(y, golden["qqmm_y_f32"])
    assert rl <= 1e-5 and ma <= 1e-4, (ma, rl)
    # bf16 x: quantised from its bf16 values (golden qqmm_x_bf16), so the target
    # is the f32 form on those values.
    xb = torch.from_numpy(golden["qqmm_x_bf16"].view(np.int16)).to(DEV).view(torch.bfloat16)
    want = orc.port.qqmm_f32(orc.f32_from_bf16_bits(golden["qqmm_x_bf16"]), golden["qqmm_wq"],
                             golden["qqmm_sq"])
    assert_close(nv.qqmm(xb, wq, sq).float().cpu().numpy(), want, what="bf16")


@pytest.mark.parametrize("M,N,K", [(1, 128, 256), (1, 4096, 2048), (2, 200, 512), (8, 384, 2048),
                                   (17, 128, 1024), (40, 256, 768), (64, 512, 512),
                                   (130, 256, 512), (512, 256, 2048)])
def test_qqmm_vs_oracle(nv, orc, M, N, K):
    wq, sq = weights(orc, N, K, seed=M * 7 + N)
    rng = np.random.default_rng(M + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    want = orc.port.qqmm_f32(x, wq, sq)
    dw, ds = to_dev_u32(wq), torch.from_numpy(sq).to(DEV)
    y32 = nv.qqmm(torch.from_numpy(x).to(DEV), dw, ds).cpu().numpy()
    ma, rl = close_report(y32, want)
    assert rl <= 1e-5, (ma, rl)
    xb = torch.from_numpy(x).to(DEV).to(torch.bfloat16)
    want_b = orc.port.qqmm_f32(xb.float().cpu().numpy(), wq, sq)
    assert_close(nv.qqmm(xb, dw, ds).float().cpu().numpy(), want_b, what=f"bf16 {M}x{N}x{K}")


def test_qqmm_full_size_vs_torch_fp32(nv):
    """config[0] at M=512 (N=4096, K=2048): against the same op in plain torch
    fp32 on the bit-exact dequantised operands (TF32 off)."""
    g = torch.Generator(device=DEV).manual_seed(5)
    w = (torch.randn(4096, 2048, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    wq, sq = nv.quantize(w)
    x = torch.randn(512, 2048, generator=g, device=DEV).to(torch.bfloat16)
    xq, xs = nv.quantize_activations(x)
    xhat = nv.dequantize(xq, xs, dtype=torch.float32)
    wd = nv.dequantize(wq, sq, dtype=torch.float32)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        want = (xhat @ wd.t()).cpu().numpy()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    got = nv.qqmm(x, wq, sq).float().cpu().numpy()
    assert_close(got, want, what="qqmm 512x4096x2048")
    got32 = nv.qqmm(x.float(), wq, sq).cpu().numpy()
    ma, rl = close_report(got32, want)
    assert rl <= 1e-5, (ma, rl)


def test_qqmm_vector_and_errors(nv, orc):
    wq, sq = weights(orc, 256, 512, seed=1)
    dw, ds = to_dev_u32(wq), torch.from_numpy(sq).to(DEV)
    x = torch.randn(512, device=DEV)
    y = nv.qqmm(x, dw, ds)
    assert y.shape == (256,)
    assert_close(y.cpu().numpy(), orc.port.qqmm_f32(x.cpu().numpy()[None], wq, sq)[0])
    with pytest.raises(ValueError):
        nv.qqmm(torch.randn(2, 3, 512, device=DEV), dw, ds)
    with pytest.raises(NotImplementedError):  # K % 256 != 0 is outside the tensor-core path
        wq2, sq2 = weights(orc, 128, 272, seed=2)
        nv.qqmm(torch.randn(1, 272, device=DEV), to_dev_u32(wq2), torch.from_numpy(sq2).to(DEV))
    assert nv.qqmm(torch.empty(0, 512, device=DEV), dw, ds).shape == (0, 256)
    nv.device_status()
