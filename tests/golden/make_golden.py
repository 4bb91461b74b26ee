"""Generate tests/golden/nvfp4_golden.npz from the reference's OWN compiled code.

Run in a container that has the reference tree (oracle/_ref/libmlxref.so built
by oracle/Makefile from Vendor/mlx-swift/Source/Cmlx/mlx/mlx/backend/cpu/
quantized.cpp).  Every output array below is produced by reference code:

  e4m3_decode      detail::FromFP8 over all 256 bytes   (backend/cpu/unary_ops.h:154-172)
  e4m3_enc_*       detail::ToFP8 on a fixed sample      (unary_ops.h:120-151)
  sigmoid_*        detail::Sigmoid on a fixed sample    (unary_ops.h:77-84)
  qmm_*            fp_qmm_t<float|bfloat16_t,16,4>      (backend/cpu/quantized.cpp:491-533)
  gather_*         the fp_bs_qmm_dispatch_mode loop     (quantized.cpp:805-844)
  fp4_enc_*        to_fp4_e2m1 on a fixed sample        (backend/cpu/quantized.cpp:1064-1091)
  qqmm_*           QQMatmul::eval_cpu's two steps: the fp_quantize_dequantize
                   group loop (quantized.cpp:1093-1129) over the reference's
                   ToFP8 / dequantize_scale / to_fp4_e2m1 / FP4_LUT, then
                   fp_qmm_t<float|bfloat16_t> on xhat (quantized.cpp:1322-1360)
  quant_*          the fp_quantize graph (ops.cpp:4909-4962) composed from the
                   reference's compiled scalar ops: bf16 division
                   (_MLX_BFloat16 operator/, types/bf16.h:71-99), ToFP8,
                   FromFP8 and the first-minimum argmin (arg_reduce.cpp:41-47).
The packed weights fed to qmm/gather are produced by the oracle's quantizer
(the reference quantizer is an MLX op graph that needs the full MLX runtime),
and quant_* pins that quantizer separately.

Seeds: numpy PCG64, fixed per array.  Usage:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "nvfp4_golden.npz")
LUT = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], np.float32)


def ref_quantize_bf16(ref, w_bits):
    """fp_quantize (ops.cpp:4909-4962) for bf16 w, one op at a time, with the
    reference's compiled scalar ops."""
    L = ref.lib
    rows, K = w_bits.shape
    six = L.ref_bf16_from_f32(6.0)
    wq = np.zeros((rows, K // 8), np.uint32)
    sq = np.zeros((rows, K // 16), np.uint8)
    lut_bf16 = [oracle.f32_from_bf16_bits(np.array([L.ref_bf16_from_f32(float(v))], np.uint16))[0]
                for v in LUT]
    for r in range(rows):
        for g in range(K // 16):
            grp = w_bits[r, 16 * g:16 * g + 16]
            mags = np.abs(oracle.f32_from_bf16_bits(grp))
            amax_bits = oracle.bf16_bits_from_f32(np.array([mags.max()], np.float32))[0]
            scale_bits = L.ref_bf16_div(int(amax_bits), int(six))          # bf16 divide
            scale_f32 = oracle.f32_from_bf16_bits(np.array([scale_bits], np.uint16))[0]
            sb = L.ref_to_fp8(float(scale_f32))                             # * f32 1.0, ToFP8
            sdec_bits = L.ref_bf16_from_f32(L.ref_from_fp8(sb))             # FromFP8 -> bf16
            sq[r, g] = sb
            for j in range(16):
                q_bits = L.ref_bf16_div(int(grp[j]), int(sdec_bits))         # bf16 divide
                q = oracle.f32_from_bf16_bits(np.array([q_bits], np.uint16))[0]
                best, bv = 0, abs(np.float32(q) - lut_bf16[0])
                for i in range(1, 16):                                       # argmin, first wins
                    d = abs(np.float32(q) - lut_bf16[i])
                    if d < bv:
                        best, bv = i, d
                wq[r, (16 * g + j) // 8] |= np.uint32(best) << np.uint32(4 * (j % 8))
    return wq, sq


def main():
    ref, port = oracle.ref, oracle.port
    if ref is None:
        raise SystemExit("oracle/_ref/libmlxref.so missing: build it with `make -f oracle/Makefile`"
                         " in a container that has the reference tree")
    L = ref.lib
    g = {}
    g["e4m3_decode"] = np.array([L.ref_from_fp8(b) for b in range(256)], np.float32)

    rng = np.random.default_rng(0)
    enc_in = np.concatenate([
        np.array([0, -0., 1e-9, 2**-10, 2**-9, 1.5 * 2**-9, 0.001953125, 0.1666, 1 / 6, 448, 449,
                  464, 465, 480, 1e4, np.inf, -np.inf, np.nan, -3.25, 0.3125], np.float32),
        (rng.standard_normal(2000) * rng.choice([1e-3, 1e-2, 0.1, 1, 50, 400], 2000)).astype(
            np.float32)])
    g["e4m3_enc_in"] = enc_in
    g["e4m3_enc_out"] = np.array([L.ref_to_fp8(float(v)) for v in enc_in], np.uint8)

    sig_in = (rng.standard_normal(512) * 6).astype(np.float32)
    g["sigmoid_in"] = sig_in
    g["sigmoid_out"] = np.array([L.ref_sigmoid(float(v)) for v in sig_in], np.float32)

    # Dense qmm: W bf16 [64, 256] ~ N(0, 0.02), x [4, 256] ~ N(0, 1).
    rng = np.random.default_rng(1)
    w = oracle.bf16_bits_from_f32((rng.standard_normal((64, 256)) * 0.02).astype(np.float32))
    wq, sq = port.quantize(w)
    x = rng.standard_normal((4, 256)).astype(np.float32)
    xb = oracle.bf16_bits_from_f32(x)
    g["qmm_w_bf16"], g["qmm_wq"], g["qmm_sq"] = w, wq, sq
    g["qmm_x_f32"], g["qmm_x_bf16"] = x, xb
    g["qmm_y_f32"] = ref.qmm_f32(x, wq, sq)
    g["qmm_y_bf16"] = ref.qmm_bf16(xb, wq, sq)

    # Gather: 6 experts [32, 128], x [3, 2, 128], 5 pairs.
    rng = np.random.default_rng(2)
    we = oracle.bf16_bits_from_f32((rng.standard_normal((6, 32, 128)) * 0.02).astype(np.float32))
    gwq, gsq = port.quantize(we)
    gx = rng.standard_normal((3, 2, 128)).astype(np.float32)
    lhs = np.array([0, 2, 1, 2, 0], np.uint32)
    rhs = np.array([5, 0, 3, 3, 1], np.uint32)
    out = np.empty((5, 2, 32), np.float32)
    L.ref_gather_qmm_f32(gx.ctypes.data, gwq.ctypes.data, gsq.ctypes.data, lhs.ctypes.data,
                         rhs.ctypes.data, 5, 2, 32, 128, out.ctypes.data)
    gxb = oracle.bf16_bits_from_f32(gx)
    outb = np.empty((5, 2, 32), np.uint16)
    L.ref_gather_qmm_bf16(gxb.ctypes.data, gwq.ctypes.data, gsq.ctypes.data, lhs.ctypes.data,
                          rhs.ctypes.data, 5, 2, 32, 128, outb.ctypes.data)
    g.update(gather_wq=gwq, gather_sq=gsq, gather_x_f32=gx, gather_x_bf16=gxb, gather_lhs=lhs,
             gather_rhs=rhs, gather_out_f32=out, gather_out_bf16=outb)

    # Quantizer pin: mixed magnitudes, zero groups, ties at LUT midpoints.
    rng = np.random.default_rng(3)
    qw = (rng.standard_normal((24, 64)) * rng.choice([1e-4, 0.02, 1, 300], (24, 1))).astype(
        np.float32)
    qw[0, :16] = 0.0                                     # all-zero group
    qw[1, :16] = np.array([6, 3, 0.25, -0.25, 0.75, -0.75, 1.25, -1.25, 1.75, 2.5, -3.5, 5,
                           -5, 0.5, -0.5, 0], np.float32)  # midpoints of the E2M1 grid at scale 1
    qb = oracle.bf16_bits_from_f32(qw)
    g["quant_w_bf16"] = qb
    g["quant_wq"], g["quant_sq"] = ref_quantize_bf16(ref, qb)

    # QQMatmul pin: activation fake-quant edge groups and a small product.
    rng = np.random.default_rng(4)
    fe = np.concatenate([
        np.array([0, -0., 0.25, -0.25, 0.2500001, 0.75, 0.7499999, 1.25, 1.2500001, 1.75, 2.5,
                  2.5000002, 3.5, 3.4999998, 5, 5.0000005, 6, 7, 1e30, np.inf, -np.inf, np.nan],
                 np.float32),
        (rng.standard_normal(500) * 3).astype(np.float32)])
    g["fp4_enc_in"] = fe
    g["fp4_enc_out"] = np.array([L.ref_to_fp4_e2m1(float(v)) for v in fe], np.uint8)
    qx = (rng.standard_normal((12, 256)) * rng.choice([1e-6, 1e-3, 1, 30, 1e4], (12, 1))).astype(
        np.float32)
    qx[0, :16] = 0.0                                     # all-zero group
    qx[1, :16] = np.nan                                  # all-NaN group (scale byte 0xFE)
    qx[2, :16] = [np.nan] * 8 + [1.0] * 8
    qx[3, :16] = np.inf
    qx[4, 16:32] = np.array([6, 3, 0.25, -0.25, 0.75, -0.75, 1.25, -1.25, 1.75, 2.5, -3.5, 5,
                             -5, 0.5, -0.5, 0], np.float32)  # E2M1 midpoints at scale 1
    g["qqmm_fq_in"] = qx
    g["qqmm_fq_out"] = ref.fake_quant_x(qx)
    rng = np.random.default_rng(5)
    w = oracle.bf16_bits_from_f32((rng.standard_normal((48, 512)) * 0.02).astype(np.float32))
    wq, sq = port.quantize(w)
    x = rng.standard_normal((3, 512)).astype(np.float32)
    xb = oracle.bf16_bits_from_f32(x)
    g["qqmm_wq"], g["qqmm_sq"], g["qqmm_x_f32"], g["qqmm_x_bf16"] = wq, sq, x, xb
    g["qqmm_y_f32"] = ref.qqmm_f32(x, wq, sq)
    g["qqmm_y_bf16"] = ref.qqmm_bf16(xb, wq, sq)

    np.savez_compressed(OUT, **g)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
