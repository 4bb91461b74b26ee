"""Pin the CPU oracle (oracle/nvfp4_oracle.c) before trusting it.

Known answers are restated from the reference's own NVFP4 tests; golden arrays
come from the reference's compiled MLX CPU kernels (tests/golden/make_golden.py).
When oracle/_ref/libmlxref.so is present the oracle is also compared with it
directly on fresh inputs.
"""
import numpy as np
import pytest

from conftest import assert_close

LUT = [0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6]


def pack(nibbles):
    words = []
    for i in range(0, len(nibbles), 8):
        w = 0
        for j in range(8):
            w |= (nibbles[i + j] & 15) << (4 * j)
        words.append(w)
    return np.array(words, np.uint32)


# --- known answers (Tests/MLXFastTests/NVFP4QuantizedMMTests.swift:101-153,
#     LagunaNVFP4KernelTests.swift:57-91) -------------------------------------

def test_low_nibble_first_decode(orc):
    w = pack(list(range(16))).reshape(1, 2)
    s = np.array([[0x38]], np.uint8)  # E4M3 1.0
    out = orc.port.dequantize(w, s)
    assert out.reshape(-1).tolist() == LUT
    assert np.signbit(out[0, 8])  # code 8 is -0


def test_e4m3_scales_per_group(orc):
    w = np.full((1, 4), 0x22222222, np.uint32)  # code 2 = 1.0
    s = np.array([[0x30, 0x40]], np.uint8)      # 0.5 and 2.0
    out = orc.port.dequantize(w, s)
    assert out.reshape(-1).tolist() == [0.5] * 16 + [2.0] * 16


def test_nibble_order_and_scale_bytes_contract(orc):
    w = np.array([[0x76543210, 0xFEDCBA98], [0x76543210, 0xFEDCBA98]], np.uint32)
    s = np.array([[0x38], [0x40]], np.uint8)
    out = orc.port.dequantize(w, s)
    assert out.reshape(-1).tolist() == LUT + [v * 2 for v in LUT]


def test_e4m3_decode_matches_reference_table(orc, golden):
    dec = np.array([orc.port.e4m3_decode(b) for b in range(256)], np.float32)
    assert np.array_equal(dec.view(np.uint32), golden["e4m3_decode"].view(np.uint32))
    assert dec[0x7F] == 480.0 and dec[0xFF] == -480.0  # MLX: no NaN encoding


def test_e4m3_encode_matches_reference(orc, golden):
    enc = np.array([orc.port.e4m3_encode(v) for v in golden["e4m3_enc_in"]], np.uint8)
    assert np.array_equal(enc, golden["e4m3_enc_out"])


def test_sigmoid_within_one_ulp_of_reference(orc, golden):
    got = np.array([orc.port.sigmoid(v) for v in golden["sigmoid_in"]], np.float32)
    assert np.abs(got - golden["sigmoid_out"]).max() <= 1.2e-7


# --- golden arrays from the reference kernels ---------------------------------

def test_qmm_f32_bit_exact_vs_reference_kernel(orc, golden):
    y = orc.port.qmm_f32(golden["qmm_x_f32"], golden["qmm_wq"], golden["qmm_sq"])
    assert np.array_equal(y.view(np.uint32), golden["qmm_y_f32"].view(np.uint32))


def test_qmm_bf16_bit_exact_vs_reference_kernel(orc, golden):
    y = orc.port.qmm_bf16(golden["qmm_x_bf16"], golden["qmm_wq"], golden["qmm_sq"])
    assert np.array_equal(y, golden["qmm_y_bf16"])


def test_gather_bit_exact_vs_reference_loop(orc, golden):
    out = orc.port.gather_qmm_f32(golden["gather_x_f32"], golden["gather_wq"], golden["gather_sq"],
                                  golden["gather_lhs"], golden["gather_rhs"], M=2)
    assert np.array_equal(out.view(np.uint32), golden["gather_out_f32"].view(np.uint32))


def test_quantizer_bit_exact_vs_reference_ops(orc, golden):
    wq, sq = orc.port.quantize(golden["quant_w_bf16"])
    assert np.array_equal(wq, golden["quant_wq"])
    assert np.array_equal(sq, golden["quant_sq"])


def test_quantizer_ties_round_to_smaller_magnitude(orc):
    # scale 1 (max 6): midpoints go to the first LUT entry (argmin, first wins).
    w = np.array([[6, 0.25, -0.25, 0.75, -0.75, 1.25, 2.5, -5] + [0] * 8], np.float32)
    wq, sq = orc.port.quantize(orc.bf16_bits_from_f32(w))
    assert sq[0, 0] == 0x38
    codes = [(int(wq[0, 0]) >> (4 * j)) & 15 for j in range(8)]
    assert codes == [7, 0, 0, 1, 9, 2, 4, 14]


# --- upstream MLX test_nvfp4_quantize_dequantize (python/tests/test_quantized.py:113-175) --

def test_lut_valued_weights_round_trip(orc):
    rng = np.random.default_rng(0)
    lut = np.array(LUT, np.float32)
    w = lut[rng.integers(0, 16, (128, 512))].reshape(-1, 16)
    w[:, 0] = 6
    w = (w + 3e-6).reshape(128, 512)
    wb = orc.bf16_bits_from_f32(w)
    wq, sq = orc.port.quantize(wb)
    w_hat = orc.port.dequantize(wq, sq)
    np.testing.assert_allclose(w_hat, orc.f32_from_bf16_bits(wb), rtol=1e-5, atol=1e-5)


def test_zeros_quantize_to_zeros(orc):
    wq, sq = orc.port.quantize(np.zeros((256, 512), np.float32))
    assert np.all(orc.port.dequantize(wq, sq) == 0)


# --- constant-weight checks (LagunaNVFP4KernelTests.swift:8-55, :93-150) --------

def test_all_ones_qmm_matches_dequantized_matmul(orc):
    x = np.ones((32, 64), np.float32)
    wq, sq = orc.port.quantize(np.ones((128, 64), np.float32))
    ref = x @ orc.port.dequantize(wq, sq).T
    assert np.abs(orc.port.qmm_f32(x, wq, sq) - ref).max() <= 1e-4


@pytest.mark.parametrize("N,K", [(512, 2048), (2048, 512)])
def test_shared_expert_shapes_constant_half(orc, N, K):
    wq, sq = orc.port.quantize(np.full((N, K), 0.5, np.float32))
    wd = orc.port.dequantize(wq, sq)
    for m in (1, 32):
        x = np.ones((m, K), np.float32)
        assert np.abs(orc.port.qmm_f32(x, wq, sq) - x @ wd.T).max() <= 1e-4


def test_routed_gather_distinct_constant_codes(orc):
    E, N, K = 256, 64, 128
    codes = np.array([((e % 7) + 1) * 0x11111111 for e in range(E)], np.uint32)
    wq = np.broadcast_to(codes[:, None, None], (E, N, K // 8)).copy()
    sq = np.full((E, N, K // 16), 0x38, np.uint8)
    ids = np.array([0, 7, 42, 255, 3, 128, 17, 99], np.uint32)
    for tokens in (1, 8):
        x = np.full((tokens, 1, K), 0.25, np.float32)
        rhs = np.tile(ids, tokens)
        lhs = np.repeat(np.arange(tokens, dtype=np.uint32), 8)
        got = orc.port.gather_qmm_f32(x, wq, sq, lhs, rhs, M=1)
        wd = orc.port.dequantize(wq[ids], sq[ids])
        want = np.einsum("tk,enk->ten", x[:, 0], wd).reshape(-1, 1, N)
        assert np.abs(got - want).max() <= 1e-4


# --- gather equals non-gather (NVFP4QuantizedMMTests.swift:309-355, :398-459) ----

def deterministic_source(shape, salt):
    n = int(np.prod(shape))
    i = np.arange(n)
    return (((i * 17 + salt) % 31) - 15).astype(np.float32).reshape(shape) / 16


@pytest.mark.parametrize("E,N,K,rows,experts", [(4, 512, 2048, 1, [3, 0, 2, 1, 2, 0, 3, 1]),
                                                 (4, 512, 2048, 32, [1, 2]),
                                                 (4, 2048, 512, 1, list(range(4)) * 4)])
def test_gather_matches_per_expert_qmm(orc, E, N, K, rows, experts):
    wq, sq = orc.port.quantize(deterministic_source((E, N, K), 5))
    x = deterministic_source((len(experts), rows, K), 18)
    rhs = np.array(experts, np.uint32)
    got = orc.port.gather_qmm_f32(x, wq, sq, None, rhs, M=rows)
    for i, e in enumerate(experts):
        want = orc.port.qmm_f32(x[i], wq[e], sq[e])
        np.testing.assert_allclose(got[i], want, rtol=2e-3, atol=2e-3)


# --- QQMatmul: activation fake-quant (quantized.cpp:1064-1129, 1322-1360) -------

def test_to_fp4_e2m1_matches_reference(orc, golden):
    got = np.array([orc.port.to_fp4_e2m1(v) for v in golden["fp4_enc_in"]], np.uint8)
    assert np.array_equal(got, golden["fp4_enc_out"])


def test_to_fp4_e2m1_ties_to_even(orc):
    # RNE on the E2M1 grid with the reference's comparisons: 0.25 -> 0,
    # 0.75 -> 1.0, 1.25 -> 1.0, 1.75 -> 2.0, 2.5 -> 2.0, 3.5 -> 4.0, 5 -> 4.0.
    for v, code in [(0.25, 0), (0.75, 2), (1.25, 2), (1.75, 4), (2.5, 4), (3.5, 6), (5.0, 6),
                    (5.01, 7), (100.0, 7), (-0.75, 10), (float("nan"), 7), (-0.0, 8)]:
        assert orc.port.to_fp4_e2m1(v) == code, v


def test_activation_fake_quant_bit_exact_vs_reference(orc, golden):
    got = orc.port.fake_quant_x(golden["qqmm_fq_in"])
    assert np.array_equal(got.view(np.uint32), golden["qqmm_fq_out"].view(np.uint32))


def test_activation_codes_dequantize_to_xhat(orc, golden):
    x = golden["qqmm_fq_in"]
    xq, s = orc.port.quantize_x(x)
    assert s.max() <= 0x7E  # UE4M3 magnitudes only (the all-NaN group is re-signed)
    assert np.array_equal(orc.port.dequantize(xq, s).view(np.uint32),
                          golden["qqmm_fq_out"].view(np.uint32))


def test_qqmm_f32_bit_exact_vs_reference(orc, golden):
    y = orc.port.qqmm_f32(golden["qqmm_x_f32"], golden["qqmm_wq"], golden["qqmm_sq"])
    assert np.array_equal(y.view(np.uint32), golden["qqmm_y_f32"].view(np.uint32))


def test_qqmm_bf16_path_bit_exact_vs_reference(orc, golden):
    # T = bfloat16_t: xhat is exact in bf16, then fp_qmm_t with per-op bf16
    # rounding (the secondary comparison; the tolerance target is the f32 form).
    x = orc.f32_from_bf16_bits(golden["qqmm_x_bf16"])
    xhat_bits = orc.bf16_bits_from_f32(orc.port.fake_quant_x(x))
    assert np.array_equal(orc.f32_from_bf16_bits(xhat_bits), orc.port.fake_quant_x(x))
    y = orc.port.qmm_bf16(xhat_bits, golden["qqmm_wq"], golden["qqmm_sq"])
    assert np.array_equal(y, golden["qqmm_y_bf16"])


# --- oracle vs the reference kernels on fresh inputs (this container only) ----

def test_port_vs_reference_library_fresh_inputs(orc):
    if orc.ref is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    rng = np.random.default_rng(7)
    w = orc.bf16_bits_from_f32((rng.standard_normal((96, 512)) * 0.02).astype(np.float32))
    wq, sq = orc.port.quantize(w)
    x = rng.standard_normal((3, 512)).astype(np.float32)
    assert np.array_equal(orc.port.qmm_f32(x, wq, sq).view(np.uint32),
                          orc.ref.qmm_f32(x, wq, sq).view(np.uint32))
    xb = orc.bf16_bits_from_f32(x)
    assert np.array_equal(orc.port.qmm_bf16(xb, wq, sq), orc.ref.qmm_bf16(xb, wq, sq))
    for v in rng.standard_normal(5000).astype(np.float32) * 100:
        assert orc.port.e4m3_encode(v) == orc.ref.lib.ref_to_fp8(float(v))
    xq = (rng.standard_normal((9, 512)) * rng.choice([1e-5, 1, 1e3], (9, 1))).astype(np.float32)
    assert np.array_equal(orc.port.fake_quant_x(xq).view(np.uint32),
                          orc.ref.fake_quant_x(xq).view(np.uint32))
    assert np.array_equal(orc.port.qqmm_f32(x, wq, sq).view(np.uint32),
                          orc.ref.qqmm_f32(x, wq, sq).view(np.uint32))


# --- router / block semantics ----------------------------------------------------

def test_router_topk_properties(orc):
    rng = np.random.default_rng(3)
    T, H, E, k = 4, 256, 64, 8
    x = orc.bf16_bits_from_f32(rng.standard_normal((T, H)).astype(np.float32))
    G = orc.bf16_bits_from_f32((rng.standard_normal((E, H)) * 0.02).astype(np.float32))
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    inds, w, logits = orc.port.router_topk(x, G, bias, k)
    s = 1 / (1 + np.exp(-logits.astype(np.float64)))
    choice = s + bias
    for t in range(T):
        order = np.argsort(-choice[t], kind="stable")[:k]
        assert set(order.tolist()) == set(inds[t].tolist())
        np.testing.assert_allclose(w[t].sum(), 1.0, rtol=1e-6)
        np.testing.assert_allclose(w[t], s[t, inds[t]] / s[t, inds[t]].sum(), rtol=1e-5)


def test_moe_block_oracle_matches_composed_ops(orc):
    rng = np.random.default_rng(4)
    T, H, I, E, k = 2, 128, 128, 8, 2
    q = lambda shape: orc.port.quantize((rng.standard_normal(shape) * 0.02).astype(np.float32))
    gw, gs = q((E, I, H)); uw, us = q((E, I, H)); dw, ds = q((E, H, I))
    sgw, sgs = q((I, H)); suw, sus = q((I, H)); sdw, sds = q((H, I))
    x = rng.standard_normal((T, H)).astype(np.float32)
    inds = np.array([[1, 5], [0, 7]], np.uint32)
    wts = np.array([[0.6, 0.4], [0.3, 0.7]], np.float32)
    routed = dict(gate_w=gw, gate_s=gs, up_w=uw, up_s=us, down_w=dw, down_s=ds)
    shared = dict(gate_w=sgw, gate_s=sgs, up_w=suw, up_s=sus, down_w=sdw, down_s=sds)
    y = orc.port.moe_block_f32(x, inds, wts, routed, shared, scaling=2.5)
    silu = lambda v: v / (1 + np.exp(-v))
    want = np.zeros_like(x)
    for t in range(T):
        for j in range(k):
            e = inds[t, j]
            a = silu(orc.port.qmm_f32(x[t:t + 1], gw[e], gs[e])) * orc.port.qmm_f32(x[t:t + 1], uw[e], us[e])
            want[t] += wts[t, j] * orc.port.qmm_f32(a, dw[e], ds[e])[0]
        want[t] *= 2.5
        a = silu(orc.port.qmm_f32(x[t:t + 1], sgw, sgs)) * orc.port.qmm_f32(x[t:t + 1], suw, sus)
        want[t] += orc.port.qmm_f32(a, sdw, sds)[0]
    assert_close(y, want, max_abs=1e-5, rel_l2=1e-6, what="oracle block")
