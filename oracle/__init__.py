"""CPU checkers for the NVFP4 MoE path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline /
``--impl reference`` arm may import this package.  It is the parity checker and
the timed CPU baseline; the product library never calls it.

``port``  -- ctypes bindings of ``liboracle.so`` (plain-C restatement,
             ``nvfp4_oracle.c``), plus numpy helpers.
``ref``   -- ctypes bindings of ``_ref/libmlxref.so``: the reference's own MLX
             CPU kernels compiled in place from the reference sources by
             ``oracle/Makefile`` (None when the file was never built).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_F = ctypes.c_float


def _ptr(a):
    return None if a is None else a.ctypes.data_as(_P)


def _load(path):
    if not os.path.exists(path):
        return None
    return ctypes.CDLL(path)


class _Port:
    def __init__(self, lib):
        self.lib = lib
        L = lib
        L.orc_bf16_from_f32.restype = ctypes.c_uint16
        L.orc_bf16_from_f32.argtypes = [_F]
        L.orc_e4m3_decode.restype = _F
        L.orc_e4m3_decode.argtypes = [ctypes.c_uint8]
        L.orc_e4m3_encode.restype = ctypes.c_uint8
        L.orc_e4m3_encode.argtypes = [_F]
        L.orc_sigmoid.restype = _F
        L.orc_sigmoid.argtypes = [_F]
        L.orc_dequantize.argtypes = [_P, _P, _I64, _I64, _P]
        L.orc_quantize_bf16.argtypes = [_P, _I64, _I64, _P, _P]
        L.orc_quantize_f32.argtypes = [_P, _I64, _I64, _P, _P]
        L.orc_qmm_f32.argtypes = [_P, _P, _P, _I64, _I64, _I64, _P]
        L.orc_qmm_bf16.argtypes = [_P, _P, _P, _I64, _I64, _I64, _P]
        L.orc_gather_qmm_f32.argtypes = [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]
        L.orc_gather_qmm_bf16.argtypes = [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]
        L.orc_router_topk.argtypes = [_P, _P, _P, _I64, _I64, _I64, _I, _I, _I, _P, _P, _P]
        L.orc_rms_norm_bf16.argtypes = [_P, _P, _I64, _I64, _F, _P]
        L.orc_moe_block_f32.argtypes = ([_P, _P, _P, _I64, _I64, _I64, _I, _F] + [_P] * 6 +
                                        [_I64] + [_P] * 6 + [_P, _P])
        L.orc_to_fp4_e2m1.restype = ctypes.c_uint8
        L.orc_to_fp4_e2m1.argtypes = [_F]
        L.orc_quantize_dequantize_x.argtypes = [_P, _I64, _I64, _P]
        L.orc_quantize_x.argtypes = [_P, _I64, _I64, _P, _P]
        L.orc_qqmm_f32.argtypes = [_P, _P, _P, _I64, _I64, _I64, _P]

    # -- scalar conversions -------------------------------------------------
    def e4m3_decode(self, b):
        return self.lib.orc_e4m3_decode(int(b))

    def e4m3_encode(self, f):
        return self.lib.orc_e4m3_encode(float(f))

    def bf16_from_f32(self, f):
        return self.lib.orc_bf16_from_f32(float(f))

    def sigmoid(self, f):
        return self.lib.orc_sigmoid(float(f))

    # -- array ops ------------------------------------------------------------
    def quantize(self, w):
        """w: bf16 bits (uint16) or float32, shape [..., K] -> (u32 [..., K/8], u8 [..., K/16])."""
        w = np.ascontiguousarray(w)
        K = w.shape[-1]
        rows = w.size // K
        wq = np.empty(w.shape[:-1] + (K // 8,), np.uint32)
        sq = np.empty(w.shape[:-1] + (K // 16,), np.uint8)
        if w.dtype == np.uint16:
            self.lib.orc_quantize_bf16(_ptr(w), rows, K, _ptr(wq), _ptr(sq))
        elif w.dtype == np.float32:
            self.lib.orc_quantize_f32(_ptr(w), rows, K, _ptr(wq), _ptr(sq))
        else:
            raise TypeError("quantize expects bf16 bits (uint16) or float32")
        return wq, sq

    def dequantize(self, wq, sq):
        wq = np.ascontiguousarray(wq, np.uint32)
        sq = np.ascontiguousarray(sq, np.uint8)
        K = wq.shape[-1] * 8
        rows = wq.size // wq.shape[-1]
        out = np.empty(wq.shape[:-1] + (K,), np.float32)
        self.lib.orc_dequantize(_ptr(wq), _ptr(sq), rows, K, _ptr(out))
        return out

    def qmm_f32(self, x, wq, sq):
        x = np.ascontiguousarray(x, np.float32)
        K = x.shape[-1]
        M = x.size // K
        N = wq.shape[-2]
        y = np.empty(x.shape[:-1] + (N,), np.float32)
        self.lib.orc_qmm_f32(_ptr(x), _ptr(np.ascontiguousarray(wq)), _ptr(np.ascontiguousarray(sq)),
                             M, N, K, _ptr(y))
        return y

    def qmm_bf16(self, x_bits, wq, sq):
        x = np.ascontiguousarray(x_bits, np.uint16)
        K = x.shape[-1]
        M = x.size // K
        N = wq.shape[-2]
        y = np.empty(x.shape[:-1] + (N,), np.uint16)
        self.lib.orc_qmm_bf16(_ptr(x), _ptr(np.ascontiguousarray(wq)), _ptr(np.ascontiguousarray(sq)),
                              M, N, K, _ptr(y))
        return y

    def gather_qmm_f32(self, x, wq, sq, lhs, rhs, M):
        """x [B, M, K] f32; wq [E, N, K/8]; rhs [P]; lhs [P] or None -> [P, M, N]."""
        x = np.ascontiguousarray(x, np.float32)
        K = x.shape[-1]
        N = wq.shape[-2]
        rhs = np.ascontiguousarray(rhs, np.uint32)
        P = rhs.size
        lhs_a = None if lhs is None else np.ascontiguousarray(lhs, np.uint32)
        out = np.empty((P, M, N), np.float32)
        self.lib.orc_gather_qmm_f32(_ptr(x), _ptr(np.ascontiguousarray(wq)),
                                    _ptr(np.ascontiguousarray(sq)), _ptr(lhs_a), _ptr(rhs), P, M, N,
                                    K, _ptr(out))
        return out

    # -- QQMatmul: activation fake-quant + NVFP4 matmul ---------------------
    def to_fp4_e2m1(self, f):
        return self.lib.orc_to_fp4_e2m1(float(f))

    def fake_quant_x(self, x):
        """xhat = fp_quantize_dequantize(x) (f32 values, groups of 16 along the last axis)."""
        x = np.ascontiguousarray(x, np.float32)
        K = x.shape[-1]
        out = np.empty_like(x)
        self.lib.orc_quantize_dequantize_x(_ptr(x), x.size // K, K, _ptr(out))
        return out

    def quantize_x(self, x):
        """x f32 [..., K] -> (codes u32 [..., K/8], scale bytes u8 [..., K/16])."""
        x = np.ascontiguousarray(x, np.float32)
        K = x.shape[-1]
        xq = np.empty(x.shape[:-1] + (K // 8,), np.uint32)
        s = np.empty(x.shape[:-1] + (K // 16,), np.uint8)
        self.lib.orc_quantize_x(_ptr(x), x.size // K, K, _ptr(xq), _ptr(s))
        return xq, s

    def qqmm_f32(self, x, wq, sq):
        x = np.ascontiguousarray(x, np.float32)
        K = x.shape[-1]
        M = x.size // K
        N = wq.shape[-2]
        y = np.empty(x.shape[:-1] + (N,), np.float32)
        self.lib.orc_qqmm_f32(_ptr(x), _ptr(np.ascontiguousarray(wq)),
                              _ptr(np.ascontiguousarray(sq)), M, N, K, _ptr(y))
        return y

    def router_topk(self, x_bits, G_bits, bias, k, norm=True, round_logits=True):
        x = np.ascontiguousarray(x_bits, np.uint16)
        G = np.ascontiguousarray(G_bits, np.uint16)
        E, H = G.shape
        T = x.size // H
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        inds = np.empty((T, k), np.uint32)
        wts = np.empty((T, k), np.float32)
        logits = np.empty((T, E), np.float32)
        self.lib.orc_router_topk(_ptr(x), _ptr(G), _ptr(b), T, H, E, k, int(norm),
                                 int(round_logits), _ptr(inds), _ptr(wts), _ptr(logits))
        return inds, wts, logits

    def rms_norm_bf16(self, x_bits, w_bits, eps):
        """RMSNorm of bf16 rows (bit patterns) with bf16 weights -> bf16 bits."""
        x = np.ascontiguousarray(x_bits, np.uint16)
        H = x.shape[-1]
        w = None if w_bits is None else np.ascontiguousarray(w_bits, np.uint16)
        y = np.empty_like(x)
        self.lib.orc_rms_norm_bf16(_ptr(x), _ptr(w), x.size // H, H, float(eps), _ptr(y))
        return y

    def moe_block_f32(self, x, inds, wts, routed, shared=None, scaling=2.5, residual=None):
        """routed / shared: dicts with gate_w, gate_s, up_w, up_s, down_w, down_s."""
        x = np.ascontiguousarray(x, np.float32)
        T, H = x.shape
        k = inds.shape[-1]
        I = routed["gate_w"].shape[-2]
        c = {n: np.ascontiguousarray(a) for n, a in routed.items()}
        sh = {n: np.ascontiguousarray(a) for n, a in shared.items()} if shared else None
        Is = shared["gate_w"].shape[-2] if shared else 0
        y = np.empty((T, H), np.float32)
        inds = np.ascontiguousarray(inds, np.uint32)
        wts = np.ascontiguousarray(wts, np.float32)
        res = None if residual is None else np.ascontiguousarray(residual, np.float32)
        sp = [None] * 6 if sh is None else [_ptr(sh[n]) for n in
                                            ("gate_w", "gate_s", "up_w", "up_s", "down_w", "down_s")]
        self.lib.orc_moe_block_f32(
            _ptr(x), _ptr(inds), _ptr(wts), T, H, I, k, float(scaling),
            *[_ptr(c[n]) for n in ("gate_w", "gate_s", "up_w", "up_s", "down_w", "down_s")],
            Is, *sp, _ptr(res), _ptr(y))
        return y


class _Ref:
    def __init__(self, lib):
        self.lib = lib
        L = lib
        L.ref_qmm_f32.argtypes = [_P, _P, _P, _I, _I, _I, _P]
        L.ref_qmm_bf16.argtypes = [_P, _P, _P, _I, _I, _I, _P]
        L.ref_qmm_bf16_mt.argtypes = [_P, _P, _P, _I, _I, _I, _P, _I]
        L.ref_gather_qmm_bf16.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P]
        L.ref_gather_qmm_f32.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P]
        L.ref_from_fp8.restype = _F
        L.ref_from_fp8.argtypes = [ctypes.c_uint8]
        L.ref_to_fp8.restype = ctypes.c_uint8
        L.ref_to_fp8.argtypes = [_F]
        L.ref_sigmoid.restype = _F
        L.ref_sigmoid.argtypes = [_F]
        L.ref_to_fp4_e2m1.restype = ctypes.c_uint8
        L.ref_to_fp4_e2m1.argtypes = [_F]
        L.ref_bf16_from_f32.restype = ctypes.c_uint16
        L.ref_bf16_from_f32.argtypes = [_F]
        for n in ("ref_bf16_mul", "ref_bf16_div"):
            getattr(L, n).restype = ctypes.c_uint16
            getattr(L, n).argtypes = [ctypes.c_uint16, ctypes.c_uint16]
        L.ref_fake_quant_f32.argtypes = [_P, _I, _I, _P]
        L.ref_qqmm_f32.argtypes = [_P, _P, _P, _I, _I, _I, _P]
        L.ref_qqmm_bf16.argtypes = [_P, _P, _P, _I, _I, _I, _P]

    def fake_quant_x(self, x):
        x = np.ascontiguousarray(x, np.float32)
        K = x.shape[-1]
        out = np.empty_like(x)
        self.lib.ref_fake_quant_f32(_ptr(x), x.size // K, K, _ptr(out))
        return out

    def qqmm_f32(self, x, wq, sq):
        x = np.ascontiguousarray(x, np.float32)
        K = x.shape[-1]
        M = x.size // K
        N = wq.shape[-2]
        y = np.empty(x.shape[:-1] + (N,), np.float32)
        self.lib.ref_qqmm_f32(_ptr(x), _ptr(np.ascontiguousarray(wq)),
                              _ptr(np.ascontiguousarray(sq)), M, N, K, _ptr(y))
        return y

    def qqmm_bf16(self, x_bits, wq, sq):
        x = np.ascontiguousarray(x_bits, np.uint16)
        K = x.shape[-1]
        M = x.size // K
        N = wq.shape[-2]
        y = np.empty(x.shape[:-1] + (N,), np.uint16)
        self.lib.ref_qqmm_bf16(_ptr(x), _ptr(np.ascontiguousarray(wq)),
                               _ptr(np.ascontiguousarray(sq)), M, N, K, _ptr(y))
        return y

    def qmm_f32(self, x, wq, sq):
        x = np.ascontiguousarray(x, np.float32)
        K = x.shape[-1]
        M = x.size // K
        N = wq.shape[-2]
        y = np.empty(x.shape[:-1] + (N,), np.float32)
        self.lib.ref_qmm_f32(_ptr(x), _ptr(np.ascontiguousarray(wq)), _ptr(np.ascontiguousarray(sq)),
                             M, N, K, _ptr(y))
        return y

    def qmm_bf16(self, x_bits, wq, sq, threads=1):
        x = np.ascontiguousarray(x_bits, np.uint16)
        K = x.shape[-1]
        M = x.size // K
        N = wq.shape[-2]
        y = np.empty(x.shape[:-1] + (N,), np.uint16)
        if threads > 1:
            self.lib.ref_qmm_bf16_mt(_ptr(x), _ptr(np.ascontiguousarray(wq)),
                                     _ptr(np.ascontiguousarray(sq)), M, N, K, _ptr(y), threads)
        else:
            self.lib.ref_qmm_bf16(_ptr(x), _ptr(np.ascontiguousarray(wq)),
                                  _ptr(np.ascontiguousarray(sq)), M, N, K, _ptr(y))
        return y


port = _Port(ctypes.CDLL(os.path.join(HERE, "liboracle.so"))) if os.path.exists(
    os.path.join(HERE, "liboracle.so")) else None
_ref_lib = _load(os.path.join(HERE, "_ref", "libmlxref.so"))
ref = _Ref(_ref_lib) if _ref_lib is not None else None


# -- numpy helpers shared by tests, smoke() and bench.py ----------------------
def bf16_bits_from_f32(a):
    """Round-to-nearest-even f32 -> bf16 bit patterns (types/bf16.h:37-58)."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + ((u >> 16) & 1) + 0x7FFF) >> 16).astype(np.uint16)
    r[np.isnan(a)] = 0x7FC0
    return r


def f32_from_bf16_bits(b):
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def build():
    """Compile liboracle.so (and _ref/libmlxref.so when the reference tree exists)."""
    import subprocess
    subprocess.run(["make", "-s", "-f", os.path.join(HERE, "Makefile")], check=True)
