"""B200-native NVFP4 MoE hot path of Layr-Labs/mlxfast-challenge (Laguna XS 2.1).

Host-side mirror of the reference's operator surface for this path, over the
C ABI of ``libnvfp4moe.so`` (``include/nvfp4moe.h``).  Names, argument meaning
and error behaviour follow MLX's Python API for the same ops:

    quantize(w, group_size=16, bits=4, mode="nvfp4")          -> (wq, scales)
        mlx ops.cpp:4980-5025 / fp_quantize :4873-4978
    dequantize(wq, scales, biases=None, ..., dtype=...)       -> w
        ops.cpp:5243-5302 / fp_dequantize :5120-5241
    quantized_matmul(x, w, scales, biases=None, transpose=True, ...)
        ops.cpp:4549-4600
    gather_qmm(x, w, scales, biases=None, lhs_indices=None, rhs_indices=None,
               transpose=True, ..., sorted_indices=False)
        ops.cpp:5338-5433
    moe_router_topk(x, gate_weight, bias, top_k, norm_topk_prob)
        LagunaMoEGate, VLM/MLXLLM/Models/Laguna.swift:149-181
    SparseMoeBlock(...)(x)
        LagunaSparseMoeBlock, Laguna.swift:183-213

Tensors are torch CUDA tensors (torch provides device memory and streams
only); every computation runs in the library's sm_100a kernels.  Invalid
arguments raise ValueError as MLX's std::invalid_argument does; modes other
than nvfp4 / transpose=False raise NotImplementedError (out of scope).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from ._lib import DeviceIndexError, DeviceTimeoutError, MoeLayerDesc, NvFp4Bank, check, lib

__all__ = [
    "quantize", "dequantize", "quantized_matmul", "gather_qmm", "moe_router_topk", "qqmm",
    "rms_norm",
    "quantize_activations",
    "SparseMoeBlock", "MoEDecodeChain", "device_status", "launch_flags", "DeviceIndexError", "DeviceTimeoutError", "library_path",
]

_DT = {torch.bfloat16: _lib.NVFP4_BF16, torch.float16: _lib.NVFP4_F16,
       torch.float32: _lib.NVFP4_F32}


def library_path() -> str:
    return _lib.LIB_PATH


def _stream(device=None) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _dtype_code(t: torch.Tensor, op: str) -> int:
    if t.dtype not in _DT:
        raise ValueError(f"[{op}] Only real floating types are supported but x.dtype() == "
                         f"{t.dtype}.")
    return _DT[t.dtype]


def _check_mode(op: str, group_size, bits, mode, biases=None, transpose=True):
    if mode != "nvfp4":
        raise NotImplementedError(f"[{op}] only mode 'nvfp4' is provided by this library "
                                  f"(got '{mode}').")
    if group_size is not None and group_size != 16:
        raise ValueError(f"[{op}] nvfp4 quantization requires group size 16 but got "
                         f"{group_size}.")
    if bits is not None and bits != 4:
        raise ValueError(f"[{op}] nvfp4 quantization requires bits to be 4 but got {bits}.")
    if biases is not None:
        raise ValueError(f"[{op}] Biases must be null for quantization mode 'nvfp4'.")
    if not transpose:
        raise NotImplementedError(f"[{op}] only transpose=True is provided by this library.")


def _require_cuda(op: str, *ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError(f"[{op}] tensors must live on a CUDA device (no CPU path).")


def _u32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == torch.uint32:
        return t
    if t.dtype == torch.int32:
        return t.view(torch.uint32)
    raise ValueError("The weight matrix should be uint32")


def quantize(w: torch.Tensor, group_size: int = 16, bits: int = 4, mode: str = "nvfp4"):
    """w [..., K] (bf16/f16/f32) -> (wq uint32 [..., K/8], scales uint8 [..., K/16])."""
    _check_mode("quantize", group_size, bits, mode)
    _require_cuda("quantize", w)
    if w.dim() < 2:
        raise ValueError("[quantize] The matrix to be quantized must have at least 2 dimension "
                         f"but it has only {w.dim()}.")
    K = w.shape[-1]
    if K % 16:
        raise ValueError("[quantize] The last dimension of the matrix needs to be divisible by "
                         f"the quantization group size 16. However the provided  matrix has shape "
                         f"{tuple(w.shape)}")
    w = w.contiguous()
    rows = w.numel() // K
    wq = torch.empty(w.shape[:-1] + (K // 8,), dtype=torch.uint32, device=w.device)
    sc = torch.empty(w.shape[:-1] + (K // 16,), dtype=torch.uint8, device=w.device)
    check(lib().nvfp4_quantize(_ptr(wq), _ptr(sc), _ptr(w), _dtype_code(w, "quantize"), rows, K,
                               _stream(w.device)))
    return wq, sc


def dequantize(wq: torch.Tensor, scales: torch.Tensor, biases=None, group_size: int = 16,
               bits: int = 4, mode: str = "nvfp4", dtype: torch.dtype = torch.bfloat16):
    _check_mode("dequantize", group_size, bits, mode, biases)
    _require_cuda("dequantize", wq, scales)
    wq = _u32(wq).contiguous()
    if wq.dim() < 2:
        raise ValueError("[dequantize] The matrix to be dequantized must have at least 2 "
                         f"dimension but it has only {wq.dim()}.")
    if scales.dtype != torch.uint8:
        raise ValueError(f"[dequantize] Scale type must be uint8 but received type "
                         f"{scales.dtype}.")
    if wq.shape[:-1] != scales.shape[:-1] or wq.shape[-1] * 8 != scales.shape[-1] * 16:
        raise ValueError("[dequantize] Shape of scales does not match the matrix given the "
                         f"quantization parameters. Provided matrix of shape {tuple(wq.shape)} "
                         f"and scales of shape {tuple(scales.shape)}.")
    K = wq.shape[-1] * 8
    rows = wq.numel() // wq.shape[-1]
    out = torch.empty(wq.shape[:-1] + (K,), dtype=dtype, device=wq.device)
    check(lib().nvfp4_dequantize(_ptr(out), _dtype_code(out, "dequantize"), _ptr(wq),
                                 _ptr(scales.contiguous()), rows, K, _stream(wq.device)))
    return out


def _qdims(op, x, w, scales):
    w = _u32(w)
    if scales.dtype != torch.uint8:
        raise ValueError(f"[{op}] Scale type must be uint8 but received type {scales.dtype}.")
    if w.shape[:-1] != scales.shape[:-1] or w.shape[-1] * 8 != scales.shape[-1] * 16:
        raise ValueError(f"[{op}] The shapes of the weight and scales are incompatible based on "
                         f"bits and group_size. w.shape() == {tuple(w.shape)} and scales.shape() "
                         f"== {tuple(scales.shape)} with group_size=16 and bits=4")
    K = w.shape[-1] * 8
    if x.shape[-1] != K:
        raise ValueError(f"[{op}] Last dimension of first input with shape (..., {x.shape[-1]}) "
                         f"does not match the expanded quantized matrix ({K}, {w.shape[-2]}) "
                         f"computed from shape {tuple(w.shape)} with group_size=16, bits=4 and "
                         f"transpose=true")
    return w, K, w.shape[-2]


def quantized_matmul(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases=None,
                     transpose: bool = True, group_size: int = 16, bits: int = 4,
                     mode: str = "nvfp4") -> torch.Tensor:
    """x [..., M, K] @ dequant(w [N, K/8])^T -> [..., M, N] in x.dtype."""
    _check_mode("quantized_matmul", group_size, bits, mode, biases, transpose)
    _require_cuda("quantized_matmul", x, w, scales)
    if w.dim() > 2 and x.dim() > 2:
        # Batched weights broadcast against x's batch dims (ops.cpp:4589-4591):
        # the same product as a gather over both batch index grids.
        nx = x.numel() // (x.shape[-2] * x.shape[-1])
        nw = w.numel() // (w.shape[-2] * w.shape[-1])
        lhs = torch.arange(nx, device=x.device).reshape(x.shape[:-2])
        rhs = torch.arange(nw, device=x.device).reshape(w.shape[:-2])
        return gather_qmm(x, w, scales, lhs_indices=lhs, rhs_indices=rhs)
    if w.dim() > 2:
        raise ValueError("[quantized_matmul] batched weights need a batched x.")
    w, K, N = _qdims("quantized_matmul", x, w, scales)
    xc = x.contiguous()
    M = xc.numel() // K
    y = torch.empty(x.shape[:-1] + (N,), dtype=x.dtype, device=x.device)
    check(lib().nvfp4_quantized_matmul(_ptr(y), _ptr(xc), _dtype_code(x, "quantized_matmul"),
                                       _ptr(w.contiguous()), _ptr(scales.contiguous()), M, N, K,
                                       _stream(x.device)))
    return y


def quantize_activations(x: torch.Tensor):
    """The activation quantisation QQMatmul applies to x (fp_quantize_dequantize,
    backend/cpu/quantized.cpp:1093-1129): x [..., K] -> (codes uint32 [..., K/8],
    scales uint8 [..., K/16]); dequantize() of them is MLX's xhat bit for bit."""
    _require_cuda("qqmm", x)
    K = x.shape[-1]
    if K % 16:
        raise ValueError("[qqmm] The last dimension of the matrix needs to be divisible by the "
                         f"quantization group size 16. However the provided matrix has K={K}.")
    xc = x.contiguous()
    M = xc.numel() // K if K else 0
    xq = torch.empty(x.shape[:-1] + (K // 8,), dtype=torch.uint32, device=x.device)
    sc = torch.empty(x.shape[:-1] + (K // 16,), dtype=torch.uint8, device=x.device)
    check(lib().nvfp4_quantize_activations(_ptr(xq), _ptr(sc), _ptr(xc), _dtype_code(x, "qqmm"),
                                           M, K, _stream(x.device)))
    return xq, sc


def qqmm(x: torch.Tensor, w: torch.Tensor, scales: Optional[torch.Tensor] = None,
         group_size: int = 16, bits: int = 4, mode: str = "nvfp4", global_scale_x=None,
         global_scale_w=None) -> torch.Tensor:
    """mlx.core.qqmm (ops.cpp:4691-4757) for mode "nvfp4" with quantized w:
    y = fake_quant(x) @ dequant(w)^T in x.dtype, on the block-scaled tensor
    cores.  x is 1-D or 2-D (qqmm's own rule); w [N, K/8] uint32."""
    _check_mode("qqmm", group_size, bits, mode)
    if global_scale_x is not None or global_scale_w is not None:
        raise ValueError("[qqmm] global scales are not supported by this build.")
    if scales is None:
        raise ValueError("[qqmm] Scales must be provided if second argument is quantized.")
    _require_cuda("qqmm", x, w, scales)
    if x.dim() > 2 or w.dim() > 2:
        raise ValueError(f"[qqmm] Only 2D inputs are supported but x.ndim() == {x.dim()} and "
                         f"w.ndim() == {w.dim()}.")
    x2 = x.unsqueeze(0) if x.dim() == 1 else x
    w, K, N = _qdims("qqmm", x2, w, scales)
    xc = x2.contiguous()
    M = xc.shape[0]
    y = torch.empty((M, N), dtype=x.dtype, device=x.device)
    ws_bytes = lib().nvfp4_qqmm_workspace_size(M, N, K)
    ws = torch.empty(max(int(ws_bytes), 256), dtype=torch.uint8, device=x.device)
    check(lib().nvfp4_qqmm(_ptr(y), _ptr(xc), _dtype_code(x, "qqmm"), _ptr(w.contiguous()),
                           _ptr(scales.contiguous()), M, N, K, _ptr(ws), ws.numel(),
                           _stream(x.device)))
    return y.squeeze(0) if x.dim() == 1 else y


def gather_qmm(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases=None,
               lhs_indices: Optional[torch.Tensor] = None,
               rhs_indices: Optional[torch.Tensor] = None, transpose: bool = True,
               group_size: int = 16, bits: int = 4, mode: str = "nvfp4",
               sorted_indices: bool = False) -> torch.Tensor:
    """out[i] = x[lhs[i]] @ dequant(w[rhs[i]])^T; shape = broadcast(lhs, rhs).shape + [M, N]."""
    if lhs_indices is None and rhs_indices is None:
        return quantized_matmul(x, w, scales, biases, transpose, group_size, bits, mode)
    _check_mode("gather_qmm", group_size, bits, mode, biases, transpose)
    _require_cuda("gather_qmm", x, w, scales, lhs_indices, rhs_indices)
    if x.dim() < 2:
        raise ValueError("[gather_qmm] Non-quantized input must have at least two dimensions "
                         f"but got input with shape {tuple(x.shape)}.")
    w, K, N = _qdims("gather_qmm", x, w, scales)
    for name, ind in (("lhs", lhs_indices), ("rhs", rhs_indices)):
        if ind is not None and (ind.dtype.is_floating_point or ind.dtype == torch.bool):
            raise ValueError(f"[gather_qmm] Got {name}_indices with invalid dtype. Indices must "
                             "be integral.")
    M = x.shape[-2]
    xb = x.reshape(-1, M, K).contiguous()
    nxb = xb.shape[0]
    wb = w.reshape(-1, N, K // 8).contiguous()
    sb = scales.reshape(-1, N, K // 16).contiguous()
    E = wb.shape[0]
    # indices_or_default (ops.cpp:67-81): arange over the batch dims.
    if lhs_indices is None:
        lhs_indices = torch.arange(nxb, device=x.device).reshape(x.shape[:-2] or (1,))
    if rhs_indices is None:
        rhs_indices = torch.arange(E, device=x.device).reshape(w.shape[:-2] or (1,))
    lhs, rhs = torch.broadcast_tensors(lhs_indices, rhs_indices)
    out_shape = tuple(lhs.shape) + (M, N)
    lhs = lhs.reshape(-1).to(torch.int32).view(torch.uint32).contiguous()
    rhs = rhs.reshape(-1).to(torch.int32).view(torch.uint32).contiguous()
    P = lhs.numel()
    out = torch.empty(out_shape, dtype=x.dtype, device=x.device)
    check(lib().nvfp4_gather_qmm(_ptr(out), _ptr(xb), _dtype_code(x, "gather_qmm"), _ptr(wb),
                                 _ptr(sb), _ptr(lhs), _ptr(rhs), P, nxb, E, M, N, K,
                                 int(bool(sorted_indices)), _stream(x.device)))
    return out


class launch_flags:
    """Context manager setting the calling thread's C-ABI launch flags
    (nvfp4_set_launch_flags): pdl=True lets the first kernel of each call
    overlap its predecessor; bulk_copy=True selects the bulk-copy fed decode
    kernels; exact_prefill=True runs the prefill GEMMs on 16-bit dequantised
    weights (kind::f16) instead of the default block-scaled FP4 path
    (activations as four NVFP4 terms); exact_decode=True runs the persistent
    decode stack on the mma.sync engine (16-bit activations) instead of the
    default block-scaled FP4 stack."""

    def __init__(self, pdl: bool = False, bulk_copy: bool = False, exact_prefill: bool = False,
                 exact_decode: bool = False):
        self.flags = (_lib.NVFP4_LAUNCH_PDL if pdl else 0) | (
            _lib.NVFP4_LAUNCH_BULK_COPY if bulk_copy else 0) | (
            _lib.NVFP4_LAUNCH_EXACT_PREFILL if exact_prefill else 0) | (
            _lib.NVFP4_LAUNCH_EXACT_DECODE if exact_decode else 0)

    def __enter__(self):
        self.old = lib().nvfp4_set_launch_flags(self.flags)
        return self

    def __exit__(self, *exc):
        lib().nvfp4_set_launch_flags(self.old)


def device_status() -> None:
    """Synchronise; raise DeviceIndexError if a kernel saw an out-of-range index,
    DeviceTimeoutError if a kernel's bounded wait gave up (the status is cleared)."""
    check(lib().nvfp4_device_status())


class _Workspace:
    """Caller-owned device workspace, zeroed once (the router's tickets reset themselves)."""

    def __init__(self):
        self.buf = None

    def get(self, nbytes: int, device) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        return self.buf


_router_ws = _Workspace()


def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float,
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """mlx.core.fast.rms_norm (mlx/fast.cpp:53-108) over the last axis:
    dtype(dtype(x * rsqrt(mean(x^2) + eps)) * weight), weight [dims] in x.dtype."""
    _require_cuda("rms_norm", x, weight, out)
    if x.dim() < 1:
        raise ValueError("[rms_norm] Input must have at least 1 dimension but got input with 0 "
                         "dimensions.")
    H = x.shape[-1]
    if weight is not None:
        if weight.dim() != 1:
            raise ValueError(f"[rms_norm] (*weight) must have 1 dimension but has "
                             f"{weight.dim()} dimensions.")
        if weight.numel() != H:
            raise ValueError("[rms_norm] (*weight) must have the same size as the last "
                             f"dimension of x but has {weight.numel()} elements.")
        weight = weight.to(x.dtype).contiguous()
    xc = x.contiguous()
    y = out if out is not None else torch.empty_like(xc)
    check(lib().nvfp4_rms_norm(_ptr(y), _ptr(xc), _ptr(weight), _dtype_code(xc, "rms_norm"),
                               xc.numel() // H, H, float(eps), _stream(x.device)))
    return y


def moe_router_topk(x: torch.Tensor, gate_weight: torch.Tensor, bias: Optional[torch.Tensor],
                    top_k: int, norm_topk_prob: bool = True):
    """LagunaMoEGate: x [..., H], gate_weight bf16 [E, H], bias f32 [E] -> (inds u32, w f32)."""
    _require_cuda("router", x, gate_weight, bias)
    if gate_weight.dtype != torch.bfloat16:
        raise ValueError("[router] gate weight must be bfloat16.")
    E, H = gate_weight.shape
    if x.shape[-1] != H:
        raise ValueError(f"[router] x last dimension {x.shape[-1]} does not match gate weight "
                         f"{tuple(gate_weight.shape)}.")
    xc = x.contiguous()
    T = xc.numel() // H
    inds = torch.empty(x.shape[:-1] + (top_k,), dtype=torch.uint32, device=x.device)
    wts = torch.empty(x.shape[:-1] + (top_k,), dtype=torch.float32, device=x.device)
    nbytes = lib().moe_router_workspace_size(T, H, E)
    ws = _router_ws.get(nbytes, x.device)
    b = None if bias is None else bias.to(torch.float32).contiguous()
    check(lib().moe_router_topk(_ptr(inds), _ptr(wts), _ptr(xc), _dtype_code(x, "router"),
                                _ptr(gate_weight.contiguous()), _ptr(b), T, H, E, int(top_k),
                                int(bool(norm_topk_prob)), _ptr(ws), ws.numel(),
                                _stream(x.device)))
    return inds, wts


class SparseMoeBlock:
    """LagunaSparseMoeBlock (Laguna.swift:183-213) over packed NVFP4 banks.

    routed: dict gate_w [E, I, H/8], gate_s [E, I, H/16], up_w, up_s, down_w [E, H, I/8], down_s.
    shared: same keys for the shared expert without the E dim, or None.
    """

    def __init__(self, routed: dict, shared: Optional[dict] = None,
                 router_weight: Optional[torch.Tensor] = None,
                 router_bias: Optional[torch.Tensor] = None, top_k: int = 8,
                 routed_scaling: float = 2.5, norm_topk_prob: bool = True):
        self.routed = {k: (v.view(torch.uint32) if v.dtype == torch.int32 else v).contiguous()
                       for k, v in routed.items()}
        self.shared = None if shared is None else {
            k: (v.view(torch.uint32) if v.dtype == torch.int32 else v).contiguous()
            for k, v in shared.items()}
        self.router_weight = None if router_weight is None else router_weight.contiguous()
        self.router_bias = None if router_bias is None else router_bias.to(
            torch.float32).contiguous()
        E, I, H8 = self.routed["gate_w"].shape
        self.E, self.I, self.H = E, I, H8 * 8
        self.Is = 0 if self.shared is None else self.shared["gate_w"].shape[0]
        self.top_k = top_k
        self.desc = MoeLayerDesc()
        d = self.desc
        d.hidden, d.inter, d.n_experts, d.top_k = self.H, self.I, E, top_k
        d.shared_inter = self.Is
        d.routed_scaling = float(routed_scaling)
        d.norm_topk_prob = int(bool(norm_topk_prob))
        d.router_w = None if self.router_weight is None else self.router_weight.data_ptr()
        d.router_bias = None if self.router_bias is None else self.router_bias.data_ptr()
        r = self.routed
        d.gate = NvFp4Bank(r["gate_w"].data_ptr(), r["gate_s"].data_ptr())
        d.up = NvFp4Bank(r["up_w"].data_ptr(), r["up_s"].data_ptr())
        d.down = NvFp4Bank(r["down_w"].data_ptr(), r["down_s"].data_ptr())
        if self.shared is not None:
            s = self.shared
            d.shared_gate = NvFp4Bank(s["gate_w"].data_ptr(), s["gate_s"].data_ptr())
            d.shared_up = NvFp4Bank(s["up_w"].data_ptr(), s["up_s"].data_ptr())
            d.shared_down = NvFp4Bank(s["down_w"].data_ptr(), s["down_s"].data_ptr())
        self._ws = _Workspace()

    def workspace_bytes(self, T: int) -> int:
        return lib().moe_block_workspace_size(ctypes.byref(self.desc), T)

    def __call__(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                 inds: Optional[torch.Tensor] = None, weights: Optional[torch.Tensor] = None,
                 return_routing: bool = False, out: Optional[torch.Tensor] = None):
        _require_cuda("moe_block", x, residual, inds, weights)
        H = self.H
        xc = x.contiguous()
        T = xc.numel() // H
        y = out if out is not None else torch.empty_like(xc)
        ws = self._ws.get(self.workspace_bytes(T), x.device)
        inds_out = wts_out = None
        if return_routing:
            inds_out = torch.empty((T, self.top_k), dtype=torch.uint32, device=x.device)
            wts_out = torch.empty((T, self.top_k), dtype=torch.float32, device=x.device)
        if inds is not None:
            inds = inds.to(torch.int32).view(torch.uint32).reshape(T, self.top_k).contiguous()
            weights = weights.to(torch.float32).reshape(T, self.top_k).contiguous()
        res = None if residual is None else residual.to(x.dtype).contiguous()
        check(lib().moe_block_forward(_ptr(y), _ptr(xc), _ptr(res), _dtype_code(x, "moe_block"),
                                      T, ctypes.byref(self.desc), _ptr(inds), _ptr(weights),
                                      _ptr(inds_out), _ptr(wts_out), _ptr(ws), ws.numel(),
                                      _stream(x.device)))
        y = y.reshape(x.shape)
        if return_routing:
            return y, inds_out, wts_out
        return y


from .decode import MoEDecodeChain  # noqa: E402
