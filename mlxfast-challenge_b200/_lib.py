"""ctypes binding of libnvfp4moe.so (include/nvfp4moe.h).

The library is built in-tree by ``build.py``.  Loading fails loudly when the
file is missing: there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libnvfp4moe.so")

NVFP4_OK = 0
NVFP4_ERR_INVALID = 1
NVFP4_ERR_UNSUPPORTED = 2
NVFP4_ERR_CUDA = 3
NVFP4_ERR_WORKSPACE = 4
NVFP4_ERR_DEVICE_INDEX = 5
NVFP4_ERR_DEVICE_TIMEOUT = 6

NVFP4_BF16, NVFP4_F16, NVFP4_F32 = 0, 1, 2
NVFP4_LAUNCH_PDL = 1
NVFP4_LAUNCH_BULK_COPY = 2
NVFP4_LAUNCH_EXACT_PREFILL = 4
NVFP4_LAUNCH_EXACT_DECODE = 8
NVFP4_LAUNCH_TEST_EXPIRE = 16

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_SZ = ctypes.c_size_t


class NvFp4Bank(ctypes.Structure):
    _fields_ = [("w", _P), ("scales", _P)]


class MoeLayerDesc(ctypes.Structure):
    _fields_ = [
        ("hidden", _I64), ("inter", _I64), ("n_experts", _I64), ("top_k", _I64),
        ("shared_inter", _I64), ("routed_scaling", ctypes.c_float), ("norm_topk_prob", _I),
        ("router_w", _P), ("router_bias", _P),
        ("gate", NvFp4Bank), ("up", NvFp4Bank), ("down", NvFp4Bank),
        ("shared_gate", NvFp4Bank), ("shared_up", NvFp4Bank), ("shared_down", NvFp4Bank),
    ]


# Every symbol declared in include/nvfp4moe.h with its ctypes signature.
SIGNATURES = {
    "nvfp4_last_error": (ctypes.c_char_p, []),
    "nvfp4_set_error_handler": (None, [_P, _P]),
    "nvfp4_version": (_I, []),
    "nvfp4_set_launch_flags": (_I, [_I]),
    "nvfp4_device_status": (_I, []),
    "nvfp4_dequantize": (_I, [_P, _I, _P, _P, _I64, _I64, _P]),
    "nvfp4_quantize": (_I, [_P, _P, _P, _I, _I64, _I64, _P]),
    "nvfp4_quantized_matmul": (_I, [_P, _P, _I, _P, _P, _I64, _I64, _I64, _P]),
    "nvfp4_quantize_activations": (_I, [_P, _P, _P, _I, _I64, _I64, _P]),
    "nvfp4_qqmm_workspace_size": (ctypes.c_size_t, [_I64, _I64, _I64]),
    "moe_ep_partial_workspace_size": (ctypes.c_size_t, [_P, _I64]),
    "moe_ep_partial_forward": (_I, [_P, _P, _I64, _I, _I64, _P, _P, _P, _I64, _I64, _I64, _P,
                                    ctypes.c_size_t, _P]),
    "moe_ep_finish": (_I, [_P, _P, _P, _P, _I, _I64, _I64, _P]),
    "moe_ep_partial_forward_typed": (_I, [_P, _I, _P, _I64, _I, _I64, _P, _P, _P, _I64, _I64,
                                          _I64, _P, ctypes.c_size_t, _P]),
    "moe_ep_finish_typed": (_I, [_P, _P, _I, _P, _P, _I, _I64, _I64, _P]),
    "nvfp4_qqmm": (_I, [_P, _P, _I, _P, _P, _I64, _I64, _I64, _P, ctypes.c_size_t, _P]),
    "nvfp4_gather_qmm": (_I, [_P, _P, _I, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64,
                              _I, _P]),
    "moe_router_workspace_size": (_SZ, [_I64, _I64, _I64]),
    "moe_router_topk": (_I, [_P, _P, _P, _I, _P, _P, _I64, _I64, _I64, _I, _I, _P, _SZ, _P]),
    "moe_block_workspace_size": (_SZ, [ctypes.POINTER(MoeLayerDesc), _I64]),
    "moe_workspace_init": (_I, [_P, _SZ, _P]),
    "nvfp4_rms_norm": (_I, [_P, _P, _P, _I, _I64, _I64, ctypes.c_float, _P]),
    "moe_block_forward": (_I, [_P, _P, _P, _I, _I64, ctypes.POINTER(MoeLayerDesc), _P, _P, _P,
                               _P, _P, _SZ, _P]),
    "moe_block_forward_noalloc": (_I, [_P, _P, _P, _I, _I64, ctypes.POINTER(MoeLayerDesc), _P,
                                       _P, _P, _P, _P]),
    "moe_gate_up_swiglu": (_I, [_P, _I64, _P, _I, _I64, ctypes.POINTER(MoeLayerDesc), _P, _P]),
    "moe_down_combine": (_I, [_P, _P, _I64, _P, _I, _I64, ctypes.POINTER(MoeLayerDesc), _P, _P,
                              _P]),
    "moe_decode_stack_workspace_size": (_SZ, [ctypes.POINTER(MoeLayerDesc), _I64]),
    "moe_decode_stack_launches": (_I, [ctypes.POINTER(MoeLayerDesc), _I64]),
    "moe_decode_stack_uses_fp4": (_I, [ctypes.POINTER(MoeLayerDesc), _I64]),
    "moe_decode_stack_forward": (_I, [_P, _P, _I, _I64, ctypes.POINTER(MoeLayerDesc), _P, _P, _P,
                                      _SZ, _P]),
    "moe_decode_stack_routed_launches": (_I, [ctypes.POINTER(MoeLayerDesc), _I64]),
    "moe_decode_stack_routed_forward": (_I, [_P, _P, _I, _I64, ctypes.POINTER(MoeLayerDesc), _I,
                                             _P, ctypes.c_float, _P, _P, _P, _SZ, _P]),
    "moe_ep_dispatch": (_I, [_P, _P, _P, _P, _P, _I, _P, _I64, _I, _I64, _I64, _I, _P]),
    "moe_ep_combine": (_I, [_P, _P, _P, _P, _P, _P, _I, _I64, _I, _I64, ctypes.c_float, _P]),
}

_lib = None


def lib():
    """Load (once) and return the CDLL with typed entry points."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libnvfp4moe.so not built at {LIB_PATH}; run build.py (there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class DeviceIndexError(IndexError):
    pass


class DeviceTimeoutError(RuntimeError):
    """A kernel's bounded wait gave up; its outputs are not valid."""


def check(status: int) -> None:
    """Raise the Python exception the reference raises for the same failure."""
    if status == NVFP4_OK:
        return
    msg = lib().nvfp4_last_error().decode(errors="replace")
    if status == NVFP4_ERR_INVALID:
        raise ValueError(msg)  # std::invalid_argument in MLX -> ValueError
    if status == NVFP4_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if status == NVFP4_ERR_WORKSPACE:
        raise ValueError(msg)
    if status == NVFP4_ERR_DEVICE_INDEX:
        raise DeviceIndexError(msg)
    if status == NVFP4_ERR_DEVICE_TIMEOUT:
        raise DeviceTimeoutError(msg)
    raise RuntimeError(msg)
