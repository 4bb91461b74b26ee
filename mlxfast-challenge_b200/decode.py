"""Serial decode of a stack of sparse MoE layers as one CUDA graph.

The reference evaluates each decode step as a lazy MLX graph (eval at
LagunaRuntimeWorker.swift:369, the per-layer chain at
LagunaRuntimeModel.swift:11460 -> :11030 -> :10678).  On the B200 the same
chain is captured once into a CUDA graph: per layer the fused gate/up+SwiGLU
kernel and the fused down+combine kernel (C ABI moe_gate_up_swiglu /
moe_down_combine), the output of layer l feeding layer l+1.  A step replays
the graph, so launch overhead is paid once per step instead of per kernel.

With uniform layer shapes (the Laguna case) and one sequence (T = 1) the step
is instead ONE persistent launch over all layers: with given routing
moe_decode_stack_forward, which streams the next layers'
expert weights while the current layer's dependent chain runs; with
route=True (config[2]) moe_decode_stack_routed_forward, which runs each
layer's router inside the launch and streams a routed expert's weights from
the moment its layer's top-k is known.  stack=False keeps the per-layer
kernels (moe_block_forward per layer: with the router when route=True, the
GEMV engine at T = 1 and the grouped GEMMs from T = 2), which also serve
T > 1 and other shapes.

residual=True makes each layer h_{l+1} = h_l + block_l(x_l), the block output
summed into the residual stream, and norms (one RMSNorm weight per layer, in
the activation dtype) makes the block input x_l = RMSNorm(h_l) (else h_l):
with both, each layer is the decoder layer's MoE half, h + mlp(
postAttentionLayerNorm(h)) (Laguna.swift:242-246), without the attention
half.  Routed decode with norms and residual is the realistic serial step: the
norm keeps every layer's input at unit scale, as in the model.

MoEDecodeChain(blocks, routing)(x_host) is the end-to-end call: it copies the
step's input from pinned host memory, replays the graph and copies the result
back.  With route=True, self.routing[l] holds layer l's routing after a step.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple

import torch

from ._lib import check, lib


class MoEDecodeChain:
    def __init__(self, blocks: Sequence, routing: Optional[Sequence[Tuple[torch.Tensor,
                                                                           torch.Tensor]]],
                 T: int = 1, dtype=torch.bfloat16, route: bool = False, device="cuda:0",
                 stack: bool = True, residual: bool = False,
                 norms: Optional[Sequence[torch.Tensor]] = None, eps: float = 1e-6):
        self.blocks = list(blocks)
        self.T = T
        self.dtype = dtype
        self.route = route
        self.residual = residual
        self.norms = None if norms is None else [w.to(dtype).contiguous() for w in norms]
        self.eps = float(eps)
        self.device = torch.device(device)
        H = self.blocks[0].H
        self.H = H
        self.x0 = torch.zeros(T, H, dtype=dtype, device=self.device)
        self.bufs = [torch.zeros(T, H, dtype=dtype, device=self.device) for _ in range(2)]
        self.xn = torch.zeros(T, H, dtype=dtype, device=self.device)  # a layer's normed input
        self.routing = []
        for l, b in enumerate(self.blocks):
            if route:
                self.routing.append((torch.empty(T, b.top_k, dtype=torch.uint32, device=self.device),
                                     torch.empty(T, b.top_k, dtype=torch.float32,
                                                 device=self.device)))
            else:
                i, w = routing[l]
                self.routing.append((i.to(torch.int32).view(torch.uint32).reshape(T, b.top_k)
                                     .contiguous(), w.to(torch.float32).reshape(T, b.top_k)
                                     .contiguous()))
        nbytes = max(b.workspace_bytes(T) for b in self.blocks)
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        self.stream = torch.cuda.Stream(device=self.device)
        self.graph = None
        self.out = None
        from . import _dtype_code
        self._dt = _dtype_code(self.x0, "decode")
        # One persistent launch for the whole stack when the library accepts it
        # (the given-routing stack has no residual form).
        self.stack = False
        self.stack_fp4 = False
        if stack and T == 1 and len(self.blocks) <= 64 and (
                route or (not residual and self.norms is None)):
            from ._lib import MoeLayerDesc
            n = len(self.blocks)
            self._descs = (MoeLayerDesc * n)(*[b.desc for b in self.blocks])
            self._inds = (ctypes.c_void_p * n)(*[r[0].data_ptr() for r in self.routing])
            self._wts = (ctypes.c_void_p * n)(*[r[1].data_ptr() for r in self.routing])
            self._norm_ptrs = None if self.norms is None else (ctypes.c_void_p * n)(
                *[w.data_ptr() for w in self.norms])
            sb = lib().moe_decode_stack_workspace_size(self._descs, n)
            self._stack_ws = torch.zeros(max(sb, 256), dtype=torch.uint8, device=self.device)
            self.stack = self._try_stack()

    def _stack_call(self, stream_ptr) -> int:
        n = len(self.blocks)
        if self.route:
            self._stack_launches = lib().moe_decode_stack_routed_launches(self._descs, n)
            self.stack_fp4 = self._stack_launches > 0
            norms = (None if self._norm_ptrs is None
                     else ctypes.cast(self._norm_ptrs, ctypes.c_void_p))
            return lib().moe_decode_stack_routed_forward(
                self.bufs[0].data_ptr(), self.x0.data_ptr(), self._dt, n, self._descs,
                int(self.residual), norms, self.eps, ctypes.cast(self._inds, ctypes.c_void_p),
                ctypes.cast(self._wts, ctypes.c_void_p), self._stack_ws.data_ptr(),
                self._stack_ws.numel(), stream_ptr)
        self._stack_launches = lib().moe_decode_stack_launches(self._descs, n)
        self.stack_fp4 = bool(lib().moe_decode_stack_uses_fp4(self._descs, n))
        return lib().moe_decode_stack_forward(
            self.bufs[0].data_ptr(), self.x0.data_ptr(), self._dt, n, self._descs,
            ctypes.cast(self._inds, ctypes.c_void_p), ctypes.cast(self._wts, ctypes.c_void_p),
            self._stack_ws.data_ptr(), self._stack_ws.numel(), stream_ptr)

    def _try_stack(self) -> bool:
        """Whether the library runs this stack as one launch (shape checks only)."""
        s = torch.cuda.Stream(device=self.device)
        # after the caller's pending work: the stack's CTAs wait on one another
        # and must not share the GPU with another persistent stack in flight
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            st = self._stack_call(ctypes.c_void_p(s.cuda_stream))
        s.synchronize()
        return st == 0

    # -- one step as raw launches (captured below) --------------------------------
    def _launch_step(self, stream_ptr):
        L = lib()
        if self.stack:
            check(self._stack_call(stream_ptr))
            self.out = self.bufs[0]
            return
        src = self.x0
        for l, b in enumerate(self.blocks):
            dst = self.bufs[l % 2]
            inds, wts = self.routing[l]
            res = src.data_ptr() if self.residual else None
            inp = src
            if self.norms is not None:
                check(L.nvfp4_rms_norm(self.xn.data_ptr(), src.data_ptr(),
                                       self.norms[l].data_ptr(), self._dt, self.T, self.H,
                                       self.eps, stream_ptr))
                inp = self.xn
            if self.route:
                # Router + gate/up + down in one call: the library knows the
                # gate/up kernel must read the fresh routing after its wait.
                check(L.moe_block_forward(dst.data_ptr(), inp.data_ptr(), res, self._dt, self.T,
                                          ctypes.byref(b.desc), None, None, inds.data_ptr(),
                                          wts.data_ptr(), self.ws.data_ptr(), self.ws.numel(),
                                          stream_ptr))
                src = dst
                continue
            # given routing: the block with it (the GEMV engine at T = 1, the
            # grouped GEMMs from T = 2, as SparseMoeBlock runs it)
            check(L.moe_block_forward(dst.data_ptr(), inp.data_ptr(), res, self._dt, self.T,
                                      ctypes.byref(b.desc), inds.data_ptr(), wts.data_ptr(),
                                      None, None, self.ws.data_ptr(), self.ws.numel(),
                                      stream_ptr))
            src = dst
        self.out = src

    def launches_per_step(self) -> int:
        """Kernel launches of one step (the stack: as of its last call, whose
        launch flags choose the FP4 or the mma.sync stack)."""
        if self.stack:
            return self._stack_launches
        # per layer: the norm, the router (one kernel for T <= 8, logits + top-k
        # beyond), then the GEMV pair (T = 1) or the sort, two term passes, two
        # grouped GEMMs and the combine (T >= 2)
        router = 0 if not self.route else (1 if self.T <= 8 else 2)
        block = 2 if self.T == 1 else 6
        return len(self.blocks) * ((1 if self.norms else 0) + router + block)

    def capture(self, pdl: bool = True):
        """Capture one step.  With pdl, every kernel may start while its
        predecessor drains (programmatic dependent launch): the next layer's
        weights stream in before the previous layer's output is ready."""
        s = self.stream
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self._launch_step(ctypes.c_void_p(s.cuda_stream))  # warm (sets kernel attributes)
        s.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        L = lib()
        old = L.nvfp4_set_launch_flags(0)
        L.nvfp4_set_launch_flags((old & ~1) | (1 if pdl else 0))  # keep other flag bits
        try:
            with torch.cuda.graph(self.graph, stream=s):
                self._launch_step(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        finally:
            L.nvfp4_set_launch_flags(old)
        return self

    def replay(self):
        """Enqueue one step (inputs already in self.x0), ordered after the
        caller's current stream; the caller's stream then waits for it."""
        if self.graph is None:
            self.capture()
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            self.graph.replay()
        cur.wait_stream(self.stream)
        return self.out

    def __call__(self, x_host: torch.Tensor, y_host: Optional[torch.Tensor] = None):
        """End-to-end step: pinned host x -> device, all layers, device -> host y."""
        if self.graph is None:
            self.capture()
        if y_host is None:
            y_host = torch.empty(self.T, self.H, dtype=self.dtype, pin_memory=True)
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            self.x0.copy_(x_host.reshape(self.T, self.H), non_blocking=True)
            self.graph.replay()
            y_host.copy_(self.out, non_blocking=True)
        self.stream.synchronize()
        return y_host
