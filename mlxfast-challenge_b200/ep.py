"""Expert parallelism for the Laguna sparse MoE block over torch.distributed.

The 256 routed experts are split over the N ranks of a process group (one
process per GPU): rank r holds experts [r*E/N, (r+1)*E/N), every rank holds
the router and the shared expert.  Each rank runs the block for its own tokens:

1. route its tokens (BF16 router top-k, moe_router_topk);
2. build the send buffer: every (token, slot) pair's activation row grouped by
   the rank that owns the pair's expert (moe_ep_dispatch);
3. exchange the per-rank row counts, then the rows and their local expert ids
   (all-to-all; NCCL over NVLink on the GPUs);
4. run its local experts over the rows it received, one expert per row, with
   the grouped NVFP4 GEMM path (moe_block_forward, top-1, weight 1);
5. send the expert outputs back (all-to-all, the reverse splits);
6. combine in the Laguna order: y = 2.5 * sum_j w_j e_j(x) + shared(x)
   (+ residual) (moe_ep_combine).

Reference semantics: the single-device block (VLM/MLXLLM/Models/Laguna.swift:
183-213, SwitchGLU with sorted indices VLM/MLXLMCommon/SwitchLayers.swift:
532-580); the exchange has no reference counterpart.  Expert outputs travel as
the activation dtype (bf16), as the reference's gather_qmm returns them.

The exchange logic (ExpertParallelBlock) only moves tensors; the compute goes
through an ops object.  CudaEPOps is the product (C ABI kernels on the GPU, no
CPU fallback); tests may drive the same exchange with CPU ops on gloo ranks.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch
import torch.distributed as dist

from ._lib import check, lib


def exchange(send: torch.Tensor, send_counts, recv_counts, group=None) -> torch.Tensor:
    """Rows of `send` (grouped by destination rank, send_counts[r] rows for
    rank r) to their ranks; returns the rows received, grouped by source rank."""
    shape = (int(sum(recv_counts)),) + tuple(send.shape[1:])
    recv = torch.empty(shape, dtype=send.dtype, device=send.device)
    dist.all_to_all_single(recv, send, output_split_sizes=[int(c) for c in recv_counts],
                           input_split_sizes=[int(c) for c in send_counts], group=group)
    return recv


def exchange_counts(send_counts: torch.Tensor, group=None) -> torch.Tensor:
    recv = torch.empty_like(send_counts)
    dist.all_to_all_single(recv, send_counts, group=group)
    return recv


class ExpertParallelBlock:
    """One sparse block, expert-parallel over `group` (see the module doc)."""

    def __init__(self, ops, group=None):
        self.ops = ops
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def __call__(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                 routing: Optional[Tuple[torch.Tensor, torch.Tensor]] = None) -> torch.Tensor:
        ops = self.ops
        # The shared expert needs neither the routing nor the exchange: it
        # runs on a side stream, overlapping the all-to-alls (which leave most
        # SMs idle) and the local experts.
        side = self._side_stream(x)
        if side is not None:
            side.wait_stream(torch.cuda.current_stream(x.device))
            with torch.cuda.stream(side):
                shared = ops.shared(x)
        else:
            shared = ops.shared(x)
        inds, wts = routing if routing is not None else ops.route(x)
        send_x, send_ids, pos, send_counts = ops.dispatch(x, inds, self.world)
        # Counts travel as int64 on the exchange's device; the row splits are
        # host integers (one small device-to-host copy per layer).
        sc = send_counts.to(torch.int64)
        rc = exchange_counts(sc, self.group)
        sc_h, rc_h = sc.tolist(), rc.tolist()
        recv_x = exchange(send_x, sc_h, rc_h, self.group)
        recv_ids = exchange(send_ids, sc_h, rc_h, self.group)
        y_recv = ops.experts(recv_x, recv_ids)
        y_back = exchange(y_recv, rc_h, sc_h, self.group)
        if side is not None:
            torch.cuda.current_stream(x.device).wait_stream(side)
            if shared is not None:
                shared.record_stream(torch.cuda.current_stream(x.device))
        return ops.combine(y_back, pos, wts, shared, residual)

    def _side_stream(self, x: torch.Tensor):
        if not x.is_cuda:
            return None
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(device=x.device)
        return self._side


class CudaEPOps:
    """The device side of one rank: router, dispatch / combine kernels, local
    experts through moe_block_forward (C ABI).  `routed` holds this rank's
    expert slice (gate_w [E/N, I, H/8], ...), `shared` the shared expert."""

    def __init__(self, routed: dict, shared: Optional[dict], router_w: torch.Tensor,
                 router_b: Optional[torch.Tensor], n_experts: int, rank: int, world: int,
                 top_k: int = 8, routed_scaling: float = 2.5, norm_topk_prob: bool = True):
        from . import SparseMoeBlock
        self.E, self.rank, self.world = n_experts, rank, world
        self.epr = n_experts // world
        self.top_k, self.scaling, self.norm = top_k, float(routed_scaling), bool(norm_topk_prob)
        # Local experts as a top-1 block: scaling and weights are applied by the
        # source rank's combine.
        self.local = SparseMoeBlock(routed, None, None, None, top_k=1, routed_scaling=1.0,
                                    norm_topk_prob=False)
        self.shared_block = None
        if shared is not None:
            one = {k: v.unsqueeze(0) for k, v in shared.items()}
            self.shared_block = SparseMoeBlock(one, None, None, None, top_k=1,
                                               routed_scaling=1.0, norm_topk_prob=False)
        self.router_w = router_w.contiguous()
        self.router_b = None if router_b is None else router_b.to(torch.float32).contiguous()
        self.H = self.local.H

    def _stream(self, t):
        return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)

    def route(self, x):
        from . import moe_router_topk
        return moe_router_topk(x, self.router_w, self.router_b, self.top_k, self.norm)

    def dispatch(self, x, inds, world):
        from . import _dtype_code
        T, k = inds.shape
        P = T * k
        send_x = torch.empty(P, self.H, dtype=x.dtype, device=x.device)
        send_ids = torch.empty(P, dtype=torch.int32, device=x.device)
        pos = torch.empty(P, dtype=torch.int32, device=x.device)
        counts = torch.empty(world, dtype=torch.int32, device=x.device)
        xi = (inds if inds.dtype == torch.uint32 else inds.to(torch.int32).view(torch.uint32))
        xi = xi.contiguous()
        check(lib().moe_ep_dispatch(send_x.data_ptr(), send_ids.data_ptr(), pos.data_ptr(),
                                    counts.data_ptr(), x.contiguous().data_ptr(),
                                    _dtype_code(x, "moe_ep_dispatch"), xi.data_ptr(), T, k, self.H,
                                    self.epr, world, self._stream(x)))
        return send_x, send_ids, pos, counts

    def experts(self, rows, ids):
        if rows.shape[0] == 0:
            return torch.empty_like(rows)
        w = torch.ones(rows.shape[0], 1, dtype=torch.float32, device=rows.device)
        return self.local(rows, inds=ids.view(-1, 1), weights=w)

    def shared(self, x):
        if self.shared_block is None:
            return None
        T = x.shape[0]
        z = torch.zeros(T, 1, dtype=torch.int32, device=x.device)
        w = torch.ones(T, 1, dtype=torch.float32, device=x.device)
        return self.shared_block(x, inds=z, weights=w)

    def combine(self, y_pairs, pos, wts, shared, residual):
        from . import _dtype_code
        T, k = wts.shape
        y = torch.empty(T, self.H, dtype=y_pairs.dtype, device=y_pairs.device)
        res = None if residual is None else residual.to(y.dtype).contiguous()
        check(lib().moe_ep_combine(y.data_ptr(), y_pairs.data_ptr(), pos.data_ptr(),
                                   wts.to(torch.float32).contiguous().data_ptr(),
                                   None if shared is None else shared.data_ptr(),
                                   None if res is None else res.data_ptr(),
                                   _dtype_code(y, "moe_ep_combine"), T, k, self.H, self.scaling,
                                   self._stream(y)))
        return y


def local_slice(raw_routed: dict, rank: int, world: int) -> dict:
    """This rank's expert slice of full routed banks (views, no copy)."""
    E = next(iter(raw_routed.values())).shape[0]
    epr = E // world
    return {k: v[rank * epr:(rank + 1) * epr] for k, v in raw_routed.items()}


# ---------------------------------------------------------------------------
# Gather / reduce-scatter form.  Every rank all-gathers all ranks' tokens with
# their routing (one fixed-size collective), computes for every token the
# contribution of its own experts (moe_ep_partial_forward: f32 partial sums,
# foreign experts skipped), and a reduce-scatter sums the partials so each
# rank receives its own tokens' sum.  The shared expert either joins the
# partial call as one more group over the rank's own rows (CUDA ops: its GEMM
# work rides in the same launches) or comes from ops.shared on a side stream;
# moe_ep_finish adds it, if separate, and the residual.  Sizes are fixed (equal T per rank): no host synchronisation, and
# the whole call can be captured in a CUDA graph.  Same per-token order of
# the routed sum as the single-device block within a rank; across ranks the
# partials add in rank order inside the reduce-scatter.

def gather_rows(t: torch.Tensor, group=None) -> torch.Tensor:
    """[R, ...] on every rank -> [world * R, ...], rank-major."""
    world = dist.get_world_size(group)
    out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype,
                      device=t.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    else:
        dist.all_gather(list(out.chunk(world)), t.contiguous(), group=group)
    return out


def reduce_scatter_rows(t: torch.Tensor, group=None) -> torch.Tensor:
    """[world * R, ...] on every rank -> this rank's [R, ...] block of the sum."""
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    rows = t.shape[0] // world
    if dist.get_backend(group) == "nccl":
        out = torch.empty((rows,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.reduce_scatter_tensor(out, t.contiguous(), op=dist.ReduceOp.SUM, group=group)
        return out
    tmp = t.contiguous().clone()
    dist.all_reduce(tmp, op=dist.ReduceOp.SUM, group=group)
    return tmp[rank * rows:(rank + 1) * rows].clone()


def pack_tokens(x: torch.Tensor, inds: torch.Tensor, wts: torch.Tensor) -> torch.Tensor:
    """One byte row per token: x, then the k expert ids (u32), then the k
    weights (f32) -- 16-byte multiple for Laguna sizes."""
    T = x.shape[0]
    xb = x.contiguous().view(torch.uint8).reshape(T, -1)
    ib = inds.contiguous().to(torch.int32).view(torch.uint8).reshape(T, -1)
    wb = wts.contiguous().to(torch.float32).view(torch.uint8).reshape(T, -1)
    return torch.cat([xb, ib, wb], dim=1)


def unpack_tokens(rows: torch.Tensor, H: int, k: int, dtype: torch.dtype):
    esz = torch.empty(0, dtype=dtype).element_size()
    xb, ib, wb = rows[:, :H * esz], rows[:, H * esz:H * esz + 4 * k], rows[:, H * esz + 4 * k:]
    return (xb, ib.contiguous().view(torch.int32), wb.contiguous().view(torch.float32))


class GatherEPBlock:
    """One sparse block, expert-parallel over `group` in the gather /
    reduce-scatter form (see above).  `ops` supplies route, shared, partial
    and finish."""

    def __init__(self, ops, group=None):
        self.ops = ops
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self._side = None

    def __call__(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None,
                 routing: Optional[Tuple[torch.Tensor, torch.Tensor]] = None) -> torch.Tensor:
        ops = self.ops
        side = None
        shared = None
        if getattr(ops, "shared_in_partial", False):
            pass
        elif x.is_cuda:
            if self._side is None:
                self._side = torch.cuda.Stream(device=x.device)
            side = self._side
            side.wait_stream(torch.cuda.current_stream(x.device))
            with torch.cuda.stream(side):
                shared = ops.shared(x)
        else:
            shared = ops.shared(x)
        inds, wts = routing if routing is not None else ops.route(x)
        rows = gather_rows(pack_tokens(x, inds, wts), self.group)
        T = x.shape[0]
        part = ops.partial(rows, x.dtype, self.rank * T, T)  # [world * T, H]
        mine = reduce_scatter_rows(part, self.group)  # [T, H], the partials' dtype
        if side is not None:
            torch.cuda.current_stream(x.device).wait_stream(side)
            if shared is not None:
                shared.record_stream(torch.cuda.current_stream(x.device))
        return ops.finish(mine, shared, residual, x.dtype)


class CudaGatherEPOps:
    """Device side of one rank for GatherEPBlock: router, this rank's routed
    experts and the shared expert (on the rank's own rows) through
    moe_ep_partial_forward_typed, moe_ep_finish_typed.  partial_dtype: the
    partial sums' type on the wire -- torch.float32, or torch.bfloat16 (half
    the reduce-scatter bytes; each rank's partial rounded once to bf16)."""

    shared_in_partial = True

    def __init__(self, routed: dict, shared: Optional[dict], router_w: torch.Tensor,
                 router_b: Optional[torch.Tensor], n_experts: int, rank: int, world: int,
                 top_k: int = 8, routed_scaling: float = 2.5, norm_topk_prob: bool = True,
                 partial_dtype: torch.dtype = torch.float32):
        from . import SparseMoeBlock
        if partial_dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("[moe_ep] partials are float32 or bfloat16")
        self.partial_dtype = partial_dtype
        self.E, self.rank, self.world = n_experts, rank, world
        self.epr = n_experts // world
        self.top_k, self.norm = top_k, bool(norm_topk_prob)
        self.local = SparseMoeBlock(routed, shared, None, None, top_k=top_k,
                                    routed_scaling=routed_scaling, norm_topk_prob=norm_topk_prob)
        self.router_w = router_w.contiguous()
        self.router_b = None if router_b is None else router_b.to(torch.float32).contiguous()
        self.H = self.local.H
        self._ws = {}

    def _stream(self, t):
        return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)

    def route(self, x):
        from . import moe_router_topk
        return moe_router_topk(x, self.router_w, self.router_b, self.top_k, self.norm)

    # moe_ep_partial_forward's FP4 GEMMs hold the batch's tile list
    # (E + ceil(T k / 32) + ceil(T / 32) entries) in shared memory; this many
    # entries always fit.  A longer gathered batch runs as several calls over
    # consecutive row ranges (tokens are independent).
    MAX_TILES = 4096

    def chunk_tokens(self, Tt: int) -> int:
        """Rows per moe_ep_partial_forward call for a gathered batch of Tt."""
        if Tt <= 1:
            return 1
        sh = self.local.desc.shared_inter > 0
        n = 1
        while True:
            c = -(-Tt // n)
            tiles = self.epr + -(-c * self.top_k // 32) + (-(-c // 32) if sh else 0)
            if tiles <= self.MAX_TILES or c <= 1:
                return c
            n += 1

    def _routed_only_desc(self):
        # the layer without its shared expert, for a row range holding none of
        # this rank's own tokens
        d = getattr(self, "_desc_routed", None)
        if d is None:
            d = type(self.local.desc).from_buffer_copy(self.local.desc)
            d.shared_inter = 0
            for f in ("shared_gate", "shared_up", "shared_down"):
                setattr(d, f, type(d.shared_gate)())
            self._desc_routed = d
        return d

    def partial(self, rows, dtype, row0, nrows):
        from . import _dtype_code
        H, k = self.H, self.top_k
        xb, ids, wts = unpack_tokens(rows, H, k, dtype)
        Tt = rows.shape[0]
        esz = torch.empty(0, dtype=dtype).element_size()
        c = self.chunk_tokens(Tt)
        nbytes = int(lib().moe_ep_partial_workspace_size(ctypes.byref(self.local.desc), c))
        ws = self._ws.get(c)
        if ws is None or ws.numel() < nbytes:
            ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=rows.device)
            self._ws[c] = ws
        y = torch.empty(Tt, H, dtype=self.partial_dtype, device=rows.device)
        probe = torch.empty(0, dtype=dtype, device=rows.device)
        sh = self.local.desc.shared_inter > 0
        for c0 in range(0, Tt, c):
            c1 = min(Tt, c0 + c)
            s0, s1 = max(row0, c0), min(row0 + nrows, c1)  # own rows in this range
            desc = self.local.desc if (not sh or s1 > s0) else self._routed_only_desc()
            r0, rn = (s0 - c0, s1 - s0) if (sh and s1 > s0) else (0, 0)
            check(lib().moe_ep_partial_forward_typed(
                y[c0:].data_ptr(), _dtype_code(y, "moe_ep"), rows[c0:].data_ptr(),
                rows.shape[1] // esz, _dtype_code(probe, "moe_ep"),
                c1 - c0, ctypes.byref(desc), ids[c0:].data_ptr(), wts[c0:].data_ptr(),
                self.rank * self.epr, r0, rn, ws.data_ptr(), ws.numel(), self._stream(rows)))
        return y

    def finish(self, mine, shared, residual, dtype):
        from . import _dtype_code
        T, H = mine.shape
        y = torch.empty(T, H, dtype=dtype, device=mine.device)
        res = None if residual is None else residual.to(dtype).contiguous()
        check(lib().moe_ep_finish_typed(y.data_ptr(), mine.data_ptr(),
                                        _dtype_code(mine, "moe_ep_finish"),
                                        None if shared is None else shared.data_ptr(),
                                        None if res is None else res.data_ptr(),
                                        _dtype_code(y, "moe_ep_finish"), T, H, self._stream(y)))
        return y
