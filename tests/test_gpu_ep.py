"""GPU checks of the expert-parallel path with the real kernels: the dispatch
plan / pack contract, the combine, and N-rank data flow simulated in one
process (the all-to-all replaced by the same row shuffle done in Python), which
must reproduce the single-GPU sparse block.  The multi-process NCCL exchange
itself is covered by the gloo test on the CPU and by bench.py --gpus N."""
import importlib

import numpy as np
import pytest
import torch

from conftest import PKG, assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.mark.parametrize("T,world", [(37, 4), (512, 8), (9, 2), (1, 2)])
def test_dispatch_contract(nv, T, world):
    ep = importlib.import_module(PKG + ".ep")
    E, k, H = 256, 8, 2048
    g = torch.Generator(device="cpu").manual_seed(T + world)
    inds = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    dev_inds, dev_x = inds.to(DEV), x.to(DEV)

    class Dummy:  # only dispatch is used
        H = 2048
        epr = E // world
        _stream = ep.CudaEPOps._stream
    send_x, send_ids, pos, counts = ep.CudaEPOps.dispatch(Dummy(), dev_x, dev_inds, world)
    torch.cuda.synchronize()
    dest = (inds.reshape(-1) // (E // world)).numpy()
    order = np.argsort(dest, kind="stable")
    want_pos = np.empty(T * k, np.int64)
    want_pos[order] = np.arange(T * k)
    assert np.array_equal(pos.cpu().numpy(), want_pos)
    assert np.array_equal(counts.cpu().numpy(), np.bincount(dest, minlength=world))
    assert np.array_equal(send_ids.cpu().numpy(), (inds.reshape(-1).numpy() % (E // world))[order])
    rows = x.reshape(T, 1, H).expand(T, k, H).reshape(T * k, H)[torch.from_numpy(order)]
    assert torch.equal(send_x.cpu(), rows)


def test_combine_matches_torch(nv):
    ep = importlib.import_module(PKG + ".ep")
    T, k, H = 33, 8, 2048
    g = torch.Generator(device=DEV).manual_seed(4)
    yp = torch.randn(T * k, H, generator=g, device=DEV).to(torch.bfloat16)
    perm = torch.randperm(T * k, generator=torch.Generator().manual_seed(1)).to(torch.int32).to(DEV)
    wts = torch.softmax(torch.randn(T, k, generator=g, device=DEV), -1)
    shared = torch.randn(T, H, generator=g, device=DEV).to(torch.bfloat16)
    res = torch.randn(T, H, generator=g, device=DEV).to(torch.bfloat16)

    class Dummy:
        H = 2048
        scaling = 2.5
        _stream = ep.CudaEPOps._stream
    y = ep.CudaEPOps.combine(Dummy(), yp, perm, wts, shared, res)
    want = (2.5 * (wts.unsqueeze(-1) * yp.float()[perm.long()].reshape(T, k, H)).sum(1)
            + shared.float() + res.float())
    assert_close(y.float().cpu().numpy(), want.cpu().numpy(), max_abs=4e-2, what="combine")


def simulate(ops, xs, routings):
    """ExpertParallelBlock's steps for len(ops) ranks in one process."""
    W = len(ops)
    sends = [ops[r].dispatch(xs[r], routings[r][0], W) for r in range(W)]
    counts = [s[3].cpu().tolist() for s in sends]
    offs = [np.concatenate([[0], np.cumsum(c)]) for c in counts]
    # rank d receives, from each source r in order, rows offs[r][d]:offs[r][d+1]
    recv_x = [torch.cat([sends[r][0][offs[r][d]:offs[r][d + 1]] for r in range(W)]) for d in range(W)]
    recv_i = [torch.cat([sends[r][1][offs[r][d]:offs[r][d + 1]] for r in range(W)]) for d in range(W)]
    y_recv = [ops[d].experts(recv_x[d], recv_i[d]) for d in range(W)]
    outs = []
    for r in range(W):
        back = []
        for d in range(W):
            start = sum(counts[q][d] for q in range(r))
            back.append(y_recv[d][start:start + counts[r][d]])
        y_back = torch.cat(back)
        outs.append(ops[r].combine(y_back, sends[r][2], routings[r][1], ops[r].shared(xs[r]),
                                   None))
    return outs


@pytest.mark.parametrize("world,T", [(2, 64), (4, 100), (8, 512)])
def test_simulated_ranks_match_single_block(nv, world, T):
    ep = importlib.import_module(PKG + ".ep")
    lag = importlib.import_module(PKG + ".laguna")
    block, raw = lag.random_sparse_layer(nv, seed=31, device=DEV)
    ops = [ep.CudaEPOps(ep.local_slice(raw["routed"], r, world), raw["shared"], raw["router_w"],
                        raw["router_b"], 256, r, world) for r in range(world)]
    xs = [torch.randn(T + r, 2048, generator=torch.Generator(device=DEV).manual_seed(r),
                      device=DEV).to(torch.bfloat16) for r in range(world)]
    routings = [ops[r].route(xs[r]) for r in range(world)]
    outs = simulate(ops, xs, routings)
    torch.cuda.synchronize()
    nv.device_status()
    for r in range(world):
        want = block(xs[r], inds=routings[r][0].view(torch.int32), weights=routings[r][1])
        # expert outputs cross the exchange as bf16 (one rounding more than the
        # single-GPU path's f32 expert sums): path-vs-path bound as for prefill
        assert_close(outs[r].float().cpu().numpy(), want.float().cpu().numpy(), max_abs=4e-2,
                     what=f"rank {r} of {world}")


@pytest.mark.parametrize("world,T,pdt", [(2, 64, torch.float32), (4, 100, torch.float32),
                                         (8, 512, torch.float32), (2, 64, torch.bfloat16),
                                         (8, 512, torch.bfloat16), (8, 2048, torch.bfloat16)])
def test_gather_form_simulated_ranks_match_single_block(nv, world, T, pdt):
    """GatherEPBlock's steps for `world` ranks in one process: every rank's
    partial over all gathered tokens (moe_ep_partial_forward_typed, foreign
    experts skipped; f32 or bf16 partials), the reduce-scatter as a sum in the
    partials' dtype, moe_ep_finish_typed with the shared expert and the
    residual -- against the single-GPU block.  At 8 x 2048 the gathered
    batch (16384 tokens) runs as two partial calls per rank, one of them
    without the rank's own rows (no shared expert)."""
    ep = importlib.import_module(PKG + ".ep")
    lag = importlib.import_module(PKG + ".laguna")
    block, raw = lag.random_sparse_layer(nv, seed=37, device=DEV)
    ops = [ep.CudaGatherEPOps(ep.local_slice(raw["routed"], r, world), raw["shared"],
                              raw["router_w"], raw["router_b"], 256, r, world,
                              partial_dtype=pdt)
           for r in range(world)]
    g = torch.Generator(device=DEV).manual_seed(world)
    xs = [torch.randn(T, 2048, generator=g, device=DEV).to(torch.bfloat16) for _ in range(world)]
    res = [torch.randn(T, 2048, generator=g, device=DEV).to(torch.bfloat16) for _ in range(world)]
    routings = [ops[r].route(xs[r]) for r in range(world)]
    rows = torch.cat([ep.pack_tokens(xs[r], *routings[r]) for r in range(world)])
    partials = [ops[d].partial(rows, torch.bfloat16, d * T, T) for d in range(world)]
    assert all(p.dtype == pdt for p in partials)
    total = sum(partials)  # the reduce-scatter, all blocks at once (bf16: rounded per add)
    torch.cuda.synchronize()
    nv.device_status()
    for r in range(world):
        mine = total[r * T:(r + 1) * T].contiguous()
        y = ops[r].finish(mine, None, res[r], torch.bfloat16)
        want = block(xs[r], residual=res[r], inds=routings[r][0].view(torch.int32),
                     weights=routings[r][1])
        assert_close(y.float().cpu().numpy(), want.float().cpu().numpy(), max_abs=4e-2,
                     what=f"gather form, rank {r} of {world}")


def test_ep_partial_skips_foreign_experts_without_error(nv):
    """Ids outside the rank's range contribute nothing and raise no device
    error; a token with no local pair gets a zero partial."""
    ep = importlib.import_module(PKG + ".ep")
    lag = importlib.import_module(PKG + ".laguna")
    _, raw = lag.random_sparse_layer(nv, seed=5, device=DEV)
    world, T = 4, 40
    op1 = ep.CudaGatherEPOps(ep.local_slice(raw["routed"], 1, world), None, raw["router_w"],
                             raw["router_b"], 256, 1, world)
    x = torch.randn(T, 2048, device=DEV).to(torch.bfloat16)
    inds, wts = op1.route(x)
    inds = inds.clone()
    inds[:10] = torch.arange(8, dtype=torch.int32, device=DEV).view(inds.dtype)  # experts 0-7: rank 0
    part = op1.partial(ep.pack_tokens(x, inds, wts), torch.bfloat16, 0, T)
    nv.device_status()
    assert torch.count_nonzero(part[:10]) == 0
    assert torch.isfinite(part).all()
