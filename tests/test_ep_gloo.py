"""Expert-parallel exchange (mlxfast-challenge_b200/ep.py) on two gloo ranks on
the CPU.  The device kernels are replaced by CPU ops built on the oracle
(test-only), so what is checked here is the distributed data flow: counts
exchange, uneven all-to-all splits, the return path and the combine order
(all-to-all form); token/routing gather, foreign-expert skipping and the
reduce-scatter of partial sums (gather form).  Each rank's output must equal
the single-process block over all experts."""
import importlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG, assert_close

E, H, I, K, T = 8, 64, 32, 2, 5
SCALING = 2.5


def make_layer(seed=0):
    import oracle
    rng = np.random.default_rng(seed)

    def bank(rows, k):
        w = (rng.standard_normal((rows, k)) * 0.05).astype(np.float32)
        return oracle.port.quantize(w)

    routed = {"gate_w": [], "gate_s": [], "up_w": [], "up_s": [], "down_w": [], "down_s": []}
    for _ in range(E):
        for name, (r, k) in {"gate": (I, H), "up": (I, H), "down": (H, I)}.items():
            q, s = bank(r, k)
            routed[name + "_w"].append(q)
            routed[name + "_s"].append(s)
    routed = {k: np.stack(v) for k, v in routed.items()}
    shared = {}
    for name, (r, k) in {"gate": (I, H), "up": (I, H), "down": (H, I)}.items():
        shared[name + "_w"], shared[name + "_s"] = bank(r, k)
    return routed, shared


class CpuOps:
    """Oracle-backed stand-in for CudaEPOps on one rank (test only)."""

    def __init__(self, routed, shared, rank, world):
        import oracle
        self.port = oracle.port
        self.epr = E // world
        self.local = {k: v[rank * self.epr:(rank + 1) * self.epr] for k, v in routed.items()}
        self.shared_b = shared

    def dispatch(self, x, inds, world):
        # The C ABI's contract: rows grouped by destination rank, pair order
        # inside a rank; pos[p] = row of pair p.
        inds = inds.numpy().astype(np.int64)
        P = inds.size
        dest = (inds.reshape(-1) // self.epr)
        order = np.argsort(dest, kind="stable")
        pos = np.empty(P, np.int32)
        pos[order] = np.arange(P, dtype=np.int32)
        send_x = x.reshape(-1, 1, H).expand(-1, K, H).reshape(P, H)[torch.from_numpy(order)]
        send_ids = torch.from_numpy((inds.reshape(-1) % self.epr)[order].astype(np.int32))
        counts = torch.from_numpy(np.bincount(dest, minlength=world).astype(np.int32))
        return send_x.contiguous(), send_ids, torch.from_numpy(pos), counts

    def experts(self, rows, ids):
        if rows.shape[0] == 0:
            return rows.clone()
        y = self.port.moe_block_f32(rows.numpy(), ids.numpy().astype(np.uint32).reshape(-1, 1),
                                    np.ones((rows.shape[0], 1), np.float32), self.local, None,
                                    scaling=1.0)
        return torch.from_numpy(y.astype(np.float32))

    def shared(self, x):
        n = x.shape[0]
        one = {k: v[None] for k, v in self.shared_b.items()}
        y = self.port.moe_block_f32(x.numpy(), np.zeros((n, 1), np.uint32),
                                    np.ones((n, 1), np.float32), one, None, scaling=1.0)
        return torch.from_numpy(y.astype(np.float32))

    def combine(self, y_pairs, pos, wts, shared, residual):
        yp = y_pairs[pos.long()].reshape(-1, K, H)
        y = SCALING * (wts.reshape(-1, K, 1) * yp).sum(1) + shared
        return y if residual is None else y + residual


def worker(rank, world, port, out):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ep = importlib.import_module(PKG + ".ep")
    routed, shared = make_layer()
    rng = np.random.default_rng(100 + rank)
    x = torch.from_numpy(rng.standard_normal((T + rank, H)).astype(np.float32))
    # Skewed routing: rank 0 sends most pairs to rank 1's experts.
    inds = torch.from_numpy(np.stack([rng.permutation(E)[:K] for _ in range(T + rank)]))
    if rank == 0:
        inds[:, 0] = E - 1
    wts = torch.softmax(torch.from_numpy(rng.standard_normal((T + rank, K)).astype(np.float32)), -1)
    block = ep.ExpertParallelBlock(CpuOps(routed, shared, rank, world))
    y = block(x, routing=(inds, wts))
    out[rank] = (x.numpy(), inds.numpy(), wts.numpy(), y.numpy())
    dist.barrier()
    dist.destroy_process_group()


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_ep_exchange_two_gloo_ranks_matches_single_block(orc):
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(worker, args=(world, free_port(), out), nprocs=world, join=True)
    routed, shared = make_layer()
    for r in range(world):
        x, inds, wts, y = out[r]
        want = orc.port.moe_block_f32(x, inds.astype(np.uint32), wts, routed, shared,
                                      scaling=SCALING)
        assert_close(y, want, what=f"rank {r}")


class CpuGatherOps:
    """Oracle-backed stand-in for CudaGatherEPOps on one rank (test only)."""

    def __init__(self, routed, shared, rank, world):
        import oracle
        self.port = oracle.port
        self.rank = rank
        self.epr = E // world
        self.local = {k: v[rank * self.epr:(rank + 1) * self.epr] for k, v in routed.items()}
        self.shared_b = shared

    def shared(self, x):
        n = x.shape[0]
        one = {k: v[None] for k, v in self.shared_b.items()}
        y = self.port.moe_block_f32(x.numpy(), np.zeros((n, 1), np.uint32),
                                    np.ones((n, 1), np.float32), one, None, scaling=1.0)
        return torch.from_numpy(y.astype(np.float32))

    def partial(self, rows, dtype, row0, nrows):
        ep = importlib.import_module(PKG + ".ep")
        xb, ids, wts = ep.unpack_tokens(rows, H, K, dtype)
        x = xb.contiguous().view(dtype).numpy()
        ids = ids.numpy().astype(np.int64) - self.rank * self.epr
        local = (ids >= 0) & (ids < self.epr)
        w = np.where(local, wts.numpy(), 0.0).astype(np.float32)   # foreign pairs weigh 0
        i = np.where(local, ids, 0).astype(np.uint32)
        y = self.port.moe_block_f32(x, i, w, self.local, None, scaling=SCALING)
        return torch.from_numpy(y.astype(np.float32))

    def finish(self, mine, shared, residual, dtype):
        y = mine + shared
        return (y if residual is None else y + residual).to(dtype)


def worker_gather(rank, world, port, out):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ep = importlib.import_module(PKG + ".ep")
    routed, shared = make_layer()
    rng = np.random.default_rng(200 + rank)
    x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32))
    inds = torch.from_numpy(np.stack([rng.permutation(E)[:K] for _ in range(T)]))
    if rank == 0:
        inds[:, 0] = E - 1  # skew: rank 0's tokens all hit one of rank 1's experts
    wts = torch.softmax(torch.from_numpy(rng.standard_normal((T, K)).astype(np.float32)), -1)
    res = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32))
    block = ep.GatherEPBlock(CpuGatherOps(routed, shared, rank, world))
    y = block(x, residual=res, routing=(inds, wts))
    out[rank] = (x.numpy(), inds.numpy(), wts.numpy(), res.numpy(), y.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_ep_gather_two_gloo_ranks_matches_single_block(orc):
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(worker_gather, args=(world, free_port(), out), nprocs=world, join=True)
    routed, shared = make_layer()
    for r in range(world):
        x, inds, wts, res, y = out[r]
        want = orc.port.moe_block_f32(x, inds.astype(np.uint32), wts, routed, shared,
                                      scaling=SCALING, residual=res)
        assert_close(y, want, what=f"rank {r}")


@pytest.mark.parametrize("Tt,epr,k,shared,want", [
    (4096, 32, 8, True, 4096),      # BASELINE config[3] at 8 GPUs: one call
    (16384, 32, 8, True, 8192),     # 8 x 2048 tokens: two calls
    (16384, 256, 8, False, 8192),   # one rank, no shared expert
    (100000, 32, 16, True, 7143),   # 14 calls (13 would need 4120 entries)
    (0, 32, 8, True, 1),            # an empty batch: no call, an empty partial
])
def test_gather_partial_chunk_rule(Tt, epr, k, shared, want):
    """CudaGatherEPOps.partial splits a gathered batch into the fewest equal
    row ranges whose FP4 tile list (E + ceil(T k / 32) + ceil(T / 32) with a
    shared expert) stays within MAX_TILES."""
    ep = importlib.import_module(PKG + ".ep")

    class Desc:
        shared_inter = 512 if shared else 0

    class Local:
        desc = Desc()

    class Ops:
        MAX_TILES = ep.CudaGatherEPOps.MAX_TILES
        local = Local()

    o = Ops()
    o.epr, o.top_k = epr, k
    c = ep.CudaGatherEPOps.chunk_tokens(o, Tt)
    assert c == want
    tiles = epr + -(-c * k // 32) + (-(-c // 32) if shared else 0)
    assert tiles <= ep.CudaGatherEPOps.MAX_TILES
