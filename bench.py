#!/usr/bin/env python
"""Benchmark of the NVFP4 MoE decode hot path (Laguna XS 2.1 sparse layers).

Headline workload (BASELINE config[2] at one sequence, the Laguna decode the
metric is quoted on): the full sparse block at decode, T=1 -- RMSNorm, the
BF16 router [256, 2048] top-8 computed on the device, 256 routed NVFP4
experts (SwiGLU gate/up [512, 2048], down [2048, 512], group 16), the NVFP4
shared expert, summed into the bf16 residual stream -- for each of the
model's 39 sparse layers in turn: h_{l+1} = h_l + block_l(RMSNorm_l(h_l)),
the decoder layers' MoE halves without the attention halves.  The routing of
layer l+1 depends on layer l's output, so no routed expert's weights can be
fetched before its layer's router has run.  Weights are random-init (bf16
N(0, 0.02) quantized with the reference's nvfp4 quantizer, router N(0, 0.02),
norm weights 1 + N(0, 0.1)); the input h_0 is bf16 N(0, 1).  One step streams
39 x ~17 MB of weights, far more than the 126 MB L2, so no timed iteration is
served from L2.

value   = algorithmic HBM bytes of all ranks' steps / device time (GB/s): per
          layer the router, the shared expert, the distinct routed experts the
          router chose (counted from its outputs), the norm weight and the
          activations; device time with CUDA events around K CUDA-graph
          replays, max over ranks.
e2e     = the same metric through the public API MoEDecodeChain(x_host): per
          step the input is copied from pinned host memory, the layers run and
          the output is read back to the host.
roofline= the dominant kernel timed alone: the routed persistent decode stack
          (moe_decode_stack_fp4_kernel, routed form), which is the whole step.

--impl reference times the reference's own MLX CPU kernel (fp_qmm_t for bf16
x, compiled from the reference sources into oracle/_ref) for the same layer
(8 routed experts and the shared expert; the router and norm, which MLX
evaluates with its generic ops, through the CPU restatement), with all host
threads, one sparse layer per step.

Also reported on the same line (rank 0, N=1 runs):
decode_given_routing = BASELINE config[1]: the routed experts only, routing
          given for all 39 layers before the step (the persistent stack
          streams later layers' experts ahead).
decode_b8 = config[2] at 8 sequences (T=8) through the per-layer kernels
          (RMSNorm, router, fused gate/up and down + combine per layer).
prefill = BASELINE config[3] on one GPU: the full sparse block (BF16 router
          top-8, 256 routed experts, shared expert, residual) at T=512 tokens,
          39 sparse layers per step (4 distinct random-init layers cycled, 452 MB
          of NVFP4 weights each, > L2), through SparseMoeBlock; 512-token
          prefill tok/s of the MoE blocks and the HBM GB/s that moving every
          used weight once would need in that time.
dense   = BASELINE config[0]: quantized_matmul x[M, 2048] @ W[4096, 2048]^T,
          M = 512 (tensor-core GEMM, TFLOP/s) and M = 1 (GEMV, GB/s), cycling 32
          weight copies (150 MB > L2).

prefill_ep (N > 1 only) = config[3] expert-parallel: each GPU holds 256/N
          experts (+ router and shared expert) and its own 512 tokens; pair
          rows go to their experts' GPU and back by NCCL; total tok/s over all
          GPUs, device time max over ranks.

--workload prefill|dense|decode prints only that measurement (used by the
committed ncu profiling commands).

Multi-GPU: serial decode does not shard (replicas only): each rank runs its own
chain; value is the aggregate.
"""
from __future__ import annotations

import argparse
import csv
import importlib
import io
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "moe_decode_hbm_gbs"
UNIT = "GB/s"
L2_NOTE = "inputs larger than L2 (~660 MB of weights per step vs 126 MB L2)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=400)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--layers", type=int, default=39)
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--workload", choices=["all", "decode", "prefill", "dense"], default="all")
    p.add_argument("--prefill-steps", type=int, default=10)
    return p.parse_args()


def layer_bytes(cfg, k, T=1):
    """Algorithmic bytes of one config[1] layer: the k selected experts' packed
    codes + scales (gate, up, down) plus bf16 x in and y out."""
    return k * cfg.routed_bytes_per_expert() + 2 * T * cfg.hidden * 2


# ----------------------------------------------------------------------------- prefill / dense
def bench_prefill(torch, nv, lag, cfg, dev, steps, warmup, layers, distinct=4, T=512):
    """config[3] on one GPU: the full sparse block at T tokens, `layers` per step."""
    distinct = max(1, min(distinct, layers))
    blocks = [lag.random_sparse_layer(nv, seed=2000 + l, device=dev)[0] for l in range(distinct)]
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(T, cfg.hidden, generator=g, device=dev).to(torch.bfloat16)
    res = torch.randn(T, cfg.hidden, generator=g, device=dev).to(torch.bfloat16)
    y = torch.empty_like(x)

    def step():
        for l in range(layers):
            blocks[l % distinct](x, residual=res, out=y)

    def timed(exact):
        with nv.launch_flags(exact_prefill=exact):
            for _ in range(max(warmup, 3)):
                step()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                step()
            e1.record()
            torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    ms_step = timed(False)            # default: block-scaled FP4 GEMMs
    ms_exact = timed(True)            # exact 16-bit path, for comparison
    us_layer = ms_step * 1e3 / layers
    # Every expert is hit at T=512 (4096 random pairs over 256 experts).
    layer_w = (cfg.n_experts * cfg.routed_bytes_per_expert() + cfg.shared_bytes() +
               cfg.router_bytes())
    layer_b = layer_w + 3 * T * cfg.hidden * 2
    peak, peak_kind = measured_peak_hbm()
    return {"workload": f"BASELINE config[3] on 1 GPU: sparse block T={T} (router top-8, 256 "
                        f"experts, shared expert, residual), {layers} layers per step "
                        f"({distinct} distinct layers cycled)",
            "path": "block-scaled FP4 tensor cores (tcgen05 kind::mxf4nvf4), activations as "
                    "four NVFP4 terms",
            "tok_per_s": T / (ms_step / 1e3), "us_per_layer": us_layer,
            "hbm_gbs_equiv": layer_b / (us_layer / 1e6) / 1e9,
            "hbm_frac": layer_b / (us_layer / 1e6) / 1e9 / peak,
            "hbm_peak_gbs": peak, "hbm_peak_source": peak_kind,
            "us_per_layer_exact_path": ms_exact * 1e3 / layers,
            "tok_per_s_exact_path": T / (ms_exact / 1e3),
            "bytes_per_layer": layer_b, "steps": steps, "layers_per_step": layers,
            "unit": "tok/s"}


def bench_prefill_ep(torch, dist, nv, lag, cfg, dev, rank, world, steps, layers, distinct=2,
                     T=512, form="gather", partial_dtype=None, check=False):
    """config[3] expert-parallel: every rank holds E/world experts, the router
    and the shared expert, and runs the sparse block for its own T tokens; the
    (token, slot) rows cross to their experts' ranks and back by NCCL
    all-to-all.  Weak scaling: T tokens per rank.  Device time per step, max
    over ranks."""
    ep = importlib.import_module("mlxfast-challenge_b200.ep")
    blocks = []
    full0 = None  # rank 0 with check: the whole layer 0 on one GPU, the reference path
    for l in range(distinct):
        full, raw = lag.random_sparse_layer(nv, seed=3000 + l, device=dev)
        if check and rank == 0 and l == 0:
            full0 = full
        del full
        # this rank's expert slice as its own tensors, so the other experts
        # are freed (256/world experts resident per GPU)
        local = {k: v.clone() for k, v in ep.local_slice(raw["routed"], rank, world).items()}
        if form == "gather":
            ops = ep.CudaGatherEPOps(local, raw["shared"], raw["router_w"], raw["router_b"],
                                     cfg.n_experts, rank, world,
                                     partial_dtype=partial_dtype or torch.bfloat16)
            blk = ep.GatherEPBlock(ops)
        else:
            ops = ep.CudaEPOps(local, raw["shared"], raw["router_w"], raw["router_b"],
                               cfg.n_experts, rank, world)
            blk = ep.ExpertParallelBlock(ops)
        del raw
        torch.cuda.empty_cache()
        blocks.append(blk)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    x = torch.randn(T, cfg.hidden, generator=g, device=dev).to(torch.bfloat16)
    res = torch.randn(T, cfg.hidden, generator=g, device=dev).to(torch.bfloat16)
    checked = None
    if check:
        # every rank takes part; rank 0 compares its tokens' output with the
        # single-GPU block on the same tokens (same router, all 256 experts)
        y_ep = blocks[0](x, residual=res)
        if rank == 0:
            want = full0(x, residual=res)
            d = (y_ep.float() - want.float())
            checked = {"vs": "single-GPU SparseMoeBlock (all 256 experts) on rank 0's tokens",
                       "rel_l2": float(d.norm() / want.float().norm()),
                       "max_abs": float(d.abs().max()), "tolerance_rel_l2": 1e-2}
            checked["ok"] = bool(checked["rel_l2"] <= 1e-2)
        full0 = None
        torch.cuda.synchronize()
        torch.cuda.empty_cache()

    def step():
        for l in range(layers):
            blocks[l % distinct](x, residual=res)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item())
    exchange = ("NCCL all-gather of tokens + routing, per-rank partial sums over its "
                "experts, NCCL reduce-scatter" if form == "gather" else
                "NCCL all-to-all dispatch/combine")
    out = {"workload": f"BASELINE config[3] expert-parallel over {world} GPUs: sparse block "
                       f"T={T} tokens per GPU (router top-8, {cfg.n_experts // world} experts "
                       f"per GPU, shared expert, residual), {layers} layers per step, "
                       f"{exchange}", "n_gpus": world, "form": form,
           "tok_per_s": world * T / (ms_step / 1e3), "us_per_layer": ms_step * 1e3 / layers,
           "scaling": "weak", "unit": "tok/s", "steps": steps}
    if form == "gather":
        out["partials"] = str(partial_dtype or torch.bfloat16).replace("torch.", "")
    if checked is not None:
        out["check"] = checked
    return out


def blocked_scales(torch, s):
    """E4M3 group scales [rows, K/16] in the block-scaling layout cuBLASLt reads
    (tiles of 128 rows x 4 groups, rows interleaved in 4 x 32; the layout
    documented for cuBLAS block-scaled matmul), flattened."""
    r, c = s.shape
    rb, cb = (r + 127) // 128, (c + 3) // 4
    p = torch.zeros(rb * 128, cb * 4, dtype=s.dtype, device=s.device)
    p[:r, :c] = s
    return (p.view(rb, 128, cb, 4).permute(0, 2, 1, 3).reshape(-1, 4, 32, 4).transpose(1, 2)
            .reshape(-1, 32, 16).flatten())


def graph_us(torch, fn, reps=96, repeats=5):
    """Device us per call of fn(i), i = 0 .. reps-1 captured into one CUDA graph
    (the calls' own launches only; host work and allocation happen at capture)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(reps):
            fn(i)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(repeats):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / (repeats * reps)


def bench_dense(torch, nv, dev, copies=32):
    """config[0]: quantized_matmul [M, 2048] x [4096, 2048]^T for M = 512 and
    M = 1 (W4A16, the reference's op), and the same shapes through qqmm
    (activations fake-quantised to NVFP4 in the call, tcgen05 kind::mxf4nvf4);
    each timed as 96 calls in one CUDA graph cycling 32 weight copies (> L2).

    NVIDIA library bar (the reference's CUDA backend runs qqmm as cuBLASLt's
    NVFP4 block-scaled matmul, VMLX/backend/cuda/quantized/cublas_qqmm.cpp):
    torch._scaled_mm on the same NVFP4 operands (x quantized by this library,
    scales in cuBLASLt's block layout), its GEMM alone and with the
    quantization and re-layout of x in the call; outputs compared bit for bit
    with qqmm's.  Its throughput at 8192 x 8192 x 8192 is reported as the
    measured NVFP4 dense tensor peak of the chip."""
    N, K = 4096, 2048
    g = torch.Generator(device=dev).manual_seed(5)
    w = (torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    wq, sq = nv.quantize(w)
    wqs = [wq.clone() for _ in range(copies)]
    sqs = [sq.clone() for _ in range(copies)]
    fp4 = lambda q: q.view(torch.uint8).view(torch.float4_e2m1fn_x2)
    e4 = lambda q: q.view(torch.float8_e4m3fn)
    Bs = [fp4(q) for q in wqs]
    sbs = [blocked_scales(torch, e4(q)) for q in sqs]
    wbytes = N * K // 2 + N * K // 16
    out = {}

    def rec(name, M, us):
        out[name] = {"us": us, "tflops": 2 * M * N * K / (us / 1e6) / 1e12,
                     "hbm_gbs": (wbytes + M * K * 2 + M * N * 2) / (us / 1e6) / 1e9}

    for M in (512, 1):
        x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
        rec(f"M{M}", M, graph_us(torch, lambda i: nv.quantized_matmul(x, wqs[i % copies],
                                                                      sqs[i % copies])))
        rec(f"qqmm_M{M}", M, graph_us(torch, lambda i: nv.qqmm(x, wqs[i % copies],
                                                               sqs[i % copies])))
        xq, xs = nv.quantize_activations(x)
        A, sa = fp4(xq), blocked_scales(torch, e4(xs))
        try:
            yc = torch._scaled_mm(A, Bs[0].t(), sa, sbs[0], out_dtype=torch.bfloat16)
        except Exception as exc:  # no cuBLASLt NVFP4 on this build
            out[f"cublaslt_nvfp4_M{M}"] = {"unavailable": repr(exc)[:200]}
            continue
        same = bool(torch.equal(yc, nv.qqmm(x, wqs[0], sqs[0])))
        rec(f"cublaslt_nvfp4_M{M}", M, graph_us(torch, lambda i: torch._scaled_mm(
            A, Bs[i % copies].t(), sa, sbs[i % copies], out_dtype=torch.bfloat16)))
        out[f"cublaslt_nvfp4_M{M}"]["bitwise_equal_to_qqmm"] = same

        def cub_q(i):
            q2, s2 = nv.quantize_activations(x)
            return torch._scaled_mm(fp4(q2), Bs[i % copies].t(), blocked_scales(torch, e4(s2)),
                                    sbs[i % copies], out_dtype=torch.bfloat16)
        rec(f"cublaslt_nvfp4_with_quant_M{M}", M, graph_us(torch, cub_q))
    try:
        P = 8192
        a = fp4(torch.randint(0, 256, (P, P // 2), dtype=torch.uint8, device=dev))
        b = fp4(torch.randint(0, 256, (P, P // 2), dtype=torch.uint8, device=dev))
        sc = blocked_scales(torch, torch.full((P, P // 16), 0x38, dtype=torch.uint8,
                                              device=dev).view(torch.float8_e4m3fn))
        us = graph_us(torch, lambda i: torch._scaled_mm(a, b.t(), sc, sc,
                                                        out_dtype=torch.bfloat16), reps=20)
        out["nvfp4_peak_measured"] = {"tflops": 2 * P ** 3 / (us / 1e6) / 1e12, "us": us,
                                      "how": "cuBLASLt NVFP4 block-scaled matmul "
                                             "(torch._scaled_mm) 8192^3, CUDA graph"}
        del a, b, sc
    except Exception as exc:
        out["nvfp4_peak_measured"] = {"unavailable": repr(exc)[:200]}
    out["workload"] = ("BASELINE config[0]: x bf16 [M, 2048] @ nvfp4 W[4096, 2048]^T, "
                       f"{copies} weight copies cycled (> L2), 96 calls per CUDA graph; qqmm_* = "
                       "the same through qqmm (x fake-quantised to NVFP4 in the call, tcgen05 "
                       "kind::mxf4nvf4); cublaslt_nvfp4_* = cuBLASLt's NVFP4 matmul on the "
                       "same operands (the reference CUDA backend's qqmm)")
    return out


# ----------------------------------------------------------------------------- CPU
class _CpuLayer:
    """One config[2] sparse layer (one sequence) for the CPU arms: 8 routed
    experts and the shared expert as packed NVFP4 banks quantized from bf16
    N(0, 0.02) by the reference's quantizer (the CPU restatement, bit-identical
    to it), a bf16 router and norm weight; x bf16 N(0, 1)."""

    def __init__(self, cfg, seed=0):
        import numpy as np
        import oracle
        self.np, self.orc = np, oracle
        rng = np.random.default_rng(seed)
        H, I, k = cfg.hidden, cfg.inter, cfg.top_k
        bits = lambda *shape: oracle.bf16_bits_from_f32(
            (rng.standard_normal(shape) * 0.02).astype(np.float32))
        q = lambda *shape: oracle.port.quantize(bits(*shape))
        self.experts = [(q(I, H), q(I, H), q(H, I)) for _ in range(k + 1)]  # k routed + shared
        self.G = bits(cfg.n_experts, H)
        self.bias = (rng.standard_normal(cfg.n_experts) * 1e-3).astype(np.float32)
        self.norm_w = oracle.bf16_bits_from_f32(
            (1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
        self.h = oracle.bf16_bits_from_f32(rng.standard_normal((1, H)).astype(np.float32))
        self.k = k
        self.bytes = (cfg.router_bytes() + cfg.shared_bytes() + k * cfg.routed_bytes_per_expert()
                      + 2 * H * 2 + H * 2)

    def run(self, impl, kind, threads):
        """The layer as MLX evaluates it for bf16 on the CPU: norm, router,
        then each expert's gate / up / down through fp_qmm_t<bfloat16_t> (the
        reference's own kernel when kind == "reference"), SwiGLU and the
        weighted sum in bf16 steps, plus the residual."""
        np, orc = self.np, self.orc
        x = orc.port.rms_norm_bf16(self.h, self.norm_w, 1e-6)
        _, w, _ = orc.port.router_topk(x, self.G, self.bias, self.k)
        if kind == "reference":
            mm = lambda a, wq: impl.qmm_bf16(a, wq[0], wq[1], threads=threads)
        else:
            mm = lambda a, wq: orc.bf16_bits_from_f32(
                impl.qmm_f32(orc.f32_from_bf16_bits(a), wq[0], wq[1]))
        acc = np.zeros(self.h.shape[-1], np.float32)
        for j, (g, u, d) in enumerate(self.experts):
            gf = orc.f32_from_bf16_bits(mm(x, g))
            uf = orc.f32_from_bf16_bits(mm(x, u))
            a = orc.bf16_bits_from_f32(gf / (1 + np.exp(-gf)) * uf)
            y = orc.f32_from_bf16_bits(mm(a, d))[0]
            acc += (2.5 * w[0][j] if j < self.k else 1.0) * y
        return acc + orc.f32_from_bf16_bits(self.h)[0]


def cpu_reference_gbs(seconds, threads, cfg, steps=None, warmup=0, layer=None):
    """The reference's MLX CPU kernel (oracle/_ref) on one config[2] layer per step."""
    import oracle
    impl = oracle.ref if oracle.ref is not None else oracle.port
    kind = "reference" if oracle.ref is not None else "port"
    layer = layer or _CpuLayer(cfg)
    for _ in range(warmup):
        layer.run(impl, kind, threads)
    t0 = time.perf_counter()
    n = 0
    while True:
        layer.run(impl, kind, threads)
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and el >= seconds):
            break
    what = ("the reference fp_qmm_t<bfloat16_t,16,4>" if kind == "reference"
            else "the CPU restatement of fp_qmm_t")
    return dict(value=layer.bytes * n / el / 1e9, unit=UNIT, cores=threads, kind=kind,
                sample=f"{n} config[2] layers (norm, router, 8 routed experts + shared expert "
                       f"x gate/up/down, T=1), bf16 x through {what} split over {threads} "
                       f"thread(s); {el:.2f} s"), n, el


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.proc = None
        self.gpu_index = gpu_index

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = [r for r in csv.reader(io.StringIO(out)) if len(r) >= 9]
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(rows)}


def measured_peak_hbm():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def stack_traffic(layers, kind="routed", launches=1):
    """DRAM bytes per launch of a decode stack over `layers` layers in
    `launches` launches (kind: "routed", "fp4" given routing, or "exact", the
    mma.sync stack), scaled from the committed ncu capture (taken on fewer
    layers; the kernel moves the same bytes per layer)."""
    name = {"routed": "moe_decode_stack_routed_traffic.json",
            "fp4": "moe_decode_stack_fp4_traffic.json",
            "exact": "moe_decode_stack_traffic.json"}[kind]
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            d = json.load(f)
        if d.get("dram_bytes_per_layer") is None:
            return None
        return d["dram_bytes_per_layer"] * layers / launches
    except Exception:
        return None


# ----------------------------------------------------------------------------- decode
def time_replays(torch, chain, steps):
    """Device ms per step over `steps` replays of the chain's graph (CUDA events
    on its stream)."""
    s = chain.stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(steps):
            chain.graph.replay()
        e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def distinct_experts(chain):
    """Distinct routed experts per layer of the chain's last step."""
    return [int(len(set(r[0].view(torch_int32()).flatten().tolist()))) for r in chain.routing]


def torch_int32():
    import torch
    return torch.int32


def step_bytes(cfg, U, T):
    """Algorithmic bytes of one step: per layer the router, the shared expert,
    the distinct routed experts U[l] (packed codes + scales of gate, up and
    down), the norm weight, and the activations in (h) and out (h_next)."""
    per_act = 2 * T * cfg.hidden * 2
    return sum(cfg.router_bytes() + cfg.shared_bytes() + u * cfg.routed_bytes_per_expert() +
               cfg.hidden * 2 + per_act for u in U)


def bench_given_routing(torch, nv, lag, cfg, dev, made, steps, warmup):
    """config[1]: the routed experts only (no shared expert, no router), the
    routing of all layers given before the step (k distinct uniform experts,
    softmax(N(0,1)) weights), 39 layers chained through the persistent stack."""
    blocks = [nv.SparseMoeBlock(m[1]["routed"], None, top_k=cfg.top_k,
                                routed_scaling=cfg.routed_scaling) for m in made]
    routing = [lag.random_routing(1, cfg, seed=5000 + l, device=dev) for l in range(len(made))]
    chain = nv.MoEDecodeChain(blocks, routing, T=1, device=dev).capture()
    chain.x0.copy_(torch.randn(1, cfg.hidden, device=dev).to(torch.bfloat16))
    for _ in range(max(warmup, 3)):
        chain.replay()
    torch.cuda.synchronize()
    ms = time_replays(torch, chain, steps)
    b = len(made) * layer_bytes(cfg, cfg.top_k)
    out = {"workload": "BASELINE config[1]: routed experts only, routing given for all "
                       f"{len(made)} layers before the step (the stack streams later layers' "
                       "experts ahead)",
           "value": b / (ms / 1e3) / 1e9, "unit": UNIT, "us_per_layer": ms * 1e3 / len(made),
           "kernel": "moe_decode_stack_fp4_kernel (given routing)" if chain.stack_fp4
           else "moe_decode_stack_kernel (mma.sync)", "bytes_per_step": b}
    del chain
    return out


def bench_decode_b8(torch, nv, cfg, dev, blocks, norms, steps, warmup, T=8):
    """config[2] at T sequences: per layer RMSNorm, router, fused gate/up +
    SwiGLU and down + combine + residual (the per-layer kernels in one CUDA
    graph); bytes from the distinct experts the router chose."""
    chain = nv.MoEDecodeChain(blocks, None, T=T, route=True, residual=True, norms=norms,
                              device=dev, stack=False).capture()
    chain.x0.copy_(torch.randn(T, cfg.hidden, device=dev).to(torch.bfloat16))
    for _ in range(max(warmup, 3)):
        chain.replay()
    torch.cuda.synchronize()
    ms = time_replays(torch, chain, steps)
    U = distinct_experts(chain)
    b = step_bytes(cfg, U, T)
    out = {"workload": f"BASELINE config[2] at {T} sequences: the same layers, T={T}, per-layer "
                       "kernels (rms_norm, router, gate/up + SwiGLU, down + combine + residual)",
           "value": b / (ms / 1e3) / 1e9, "unit": UNIT, "us_per_layer": ms * 1e3 / len(blocks),
           "tok_per_s_moe_only": T * 1e3 / ms, "mean_distinct_experts": sum(U) / len(U),
           "bytes_per_step": b, "launches_per_step": chain.launches_per_step()}
    del chain
    return out


# ----------------------------------------------------------------------------- main
def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    lag = importlib.import_module("mlxfast-challenge_b200.laguna")
    cfg = lag.LAGUNA_XS_2_1

    if args.impl == "reference":
        if rank != 0:
            return
        threads = os.cpu_count() or 1
        cb, n, el = cpu_reference_gbs(None, threads, cfg, steps=args.steps, warmup=args.warmup)
        line = {"metric": METRIC, "value": cb["value"], "unit": UNIT, "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / n * 1e3,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "BASELINE config[2] at one sequence: Laguna sparse "
                                       "block at decode T=1 (RMSNorm, router top-8, 8 of 256 "
                                       "routed experts, shared expert, residual), H=2048 "
                                       "I=512, one layer per step",
                           "l2": "CPU"},
                "impl": "reference", "cpu_baseline": cb,
                "e2e": {"value": cb["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    nv = importlib.import_module("mlxfast-challenge_b200")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    if args.workload in ("prefill", "dense"):
        if rank == 0:
            if args.workload == "prefill":
                r = bench_prefill(torch, nv, lag, cfg, dev, args.steps, args.warmup, args.layers)
            else:
                r = bench_dense(torch, nv, dev)
            print(json.dumps({"workload": args.workload, "result": r}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return

    # Setup: L random-init sparse layers (config[2]: router, routed experts,
    # shared expert, the decoder layer's norm weight).
    made = [lag.random_sparse_layer(nv, seed=1000 + l, device=dev) for l in range(args.layers)]
    blocks = [m[0] for m in made]
    norms = [m[1]["norm_w"] for m in made]
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    x0 = torch.randn(1, cfg.hidden, generator=g, device=dev).to(torch.bfloat16)
    chain = nv.MoEDecodeChain(blocks, None, T=1, route=True, residual=True, norms=norms,
                              device=dev).capture()
    chain.x0.copy_(x0)
    s = chain.stream

    # Warm-up, then K timed replays bracketed by barrier + synchronize.
    for _ in range(max(args.warmup, 3)):
        chain.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    gpu_index = int(vis.split(",")[local]) if vis else local
    sampler = ClockSampler(gpu_index)
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    ms = time_replays(torch, chain, args.steps)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = sampler.stop() if rank == 0 else None
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    # The step's algorithmic bytes from the routing it used (the same every
    # replay: the input and the weights do not change).
    U = distinct_experts(chain)
    bytes_step = step_bytes(cfg, U, T=1)
    value = world * bytes_step / (ms_max / 1e3) / 1e9

    # Dominant kernel alone: the routed stack is the whole step (its launches,
    # with their counter resets).
    import ctypes
    peak, peak_kind = measured_peak_hbm()
    peak_src = (f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6650 GB/s")
    reps = max(20, args.steps // 4)
    with torch.cuda.stream(s):
        sp = ctypes.c_void_p(s.cuda_stream)
        for _ in range(3):
            nv._lib.check(chain._stack_call(sp))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(reps):
            nv._lib.check(chain._stack_call(sp))
        e1.record(s)
    torch.cuda.synchronize()
    k_ms = e0.elapsed_time(e1) / reps
    achieved = bytes_step / (k_ms / 1e3) / 1e9
    tr = stack_traffic(args.layers, "routed", chain.launches_per_step())
    roofline = {"bound": "hbm",
                "kernel": f"moe_decode_stack_fp4_kernel, routed form (tcgen05 kind::mxf4nvf4; "
                          f"norm, router, experts, residual on the device), {args.layers} layers, "
                          f"{chain.launches_per_step()} persistent launches",
                "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "peak_source": peak_src, "traffic": tr,
                "traffic_note": (None if tr is not None else
                                 "ncu cannot launch this cooperative cluster kernel "
                                 "(profiles/moe_decode_stack_routed_traffic.json)"),
                "algorithmic_bytes_per_launch": bytes_step / chain.launches_per_step(),
                "algorithmic_bytes_per_step": bytes_step, "us_per_step": k_ms * 1e3,
                "us_per_layer": k_ms * 1e3 / args.layers}

    # End to end through the public API: pinned host x in, host y out, every step.
    xh = x0.cpu().pin_memory()
    yh = torch.empty(1, cfg.hidden, dtype=torch.bfloat16).pin_memory()
    for _ in range(3):
        chain(xh, yh)
    if world > 1:
        dist.barrier()
    e2e_steps = max(10, args.steps // 2)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        chain(xh, yh)
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_val = world * e2e_steps * bytes_step / float(te.item()) / 1e9
    launches = args.steps * chain.launches_per_step()
    del chain

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        layer = _CpuLayer(cfg)
        cpu, _, _ = cpu_reference_gbs(args.cpu_seconds, threads, cfg, layer=layer)
        one, _, _ = cpu_reference_gbs(max(2.0, args.cpu_seconds / 3), 1, cfg, layer=layer)
        cpu["one_thread"] = {"value": one["value"], "unit": UNIT, "cores": 1,
                             "sample": one["sample"],
                             "note": "MLX runs its CPU stream on one thread"}
    given = b8 = prefill = dense = prefill_ep = None
    if world > 1 and args.workload == "all":
        # every rank takes part (the exchange is collective)
        prefill_ep = bench_prefill_ep(torch, dist, nv, lag, cfg, dev, rank, world,
                                      args.prefill_steps, cfg.num_sparse_layers, form="gather",
                                      partial_dtype=torch.bfloat16, check=True)
        f32 = bench_prefill_ep(torch, dist, nv, lag, cfg, dev, rank, world, args.prefill_steps,
                               cfg.num_sparse_layers, form="gather",
                               partial_dtype=torch.float32)
        prefill_ep["f32_partials"] = {"tok_per_s": f32["tok_per_s"],
                                      "us_per_layer": f32["us_per_layer"]}
        a2a = bench_prefill_ep(torch, dist, nv, lag, cfg, dev, rank, world, args.prefill_steps,
                               cfg.num_sparse_layers, form="all2all")
        prefill_ep["all2all_form"] = {"tok_per_s": a2a["tok_per_s"],
                                      "us_per_layer": a2a["us_per_layer"]}
    if rank == 0 and world == 1 and args.workload == "all":
        given = bench_given_routing(torch, nv, lag, cfg, dev, made, args.steps, args.warmup)
        b8 = bench_decode_b8(torch, nv, cfg, dev, blocks, norms, max(10, args.steps // 4),
                             args.warmup)
        del made, blocks, norms
        torch.cuda.empty_cache()
        prefill = bench_prefill(torch, nv, lag, cfg, dev, args.prefill_steps, 3,
                                cfg.num_sparse_layers)
        dense = bench_dense(torch, nv, dev)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE config[2] at one sequence: Laguna sparse block at "
                                   "decode T=1 (RMSNorm, BF16 router top-8 on the device, 256 "
                                   "NVFP4 g16 routed experts, NVFP4 shared expert, residual), "
                                   "H=2048, I=512, x 39 sparse layers per step, each layer's "
                                   "input the previous layer's output",
                       "layers_per_step": args.layers, "bytes_per_step": bytes_step,
                       "distinct_experts_per_layer": U,
                       "l2": L2_NOTE, "parallelism": f"replicas{world}",
                       "weights": "nvfp4 e2m1/e4m3-g16 (router, norm: bf16)",
                       "activations": "bf16", "accumulate": "f32"},
            "tok_per_s_moe_only": world * 1e3 / ms_max,
            "us_per_layer": ms_max * 1e3 / args.layers,
            "gpu_launches": launches,
            "clocks": clocks,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": cfg.hidden * 2,
                    "d2h_bytes_per_step": cfg.hidden * 2,
                    "api": "MoEDecodeChain.__call__ (pinned host x -> device -> host y)"},
            "decode_given_routing": given,
            "decode_b8": b8,
            "prefill": prefill,
            "prefill_ep": prefill_ep,
            "dense": dense,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
