"""Benchmark of the MoE block hot path (BASELINE metric: "MoE block us/token @decode M=1 (% HBM peak)").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (BASELINE configs[1] at M=1, run as configs[4](a) runs it): a synthetic 16-layer stack of the bf16
Ling-style MoE block (H=2048, 64 routed experts of I=1408 + a 2816-wide shared expert as two I-wide slots,
softmax top-6 router, RMSNorm eps 1e-6, residual), random-init N(0, 0.02) weights generated on the device,
one decode token. A "step" is one token through all 16 blocks, captured once in a CUDA graph and replayed:
each block is ONE kernel (mv_block_decode). Weights touched per step (16 x ~139 MB) exceed the 126 MB L2,
so no flush is needed between steps. value = device time per step / (16 blocks x N ranks), i.e. the
whole-job time per block-token (lower is better; N > 1 runs independent replicas: decode does not shard).

Keys beyond the base contract: roofline (HBM, measured copy peak), cpu_baseline (the oracle's torch-eager
fp32 block on the host cores), e2e (the same metric through the public MoeBlock.decode API with the token
copied host->device and the result device->host every step), gpu_launches, clocks (sampled from the first timed
region to the end of the last); decode_sweep (M = 1, 2, 4, 8, 16 through the same graph
chain, us/token and HBM fraction); int8_decode (configs[2] at M = 1, 4, 16, with its HBM roofline); prefill
(configs[3]: the 2043-token ragged pass in a CUDA graph on one GPU, expert parallel over N > 1 ranks, weak
scaling) with its tensor roofline; stack_prefill (configs[4](b): 8192 tokens through the 16 layers, strong
scaling over N ranks); reference_kernels (why the reference's Triton kernels are not timed here). --decode-m M
measures the headline at another token count, --prefill-only the prefill pass alone; --no-prefill / --no-int8 /
--no-sweep / --no-stack skip those parts. --impl reference times the reference's CPU path (the oracle's fp32
restatement) on the same 16-layer decode workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "ming-voice_b200"))

import torch  # noqa: E402

METRIC = "MoE block us/token @decode M=1 (% HBM peak); prefill tokens/s @1/2/4/8 GPU"
UNIT = "us/token"
LAYERS = 16
H, I, E, TOPK, IS = 2048, 1408, 64, 6, 2816
EP_REPLICATED = 8  # experts replicated on every rank in the expert-parallel prefill (the Zipf-hot head)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def peaks_tensor():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured (burst)"
    except Exception:
        return 1590.0, "fallback"


def ncu_traffic():
    """dram read+write bytes per launch of the decode kernel (the one-token kernel at M=1) from the committed ncu
    summary (or None)."""
    import re
    path = os.path.join(ROOT, "profiles", "decode_m1_kernel_block_m1.md")
    try:
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.e+]+)", open(path).read())
        return float(m.group(1)) if m else None
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""

    def __init__(self, index):
        self.index, self.samples, self.proc = index, [], None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 6:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[2 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def make_stack(device, layers, seed=3, int8=False):
    """16 blocks of random N(0, 0.02) weights, generated on the device (seeded). int8: every expert, shared and
    router weight quantised per output row (symmetric, scale max|w|/127 stored bf16)."""
    from mingmoe.block import MoeBlock
    import fused_moe
    g = torch.Generator(device=device).manual_seed(seed)
    blocks = []
    for _ in range(layers):
        E1 = E + IS // I
        w_gu = (torch.randn(E1, 2 * I, H, generator=g, device=device) * 0.02).to(torch.bfloat16)
        w_d = (torch.randn(E1, H, I, generator=g, device=device) * 0.02).to(torch.bfloat16)
        rw = (torch.randn(E, H, generator=g, device=device) * 0.02).to(torch.bfloat16)
        nw = torch.ones(H, dtype=torch.bfloat16, device=device)
        if int8:
            q_gu, s_gu = fused_moe.quantize_rows_int8(w_gu, scale_dtype=torch.bfloat16)
            q_d, s_d = fused_moe.quantize_rows_int8(w_d, scale_dtype=torch.bfloat16)
            q_rw, s_rw = fused_moe.quantize_rows_int8(rw, scale_dtype=torch.bfloat16)
            del w_gu, w_d, rw
            blocks.append(MoeBlock(q_gu, q_d, q_rw, nw, top_k=TOPK, shared_ids=tuple(range(E, E1)), eps=1e-6,
                                   s_gu=s_gu, s_d=s_d, router_s=s_rw))
        else:
            blocks.append(MoeBlock(w_gu, w_d, rw, nw, top_k=TOPK, shared_ids=tuple(range(E, E1)), eps=1e-6))
    for layer, blk in enumerate(blocks):  # block l prefetches the routing weights of block l + 1 (a step repeats)
        blk.link(blocks[(layer + 1) % len(blocks)])
    return blocks


def chain_us_per_block(blocks, dev, Md, steps, warmup, ids=None):
    """Device time per block of an Md-token step through the stack, one CUDA graph per step (Md tokens, seeded),
    and the number of distinct routed experts of the first block's step."""
    from oracle import moe_oracle as O
    layers = len(blocks)
    bufs = [torch.empty(Md, H, dtype=torch.bfloat16, device=dev) for _ in range(layers + 1)]
    bufs[0].copy_(O.make_tokens(Md, seed=3).to(dev))
    ids = torch.empty(Md, TOPK + 2, dtype=torch.int32, device=dev)

    def step():
        for layer, blk in enumerate(blocks):
            blk.decode(bufs[layer], out=bufs[layer + 1], ids=ids if layer == 0 else None)

    step()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        step()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
    torch.cuda.current_stream(dev).wait_stream(stream)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(True), torch.cuda.Event(True)
    s_ev.record()
    for _ in range(steps):
        graph.replay()
    e_ev.record()
    torch.cuda.synchronize()
    us = s_ev.elapsed_time(e_ev) / steps * 1e3 / layers
    U = O.distinct_experts(ids.cpu()[:, :TOPK])
    del graph
    return us, U


def decode_sweep_lines(blocks, dev, steps, warmup, ms=(1, 2, 4, 8, 16)):
    """decode at M in {1, 2, 4, 8, 16} tokens through the same 16-layer graph chain: us per
    token and the HBM roofline of the weights touched (U distinct routed experts + the shared expert + router)."""
    from oracle import moe_oracle as O
    peak, _ = peaks()
    out = []
    for Md in ms:
        us, U = chain_us_per_block(blocks, dev, Md, steps, warmup)
        byts = O.decode_bytes(U, M=Md)
        gbs = byts / (us * 1e-6) / 1e9
        out.append({"M": Md, "us_per_token": round(us / Md, 3), "us_per_block": round(us, 2), "routed_experts_hit": U,
                    "bytes_per_block": byts, "hbm_gbs": round(gbs, 1), "hbm_frac": round(gbs / peak, 4)})
    return out


def int8_decode_lines(dev, steps, warmup, layers=16, ms=(1, 4, 16)):
    """BASELINE configs[2] (int8 weights, bf16 scales) at decode M in {1, 4, 16}, through the same 16-layer graph chain
    as the headline: us per token and the HBM roofline (int8 bytes + bf16 scales)."""
    from oracle import moe_oracle as O
    blocks = make_stack(dev, layers, seed=4, int8=True)
    peak, _ = peaks()
    rows = []
    for Md in ms:
        us, U = chain_us_per_block(blocks, dev, Md, steps, warmup)
        byts = O.decode_bytes(U, M=Md, esz=1, scale_bytes=2)
        achieved = byts / (us * 1e-6) / 1e9
        rows.append({"M": Md, "us_per_token": round(us / Md, 3), "us_per_block": round(us, 2),
                     "routed_experts_hit": U, "bytes_per_block": byts,
                     "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                                  "frac": round(achieved / peak, 4)}})
    del blocks
    torch.cuda.empty_cache()
    m1 = rows[0]
    return {"metric": "int8 decode us/token (BASELINE configs[2], 16-layer graph chain)", "value": m1["us_per_token"],
            "unit": "us/token", "bytes_per_block": m1["bytes_per_block"], "roofline": m1["roofline"], "sweep": rows}


def cpu_block_time_us(reps=5):
    """The oracle's torch-eager fp32 block on the host cores: us per block-token at M=1."""
    from oracle import moe_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    p = O.make_block_params(seed=3, dtype=torch.float32)
    x = O.make_tokens(1, seed=3, dtype=torch.float32)
    O.moe_block(x, p)  # warm-up
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        O.moe_block(x, p)
        ts.append((time.perf_counter() - t0) * 1e6)
    return statistics.median(ts), torch.get_num_threads(), f"1 token through 1 fp32 block, median of {reps}"


def dist_setup(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    return rank, world, local


def run_reference(args):
    rank, world, _ = dist_setup(args.gpus) if int(os.environ.get("WORLD_SIZE", "1")) > 1 else (0, 1, 0)
    if rank != 0:
        return
    # the reference's CPU torch-eager path (restated in oracle/), all host threads: the headline workload, one token
    # through a 16-layer chain of fp32 blocks per step (the blocks share one set of weights: CPU time does not
    # depend on their values, and 16 distinct fp32 blocks would hold 37 GB of host memory)
    from oracle import moe_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    p = O.make_block_params(seed=3, dtype=torch.float32)
    x0 = O.make_tokens(1, seed=3, dtype=torch.float32)

    def step():
        h = x0
        for _ in range(args.layers):
            h = O.moe_block(h, p)[0]
        return h

    for _ in range(args.warmup):
        step()
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        ts.append((time.perf_counter() - t0) * 1e6 / args.layers)
    v = sum(ts) / len(ts)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 2), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(v * args.layers / 1e3, 4),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"decode M=1 through a {args.layers}-layer chain of MoE blocks (BASELINE configs[1] "
                               "at M=1, run as configs[4](a)); CPU torch-eager reference path, fp32",
                   "tokens_per_step": 1, "layers": args.layers, "H": H, "I": I, "E": E, "top_k": TOPK,
                   "shared_I": IS},
        "cpu_baseline": {"value": round(v, 2), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"1 token through {args.layers} fp32 blocks per step, us per block-token"},
        "e2e": {"value": round(v, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def prefill_lines(dev, steps, warmup):
    """BASELINE C4 on one block: 2043 packed tokens (37/211/512/1283), Zipf router bias, seed 2; one CUDA
    graph per pass (RMSNorm, router, expert sort, gather, two tcgen05 grouped GEMMs, finalize)."""
    from mingmoe.block import MoeBlock
    from oracle import moe_oracle as O
    p = O.make_block_params(seed=2, dtype=torch.bfloat16)
    blk = MoeBlock.from_params(p, device=dev, router_bias=O.zipf_bias(E))
    del p
    N = sum(O.PREFILL_LENS)
    x = O.make_tokens(N, seed=2).to(dev)
    out = {}
    blk.prefill(x)  # workspaces exist before capture
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        blk.prefill(x)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            y = blk.prefill(x)
    torch.cuda.current_stream(dev).wait_stream(stream)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(True), torch.cuda.Event(True)
    s_ev.record()
    for _ in range(steps):
        graph.replay()
    e_ev.record()
    torch.cuda.synchronize()
    us = s_ev.elapsed_time(e_ev) / steps * 1e3
    # end to end through MoeBlock.prefill: pinned host tokens in, result out, every pass
    h_in = x.cpu().pin_memory()
    h_out = torch.empty_like(h_in).pin_memory()
    for _ in range(warmup):
        h_out.copy_(blk.prefill(h_in.to(dev, non_blocking=True)), non_blocking=True)
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(True), torch.cuda.Event(True)
    s2.record()
    for _ in range(steps):
        h_out.copy_(blk.prefill(h_in.to(dev, non_blocking=True)), non_blocking=True)
    e2.record()
    torch.cuda.synchronize()
    us_e2e = s2.elapsed_time(e2) / steps * 1e3
    flops = O.prefill_flops(N)
    del graph, y
    return {"tokens": N, "us_per_pass": round(us, 1), "tokens_per_s": round(N / us * 1e6, 0),
            "tflops": round(flops / us / 1e6, 1), "e2e_tokens_per_s": round(N / us_e2e * 1e6, 0),
            "launches_per_pass": 9, "flops_per_pass": flops}


def ep_prefill_lines(dev, world, rank, steps, warmup):
    """BASELINE C4 with expert parallelism over `world` ranks (NCCL): every rank prefills its own 2043 packed
    tokens (seed 2 + rank), owns E / world routed experts and keeps the router, norm and shared expert; one
    all-to-all exchange each way. Weak scaling: tokens/s of the whole job = world * 2043 / max time."""
    from mingmoe.block import MoeBlock
    from mingmoe.ep import EPMoeBlock
    from oracle import moe_oracle as O
    g = torch.Generator(device=dev).manual_seed(2)  # the same weights on every rank
    E1 = E + IS // I
    w_gu = (torch.randn(E1, 2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w_d = (torch.randn(E1, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    rw = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    from mingmoe.ep import placement
    replicated = tuple(range(EP_REPLICATED))  # the Zipf-hot experts (lowest ids) on every rank
    stacks = placement(E, world, replicated)[2]
    n_loc = len(stacks[rank])
    sel = torch.tensor(stacks[rank] + list(range(E, E1)), device=dev)
    blk = MoeBlock(w_gu.index_select(0, sel).contiguous(), w_d.index_select(0, sel).contiguous(), rw,
                   torch.ones(H, dtype=torch.bfloat16, device=dev), top_k=TOPK,
                   shared_ids=tuple(range(n_loc, n_loc + E1 - E)), eps=1e-6, router_bias=O.zipf_bias(E).to(dev))
    del w_gu, w_d
    ep = EPMoeBlock(blk, E, replicated=replicated)
    N = sum(O.PREFILL_LENS)
    x = O.make_tokens(N, seed=2 + rank).to(dev)
    cap = ep.calibrate(x)  # the exchange capacity per peer, from this batch (before the timed region)
    for _ in range(warmup):
        ep.forward(x)
    torch.cuda.synchronize()
    # the step has no host synchronisation, so it is captured whole (NCCL all-to-alls included) in one CUDA graph,
    # as the single-GPU pass is; every rank captures and replays the same collectives in the same order
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        ep.forward(x)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            ep.forward(x)
    torch.cuda.current_stream(dev).wait_stream(stream)
    for _ in range(warmup):
        graph.replay()
    torch.distributed.barrier()
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(True), torch.cuda.Event(True)
    s_ev.record()
    for _ in range(steps):
        graph.replay()
    e_ev.record()
    torch.cuda.synchronize()
    t = torch.tensor([s_ev.elapsed_time(e_ev) / steps], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    us = t.item() * 1e3
    torch.distributed.barrier()
    del graph  # a graph holding NCCL calls is released before the process group
    errs = ep.errors()
    if errs:
        raise RuntimeError(f"EP prefill device errors: {errs}")
    # per-phase device times (graph replays, event nodes at the phase boundaries), max over ranks
    ph = torch.tensor(ep.phase_times(x), dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(ph, op=torch.distributed.ReduceOp.MAX)
    phases = {n: round(v, 1) for n, v in zip(ep.PHASES, ph.tolist())}
    flops = O.prefill_flops(N) * world
    return {"tokens_per_gpu": N, "us_per_pass": round(us, 1), "tokens_per_s": round(world * N / us * 1e6, 0),
            "tflops": round(flops / us / 1e6, 1),
            "parallelism": f"ep{world}: experts 0-{EP_REPLICATED - 1} replicated, {E - EP_REPLICATED} dealt as a snake",
            "exchange": f"NCCL all-to-all of fixed capacity {cap} pairs per peer: bf16 rows out, bf16 outputs back "
                        "(device-side plan / pack / combine, no host synchronisation; the step replayed as one CUDA "
                        "graph)", "flops_per_pass": flops,
            "phases_us": {**phases, "note": "graph replays with event nodes at the phase boundaries, each phase's max "
                                            "over ranks (an exchange phase includes waiting for the slowest peer)"}}


def stack_prefill_lines(dev, world, rank, steps, warmup, blocks=None, layers=LAYERS, tokens=8192):
    """BASELINE configs[4](b): 8 packed sequences of 1024 tokens (8192) through the 16-layer stack, one step = the
    whole prefill. One GPU: MoeBlock.prefill per layer (norm, router, expert sort, grouped GEMMs, finalize) on the
    decode stack's blocks. N ranks: expert parallel, strong scaling (8192 / N tokens per rank; every rank holds
    the router, norm, shared expert and experts 0-7 of each layer and its share of the others, dealt as a snake).
    The step is replayed as one CUDA graph."""
    from oracle import moe_oracle as O
    per_rank = tokens // world
    x = O.make_tokens(per_rank, seed=30 + rank).to(dev)
    if world == 1:
        fwd_blocks = blocks

        def step():
            h = x
            for blk in fwd_blocks:
                h = blk.prefill(h)
            return h
    else:
        from mingmoe.block import MoeBlock
        from mingmoe.ep import EPMoeBlock, placement
        replicated = tuple(range(EP_REPLICATED))
        stacks = placement(E, world, replicated)[2]
        n_loc = len(stacks[rank])
        E1 = E + IS // I
        sel = torch.tensor(stacks[rank] + list(range(E, E1)), device=dev)
        g = torch.Generator(device=dev).manual_seed(3)  # the same weights on every rank
        eps_blocks = []
        for _ in range(layers):
            w_gu = (torch.randn(E1, 2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            w_d = (torch.randn(E1, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            rw = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            blk = MoeBlock(w_gu.index_select(0, sel).contiguous(), w_d.index_select(0, sel).contiguous(), rw,
                           torch.ones(H, dtype=torch.bfloat16, device=dev), top_k=TOPK,
                           shared_ids=tuple(range(n_loc, n_loc + E1 - E)), eps=1e-6)
            del w_gu, w_d
            eps_blocks.append(EPMoeBlock(blk, E, replicated=replicated))
        h = x
        for ep in eps_blocks:  # the exchange capacity of each layer, from this batch (before the timed region)
            ep.calibrate(h)
            h = ep.forward(h).clone()

        def step():
            h = x
            for ep in eps_blocks:
                h = ep.forward(h)
            return h
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    # the whole 16-layer step (with EP: its 32 NCCL all-to-alls too) in one CUDA graph: no host synchronisation
    # anywhere in it, and every rank captures and replays the same collectives in the same order
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        step()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
    torch.cuda.current_stream(dev).wait_stream(stream)
    for _ in range(warmup):
        graph.replay()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(True), torch.cuda.Event(True)
    s_ev.record()
    for _ in range(steps):
        graph.replay()
    e_ev.record()
    torch.cuda.synchronize()
    t = torch.tensor([s_ev.elapsed_time(e_ev) / steps], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.barrier()
    del graph  # (a graph holding NCCL calls is released before the process group)
    if world > 1:
        errs = {k: v for ep in eps_blocks for k, v in ep.errors().items()}
        if errs:
            raise RuntimeError(f"stack prefill EP device errors: {errs}")
    ms = t.item()
    flops = O.prefill_flops(per_rank * world) * layers
    tf_peak, tf_kind = peaks_tensor()
    tflops = flops / (ms * 1e-3) / 1e12
    return {"metric": f"prefill tokens/s (BASELINE configs[4](b): {tokens} tokens through {layers} layers, "
                      + ("1 GPU" if world == 1 else f"expert parallel over {world} GPUs, strong scaling") + ")",
            "tokens": per_rank * world, "tokens_per_gpu": per_rank, "layers": layers, "ms_per_step": round(ms, 3),
            "tokens_per_s": round(per_rank * world / (ms * 1e-3), 0), "tflops": round(tflops, 1),
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": tf_peak * world, "unit": "TFLOP/s",
                         "frac": round(tflops / (tf_peak * world), 4),
                         "note": f"algorithmic FLOPs / step time; peak {tf_kind}" + (f" x {world} GPUs" if world > 1 else "")}}


def run_ours(args):
    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from oracle import moe_oracle as O
    LAYERS = args.layers
    blocks = make_stack(dev, LAYERS)
    Md = args.decode_m
    x0 = O.make_tokens(Md, seed=3).to(dev)
    bufs = [torch.empty(Md, H, dtype=torch.bfloat16, device=dev) for _ in range(LAYERS + 1)]
    bufs[0].copy_(x0)
    ids = torch.empty(Md, TOPK + 2, dtype=torch.int32, device=dev)

    def step():
        for layer, blk in enumerate(blocks):
            blk.decode(bufs[layer], out=bufs[layer + 1], ids=ids if layer == 0 else None)

    step()  # creates the workspaces before capture
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        step()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
    torch.cuda.current_stream(dev).wait_stream(stream)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    U = O.distinct_experts(ids.cpu()[:, :TOPK])

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    # clocks are sampled from the first timed region to the end of the last (decode, e2e, prefill, int8, sweep, stack)
    clk = ClockSampler(local).__enter__()
    barrier()
    s_ev, e_ev = torch.cuda.Event(True), torch.cuda.Event(True)
    s_ev.record()
    for _ in range(args.steps):
        graph.replay()
    e_ev.record()
    barrier()
    elapsed_ms = s_ev.elapsed_time(e_ev)
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    elapsed_ms = t.item()
    ms_per_step = elapsed_ms / args.steps
    us_per_block = ms_per_step * 1e3 / LAYERS

    # end to end through the public API: pinned host token in, result out, every step (eager calls)
    h_in = torch.empty(Md, H, dtype=torch.bfloat16).pin_memory()
    h_in.copy_(x0.cpu())
    h_out = torch.empty(Md, H, dtype=torch.bfloat16).pin_memory()
    for _ in range(args.warmup):
        bufs[0].copy_(h_in, non_blocking=True)
        step()
        h_out.copy_(bufs[LAYERS], non_blocking=True)
    barrier()
    s2, e2 = torch.cuda.Event(True), torch.cuda.Event(True)
    s2.record()
    for _ in range(args.steps):
        bufs[0].copy_(h_in, non_blocking=True)
        step()
        h_out.copy_(bufs[LAYERS], non_blocking=True)
    e2.record()
    barrier()
    t2 = torch.tensor([s2.elapsed_time(e2)], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t2, op=torch.distributed.ReduceOp.MAX)
    e2e_us = t2.item() / args.steps * 1e3 / LAYERS

    pre = None
    if not args.no_prefill:
        if world > 1:
            pre = ep_prefill_lines(dev, world, rank, max(3, min(args.steps, 20)), args.warmup)
        else:
            pre = prefill_lines(dev, max(3, min(args.steps, 50)), args.warmup)
    q8 = None
    if world == 1 and not args.no_int8 and Md == 1:
        q8 = int8_decode_lines(dev, max(3, min(args.steps, 300)), args.warmup, layers=LAYERS)
    sweep = None
    if world == 1 and not args.no_sweep and Md == 1:
        sweep = decode_sweep_lines(blocks, dev, max(3, min(args.steps, 100)), args.warmup, ms=(2, 4, 8, 16))
    stack = None
    if not args.no_stack:
        stack = stack_prefill_lines(dev, world, rank, max(3, min(args.steps, 10)), args.warmup, blocks=blocks,
                                    layers=LAYERS)
    clk.__exit__()
    peak, peak_kind = peaks()
    byts = O.decode_bytes(U, M=Md)  # algorithmic bytes of one block step
    achieved = byts / (us_per_block * 1e-6) / 1e9
    out = None
    if rank == 0:
        cpu_v, cores, sample = cpu_block_time_us() if world == 1 else (None, None, None)
        out = {
            "metric": METRIC, "value": round(us_per_block / Md / world, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) weights generated on the device; N(0,1) token)",
            "config": {"workload": f"decode M={Md} through a 16-layer chain of MoE blocks (BASELINE configs[1] at "
                                   f"M={Md}, run as configs[4](a): one CUDA graph per step, one kernel per block)",
                       "tokens_per_step": Md,
                       "layers": LAYERS, "H": H, "I": I, "E": E, "top_k": TOPK, "shared_I": IS,
                       "routed_experts_hit": U, "parallelism": f"replicas x{world}",
                       "l2": "weights per step (16 x 139 MB) exceed L2; no flush"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": ncu_traffic(),
                         "note": f"{byts / 1e6:.1f} MB algorithmic per block / (graph step time / 16); "
                                 f"peak {peak_kind}"},
            "cpu_baseline": ({"value": round(cpu_v, 1), "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
                             if world == 1 else None),
            "e2e": {"value": round(e2e_us / Md / world, 3), "unit": UNIT, "h2d_bytes_per_step": H * 2 * Md,
                    "d2h_bytes_per_step": H * 2 * Md},
            "gpu_launches": LAYERS * args.steps,
            "clocks": clk.summary(),
        }
        if pre is not None:
            tf_peak, tf_kind = peaks_tensor()
            name = ("prefill tokens/s (BASELINE configs[3], 1 GPU, one block)" if world == 1 else
                    f"prefill tokens/s (BASELINE configs[3] per rank, expert parallel over {world} GPUs, one block)")
            out["prefill"] = {"metric": name, **pre,
                              "roofline": {"bound": "tensor", "achieved": pre["tflops"], "peak": tf_peak * world,
                                           "unit": "TFLOP/s", "frac": round(pre["tflops"] / (tf_peak * world), 4),
                                           "note": f"algorithmic FLOPs / pass time; peak {tf_kind}"
                                                   + (f" x {world} GPUs" if world > 1 else "")}}
        if q8 is not None:
            out["int8_decode"] = q8
        if sweep is not None:
            m1 = {"M": 1, "us_per_token": out["value"], "us_per_block": round(us_per_block, 2),
                  "routed_experts_hit": U, "bytes_per_block": byts, "hbm_gbs": round(achieved, 1),
                  "hbm_frac": round(achieved / peak, 4)}
            out["decode_sweep"] = {"metric": "decode us/token at M tokens (BASELINE configs[1], 16-layer graph chain)",
                                   "rows": [m1] + sweep}
        if stack is not None:
            out["stack_prefill"] = stack
        out["reference_kernels"] = {
            "unavailable": "the reference's own GPU kernels are Triton source inside the ming-voice application, "
                           "which is not an installable package (no setup.py / pyproject.toml), so they cannot be "
                           "installed into baseline/_ref or travel to the GPU box; their numerics are pinned on the "
                           "CPU by the golden fixtures (tests/golden) instead"}
    if world > 1:
        torch.distributed.barrier()
        del graph
        torch.distributed.destroy_process_group()
    if out is not None:
        print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=LAYERS, help="blocks in the chain (1 = the small profiling case)")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill (configs[3]) measurement")
    ap.add_argument("--no-int8", action="store_true", help="skip the int8 decode (configs[2]) measurement")
    ap.add_argument("--no-sweep", action="store_true", help="skip the decode token-count sweep (configs[1])")
    ap.add_argument("--no-stack", action="store_true", help="skip the 16-layer 8192-token prefill (configs[4](b))")
    ap.add_argument("--decode-m", type=int, default=1, choices=range(1, 17), metavar="M",
                    help="tokens per decode step (1 = the headline; 2..16 = the other configs[1] points)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="run only the prefill measurement (the profiling case for the grouped GEMMs)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.prefill_only:
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(dev)
        print(json.dumps(prefill_lines(dev, args.steps, args.warmup)), flush=True)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
