#!/usr/bin/env python
"""Benchmark of the quantized-expert MoE decode path.

Workload at N=1: the full 40-layer expert stack, 40 x 256 three-bit experts
(14.09 GB, resident in HBM, device-generated synthetic values), one 4-bit shared
expert per layer, batch 8 (headline) and batch 1 (reported under "batch1"),
per-layer top-8 ids drawn from a Zipf(1.1) popularity, hidden ~N(0,1) bf16.
One step = one pass of the 40 layers (40 calls of the per-layer entry point).
Metric = algorithmic HBM bytes per second: every distinct selected expert block
(1,376,256 B) plus the shared expert (1,769,472 B) per layer, divided by the
device time of the step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`--impl reference` times the CPU restatement of the reference's own CPU expert
path (oracle/finch_oracle.c; the reference's Objective-C file does not compile
here) on the host cores, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from finchmoe_b200 import synth  # noqa: E402

HIDDEN, INTER, NEXP, TOPK, LAYERS = 2048, 512, 256, 8, 40
EXPERT_BYTES = 1376256
SHARED_BYTES = 3 * 589824
GATEUP_BYTES = 2 * (393216 + 2 * 32768)  # gate + up codes, scales, biases of one expert
SCALE_FP16, ACT_BF16 = 1, 0
METRIC = "moe3_decode_hbm_gbs"


def routing_sets(batch: int, n_sets: int, n_layers: int | None = None):
    """[set][layer] -> (ids [B,8], weights [B,8]); Zipf(1.1) popularity per layer."""
    n_layers = LAYERS if n_layers is None else n_layers
    out = []
    for s in range(n_sets):
        per_layer = []
        for l in range(n_layers):
            per_layer.append(synth.zipf_routing(synth.rng_for(2, l, 100 + s), batch, NEXP, TOPK))
        out.append(per_layer)
    return out


def alg_bytes(ids: np.ndarray, shared: bool = True) -> int:
    return len(set(ids.ravel().tolist())) * EXPERT_BYTES + (SHARED_BYTES if shared else 0)


class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "100",
                                       "-i", str(gpu_index)], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            pass

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.p.terminate()
        self.p.wait()
        self.f.flush()
        self.f.seek(0)
        sm, mx, reasons, pw = [], [], set(), []
        for line in self.f.read().splitlines():
            c = [x.strip() for x in line.split(",")]
            if len(c) < 9:
                continue
            try:
                sm.append(float(c[1]))
                mx.append(float(c[2]))
                pw.append(float(c[3]))
            except ValueError:
                continue
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), c[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        self.f.close()
        os.unlink(self.f.name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        # "under load" = samples at or above the median power draw
        med_p = float(np.median(pw))
        load = [s for s, p in zip(sm, pw) if p >= med_p] or sm
        return {"sm_mhz": float(np.median(load)), "sm_max_mhz": float(max(mx)), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": float(max(pw))}


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# --------------------------------------------------------------------- CPU arm
def cpu_arm(batch: int, sample_layers: int, threads: int, steps: int = 1, warmup: int = 0, blocks_from=None):
    """Times the oracle's CPU expert path on `sample_layers` layers of the
    batch-`batch` workload.  Returns (GB/s by the same byte definition, seconds per pass, description)."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle as orc
    orc.build()
    rs = routing_sets(batch, 1, sample_layers)[0]
    x = synth.activations(synth.rng_for(2, 0, 7), batch, HIDDEN)
    layers = []
    total_bytes = 0
    for l, (ids, w) in enumerate(rs):
        uniq = sorted(set(ids.ravel().tolist()))
        if blocks_from is not None:
            blocks = {e: blocks_from(l, e) for e in uniq}
        else:
            rng = synth.rng_for(2, l, 55)
            one = synth.expert_block(rng, scale_dtype=SCALE_FP16)
            # distinct contents per expert are irrelevant to CPU speed: rotate one block's bytes
            blocks = {e: np.roll(one, 3 * i) if i else one for i, e in enumerate(uniq)}
        sh = synth.shared_expert(synth.rng_for(2, l, 56), scale_dtype=SCALE_FP16)
        layers.append((ids, w, blocks, sh))
        total_bytes += alg_bytes(ids)
    per_tok_threads = min(TOPK, max(1, threads))
    tok_workers = max(1, threads // per_tok_threads)

    def one_pass():
        for ids, w, blocks, sh in layers:
            def tok(t):
                return orc.moe_layer([blocks[int(e)] for e in ids[t]], w[t], None, x[t], scale_dtype=SCALE_FP16,
                                     shared=sh, shared_gate_score=0.1, accum=orc.ACC_F32, nthreads=per_tok_threads)
            if tok_workers > 1 and batch > 1:
                with ThreadPoolExecutor(tok_workers) as ex:
                    list(ex.map(tok, range(batch)))
            else:
                for t in range(batch):
                    tok(t)
    for _ in range(warmup):
        one_pass()
    t0 = time.perf_counter()
    for _ in range(steps):
        one_pass()
    dt = (time.perf_counter() - t0) / steps
    return total_bytes / dt / 1e9, dt, f"{sample_layers} of {LAYERS} layers, batch {batch}, sequential-fp32 C port"


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    # sized so warmup + steps stay within a few minutes: ~0.03 s per (token, expert) on one core
    budget_s = 20.0
    per_layer_s = 8 * 8 * 0.012 / min(cores, 64) + 0.02
    sample_layers = int(max(1, min(LAYERS, budget_s / max(1, args.steps + args.warmup) / per_layer_s)))
    gbs, dt, what = cpu_arm(8, sample_layers, cores, steps=args.steps, warmup=args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt * 1e3 * LAYERS / sample_layers, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "C2: 40-layer 3-bit expert stack decode, batch 8, top-8 of 256, Zipf(1.1)", "batch": 8,
                   "layers": LAYERS, "hidden": HIDDEN, "moe_inter": INTER, "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port", "sample": what},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line))


# --------------------------------------------------------------------- GPU arm
class Stack:
    """The 40-layer expert stack resident on one GPU."""

    def __init__(self, device: int, max_tokens: int, layers: int = LAYERS, seed: int = 2024, shard=None):
        """shard = (rank, world): keep only this rank's contiguous block of experts (expert parallelism)."""
        import torch

        from finchmoe_b200 import api, lib as L
        self.torch, self.L = torch, L
        torch.cuda.set_device(device)
        self.ctx = api.Context(device=device, n_layers=layers, max_tokens=max_tokens, scale_dtype=L.FP16, act_dtype=L.BF16)
        if shard is None:
            self.pool = self.ctx.pool()
            self.pool.fill_synthetic(0, layers, seed)
        else:
            rank, world = shard
            per = NEXP // world
            self.pool = self.ctx.pool(max_slots=layers * per)
            self.ctx.check(self.ctx.lib.finch_pool_fill_synthetic_range(self.pool.h, 0, layers, rank * per, (rank + 1) * per, seed))
        self.layers = layers
        self.shared = []
        for l in range(layers):
            sh = synth.shared_expert(synth.rng_for(2, l, 56), scale_dtype=SCALE_FP16)
            self.shared.append([self.ctx.upload_tensor(t) for t in sh])
        self.stream = torch.cuda.Stream(device=device)

    def device_inputs(self, rsets, batch):
        torch = self.torch
        dev = []
        for rs in rsets:
            ids = torch.from_numpy(np.stack([r[0] for r in rs])).cuda()      # [L,B,8] int32
            w = torch.from_numpy(np.stack([r[1] for r in rs])).cuda()        # [L,B,8] fp32
            dev.append((ids, w))
        x = synth.activations(synth.rng_for(2, 0, 7), batch, HIDDEN)
        xd = torch.from_numpy(x).cuda().to(torch.bfloat16)
        score = torch.full((batch,), 0.1, device="cuda")
        out = torch.empty((self.layers, batch, HIDDEN), device="cuda")
        return dev, xd, score, out, x

    def encode_step(self, ids, w, xd, score, out, batch):
        st = self.stream.cuda_stream
        for l in range(self.layers):
            sh = self.ctx.make_shared(*self.shared[l], gate_score=score)
            self.ctx.encode_moe_decode(self.pool, l, xd, ids[l], w[l], None, sh, None, out[l], batch, stream=st)

    def capture(self, rsets_dev, xd, score, out, batch):
        """One CUDA graph per routing set: the 40 per-layer calls of a step, captured from the stream."""
        torch = self.torch
        ids, w = rsets_dev[0]
        self.encode_step(ids, w, xd, score, out, batch)  # first call sets kernel attributes: keep it out of capture
        torch.cuda.synchronize()
        graphs = []
        for ids, w in rsets_dev:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                self.encode_step(ids, w, xd, score, out, batch)
            graphs.append(g)
        return graphs

    def time_steps(self, rsets_dev, xd, score, out, batch, steps, warmup, barrier=None, use_graph=True):
        torch = self.torch
        graphs = self.capture(rsets_dev, xd, score, out, batch) if use_graph else None

        def run(i):
            if graphs is not None:
                with torch.cuda.stream(self.stream):
                    graphs[i % len(graphs)].replay()
            else:
                ids, w = rsets_dev[i % len(rsets_dev)]
                self.encode_step(ids, w, xd, score, out, batch)
        for i in range(warmup):
            run(i)
        torch.cuda.synchronize()
        if barrier:
            barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for i in range(steps):
            run(warmup + i)
        e1.record(self.stream)
        torch.cuda.synchronize()
        if barrier:
            barrier()
        return e0.elapsed_time(e1) / 1e3  # seconds for `steps` steps

    def time_prefill(self, T, steps, warmup):
        """One chunk of T tokens through finch_encode_moe_prefill on every layer; seconds per pass, distinct experts."""
        torch = self.torch
        rs = routing_sets(T, 1, self.layers)
        dev, xd, score, out, _ = self.device_inputs(rs, T)
        ids, w = dev[0]

        def step():
            st = self.stream.cuda_stream
            for l in range(self.layers):
                sh = self.ctx.make_shared(*self.shared[l], gate_score=score)
                self.ctx.encode_moe_decode(self.pool, l, xd, ids[l], w[l], None, sh, None, out[l], T, stream=st, prefill=True)
        for _ in range(max(1, warmup)):
            step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for _ in range(steps):
            step()
        e1.record(self.stream)
        torch.cuda.synchronize()
        uniq = sum(len(set(i_.ravel().tolist())) for i_, _ in rs[0])
        return e0.elapsed_time(e1) / 1e3 / steps, uniq

    def time_e2e(self, rsets, x, batch, steps, warmup):
        """Host buffers in and out through finch_moe_forward_host, layer by layer.  Every call stages its inputs in
        pinned host memory and the bytes cross the bus inside the timed region, both ways: for decode-sized calls as
        reads and writes of the layer's kernels on the pinned block, otherwise as one copy in and one copy out."""
        torch = self.torch
        xw = self.ctx.acts_to_wire(x)
        score = np.full(batch, 0.1, np.float32)
        h2d = xw.nbytes + batch * TOPK * 8 + score.nbytes
        d2h = batch * HIDDEN * 4

        shs = [self.ctx.make_shared(*self.shared[l]) for l in range(self.layers)]

        def step(rs):
            last = None
            for l in range(self.layers):
                last = self.ctx.moe_forward_host(self.pool, l, xw, rs[l][0], rs[l][1], shared=shs[l], gate_score=score)
            return last
        for i in range(warmup):
            step(rsets[i % len(rsets)])
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(steps):
            step(rsets[(warmup + i) % len(rsets)])
        torch.cuda.synchronize()
        return (time.perf_counter() - t0), h2d * self.layers, d2h * self.layers


def run_ours(args):
    import torch
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    if world > 1:
        return run_ep(args, rank, local_rank, world)
    batch = 8
    stack = Stack(local_rank, max_tokens=512, layers=LAYERS)
    n_sets = 4
    rsets = [[(ids, w) for ids, w in rs] for rs in routing_sets(batch, n_sets)]
    dev, xd, score, out, x = stack.device_inputs(rsets, batch)

    sampler = ClockSampler(local_rank)
    secs = stack.time_steps(dev, xd, score, out, batch, args.steps, args.warmup, None, use_graph=not args.no_graph)
    launches = 4 * LAYERS * args.steps  # four kernels per layer call (graph replays launch them without the host counter)
    clocks = sampler.stop()
    step_bytes = [sum(alg_bytes(ids) for ids, _ in rs) for rs in rsets]
    timed_bytes = sum(step_bytes[(args.warmup + i) % n_sets] for i in range(args.steps))
    value = timed_bytes / secs / 1e9

    # end to end through the host-pointer entry point
    e2e_warm = max(3, args.warmup)
    e2e_secs, h2d, d2h = stack.time_e2e(rsets, x, batch, args.steps, e2e_warm)
    e2e_bytes = sum(step_bytes[(e2e_warm + i) % n_sets] for i in range(args.steps))   # the routing sets its timed steps used
    e2e_value = e2e_bytes / e2e_secs / 1e9

    peaks, peak_kind = measured_peaks()
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "C2: 40-layer 3-bit expert stack decode, batch 8, top-8 of 256, Zipf(1.1)", "batch": batch,
                   "layers": LAYERS, "hidden": HIDDEN, "moe_inter": INTER, "scale_dtype": "fp16", "act_dtype": "bf16",
                   "pool_gb": LAYERS * NEXP * EXPERT_BYTES / 1e9, "parallelism": "1 GPU",
                   "l2": "inputs larger than L2: every step streams >= 0.5 GB of a 14 GB pool; 4 routing sets rotate"},
        "clocks": clocks,
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "hbm_frac_of_" + peak_kind: value / world / peaks["hbm_gbs"],
    }

    if world == 1:
        # batch 1 (single-stream decode) on the same pool
        r1 = [[(ids, w) for ids, w in rs] for rs in routing_sets(1, n_sets)]
        dev1, xd1, score1, out1, _ = stack.device_inputs(r1, 1)
        s1 = stack.time_steps(dev1, xd1, score1, out1, 1, args.steps, args.warmup, use_graph=not args.no_graph)
        b1 = sum(sum(alg_bytes(ids) for ids, _ in r1[(args.warmup + i) % n_sets]) for i in range(args.steps))
        line["batch1"] = {"value": b1 / s1 / 1e9, "unit": "GB/s", "ms_per_step": s1 / args.steps * 1e3,
                          "us_per_layer": s1 / args.steps / LAYERS * 1e6, "frac_of_" + peak_kind: b1 / s1 / 1e9 / peaks["hbm_gbs"]}
        # per-kernel roofline of the dominant kernel (gate/up/SiLU)
        line["roofline"] = kernel_roofline(stack, dev, rsets, xd, score, out, batch, args, peaks, peak_kind)
        # chunked prefill: 512-token chunks through the grouped dequant-GEMM (tcgen05), the whole stack
        T = 512
        ps, uniq = stack.time_prefill(T, max(2, args.steps // 4), 1)
        flops = LAYERS * (T * TOPK * 6291456 + T * 3 * 2 * 512 * HIDDEN)
        pbytes = uniq * EXPERT_BYTES + LAYERS * SHARED_BYTES
        ai = flops / pbytes
        ceil_tf = min(peaks["bf16_tflops_sustained"], ai * peaks["hbm_gbs"] / 1e3)
        line["prefill"] = {"metric": "moe3_prefill_tokens_per_s", "chunk": T, "value": T / ps, "unit": "tokens/s (40 MoE layers per token)",
                           "ms_per_chunk": ps * 1e3, "tflops": flops / ps / 1e12, "hbm_gbs": pbytes / ps / 1e9,
                           "roofline": {"bound": "hbm", "note": "8T/256 pairs per expert: below the tensor ridge", "ceiling_tflops": ceil_tf,
                                        "frac": flops / ps / 1e12 / ceil_tf, "peak_kind": peak_kind}}
        line["other_rows"] = aux_rooflines(stack, peaks, peak_kind)
        # CPU baseline: bounded sample of the same workload on the expert blocks of this pool
        cores = os.cpu_count() or 1
        sample_layers = 2
        gbs, dt, what = cpu_arm(batch, sample_layers, cores, blocks_from=lambda l, e: stack.pool.get(l, e))
        line["cpu_baseline"] = {"value": gbs, "unit": "GB/s", "cores": cores, "kind": "port", "sample": what,
                                "seconds": dt}
    print(json.dumps(line))



def run_ep(args, rank, local_rank, world):
    """N > 1: the batched-decode layer is expert parallel.  Every rank owns 8 tokens per step (weak scaling:
    8 N tokens per step in all) and the contiguous block of 256 / N experts of every layer; per layer the
    ranks exchange activation rows and partial outputs (finchmoe_b200/ep.py).  value = bytes of the distinct
    local experts each rank streams per step (plus its copy of the shared expert), summed over ranks, per
    second of the slowest rank."""
    import torch
    import torch.distributed as dist

    from finchmoe_b200 import ep
    batch, n_sets = 8, 4
    stack = Stack(local_rank, max_tokens=8 * world, layers=LAYERS, shard=(rank, world))
    per = NEXP // world
    # every rank can regenerate every rank's routing (seeded), which is all the byte count needs
    all_sets = [[[synth.zipf_routing(synth.rng_for(2, l, 100 + s + 1000 * r), batch, NEXP, TOPK) for l in range(LAYERS)]
                 for s in range(n_sets)] for r in range(world)]
    rsets = all_sets[rank]
    dev, xd, score, out, x = stack.device_inputs(rsets, batch)
    backend = ep.GpuBackend(stack.ctx, stack.pool, batch * world)
    shared = [stack.ctx.make_shared(*stack.shared[l], gate_score=score) for l in range(LAYERS)]

    # Decode batches are small and the same size on every rank: the fixed-capacity exchange (every token to
    # every rank, known message sizes) needs no row counts and no host synchronisation, so a whole step is a
    # fixed sequence of launches and all-to-alls, recorded once per routing set into a CUDA graph.
    def layers_of(s):
        ids, w = dev[s]
        for l in range(LAYERS):
            ep.ep_layer_static(backend, dist, None, l, xd, ids[l], w[l], None, shared[l], None, out[l], in_scope=True)

    def step_eager(i):
        with backend.stream_scope():
            layers_of(i % n_sets)

    graphs, graph_note = None, "launched from the host every step"
    if not args.no_graph:
        try:
            for s in range(n_sets):          # communicators, lazily made buffers and tables exist before capture
                step_eager(s)
            torch.cuda.synchronize()
            dist.barrier()
            graphs = []
            for s in range(n_sets):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=backend.stream, capture_error_mode="thread_local"):
                    layers_of(s)
                graphs.append(g)
            torch.cuda.synchronize()
            graph_note = "one CUDA graph per routing set (kernels and all-to-alls)"
        except Exception as e:               # capture of the collectives unavailable: keep launching from the host
            graphs = None
            graph_note = "launched from the host every step (graph capture failed: %s)" % (str(e).splitlines()[0][:120] if str(e) else type(e).__name__)
            torch.cuda.synchronize()
    # every rank must take the same path: a rank that replays graphs cannot pair with one that launches eagerly
    flag = torch.tensor([1 if graphs is not None else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if int(flag.item()) == 0:
        graphs = None

    def step(i):
        if graphs is not None:
            graphs[i % n_sets].replay()
        else:
            step_eager(i)

    def timed(n, w0, fn):
        for i in range(w0):
            fn(i)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(n):
            fn(w0 + i)
        e1.record()
        torch.cuda.synchronize()
        dist.barrier()
        t = torch.tensor([e0.elapsed_time(e1) / 1e3], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    sampler = ClockSampler(local_rank) if rank == 0 else None
    secs = timed(args.steps, args.warmup, step)
    clocks = sampler.stop() if sampler else None

    # end to end: the step's inputs come from pinned host memory and its result goes back to the host
    xh = torch.from_numpy(stack.ctx.acts_to_wire(x).view(np.int16)).pin_memory()
    res = torch.empty((batch, HIDDEN), dtype=torch.float32).pin_memory()

    def step_e2e(i):
        xd.view(torch.int16).copy_(xh, non_blocking=True)
        step(i)
        res.copy_(out[LAYERS - 1], non_blocking=True)
        torch.cuda.current_stream().synchronize()
    e2e_secs = timed(args.steps, max(3, args.warmup), step_e2e)

    def step_bytes(s):
        total = 0
        for l in range(LAYERS):
            touched = set()
            for r in range(world):
                touched |= set(all_sets[r][s][l][0].ravel().tolist())
            total += len(touched) * EXPERT_BYTES + world * SHARED_BYTES     # every rank reads its own copy of the shared expert
        return total
    timed_bytes = sum(step_bytes((args.warmup + i) % n_sets) for i in range(args.steps))
    e2e_bytes = sum(step_bytes((max(3, args.warmup) + i) % n_sets) for i in range(args.steps))
    if rank == 0:
        peaks, peak_kind = measured_peaks()
        value = timed_bytes / secs / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": "C5: expert-parallel batched decode, 40 layers, 8 tokens per GPU per step, top-8 of 256, Zipf(1.1)",
                       "batch": batch * world, "layers": LAYERS, "hidden": HIDDEN, "moe_inter": INTER, "scale_dtype": "fp16",
                       "act_dtype": "bf16", "experts_per_gpu": per, "parallelism": f"ep{world}",
                       "exchange": "fixed capacity: 2 all-to-alls per layer over NCCL (records, partial rows), no host synchronisation",
                       "launch": graph_note,
                       "l2": "inputs larger than L2: the pool shards exceed it; 4 routing sets rotate"},
            "clocks": clocks,
            "e2e": {"value": e2e_bytes / e2e_secs / 1e9, "unit": "GB/s", "h2d_bytes_per_step": int(xh.numel() * 2 * world),
                    "d2h_bytes_per_step": int(res.numel() * 4 * world)},
            "gpu_launches": int(stack.ctx.launch_count()),
            "tokens_per_s": batch * world * args.steps / secs,
            "us_per_layer": secs / args.steps / LAYERS * 1e6,
            "hbm_frac_of_" + peak_kind: value / world / peaks["hbm_gbs"],
        }
        print(json.dumps(line), flush=True)
    # The graphs hold the recorded all-to-alls: they go before the communicator does, and the process then
    # leaves without tearing NCCL down (a communicator destroyed after graphs had captured its collectives did
    # not return on this stack).
    graphs = None
    torch.cuda.synchronize()
    dist.barrier()
    sys.stdout.flush()
    sys.stderr.flush()
    os._exit(0)


def aux_rooflines(stack, peaks, peak_kind, iters=8):
    """The other matvec rows of the path, each timed alone with CUDA events and the L2 flushed (a 256 MB
    write) before every timed launch: 4-bit g64 projections and GGUF Q4_K / Q6_K tensors through
    finch_encode_batch_matvec at 1 / 8 (/ 90) positions, and the 4-bit projections at 64 / 512 positions
    through the tensor-core GEMM.  bytes = packed weights + scales (+ activations); flops = 2 T out in."""
    import ctypes as C

    import torch
    ctx, L = stack.ctx, stack.L
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    rng = synth.rng_for(4, 0, 99)
    st = stack.stream
    rows = []

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(iters):
            with torch.cuda.stream(st):
                flush.fill_(1)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
                fn()
                e1.record(st)
            torch.cuda.synchronize()
            tot += e0.elapsed_time(e1)
        return tot / iters * 1e-3

    def wbytes(t):
        return int(t["W"].nbytes + (t["S"].nbytes if t.get("S") is not None else 0) + (t["B"].nbytes if t.get("B") is not None else 0))

    cases = [("4bit_g64", synth.affine_tensor(rng, 8192, 2048, 4, SCALE_FP16), (1, 8)),
             ("4bit_g64", synth.affine_tensor(rng, 2048, 4096, 4, SCALE_FP16), (1, 8)),
             ("q4_k", synth.gguf_tensor(rng, 8192, 2048, 12), (1, 8, 90)),
             ("q6_k", synth.gguf_tensor(rng, 8192, 2048, 14), (1, 8, 90)),
             ("q4_k", synth.gguf_tensor(rng, 2048, 512, 12), (1, 8)),
             ("q6_k", synth.gguf_tensor(rng, 512, 2048, 14), (1, 8))]
    for name, t, Ts in cases:
        w = ctx.upload_tensor(t)
        for T in Ts:
            x = torch.from_numpy(synth.activations(rng, T, t["in_dim"])).cuda().to(torch.bfloat16)
            out = torch.empty((T, t["out_dim"]), dtype=torch.float32, device="cuda")
            secs = timed(lambda: ctx.fast_batch_matvec(x, L.BF16, [w], [out], M=T, stream=st.cuda_stream))
            b = wbytes(t) + T * t["in_dim"] * 2 + T * t["out_dim"] * 4
            rows.append({"op": f"matvec_{name}", "shape": [t["out_dim"], t["in_dim"]], "T": T, "us": secs * 1e6, "gbs": b / secs / 1e9,
                         "frac_hbm_" + peak_kind: b / secs / 1e9 / peaks["hbm_gbs"]})
    for shape in ((8192, 2048), (2048, 4096)):
        t = synth.affine_tensor(rng, shape[0], shape[1], 4, SCALE_FP16)
        w = ctx.upload_tensor(t)
        for T in (64, 512):
            x = torch.from_numpy(synth.activations(rng, T, shape[1])).cuda().to(torch.bfloat16)
            out = torch.empty((T, shape[0]), dtype=torch.float32, device="cuda")
            secs = timed(lambda: ctx.check(ctx.lib.finch_encode_dense_gemm(ctx.h, st.cuda_stream, C.byref(w), x.data_ptr(), out.data_ptr(), T)))
            fl, b = 2.0 * T * shape[0] * shape[1], wbytes(t) + T * shape[1] * 2 + T * shape[0] * 4
            ceil = min(peaks["bf16_tflops"], fl / b * peaks["hbm_gbs"] / 1e3)
            rows.append({"op": "dense_gemm_4bit_g64_tcgen05", "shape": list(shape), "T": T, "us": secs * 1e6, "tflops": fl / secs / 1e12,
                         "gbs": b / secs / 1e9, "ceiling_tflops": ceil, "frac_" + peak_kind: fl / secs / 1e12 / ceil})
    return rows


def kernel_roofline(stack, dev, rsets, xd, score, out, batch, args, peaks, peak_kind):
    """Average duration of the gate/up/SiLU kernel over the same steps, from CUDA
    events recorded around every launch on the launching stream (a separate pass
    with per-kernel events, so the headline timing carries no event overhead)."""
    import ctypes as C
    lib = stack.ctx.lib
    if not hasattr(lib, "finch_profile_enable"):
        return None
    lib.finch_profile_enable.argtypes = [C.c_void_p, C.c_int]
    lib.finch_profile_read.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_float), C.POINTER(C.c_int)]
    n_sets = len(dev)
    lib.finch_profile_enable(stack.ctx.h, 1)
    gate_bytes = 0
    for i in range(args.steps):
        ids, w = dev[(args.warmup + i) % n_sets]
        stack.encode_step(ids, w, xd, score, out, batch)
        gate_bytes += sum(len(set(i_.ravel().tolist())) * GATEUP_BYTES + 2 * 589824 for i_, _ in rsets[(args.warmup + i) % n_sets])
    stack.torch.cuda.synchronize()
    ms_a, ms_b, n = C.c_float(), C.c_float(), C.c_int()
    lib.finch_profile_read(stack.ctx.h, C.byref(ms_a), C.byref(ms_b), C.byref(n))
    lib.finch_profile_enable(stack.ctx.h, 0)
    if n.value == 0:
        return None
    per_launch_bytes = gate_bytes / n.value
    achieved = per_launch_bytes / (ms_a.value / n.value * 1e-3) / 1e9
    return {"bound": "hbm", "kernel": "moe_gateup_kernel", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / peaks["hbm_gbs"], "peak_kind": peak_kind,
            # dram__bytes_read + write of one launch with 38 distinct experts (36,044,800 algorithmic bytes):
            # 38,070,528 B (profiles/moe_decode_batch8_gateup_down_full.md), scaled to this run's average launch
            "traffic": per_launch_bytes * (38070528 / 36044800), "traffic_source": "ncu, 38-expert launch, scaled by bytes",
            "bytes_per_launch": per_launch_bytes, "us_per_launch": ms_a.value / n.value * 1e3,
            "down_combine_us_per_launch": ms_b.value / n.value * 1e3, "launches_timed": n.value}


def main():
    global LAYERS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=LAYERS, help="fewer layers = a small case for profiler captures")
    ap.add_argument("--no-graph", action="store_true", help="launch from the host every step instead of replaying CUDA graphs")
    ap.add_argument("--only", default="", choices=["", "prefill"], help="prefill: just the 512-token chunk on --layers layers (profiler captures)")
    args = ap.parse_args()
    LAYERS = args.layers
    if args.only == "prefill":
        stack = Stack(0, max_tokens=512, layers=LAYERS)
        ps, uniq = stack.time_prefill(512, max(1, args.steps), max(1, args.warmup))
        print(json.dumps({"only": "prefill", "chunk": 512, "layers": LAYERS, "ms_per_chunk": ps * 1e3, "tokens_per_s": 512 / ps,
                          "distinct_experts": uniq, "status": stack.ctx.device_status()}))
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
