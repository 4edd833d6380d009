#!/usr/bin/env python
"""Benchmark of the quantized-expert MoE path: the 40-layer 3-bit expert stack.

N = 1.  The full stack, 40 x 256 three-bit experts (14.09 GB resident in HBM, device-generated synthetic
values), one 4-bit shared expert per layer, batch 8 (headline) and batch 1, top-8 ids per layer drawn from a
Zipf(1.1) popularity that all tokens of a layer share, hidden ~N(0,1) bf16.  One step = one pass of the 40
layers (40 calls of the per-layer entry point).  Metric = algorithmic HBM bytes per second: every distinct
selected expert block (1,376,256 B) plus the shared expert (1,769,472 B) per layer, over the device time of
the step.  The same line carries the 512-token chunked prefill, the expert-parallel layer run by one rank,
the other matvec tiers and the CPU baseline.

N > 1 (under torchrun).  The expert-parallel layer: every rank holds 256 / N experts of every layer and owns
8 tokens per decode step and 512 tokens per prefill chunk (64 and 4096 in all at N = 8).  The line carries
tokens/s of both, the parity of what was timed, and the all-to-all's share of the time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`--impl reference` times the reference's own CPU expert path on the host cores (its C functions compiled into
oracle/_ref when that build is present, else the restatement in oracle/finch_oracle.c).
"""
from __future__ import annotations

import argparse
import gc
import json
import os
import re
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
PREFILL_CHUNK = 512
KERNELS_PER_LAYER = 3            # gate/up/SiLU, down, combine


def layer_popularity(layer: int) -> np.ndarray:
    return synth.zipf_popularity(synth.rng_for(2, layer, 7), NEXP)


def routing_sets(batch: int, n_sets: int, n_layers: int | None = None, rank: int = 0):
    """[set][layer] -> (ids [B,8], weights [B,8]).  A layer's Zipf(1.1) popularity is the same for every token,
    set and rank; the draws differ."""
    n_layers = LAYERS if n_layers is None else n_layers
    perms = [layer_popularity(l) for l in range(n_layers)]
    return [[synth.zipf_routing_shared(synth.rng_for(2, l, 100 + s + 1000 * rank), batch, perms[l], TOPK) for l in range(n_layers)]
            for s in range(n_sets)]


def alg_bytes(ids: np.ndarray, shared: bool = True) -> int:
    return len(set(ids.ravel().tolist())) * EXPERT_BYTES + (SHARED_BYTES if shared else 0)


def spread(ms) -> dict:
    a = np.asarray(ms, np.float64)
    return {"median": float(np.median(a)), "p10": float(np.percentile(a, 10)), "p90": float(np.percentile(a, 90)),
            "min": float(a.min()), "max": float(a.max()), "n": int(a.size)}


def cos_and_rel(got, want) -> dict:
    """cos and max |a - b| / max(|b|, rms(b)): the parity tests' two figures."""
    a, b = np.asarray(got, np.float64).ravel(), np.asarray(want, np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    cos = 1.0 if na == 0 and nb == 0 else float(a @ b / (na * nb + 1e-300))
    floor = np.sqrt(np.mean(b * b)) + 1e-30
    return {"cos": cos, "max_rel": float(np.max(np.abs(a - b) / np.maximum(np.abs(b), floor))), "finite": bool(np.all(np.isfinite(a)))}


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


def profiled_traffic_ratio():
    """DRAM bytes per algorithmic byte of the gate/up kernel, from the committed profiler summary
    (a line `traffic_ratio: dram_bytes / algorithmic_bytes`); None when the summary carries none."""
    p = os.path.join(ROOT, "profiles", "moe_gateup_kernel_batch8.md")
    try:
        m = re.search(r"^traffic_ratio:\s*([0-9]+)\s*/\s*([0-9]+)", open(p).read(), re.M)
    except OSError:
        return None, None
    if not m:
        return None, None
    return int(m.group(1)) / int(m.group(2)), os.path.relpath(p, ROOT)


# --------------------------------------------------------------------- CPU arm
class CpuExpertPath:
    """The reference's CPU expert path (serial over a token's experts, finchmoe/infer.m:10109-10204: gate and up
    matvec, SwiGLU, down matvec, weighted add), on expert blocks of the bench's shapes.  kind "reference" drives
    the reference's own functions (oracle/_ref); "port" the restatement."""

    def __init__(self):
        from oracle import oracle as orc
        self.orc = orc
        orc.build()
        self.ref = orc.ref_lib()
        self.kind = "reference" if self.ref is not None else "port"
        rng = synth.rng_for(2, 0, 55)
        self.blocks = [synth.expert_block(rng, scale_dtype=SCALE_FP16) for _ in range(8)]
        self.block = self.blocks[0]
        self.lay = synth.expert_layout()
        self.x = synth.activations(synth.rng_for(2, 0, 7), 8, HIDDEN)

    def blocks_for(self, uniq):
        # which values an expert holds is irrelevant to CPU speed: eight generated blocks take turns
        return {e: self.blocks[i % len(self.blocks)] for i, e in enumerate(uniq)}

    def pair(self, blk, x, w, acc):
        """acc += w * expert(x) for one (token, expert) pair."""
        if self.ref is None:
            acc += w * self.orc.expert_forward(blk, 3, SCALE_FP16, HIDDEN, INTER, 64, x, accum=self.orc.ACC_F32)
            return
        import ctypes as C
        R, L = self.ref, self.lay
        f32p = C.POINTER(C.c_float)
        base = blk.ctypes.data
        g, u, a, d = (np.empty(n, np.float32) for n in (INTER, INTER, INTER, HIDDEN))
        xp = x.ctypes.data_as(f32p)
        # the reference's function reads the 16-bit scale words as bf16; the arithmetic per weight is the same
        R.ref_cpu_dequant_matvec(base + L["gate_w"], base + L["gate_s"], base + L["gate_b"], xp, g.ctypes.data_as(f32p), INTER, HIDDEN, 64, 3)
        R.ref_cpu_dequant_matvec(base + L["up_w"], base + L["up_s"], base + L["up_b"], xp, u.ctypes.data_as(f32p), INTER, HIDDEN, 64, 3)
        R.ref_cpu_swiglu(g.ctypes.data_as(f32p), u.ctypes.data_as(f32p), a.ctypes.data_as(f32p), INTER)
        R.ref_cpu_dequant_matvec(base + L["down_w"], base + L["down_s"], base + L["down_b"], a.ctypes.data_as(f32p), d.ctypes.data_as(f32p),
                                 HIDDEN, INTER, 64, 3)
        R.ref_cpu_vec_madd(acc.ctypes.data_as(f32p), d.ctypes.data_as(f32p), float(w), HIDDEN)

    def time_layers(self, rs, batch, threads):
        """One pass over the layers of routing set rs ([layer] -> (ids, w)); returns (seconds, algorithmic bytes).
        The routed experts only, as the reference's CPU fallback runs them; threads > 1 = one pair per thread."""
        from concurrent.futures import ThreadPoolExecutor
        x = np.ascontiguousarray(self.x[:batch])
        jobs, nbytes = [], 0
        for ids, w in rs:
            blocks = self.blocks_for(sorted(set(ids.ravel().tolist())))
            accs = [np.zeros(HIDDEN, np.float32) for _ in range(batch)]
            jobs.append([(blocks[int(ids[t, k])], x[t], float(w[t, k]), accs[t], t) for t in range(batch) for k in range(TOPK)])
            nbytes += alg_bytes(ids, shared=False)
        t0 = time.perf_counter()
        if threads <= 1:
            for layer in jobs:
                for blk, xt, wk, acc, _ in layer:
                    self.pair(blk, xt, wk, acc)
        else:
            with ThreadPoolExecutor(threads) as ex:
                for layer in jobs:
                    # pairs of one token go to one worker in order (its accumulator is not shared)
                    per_tok = {}
                    for j in layer:
                        per_tok.setdefault(j[4], []).append(j)
                    chunks = []
                    for lst in per_tok.values():
                        n = max(1, min(len(lst), threads // max(1, len(per_tok))))
                        chunks += [lst[i::n] for i in range(n)]

                    def run(chunk):
                        part = np.zeros(HIDDEN, np.float32)
                        for blk, xt, wk, _, _ in chunk:
                            self.pair(blk, xt, wk, part)
                        return chunk[0][3], part
                    for acc, part in list(ex.map(run, chunks)):
                        acc += part
        return time.perf_counter() - t0, nbytes

    def numpy_row(self, rs, batch):
        """numpy: dequantise the tile (codes * scale + bias), then W @ x (BLAS threads as configured)."""
        x = self.x[:batch]
        n_pairs = sum(ids.size for ids, _ in rs)
        t0 = time.perf_counter()
        reps = min(n_pairs, 16)
        for _ in range(reps):
            for which in ("gate", "up", "down"):
                tt = synth.block_tensor(self.block, which, scale_dtype=SCALE_FP16)
                W = self.orc.np_dequant_affine(tt["W"], tt["S"], tt["B"], SCALE_FP16, tt["out_dim"], tt["in_dim"], 64, 3)
                _ = W @ (x[0] if which != "down" else np.zeros(INTER, np.float32))
        dt = (time.perf_counter() - t0) / reps
        return dt   # seconds per (token, expert) pair


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    cpu = CpuExpertPath()
    rs_all = routing_sets(8, 1)[0]
    # one probe pair sizes the step: all 40 layers when warm-up + steps fit in about two minutes, else fewer layers
    acc = np.zeros(HIDDEN, np.float32)
    cpu.pair(cpu.block, cpu.x[0], 1.0, acc)
    t0 = time.perf_counter()
    cpu.pair(cpu.block, cpu.x[0], 1.0, acc)
    pair_s = time.perf_counter() - t0
    threads = min(cores, 64)
    est_layer = 64 * pair_s / min(threads, 64) * 1.3 + 0.005
    n_layers = int(max(1, min(LAYERS, 120.0 / max(1, args.steps + args.warmup) / est_layer)))
    rs = rs_all[:n_layers]
    for _ in range(args.warmup):
        cpu.time_layers(rs, 8, threads)
    secs, nbytes = [], 0
    for _ in range(args.steps):
        dt, b = cpu.time_layers(rs, 8, threads)
        secs.append(dt)
        nbytes += b
    total = float(sum(secs))
    gbs = nbytes / total / 1e9
    # rows beside it, on one layer: the single-thread loop the reference's fallback runs, 8 threads, numpy
    one = rs_all[:1]
    dt1, b1 = cpu.time_layers(one, 8, 1)
    dt8, _ = cpu.time_layers(one, 8, 8)
    np_pair = cpu.numpy_row(one, 8)
    what = (f"{n_layers} of {LAYERS} layers per step, batch 8, routed experts, {threads} threads (one (token, expert) pair per task), "
            + ("the reference's C functions (finchmoe/infer.m:1676-1763, 1780-1786, 1849-1851) compiled with gcc -O2"
               if cpu.kind == "reference" else "sequential-fp32 C restatement"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3, "step_ms": spread([s * 1e3 for s in secs]),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "C2: 40-layer 3-bit expert stack decode, batch 8, top-8 of 256, Zipf(1.1)"
                   + ("" if world == 1 else f" (the one-process CPU path; it stands in for C5, the expert-parallel layer on {world} GPUs, which has no CPU form)"),
                   "batch": 8, "layers": LAYERS, "layers_per_step": n_layers, "hidden": HIDDEN, "moe_inter": INTER, "scale_dtype": "fp16",
                   "act_dtype": "f32", "pool_gb": LAYERS * NEXP * EXPERT_BYTES / 1e9, "parallelism": f"{threads} host threads",
                   "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": cpu.kind, "sample": what},
        "cpu_rows": {"single_thread": {"value": b1 / dt1 / 1e9, "unit": "GB/s", "ms_per_layer": dt1 * 1e3, "cores": 1,
                                       "note": "the reference's --cpu-experts loop is serial over experts (finchmoe/infer.m:10109-10204)"},
                     "threads_8": {"value": b1 / dt8 / 1e9, "unit": "GB/s", "ms_per_layer": dt8 * 1e3, "cores": 8},
                     "numpy": {"ms_per_pair": np_pair * 1e3, "note": "dequantise three tiles with numpy, then W @ x"}},
        "tokens_per_s": 8 * n_layers / LAYERS * args.steps / total,
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
        self.seed = seed
        self.ctx = api.Context(device=device, n_layers=layers, max_tokens=max_tokens, scale_dtype=L.FP16, act_dtype=L.BF16)
        if shard is None or shard[1] == 1:
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

    def time_steps(self, rsets_dev, xd, score, out, batch, steps, warmup, use_graph=True):
        """Returns (seconds for `steps` steps, [ms of every step]) from CUDA events on the launching stream: one
        event before the first step and one after each."""
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
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        ev[0].record(self.stream)
        for i in range(steps):
            run(warmup + i)
            ev[i + 1].record(self.stream)
        torch.cuda.synchronize()
        return ev[0].elapsed_time(ev[steps]) / 1e3, [ev[i].elapsed_time(ev[i + 1]) for i in range(steps)]

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
        pinned host memory and the bytes cross the bus inside the timed region, both ways: the inputs as one copy
        to the device, the result as the combine kernel's writes to the pinned block (decode-sized calls) or one
        copy back."""
        torch = self.torch
        xw = self.ctx.acts_to_wire(x)
        score = np.full(batch, 0.1, np.float32)
        h2d = xw.nbytes + batch * TOPK * 8 + score.nbytes
        d2h = batch * HIDDEN * 4

        import ctypes as C
        shs = [C.byref(self.ctx.make_shared(*self.shared[l])) for l in range(self.layers)]
        # host arrays of every (routing set, layer), converted once: a step then is 40 calls of the C entry point on
        # host addresses, as a C host would make them
        ids_h = [[np.ascontiguousarray(rs[l][0], np.int32) for l in range(self.layers)] for rs in rsets]
        w_h = [[np.ascontiguousarray(rs[l][1], np.float32) for l in range(self.layers)] for rs in rsets]
        outs = np.empty((batch, HIDDEN), np.float32)
        self._e2e_keep = (xw, score, ids_h, w_h, outs, shs)
        xp, sp, op = xw.ctypes.data, score.ctypes.data, outs.ctypes.data
        ids_p = [[a.ctypes.data for a in row] for row in ids_h]
        w_p = [[a.ctypes.data for a in row] for row in w_h]
        index = {id(rs): i for i, rs in enumerate(rsets)}
        call, pool = self.ctx.moe_forward_host_ptrs, self.pool

        def step(rs):
            si = index[id(rs)]
            ip, wp = ids_p[si], w_p[si]
            for l in range(self.layers):
                call(pool, l, xp, ip[l], wp[l], None, shs[l], sp, None, op, batch)
            return outs
        for i in range(warmup):
            step(rsets[i % len(rsets)])
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(steps):
            step(rsets[(warmup + i) % len(rsets)])
        torch.cuda.synchronize()
        return (time.perf_counter() - t0), h2d * self.layers, d2h * self.layers


# ------------------------------------------------------- expert-parallel layer
class EpBench:
    """The expert-parallel layer at any number of ranks (one rank: the same protocol, its exchanges are copies).
    Decode: 8 tokens per rank per step through ep_layer_static, one CUDA graph per routing set.  Prefill: 512
    tokens per rank per chunk through ep_layer (planned exchange)."""

    BATCH, N_SETS = 8, 4

    def __init__(self, stack, dist, rank, world, args):
        import torch

        from finchmoe_b200 import ep
        self.torch, self.ep, self.stack, self.dist, self.rank, self.world, self.args = torch, ep, stack, dist, rank, world, args
        self.backend = ep.GpuBackend(stack.ctx, stack.pool, max(self.BATCH, PREFILL_CHUNK) * world)
        self.backend.tc_mode = args.ep_prefill_mode
        self.score_val = 0.1
        self.graphs = None
        self.graphs_extra = None
        # decode: the exchange goes through the ranks' own kernels over peer memory unless told (or forced) otherwise
        self.exchange = "none (one rank)"
        if world > 1:
            self.exchange = "2 all-to-alls per layer over NCCL (records, partial rows)"
            if args.exchange == "peer":
                self.backend.peer = ep.PeerExchange.connect(stack.ctx, dist, None, self.BATCH)
                if self.backend.peer is not None:
                    self.exchange = "the ranks' own kernels over NVLink peer memory: stores into the peers' receive areas, one flag per slot, bounded waits"
                else:
                    self.exchange += " (the peer areas could not be mapped)"

    # ---- helpers
    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()

    def max_over_ranks(self, v: float) -> float:
        if self.dist is None:
            return v
        t = self.torch.tensor([v], device="cuda", dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(self, v: float) -> float:
        if self.dist is None:
            return v
        t = self.torch.tensor([v], device="cuda", dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return float(t.item())

    def gather_ints(self, v: int):
        if self.dist is None:
            return [int(v)]
        t = self.torch.zeros(self.world, device="cuda", dtype=self.torch.int64)
        t[self.rank] = int(v)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return [int(a) for a in t.cpu().tolist()]

    def timed(self, n, w0, fn):
        """w0 warm-up calls, then n timed: barrier and synchronize on both sides, one event per step, the total as
        the maximum over ranks.  Returns (seconds, [ms per step on this rank])."""
        torch = self.torch
        for i in range(w0):
            fn(i)
        torch.cuda.synchronize()
        self.barrier()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(n + 1)]
        ev[0].record()
        for i in range(n):
            fn(w0 + i)
            ev[i + 1].record()
        torch.cuda.synchronize()
        self.barrier()
        return self.max_over_ranks(ev[0].elapsed_time(ev[n]) / 1e3), [ev[i].elapsed_time(ev[i + 1]) for i in range(n)]

    # ---- decode
    def setup_decode(self):
        st, world, rank = self.stack, self.world, self.rank
        # every rank can regenerate every rank's routing (seeded), which is all the byte count needs
        self.all_sets = [routing_sets(self.BATCH, self.N_SETS, LAYERS, r) for r in range(world)]
        self.dev, self.xd, self.score, self.out, self.x = st.device_inputs(self.all_sets[rank], self.BATCH)
        self.shared = [st.ctx.make_shared(*st.shared[l], gate_score=self.score) for l in range(LAYERS)]

    def decode_layers(self, s):
        ids, w = self.dev[s]
        for l in range(LAYERS):
            self.ep.ep_layer_static(self.backend, self.dist, None, l, self.xd, ids[l], w[l], None, self.shared[l], None, self.out[l], in_scope=True)

    def decode_eager(self, i):
        with self.backend.stream_scope():
            self.decode_layers(i % self.N_SETS)

    def capture_decode(self):
        """One CUDA graph per routing set (kernels and all-to-alls).  Every rank must take the same path: a rank
        that replays graphs cannot pair with one that launches from the host."""
        torch = self.torch
        note = "launched from the host every step"
        graphs = None
        if not self.args.no_graph:
            try:
                for s in range(self.N_SETS):      # communicators, lazily made buffers and tables exist before capture
                    self.decode_eager(s)
                torch.cuda.synchronize()
                self.barrier()
                graphs = []
                for s in range(self.N_SETS):
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=self.backend.stream, capture_error_mode="thread_local"):
                        self.decode_layers(s)
                    graphs.append(g)
                    del g
                torch.cuda.synchronize()
                note = "one CUDA graph per routing set (kernels and all-to-alls)"
            except Exception as e:                # capture of the collectives unavailable: keep launching from the host
                graphs = None
                note = "launched from the host every step (graph capture failed: %s)" % (str(e).splitlines()[0][:120] if str(e) else type(e).__name__)
                torch.cuda.synchronize()
        ok = 1 if graphs is not None else 0
        if self.dist is not None:
            flag = torch.tensor([ok], device="cuda")
            self.dist.all_reduce(flag, op=self.dist.ReduceOp.MIN)
            ok = int(flag.item())
        self.graphs = graphs if ok else None
        return note

    def decode_step(self, i):
        if self.graphs is not None:
            self.graphs[i % self.N_SETS].replay()
        else:
            self.decode_eager(i)

    def decode_step_bytes(self, s):
        """Distinct experts touched by all ranks' tokens (each lives on one rank), plus every rank's copy of the
        shared expert."""
        total = 0
        for l in range(LAYERS):
            touched = set()
            for r in range(self.world):
                touched |= set(self.all_sets[r][s][l][0].ravel().tolist())
            total += len(touched) * EXPERT_BYTES + self.world * SHARED_BYTES
        return total

    def run_decode(self):
        args, torch = self.args, self.torch
        self.setup_decode()
        c0 = int(self.stack.ctx.launch_count())
        self.decode_eager(0)
        torch.cuda.synchronize()
        launches_per_step = int(self.stack.ctx.launch_count()) - c0      # graph replays do not pass the host counter
        note = self.capture_decode()
        secs, per_step = self.timed(args.steps, args.warmup, self.decode_step)
        # end to end: the step's inputs come from pinned host memory and its result goes back to the host
        xh = torch.from_numpy(self.stack.ctx.acts_to_wire(self.x).view(np.int16)).pin_memory()
        res = torch.empty((self.BATCH, HIDDEN), dtype=torch.float32).pin_memory()

        def step_e2e(i):
            self.xd.view(torch.int16).copy_(xh, non_blocking=True)
            self.decode_step(i)
            res.copy_(self.out[LAYERS - 1], non_blocking=True)
            torch.cuda.current_stream().synchronize()
        e2e_w = max(3, args.warmup)
        e2e_secs, _ = self.timed(args.steps, e2e_w, step_e2e)
        timed_bytes = sum(self.decode_step_bytes((args.warmup + i) % self.N_SETS) for i in range(args.steps))
        e2e_bytes = sum(self.decode_step_bytes((e2e_w + i) % self.N_SETS) for i in range(args.steps))
        rec = self.backend.record_bytes()
        link_bytes = (self.world - 1) * self.BATCH * (rec + HIDDEN * 4) * LAYERS       # sent by one rank per step (it receives as much)
        return {"launches_per_step": launches_per_step, "secs": secs, "per_step": per_step, "e2e_secs": e2e_secs, "bytes": timed_bytes, "e2e_bytes": e2e_bytes, "note": note,
                "h2d": int(xh.numel() * 2 * self.world), "d2h": int(res.numel() * 4 * self.world),
                "tokens_per_s": self.BATCH * self.world * args.steps / secs, "us_per_layer": secs / args.steps / LAYERS * 1e6,
                "nvlink_gbs_per_gpu_per_direction": link_bytes * args.steps / secs / 1e9 if self.world > 1 else 0.0,
                "link_bytes_per_gpu_per_step": link_bytes if self.world > 1 else 0}

    # ---- prefill
    def run_prefill(self, steps, warmup):
        torch, st, T = self.torch, self.stack, PREFILL_CHUNK
        rs = routing_sets(T, 1, LAYERS, self.rank)[0]
        ids = torch.from_numpy(np.stack([r[0] for r in rs])).cuda()
        w = torch.from_numpy(np.stack([r[1] for r in rs])).cuda()
        x = synth.activations(synth.rng_for(2, 0, 9 + 1000 * self.rank), T, HIDDEN)
        xd = torch.from_numpy(x).cuda().to(torch.bfloat16)
        score = torch.full((T,), self.score_val, device="cuda")
        out = torch.empty((2, T, HIDDEN), device="cuda")
        shared = [st.ctx.make_shared(*st.shared[l], gate_score=score) for l in range(LAYERS)]
        self.pf = (rs, ids, w, x, xd, score, shared)
        self.backend.stats = []

        fixed = self.args.ep_prefill_exchange == "fixed" and self.world > 1
        layer_fn = self.ep.ep_layer_static if fixed else self.ep.ep_layer
        self.pf_layer = layer_fn

        def layers(in_scope):
            for l in range(LAYERS):
                if fixed:
                    layer_fn(self.backend, self.dist, None, l, xd, ids[l], w[l], None, shared[l], None, out[l & 1], in_scope=in_scope)
                else:
                    layer_fn(self.backend, self.dist, None, l, xd, ids[l], w[l], None, shared[l], None, out[l & 1])

        def eager(_):
            if fixed:
                with self.backend.stream_scope():
                    layers(True)
            else:
                layers(False)
        step, launch = eager, "launched from the host every step"
        if fixed and not self.args.no_graph:
            # the fixed-capacity layer has no host step: the chunk's 40 layers (kernels and all-to-alls) replay from one CUDA graph
            g, ok = None, 1
            try:
                eager(0)                              # workspaces, attributes and communicators exist before capture
                torch.cuda.synchronize()
                self.barrier()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=self.backend.stream, capture_error_mode="thread_local"):
                    layers(True)
                torch.cuda.synchronize()
            except Exception:
                g, ok = None, 0
                torch.cuda.synchronize()
            flag = torch.tensor([ok], device="cuda")
            self.dist.all_reduce(flag, op=self.dist.ReduceOp.MIN)
            if int(flag.item()) == 1:
                self.graphs_extra = g                 # released with the others, no other name holds it
                step, launch = (lambda _: self.graphs_extra.replay()), "one CUDA graph per chunk (kernels and all-to-alls)"
            del g
        secs, per_step = self.timed(steps, warmup, step)
        stats, self.backend.stats = self.backend.stats, None
        if fixed:       # every token to every rank
            rows_sent, rows_recv = T * (self.world - 1) * LAYERS, T * self.world * LAYERS
        else:
            per_call = stats[-LAYERS:]                                   # the last step's layers
            rows_sent = sum(sum(c for d, c in enumerate(cs) if d != self.rank) for cs, _ in per_call)
            rows_recv = sum(sum(cr) for _, cr in per_call)
        rec = self.backend.record_bytes()
        pairs_local = sum(int(((r[0] // (NEXP // self.world)) == self.rank).sum()) for r in rs)   # of this rank's own tokens
        link = rows_sent * (rec + HIDDEN * 4)
        return {"exchange": "fixed capacity (every token to every rank: two all-to-alls with equal splits, no host synchronisation)" if fixed
                else "planned (a token goes where it has an expert; row counts exchanged first, one host synchronisation per layer)",
                "launch": launch,
                "chunk_tokens_per_gpu": T, "tokens_per_step": T * self.world, "steps": steps, "ms_per_step": secs / steps * 1e3,
                "step_ms": spread(per_step), "tokens_per_s": T * self.world * steps / secs,
                "rows_received_per_gpu_per_step": self.gather_ints(rows_recv),
                "rows_sent_per_gpu_per_step": self.gather_ints(rows_sent),
                "nvlink_gbs_per_gpu_per_direction": self.max_over_ranks(link * steps / secs / 1e9) if self.world > 1 else 0.0,
                "own_pairs_on_own_experts": self.gather_ints(pairs_local)}

    # ---- parity of what was timed
    def parity(self):
        """Layer 0 of routing set 0 (decode) and of the prefill chunk, as the expert-parallel layer computed them
        for this rank's tokens, against the one-GPU entry point on a pool that holds all 256 experts of that
        layer (the same synthetic contents).  The worst figures over the ranks are reported."""
        torch, st, ctx = self.torch, self.stack, self.stack.ctx
        full = ctx.pool(n_layers=1)
        full.fill_synthetic(0, 1, st.seed)
        res = {}
        try:
            ids, w = self.dev[0]
            with self.backend.stream_scope():
                self.ep.ep_layer_static(self.backend, self.dist, None, 0, self.xd, ids[0], w[0], None, self.shared[0], None, self.out[0], in_scope=True)
            torch.cuda.synchronize()
            got = self.out[0].cpu().numpy()
            want_d = torch.empty_like(self.out[0])
            ctx.encode_moe_decode(full, 0, self.xd, ids[0], w[0], None, self.shared[0], None, want_d, self.BATCH)
            torch.cuda.synchronize()
            res["decode"] = cos_and_rel(got, want_d.cpu().numpy())
            rs, pids, pw, x, xd, score, shared = self.pf
            T = PREFILL_CHUNK
            out = torch.empty((T, HIDDEN), device="cuda")
            self.pf_layer(self.backend, self.dist, None, 0, xd, pids[0], pw[0], None, shared[0], None, out)
            torch.cuda.synchronize()
            want_p = torch.empty_like(out)
            ctx.set_prefill_mode(1)            # the exact sub-batch path: the decode kernels, 8 tokens at a time
            ctx.encode_moe_decode(full, 0, xd, pids[0], pw[0], None, shared[0], None, want_p, T, prefill=True)
            ctx.set_prefill_mode(0)
            torch.cuda.synchronize()
            res["prefill"] = cos_and_rel(out.cpu().numpy(), want_p.cpu().numpy())
        finally:
            full.destroy()
        status = int(ctx.device_status())
        worst = {}
        for k, v in res.items():
            worst[k] = {"cos": -self.max_over_ranks(-v["cos"]), "max_rel": self.max_over_ranks(v["max_rel"]),
                        "finite": self.max_over_ranks(0.0 if v["finite"] else 1.0) == 0.0}
        worst["device_status"] = int(self.max_over_ranks(float(abs(status))))
        worst["against"] = "finch_encode_moe_decode on a rank-local pool holding all 256 experts of layer 0 (prefill rows: its sub-batch path)"
        worst["ok"] = bool(worst["device_status"] == 0 and all(worst[k]["finite"] and worst[k]["cos"] >= 0.99999 and worst[k]["max_rel"] <= 1e-3
                                                                for k in ("decode", "prefill")))
        return worst

    # ---- the exchanges alone
    def time_exchanges(self, reps=5):
        """The exchange of a decode layer with nothing between its steps, 40 layers per CUDA graph: what it costs alone.
        Through peer memory: dispatch, receive, return, combine; over NCCL: the two all-to-alls."""
        if self.world == 1:
            return None
        torch, dist = self.torch, self.dist
        n = self.BATCH * self.world
        be = self.backend
        if be.peer is not None:
            ids, w = self.dev[0]
            what = "dispatch, receive, return and combine kernels of every layer, nothing else"

            def pairs():
                for _ in range(LAYERS):
                    be.peer_dispatch(self.xd, ids[0], w[0], None)
                    be.peer_receive(False)
                    be.peer_return(be.rout)
                    be.peer_combine(self.out[0])
        else:
            a = torch.zeros(n * self.backend.record_bytes(), dtype=torch.uint8, device="cuda")
            b = torch.empty_like(a)
            c = torch.zeros(n * HIDDEN, dtype=torch.float32, device="cuda")
            d = torch.empty_like(c)
            what = "two all_to_all_single per layer (records out, fp32 rows back), nothing else"

            def pairs():
                for _ in range(LAYERS):
                    dist.all_to_all_single(b, a)
                    dist.all_to_all_single(d, c)
        run = None
        if self.graphs is not None:
            try:
                with self.backend.stream_scope():
                    pairs()
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=self.backend.stream, capture_error_mode="thread_local"):
                    pairs()
                self.graphs.append(g)      # released with the others
                run = g.replay
                del g
            except Exception:
                run = None
        ok = 1 if run is not None else 0
        flag = torch.tensor([ok], device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if int(flag.item()) == 0:
            def run():
                with self.backend.stream_scope():
                    pairs()
        secs, _ = self.timed(reps, 2, lambda i: run())
        return {"us_per_layer": secs / reps / LAYERS * 1e6, "what": what}

    def release(self):
        self.graphs = None
        self.graphs_extra = None
        gc.collect()


def run_ours(args):
    import torch
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
        return run_ep(args, rank, local_rank, world, dist)
    batch = 8
    stack = Stack(local_rank, max_tokens=PREFILL_CHUNK, layers=LAYERS)
    n_sets = 4
    rsets = routing_sets(batch, n_sets)
    dev, xd, score, out, x = stack.device_inputs(rsets, batch)

    sampler = ClockSampler(local_rank)
    secs, per_step = stack.time_steps(dev, xd, score, out, batch, args.steps, args.warmup, use_graph=not args.no_graph)
    launches = KERNELS_PER_LAYER * LAYERS * args.steps  # graph replays launch them without passing the host counter
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
        "ms_per_step": secs / args.steps * 1e3, "step_ms": spread(per_step), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "C2: 40-layer 3-bit expert stack decode, batch 8, top-8 of 256, Zipf(1.1)", "batch": batch,
                   "layers": LAYERS, "layers_per_step": LAYERS, "hidden": HIDDEN, "moe_inter": INTER, "scale_dtype": "fp16", "act_dtype": "bf16",
                   "pool_gb": LAYERS * NEXP * EXPERT_BYTES / 1e9, "parallelism": "1 GPU",
                   "l2": "inputs larger than L2: every step streams >= 0.5 GB of a 14 GB pool; 4 routing sets rotate"},
        "clocks": clocks,
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "tokens_per_s": batch * args.steps / secs,
        "us_per_layer": secs / args.steps / LAYERS * 1e6,
        "hbm_frac_of_" + peak_kind: value / peaks["hbm_gbs"],
    }

    # batch 1 (single-stream decode) on the same pool
    r1 = routing_sets(1, n_sets)
    dev1, xd1, score1, out1, _ = stack.device_inputs(r1, 1)
    s1, per1 = stack.time_steps(dev1, xd1, score1, out1, 1, args.steps, args.warmup, use_graph=not args.no_graph)
    b1 = sum(sum(alg_bytes(ids) for ids, _ in r1[(args.warmup + i) % n_sets]) for i in range(args.steps))
    line["batch1"] = {"value": b1 / s1 / 1e9, "unit": "GB/s", "ms_per_step": s1 / args.steps * 1e3, "step_ms": spread(per1),
                      "us_per_layer": s1 / args.steps / LAYERS * 1e6, "tokens_per_s": args.steps / s1,
                      "frac_of_" + peak_kind: b1 / s1 / 1e9 / peaks["hbm_gbs"]}
    # per-kernel roofline of the dominant kernel (gate/up/SiLU)
    line["roofline"] = kernel_roofline(stack, dev, rsets, xd, score, out, batch, args, peaks, peak_kind)
    # chunked prefill: 512-token chunks through the grouped dequant-GEMM (tcgen05), the whole stack
    T = PREFILL_CHUNK
    pf_steps = max(3, args.steps // 8)
    ps, uniq = stack.time_prefill(T, pf_steps, 2)
    flops = LAYERS * (T * TOPK * 6291456 + T * 3 * 2 * 512 * HIDDEN)
    pbytes = uniq * EXPERT_BYTES + LAYERS * SHARED_BYTES
    ai = flops / pbytes
    ceil_tf = min(peaks["bf16_tflops_sustained"], ai * peaks["hbm_gbs"] / 1e3)
    line["prefill"] = {"metric": "moe3_prefill_tokens_per_s", "chunk": T, "value": T / ps, "unit": "tokens/s (40 MoE layers per token)",
                       "ms_per_chunk": ps * 1e3, "tflops": flops / ps / 1e12, "hbm_gbs": pbytes / ps / 1e9,
                       "roofline": {"bound": "hbm", "note": "8T/256 pairs per expert: below the tensor ridge", "ceiling_tflops": ceil_tf,
                                    "frac": flops / ps / 1e12 / ceil_tf, "peak_kind": peak_kind}}
    # the expert-parallel layer run by one rank: the code path of --gpus N with its exchanges as copies
    epb = EpBench(stack, None, 0, 1, args)
    d = epb.run_decode()
    p = epb.run_prefill(pf_steps, 2)
    line["ep"] = {"n_gpus": 1, "decode": {"tokens_per_step": epb.BATCH, "tokens_per_s": d["tokens_per_s"], "us_per_layer": d["us_per_layer"],
                                          "step_ms": spread(d["per_step"]), "launch": d["note"]},
                  "prefill": p, "ep_parity": epb.parity()}
    epb.release()
    line["other_rows"] = aux_rooflines(stack, peaks, peak_kind)
    # CPU baseline: a bounded sample of the same workload, all host threads
    cores = os.cpu_count() or 1
    cpu = CpuExpertPath()
    sample = rsets[0][:2]
    dt, nb = cpu.time_layers(sample, batch, min(cores, 64))
    line["cpu_baseline"] = {"value": nb / dt / 1e9, "unit": "GB/s", "cores": min(cores, 64), "kind": cpu.kind,
                            "sample": f"2 of {LAYERS} layers, batch {batch}, routed experts, one (token, expert) pair per task", "seconds": dt}
    print(json.dumps(line))


def run_ep(args, rank, local_rank, world, dist):
    """N > 1: the layer is expert parallel.  Every rank owns 8 tokens per decode step and 512 tokens per prefill
    chunk (weak scaling) and the contiguous block of 256 / N experts of every layer; per layer the ranks exchange
    activation rows and partial outputs (finchmoe_b200/ep.py).  value = bytes of the distinct experts the ranks
    stream per decode step (plus every rank's copy of the shared expert) per second of the slowest rank."""
    import torch
    stack = Stack(local_rank, max_tokens=PREFILL_CHUNK * world, layers=LAYERS, shard=(rank, world))
    epb = EpBench(stack, dist, rank, world, args)
    sampler = ClockSampler(local_rank) if rank == 0 else None
    d = epb.run_decode()
    clocks = sampler.stop() if sampler else None
    p = epb.run_prefill(max(3, args.steps // 8), 2)
    parity = epb.parity()
    exch = epb.time_exchanges()
    status = int(stack.ctx.device_status())
    if rank == 0:
        peaks, peak_kind = measured_peaks()
        secs = d["secs"]
        value = d["bytes"] / secs / 1e9
        per = NEXP // world
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": secs / args.steps * 1e3, "step_ms": spread(d["per_step"]), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "C5: expert-parallel batched decode, 40 layers, 8 tokens per GPU per step, top-8 of 256, Zipf(1.1) (one popularity per layer for all ranks)",
                       "batch": epb.BATCH * world, "layers": LAYERS, "layers_per_step": LAYERS, "hidden": HIDDEN, "moe_inter": INTER,
                       "scale_dtype": "fp16", "act_dtype": "bf16", "pool_gb": LAYERS * NEXP * EXPERT_BYTES / 1e9, "experts_per_gpu": per,
                       "parallelism": f"ep{world}",
                       "exchange": "fixed capacity, no host synchronisation: " + epb.exchange,
                       "launch": d["note"],
                       "l2": "inputs larger than L2: the pool shards exceed it; 4 routing sets rotate"},
            "clocks": clocks,
            "e2e": {"value": d["e2e_bytes"] / d["e2e_secs"] / 1e9, "unit": "GB/s", "h2d_bytes_per_step": d["h2d"], "d2h_bytes_per_step": d["d2h"]},
            "gpu_launches": d["launches_per_step"] * args.steps * world,
            "tokens_per_s": d["tokens_per_s"],
            "us_per_layer": d["us_per_layer"],
            "decode": {"tokens_per_step": epb.BATCH * world, "tokens_per_gpu_per_step": epb.BATCH, "tokens_per_s": d["tokens_per_s"],
                       "us_per_layer": d["us_per_layer"], "nvlink_gbs_per_gpu_per_direction": d["nvlink_gbs_per_gpu_per_direction"],
                       "link_bytes_per_gpu_per_step": d["link_bytes_per_gpu_per_step"], "exchange_alone": exch},
            "prefill": dict(p, metric="moe3_prefill_tokens_per_s", value=p["tokens_per_s"], unit="tokens/s (40 MoE layers per token)"),
            "ep_parity": parity,
            "device_status": status,
            "hbm_frac_of_" + peak_kind: value / world / peaks["hbm_gbs"],
        }
        print(json.dumps(line), flush=True)
    # The graphs hold the recorded all-to-alls.  NCCL keeps a communicator alive while a graph that captured its
    # collectives exists (destroying it waits for those graphs to be released), so the graphs go first and no name
    # may still hold one; the process then leaves without tearing the process group down.
    epb.release()
    torch.cuda.synchronize()
    dist.barrier()
    sys.stdout.flush()
    sys.stderr.flush()
    os._exit(0)


def aux_rooflines(stack, peaks, peak_kind, iters=8):
    """The other matvec rows of the path, each timed alone with CUDA events and the L2 flushed (a 256 MB
    write) before every timed launch: 4-bit g64 projections and GGUF Q4_K / Q6_K tensors through
    finch_encode_batch_matvec at 1 / 8 (/ 90) positions, the 4-bit projections at 64 / 512 positions
    through the tensor-core GEMM, and the 248,320-row output projection in 8 and 4 bits (larger than L2 by
    itself: no flush, which would leave dirty lines to be written back under the timed launch).
    bytes = packed weights + scales (+ activations); flops = 2 T out in."""
    import ctypes as C

    import torch
    ctx, L = stack.ctx, stack.L
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    rng = synth.rng_for(4, 0, 99)
    st = stack.stream
    rows = []

    def timed(fn, do_flush=True):
        fn()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(iters):
            with torch.cuda.stream(st):
                if do_flush:
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
    rows += lm_head_rows(stack, peaks, peak_kind, timed)
    rows += gguf_expert_rows(stack, peaks, peak_kind, timed)
    return rows


def gguf_expert_rows(stack, peaks, peak_kind, timed):
    """The GGUF expert MLP (Q4_K gate / up, Q6_K down: the Q4_K_M mix) of a 90-token prefill chunk and of one decode
    token at the model's size, from stacked slabs of all 256 experts (device-generated codes, |N(0, 0.01)| block
    scales).  bytes = the distinct selected experts' slabs."""
    import torch
    ctx, L, st = stack.ctx, stack.L, stack.stream
    rng = synth.rng_for(4, 0, 97)

    def slab(rows, cols, block, d_at, n_d):
        nb = cols // 256
        W = torch.randint(0, 256, (NEXP, rows, nb, block), dtype=torch.uint8, device="cuda")
        d = (torch.randn((NEXP, rows, nb, n_d), device="cuda").abs() * 0.01).to(torch.float16)
        W[..., d_at:d_at + 2 * n_d] = d.view(torch.uint8).reshape(NEXP, rows, nb, 2 * n_d)
        return W
    gate, up, down = slab(INTER, HIDDEN, 144, 0, 2), slab(INTER, HIDDEN, 144, 0, 2), slab(HIDDEN, INTER, 210, 208, 1)
    ge = L.GgufExperts(gate.data_ptr(), up.data_ptr(), down.data_ptr(), gate[0].numel(), up[0].numel(), down[0].numel(), 10, 10, 11)
    per_expert = gate[0].numel() + up[0].numel() + down[0].numel()
    rows = []
    perm = layer_popularity(0)
    for T in (1, 90):
        ids, w = synth.zipf_routing_shared(rng, T, perm, TOPK)
        x = torch.from_numpy(synth.activations(rng, T, HIDDEN)).cuda().to(torch.bfloat16)
        idd, wd = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
        out = torch.empty((T, HIDDEN), dtype=torch.float32, device="cuda")
        secs = timed(lambda: ctx.encode_moe_gguf(ge, x, idd, wd, None, None, out, T, stream=st.cuda_stream))
        b = len(set(ids.ravel().tolist())) * per_expert
        rows.append({"op": "gguf_expert_mlp_q4k_q4k_q6k", "T": T, "distinct_experts": len(set(ids.ravel().tolist())), "us": secs * 1e6, "gbs": b / secs / 1e9,
                     "path": "grouped by expert, one pass per expert" if T >= 9 else "token by token", "frac_hbm_" + peak_kind: b / secs / 1e9 / peaks["hbm_gbs"]})
    del gate, up, down
    return rows


def lm_head_rows(stack, peaks, peak_kind, timed=None, iters=8):
    """The output projection (lm_head tier): 248,320 rows of 2048 in 8 and 4 bits, device-generated bytes, one
    position.  The tensor is larger than L2 by itself, so nothing is flushed between the timed launches."""
    import torch
    ctx, L, st = stack.ctx, stack.L, stack.stream
    rng = synth.rng_for(4, 0, 98)
    if timed is None:
        def timed(fn, do_flush=True):
            fn()
            torch.cuda.synchronize()
            tot = 0.0
            for _ in range(iters):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(st):
                    e0.record(st)
                    fn()
                    e1.record(st)
                torch.cuda.synchronize()
                tot += e0.elapsed_time(e1)
            return tot / iters * 1e-3
    rows = []
    rows_out, in_dim = 248320, 2048
    for bits in (8, 4):
        Wd = torch.randint(0, 256, (rows_out, in_dim * bits // 8), dtype=torch.uint8, device="cuda")
        Sd = (torch.rand((rows_out, in_dim // 64), device="cuda") * 0.01 + 1e-4).to(torch.float16)
        Bd = (Sd.float() * -(128.0 if bits == 8 else 8.0)).to(torch.float16)
        w = L.WDesc(Wd.data_ptr(), Sd.data_ptr(), Bd.data_ptr(), rows_out, in_dim, 64, bits, L.FP16)
        x = torch.from_numpy(synth.activations(rng, 1, in_dim)).cuda().to(torch.bfloat16)
        out = torch.empty((1, rows_out), dtype=torch.float32, device="cuda")
        secs = timed(lambda: ctx.fast_batch_matvec(x, L.BF16, [w], [out], M=1, stream=st.cuda_stream), do_flush=False)
        b = Wd.numel() + Sd.numel() * 2 + Bd.numel() * 2 + in_dim * 2 + rows_out * 4
        rows.append({"op": f"lm_head_matvec_{bits}bit_g64", "shape": [rows_out, in_dim], "T": 1, "us": secs * 1e6, "gbs": b / secs / 1e9,
                     "bytes": int(b), "frac_hbm_" + peak_kind: b / secs / 1e9 / peaks["hbm_gbs"]})
        del Wd, Sd, Bd
    # the same projection as GGUF K-quants (the tier a GGUF model's output tensor uses): 256-value blocks, uniform bytes,
    # block scales d (and dmin) = 0.003 as fp16
    import numpy as _np
    lo, hi = (int(v) for v in _np.array([0.003], _np.float16).view(_np.uint8))
    for name, bs, bits, dpos in (("q6_k", 210, 11, (208,)), ("q4_k", 144, 10, (0, 2))):
        nb = in_dim // 256
        Wd = torch.randint(0, 256, (rows_out * nb, bs), dtype=torch.uint8, device="cuda")
        for o in dpos:
            Wd[:, o] = lo
            Wd[:, o + 1] = hi
        w = L.WDesc(Wd.data_ptr(), None, None, rows_out, in_dim, 256, bits, L.FP16)
        x = torch.from_numpy(synth.activations(rng, 1, in_dim)).cuda().to(torch.bfloat16)
        out = torch.empty((1, rows_out), dtype=torch.float32, device="cuda")
        secs = timed(lambda: ctx.fast_batch_matvec(x, L.BF16, [w], [out], M=1, stream=st.cuda_stream), do_flush=False)
        b = Wd.numel() + in_dim * 2 + rows_out * 4
        rows.append({"op": f"lm_head_matvec_{name}", "shape": [rows_out, in_dim], "T": 1, "us": secs * 1e6, "gbs": b / secs / 1e9,
                     "bytes": int(b), "frac_hbm_" + peak_kind: b / secs / 1e9 / peaks["hbm_gbs"]})
        del Wd
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
    ratio, src = profiled_traffic_ratio()
    return {"bound": "hbm", "kernel": "moe_gateup_kernel", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / peaks["hbm_gbs"], "peak_kind": peak_kind,
            # DRAM bytes of one profiled launch over its algorithmic bytes, applied to this run's average launch
            "traffic": per_launch_bytes * ratio if ratio else None, "traffic_source": src,
            "bytes_per_launch": per_launch_bytes, "us_per_launch": ms_a.value / n.value * 1e3,
            "down_combine_us_per_launch": ms_b.value / n.value * 1e3, "launches_timed": n.value}


def main():
    global LAYERS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=LAYERS, help="fewer layers = a small case for profiler captures")
    ap.add_argument("--no-graph", action="store_true", help="launch from the host every step instead of replaying CUDA graphs")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"], help="N > 1, decode: the ranks' own kernels over peer memory, or NCCL all-to-alls")
    ap.add_argument("--ep-prefill-mode", type=int, default=0, choices=[0, 2, 3],
                    help="N > 1, prefill: the received rows through the tcgen05 grouped GEMMs (2), the grouped mma.sync passes (3), or by tokens per expert (0)")
    ap.add_argument("--ep-prefill-exchange", default="fixed", choices=["fixed", "planned"],
                    help="N > 1, prefill: every token to every rank with equal splits and no host step, or the planned exchange")
    ap.add_argument("--prefill-mode", type=int, default=0, choices=[0, 1, 2, 3, 4],
                    help="with --only prefill: which kernels take the routed experts of a chunk (0: the library's choice)")
    ap.add_argument("--only", default="", choices=["", "prefill", "decode", "lmhead"],
                    help="just the 512-token chunk, just the batch-8 decode steps (both on --layers layers), or just the output-projection matvecs (profiler captures)")
    args = ap.parse_args()
    LAYERS = args.layers
    if args.only == "prefill":
        stack = Stack(0, max_tokens=PREFILL_CHUNK, layers=LAYERS)
        stack.ctx.set_prefill_mode(args.prefill_mode)
        ps, uniq = stack.time_prefill(PREFILL_CHUNK, max(1, args.steps), max(1, args.warmup))
        print(json.dumps({"only": "prefill", "chunk": PREFILL_CHUNK, "layers": LAYERS, "ms_per_chunk": ps * 1e3, "tokens_per_s": PREFILL_CHUNK / ps,
                          "distinct_experts": uniq, "status": stack.ctx.device_status()}))
    elif args.only == "decode":
        stack = Stack(0, max_tokens=8, layers=LAYERS)
        rsets = routing_sets(8, 4)
        dev, xd, score, out, _ = stack.device_inputs(rsets, 8)
        secs, per_step = stack.time_steps(dev, xd, score, out, 8, args.steps, args.warmup, use_graph=not args.no_graph)
        print(json.dumps({"only": "decode", "layers": LAYERS, "ms_per_step": secs / args.steps * 1e3, "step_ms": spread(per_step),
                          "status": stack.ctx.device_status()}))
    elif args.only == "lmhead":
        stack = Stack(0, max_tokens=8, layers=1)
        peaks, peak_kind = measured_peaks()
        print(json.dumps({"only": "lmhead", "rows": lm_head_rows(stack, peaks, peak_kind, iters=max(1, args.steps)), "status": stack.ctx.device_status()}))
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
