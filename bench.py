#!/usr/bin/env python
"""Benchmark of the B200 nomic-bert encoder (BASELINE.json metric:
"embeddings/s at seq128 on 1/2/4/8 B200; p50 batch-1 8-token latency").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--sections headline,latency,configs,sweep,load,tokenizer]

Headline workload: BASELINE.json configs[2], one batch of 256 sequences
(lengths U[16, 128], seed 1, packed without padding) on the Q8_0 random-init
12-layer model.  With N GPUs (torchrun, one process per GPU) the one batch is
sharded: rank r embeds the contiguous, work-balanced shard
llm_embed_b200.dist.local_shard gives it, on its own replica (no data-path
collective; strong scaling, as configs[2] states "1 GPU then batch-sharded
across 2/4/8 GPUs").  The timed region is bracketed by a barrier and a
synchronize; times are the max over ranks.  Rank 0 prints one JSON line.

  value     embeddings/s of the whole batch: 256 * K / (max over ranks of the
            CUDA-event time of K steps on the launching stream), inputs
            resident in HBM, L2 flushed between steps (outside the events).
  e2e       the same through the public host API (Embedder.EmbedIDs): host
            ids in, host embeddings out, copies inside the timed region.
  roofline  the kernel class with the largest device time, against the
            measured burst peak (kernels timed inside a sub-second region
            run at full clock); `roofline_classes` gives every class as
            achieved / max(FLOP floor, byte floor).  Per-class device times
            come from a second pass with CUDA events around every launch.
  cpu_baseline  the CPU restatement of the reference (oracle/, test
            infrastructure) on this host's cores, rank 0, N=1.

Extra keys: weak scaling (N>1: each rank its own 256-sequence batch),
the optional NCCL all-gather of the embeddings (N>1, outside the timed step),
per-rank shard sizes and kernel times, configs[3] and configs[4] at their
stated sizes (sharded the same way), the configs[1] op sweep (N=1), model
load phases (f2) and host tokenizer throughput (f1).

--impl reference times the reference path's CPU restatement alone (the Go
reference cannot be built: no Go toolchain in the image).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from llm_embed_b200 import dist as ldist  # noqa: E402
from llm_embed_b200 import synth  # noqa: E402

METRIC = "embeddings/s at seq128 on 1/2/4/8 B200; p50 batch-1 8-token latency"
H, F, LAYERS = 768, 3072, 12
GEMM_FLOP_PER_TOKEN = 226492416.0
ALL_SECTIONS = ("headline", "latency", "configs", "sweep", "load", "tokenizer")
# Bytes per weight of each GGUF block type.
BPE = {synth.GGML_F32: 4.0, synth.GGML_Q8_0: 34 / 32, synth.GGML_Q4_K: 144 / 256, synth.GGML_Q5_K: 176 / 256,
       synth.GGML_Q6_K: 210 / 256}
EMB_ROW_BYTES = {synth.GGML_Q8_0: 816, synth.GGML_Q4_K: 432, synth.GGML_Q5_K: 528, synth.GGML_Q6_K: 630,
                 synth.GGML_F32: 3072}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm": p["hbm_gbs"], "tf": p["bf16_tflops"], "tf_sust": p["bf16_tflops_sustained"],
                "src": "measured"}
    except Exception:  # noqa: BLE001
        return {"hbm": 6650.0, "tf": 1590.0, "tf_sust": 1400.0, "src": "fallback"}


class Clocks:
    """nvidia-smi sampling of one GPU during a timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: int):
        self.dev = dev
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.dev)], stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except Exception:  # noqa: BLE001
            self.proc = None
        time.sleep(0.3)  # first sample before the timed work starts

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) == 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        num = lambda v: v.replace(".", "").isdigit()  # noqa: E731
        sm = [float(r[1]) for r in rows if num(r[1])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if num(rows[0][2]) else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max((float(r[3]) for r in rows if num(r[3])), default=None)}


# ------------------------------------------------------------- CPU arm -----

def time_oracle(path, ids, offs, n, threads, reps=1):
    """The CPU restatement (oracle/, test infrastructure) on the first n
    sequences, all of them in one call per rep: `threads` workers take one
    sequence at a time (dynamic schedule), each sequence's GEMMs on its own
    worker.  Returns seconds per rep."""
    import oracle
    m = oracle.Model(path)
    try:
        sub_ids, sub_offs = ids[:offs[n]], offs[:n + 1]
        t0 = time.perf_counter()
        for _ in range(reps):
            m.embed_ids(sub_ids, sub_offs, nthreads=threads)
        return (time.perf_counter() - t0) / reps
    finally:
        m.close()


WORKERS = ("{t} host threads, one sequence per worker at a time, GEMMs single-threaded inside a sequence (the "
           "reference runs <= 8 batch workers x <= 8 GEMM workers, embedder.go:95-97, ops_fast.go:217-226); "
           "C++ restatement of the Go reference (no Go toolchain to build the reference)")


def cpu_sample_size(path, ids, offs, threads, budget_s):
    """Sequences that take about budget_s on the CPU arm (calibrated)."""
    n_cal = min(offs.size - 1, max(threads, 16))
    per_seq = time_oracle(path, ids, offs, n_cal, threads) / n_cal
    return int(min(offs.size - 1, max(n_cal, budget_s / per_seq)))


def cpu_baseline(path, ids, offs, budget_s=12.0):
    threads = os.cpu_count() or 1
    n = cpu_sample_size(path, ids, offs, threads, budget_s)
    dt = time_oracle(path, ids, offs, n, threads)
    return {"value": n / dt, "unit": "embeddings/s", "cores": threads, "kind": "port",
            "sample": f"first {n} of {offs.size - 1} configs[2] sequences ({int(offs[n])} tokens) in one call, "
                      f"{dt:.1f} s; " + WORKERS.format(t=threads)}


def run_reference(args, rank):
    if rank != 0:
        return
    path = synth.cached_model("q8_0")
    ids, offs = synth.config_inputs(2)
    threads = os.cpu_count() or 1
    total_steps = args.steps + args.warmup
    n = cpu_sample_size(path, ids, offs, threads, 150.0 / total_steps)
    for _ in range(args.warmup):
        time_oracle(path, ids, offs, n, threads)
    dt = time_oracle(path, ids, offs, n, threads, reps=args.steps)
    v = n / dt
    sample = f"first {n} of 256 configs[2] sequences ({int(offs[n])} tokens) per step; " + WORKERS.format(t=threads)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "embeddings/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "configs[2] sample: Q8_0 nomic-bert, 12 layers, L~U[16,128]", "sequences_per_step": n},
        "cpu_baseline": {"value": v, "unit": "embeddings/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "embeddings/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ------------------------------------------------------------- work model --

LAYER_CLASSES = ("gemm_qkv", "gemm_attn_out", "gemm_ffn_upgate", "gemm_ffn_down", "attention", "layernorm")


def class_work(cls, T, nseq, sum_l2, wtypes, emb_type):
    """(FLOP, bytes) of kernel class `cls` for one device call of T valid
    tokens: per layer for the layer classes (LAYER_CLASSES; the attention
    class counts all its launches of a layer together), per call for the
    others.  Algorithmic: valid tokens only, weights at their GGUF size,
    each activation read or written once.  wtypes: GGUF types of (qkv, out,
    up/gate, down)."""
    fused = T >= 256  # the out and down projections carry the residual LayerNorm
    wb = lambda n, k, t: n * k * BPE[t]  # noqa: E731
    if cls == "gemm_qkv":
        return 2.0 * T * 3 * H * H, T * H * 2 + T * 3 * H * 2 + wb(3 * H, H, wtypes[0])
    if cls == "gemm_attn_out":
        io = T * H * 2 + (T * H * 10 if fused else T * H * 4)
        return 2.0 * T * H * H, io + wb(H, H, wtypes[1])
    if cls == "gemm_ffn_upgate":
        return 2.0 * T * 2 * F * H, T * H * 2 + T * F * 2 + wb(2 * F, H, wtypes[2])
    if cls == "gemm_ffn_down":
        io = T * F * 2 + (T * H * 10 if fused else T * H * 4)
        return 2.0 * T * H * F, io + wb(H, F, wtypes[3])
    if cls == "attention":
        return 4.0 * H * sum_l2, T * 3 * H * 2 + T * H * 2
    if cls == "layernorm":
        return 0.0, T * H * 14
    if cls == "embed_ln":
        return 0.0, T * (EMB_ROW_BYTES.get(emb_type, 816) + 4 + H * 6)
    if cls == "positions_pool":
        return 0.0, T * H * 4 + nseq * H * 4
    if cls == "fused_small":
        wbytes = sum(wb(n, k, t) for (n, k), t in zip(((3 * H, H), (H, H), (2 * F, H), (H, F)), wtypes)) * LAYERS
        return GEMM_FLOP_PER_TOKEN * T + 36864.0 * sum_l2, wbytes + T * EMB_ROW_BYTES.get(emb_type, 816)
    return 0.0, 0.0


def class_roofline(stats, calls, wtypes, emb_type, pk, sm_mhz=None, steps=1):
    """Per kernel class over `steps` repetitions of the device calls `calls`
    [(T, nseq, sum of L^2)]: average launch time, achieved rate and the
    fraction of the floor (max(FLOP / burst bf16 peak, bytes / HBM peak)) the
    class's total time reaches."""
    out = {}
    for cls, c in stats["classes"].items():
        if not c["count"]:
            continue
        flop = byt = 0.0
        for T, nseq, sl2 in calls:
            f, b = class_work(cls, T, nseq, sl2, wtypes, emb_type)
            mult = LAYERS if cls in LAYER_CLASSES else 1
            flop += f * mult * steps
            byt += b * mult * steps
        total_s = c["ms"] / 1e3
        t_flop, t_byte = flop / (pk["tf"] * 1e12), byt / (pk["hbm"] * 1e9)
        tensor = t_flop >= t_byte
        launches = c["count"]
        rec = {"launches": launches, "avg_launch_us": total_s / launches * 1e6,
               "flop_per_launch": flop / launches, "bytes_per_launch": byt / launches,
               "floor_us_per_launch": max(t_flop, t_byte) / launches * 1e6, "bound": "tensor" if tensor else "hbm",
               "frac": max(t_flop, t_byte) / total_s if total_s > 0 else None}
        rec["achieved"] = flop / total_s / 1e12 if tensor else byt / total_s / 1e9
        rec["unit"] = "TFLOP/s" if tensor else "GB/s"
        if tensor and sm_mhz:
            rec["frac_at_sampled_clock"] = rec["frac"] * 1965.0 / sm_mhz
        out[cls] = rec
    return out


# ------------------------------------------------------------- GPU arm -----

class DeviceBatch:
    """A packed batch resident on the device, split into calls of at most
    MAX_DEVICE_TOKENS tokens (whole sequences)."""

    def __init__(self, e, ids, offs, stream):
        import torch
        from llm_embed_b200.embed import MAX_DEVICE_TOKENS
        self.e, self.stream = e, stream
        self.nseq, self.T = offs.size - 1, int(offs[-1])
        self.lens = np.diff(offs)
        self.sum_l2 = float((self.lens.astype(np.float64) ** 2).sum())
        self.out = torch.empty(max(self.nseq, 1), H, device="cuda")
        self.calls = []
        self.work = []  # (T, nseq, sum of L^2) of each device call
        s0 = 0
        while s0 < self.nseq:
            s1 = s0 + 1
            while s1 < self.nseq and offs[s1 + 1] - offs[s0] <= MAX_DEVICE_TOKENS:
                s1 += 1
            sub = (offs[s0:s1 + 1] - offs[s0]).astype(np.int32)
            d_ids = torch.from_numpy(np.ascontiguousarray(ids[offs[s0]:offs[s1]])).cuda()
            d_offs = torch.from_numpy(sub).cuda()
            self.calls.append((d_ids, d_offs, s1 - s0, int(sub[-1]), int(np.diff(sub).max()), s0))
            lens = np.diff(sub).astype(np.float64)
            self.work.append((int(sub[-1]), s1 - s0, float((lens ** 2).sum())))
            s0 = s1

    def step(self):
        for d_ids, d_offs, n, T, maxlen, s0 in self.calls:
            self.e.embed_device(d_ids.data_ptr(), d_offs.data_ptr(), n, T, maxlen, self.out[s0:].data_ptr(),
                                self.stream.cuda_stream)


class Ctx:
    def __init__(self, rank, world, local_rank):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.rank, self.world, self.local_rank = rank, world, local_rank
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        self.stream = torch.cuda.Stream()
        torch.cuda.set_stream(self.stream)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, x):
        if self.world == 1:
            return x
        t = self.torch.tensor([float(x)], dtype=self.torch.float64, device="cuda")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return t.item()

    def gather(self, obj):
        if self.world == 1:
            return [obj]
        out = [None] * self.world
        self.dist.all_gather_object(out, obj)
        return out

    def time_steps(self, b, steps, warmup, clocks=None):
        """CUDA-event ms of each of `steps` steps on the launching stream,
        L2 flushed before each (outside the events); and our kernel launches
        inside the timed region."""
        torch = self.torch
        for _ in range(max(warmup, 3)):
            b.step()
        torch.cuda.synchronize()
        b.e.sync()
        b.e.stats(reset=True)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        self.barrier()
        torch.cuda.synchronize()
        if clocks:
            clocks.start()
        for i in range(steps):
            self.flush.zero_()
            ev[i][0].record(self.stream)
            b.step()
            ev[i][1].record(self.stream)
        torch.cuda.synchronize()
        self.barrier()
        clk = clocks.stop() if clocks else None
        launches = b.e.stats(reset=True)["launches"]
        return [a.elapsed_time(c) for a, c in ev], launches, clk

    def profile(self, b, steps):
        """Per-class device time from a pass with events around every launch.
        A spin kernel ahead of each step keeps the GPU busy while the host
        enqueues the step, so an event pair times the kernel between them,
        not the host's launch work (kernels still run one after another:
        no programmatic overlap between them in this pass)."""
        torch = self.torch
        b.e.set_profiling(True)
        for _ in range(steps):
            self.flush.zero_()
            torch.cuda._sleep(4_000_000 * len(b.calls))  # ~2 ms per device call at ~2 GHz
            b.step()
        torch.cuda.synchronize()
        st = b.e.stats(reset=True)
        b.e.set_profiling(False)
        b.e.sync()
        return st


def model_types(name):
    spec = synth.CONFIG_SPECS[name]
    w = spec.weight_types
    return (w[0], w[1], w[2], w[4]), spec.embd_type


def headline(ctx, args, pk, res):
    from llm_embed_b200.embed import Embedder
    torch = ctx.torch
    path = synth.cached_model("q8_0")
    e = Embedder.Load(path, devices=[ctx.local_rank])
    ids, offs = synth.config_inputs(2)
    l_ids, l_offs, a, b_ = ldist.local_shard(ids, offs, ctx.rank, ctx.world)
    b = DeviceBatch(e, l_ids, l_offs, ctx.stream)
    clocks = Clocks(ctx.local_rank)
    step_ms, launches, clk = ctx.time_steps(b, args.steps, args.warmup, clocks)
    total_ms = ctx.max(sum(step_ms))
    st = ctx.profile(b, args.steps)
    nseq_all = offs.size - 1
    value = nseq_all * args.steps / (total_ms / 1e3)

    # e2e through the public API with host buffers (this rank's shard).
    for _ in range(2):
        e.EmbedIDs(l_ids, l_offs)
    ctx.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = e.EmbedIDs(l_ids, l_offs)
    e2e_s = ctx.max(time.perf_counter() - t0)
    assert np.isfinite(out).all()

    wtypes, etype = model_types("q8_0")
    classes = class_roofline(st, b.work, wtypes, etype, pk, clk.get("sm_mhz"), steps=args.steps)
    kernel_ms = {k: round(v["ms"] / args.steps, 4) for k, v in st["classes"].items() if v["count"]}
    per_rank = ctx.gather({"rank": ctx.rank, "sequences": [a, b_], "tokens": b.T,
                           "ms_per_step": sum(step_ms) / args.steps, "kernel_ms_per_step": kernel_ms,
                           "gpu_launches_per_step": launches / args.steps, "clocks": clk})

    gather = None
    if ctx.world > 1:
        # The optional collective of the multi-GPU row: every rank's
        # embeddings to every rank (NCCL all-gather over NVLink), shards
        # padded to the largest one.  Not part of the path or of `value`.
        counts = [int(ldist.local_shard(ids, offs, r, ctx.world)[1].size - 1) for r in range(ctx.world)]
        mx = max(counts)
        send = torch.zeros(mx, H, device="cuda")
        send[:b.nseq].copy_(b.out[:b.nseq])
        recv = torch.empty(ctx.world * mx, H, device="cuda")
        for _ in range(3):
            ctx.dist.all_gather_into_tensor(recv, send)
        torch.cuda.synchronize()
        ctx.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        g0.record(ctx.stream)
        for _ in range(reps):
            ctx.dist.all_gather_into_tensor(recv, send)
        g1.record(ctx.stream)
        torch.cuda.synchronize()
        g_ms = ctx.max(g0.elapsed_time(g1) / reps)
        got = recv.view(ctx.world, mx, H)[ctx.rank, :b.nseq]
        assert torch.equal(got, b.out[:b.nseq])
        nbytes = ctx.world * mx * H * 4
        gather = {"ms": g_ms, "bytes_gathered": nbytes, "algbw_gbs": nbytes / (g_ms * 1e6),
                  "busbw_gbs": nbytes * (ctx.world - 1) / ctx.world / (g_ms * 1e6),
                  "note": "NCCL all_gather_into_tensor of every rank's [max shard x 768] f32 embeddings, CUDA events "
                          "on the bench stream, mean of 20 after 3 warm-up, max over ranks; outside the timed step"}

    weak = None
    if ctx.world > 1:
        # Weak scaling: every rank its own 256-sequence batch (seed 1 + rank).
        w_ids, w_offs = synth.config_inputs(2, seed=1 + ctx.rank)
        wb = DeviceBatch(e, w_ids, w_offs, ctx.stream)
        w_ms, _, _ = ctx.time_steps(wb, args.steps, args.warmup)
        w_total = ctx.max(sum(w_ms))
        weak = {"value": 256 * ctx.world * args.steps / (w_total / 1e3), "unit": "embeddings/s",
                "ms_per_step": w_total / args.steps,
                "config": "each rank embeds its own configs[2]-shaped batch (256 sequences, seed 1 + rank)"}

    if ctx.rank == 0:
        dom = max(classes, key=lambda c: classes[c]["avg_launch_us"] * classes[c]["launches"])
        d = classes[dom]
        peak = pk["tf"] if d["bound"] == "tensor" else pk["hbm"]
        roof = {"kernel": dom, "bound": d["bound"], "achieved": d["achieved"], "peak": peak, "unit": d["unit"],
                "frac": d["frac"], "traffic": None, "floor_us": d["floor_us_per_launch"],
                "avg_launch_ms": d["avg_launch_us"] / 1e3,
                "algorithmic_per_launch": {"flop": d["flop_per_launch"], "bytes": d["bytes_per_launch"],
                                           "tokens": b.T},
                "peak_source": (f"{pk['src']} bf16_tflops (burst: kernel timed inside a sub-second region)"
                                if d["bound"] == "tensor" else f"{pk['src']} hbm_gbs"),
                "sm_mhz_sampled": clk.get("sm_mhz")}
        if d["bound"] == "tensor":
            roof["frac_vs_sustained_peak"] = d["achieved"] / pk["tf_sust"]
        tr_path = os.path.join(ROOT, "profiles", "traffic.json")
        if ctx.world == 1 and os.path.exists(tr_path):
            with open(tr_path) as f:
                tr = json.load(f).get(dom)
            roof["traffic"] = tr.get("bytes_per_launch") if isinstance(tr, dict) else tr
        res.update({
            "metric": METRIC, "value": value, "unit": "embeddings/s", "n_gpus": ctx.world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp16 operands, fp32 accumulate", "data": "synthetic",
            "config": {"workload": "configs[2]: 256 sequences, L~U[16,128] packed (no padding), Q8_0 nomic-bert "
                                   "12x768, random-init N(0,0.02), sharded over the GPUs",
                       "sequences": nseq_all, "tokens": int(offs[-1]), "parallelism": f"replica x{ctx.world}",
                       "l2": "flushed between steps (256 MiB memset outside the timed events); weights 120 MB + "
                             "activations > L2"},
            "e2e": {"value": nseq_all * args.steps / e2e_s, "unit": "embeddings/s",
                    "h2d_bytes_per_step": int(ids.nbytes + offs.nbytes), "d2h_bytes_per_step": int(nseq_all * H * 4),
                    "timing": "host wall clock per rank around K synchronous EmbedIDs calls on its shard, max over "
                              "ranks"},
            "roofline": roof,
            "roofline_classes": classes,
            "gpu_launches": launches,
            "kernel_ms_per_step": kernel_ms,
            "per_rank": per_rank,
            "clocks": clk,
        })
        if weak:
            res["weak_scaling"] = weak
        if gather:
            res["allgather_embeddings"] = gather
        res["clocks"]["reasons"] = sorted({r for p in per_rank for r in (p["clocks"] or {}).get("reasons", [])})
    return e


def latency(ctx, e, res):
    """batch 1, 8 tokens; p50 over 50 calls, L2 flushed first."""
    torch = ctx.torch
    if ctx.rank != 0:
        return
    ids8, offs8 = synth.config_inputs(0)
    d_ids = torch.from_numpy(ids8).cuda()
    d_offs = torch.from_numpy(offs8).cuda()
    d_out = torch.empty(1, H, device="cuda")
    lat_dev, lat_e2e = [], []
    for i in range(60):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ctx.flush.zero_()
        # The GPU spins while the host enqueues the call, so the events
        # time the forward on the device, not the host's launch work.
        torch.cuda._sleep(2_000_000)
        a.record(ctx.stream)
        e.embed_device(d_ids.data_ptr(), d_offs.data_ptr(), 1, 8, 8, d_out.data_ptr(), ctx.stream.cuda_stream)
        b.record(ctx.stream)
        torch.cuda.synchronize()
        if i >= 10:
            lat_dev.append(a.elapsed_time(b) * 1e3)
    for i in range(60):
        t0 = time.perf_counter()
        e.Embed(ids8)
        if i >= 10:
            lat_e2e.append((time.perf_counter() - t0) * 1e6)
    floor_us = 120324096 / (peaks()["hbm"] * 1e3)
    res["latency_batch1_8tok_p50_us"] = {
        "device": statistics.median(lat_dev), "e2e": statistics.median(lat_e2e),
        "weight_read_floor_us": floor_us, "x_floor": statistics.median(lat_dev) / floor_us,
        "config": "configs[0], L2 flushed before each call; floor = Q8_0 layer weights (120,324,096 B) / hbm_gbs"}


def other_configs(ctx, args, pk, res):
    """configs[3] (1024 x U[64,256], Q4_K_M mix) and configs[4] (4096 x 512,
    Q6_K and Q5_K) at their stated sizes, sharded over the ranks."""
    from llm_embed_b200.embed import Embedder
    out = {}
    for key, cfg, model in (("configs3_q4_k_m", 3, "q4_k_m"), ("configs4_q6_k", 4, "q6_k"),
                            ("configs4_q5_k", 4, "q5_k")):
        e = Embedder.Load(synth.cached_model(model), devices=[ctx.local_rank])
        ids, offs = synth.config_inputs(cfg)
        l_ids, l_offs, a, b_ = ldist.local_shard(ids, offs, ctx.rank, ctx.world)
        b = DeviceBatch(e, l_ids, l_offs, ctx.stream)
        steps = 2
        ms, launches, _ = ctx.time_steps(b, steps, 1)
        total = ctx.max(sum(ms))
        st = ctx.profile(b, 1)
        wtypes, etype = model_types(model)
        classes = class_roofline(st, b.work, wtypes, etype, pk)
        all_l = np.diff(offs).astype(np.float64)
        flop = GEMM_FLOP_PER_TOKEN * all_l.sum() + 36864.0 * (all_l ** 2).sum()
        t_step = total / steps / 1e3
        if ctx.rank == 0:
            out[key] = {
                "sequences": int(offs.size - 1), "tokens": int(offs[-1]), "model": model,
                "ms_per_step": total / steps, "embeddings_per_s": (offs.size - 1) / t_step,
                "tensor_roofline": {"achieved_tflops": flop / t_step / 1e12, "peak": pk["tf"] * ctx.world,
                                    "frac": flop / t_step / 1e12 / (pk["tf"] * ctx.world),
                                    "flop_per_step": flop,
                                    "note": "GEMM + attention FLOPs of valid tokens over the whole forward "
                                            "(every kernel, launch gaps included) against burst bf16 x GPUs"},
                "rank0_kernel_ms": {k: round(v["ms"], 3) for k, v in st["classes"].items() if v["count"]},
                "rank0_classes": {k: {"frac": v["frac"], "bound": v["bound"]} for k, v in classes.items()},
                "gpu_launches_per_step": launches / steps,
            }
        e.Close()
    res["configs"] = out


def op_sweep(ctx, pk, res):
    """le_qgemm_device (fp32 x in, fp32 y out) over M x K x N x
    type, median of 5 calls with L2 flushed between them (the GPU kept ahead
    of the host, so the events time the two kernels of a call)."""
    from llm_embed_b200.embed import QWeight
    torch = ctx.torch
    rows = []
    xs = {}
    for qtype, tname in ((synth.GGML_Q8_0, "q8_0"), (synth.GGML_Q6_K, "q6_k"), (synth.GGML_Q5_K, "q5_k"),
                         (synth.GGML_Q4_K, "q4_k")):
        for K in (768, 3072):
            for N in (768, 2304, 3072):
                rng = np.random.default_rng([0, qtype, K, N])
                w = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
                qw = QWeight(qtype, synth.quantize(w, qtype), N, K)
                for M in (8, 512, 32768):
                    if (M, K) not in xs:
                        xs[(M, K)] = torch.randn(M, K, device="cuda", generator=torch.Generator("cuda").manual_seed(M + K))
                    x = xs[(M, K)]
                    y = torch.empty(M, N, device="cuda")
                    for _ in range(2):
                        qw.matmul_device(x.data_ptr(), M, y.data_ptr(), ctx.stream.cuda_stream)
                    ts = []
                    for _ in range(5):
                        ctx.flush.zero_()
                        torch.cuda._sleep(1_000_000)  # the GPU ahead of the host's enqueue
                        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        a.record(ctx.stream)
                        qw.matmul_device(x.data_ptr(), M, y.data_ptr(), ctx.stream.cuda_stream)
                        b.record(ctx.stream)
                        torch.cuda.synchronize()
                        ts.append(a.elapsed_time(b) / 1e3)
                    qw.sync()
                    t = statistics.median(ts)
                    flop = 2.0 * M * N * K
                    byt = N * K * BPE[qtype] + 4.0 * M * K + 4.0 * M * N
                    rec = {"type": tname, "M": M, "K": K, "N": N, "us": t * 1e6, "tflops": flop / t / 1e12,
                           "gbs": byt / t / 1e9}
                    rec["frac_hbm"] = rec["gbs"] / pk["hbm"]
                    rec["frac_tensor"] = rec["tflops"] / pk["tf"]
                    rec["bound"] = "hbm" if M == 8 else ("tensor" if M == 32768 else "both")
                    rows.append(rec)
                qw.close()
    res["op_sweep_configs1"] = {
        "rows": rows,
        "note": "bytes = N*K*bytes_per_weight + 4*M*K + 4*M*N (fp32 x and y); M=8 against hbm_gbs, M=32768 "
                "against burst bf16_tflops; the call converts x to fp16 and runs the GEMM (two kernels)"}


def load_phases(ctx, res):
    from llm_embed_b200.embed import Embedder
    path = synth.cached_model("q8_0")
    t0 = time.perf_counter()
    e = Embedder.Load(path, devices=[ctx.local_rank])
    wall = (time.perf_counter() - t0) * 1e3
    st = e.load_stats()
    e.Close()
    st["wall_ms_python_load"] = wall
    st["model"] = "configs[0]/[2] Q8_0 GGUF (the file is in the page cache: written earlier in this run)"
    res["load_f2"] = st


def tokenizer_rate(res):
    """Host tokenizer throughput (f1): the C++ encoder (le_tokenize) on one
    thread and on all host threads, and the Python restatement, over the
    same synthetic texts (vocabulary words, unknown words, punctuation)."""
    from llm_embed_b200.embed import Tokenizer
    from llm_embed_b200.tokenizer import WordPieceTokenizer
    path = synth.cached_model("q8_0")
    words = synth._VOCAB_WORDS + ["unknownword", "tokenization", "café", "hello,", "world!", "Machine", "(x)"]
    rng = np.random.default_rng(5)
    texts = [" ".join(rng.choice(words, size=int(rng.integers(20, 90)))) for _ in range(20000)]
    py = WordPieceTokenizer.Load(path)
    t0 = time.perf_counter()
    n_py = sum(len(py.Encode("search_query: " + t, 2048)[0]) for t in texts[:400])
    py_rate = n_py / (time.perf_counter() - t0)
    nat = Tokenizer.Load(path)
    t0 = time.perf_counter()
    buf, toffs = Tokenizer.pack_texts(texts)
    pack_s = time.perf_counter() - t0
    rates = {}
    for threads in (1, os.cpu_count() or 1):
        nat.encode_packed(buf, toffs, 2048, "search_query: ", threads)
        best = 1e9
        for _ in range(3):
            t0 = time.perf_counter()
            ids, _ = nat.encode_packed(buf, toffs, 2048, "search_query: ", threads)
            best = min(best, time.perf_counter() - t0)
        rates[threads] = ids.size / best
    nat.close()
    res["tokenizer_f1"] = {
        "native_tokens_per_s_1_thread": rates[1], "native_tokens_per_s_all_threads": rates[max(rates)],
        "threads": max(rates), "python_restatement_tokens_per_s": py_rate, "texts": len(texts),
        "tokens": int(ids.size), "python_packing_ms": pack_s * 1e3,
        "needed_for_8_gpus_tokens_per_s": 8 * 55000 * 73,
        "note": "le_tokenize on texts packed into one UTF-8 buffer (what a Go host passes), best of 3; the "
                "Python list -> buffer packing is timed apart; needed = 8 GPUs x ~55K embeddings/s x 73 tokens"}


def run_ours(args, rank, world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    if rank == 0:
        for name in ("q8_0",) + (("q4_k_m", "q6_k", "q5_k") if "configs" in args.sections else ()):
            synth.cached_model(name)
    ctx = Ctx(rank, world, local_rank)
    ctx.barrier()
    pk = peaks()
    res = {}
    e = headline(ctx, args, pk, res)
    if "latency" in args.sections:
        latency(ctx, e, res)
    e.Close()
    ctx.barrier()
    if "configs" in args.sections:
        other_configs(ctx, args, pk, res)
    if world == 1 and "sweep" in args.sections:
        op_sweep(ctx, pk, res)
    if world == 1 and "load" in args.sections:
        load_phases(ctx, res)
    if rank == 0 and "tokenizer" in args.sections:
        tokenizer_rate(res)
    ctx.barrier()
    return res if rank == 0 else None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sections", default=",".join(ALL_SECTIONS),
                    help="comma list of " + ",".join(ALL_SECTIONS) + " (the headline always runs)")
    args = ap.parse_args()
    args.sections = set(args.sections.split(","))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        result = run_ours(args, rank, world, local_rank)
        if rank == 0:
            if world == 1 and not args.no_cpu_baseline:
                ids, offs = synth.config_inputs(2)
                result["cpu_baseline"] = cpu_baseline(synth.cached_model("q8_0"), ids, offs)
            print(json.dumps(result), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
