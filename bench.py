#!/usr/bin/env python
"""Benchmark of the B200 nomic-bert encoder (BASELINE.json metric:
"embeddings/s at seq128 on 1/2/4/8 B200; p50 batch-1 8-token latency").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step embeds one configs[2] batch per GPU: 256 sequences, lengths
U[16, 128], Q8_0 random-init 12-layer model (synthetic data, seeded; rank r
uses input seed 1 + r).  Multi-GPU runs are one process per GPU (torchrun),
each with its own replica and its own batch (weak scaling, no data-path
collective); the timed region is bracketed by a barrier and synchronize and
the max over ranks is reported.  One JSON line is printed by rank 0.

  value     embeddings/s over all ranks, inputs resident in HBM, CUDA-event
            time of the K steps on the launching stream (L2 flushed between
            steps, outside the events).
  e2e       same metric through the public host API (Embedder.EmbedIDs):
            host ids in, host embeddings out, copies inside the timed region.
  roofline  the dominant kernel class (largest device time), timed with the
            library's per-launch CUDA events in a second pass over the same
            steps (events around every launch would inflate `value`).
  cpu_baseline  the CPU restatement of the reference (oracle/) timed on this
            host's cores on a bounded sample of the same batch (rank 0, N=1).

--impl reference times that CPU restatement of the reference's Go path alone
(the Go reference cannot be built: no Go toolchain in the image).
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

from llm_embed_b200 import synth  # noqa: E402

METRIC = "embeddings/s at seq128 on 1/2/4/8 B200; p50 batch-1 8-token latency"
H, F, LAYERS = 768, 3072, 12
GEMM_SHAPES = {"gemm_qkv": (3 * H, H), "gemm_attn_out": (H, H), "gemm_ffn_upgate": (2 * F, H), "gemm_ffn_down": (H, F)}
Q8_0_LAYER_BYTES = 9437184 * 34 // 32  # per layer, all five projections


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p["bf16_tflops_sustained"], "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, 1590.0, 1400.0, "fallback"


class Clocks:
    """nvidia-smi sampling of one GPU during the timed region."""

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
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def cpu_baseline(path, ids, offs, budget_s=12.0):
    """The CPU restatement (oracle/, test infrastructure) on a bounded sample
    of the batch, all host threads: embeddings/s."""
    import oracle
    m = oracle.Model(path)
    threads = os.cpu_count() or 1
    done, tokens, t_total = 0, 0, 0.0
    nseq = offs.size - 1
    chunk = max(threads, 8)
    while t_total < budget_s and done < nseq:
        b = min(nseq, done + chunk)
        sub_offs = (offs[done:b + 1] - offs[done]).astype(np.int32)
        t0 = time.perf_counter()
        m.embed_ids(ids[offs[done]:offs[b]], sub_offs, nthreads=threads)
        t_total += time.perf_counter() - t0
        tokens += int(offs[b] - offs[done])
        done = b
    m.close()
    return {"value": done / t_total, "unit": "embeddings/s", "cores": threads, "kind": "port",
            "sample": f"first {done} of {nseq} configs[2] sequences ({tokens} tokens), {t_total:.1f} s, "
                      "C++ restatement of the Go reference (no Go toolchain to build the reference)"}


def run_reference(args, rank):
    if rank != 0:
        return
    import oracle
    path = synth.cached_model("q8_0")
    ids, offs = synth.config_inputs(2)
    m = oracle.Model(path)
    threads = os.cpu_count() or 1
    # One step = a bounded sample of the batch, sized from a calibration run
    # so the whole run stays within a few minutes.
    n_cal = min(threads, 32)
    t0 = time.perf_counter()
    m.embed_ids(ids[:offs[n_cal]], offs[:n_cal + 1], nthreads=threads)
    per_seq = (time.perf_counter() - t0) / n_cal
    total_steps = args.steps + args.warmup
    n = int(max(threads, min(256, 150.0 / total_steps / per_seq)))
    n = min(n, 256)
    sub_ids, sub_offs = ids[:offs[n]], offs[:n + 1]
    for _ in range(args.warmup):
        m.embed_ids(sub_ids, sub_offs, nthreads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.embed_ids(sub_ids, sub_offs, nthreads=threads)
    dt = time.perf_counter() - t0
    m.close()
    v = n * args.steps / dt
    sample = (f"first {n} of 256 configs[2] sequences ({int(offs[n])} tokens) per step, "
              "C++ restatement of the Go reference (no Go toolchain to build the reference)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "embeddings/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "configs[2] sample: Q8_0 nomic-bert, 12 layers, L~U[16,128]", "sequences_per_step": n},
        "cpu_baseline": {"value": v, "unit": "embeddings/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "embeddings/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from llm_embed_b200.embed import CLASS_NAMES, Embedder

    torch.cuda.set_device(local_rank)
    if rank == 0:
        path = synth.cached_model("q8_0")
    if world > 1:
        dist.barrier()
    path = synth.cached_model("q8_0")
    e = Embedder.Load(path, devices=[local_rank])
    ids, offs = synth.config_inputs(2, seed=1 + rank)
    nseq, T = offs.size - 1, int(offs[-1])
    maxlen = int(np.diff(offs).max())
    d_ids = torch.from_numpy(ids).cuda()
    d_offs = torch.from_numpy(offs).cuda()
    d_out = torch.empty(nseq, H, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    # A dedicated stream: the library launches on it and the timing events
    # are recorded on it (handle 0 would mean "the model's own stream").
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    assert stream.cuda_stream != 0

    def step():
        e.embed_device(d_ids.data_ptr(), d_offs.data_ptr(), nseq, T, maxlen, d_out.data_ptr(), stream.cuda_stream)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    e.sync()
    e.stats(reset=True)

    clocks = Clocks(local_rank)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    enqueue_s = 0.0
    for i in range(args.steps):
        flush.zero_()
        ev[i][0].record(stream)
        t0 = time.perf_counter()
        step()
        enqueue_s += time.perf_counter() - t0
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    launches = e.stats(reset=True)["launches"]
    total_ms = max_over_ranks(sum(step_ms))

    # Kernel breakdown: the same steps again with a CUDA event pair around
    # every launch (kept out of the timed region above).
    e.set_profiling(True)
    for i in range(args.steps):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    st = e.stats(reset=True)
    e.set_profiling(False)
    e.sync()
    value = nseq * world * args.steps / (total_ms / 1e3)

    # e2e through the public API with host buffers.
    for _ in range(2):
        e.EmbedIDs(ids, offs)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = e.EmbedIDs(ids, offs)
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    assert np.isfinite(out).all()
    e2e = {"value": nseq * world * args.steps / e2e_s, "unit": "embeddings/s",
           "h2d_bytes_per_step": int(ids.nbytes + offs.nbytes), "d2h_bytes_per_step": int(nseq * H * 4),
           "timing": "host wall clock per rank around K synchronous EmbedIDs calls, max over ranks"}

    # Batch-1 8-token latency.
    ids8, offs8 = synth.config_inputs(0)
    d8_ids = torch.from_numpy(ids8).cuda()
    d8_offs = torch.from_numpy(offs8).cuda()
    d8_out = torch.empty(1, H, device="cuda")
    lat_dev, lat_e2e = [], []
    for i in range(60):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        flush.zero_()
        a.record(stream)
        e.embed_device(d8_ids.data_ptr(), d8_offs.data_ptr(), 1, 8, 8, d8_out.data_ptr(), stream.cuda_stream)
        b.record(stream)
        torch.cuda.synchronize()
        if i >= 10:
            lat_dev.append(a.elapsed_time(b) * 1e3)
    for i in range(60):
        t0 = time.perf_counter()
        e.Embed(ids8)
        if i >= 10:
            lat_e2e.append((time.perf_counter() - t0) * 1e6)

    # Roofline of the dominant kernel class.
    hbm, tf_burst, tf_sust, src = peaks()
    cls = max(CLASS_NAMES, key=lambda c: st["classes"][c]["ms"])
    c = st["classes"][cls]
    avg_ms = c["ms"] / max(c["count"], 1)
    if cls in GEMM_SHAPES:
        n, k = GEMM_SHAPES[cls]
        flop = 2.0 * T * n * k
        achieved = flop / (avg_ms / 1e3) / 1e12
        roof = {"kernel": cls, "bound": "tensor", "achieved": achieved, "peak": tf_sust, "unit": "TFLOP/s",
                "frac": achieved / tf_sust, "traffic": None,
                "peak_source": f"{src} bf16_tflops_sustained (kernel timed inside a long step)",
                "algorithmic_per_launch": f"2*T*N*K = {flop:.4g} FLOP (T={T} valid tokens, N={n}, K={k})",
                "avg_launch_ms": avg_ms}
    elif cls == "attention":
        flop = 4.0 * 64 * sum(int(L) ** 2 for L in np.diff(offs)) * 12
        achieved = flop / (avg_ms / 1e3) / 1e12
        roof = {"kernel": cls, "bound": "tensor", "achieved": achieved, "peak": tf_sust, "unit": "TFLOP/s",
                "frac": achieved / tf_sust, "traffic": None, "avg_launch_ms": avg_ms,
                "peak_source": f"{src} bf16_tflops_sustained"}
    else:
        byt = 2.0 * T * H * 4
        achieved = byt / (avg_ms / 1e3) / 1e9
        roof = {"kernel": cls, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": None, "avg_launch_ms": avg_ms, "peak_source": f"{src} hbm_gbs"}
    tr_path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tr_path):
        with open(tr_path) as f:
            roof["traffic"] = json.load(f).get(cls)
    breakdown = {k: round(v["ms"] / args.steps, 4) for k, v in st["classes"].items()}

    result = None
    if rank == 0:
        result = {
            "metric": METRIC, "value": value, "unit": "embeddings/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 operands, fp32 accumulate", "data": "synthetic",
            "config": {"workload": "configs[2]: 256 seqs/GPU, L~U[16,128] packed (no padding), Q8_0 nomic-bert "
                                   "12x768, random-init N(0,0.02)",
                       "sequences_per_gpu": nseq, "tokens_per_gpu": T, "parallelism": f"replica x{world}",
                       "l2": "flushed between steps (256 MiB memset outside the timed events); weights 120 MB + "
                             "activations > L2"},
            "e2e": e2e,
            "latency_batch1_8tok_p50_us": {"device": statistics.median(lat_dev), "e2e": statistics.median(lat_e2e),
                                           "config": "configs[0], L2 flushed before each call"},
            "roofline": roof,
            "gpu_launches": launches,
            "host_enqueue_ms_per_step": enqueue_s * 1e3 / args.steps,
            "kernel_ms_per_step": breakdown,
            "clocks": clk,
        }
    if world > 1:
        dist.barrier()
    e.Close()
    return result


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
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
