"""Time the forward pass on a BASELINE.json config's synthetic workload.

    python -m llm_embed_b200.workloads --config 4 --model q6_k --seqs 128 [--steps 3]

Loads the config's synthetic model, takes the first --seqs sequences of the
config's batch (one device chunk: at most 65,536 tokens), runs the forward on
device-resident ids (L2 flushed between steps, outside the CUDA events) and
prints one JSON line: embeddings/s, ms per step and the device time of each
kernel class from a separate profiled step.  bench.py measures the headline
config; this covers the others.
"""
from __future__ import annotations

import argparse
import json

import numpy as np

from . import synth
from .embed import Embedder

DEFAULT_MODEL = {2: "q8_0", 3: "q4_k_m", 4: "q6_k"}


def run(config: int, model: str, seqs: int, steps: int) -> dict:
    import torch

    e = Embedder.Load(synth.cached_model(model))
    ids, offs = synth.config_inputs(config)
    n = min(seqs, offs.size - 1)
    ids, offs = ids[:offs[n]], offs[:n + 1]
    T, max_len = int(offs[-1]), int(np.diff(offs).max())
    d_ids = torch.from_numpy(ids).cuda()
    d_offs = torch.from_numpy(offs).cuda()
    d_out = torch.empty(n, e.Dim(), device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    st = torch.cuda.Stream()
    torch.cuda.set_stream(st)
    torch.cuda.synchronize()

    def step():
        e.embed_device(d_ids.data_ptr(), d_offs.data_ptr(), n, T, max_len, d_out.data_ptr(), st.cuda_stream)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    e.sync()
    ms = []
    for _ in range(steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        step()
        b.record(st)
        torch.cuda.synchronize()
        ms.append(a.elapsed_time(b))
    e.stats(reset=True)
    e.set_profiling(True)
    flush.zero_()
    step()
    torch.cuda.synchronize()
    st_ = e.stats(reset=True)
    e.sync()
    e.Close()
    t = float(np.median(ms))
    return {"config": config, "model": model, "sequences": n, "tokens": T, "max_len": max_len,
            "ms_per_step": t, "embeddings_per_s": n / t * 1e3,
            "kernel_ms": {k: round(v["ms"], 4) for k, v in st_["classes"].items() if v["count"]}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", type=int, default=4, choices=[2, 3, 4])
    ap.add_argument("--model", default=None, help="synthetic model name (default: the config's)")
    ap.add_argument("--seqs", type=int, default=128)
    ap.add_argument("--steps", type=int, default=3)
    a = ap.parse_args()
    print(json.dumps(run(a.config, a.model or DEFAULT_MODEL[a.config], a.seqs, a.steps)), flush=True)


if __name__ == "__main__":
    main()
