"""World-size-2 gloo run of the multi-rank path on CPU: each rank embeds its
token-balanced shard (here with the oracle standing in for the device) and
rank 0 gathers; the result equals one process embedding everything."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from llm_embed_b200 import dist as ld
from llm_embed_b200 import synth
from helpers import MODEL_DIR, small_spec


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, path, ids, offs, q):
    import torch.distributed as dist

    import oracle
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    m = oracle.Model(path)
    try:
        out = ld.embed_sharded(lambda i, o: m.embed_ids(i, o, nthreads=2), ids, offs, m.hidden)
        if rank == 0:
            q.put(out)
    finally:
        m.close()
        dist.destroy_process_group()


def test_shard_bounds_balanced_and_contiguous():
    ids, offs = synth.config_inputs(2)
    for n in (1, 2, 4, 8):
        c = ld.shard_bounds(offs, n)
        assert c[0] == 0 and c[-1] == 256 and all(a <= b for a, b in zip(c, c[1:]))
        w = ld.seq_work(np.diff(offs))
        parts = [w[c[i]:c[i + 1]].sum() for i in range(n)]
        assert max(parts) - min(parts) <= 2 * w.max()


def test_shard_bounds_more_ranks_than_sequences():
    offs = np.array([0, 5, 9], np.int32)
    c = ld.shard_bounds(offs, 4)
    assert c[0] == 0 and c[-1] == 2 and sorted(c) == c


def test_gloo_world2_matches_single_process():
    path = synth.cached_model(small_spec(layers=1, vocab=2048, seed=31), MODEL_DIR)
    ids, offs = synth.make_ids([7, 19, 3, 40, 11, 1], seed=9, vocab=2048)
    import oracle
    m = oracle.Model(path)
    ref = m.embed_ids(ids, offs, nthreads=2)
    m.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, path, ids, offs, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert np.array_equal(got, ref)
