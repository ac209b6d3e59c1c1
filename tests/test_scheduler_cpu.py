"""Multi-rank host logic on CPU: LPT sharding of utterances and the gather of
results over a world-size-2 gloo group (each rank runs the CPU oracle on its
share; rank 0 checks the merged result against a single-rank run)."""
from __future__ import annotations

import os
import socket

import numpy as np
import torch.multiprocessing as mp

from conftest import ROOT, load_pkg


def _utts(n=7):
    sched = load_pkg().scheduler
    rng = np.random.default_rng(0)
    return [sched.Utterance(uid=i, prefill=int(rng.integers(32, 512)), frames=int(rng.integers(2, 5)),
                            payload=rng.integers(0, 151643, 12).astype(np.int32)) for i in range(n)]


def test_lpt_partition_properties():
    sched = load_pkg().scheduler
    utts = _utts(64)
    for world in (1, 2, 4, 8):
        parts = sched.lpt_partition(utts, world)
        uids = sorted(u.uid for p in parts for u in p)
        assert uids == list(range(64))                      # every utterance exactly once
        lb = max(max(u.cost for u in utts), sum(u.cost for u in utts) / world)
        assert sched.makespan(parts) <= 4.0 / 3.0 * lb + 1  # LPT bound
        assert parts == sched.lpt_partition(utts, world)    # deterministic


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, model, out_q):
    import sys
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from oracle import Oracle
    sched = load_pkg().scheduler
    o = Oracle(model, threads=2)

    def run_one(u):
        return o.generate(u.payload, u.frames, eos_bias=-1e9)["codes"]

    res = sched.run_sharded(_utts(), run_one, rank, world)
    if rank == 0:
        out_q.put({k: v.tolist() for k, v in res.items()})
    dist.destroy_process_group()


def test_two_rank_gloo_shard_and_gather(tiny_f16):
    sched = load_pkg().scheduler
    from oracle import Oracle
    o = Oracle(tiny_f16, threads=2)
    single = sched.run_sharded(_utts(), lambda u: o.generate(u.payload, u.frames, eos_bias=-1e9)["codes"], 0, 1)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, tiny_f16, q)) for r in range(2)]
    for p in procs:
        p.start()
    merged = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(merged) == sorted(single)
    for uid, codes in single.items():
        assert merged[uid] == codes.tolist()
