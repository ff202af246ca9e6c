"""The multi-GPU host logic on CPU: two gloo ranks (world size 2) on 127.0.0.1.

The kernels need a GPU, so the compute here is the oracle; what is under test is the partitioning
and the record exchange of select_dist (the same calls run over NCCL on B200):
  - row partition: each rank samples its rows, the gathered results equal one rank doing all rows;
  - vocabulary shards: each rank makes the records of its slice, all_gather puts them in rank
    order, the merge equals the unsharded chain on both ranks.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(31)
    rows, V = 6, 3001
    x = rng.normal(0, 3, (rows, V)).astype(np.float32)
    x[1, 1400:1700] = 9.0  # a tie across the shard boundary
    hist = rng.integers(0, V, (rows, 40)).astype(np.int32)
    u = rng.random(rows).astype(np.float32)
    return x, hist, u


def _worker(rank, world, port, queue):
    import sys

    for p in (os.path.join(ROOT, "loom.cpp_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    import oracle_binding as ob
    import select_dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        x, hist, u = _inputs()
        rows, V = x.shape
        T, r, k, p = 0.8, 1.2, 16, 0.9
        full = ob.sample_rows(x, u, T, r, k, p, hist)

        # rows: this rank's share, gathered
        lo, hi = select_dist.split(rows, world, rank)
        mine = ob.sample_rows(x[lo:hi], u[lo:hi], T, r, k, p, hist[lo:hi])
        ids = torch.from_numpy(np.pad(mine["ids"], (0, rows - (hi - lo)))).contiguous()
        gathered = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(gathered, ids)
        row_ids = np.concatenate([g.numpy()[: select_dist.split(rows, world, q)[1] - select_dist.split(rows, world, q)[0]]
                                  for q, g in enumerate(gathered)])

        # vocabulary: this rank's slice -> records -> all_gather -> merge
        vlo, vhi = select_dist.split(V, world, rank)
        st, rec = ob.shard_partial(np.ascontiguousarray(x[:, vlo:vhi]), vlo, V, T, r, k, hist)
        assert st == 0
        records = select_dist.gather_records(torch.from_numpy(rec))
        merged = ob.shard_merge(records.numpy().reshape(-1), world, rows, u, T, k, p)
        ok = (np.array_equal(row_ids, full["ids"]) and np.array_equal(merged["ids"], full["ids"])
              and np.array_equal(merged["topk"], full["topk"])
              and np.array_equal(merged["prob"].view(np.uint32), full["prob"].view(np.uint32)))
        queue.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_two_rank_partitions_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    codes = [p.exitcode for p in procs]
    results = dict(q.get(timeout=5) for _ in range(2))
    assert codes == [0, 0], codes
    assert results == {0: True, 1: True}, results
