"""Several GPUs, one process each, NCCL: the row partition and the vocabulary shards end to end.

Needs at least 2 visible GPUs (skipped otherwise). Each rank checks its results against the oracle.
NVLS is switched off (NCCL_NVLS_ENABLE=0): the exchange is one small all-gather.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    import sys

    for p in (os.path.join(ROOT, "loom.cpp_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    import torch.distributed as dist

    import loom_select as sel
    import oracle_binding as ob
    import select_dist
    import synth

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    ok = True
    try:
        nt = max(1, (os.cpu_count() or 4) // world)
        # rows: every rank samples its own share of a 64-row batch
        x, hist, u = synth.sample_chain(64, seed=42, device="cpu")
        lo, hi = select_dist.split(64, world, rank)
        ids, prob = sel.sample_rows(x[lo:hi].to(dev), u[lo:hi].to(dev), 0.7, 1.1, 40, 0.9,
                                    history=hist[lo:hi].to(dev))
        want = ob.sample_rows(x[lo:hi].numpy(), u[lo:hi].numpy(), 0.7, 1.1, 40, 0.9, hist[lo:hi].numpy(),
                              want_logp=False, nthreads=nt)
        ok &= np.array_equal(ids.cpu().numpy(), want["ids"])

        # vocabulary: [32, 262144] bf16 split `world` ways, records all-gathered over NCCL
        xg, ug = synth.gemma_vocab(32, device="cpu")
        V = xg.shape[1]
        vlo, vhi = select_dist.split(V, world, rank)
        shard = xg[:, vlo:vhi].contiguous().to(dev)
        ids, prob, logp = select_dist.sample_vocab_sharded(shard, vlo, V, ug.to(dev), 1.0, 1.0, 64, 0.95,
                                                           want_logp=True)
        want = ob.sample_rows(synth.bf16_bits(xg), ug.numpy(), 1.0, 1.0, 64, 0.95, None, nthreads=nt)
        ok &= np.array_equal(ids.cpu().numpy(), want["ids"])
        ok &= bool(np.all(np.abs(prob.cpu().numpy() - want["prob"]) <= 1e-5 * np.abs(want["prob"])))
        wl = want["logp"].astype(np.float64)
        ok &= bool(np.all(np.abs(logp.cpu().numpy() - wl) <= 1e-5 * np.maximum(1.0, np.abs(wl))))
        torch.cuda.synchronize()
        dist.barrier()
    except Exception as e:  # report, never hang the other rank
        ok = False
        print(f"rank {rank}: {e!r}", flush=True)
    finally:
        dist.destroy_process_group()
    queue.put((rank, bool(ok)))


def test_rows_and_vocab_shards_over_nccl():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip(f"needs 2 or more GPUs, {n} visible")
    world = min(n, 8)
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    codes = [p.exitcode for p in procs]
    results = dict(q.get(timeout=5) for _ in range(world))
    assert codes == [0] * world, codes
    assert all(results[r] for r in range(world)), results
