"""CPU, world size 2 (gloo): the multi-GPU host logic of the reductions.

The GPU partial kernels cannot run here, so each rank computes its chunk partials with a fixed-order
numpy stand-in; what is under test is the host side the GPU path uses: chunk-aligned shard ranges
that tile the element range, the padded all-gather that restores global chunk order for uneven
shards, and a fixed-order finish giving bit-identical results for 1 and 2 ranks.  A rank that
raises before the collective is also tested: the other rank's collective ends with an error within
the process-group timeout instead of hanging.
"""
import datetime
import importlib
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent
CHUNK = 8192


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partials(a, b):
    """Stand-in for the GPU chunk kernel: fp64 sum of each chunk's elements, fixed order."""
    n = a.size
    out = np.empty((n + CHUNK - 1) // CHUNK)
    for c in range(out.size):
        d = a[c * CHUNK:(c + 1) * CHUNK].astype(np.float64) - b[c * CHUNK:(c + 1) * CHUNK]
        out[c] = np.sum(np.sqrt(d * d + 1e-6))
    return out


def _finish(parts, n_total):
    s = 0.0
    for v in parts:  # fixed order: chunk order
        s += float(v)
    return s / n_total


def _worker(rank, world, port, n_total, q, fail_rank):
    sys.path.insert(0, str(REPO))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        d = importlib.import_module("cuda-optimization-benchmark_b200.dist")
        g = np.random.default_rng(0)
        a = g.standard_normal(n_total).astype(np.float32)
        b = g.standard_normal(n_total).astype(np.float32)
        lo, hi = d.shard_range(n_total, CHUNK, world, rank)
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        local = torch.from_numpy(_partials(a[lo:hi], b[lo:hi]))
        rows = d.gather_rows(local, d.shard_chunks(n_total, CHUNK, world))
        q.put((rank, "ok", lo, hi, _finish(rows.numpy(), n_total)))
    except Exception as e:  # reported to the parent, which checks who failed and how
        q.put((rank, "error", type(e).__name__, str(e)[:200], None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, n_total, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_total, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    return sorted(res)


def test_shard_ranges_tile_the_range():
    d = importlib.import_module("cuda-optimization-benchmark_b200.dist")
    for n in (1, CHUNK - 1, CHUNK, 5 * CHUNK + 7, 1 << 20):
        for world in (1, 2, 3, 8):
            ranges = [d.shard_range(n, CHUNK, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            for (l0, h0), (l1, h1) in zip(ranges, ranges[1:]):
                assert h0 == l1 and l1 % CHUNK == 0
            assert sum(d.shard_chunks(n, CHUNK, world)) == (n + CHUNK - 1) // CHUNK


@pytest.mark.parametrize("n_total", [5 * CHUNK + 123, 64 * CHUNK])
def test_two_ranks_match_one_rank_bitwise(n_total):
    one = _run(1, n_total)
    two = _run(2, n_total)
    assert [r[1] for r in two] == ["ok", "ok"]
    assert two[0][4] == two[1][4] == one[0][4]   # identical bits on every rank and vs one rank
    assert two[0][3] == two[1][2]                 # rank 0 ends where rank 1 begins


def test_failing_rank_is_reported_not_hung():
    res = _run(2, 8 * CHUNK, fail_rank=1)
    by_rank = {r[0]: r for r in res}
    assert by_rank[1][1] == "error" and "injected" in by_rank[1][3]
    assert by_rank[0][1] == "error"   # its all-gather ended with an error (peer gone / timeout)
