"""CPU, world sizes 2 and 3 (gloo): the host logic of reward-to-go sharded over time.

The GPU kernels cannot run here, so each rank's slice maps and slice scan are numpy stand-ins with
the C ABI's contract (a [B, 2] fp64 map per row, y_left = b + a * y_right over the rank's steps;
the scan composes the maps of the later ranks, in rank order, into its carry-in).  Under test is
what the GPU path runs unchanged: `ops.reward_to_go_time_sharded`'s all-gather of the maps in rank
order (the layout both NCCL and gloo accept), the rank indexing of the carry-in, and
`dist.time_range`'s contiguous split (ragged lengths included); the concatenated outputs must meet
the reward-to-go oracle.
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


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _maps(reward, done, gamma):
    r = reward.double().numpy()
    d = done.numpy()
    B, T = r.shape
    a = np.ones(B)
    b = np.zeros(B)
    for t in range(T - 1, -1, -1):
        at = np.where(d[:, t], 0.0, float(np.float32(gamma)))
        b = r[:, t] + at * b
        a = at * a
    return torch.from_numpy(np.stack([a, b], axis=1))


def _scan(reward, done, gamma, all_maps, rank, out=None):
    m = all_maps.numpy()
    y = np.zeros(m.shape[1])
    for k in range(m.shape[0] - 1, rank, -1):
        y = m[k, :, 1] + m[k, :, 0] * y
    r = reward.double().numpy()
    d = done.numpy()
    o = np.empty_like(r)
    g = float(np.float32(gamma))
    for t in range(r.shape[1] - 1, -1, -1):
        y = r[:, t] + np.where(d[:, t], 0.0, g) * y
        o[:, t] = y
    return torch.from_numpy(o)


def _worker(rank, world, port, q):
    sys.path.insert(0, str(REPO))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        ops = importlib.import_module("cuda-optimization-benchmark_b200.ops")
        d = importlib.import_module("cuda-optimization-benchmark_b200.dist")
        ops.reward_to_go_slice_maps = _maps   # the GPU kernels' stand-ins
        ops.reward_to_go_slice_scan = _scan
        B, T = 5, 1001
        g = torch.Generator().manual_seed(9)
        reward = torch.rand(B, T, generator=g)
        done = torch.rand(B, T, generator=g) < 0.01
        t0, t1 = d.time_range(T, world, rank)
        out = ops.reward_to_go_time_sharded(reward[:, t0:t1].contiguous(), done[:, t0:t1].contiguous(), 0.99)
        parts = [None] * world
        dist.all_gather_object(parts, (t0, t1, out.numpy()))
        if rank == 0:
            parts.sort(key=lambda p: p[0])
            assert parts[0][0] == 0 and parts[-1][1] == T
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            full = np.concatenate([p[2] for p in parts], axis=1)
            from oracle import exact
            ref = exact.reward_to_go({"reward": reward, "done": done, "gamma": 0.99})["output"]
            bad, worst = exact.within(full, ref, *exact.TOLERANCE["reward_to_go"])
            q.put((rank, "ok" if bad == 0 else f"bad {bad} {worst}"))
        else:
            q.put((rank, "ok"))
    except Exception as e:
        q.put((rank, f"error {type(e).__name__}: {str(e)[:200]}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.parametrize("world", [2, 3])
def test_time_sharded_host_logic(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(s == "ok" for _, s in got), got
