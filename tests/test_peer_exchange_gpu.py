"""GPU, 2 devices: the fused multi-GPU RL step (b200_rl_step_exchange_async), one process per GPU,
each rank's PPO totals exchanged over NVLink peer memory inside the kernel.

- Every rank's PPO outputs are bit-identical to each other over several consecutive steps (the
  exchange alternates buffer halves by step), with and without entropy, with and without the
  inputs-ready declaration; they equal one GPU running the ranks' batches back to back within a
  few fp32 ulps (the ranks' totals are added in rank order, one GPU adds all chunk partials in one
  tree) and meet the fp64 oracle.
- Each rank's returns are bit-identical to reward_to_go on its own batch.
- With a per-rank sample count that is not a multiple of the chunk, the same holds.
- On a box with more than two GPUs, the same over all of them (up to 8 ranks).
Skipped on a box with fewer than two GPUs.
"""
import os
import socket

import pytest
import torch

from conftest import REPO

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(rank, B, T, n, ent, seed):
    g = torch.Generator(device="cpu").manual_seed(seed * 100 + rank)
    reward = torch.randn(B, T, generator=g)
    done = torch.rand(B, T, generator=g) < 0.01
    new = torch.randn(n, generator=g) * 0.5 - 1.0
    old = new + torch.randn(n, generator=g) * 0.1
    adv = torch.randn(n, generator=g)
    e = torch.rand(n, generator=g) * 2.0 if ent else None
    return reward, done, new, old, adv, e


def _worker(rank, world, port, B, T, n, ent, steps, q):
    import sys
    sys.path.insert(0, str(REPO))
    import importlib
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pkg = importlib.import_module("cuda-optimization-benchmark_b200")
        lib = pkg.load()
        ops = pkg.ops
        ex = ops.PeerExchange(world, rank, n)
        outs = []
        for step in range(steps):
            mine = [t.cuda() if t is not None else None for t in _inputs(rank, B, T, n, ent, step)]
            rtg, ppo = ops.rl_step_exchange(ex, mine[0], mine[1], 0.99, mine[2], mine[3], mine[4], 0.2, mine[5],
                                            inputs_ready=bool(step & 1))
            torch.cuda.synchronize()
            own_rtg = ops.reward_to_go(mine[0], mine[1], 0.99)
            single = None
            if rank == 0:
                parts = [_inputs(r, B, T, n, ent, step) for r in range(world)]
                cat = [torch.cat([p[i] for p in parts]).cuda() if parts[0][i] is not None else None for i in range(6)]
                _, single = ops.rl_step(cat[0], cat[1], 0.99, cat[2], cat[3], cat[4], 0.2, cat[5])
                single = single.cpu()
            outs.append((ppo.cpu(), torch.equal(rtg.cpu().view(torch.int32), own_rtg.cpu().view(torch.int32)), single))
            dist.barrier()  # keep the ranks in step: rank 0's extra check must not stall the other's wait
        dist.barrier()
        ex.close()
        dist.barrier()
        q.put((rank, outs, lib.b200_device_fault()))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e), -1))
    finally:
        dist.destroy_process_group()


def _run(B, T, n, ent, steps=3, world=2):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, B, T, n, ent, steps, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict()
    for _ in procs:
        r, outs, fault = q.get(timeout=240)
        assert not isinstance(outs, str), outs
        assert fault == 0, "a bounded device wait gave up"
        res[r] = outs
    for p in procs:
        p.join(timeout=60)
    return res


def _check_against_oracle(ppo, parts, ent):
    import numpy as np
    from oracle import exact
    s = {"current_log_prob": torch.cat([p[2] for p in parts]), "old_log_prob": torch.cat([p[3] for p in parts]),
         "advantage": torch.cat([p[4] for p in parts]), "clip_epsilon": 0.2}
    ref = exact.ppo_clip(s, entropy=torch.cat([p[5] for p in parts]) if ent else None)["output"]
    bad, worst = exact.within(ppo.double().numpy(), np.asarray(ref), 1e-5, 1e-4)
    assert bad == 0, worst


@pytest.mark.timeout(300)
@pytest.mark.parametrize("ent", [True, False], ids=["ent", "noent"])
def test_exchange_ranks_agree_and_match_one_gpu(ent):
    B, T = 64, 512
    n = 8 * 4096
    res = _run(B, T, n, ent, steps=4)
    for step in range(4):
        p0, rtg_ok0, single = res[0][step]
        p1, rtg_ok1, _ = res[1][step]
        assert rtg_ok0 and rtg_ok1
        assert torch.equal(p0.view(torch.int32), p1.view(torch.int32)), (step, p0, p1)
        # The same sums in another order: a few fp32 ulps at most.
        assert torch.allclose(p0, single, rtol=4e-7, atol=1e-9), (step, p0, single)
        _check_against_oracle(p0, [_inputs(r, B, T, n, ent, step) for r in range(2)], ent)


@pytest.mark.timeout(300)
def test_exchange_ragged_ranks_agree():
    B, T, n = 3, 1000, 3 * 4096 + 777
    res = _run(B, T, n, True, steps=2)
    for step in range(2):
        p0, _, _ = res[0][step]
        p1, _, _ = res[1][step]
        assert torch.equal(p0.view(torch.int32), p1.view(torch.int32))
        _check_against_oracle(p0, [_inputs(r, B, T, n, True, step) for r in range(2)], True)


@pytest.mark.timeout(400)
def test_exchange_all_gpus():
    """Every GPU of the box as one rank each (3 to 8 ranks): all ranks agree bit for bit, meet the
    fp64 oracle over all ranks' samples and match one GPU within a few ulps."""
    world = min(torch.cuda.device_count(), 8)
    if world < 3:
        pytest.skip("needs more than two GPUs")
    B, T, n = 16, 700, 5 * 4096 + 123
    res = _run(B, T, n, True, steps=3, world=world)
    for step in range(3):
        p0, rtg_ok0, single = res[0][step]
        assert rtg_ok0
        for r in range(1, world):
            pr, rtg_ok, _ = res[r][step]
            assert rtg_ok
            assert torch.equal(p0.view(torch.int32), pr.view(torch.int32)), (step, r, p0, pr)
        assert torch.allclose(p0, single, rtol=4e-7, atol=1e-9), (step, p0, single)
        _check_against_oracle(p0, [_inputs(r, B, T, n, True, step) for r in range(world)], True)
