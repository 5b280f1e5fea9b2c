"""GPU: robust-L1 over GPUs with the chunk-partial exchange fused into the kernel
(b200_robust_l1_exchange_async), one process per GPU, partials pushed over NVLink peer memory.

- One rank (any box): the exchange form is bit-identical to b200_robust_l1_async over the same
  range, over consecutive calls (the exchange alternates buffer halves by call), for ragged sizes
  (a partial last chunk) and a single element.
- Two or more ranks (boxes with several GPUs; skipped otherwise): every rank's output is the same
  bits, those of one GPU over the concatenated range, over consecutive calls, for an even and a
  ragged split, and meets the fp64 oracle at the BASELINE tolerance (rtol 1e-5).
"""
import os
import socket

import pytest
import torch

from conftest import REPO, pkg

pytestmark = pytest.mark.gpu


def _data(n, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(n, generator=g), torch.randn(n, generator=g)


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    p = pkg()
    p.load()
    return p.ops


@pytest.mark.parametrize("n", [1, 8192, (1 << 20) + 123, 1 << 24])
def test_one_rank_matches_single_gpu(ops, n):
    ex = ops.RobustL1Exchange(1, 0, n, swap=lambda h: [h])
    try:
        for call in range(3):
            a, b = (t.cuda() for t in _data(n, 1000 * call + n % 997))
            got = ops.robust_l1_exchange(ex, a, b)
            want = ops.robust_l1(a, b)
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int32), want.view(torch.int32)), (call, float(got), float(want))
    finally:
        torch.cuda.synchronize()
        ex.close()
    assert pkg().load().b200_device_fault() == 0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, steps, q):
    import sys
    sys.path.insert(0, str(REPO))
    import importlib
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p = importlib.import_module("cuda-optimization-benchmark_b200")
        lib = p.load()
        ops = p.ops
        ex = ops.RobustL1Exchange(world, rank, n)
        lo, hi = ex.shard_range()
        outs = []
        for step in range(steps):
            a, b = _data(n, 7 * step + 1)
            got = ops.robust_l1_exchange(ex, a[lo:hi].cuda(), b[lo:hi].cuda())
            torch.cuda.synchronize()
            whole = ops.robust_l1(a.cuda(), b.cuda()).cpu() if rank == 0 else None
            outs.append((got.cpu(), whole))
            dist.barrier()
        dist.barrier()
        ex.close()
        dist.barrier()
        q.put((rank, outs, lib.b200_device_fault()))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e), -1))
    finally:
        dist.destroy_process_group()


def _run(n, world, steps=3):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = torch.multiprocessing.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, steps, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, outs, fault = q.get(timeout=240)
        assert not isinstance(outs, str), outs
        assert fault == 0, "a bounded device wait gave up"
        res[r] = outs
    for p in procs:
        p.join(timeout=60)
    return res


def _check(res, world, n, steps):
    from oracle import exact
    for step in range(steps):
        got0, whole = res[0][step]
        assert torch.equal(got0.view(torch.int32), whole.view(torch.int32)), (step, float(got0), float(whole))
        for r in range(1, world):
            assert torch.equal(res[r][step][0].view(torch.int32), got0.view(torch.int32)), (step, r)
        a, b = _data(n, 7 * step + 1)
        ref = float(exact.pow_abs_sqrt_mean({"inp": a, "target": b})["output"])
        assert abs(float(got0) - ref) <= 1e-5 * abs(ref)


@pytest.mark.timeout(300)
@pytest.mark.parametrize("n", [1 << 22, (1 << 22) + 5 * 8192 + 77], ids=["even", "ragged"])
def test_two_ranks_bit_identical_to_one_gpu(n):
    res = _run(n, 2)
    _check(res, 2, n, 3)


@pytest.mark.timeout(400)
def test_all_gpus_bit_identical_to_one_gpu():
    world = min(torch.cuda.device_count(), 8)
    if world < 3:
        pytest.skip("needs more than two GPUs")
    n = (1 << 23) + 3 * 8192 + 11
    res = _run(n, world)
    _check(res, world, n, 3)
