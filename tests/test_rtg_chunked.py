"""Reward-to-go parallel along T (b200_reward_to_go_chunked_async) and sharded along T across ranks
(b200_reward_to_go_slice_maps_async + an all-gather + b200_reward_to_go_slice_scan_async).

No reference counterpart (the reference runs one row per block); the oracle is the reference's own
reward_to_go oracle (oracle.exact.reward_to_go, fp64), at the task tolerance (1e-5 / 1e-5).

GPU, through the C ABI:
- the chunked scan against the oracle on rows shorter than, equal to and longer than one
  1056-step chunk, up to 100,003 steps, with done as bytes and as bits (the two bit-identical);
- the time-sharded form with 2, 3, 4 and 8 ranks emulated on one GPU (each rank's slice a separate
  buffer and workspace, slice maps stacked in rank order as the all-gather would), with ragged
  slice lengths, against the oracle and against the one-GPU chunked scan;
- with several GPUs, the same through torch.distributed (NCCL) with one process per GPU;
- the one-launch form's carry paths at large sizes (CTA ranges across rows, many superblocks, the
  global-memory path) against the one-warp-per-row scan, and its grid barrier's bounded wait run
  out on purpose (the device fault bit, then recovery);
- status codes.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import REPO, golden_cases, pkg
from oracle import exact, inputs

pytestmark = pytest.mark.gpu
TOL = exact.TOLERANCE["reward_to_go"]


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    p = pkg()
    p.load()
    return p.ops


def make(B, T, seed, p=0.01):
    g = torch.Generator().manual_seed(seed)
    r = torch.rand(B, T, generator=g)
    d = torch.rand(B, T, generator=g) < p
    return r, d


def check(got, r, d, gamma):
    ref = exact.reward_to_go({"reward": r, "done": d, "gamma": gamma})["output"]
    bad, worst = exact.within(got.cpu().double().numpy(), ref, *TOL)
    assert bad == 0, worst


SHAPES = [(1, 1), (3, 31), (2, 1056), (2, 1057), (5, 2111), (1, 8000), (3, 9000), (64, 1000), (2, 100_003)]


@pytest.mark.parametrize("B,T", SHAPES, ids=[f"B{b}_T{t}" for b, t in SHAPES])
@pytest.mark.parametrize("gamma", [0.99, 0.5])
def test_chunked_against_oracle(ops, B, T, gamma):
    r, d = make(B, T, seed=B * 7 + T)
    rc, dc = r.cuda(), d.cuda()
    got = ops.reward_to_go_chunked(rc, dc, gamma).clone()
    got_bits = ops.reward_to_go_chunked(rc, ops.pack_done(dc), gamma)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), got_bits.view(torch.int32))
    check(got, r, d, gamma)


@pytest.mark.parametrize("cid,rec", golden_cases("reward_to_go"), ids=[c for c, _ in golden_cases("reward_to_go")])
def test_chunked_golden(ops, cid, rec):
    s = inputs.task_inputs("reward_to_go", rec["case"], int(rec["case"]["seed"]))
    got = ops.reward_to_go_chunked(s["reward"].cuda(), s["done"].cuda(), s["gamma"])
    torch.cuda.synchronize()
    check(got, s["reward"], s["done"], s["gamma"])


LARGE = [
    (8, 1 << 21),   # CTA ranges that cross rows; 8 superblocks per row (shared-memory carry path)
    (1, 1 << 24),   # one row over every CTA: up to 62 superblocks before a CTA's range
    (1, 70_000_000),  # more than 256 superblocks in the row: the global-memory carry path
    (4096, 160_000),  # more than 512 blocks per CTA: the global-memory carry path over many rows
]


@pytest.mark.parametrize("B,T", LARGE, ids=[f"B{b}_T{t}" for b, t in LARGE])
def test_chunked_large_paths(ops, B, T):
    """Every carry path of the one-launch form against the one-warp-per-row scan (each within the
    task tolerance of the fp64 oracle, so within twice of each other), with done as bytes and as
    bits (the same bits), and run twice (the same bits)."""
    g = torch.Generator(device="cuda").manual_seed(B + T)
    r = torch.rand(B, T, device="cuda", generator=g)
    d = torch.rand(B, T, device="cuda", generator=g) < 0.001
    ref = ops.reward_to_go(r, d, 0.99)
    got = ops.reward_to_go_chunked(r, d, 0.99).clone()
    again = ops.reward_to_go_chunked(r, d, 0.99).clone()
    bits = ops.reward_to_go_chunked(r, ops.pack_done(d), 0.99)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), again.view(torch.int32))
    assert torch.equal(got.view(torch.int32), bits.view(torch.int32))
    atol, rtol = TOL
    err = ((got - ref).abs() - 2 * (atol + rtol * ref.abs())).max().item()
    assert err <= 0, err
    del r, d, ref, got, again, bits
    torch.cuda.empty_cache()


def test_grid_barrier_wait_runs_out(ops):
    """Failure detection of the one-launch form's grid barrier, without a GPU fault: a workspace
    whose arrival count is not a multiple of the grid size (one that was not zero-filled before its
    first use) leaves a CTA waiting for a count that never comes.  Its bounded wait gives up after
    2 s and sets bit 0 of the device fault word; the launch completes (its outputs are not
    meaningful), and a zero-filled workspace works again."""
    lib = pkg().load()
    B, T = 4, 50_000
    r, d = make(B, T, seed=11)
    rc, dc = r.cuda(), d.cuda()
    nbytes = lib.b200_reward_to_go_chunked_workspace_bytes(B, T)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    ws[:8].view(torch.int64).fill_(1)
    out = torch.empty_like(rc)
    torch.cuda.synchronize()
    lib.b200_device_fault()  # read and clear
    st = lib.b200_reward_to_go_chunked_async(rc.data_ptr(), dc.data_ptr(), 0, 0.99, B, T, out.data_ptr(),
                                             ws.data_ptr(), nbytes, None)
    assert st == 0
    torch.cuda.synchronize()
    fault = lib.b200_device_fault()
    assert fault > 0 and fault & 1, fault
    ws.zero_()
    st = lib.b200_reward_to_go_chunked_async(rc.data_ptr(), dc.data_ptr(), 0, 0.99, B, T, out.data_ptr(),
                                             ws.data_ptr(), nbytes, None)
    assert st == 0
    torch.cuda.synchronize()
    assert lib.b200_device_fault() == 0
    check(out, r, d, 0.99)


def emulate(ops, r, d, gamma, cuts, bits=False):
    """Ranks emulated on one GPU: rank k holds steps [cuts[k], cuts[k+1]) of every row."""
    lib = pkg().load()
    world = len(cuts) - 1
    B = r.shape[0]
    parts, wss, maps = [], [], []
    for k in range(world):
        rk = r[:, cuts[k]:cuts[k + 1]].contiguous().cuda()
        dk = d[:, cuts[k]:cuts[k + 1]].contiguous().cuda()
        if bits:
            dk = ops.pack_done(dk)
        Tk = rk.shape[1]
        ws = torch.empty(max(1, lib.b200_reward_to_go_chunked_workspace_bytes(B, Tk)), dtype=torch.uint8,
                         device="cuda")
        m = torch.empty((B, 2), dtype=torch.float64, device="cuda")
        assert lib.b200_reward_to_go_slice_maps_async(rk.data_ptr(), dk.data_ptr(), int(bits), gamma, B, Tk,
                                                      m.data_ptr(), ws.data_ptr(), ws.numel(), None) == 0
        parts.append((rk, dk, Tk))
        wss.append(ws)
        maps.append(m)
    all_maps = torch.stack(maps)
    outs = []
    for k, (rk, dk, Tk) in enumerate(parts):
        o = torch.empty_like(rk)
        assert lib.b200_reward_to_go_slice_scan_async(rk.data_ptr(), dk.data_ptr(), int(bits), gamma, B, Tk,
                                                      all_maps.data_ptr(), world, k, o.data_ptr(), wss[k].data_ptr(),
                                                      wss[k].numel(), None) == 0
        outs.append(o)
    torch.cuda.synchronize()
    return torch.cat(outs, dim=1)


CUTS = [[0, 500, 1000], [0, 1, 2000, 4001], [0, 1056, 2112, 3168, 4224], [0, 3, 1500, 1501, 7000, 9000, 9001, 12000,
                                                                          20000]]


@pytest.mark.parametrize("cuts", CUTS, ids=[f"world{len(c) - 1}" for c in CUTS])
@pytest.mark.parametrize("bits", [False, True], ids=["bytes", "bits"])
def test_time_sharded_emulated(ops, cuts, bits):
    B, T = 6, cuts[-1]
    r, d = make(B, T, seed=T + len(cuts), p=0.002)
    got = emulate(ops, r, d, 0.99, cuts, bits=bits)
    check(got, r, d, 0.99)
    one = ops.reward_to_go_chunked(r.cuda(), d.cuda(), 0.99)
    torch.cuda.synchronize()
    np.testing.assert_allclose(got.cpu().numpy(), one.cpu().numpy(), rtol=2e-6, atol=1e-6)


def test_time_sharded_no_done_long_memory(ops):
    """gamma = 1 and no done flag: every carry crosses every rank boundary."""
    B, T = 2, 6000
    r, _ = make(B, T, seed=3)
    d = torch.zeros(B, T, dtype=torch.bool)
    got = emulate(ops, r, d, 1.0, [0, 1000, 3000, 6000])
    check(got, r, d, 1.0)


def test_status_codes(ops):
    lib = pkg().load()
    x = torch.zeros(64, device="cuda")
    p = x.data_ptr()
    assert lib.b200_reward_to_go_chunked_workspace_bytes(-1, 5) == -1
    assert lib.b200_reward_to_go_chunked_async(p, p, 0, 0.9, 2, 4, p, p, 8, None) == 4
    assert lib.b200_reward_to_go_chunked_async(p, None, 0, 0.9, 2, 4, p, p, 4096, None) == 1
    assert lib.b200_reward_to_go_slice_maps_async(p, p, 0, 0.9, 2, 0, p, p, 4096, None) == 1
    assert lib.b200_reward_to_go_slice_scan_async(p, p, 0, 0.9, 2, 4, p, 2, 2, p, p, 4096, None) == 1


# ------------------------------------------------------------------------- several GPUs (NCCL)
WORKER = r"""
import os, sys, torch, torch.distributed as dist
sys.path.insert(0, os.environ["B200_REPO"])
from conftest import pkg
from oracle import exact
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=60))
ops = pkg().ops
B, T_loc = 4, 3000
g = torch.Generator().manual_seed(5)
r = torch.rand(B, T_loc * world, generator=g)
d = torch.rand(B, T_loc * world, generator=g) < 0.003
mine = slice(rank * T_loc, (rank + 1) * T_loc)
out = ops.reward_to_go_time_sharded(r[:, mine].contiguous().cuda(), d[:, mine].contiguous().cuda(), 0.99)
full = [torch.empty_like(out) for _ in range(world)]
dist.all_gather(full, out)
got = torch.cat(full, dim=1).cpu().double().numpy()
ref = exact.reward_to_go({"reward": r, "done": d, "gamma": 0.99})["output"]
bad, worst = exact.within(got, ref, *exact.TOLERANCE["reward_to_go"])
dist.barrier()
dist.destroy_process_group()
assert bad == 0, worst
print("ok", rank)
"""


def test_time_sharded_nccl(tmp_path):
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs two GPUs")
    world = min(n, 4)
    script = tmp_path / "worker.py"
    script.write_text(WORKER)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, B200_REPO=str(REPO), NCCL_NVLS_ENABLE="0",
               PYTHONPATH=os.pathsep.join([str(REPO), str(REPO / "tests")]))
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={port}", str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert r.stdout.count("ok") == world
