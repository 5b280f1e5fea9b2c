"""GPU: the reference grader's call counter around the drop-ins.

The reference grader preloads graders/interpose.c into the graded process and counts, around each
call of the answer only, the CUDA runtime calls its task header forbids: allocations and frees,
host copies, device-wide synchronizations, work on a stream other than the caller's, and launches
(graders/interpose.c:14-23,46-55,104-115; armed by graders/child.py:103-118).  Its target is no
allocation, host copy or device synchronization from the second call on (a library may allocate
its scratch once, on the first call).

oracle/ref_build.py compiles interpose.c from the reference's sources with the grader's own gcc
line into oracle/_ref/interpose.so; each case runs tests/call_count_child.py in a fresh process
with that library preloaded, on the grader-built drop-in (abi/_build/<task>/kernel.so, built with
`-cudart shared` exactly as the grader builds it, so every runtime call passes the counter), over
the grader's three calls (set A, set B, set A) on guarded buffers.  The reference's expert library
runs the same way beside it when it is present; its counts are recorded, not asserted.

Asserted for the drop-ins: calls 2 and 3 make no allocation, host copy, device-wide or stream
synchronization and put no work on another stream; they launch the same number of kernels as each
other, which is the count pinned per task below; guards and inputs are intact and call 3 repeats
call 1's bits.  The per-task counts are written to the file named by B200_CALL_COUNTS when set.
"""
import json
import os
import subprocess
import sys

import pytest

from conftest import REPO, golden_cases
from oracle import ref_build

pytestmark = pytest.mark.gpu

CHILD = REPO / "tests" / "call_count_child.py"
ABI_BUILD = REPO / "cuda-optimization-benchmark_b200" / "abi" / "_build"
TASKS = ["pow_abs_sqrt_mean", "ppo_clip", "reward_to_go", "leaky", "efficient_kan", "fp8_linear"]
# Kernels one call launches: one per op, except KAN (weight planes with the row scales, activation
# planes, the tensor-core GEMM).
LAUNCHES = {"pow_abs_sqrt_mean": 1, "ppo_clip": 1, "reward_to_go": 1, "leaky": 1, "efficient_kan": 3,
            "fp8_linear": 1}
ROWS = []


def _cases():
    out = []
    for t in TASKS:
        cases = golden_cases(t)
        small = next(rec for cid, rec in cases if not rec["case"].get("timed"))
        timed = next(rec for cid, rec in cases if rec["case"].get("timed"))
        out += [(t, small), (t, timed)]
    return out


CASES = _cases()


def run_child(task, case, lib):
    env = dict(os.environ, LD_PRELOAD=str(ref_build.counter_library()))
    r = subprocess.run([sys.executable, str(CHILD), task, json.dumps(case), str(lib)], capture_output=True,
                       text=True, timeout=600, env=env, cwd=str(REPO))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("task,rec", CASES, ids=[f"{t}-{r['case']['name']}" for t, r in CASES])
def test_call_counts(task, rec):
    if not ref_build.counter_library().exists():
        pytest.skip("oracle/_ref/interpose.so not built (needs the reference checkout at build time)")
    lib = ABI_BUILD / task / "kernel.so"
    if not lib.exists():
        pytest.skip(f"{lib} not built (run __graft_entry__.build())")
    ours = run_child(task, rec["case"], lib)
    assert ours["counter"], "the call counter did not load"
    row = {"task": task, "case": rec["case"]["name"], "b200": [c["count"] for c in ours["calls"]]}
    exp_lib = ref_build.library(task)
    if exp_lib.exists():
        row["expert"] = [c["count"] for c in run_child(task, rec["case"], exp_lib)["calls"]]
    ROWS.append(row)
    for c in ours["calls"]:
        assert c["guards_ok"] and c["inputs_unchanged"], ours
    assert ours["identical_repeat"], "call 3 did not repeat call 1's bits"
    c2, c3 = ours["calls"][1]["count"], ours["calls"][2]["count"]
    for c in (c2, c3):
        for k in ("alloc", "host_copy", "device_sync", "other_stream", "stream_sync"):
            assert c[k] == 0, (k, c)
    assert c2["launch"] == c3["launch"] == LAUNCHES[task], (c2, c3)


def test_zz_call_count_table():
    if not ROWS:
        pytest.skip("no counts collected")
    keys = ["alloc", "host_copy", "device_sync", "other_stream", "stream_sync", "launch"]
    lines = [f"{'task / case':44s} {'side':7s} " + " ".join(f"{k:>12s}" for k in keys) + "   (call 1 / 2 / 3)"]
    for r in ROWS:
        for side in ("b200", "expert"):
            if side in r:
                cells = " ".join(f"{'/'.join(str(c[k]) for c in r[side]):>12s}" for k in keys)
                lines.append(f"{r['task'] + ' ' + r['case']:44s} {side:7s} {cells}")
    print("\n" + "\n".join(lines))
    out = os.environ.get("B200_CALL_COUNTS")
    if out:
        with open(out, "w") as f:
            json.dump(ROWS, f, indent=1)
