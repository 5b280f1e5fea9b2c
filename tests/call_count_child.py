"""Child process of tests/test_call_counts_gpu.py (run with the reference grader's call counter,
oracle/_ref/interpose.so, in LD_PRELOAD; never imported by pytest).

    python tests/call_count_child.py <task> <case json> [<library>]

Loads a drop-in library (default: the grader-built abi/_build/<task>/kernel.so) and makes the
grader's three calls (set A, set B = seed + 7919, set A again; graders/child.py:178-207) on guarded
buffers, with the counter armed around each call only (graders/child.py:103-118).  Prints one JSON
line: per call the counts of allocations, host copies, device-wide synchronizations, off-stream
work, stream synchronizations and launches (graders/interpose.c:14), the guard and input checks,
and whether call 3 repeated call 1's bits.
"""
import ctypes
import importlib.util
import json
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

from harness import SET_B, Guarded, as_bytes, guarded_like  # noqa: E402
from oracle import inputs  # noqa: E402

ABI = REPO / "cuda-optimization-benchmark_b200" / "abi"
_spec = importlib.util.spec_from_file_location("b200_amalgamate_cc", ABI / "amalgamate.py")
am = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(am)

SCALAR = {"int64_t": ctypes.c_int64, "int32_t": ctypes.c_int32, "float": ctypes.c_float}
OUTPUTS = {"pow_abs_sqrt_mean": {"output": (torch.float32, lambda s: ())},
           "ppo_clip": {"output": (torch.float32, lambda s: (6,))},
           "reward_to_go": {"output": (torch.float32, lambda s: (s["B"], s["T"]))},
           "leaky": {"spikes": (torch.float32, lambda s: (s["T"], s["B"], s["H"])),
                     "final_mem": (torch.float32, lambda s: (s["B"], s["H"]))},
           "efficient_kan": {"out": (torch.float32, lambda s: (s["B"], s["O"]))},
           "fp8_linear": {"output": (torch.bfloat16, lambda s: (s["M"], s["N"]))}}
NAMES = ["alloc", "host_copy", "device_sync", "other_stream", "stream_sync", "launch"]


def counter():
    lib = ctypes.CDLL(None)
    try:
        fns = (lib.grader_counter_arm, lib.grader_counter_reset, lib.grader_counter_read, lib.grader_counter_n)
    except AttributeError:
        return None
    arm, reset, read, n = fns
    k = n()

    def wrap(fn):
        reset()
        arm(1)
        try:
            fn()
        finally:
            arm(0)
        c = (ctypes.c_long * k)()
        read(c)
        return {NAMES[i]: int(c[i]) for i in range(min(k, len(NAMES)))}
    return wrap


def main():
    task, case = sys.argv[1], json.loads(sys.argv[2])
    path = Path(sys.argv[3]) if len(sys.argv) > 3 else am.BUILD / task / "kernel.so"
    torch.cuda.init()
    torch.zeros(1, device="cuda")
    count = counter()
    fn = ctypes.CDLL(str(path)).grader_entry
    fn.argtypes = [ctypes.POINTER(ctypes.c_void_p)]
    fn.restype = None
    seed = int(case["seed"])
    sets = [inputs.task_inputs(task, case, seed), inputs.task_inputs(task, case, seed + SET_B)]
    ins = [n for c, n in am.params(task) if "*" in c and n not in OUTPUTS[task]]
    bufs = {k: guarded_like(sets[0][k]) for k in ins}
    for k, (dt, shp) in OUTPUTS[task].items():
        shape = shp(sets[0])
        nb = int(torch.empty(shape, dtype=dt).numel()) * torch.empty((), dtype=dt).element_size()
        bufs[k] = Guarded(nb, dt, shape)
    calls, outs = [], []
    for idx in (0, 1, 0):
        s = sets[idx]
        for k in OUTPUTS[task]:
            bufs[k].poison()
        for k in ins:
            bufs[k].load(s[k])
        torch.cuda.synchronize()
        keep = []
        for ctype, name in am.params(task):
            if "*" in ctype:
                keep.append(bufs[name].ptr)
            else:
                keep.append(SCALAR[ctype.replace("const ", "").strip()](s[name]))
        arr = (ctypes.c_void_p * len(keep))(*[ctypes.addressof(v) for v in keep])
        c = count(lambda: fn(arr)) if count else None
        torch.cuda.synchronize()
        calls.append({"count": c, "guards_ok": all(b.guards_ok() for b in bufs.values()),
                      "inputs_unchanged": all(torch.equal(as_bytes(bufs[k].t), as_bytes(s[k])) for k in ins)})
        outs.append({k: as_bytes(bufs[k].t).clone() for k in OUTPUTS[task]})
    same = all(torch.equal(outs[0][k], outs[2][k]) for k in OUTPUTS[task])
    print(json.dumps({"task": task, "case": case.get("name"), "counter": count is not None, "calls": calls,
                      "identical_repeat": same}), flush=True)


if __name__ == "__main__":
    main()
