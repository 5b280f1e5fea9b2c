"""GPU: the per-task drop-in sources abi/<task>/solution.cu, built exactly as the reference grader
builds a solution (its nvcc line, -arch=sm_100a, a shim that includes solution.cu and exposes
`grader_entry(void** a)`), called through that entry with the grader's argument protocol (a[i] is
the address of argument i's value, graders/child.py:85-97), on golden cases, against the oracle.
The libraries are built by __graft_entry__.build() (abi/_build/<task>/kernel.so)."""
import ctypes
import importlib.util

import numpy as np
import pytest
import torch

from conftest import REPO, golden_cases
from oracle import exact, inputs

pytestmark = pytest.mark.gpu

ABI = REPO / "cuda-optimization-benchmark_b200" / "abi"
_spec = importlib.util.spec_from_file_location("b200_amalgamate_t", ABI / "amalgamate.py")
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


def call_entry(task, s):
    lib_path = am.BUILD / task / "kernel.so"
    if not lib_path.exists():
        pytest.skip(f"{lib_path} not built (run __graft_entry__.build())")
    fn = ctypes.CDLL(str(lib_path)).grader_entry
    fn.argtypes = [ctypes.POINTER(ctypes.c_void_p)]
    fn.restype = None
    dev = {k: v.cuda() for k, v in s.items() if isinstance(v, torch.Tensor)}
    outs = {k: torch.empty(shp(s), dtype=dt, device="cuda") for k, (dt, shp) in OUTPUTS[task].items()}
    keep = []
    for ctype, name in am.params(task):
        if "*" in ctype:
            t = outs[name] if name in outs else dev[name]
            keep.append(ctypes.c_void_p(t.data_ptr()))
        else:
            keep.append(SCALAR[ctype.replace("const ", "").strip()](s[name]))
    arr = (ctypes.c_void_p * len(keep))(*[ctypes.addressof(v) for v in keep])
    fn(arr)
    torch.cuda.synchronize()
    return {k: v.cpu() for k, v in outs.items()}


CASES = [(t, cid, rec) for t in OUTPUTS for cid, rec in golden_cases(t)[:3]]


@pytest.mark.parametrize("task,cid,rec", CASES, ids=[f"{t}-{c}" for t, c, _ in CASES])
def test_grader_built_solution(task, cid, rec):
    s = inputs.task_inputs(task, rec["case"], int(rec["case"]["seed"]))
    got = call_entry(task, s)
    ref = exact.TASKS[task](s)
    atol, rtol = exact.TOLERANCE[task]
    for k, v in got.items():
        if task == "fp8_linear":
            have = exact.bf16_bits_to_f64(v.view(torch.int16).numpy().view(np.uint16))
            want = ref["output_f64"]
        else:
            have, want = v.double().numpy(), ref[k]
        bad, worst = exact.within(have, want, atol, rtol)
        assert bad == 0, (k, worst)
