"""CPU: the planted-mistake check of the reference grader, mirrored on the host.

The reference grader proves its own checks by grading deliberately wrong kernels made from each
task's expert (graders/planted.py:16-53): a wrong first output value must fail as "wrong value", a
kernel that caches its first result as "stale state", a write one byte before the output as
"out-of-bounds write".  Here the same mistakes are planted in a host-side stand-in of each drop-in
(the oracle's result written into guarded host buffers) and run through this repository's copy of
the grader's three-call protocol and verdict (tests/harness.py: protocol_record, case_label, which
the GPU parity tests use for the real kernels).  Each plant must get its label, and the unplanted
stand-in must pass: the checks that guard the GPU results are shown to catch these mistakes.
Two more labels of the same verdict are covered: an output never written ("unwritten output") and
an input overwritten ("input modified").  No GPU is involved: nothing is planted in a kernel.
"""
import numpy as np
import pytest
import torch

from conftest import golden_cases
from harness import GUARD, SET_B, case_label, protocol_record
from oracle import exact, inputs

OUT_SPECS = {"pow_abs_sqrt_mean": {"output": (torch.float32, lambda s: ())},
             "ppo_clip": {"output": (torch.float32, lambda s: (6,))},
             "reward_to_go": {"output": (torch.float32, lambda s: (s["B"], s["T"]))},
             "leaky": {"spikes": (torch.float32, lambda s: (s["T"], s["B"], s["H"])),
                       "final_mem": (torch.float32, lambda s: (s["B"], s["H"]))},
             "efficient_kan": {"out": (torch.float32, lambda s: (s["B"], s["O"]))},
             "fp8_linear": {"output": (torch.bfloat16, lambda s: (s["M"], s["N"]))}}
IN_NAMES = {"pow_abs_sqrt_mean": ["inp", "target"],
            "ppo_clip": ["current_log_prob", "old_log_prob", "advantage"],
            "reward_to_go": ["reward", "done"],
            "leaky": ["input_current", "mem0", "beta", "threshold"],
            "efficient_kan": ["x", "grid", "base_weight", "spline_weight", "spline_scaler"],
            "fp8_linear": ["x_fp8", "w_fp8", "bias"]}
EXPECT = {"none": None, "wrong_value": "wrong value", "cached_result": "stale state",
          "oob_write": "out-of-bounds write", "unwritten": "unwritten output", "input_modified": "input modified"}


def oracle_outputs(task, s):
    """The oracle's outputs for input set `s`, as tensors of the drop-in's output dtypes."""
    ref = exact.TASKS[task](s)
    if task == "fp8_linear":
        return {"output": torch.from_numpy(ref["output"].astype(np.int16)).view(torch.bfloat16)}
    return {k: torch.from_numpy(np.asarray(ref[k], dtype=np.float32)) for k in OUT_SPECS[task]}


def stand_in(task, plant):
    """A host-side stand-in of the drop-in with one planted mistake (or none)."""
    state = {"calls": 0}

    def call(bufs, s):
        state["calls"] += 1
        if plant == "cached_result" and state["calls"] > 1:
            return  # assumes the inputs never change between calls (graders/planted.py:24-30)
        if plant == "input_modified":
            first = IN_NAMES[task][0]
            bufs[first].raw[GUARD] ^= 0x01
        if plant == "unwritten":
            return
        for k, v in oracle_outputs(task, {**s, **{n: bufs[n].t.clone() for n in IN_NAMES[task]}}).items():
            bufs[k].t.copy_(v.reshape(bufs[k].t.shape))
        out = next(iter(OUT_SPECS[task]))
        if plant == "wrong_value":  # first output element far from any reference (planted.py:9-11)
            bufs[out].t.reshape(-1)[0] = 12345.0
        if plant == "oob_write":     # one byte before the output (planted.py:31-36)
            bufs[out].raw[GUARD - 1] = 0
    return call


def bad_mask(task, got, s):
    atol, rtol = exact.TOLERANCE[task]
    want = exact.TASKS[task](s)
    res = {}
    for k, v in got.items():
        if task == "fp8_linear":
            have = exact.bf16_bits_to_f64(v.view(torch.int16).numpy().view(np.uint16))
            ref = want["output_f64"]
        else:
            have, ref = v.double().numpy(), np.asarray(want[k], dtype=np.float64)
        ok = np.abs(have - ref) <= atol + rtol * np.abs(ref)
        ok |= np.isnan(have) & np.isnan(ref)
        res[k] = torch.from_numpy(~ok.reshape(-1))
    return res


def _small_case(task):
    return next(rec for cid, rec in golden_cases(task) if rec["case"].get("small"))


CASES = [(t, p) for t in OUT_SPECS for p in EXPECT]


@pytest.mark.parametrize("task,plant", CASES, ids=[f"{t}-{p}" for t, p in CASES])
def test_planted_mistake_gets_its_label(task, plant):
    case = _small_case(task)["case"]
    seed = int(case["seed"])
    sets = [inputs.task_inputs(task, case, seed), inputs.task_inputs(task, case, seed + SET_B)]
    outs = {k: (dt, shp(sets[0])) for k, (dt, shp) in OUT_SPECS[task].items()}
    rec = protocol_record(stand_in(task, plant), sets, IN_NAMES[task], outs, device="cpu")
    bad1 = bad_mask(task, rec["calls"][0]["outputs"], sets[0])
    bad2 = bad_mask(task, rec["calls"][1]["outputs"], sets[1])
    assert case_label(rec, bad1, bad2) == EXPECT[plant]
    if plant == "none":
        assert rec["identical_repeat"]
