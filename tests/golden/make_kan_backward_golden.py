"""Generate tests/golden/efficient_kan_backward.json: gradients of the reference's own KAN forward.

Runs only where the reference checkout is present (its path is the first argument, or the
REFERENCE_ROOT environment variable); the GPU box never runs it.  For each case below it builds the
inputs with oracle.inputs.task_inputs (the reference's make_inputs, draw for draw), an incoming
gradient grad_out ~ N(0, 1) [B, O] from torch.Generator().manual_seed(seed + 1), and runs torch
autograd in fp64 through the reference's `_forward` (tasks/efficient_kan/reference.py:42-46), as
its `reference_exact` does for the forward; it records every gradient value.

Usage: python tests/golden/make_kan_backward_golden.py /path/to/reference
"""
import hashlib
import importlib.util
import json
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import inputs  # noqa: E402

CASES = [
    {"name": "B4_I5_O3_G8", "B": 4, "I": 5, "O": 3, "grid_size": 8, "spline_order": 3, "seed": 11},
    {"name": "B3_I7_O2_G5_range2", "B": 3, "I": 7, "O": 2, "grid_size": 5, "spline_order": 3, "x_range": 2.0,
     "seed": 12},
    {"name": "B6_I4_O5_G4_K2", "B": 6, "I": 4, "O": 5, "grid_size": 4, "spline_order": 2, "seed": 13},
    {"name": "B1_I1_O1_G8", "B": 1, "I": 1, "O": 1, "grid_size": 8, "spline_order": 3, "seed": 14},
    {"name": "B9_I33_O7_G5", "B": 9, "I": 33, "O": 7, "grid_size": 5, "spline_order": 3, "seed": 15},
]


def grad_out_for(case):
    g = torch.Generator().manual_seed(int(case["seed"]) + 1)
    return torch.randn(case["B"], case["O"], generator=g)


def main(root):
    spec = importlib.util.spec_from_file_location("ref_kan", Path(root) / "tasks" / "efficient_kan" / "reference.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    out = []
    for case in CASES:
        s = inputs.task_inputs("efficient_kan", case, int(case["seed"]))
        d = {k: s[k].double().requires_grad_(k != "grid") for k in
             ("x", "grid", "base_weight", "spline_weight", "spline_scaler")}
        y = ref._forward(d["x"], d["grid"], d["base_weight"], d["spline_weight"], d["spline_scaler"],
                         s["spline_order"])
        go = grad_out_for(case)
        y.backward(go.double())
        rec = {"case": case,
               "input_sha256": hashlib.sha256(b"".join(s[k].numpy().tobytes() for k in
                                                       ("x", "grid", "base_weight", "spline_weight",
                                                        "spline_scaler"))).hexdigest(),
               "grad_out_sha256": hashlib.sha256(go.numpy().tobytes()).hexdigest()}
        for k, name in (("x", "grad_x"), ("base_weight", "grad_base_weight"),
                        ("spline_weight", "grad_spline_weight"), ("spline_scaler", "grad_spline_scaler")):
            rec[name] = d[k].grad.reshape(-1).tolist()
        out.append(rec)
    path = HERE / "efficient_kan_backward.json"
    path.write_text(json.dumps({"source": "torch autograd (fp64) through tasks/efficient_kan/reference.py:42-46",
                                "cases": out}) + "\n")
    print(path, len(out), "cases")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT", "/root/reference"))
