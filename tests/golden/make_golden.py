"""Generate the golden fixtures in this folder from the reference's own oracle.

Runs only where the reference checkout is present (its path is the first argument, or the
REFERENCE_ROOT environment variable); the GPU box never runs it.  For every case of every task's
`tests/task.json` and `environment/public_cases.json` it:

1. builds the inputs with the reference's `make_inputs(case, seed, "cpu")` and with
   `oracle.inputs.task_inputs`, and records the SHA-256 of each input tensor (they must agree);
2. runs the reference's `reference_exact` and records its outputs: every value for small outputs,
   otherwise a fixed sample of positions plus the SHA-256 and sum of the whole output;
3. records the case list itself (names, seeds, sizes, tolerance), so the tests do not need the
   reference checkout.

Usage: python tests/golden/make_golden.py /path/to/reference
"""
import hashlib
import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle import inputs as oracle_inputs  # noqa: E402

TASKS = ["pow_abs_sqrt_mean", "ppo_clip", "reward_to_go", "leaky", "efficient_kan", "fp8_linear"]
FULL_LIMIT = 4096     # outputs with at most this many elements are stored whole
SAMPLE = 1024         # sampled positions of larger outputs


def tensor_bytes(t):
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.float8_e4m3fn, torch.bool):
        t = t.view(torch.uint8)
    elif t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return t.numpy().tobytes()


def sha(t):
    return hashlib.sha256(tensor_bytes(t)).hexdigest()


def as_f64(t):
    if t.dtype == torch.bfloat16:
        return t.float().double().numpy()
    return t.detach().double().numpy()


def load_ref(root, task):
    p = Path(root) / "tasks" / task / "reference.py"
    spec = importlib.util.spec_from_file_location(f"ref_{task}", p)
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def record_output(name, t):
    v = as_f64(t).ravel()
    rec = {"name": name, "shape": list(t.shape), "dtype": str(t.dtype).replace("torch.", ""),
           "sha256": sha(t), "sum": float(np.sum(v)) if v.size else 0.0, "numel": int(v.size)}
    if v.size <= FULL_LIMIT:
        rec["values"] = [float(x) for x in v]
    else:
        idx = np.sort(np.random.default_rng(12345).choice(v.size, size=SAMPLE, replace=False))
        rec["index"] = [int(i) for i in idx]
        rec["values"] = [float(v[i]) for i in idx]
    return rec


def main(root):
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for task in TASKS:
        spec = json.loads((Path(root) / "tasks" / task / "tests" / "task.json").read_text())
        public = json.loads((Path(root) / "tasks" / task / "environment" / "public_cases.json").read_text())
        ref = load_ref(root, task)
        cases = [dict(c, source="tests/task.json") for c in spec["cases"]]
        cases += [dict(c, source="environment/public_cases.json") for c in public["cases"]]
        out = {"task": task, "signature": spec["signature"], "tolerance": spec["tolerance"],
               "outputs": spec["outputs"], "cases": []}
        for case in cases:
            seed = int(case["seed"])
            r_in = ref.make_inputs(case, seed, "cpu")
            m_in = oracle_inputs.task_inputs(task, case, seed)
            in_rec = {}
            for k, v in r_in.items():
                if isinstance(v, torch.Tensor):
                    a, b = sha(v), sha(m_in[k])
                    if a != b:
                        raise SystemExit(f"{task}/{case['name']}: input {k} differs from oracle.inputs")
                    in_rec[k] = {"sha256": a, "shape": list(v.shape), "dtype": str(v.dtype).replace("torch.", "")}
                else:
                    if v != m_in[k]:
                        raise SystemExit(f"{task}/{case['name']}: scalar {k} differs: {v} vs {m_in[k]}")
                    in_rec[k] = {"value": v}
            exact = ref.reference_exact(r_in)
            outs = [record_output(k, v) for k, v in exact.items()]
            out["cases"].append({"case": case, "inputs": in_rec, "outputs": outs})
            print(task, case["name"], "ok", flush=True)
        (HERE / f"{task}.json").write_text(json.dumps(out, indent=1) + "\n")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ["REFERENCE_ROOT"])
