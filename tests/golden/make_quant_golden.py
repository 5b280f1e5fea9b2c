"""Generate tests/golden/fp8_quantize.json from the reference's own E4M3 quantisation.

Runs only where the reference checkout is present (its path is the first argument, or the
REFERENCE_ROOT environment variable); the GPU box never runs it.  For every case of
oracle.inputs.QUANT_CASES it builds the fp32 input, runs the reference's `_quantize`
(tasks/fp8_linear/reference.py:15-18) and records the scale and the E4M3 bytes: every byte for
inputs of at most 4096 elements, otherwise the SHA-256 of all bytes and a fixed sample of positions.

Usage: python tests/golden/make_quant_golden.py /path/to/reference
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

from oracle import inputs  # noqa: E402

FULL_LIMIT = 4096
SAMPLE = 1024


def main(root):
    spec = importlib.util.spec_from_file_location("ref_fp8", Path(root) / "tasks" / "fp8_linear" / "reference.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    cases = []
    for name, shape, kind, bf16, seed in inputs.QUANT_CASES:
        x = inputs.quant_input(name)
        q, scale = ref._quantize(x)
        qb = q.view(torch.uint8).numpy().ravel()
        rec = {"name": name, "shape": list(shape), "bf16": bf16,
               "input_sha256": hashlib.sha256(x.numpy().tobytes()).hexdigest(),
               "scale": float(scale), "scale_hex": float(scale).hex(),
               "q_sha256": hashlib.sha256(qb.tobytes()).hexdigest()}
        if qb.size <= FULL_LIMIT:
            rec["q"] = qb.tobytes().hex()
        else:
            pos = np.sort(np.random.default_rng(seed).choice(qb.size, size=SAMPLE, replace=False))
            rec["positions"] = pos.tolist()
            rec["q_at"] = qb[pos].tobytes().hex()
        cases.append(rec)
    out = HERE / "fp8_quantize.json"
    out.write_text(json.dumps({"source": "tasks/fp8_linear/reference.py:15-18 (_quantize)", "cases": cases},
                              indent=1) + "\n")
    print(out, len(cases), "cases")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT", "/root/reference"))
