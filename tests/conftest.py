import hashlib
import importlib
import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
sys.path.insert(0, str(REPO))

TASKS = ["pow_abs_sqrt_mean", "ppo_clip", "reward_to_go", "leaky", "efficient_kan", "fp8_linear"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def golden(task):
    return json.loads((GOLDEN / f"{task}.json").read_text())


def golden_cases(task):
    """(id, case record) for every golden case of a task, ids unique per task."""
    g = golden(task)
    seen, out = set(), []
    for rec in g["cases"]:
        name = rec["case"]["name"]
        cid = name if name not in seen else f"{name}@public"
        seen.add(name)
        out.append((cid, rec))
    return out


def tensor_sha(t):
    import torch
    t = t.detach().cpu().contiguous()
    if t.dtype in (torch.float8_e4m3fn, torch.bool):
        t = t.view(torch.uint8)
    elif t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def array_sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def pkg():
    """The product package (its directory name is not an identifier, so import it by name)."""
    return importlib.import_module("cuda-optimization-benchmark_b200")


@pytest.fixture(scope="session")
def b200():
    return pkg()
