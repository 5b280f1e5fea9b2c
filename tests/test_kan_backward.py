"""Backward of the KAN layer (b200_efficient_kan_backward_async).

No reference implementation of the backward exists in the reference repository; the gradients
are those torch autograd forms through its forward (tasks/efficient_kan/reference.py:33-46).

CPU: tests/golden/efficient_kan_backward.json holds those autograd gradients (fp64) for five
cases built by the reference's make_inputs (out-of-grid inputs, K = 2, a single element), made by
tests/golden/make_kan_backward_golden.py; the numpy oracle (oracle.exact.efficient_kan_backward)
reproduces them to 1e-12.

GPU, through the C ABI: every gradient against the oracle within 2e-5 times the sum of its terms'
magnitudes plus 1e-6 (the two GEMMs run on split-fp16 tensor-core products, 22 significant bits,
with fp32 accumulation), on the golden cases, ragged shapes (B, I, O not multiples of 32 or 64,
G = 5, 8 and K = 2), each gradient requested alone, the BASELINE.json KAN size (grad_x on a row
subset, the weight gradients in full), knot grids that are not uniform and for a few inputs not
increasing (the sparse-basis kernels and their full-recurrence fallback), and through
torch.autograd (KANLinearFunction).
"""
import hashlib
import json
import sys

import numpy as np
import pytest
import torch

from conftest import REPO, pkg
from oracle import exact, inputs

sys.path.insert(0, str(REPO / "tests" / "golden"))
from make_kan_backward_golden import grad_out_for  # noqa: E402

GOLDEN = json.loads((REPO / "tests" / "golden" / "efficient_kan_backward.json").read_text())["cases"]
IDS = [c["case"]["name"] for c in GOLDEN]
NAMES = ("grad_x", "grad_base_weight", "grad_spline_weight", "grad_spline_scaler")
TOL = (1e-6, 2e-5)  # atol, fraction of the summed magnitudes
KEYS = ("x", "grid", "base_weight", "spline_weight", "spline_scaler")


@pytest.mark.parametrize("rec", GOLDEN, ids=IDS)
def test_oracle_matches_reference_autograd(rec):
    case = rec["case"]
    s = inputs.task_inputs("efficient_kan", case, int(case["seed"]))
    h = hashlib.sha256(b"".join(s[k].numpy().tobytes() for k in KEYS)).hexdigest()
    assert h == rec["input_sha256"]
    go = grad_out_for(case)
    assert hashlib.sha256(go.numpy().tobytes()).hexdigest() == rec["grad_out_sha256"]
    o = exact.efficient_kan_backward(s, go)
    for k in NAMES:
        np.testing.assert_allclose(o[k].reshape(-1), np.array(rec[k]), rtol=1e-12, atol=1e-12)


# ---------------------------------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    p = pkg()
    p.load()
    return p.ops


def check(got, ref, names=NAMES, rows=None):
    for k, v in zip(NAMES, got):
        if k not in names or v is None:
            continue
        have = v.cpu().double().numpy()
        if rows is not None and k == "grad_x":
            have = have[rows]
        err = np.abs(have - ref[k])
        lim = TOL[0] + TOL[1] * ref[k + "_abs"]
        assert (err <= lim).all(), (k, float((err / lim).max()))


def run(ops, s, go, need_x=True, need_w=True):
    d = {k: s[k].cuda() for k in KEYS}
    out = ops.efficient_kan_backward(d["x"], d["grid"], d["base_weight"], d["spline_weight"], d["spline_scaler"],
                                     s["grid_size"], s["spline_order"], go.cuda(), need_x, need_w)
    torch.cuda.synchronize()
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("rec", GOLDEN, ids=IDS)
def test_golden_cases(ops, rec):
    case = rec["case"]
    s = inputs.task_inputs("efficient_kan", case, int(case["seed"]))
    go = grad_out_for(case)
    got = run(ops, s, go)
    check(got, exact.efficient_kan_backward(s, go))


SHAPES = [(130, 37, 65, 5, 3, 1.0), (64, 128, 128, 8, 3, 1.0), (300, 64, 200, 5, 3, 2.0), (33, 20, 17, 4, 2, 1.0),
          (1, 1, 1, 5, 3, 1.0), (257, 96, 130, 8, 3, 1.5)]


@pytest.mark.gpu
@pytest.mark.parametrize("B,I,O,G,K,xr", SHAPES, ids=[f"B{b}_I{i}_O{o}_G{g}_K{k}" for b, i, o, g, k, _ in SHAPES])
def test_shapes(ops, B, I, O, G, K, xr):
    case = {"B": B, "I": I, "O": O, "grid_size": G, "spline_order": K, "x_range": xr}
    s = inputs.task_inputs("efficient_kan", case, B + I + O)
    go = torch.randn(B, O, generator=torch.Generator().manual_seed(B * O))
    ref = exact.efficient_kan_backward(s, go)
    check(run(ops, s, go), ref)
    gx, gwb, gsw, gsc = run(ops, s, go, need_w=False)
    assert gwb is None and gsw is None and gsc is None
    check((gx, None, None, None), ref, names=("grad_x",))
    gx, gwb, gsw, gsc = run(ops, s, go, need_x=False)
    assert gx is None
    check((None, gwb, gsw, gsc), ref, names=NAMES[1:])


@pytest.mark.gpu
def test_baseline_size(ops):
    s = inputs.baseline_inputs("kan", seed=0)
    B, O = s["B"], s["O"]
    go = torch.randn(B, O, generator=torch.Generator().manual_seed(7))
    got = run(ops, s, go)
    rows = np.random.default_rng(0).choice(B, size=256, replace=False)
    check(got, exact.efficient_kan_backward(s, go, rows=rows), rows=rows)


@pytest.mark.gpu
@pytest.mark.parametrize("G", [5, 8])
def test_uneven_and_unordered_knots(ops, G):
    from test_kan_gpu import uneven_grid
    case = {"B": 130, "I": 64, "O": 40, "grid_size": G, "spline_order": 3, "x_range": 1.6}
    s = inputs.task_inputs("efficient_kan", case, 41 + G)
    s["grid"] = uneven_grid(64, G, 3, 17 + G)
    go = torch.randn(130, 40, generator=torch.Generator().manual_seed(G))
    check(run(ops, s, go), exact.efficient_kan_backward(s, go))


@pytest.mark.gpu
def test_autograd_function(ops):
    case = {"B": 70, "I": 40, "O": 33, "grid_size": 5, "spline_order": 3}
    s = inputs.task_inputs("efficient_kan", case, 3)
    go = torch.randn(70, 33, generator=torch.Generator().manual_seed(4))
    d = {k: s[k].cuda().requires_grad_(k != "grid") for k in KEYS}
    y = ops.KANLinearFunction.apply(d["x"], d["grid"], d["base_weight"], d["spline_weight"], d["spline_scaler"], 5, 3)
    y.backward(go.cuda())
    got = [d[k].grad for k in ("x", "base_weight", "spline_weight", "spline_scaler")]
    check(got, exact.efficient_kan_backward(s, go))


@pytest.mark.gpu
def test_status_codes(ops):
    lib = pkg().load()
    x = torch.zeros(64, device="cuda")
    p = x.data_ptr()
    assert lib.b200_efficient_kan_backward_async(p, p, p, p, p, 0, 3, 2, 2, 2, p, p, p, p, p, p, 1 << 20, None) == 1
    assert lib.b200_efficient_kan_backward_async(p, p, p, p, p, 5, 3, 2, 2, 2, p, p, p, p, p, p, 8, None) == 4
    assert lib.b200_efficient_kan_backward_async(p, p, p, p, p, 60, 3, 2, 2, 2, p, p, p, p, p, p, 1 << 20, None) == 3
