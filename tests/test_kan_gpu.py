"""GPU parity of the KAN linear layer (efficient_kan) through the C ABI.

- Every case of tests/task.json and public_cases.json (G = 8, K = 3; B from 1 to 4096; I = 100;
  x outside the grid) under the grader's 3-call protocol on the drop-in entry point, against the
  fp64 oracle at the task tolerance 1e-5/1e-5 and against the reference oracle's recorded outputs.
- The BASELINE.json configuration (B 8192, I 1024, O 1024, G 5, K 3) against the fp64 oracle on a
  seeded subset of rows.
- Inputs with |silu(x)| far beyond the fp16 range (the row scaling path).
- The row-major A-plane preparation (odd I, or x not 8-byte aligned), beside the column-major one
  the cubic cases take otherwise.
- An output buffer that is not 16-byte aligned (the GEMM epilogue's scalar stores).
- Knot grids that are not uniform, and for a few inputs not increasing (the sparse-basis A planes
  and their full-recurrence fallback), against the fp64 oracle.
- A shape whose GEMM tiles leave a partial last round (168 tiles on 148 SMs), so its last 20 tiles
  run as two K halves whose partial tiles are added: every row against the fp64 oracle, and three
  calls bit-identical (the per-call counters start at zero each call).
"""
import numpy as np
import pytest
import torch

from conftest import golden_cases, pkg
from harness import SET_B, three_call
from oracle import exact, inputs

pytestmark = pytest.mark.gpu
CASES = golden_cases("efficient_kan")
ATOL, RTOL = exact.TOLERANCE["efficient_kan"]
IN_NAMES = ["x", "grid", "base_weight", "spline_weight", "spline_scaler"]


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return pkg().load()


def call_dropin(lib, b, s):
    lib.b200_efficient_kan(b["x"].ptr, b["grid"].ptr, b["base_weight"].ptr, b["spline_weight"].ptr,
                           b["spline_scaler"].ptr, s["grid_size"], s["spline_order"], s["B"], s["I"], s["O"],
                           b["out"].ptr)


@pytest.mark.parametrize("cid,rec", CASES, ids=[c for c, _ in CASES])
def test_case_parity(lib, cid, rec):
    case = rec["case"]
    sets = [inputs.task_inputs("efficient_kan", case, int(case["seed"])),
            inputs.task_inputs("efficient_kan", case, int(case["seed"]) + SET_B)]
    outs = {"out": (torch.float32, (case["B"], case["O"]))}
    results, same = three_call(lambda b, s: call_dropin(lib, b, s), sets, IN_NAMES, outs)
    assert lib.b200_last_status() == 0
    assert same
    for s, r in zip(sets, results):
        bad, worst = exact.within(r["out"].double().numpy(), exact.efficient_kan(s)["out"], ATOL, RTOL)
        assert bad == 0, f"{bad} bad, worst {worst:.3g}"
    o = rec["outputs"][0]
    got = results[0]["out"].double().numpy().ravel()
    have = got[o["index"]] if "index" in o else got
    bad, worst = exact.within(have, o["values"], ATOL, RTOL)
    assert bad == 0, worst


def _run_async(lib, s):
    dev = torch.device("cuda")
    t = {k: s[k].to(dev) for k in IN_NAMES}
    out = torch.empty(s["B"], s["O"], device=dev)
    nbytes = lib.b200_efficient_kan_workspace_bytes(s["grid_size"], s["spline_order"], s["B"], s["I"], s["O"])
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    st = lib.b200_efficient_kan_async(*(t[k].data_ptr() for k in IN_NAMES), s["grid_size"], s["spline_order"],
                                      s["B"], s["I"], s["O"], out.data_ptr(), ws.data_ptr(), nbytes, None)
    torch.cuda.synchronize()
    assert st == 0
    return out


def test_baseline_config_row_subset(lib):
    s = inputs.baseline_inputs("kan", seed=0)
    out = _run_async(lib, s)
    rows = np.sort(np.random.default_rng(2).choice(s["B"], size=64, replace=False))
    ref = exact.efficient_kan(s, rows=rows)["out"]
    got = out[torch.from_numpy(rows).cuda()].double().cpu().numpy()
    bad, worst = exact.within(got, ref, ATOL, RTOL)
    assert bad == 0, worst
    assert pkg().load().b200_device_fault() == 0


def test_large_inputs_use_row_scaling(lib):
    s = inputs.task_inputs("efficient_kan", {"B": 5, "I": 40, "O": 70}, 9)
    s["x"][0, 3] = 90000.0      # silu(x) = x, beyond fp16
    s["x"][2, 7] = -3.0e4
    s["base_weight"][5, 1] = 3.0e5  # a weight beyond fp16
    out = _run_async(lib, s)
    ref = exact.efficient_kan(s)["out"]
    bad, worst = exact.within(out.double().cpu().numpy(), ref, ATOL, RTOL)
    assert bad == 0, worst


@pytest.mark.parametrize("I,shift", [(41, 0), (100, 1)], ids=["odd_I", "x_4_byte_aligned"])
def test_row_major_prep_path(lib, I, shift):
    s = inputs.task_inputs("efficient_kan", {"B": 9, "I": I, "O": 70}, 11)
    dev = torch.device("cuda")
    t = {k: s[k].to(dev) for k in IN_NAMES}
    if shift:
        raw = torch.empty(s["x"].numel() + shift, dtype=torch.float32, device=dev)
        t["x"] = raw[shift:].view(s["x"].shape)
        t["x"].copy_(s["x"])
    out = torch.empty(s["B"], s["O"], device=dev)
    nbytes = lib.b200_efficient_kan_workspace_bytes(s["grid_size"], s["spline_order"], s["B"], s["I"], s["O"])
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    st = lib.b200_efficient_kan_async(*(t[k].data_ptr() for k in IN_NAMES), s["grid_size"], s["spline_order"],
                                      s["B"], s["I"], s["O"], out.data_ptr(), ws.data_ptr(), nbytes, None)
    torch.cuda.synchronize()
    assert st == 0
    ref = exact.efficient_kan(s)["out"]
    bad, worst = exact.within(out.double().cpu().numpy(), ref, ATOL, RTOL)
    assert bad == 0, worst


def test_split_tail_tiles(lib):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    n_tiles = sms + 20  # O = 1024 gives 8 column tiles per 128-row block
    B = 128 * ((n_tiles + 7) // 8)
    s = inputs.task_inputs("efficient_kan", {"B": B, "I": 64, "O": 1024}, 21)
    outs = [_run_async(lib, s) for _ in range(3)]
    for o in outs[1:]:
        assert torch.equal(o.view(torch.int32), outs[0].view(torch.int32))
    ref = exact.efficient_kan(s)["out"]
    bad, worst = exact.within(outs[0].double().cpu().numpy(), ref, ATOL, RTOL)
    assert bad == 0, worst
    assert pkg().load().b200_device_fault() == 0


def uneven_grid(I, G, K, seed):
    """Per-input knots: sorted uniform draws on [-1.5, 1.5]; inputs 3 and 10 get two middle knots
    swapped (a decreasing pair), which the kernels meet with the full recurrence."""
    g = torch.Generator().manual_seed(seed)
    knots = torch.sort(torch.rand(I, G + 2 * K + 1, generator=g) * 3.0 - 1.5, dim=1).values
    for i in (3, 10):
        if i < I:
            m = knots.shape[1] // 2
            knots[i, m], knots[i, m + 1] = knots[i, m + 1].clone(), knots[i, m].clone()
    return knots.contiguous()


@pytest.mark.parametrize("G", [5, 8])
def test_uneven_and_unordered_knots(lib, G):
    s = inputs.task_inputs("efficient_kan", {"B": 96, "I": 64, "O": 70, "grid_size": G, "spline_order": 3,
                                             "x_range": 1.6}, 31 + G)
    s["grid"] = uneven_grid(64, G, 3, 7 + G)
    out = _run_async(lib, s)
    ref = exact.efficient_kan(s)["out"]
    bad, worst = exact.within(out.double().cpu().numpy(), ref, ATOL, RTOL)
    assert bad == 0, worst


def test_unaligned_output(lib):
    s = inputs.task_inputs("efficient_kan", {"B": 130, "I": 64, "O": 72}, 13)
    dev = torch.device("cuda")
    t = {k: s[k].to(dev) for k in IN_NAMES}
    raw = torch.empty(130 * 72 + 1, device=dev)
    out = raw[1:].view(130, 72)  # 4 bytes past a 16-byte boundary
    nbytes = lib.b200_efficient_kan_workspace_bytes(s["grid_size"], s["spline_order"], 130, 64, 72)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    st = lib.b200_efficient_kan_async(*(t[k].data_ptr() for k in IN_NAMES), s["grid_size"], s["spline_order"],
                                      130, 64, 72, out.data_ptr(), ws.data_ptr(), nbytes, None)
    torch.cuda.synchronize()
    assert st == 0
    bad, worst = exact.within(out.double().cpu().numpy(), exact.efficient_kan(s)["out"], ATOL, RTOL)
    assert bad == 0, worst
