"""Seeded CPU input generators (test infrastructure; see the package docstring).

`task_inputs(task, case, seed)` reproduces the reference's `make_inputs(case, seed, "cpu")`
for every task: the same distributions drawn from one `torch.Generator("cpu")` in the same call
order, because the values themselves are the fixture (each draw below cites the line it follows).
`baseline_inputs(name, seed)` builds the BASELINE.json configurations restated in the reference's
ABI shapes.
"""
import math

import numpy as np
import torch

E4M3_MAX = 448.0


def _gen(seed):
    return torch.Generator(device="cpu").manual_seed(int(seed))


def _quantize_e4m3(x):
    """Per-tensor max-abs E4M3 quantisation; tasks/fp8_linear/reference.py:15-18.

    The scale is rounded to fp32 because that is the type the kernel receives.
    """
    amax = max(float(x.abs().max().item()), 1e-9)
    scale = float(np.float32(E4M3_MAX / amax))
    q = (x * scale).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q, scale


# Seeded inputs of the E4M3 quantisation step (tests/golden/fp8_quantize.json): name, shape, the
# value recipe and whether the values are bf16-representable (the BASELINE sources are bf16).
QUANT_CASES = [
    ("randn_64x100", (64, 100), "randn", False, 1),
    ("single", (1, 1), "randn", False, 2),
    ("zeros_16x16", (16, 16), "zeros", False, 3),
    ("tiny_17x33", (17, 33), "tiny", False, 4),
    ("bf16_128x257", (128, 257), "randn", True, 5),
    ("wide_31x129", (31, 129), "wide", False, 6),
    ("negative_8x64", (8, 64), "negative", False, 7),
    ("uniform_333x77", (333, 77), "uniform", False, 8),
    ("randn_1024x1024", (1024, 1024), "randn", False, 9),
    ("bf16_512x4096", (512, 4096), "randn", True, 10),
]


def quant_input(name):
    """fp32 input of quantisation case `name` (values bf16-representable for the bf16 cases)."""
    for nm, shape, kind, bf16, seed in QUANT_CASES:
        if nm == name:
            g = torch.Generator(device="cpu").manual_seed(seed)
            if kind == "zeros":
                x = torch.zeros(shape)
            elif kind == "tiny":
                x = torch.randn(shape, generator=g) * 1e-6
            elif kind == "wide":
                x = torch.randn(shape, generator=g) * torch.exp2(torch.randint(-20, 20, shape, generator=g).float())
            elif kind == "negative":
                x = -torch.randn(shape, generator=g).abs()
            elif kind == "uniform":
                x = torch.rand(shape, generator=g) * 6.0 - 3.0
            else:
                x = torch.randn(shape, generator=g)
            return x.to(torch.bfloat16).float() if bf16 else x
    raise KeyError(name)


def task_inputs(task, case, seed):
    """Inputs of one reference test case on the CPU, as `make_inputs(case, seed, "cpu")`."""
    g = _gen(seed)
    f32 = dict(generator=g, dtype=torch.float32)
    if task == "pow_abs_sqrt_mean":  # tasks/pow_abs_sqrt_mean/reference.py:12-19
        shape = (case["batch_size"], 4, case["height"], case["width"])
        scale = float(case.get("scale", 1.0))
        inp = torch.rand(shape, **f32) * scale
        target = torch.rand(shape, **f32) * scale
        return {"inp": inp, "target": target, "batch_size": case["batch_size"], "height": case["height"],
                "width": case["width"]}
    if task == "ppo_clip":  # tasks/ppo_clip/reference.py:14-24
        shape = (case["B"], case["T"], case["H"])
        old = torch.randn(shape, **f32) * 0.5
        delta = (torch.randn(shape, **f32) * float(case.get("delta_std", 0.12))).clamp(-20.0, 20.0)
        cur = old + delta
        adv = torch.randn(shape, **f32)
        return {"B": case["B"], "T": case["T"], "H": case["H"], "current_log_prob": cur, "old_log_prob": old,
                "advantage": adv, "clip_epsilon": float(case.get("clip_epsilon", 0.2))}
    if task == "reward_to_go":  # tasks/reward_to_go/reference.py:12-19
        B, T = case["B"], case["T"]
        reward = torch.rand(B, T, **f32)
        done = torch.rand(B, T, generator=g) < float(case["done_p"])
        done[:, -1] = True
        gamma = float(np.float32(case["gamma"]))
        return {"reward": reward, "done": done, "gamma": gamma, "B": B, "T": T}
    if task == "leaky":  # tasks/leaky/reference.py:12-23
        T, B, H = case["T"], case["B"], case["H"]
        x = torch.randn(T, B, H, **f32) * 0.35 + 0.12
        mem0_std = float(case.get("mem0_std", 0.0))
        mem0 = torch.randn(B, H, **f32) * mem0_std if mem0_std else torch.zeros(B, H)
        lo, hi = case.get("beta_range", [0.65, 0.98])
        beta = torch.rand(H, **f32) * (hi - lo) + lo
        threshold = torch.rand(H, **f32) * 0.6 + 0.8
        return {"input_current": x, "mem0": mem0, "beta": beta, "threshold": threshold, "T": T, "B": B, "H": H}
    if task == "efficient_kan":  # tasks/efficient_kan/reference.py:15-30
        B, I, O = case["B"], case["I"], case["O"]
        G, K = case.get("grid_size", 8), case.get("spline_order", 3)
        xr = float(case.get("x_range", 1.0))
        x = (torch.rand(B, I, **f32) * 2.0 - 1.0) * xr
        knots = torch.arange(-K, G + K + 1, dtype=torch.float32)
        grid = (knots * (2.0 / G) - 1.0).expand(I, -1).contiguous()
        bound = 1.0 / math.sqrt(I)
        base_weight = (torch.rand(O, I, **f32) * 2.0 - 1.0) * bound
        spline_weight = torch.randn(O, I, G + K, **f32) * 0.05
        spline_scaler = torch.randn(O, I, **f32) * 0.1 + 1.0
        return {"x": x, "grid": grid, "base_weight": base_weight, "spline_weight": spline_weight,
                "spline_scaler": spline_scaler, "grid_size": G, "spline_order": K, "B": B, "I": I, "O": O}
    if task == "fp8_linear":  # tasks/fp8_linear/reference.py:21-31
        M, K, N = case["M"], case["K"], case["N"]
        x = torch.randn(M, K, **f32)
        w = torch.randn(N, K, **f32) * (1.0 / K ** 0.5)
        bias = (torch.randn(N, **f32) * 0.05).to(torch.bfloat16)
        x_fp8, scale_x = _quantize_e4m3(x)
        w_fp8, scale_w = _quantize_e4m3(w)
        return {"M": M, "K": K, "N": N, "x_fp8": x_fp8, "scale_x": scale_x, "w_fp8": w_fp8, "scale_w": scale_w,
                "bias": bias}
    raise KeyError(task)


# ------------------------------------------------------------------------------------------------
# BASELINE.json configurations (synthetic; the reference measures no public dataset).
# ------------------------------------------------------------------------------------------------
BASELINE_SHAPES = {
    "robust_l1": {"batch_size": 16, "height": 1024, "width": 1024},            # 2^26 elements
    "rl_pipeline": {"B": 4096, "T": 1000, "gamma": 0.99, "done_p": 0.01, "clip_epsilon": 0.2},
    "lif": {"T": 256, "B": 64, "H": 4096},
    "kan": {"B": 8192, "I": 1024, "O": 1024, "grid_size": 5, "spline_order": 3},
    "fp8_linear": [(16, 4096, 4096), (1024, 4096, 4096), (8192, 8192, 8192), (16384, 28672, 8192)],
}


def baseline_inputs(name, seed=0, **override):
    """One BASELINE.json configuration in ABI shapes (configs[0..4])."""
    g = _gen(seed)
    f32 = dict(generator=g, dtype=torch.float32)
    if name == "robust_l1":  # configs[0]: x, y ~ N(0, 1), 2^26 elements each
        s = dict(BASELINE_SHAPES["robust_l1"], **override)
        shape = (s["batch_size"], 4, s["height"], s["width"])
        return {"inp": torch.randn(shape, **f32), "target": torch.randn(shape, **f32), **s}
    if name == "rl_pipeline":  # configs[1]: reward-to-go and PPO over B x T samples
        s = dict(BASELINE_SHAPES["rl_pipeline"], **override)
        B, T = s["B"], s["T"]
        reward = torch.randn(B, T, **f32)
        done = torch.rand(B, T, generator=g) < s["done_p"]
        done[:, -1] = True
        new = torch.randn(B, T, 1, **f32) * 0.5 - 1.0
        old = new + torch.randn(B, T, 1, **f32) * 0.1
        adv = torch.randn(B, T, 1, **f32)
        ent = torch.rand(B, T, 1, **f32) * 2.0
        return {"reward": reward, "done": done, "gamma": float(np.float32(s["gamma"])), "B": B, "T": T, "H": 1,
                "current_log_prob": new, "old_log_prob": old, "advantage": adv, "entropy": ent,
                "clip_epsilon": float(s["clip_epsilon"])}
    if name == "lif":  # configs[2]: x ~ N(0.3, 0.5), beta 0.9, threshold 1.0, mem0 0
        s = dict(BASELINE_SHAPES["lif"], **override)
        T, B, H = s["T"], s["B"], s["H"]
        return {"input_current": torch.randn(T, B, H, **f32) * 0.5 + 0.3, "mem0": torch.zeros(B, H),
                "beta": torch.full((H,), 0.9), "threshold": torch.full((H,), 1.0), "T": T, "B": B, "H": H}
    if name == "kan":  # configs[3]: G=5, K=3 on [-1, 1]; x ~ U(-1, 1); weights ~ N(0, 1/sqrt(I)); scaler 1
        s = dict(BASELINE_SHAPES["kan"], **override)
        B, I, O, G, K = s["B"], s["I"], s["O"], s["grid_size"], s["spline_order"]
        x = torch.rand(B, I, **f32) * 2.0 - 1.0
        knots = torch.arange(-K, G + K + 1, dtype=torch.float32)
        grid = (knots * (2.0 / G) - 1.0).expand(I, -1).contiguous()
        std = 1.0 / math.sqrt(I)
        base_weight = torch.randn(O, I, **f32) * std
        spline_weight = torch.randn(O, I, G + K, **f32) * std
        spline_scaler = torch.ones(O, I)
        return {"x": x, "grid": grid, "base_weight": base_weight, "spline_weight": spline_weight,
                "spline_scaler": spline_scaler, "grid_size": G, "spline_order": K, "B": B, "I": I, "O": O}
    if name == "fp8_linear":  # configs[4]: x, W ~ N(0, 1) bf16 -> per-tensor E4M3; bias ~ N(0, 0.02) bf16
        M, N, K = override.get("shape", BASELINE_SHAPES["fp8_linear"][0])
        x = torch.randn(M, K, **f32).to(torch.bfloat16).float()
        w = torch.randn(N, K, **f32).to(torch.bfloat16).float()
        bias = (torch.randn(N, **f32) * 0.02).to(torch.bfloat16)
        x_fp8, scale_x = _quantize_e4m3(x)
        w_fp8, scale_w = _quantize_e4m3(w)
        return {"M": M, "K": K, "N": N, "x_fp8": x_fp8, "scale_x": scale_x, "w_fp8": w_fp8, "scale_w": scale_w,
                "bias": bias}
    raise KeyError(name)
