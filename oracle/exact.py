"""numpy restatement of each task's correctness oracle `reference_exact` (test infrastructure).

fp64 for pow_abs_sqrt_mean, ppo_clip, reward_to_go and efficient_kan; the fp32 step order for
leaky (whose oracle is the fp32 reference itself); fp64 then one rounding to bf16 for fp8_linear.
Each function cites the reference lines it restates.  Inputs are the dicts built by
`oracle.inputs` (torch CPU tensors or numpy arrays); outputs are numpy arrays keyed like the
reference's output names.
"""
import math

import numpy as np

TOLERANCE = {  # tasks/<task>/tests/task.json "tolerance"
    "pow_abs_sqrt_mean": (1e-3, 1e-3),
    "ppo_clip": (1e-5, 1e-4),
    "reward_to_go": (1e-5, 1e-5),
    "leaky": (1e-6, 1e-5),
    "efficient_kan": (1e-5, 1e-5),
    "fp8_linear": (1e-2, 1e-2),
}


def _np(t):
    if hasattr(t, "detach"):
        t = t.detach().cpu()
        if str(t.dtype) == "torch.float8_e4m3fn":
            return t.view(__import__("torch").uint8).numpy()
        if str(t.dtype) == "torch.bfloat16":
            return t.view(__import__("torch").int16).numpy().view(np.uint16)
        return t.numpy()
    return np.asarray(t)


# -------------------------------------------------------------------------------- robust-L1
def pow_abs_sqrt_mean(inp):
    """tasks/pow_abs_sqrt_mean/reference.py:22-24,31-32: mean(sqrt(|a-b|^2 + 0.001*0.001)) in fp64."""
    a = _np(inp["inp"]).astype(np.float64).ravel()
    b = _np(inp["target"]).astype(np.float64).ravel()
    d = np.abs(a - b)
    v = np.sqrt(d * d + (0.001 * 0.001))
    return {"output": np.array(v.mean() if v.size else np.nan)}


# ------------------------------------------------------------------------------------- PPO
def _logsumexp(v):
    m = np.max(v)
    return m + math.log(np.sum(np.exp(v - m)))


def ppo_clip(inp, entropy=None):
    """tasks/ppo_clip/reference.py:27-35,42-45 in fp64, eps first rounded to fp32 (:43).

    With `entropy`, a 7th value (its mean) is appended: the extended form's diagnostic.
    """
    cur = _np(inp["current_log_prob"]).astype(np.float64).ravel()
    old = _np(inp["old_log_prob"]).astype(np.float64).ravel()
    adv = _np(inp["advantage"]).astype(np.float64).ravel()
    eps = float(np.float32(inp["clip_epsilon"]))
    lw = cur - old
    ratio = np.exp(lw)
    lwc = np.clip(lw, math.log1p(-eps), math.log1p(eps))
    gain = np.minimum(ratio * adv, np.exp(lwc) * adv)
    n = lw.size
    ess = math.exp(2.0 * _logsumexp(lw) - _logsumexp(2.0 * lw)) / n
    out = [-gain.mean(), (lwc != lw).astype(np.float64).mean(), ((ratio - 1.0) - lw).mean(), ess, ratio.max(),
           ratio.mean()]
    if entropy is not None:
        out.append(_np(entropy).astype(np.float64).mean())
    return {"output": np.array(out)}


# ---------------------------------------------------------------------------- reward-to-go
def reward_to_go(inp):
    """tasks/reward_to_go/reference.py:34-42: fp64 backward loop, nxt = r + gamma*keep*nxt."""
    r = _np(inp["reward"]).astype(np.float64)
    keep = (~_np(inp["done"]).astype(bool)).astype(np.float64)
    gamma = float(inp["gamma"])
    out = np.empty_like(r)
    nxt = np.zeros(r.shape[0])
    for t in range(r.shape[1] - 1, -1, -1):
        nxt = r[:, t] + gamma * keep[:, t] * nxt
        out[:, t] = nxt
    return {"output": out}


# ---------------------------------------------------------------------------------------- LIF
def leaky(inp):
    """tasks/leaky/reference.py:26-40: the fp32 loop, one rounding per product and sum."""
    x = _np(inp["input_current"]).astype(np.float32)
    T, B, H = x.shape
    beta = np.clip(_np(inp["beta"]).astype(np.float32), np.float32(0), np.float32(1)).reshape(1, H)
    th = _np(inp["threshold"]).astype(np.float32).reshape(1, H)
    mem = _np(inp["mem0"]).astype(np.float32).copy()
    spikes = np.empty_like(x)
    for t in range(T):
        reset = (mem >= th).astype(np.float32)
        mem = (beta * mem + x[t]) - reset * th
        spikes[t] = (mem >= th).astype(np.float32)
    return {"spikes": spikes, "final_mem": mem}


# ---------------------------------------------------------------------------------------- KAN
def kan_bases(x, grid, k_order):
    """Cox-de Boor bases; tasks/efficient_kan/reference.py:33-39 (indicator, then K rounds)."""
    xe = x[:, :, None]
    bases = ((xe >= grid[None, :, :-1]) & (xe < grid[None, :, 1:])).astype(x.dtype)
    for k in range(1, k_order + 1):
        left = (xe - grid[None, :, :-(k + 1)]) / (grid[None, :, k:-1] - grid[None, :, :-(k + 1)])
        right = (grid[None, :, k + 1:] - xe) / (grid[None, :, k + 1:] - grid[None, :, 1:-k])
        bases = left * bases[:, :, :-1] + right * bases[:, :, 1:]
    return bases


def efficient_kan(inp, rows=None):
    """tasks/efficient_kan/reference.py:42-46,54-57 in fp64.  `rows` limits the batch rows."""
    x = _np(inp["x"]).astype(np.float64)
    if rows is not None:
        x = x[rows]
    grid = _np(inp["grid"]).astype(np.float64)
    wb = _np(inp["base_weight"]).astype(np.float64)
    sw = _np(inp["spline_weight"]).astype(np.float64)
    sc = _np(inp["spline_scaler"]).astype(np.float64)
    bases = kan_bases(x, grid, int(inp["spline_order"]))
    silu = x / (1.0 + np.exp(-x))
    w = (sw * sc[:, :, None]).reshape(wb.shape[0], -1)
    out = silu @ wb.T + bases.reshape(x.shape[0], -1) @ w.T
    return {"out": out}


# ---------------------------------------------------------------------------------- FP8 linear
def e4m3_table():
    """Value of every E4M3 (fn variant) byte: 1 sign, 4 exponent (bias 7), 3 mantissa bits;
    exponent 0 is subnormal, S.1111.111 is NaN, no infinities."""
    vals = np.empty(256, dtype=np.float64)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            vals[b] = np.nan
        elif e == 0:
            vals[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            vals[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


def f32_to_bf16_bits(v32):
    """Round fp32 values to bf16 (round to nearest, ties to even); returns uint16 bits."""
    u = np.ascontiguousarray(v32, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(v32)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f64(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def fp8_linear(inp, rows=None):
    """tasks/fp8_linear/reference.py:34-37,44-45: (q_x/sx) @ (q_w/sw)^T + bias in fp64, then one
    conversion to bf16.  The conversion goes through fp32 (fp64 -> fp32 -> bf16, each round to
    nearest even), which is how the reference's `.to(torch.bfloat16)` of an fp64 tensor rounds.
    Returns bf16 bits (uint16) and the fp64 values before rounding."""
    tab = e4m3_table()
    xq = _np(inp["x_fp8"]).astype(np.uint8)
    if rows is not None:
        xq = xq[rows]
    x = tab[xq]
    x /= float(inp["scale_x"])
    w = tab[_np(inp["w_fp8"]).astype(np.uint8)]
    w /= float(inp["scale_w"])
    bias = bf16_bits_to_f64(_np(inp["bias"]))
    y = x @ w.T
    del w
    y += bias[None, :]
    return {"output": f32_to_bf16_bits(y.astype(np.float32)), "output_f64": y}


TASKS = {
    "pow_abs_sqrt_mean": pow_abs_sqrt_mean,
    "ppo_clip": ppo_clip,
    "reward_to_go": reward_to_go,
    "leaky": leaky,
    "efficient_kan": efficient_kan,
    "fp8_linear": fp8_linear,
}


def within(out, ref, atol, rtol):
    """Reference pass rule per element: |o - r| <= atol + rtol*|r|, NaN matches NaN
    (graders/child.py:150-175).  Returns (number of bad elements, worst |o-r|/(atol+rtol|r|))."""
    o = np.asarray(out, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    both_nan = np.isnan(o) & np.isnan(r)
    err = np.abs(o - r)
    lim = atol + rtol * np.abs(r)
    ok = (err <= lim) | both_nan
    ratio = np.where(both_nan, 0.0, err / lim)
    worst = float(np.nanmax(ratio)) if ratio.size else 0.0
    return int((~ok).sum()), worst


def gae(inp):
    """Generalised advantage estimation in fp64 (no reference implementation in the reference
    repository: the published algorithm of Schulman et al. 2016 in the form of TorchRL's
    generalized_advantage_estimate, with separate done and terminated flags):
    delta = r + gamma * next_value * (1 - terminated) - value; A[t] = delta[t] + gamma * lambda *
    (1 - done[t]) * A[t + 1], A past the last step 0; value_target = A + value.  gamma and lambda
    are taken as the fp32 values the kernel receives."""
    r = _np(inp["reward"]).astype(np.float64)
    v = _np(inp["value"]).astype(np.float64)
    nv = _np(inp["next_value"]).astype(np.float64)
    done = _np(inp["done"]).astype(bool)
    term = _np(inp["terminated"]).astype(bool)
    g = float(np.float32(inp["gamma"]))
    lam = float(np.float32(inp["lmbda"]))
    delta = r + g * nv * (~term) - v
    adv = np.zeros_like(delta)
    a = np.zeros(delta.shape[0])
    for t in range(delta.shape[1] - 1, -1, -1):
        a = delta[:, t] + g * lam * (~done[:, t]) * a
        adv[:, t] = a
    return {"advantage": adv, "value_target": adv + v}


def atan_surrogate_grad(u, alpha):
    """Derivative of the arctangent spike surrogate (Fang et al., "Incorporating Learnable
    Membrane Time Constant to Enhance Learning of Spiking Neural Networks", 2021; snnTorch's
    default surrogate for Leaky): d spike / d u = (alpha / 2) / (1 + (pi / 2 * alpha * u)^2)."""
    return (alpha / 2.0) / (1.0 + (math.pi / 2.0 * alpha * u) ** 2)


def leaky_backward(inp, grad_spikes, grad_final_mem=None, alpha=2.0):
    """Surrogate-gradient backward of the leaky layer (no reference implementation in the reference
    repository: snnTorch's Leaky, the layer tasks/leaky restates, trained through its arctangent
    surrogate with the reset detached).  The forward is the reference's own fp32 loop
    (tasks/leaky/reference.py:26-40, `leaky` above), so every reset and spike decision is the
    reference's; the backward is then fp64 over those fp32 membrane values:

        u[t] = mem[t] - th,   s'[t] = atan_surrogate_grad(u[t]),   r[t] = (mem[t-1] >= th)
        g[t] = grad_spikes[t] * s'[t] + beta * g[t+1]         (beta * g[T] := grad_final_mem)
        grad_x[t] = g[t];   grad_mem0 = beta * g[0]
        grad_beta[h] = [0 <= beta_raw[h] <= 1] * sum_{b,t} g[t] * mem[t-1]
        grad_threshold[h] = -sum_{b,t} (grad_spikes[t] * s'[t] + r[t] * g[t])

    with mem[-1] = mem0 and beta the clamped value the forward uses."""
    x = _np(inp["input_current"]).astype(np.float32)
    T, B, H = x.shape
    braw = _np(inp["beta"]).astype(np.float32)
    beta32 = np.clip(braw, np.float32(0), np.float32(1)).reshape(1, H)
    th32 = _np(inp["threshold"]).astype(np.float32).reshape(1, H)
    mem = _np(inp["mem0"]).astype(np.float32).copy()
    mems = np.empty((T + 1, B, H), dtype=np.float32)
    mems[0] = mem
    for t in range(T):
        reset = (mem >= th32).astype(np.float32)
        mem = (beta32 * mem + x[t]) - reset * th32
        mems[t + 1] = mem
    gs = _np(grad_spikes).astype(np.float64).reshape(T, B, H)
    c = (np.zeros((B, H)) if grad_final_mem is None
         else _np(grad_final_mem).astype(np.float64).reshape(B, H))
    beta = beta32.astype(np.float64)
    th = th32.astype(np.float64)
    gx = np.empty((T, B, H))
    gb = np.zeros((B, H))
    gt = np.zeros((B, H))
    gb_abs = np.zeros((B, H))
    gt_abs = np.zeros((B, H))
    for t in range(T - 1, -1, -1):
        gsp = gs[t] * atan_surrogate_grad(mems[t + 1].astype(np.float64) - th, alpha)
        g = gsp + c
        gx[t] = g
        prev = mems[t].astype(np.float64)
        gb += g * prev
        gb_abs += np.abs(g * prev)
        term = gsp + (prev >= th) * g
        gt -= term
        gt_abs += np.abs(term)
        c = beta * g
    mask = ((braw >= 0) & (braw <= 1)).astype(np.float64)
    # *_abs: the sums of the terms' magnitudes, the scale of a summation's rounding error.
    return {"grad_input": gx, "grad_mem0": c, "grad_beta": mask * gb.sum(axis=0),
            "grad_threshold": gt.sum(axis=0), "grad_beta_abs": gb_abs.sum(axis=0),
            "grad_threshold_abs": gt_abs.sum(axis=0), "spikes": (mems[1:] >= th32).astype(np.float32),
            "final_mem": mems[T], "checkpoints": mems[0:T:16]}


def pack_done_bits(done):
    """Done flags [B, T] -> uint32 words [B, ceil(T/32)]: bit t % 32 of word [b, t // 32] is
    done[b, t], bits past T zero (the bit layout beside the reference's one-bool-per-step ABI)."""
    d = _np(done).astype(bool)
    B, T = d.shape
    W = (T + 31) // 32
    padded = np.zeros((B, W * 32), dtype=np.uint64)
    padded[:, :T] = d
    weights = np.left_shift(np.uint64(1), np.arange(32, dtype=np.uint64))
    return (padded.reshape(B, W, 32) * weights).sum(axis=2).astype(np.uint32)


def efficient_kan_backward(inp, grad_out, rows=None):
    """Backward of the KAN layer in fp64 (no reference implementation in the reference repository:
    the gradients of tasks/efficient_kan/reference.py:33-46, the KANLinear forward, that torch
    autograd forms through it).  With W_spl = spline_weight * spline_scaler and the bases B_c(x)
    and their derivatives from forward-mode differentiation of the same Cox-de Boor recurrence:

        grad_x[b,i]      = silu'(x) * (G @ W_base)[b,i] + sum_c B'_c(x[b,i]) * (G @ W_spl)[b,i,c]
        grad_W_base      = G^T @ silu(x)
        grad_W_spl       = G^T @ B(x)                       ([O, I, C])
        grad_sw          = grad_W_spl * spline_scaler;  grad_scaler = sum_c grad_W_spl * sw

    `rows` limits grad_x to a subset of batch rows (the weight gradients always use every row).
    *_abs: the same sums over the terms' magnitudes (the scale of a summation's rounding error)."""
    x = _np(inp["x"]).astype(np.float64)
    g = _np(inp["grid"]).astype(np.float64)
    wb = _np(inp["base_weight"]).astype(np.float64)
    sw = _np(inp["spline_weight"]).astype(np.float64)
    sc = _np(inp["spline_scaler"]).astype(np.float64)
    G = _np(grad_out).astype(np.float64)
    K = int(inp["spline_order"])
    B, I = x.shape
    O = wb.shape[0]
    C = sw.shape[2]
    xe = x[:, :, None]
    bases = ((xe >= g[None, :, :-1]) & (xe < g[None, :, 1:])).astype(np.float64)
    dbases = np.zeros_like(bases)
    for k in range(1, K + 1):
        dl = 1.0 / (g[None, :, k:-1] - g[None, :, :-(k + 1)])
        dr = -1.0 / (g[None, :, k + 1:] - g[None, :, 1:-k])
        left = (xe - g[None, :, :-(k + 1)]) * dl
        right = (g[None, :, k + 1:] - xe) * -dr
        nb = left * bases[:, :, :-1] + right * bases[:, :, 1:]
        dbases = dl * bases[:, :, :-1] + left * dbases[:, :, :-1] + dr * bases[:, :, 1:] + right * dbases[:, :, 1:]
        bases = nb
    s = 1.0 / (1.0 + np.exp(-x))
    silu = x * s
    dsilu = s * (1.0 + x * (1.0 - s))
    wspl = (sw * sc[:, :, None]).reshape(O, I * C)
    xr = slice(None) if rows is None else rows
    Gr = G[xr]
    ga_base = Gr @ wb
    ga_spl = (Gr @ wspl).reshape(-1, I, C)
    ga_base_abs = np.abs(Gr) @ np.abs(wb)
    ga_spl_abs = (np.abs(Gr) @ np.abs(wspl)).reshape(-1, I, C)
    grad_x = ga_base * dsilu[xr] + (ga_spl * dbases[xr]).sum(axis=2)
    grad_x_abs = ga_base_abs * np.abs(dsilu[xr]) + (ga_spl_abs * np.abs(dbases[xr])).sum(axis=2)
    gw_base = G.T @ silu
    gw_base_abs = np.abs(G).T @ np.abs(silu)
    bflat = bases.reshape(B, I * C)
    gw_spl = (G.T @ bflat).reshape(O, I, C)
    gw_spl_abs = (np.abs(G).T @ np.abs(bflat)).reshape(O, I, C)  # bases can be negative on unordered knots
    return {"grad_x": grad_x, "grad_base_weight": gw_base, "grad_spline_weight": gw_spl * sc[:, :, None],
            "grad_spline_scaler": (gw_spl * sw).sum(axis=2),
            "grad_x_abs": grad_x_abs, "grad_base_weight_abs": gw_base_abs,
            "grad_spline_weight_abs": gw_spl_abs * np.abs(sc[:, :, None]),
            "grad_spline_scaler_abs": (gw_spl_abs * np.abs(sw)).sum(axis=2)}
