"""PyTorch-eager fp32 restatement of each task's `reference` (test infrastructure).

The reference times its kernels against these eager op sequences (graders/child.py:247-265);
here they run on the host CPU as the reported CPU baseline of `bench.py`.  The op sequence of
each function follows the cited reference lines, since the baseline's cost is the cost of that
sequence.
"""
import math

import torch
import torch.nn.functional as F


def pow_abs_sqrt_mean(inp, target):
    """tasks/pow_abs_sqrt_mean/reference.py:22-24."""
    return torch.sqrt(torch.pow(torch.abs(inp - target), 2) + (0.001 * 0.001)).mean()


def ppo_clip(cur, old, adv, eps, entropy=None):
    """tasks/ppo_clip/reference.py:27-35; with `entropy`, its mean appended (extended form)."""
    lw = cur - old
    ratio = torch.exp(lw)
    lwc = lw.clamp(math.log1p(-eps), math.log1p(eps))
    gain = torch.minimum(ratio * adv, torch.exp(lwc) * adv)
    flat = lw.reshape(-1)
    ess = torch.exp(2.0 * flat.logsumexp(0) - (2.0 * flat).logsumexp(0)) / flat.numel()
    vals = [-gain.mean(), (lwc != lw).to(lw.dtype).mean(), ((ratio - 1.0) - lw).mean(), ess, ratio.max(),
            ratio.mean()]
    if entropy is not None:
        vals.append(entropy.mean())
    return torch.stack(vals)


def reward_to_go(reward, done, gamma):
    """tasks/reward_to_go/reference.py:22-31: log-depth affine scan, out[t] = a[t]*out[t+1] + r[t]."""
    a = torch.where(done, 0.0, gamma).to(torch.float32)
    b = reward.clone()
    T, d = b.shape[1], 1
    while d < T:
        b = torch.cat([b[:, :-d] + a[:, :-d] * b[:, d:], b[:, -d:]], dim=1)
        a = torch.cat([a[:, :-d] * a[:, d:], a[:, -d:] * 0.0], dim=1)
        d *= 2
    return b


def leaky(x, mem0, beta, threshold):
    """tasks/leaky/reference.py:26-37."""
    T, B, H = x.shape
    beta = beta.clamp(0.0, 1.0).view(1, H)
    th = threshold.view(1, H)
    mem = mem0.clone()
    spikes = torch.empty_like(x)
    for t in range(T):
        reset = (mem >= th).to(x.dtype)
        mem = beta * mem + x[t] - reset * th
        spikes[t] = (mem >= th).to(x.dtype)
    return spikes, mem


def _b_splines(x, grid, k_order):
    xe = x.unsqueeze(-1)
    bases = ((xe >= grid[:, :-1]) & (xe < grid[:, 1:])).to(x.dtype)
    for k in range(1, k_order + 1):
        bases = ((xe - grid[:, :-(k + 1)]) / (grid[:, k:-1] - grid[:, :-(k + 1)])) * bases[:, :, :-1] + \
                ((grid[:, k + 1:] - xe) / (grid[:, k + 1:] - grid[:, 1:-k])) * bases[:, :, 1:]
    return bases.contiguous()


def efficient_kan(x, grid, base_weight, spline_weight, spline_scaler, k_order):
    """tasks/efficient_kan/reference.py:33-46."""
    bases = _b_splines(x, grid, k_order)
    base_out = F.linear(F.silu(x), base_weight)
    w = (spline_weight * spline_scaler.unsqueeze(-1)).reshape(base_weight.shape[0], -1)
    return base_out + F.linear(bases.reshape(x.shape[0], -1), w)


def fp8_linear(x_fp8, scale_x, w_fp8, scale_w, bias):
    """tasks/fp8_linear/reference.py:34-37 in fp32."""
    x = x_fp8.to(torch.float32) / scale_x
    w = w_fp8.to(torch.float32) / scale_w
    return (x @ w.t() + bias.to(torch.float32)).to(torch.bfloat16)
