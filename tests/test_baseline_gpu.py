"""GPU parity at the BASELINE.json sizes, and the reduction properties the multi-GPU path needs.

- robust-L1 at 2^26 N(0,1) elements against the fp64 oracle with rtol 1e-5;
- reward-to-go [4096, 1000] (rewards N(0,1), done p=0.01) against the fp64 oracle at the task
  tolerance 1e-5/1e-5, and PPO with entropy over the same 4,096,000 samples;
- LIF [256, 64, 4096] bit-exact against the fp32 oracle;
- robust-L1 and PPO results are bit-identical when the element range is split into 1, 2, 3, 4, 8
  chunk-aligned shards (the exchange the multi-GPU path performs), and across repeat calls.
"""
import numpy as np
import pytest
import torch

from conftest import pkg
from oracle import exact, inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    p = pkg()
    p.load()
    return p.ops


def cuda(d):
    return {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


def test_robust_l1_baseline(ops):
    s = inputs.baseline_inputs("robust_l1", seed=0)
    g = cuda(s)
    out = ops.robust_l1(g["inp"], g["target"])
    ref = exact.pow_abs_sqrt_mean(s)["output"]
    bad, worst = exact.within(out.cpu().double().numpy(), ref, 0.0, 1e-5)
    assert bad == 0, worst
    again = ops.robust_l1(g["inp"], g["target"])
    assert torch.equal(out.reshape(1).view(torch.uint8), again.reshape(1).view(torch.uint8))


def test_rl_pipeline_baseline(ops):
    s = inputs.baseline_inputs("rl_pipeline", seed=0)
    g = cuda(s)
    rtg = ops.reward_to_go(g["reward"], g["done"], g["gamma"])
    ppo = ops.ppo_clip(g["current_log_prob"], g["old_log_prob"], g["advantage"], g["clip_epsilon"], g["entropy"])
    ref_rtg = exact.reward_to_go(s)["output"]
    bad, worst = exact.within(rtg.cpu().double().numpy(), ref_rtg, 1e-5, 1e-5)
    assert bad == 0, worst
    ref_ppo = exact.ppo_clip(s, entropy=s["entropy"])["output"]
    bad, worst = exact.within(ppo.cpu().double().numpy(), ref_ppo, 1e-5, 1e-4)
    assert bad == 0, (worst, ppo.cpu().numpy(), ref_ppo)


def test_lif_baseline_bit_exact(ops):
    s = inputs.baseline_inputs("lif", seed=0)
    g = cuda(s)
    spikes, mem = ops.leaky(g["input_current"], g["mem0"], g["beta"], g["threshold"])
    ref = exact.leaky(s)
    assert np.array_equal(spikes.cpu().numpy(), ref["spikes"])
    assert np.array_equal(mem.cpu().numpy(), ref["final_mem"])


def _splits(n_chunks, parts):
    """Chunk-aligned shard boundaries (in chunks) for `parts` shards."""
    b = [round(i * n_chunks / parts) for i in range(parts + 1)]
    return list(zip(b[:-1], b[1:]))


@pytest.mark.parametrize("parts", [1, 2, 3, 4, 8])
def test_robust_l1_shards_bit_identical(ops, parts):
    n = (1 << 22) + 12345
    g = torch.Generator().manual_seed(5)
    a = torch.randn(n, generator=g).cuda()
    b = torch.randn(n, generator=g).cuda()
    whole = ops.robust_l1(a, b)
    chunk = pkg().load().b200_robust_l1_chunk_elems()
    n_chunks = (n + chunk - 1) // chunk
    pieces = []
    for c0, c1 in _splits(n_chunks, parts):
        lo, hi = c0 * chunk, min(c1 * chunk, n)
        pieces.append(ops.robust_l1_partials(a[lo:hi], b[lo:hi]))
    out = ops.robust_l1_finish(torch.cat(pieces), n)
    assert torch.equal(whole.reshape(1).view(torch.uint8), out.reshape(1).view(torch.uint8))


@pytest.mark.parametrize("parts", [1, 2, 3, 4, 8])
def test_ppo_shards_bit_identical(ops, parts):
    s = inputs.baseline_inputs("rl_pipeline", seed=3, B=997, T=1003)
    g = cuda(s)
    cur, old, adv, ent = (g[k].reshape(-1) for k in ("current_log_prob", "old_log_prob", "advantage", "entropy"))
    n = cur.numel()
    whole = ops.ppo_clip(cur, old, adv, 0.2, ent)
    chunk = pkg().load().b200_ppo_chunk_elems()
    n_chunks = (n + chunk - 1) // chunk
    pieces = []
    for c0, c1 in _splits(n_chunks, parts):
        lo, hi = c0 * chunk, min(c1 * chunk, n)
        pieces.append(ops.ppo_partials(cur[lo:hi], old[lo:hi], adv[lo:hi], 0.2, ent[lo:hi]))
    out = ops.ppo_finish(torch.cat(pieces), n, True)
    assert torch.equal(whole.view(torch.uint8), out.view(torch.uint8))


def test_ppo_boundary_clip_decisions(ops):
    """Samples within a few ulps of the clip bounds are counted exactly as the fp64 oracle does."""
    eps = 0.2
    e = np.float64(np.float32(eps))
    cur, old = [], []
    for bound in (np.log1p(-e), np.log1p(e)):
        for shift in (0.0, 0.5, -0.75, 3.0):
            v0 = np.float32(bound + shift)
            for k in range(-12, 13):
                v = v0
                for _ in range(abs(k)):
                    v = np.nextafter(v, np.float32(np.inf) if k > 0 else np.float32(-np.inf))
                cur.append(v)
                old.append(np.float32(shift))
    cur = np.array(cur * 20, dtype=np.float32)
    old = np.array(old * 20, dtype=np.float32)
    adv = np.linspace(-2, 2, cur.size, dtype=np.float32)
    s = {"current_log_prob": torch.from_numpy(cur), "old_log_prob": torch.from_numpy(old),
         "advantage": torch.from_numpy(adv), "clip_epsilon": eps}
    got = ops.ppo_clip(s["current_log_prob"].cuda(), s["old_log_prob"].cuda(), s["advantage"].cuda(), eps)
    ref = exact.ppo_clip(s)["output"]
    assert float(got[1].cpu()) == float(np.float32(ref[1])), "clip fraction differs from the fp64 decision"
    bad, worst = exact.within(got.cpu().double().numpy(), ref, 1e-5, 1e-4)
    assert bad == 0, worst
