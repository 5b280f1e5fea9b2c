"""GPU: the fused RL loss step (reward-to-go and PPO in one launch, b200_rl_step_async) gives the
same bits as the two separate entry points, at the BASELINE.json configs[1] size and at ragged,
empty and misaligned shapes, with and without entropy; its shard form gives the same per-chunk
partials as b200_ppo_shard_partials.  Through that identity the fused step inherits the separate
ops' oracle parity (tests/test_stream_ops_gpu.py, tests/test_baseline_gpu.py), which is checked
again here at the full size.
"""
import ctypes

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


def bits(t):
    return t.reshape(-1).contiguous().view(torch.uint8)


def make(B, T, n, seed, phase=0, entropy=True):
    """Reward-to-go inputs [B, T] and PPO inputs over n samples, each view `phase` floats (or
    bytes, for done) past a 256-byte boundary."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    dev = torch.device("cuda")

    def view(src, dtype=torch.float32):
        raw = torch.empty(src.numel() + phase + 1, dtype=dtype, device=dev)
        v = raw[phase:phase + src.numel()].view(src.shape)
        v.copy_(src)
        return v

    reward = view(torch.randn(B, T, generator=g))
    done = view(torch.rand(B, T, generator=g) < 0.02, torch.bool)
    cur = view(torch.randn(n, generator=g) * 0.1 - 1.0)
    old = view(cur.cpu() + torch.randn(n, generator=g) * 0.1)
    adv = view(torch.randn(n, generator=g))
    ent = view(torch.rand(n, generator=g) * 2.0) if entropy else None
    return reward, done, cur, old, adv, ent


SHAPES = [
    (4096, 1000, 4_096_000),   # configs[1]
    (1, 1, 1),
    (7, 2111, 12_345),
    (33, 64, 4096),
    (1000, 3, 4095),
    (0, 5, 100_000),           # no reward-to-go rows
    (5, 0, 1000),              # zero-length rows
    (12, 700, 0),              # no PPO samples
    (3, 9000, 2_000_003),      # long rows, ragged PPO tail
    (20_000, 17, 64),          # many short rows, tiny PPO
]


@pytest.mark.parametrize("B,T,n", SHAPES, ids=[f"B{b}_T{t}_n{n}" for b, t, n in SHAPES])
@pytest.mark.parametrize("entropy", [True, False], ids=["ent", "noent"])
def test_fused_matches_separate(ops, B, T, n, entropy):
    reward, done, cur, old, adv, ent = make(B, T, n, seed=B * 31 + T + n, entropy=entropy)
    rtg_sep = ops.reward_to_go(reward, done, 0.99)
    ppo_sep = ops.ppo_clip(cur, old, adv, 0.2, ent)
    rtg_f = torch.full_like(reward, float("nan"))
    ppo_f = torch.full_like(ppo_sep, float("nan"))
    for _ in range(2):  # twice: the completion counter is left ready for the next call
        ops.rl_step(reward, done, 0.99, cur, old, adv, 0.2, ent, rtg_out=rtg_f, ppo_out=ppo_f)
        torch.cuda.synchronize()
        assert torch.equal(bits(rtg_f), bits(rtg_sep))
        assert torch.equal(bits(ppo_f), bits(ppo_sep))


@pytest.mark.parametrize("phase", [1, 2, 3])
def test_fused_misaligned(ops, phase):
    """Unaligned PPO streams take the scalar path; the bits still match the separate ops."""
    reward, done, cur, old, adv, ent = make(61, 333, 100_001, seed=phase, phase=phase)
    rtg_f, ppo_f = ops.rl_step(reward, done, 0.95, cur, old, adv, 0.2, ent)
    assert torch.equal(bits(rtg_f), bits(ops.reward_to_go(reward, done, 0.95)))
    assert torch.equal(bits(ppo_f), bits(ops.ppo_clip(cur, old, adv, 0.2, ent)))


def test_fused_baseline_against_oracle(ops):
    """configs[1] inputs of the oracle's generator, checked against the fp64 oracle directly."""
    s = inputs.baseline_inputs("rl_pipeline", seed=0)
    g = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in s.items()}
    rtg, ppo = ops.rl_step(g["reward"], g["done"], g["gamma"], g["current_log_prob"], g["old_log_prob"],
                           g["advantage"], g["clip_epsilon"], g["entropy"])
    bad, worst = exact.within(rtg.cpu().double().numpy(), exact.reward_to_go(s)["output"], 1e-5, 1e-5)
    assert bad == 0, worst
    ref = exact.ppo_clip(s, entropy=s["entropy"])["output"]
    bad, worst = exact.within(ppo.cpu().double().numpy(), ref, 1e-5, 1e-4)
    assert bad == 0, worst


def test_fused_shard_form(ops):
    """The shard form's partials equal b200_ppo_shard_partials' and finish to the same bits."""
    lib = pkg().load()
    reward, done, cur, old, adv, ent = make(300, 500, 1_000_003, seed=5)
    n = cur.numel()
    want = ops.ppo_partials(cur, old, adv, 0.2, ent)
    got = torch.zeros_like(want)
    rtg = torch.empty_like(reward)
    st = lib.b200_rl_step_shard_async(reward.data_ptr(), done.data_ptr(), 0.9, 300, 500, rtg.data_ptr(),
                                      cur.data_ptr(), old.data_ptr(), adv.data_ptr(), ent.data_ptr(), n, 0.2,
                                      got.data_ptr(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert torch.equal(bits(rtg), bits(ops.reward_to_go(reward, done, 0.9)))
    assert torch.equal(bits(ops.ppo_finish(got, n, True)), bits(ops.ppo_clip(cur, old, adv, 0.2, ent)))


def test_fused_status_codes(ops):
    lib = pkg().load()
    x = torch.zeros(64, device="cuda")
    out = torch.zeros(8, device="cuda")
    p = x.data_ptr()
    # negative sizes
    assert lib.b200_rl_step_async(p, p, 0.9, -1, 4, p, p, p, p, None, 16, 0.2, out.data_ptr(), p, 256, None) == 1
    assert lib.b200_rl_step_async(p, p, 0.9, 1, 4, p, p, p, p, None, -16, 0.2, out.data_ptr(), p, 256, None) == 1
    # workspace too small
    assert lib.b200_rl_step_async(p, p, 0.9, 1, 4, p, p, p, p, None, 16, 0.2, out.data_ptr(), p, 8, None) == 4
    # shard form without a partials buffer
    assert lib.b200_rl_step_shard_async(p, p, 0.9, 1, 4, p, p, p, p, None, 16, 0.2, None, None) == 1
