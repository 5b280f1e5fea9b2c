// Drop-in body of task ppo_clip: the reference's `void reference(const int32_t B, const int32_t T,
// const int32_t H, const float* current_log_prob, const float* old_log_prob, const float*
// advantage, const float clip_epsilon, float* output)` (tasks/ppo_clip/tests/task.json:3), on
// the legacy default stream, scratch from the per-device arena.  `entropy` may be null (the
// reference's six outputs) or a per-sample stream (a seventh output, its mean).
#pragma once

#include "../common/workspace.cuh"
#include "../ops/ppo_clip.cuh"

namespace b200 {
namespace dropin {

inline int ppo_clip(int32_t B, int32_t T, int32_t H, const float* cur, const float* old, const float* adv,
                    const float* entropy, float clip_epsilon, float* output) {
  const int64_t n = ppo::abi_count(B, T, H);
  if (n < 0) return kInvalidArgument;
  int st = 0;
  const size_t ws = ppo::workspace_bytes(n);
  void* w = arena_get(kArenaPpo, ws, nullptr, &st);
  if (st != kOk) return st;
  return ppo::run(cur, old, adv, entropy, n, clip_epsilon, output, w, ws, nullptr);
}

}  // namespace dropin
}  // namespace b200
