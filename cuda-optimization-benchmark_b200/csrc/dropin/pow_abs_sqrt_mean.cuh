// Drop-in body of task pow_abs_sqrt_mean: the reference's `void reference(const float* inp,
// const float* target, int64_t batch_size, int64_t height, int64_t width, float* output)`
// (tasks/pow_abs_sqrt_mean/tests/task.json:3), on the legacy default stream, scratch from the
// per-device arena.  Returns a b200 status.
#pragma once

#include "../common/workspace.cuh"
#include "../ops/robust_l1.cuh"

namespace b200 {
namespace dropin {

inline int pow_abs_sqrt_mean(const float* inp, const float* target, int64_t batch_size, int64_t height, int64_t width,
                             float* output) {
  const int64_t n = robust_l1::abi_count(batch_size, height, width);
  if (n < 0) return kInvalidArgument;
  int st = 0;
  const size_t ws = robust_l1::workspace_bytes(n);
  void* w = arena_get(kArenaRobustL1, ws, nullptr, &st);
  if (st != kOk) return st;
  return robust_l1::run(inp, target, n, output, w, ws, nullptr);
}

}  // namespace dropin
}  // namespace b200
