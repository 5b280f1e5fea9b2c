// Drop-in body of task leaky: the reference's `void reference(const float* input_current,
// const float* mem0, const float* beta, const float* threshold, int32_t T, int32_t B, int32_t H,
// float* spikes, float* final_mem)` (tasks/leaky/tests/task.json:3), on the legacy default stream.
#pragma once

#include "../ops/lif.cuh"

namespace b200 {
namespace dropin {

inline int leaky(const float* input_current, const float* mem0, const float* beta, const float* threshold, int32_t T,
                 int32_t B, int32_t H, float* spikes, float* final_mem) {
  return lif::run(input_current, mem0, beta, threshold, T, B, H, spikes, final_mem, nullptr);
}

}  // namespace dropin
}  // namespace b200
