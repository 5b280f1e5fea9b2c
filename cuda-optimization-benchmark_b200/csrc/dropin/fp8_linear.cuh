// Drop-in body of task fp8_linear: the reference's `void reference(const int32_t M, const int32_t K,
// const int32_t N, const __nv_fp8_e4m3* x_fp8, float scale_x, const __nv_fp8_e4m3* w_fp8, float
// scale_w, const __nv_bfloat16* bias, __nv_bfloat16* output)` (tasks/fp8_linear/tests/task.json:3),
// with the fp8 and bf16 buffers passed as their raw bytes, on the legacy default stream.
#pragma once

#include "../ops/fp8_linear.cuh"

namespace b200 {
namespace dropin {

inline int fp8_linear(int32_t M, int32_t K, int32_t N, const uint8_t* x_fp8, float scale_x, const uint8_t* w_fp8,
                      float scale_w, const uint16_t* bias, uint16_t* output) {
  return fp8::run(M, K, N, x_fp8, scale_x, w_fp8, scale_w, bias, output, nullptr);
}

}  // namespace dropin
}  // namespace b200
