// Drop-in body of task efficient_kan: the reference's `void reference(const float* x, const float*
// grid, const float* base_weight, const float* spline_weight, const float* spline_scaler, int32_t
// grid_size, int32_t spline_order, int32_t B, int32_t I, int32_t O, float* out)`
// (tasks/efficient_kan/tests/task.json:3), on the legacy default stream, scratch (the fp16 operand
// planes) from the per-device arena.
#pragma once

#include "../common/workspace.cuh"
#include "../ops/kan.cuh"

namespace b200 {
namespace dropin {

inline int efficient_kan(const float* x, const float* grid, const float* base_weight, const float* spline_weight,
                         const float* spline_scaler, int32_t grid_size, int32_t spline_order, int32_t B, int32_t I,
                         int32_t O, float* out) {
  if (B < 0 || I < 0 || O < 0 || grid_size < 1 || spline_order < 0) return kInvalidArgument;
  int st = 0;
  const size_t ws = kan::workspace_bytes(B, I, O, grid_size + spline_order);
  void* w = arena_get(kArenaKan, ws, nullptr, &st);
  if (st != kOk) return st;
  return kan::run(x, grid, base_weight, spline_weight, spline_scaler, grid_size, spline_order, B, I, O, out, w, ws,
                  nullptr);
}

}  // namespace dropin
}  // namespace b200
