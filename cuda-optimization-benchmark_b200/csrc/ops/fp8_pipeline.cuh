// FP8 linear layer from a bf16 activation: the per-tensor E4M3 quantisation of x
// (tasks/fp8_linear/reference.py:15-18) and the E4M3 GEMM (reference.py:34-37) in one call, the
// activation scale never leaving the device.  x is quantised into the workspace (amax, scale, cast:
// fp8_quant.cuh); the GEMM kernels read the epilogue factor 1 / (scale_x * scale_w) that the amax
// kernel leaves in the workspace header, computed in fp64 exactly as fp8_linear computes it on the
// host, so the output is bit-identical to quantising x and calling fp8_linear with the scales.
#pragma once

#include "fp8_linear.cuh"
#include "fp8_quant.cuh"

namespace b200 {
namespace fp8q {

inline size_t linear_workspace_bytes(int64_t M, int64_t K) {
  return workspace_bytes() + align256(size_t(M) * size_t(K));
}

// workspace: linear_workspace_bytes(M, K), its first 4 bytes zero before the first call.
// scale_x_out (device, may be null) receives the activation scale.
inline int linear_bf16(int32_t M, int32_t K, int32_t N, const void* x, const uint8_t* w, float scale_w,
                       const uint16_t* bias, uint16_t* out, float* scale_x_out, void* workspace, size_t ws_bytes,
                       cudaStream_t stream) {
  if (M < 0 || K < 0 || N < 0) return kInvalidArgument;
  if (int64_t(M) * K > 0 && x == nullptr) return kInvalidArgument;
  if (workspace == nullptr || ws_bytes < linear_workspace_bytes(M, K)) return kWorkspaceTooSmall;
  uint8_t* q = static_cast<uint8_t*>(workspace) + workspace_bytes();
  const int st = run(x, true, int64_t(M) * K, q, scale_x_out, scale_w, workspace, workspace_bytes(), stream);
  if (st != kOk) return st;
  const Header* hdr = static_cast<const Header*>(workspace);
  return fp8::run(M, K, N, q, 1.0f, w, scale_w, bias, out, stream, &hdr->epi);
}

}  // namespace fp8q
}  // namespace b200
