// Generalised advantage estimation (GAE), the step between the returns and the PPO loss in an RL
// pipeline (TorchRL's generalized_advantage_estimate, the caller of reward-to-go and ppo_clip in
// the reference's source library; the algorithm of Schulman et al., "High-Dimensional Continuous
// Control Using Generalized Advantage Estimation", 2016).  Per row of [B, T], time along T:
//
//   delta[t]        = reward[t] + gamma * next_value[t] * (1 - terminated[t]) - value[t]
//   advantage[t]    = delta[t] + gamma * lambda * (1 - done[t]) * advantage[t + 1]   (0 past T-1)
//   value_target[t] = advantage[t] + value[t]
//
// done ends the recursion (a trajectory boundary); terminated drops the bootstrap value (a
// terminal state, as opposed to a truncation).  The advantage recursion is the reward-to-go scan
// with delta in place of the reward and gamma * lambda in place of gamma, so it runs through
// rtg::run (fp64 composition of each lane's run, fp32 re-run from exact carries), with delta
// staged in the value-target buffer:
//   1. delta_kernel: delta into value_target (13 bytes read, 4 written per element);
//   2. rtg::run from value_target into advantage (9 read, 4 written);
//   3. target_kernel: value_target = advantage + value (8 read, 4 written).
#pragma once

#include "../common/b200_common.cuh"
#include "reward_to_go.cuh"

namespace b200 {
namespace gae {

constexpr int kThreads = 256;

__device__ __forceinline__ float delta1(float r, float v, float nv, unsigned char term, float gamma) {
  const float boot = term ? 0.0f : __fmul_rn(gamma, nv);
  return __fsub_rn(__fadd_rn(r, boot), v);
}

// kVec: four elements per thread per step (16-byte aligned float streams, done bytes in 4s).
template <bool kVec>
__global__ void __launch_bounds__(kThreads) delta_kernel(const float* __restrict__ r, const float* __restrict__ v,
                                                         const float* __restrict__ nv,
                                                         const unsigned char* __restrict__ term, float gamma,
                                                         int64_t n, float* __restrict__ delta) {
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  const int64_t stride = int64_t(gridDim.x) * kThreads, t0 = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t quads = kVec ? n / 4 : 0;
  for (int64_t q = t0; q < quads; q += stride) {
    const float4 a = ld_stream_f4(r + 4 * q), b = ld_stream_f4(v + 4 * q), c = ld_stream_f4(nv + 4 * q);
    const uint32_t m = __ldg(reinterpret_cast<const uint32_t*>(term) + q);
    float4 d;
    d.x = delta1(a.x, b.x, c.x, (unsigned char)(m & 0xffu), gamma);
    d.y = delta1(a.y, b.y, c.y, (unsigned char)((m >> 8) & 0xffu), gamma);
    d.z = delta1(a.z, b.z, c.z, (unsigned char)((m >> 16) & 0xffu), gamma);
    d.w = delta1(a.w, b.w, c.w, (unsigned char)(m >> 24), gamma);
    *reinterpret_cast<float4*>(delta + 4 * q) = d;  // re-read at once by the scan: keep it in L2
  }
  for (int64_t i = quads * 4 + t0; i < n; i += stride) delta[i] = delta1(r[i], v[i], nv[i], term[i], gamma);
}

template <bool kVec>
__global__ void __launch_bounds__(kThreads) target_kernel(const float* __restrict__ adv, const float* __restrict__ v,
                                                          int64_t n, float* __restrict__ target) {
  pdl_begin();  // the advantages are written by the scan just before this kernel
  const int64_t stride = int64_t(gridDim.x) * kThreads, t0 = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t quads = kVec ? n / 4 : 0;
  for (int64_t q = t0; q < quads; q += stride) {
    const float4 a = ld_stream_f4(adv + 4 * q), b = ld_stream_f4(v + 4 * q);
    st_stream_f4(target + 4 * q, make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z),
                                             __fadd_rn(a.w, b.w)));
  }
  for (int64_t i = quads * 4 + t0; i < n; i += stride) target[i] = __fadd_rn(adv[i], v[i]);
}

inline int elementwise_grid(int64_t n) {
  const int64_t want = (n / 4 + kThreads - 1) / kThreads;
  const int64_t cap = int64_t(sm_count()) * 8;
  return int(want < 1 ? 1 : (want < cap ? want : cap));
}

// All tensors [B, T] row-major; done and terminated hold one byte per element (bool).
inline int run(const float* reward, const float* value, const float* next_value, const unsigned char* done,
               const unsigned char* terminated, float gamma, float lmbda, int32_t B, int32_t T, float* advantage,
               float* value_target, cudaStream_t stream) {
  if (B < 0 || T < 0) return kInvalidArgument;
  const int64_t n = int64_t(B) * int64_t(T);
  if (n == 0) return kOk;
  if (reward == nullptr || value == nullptr || next_value == nullptr || done == nullptr || terminated == nullptr ||
      advantage == nullptr || value_target == nullptr)
    return kInvalidArgument;
  const bool vec = aligned16(reward) && aligned16(value) && aligned16(next_value) && aligned16(advantage) &&
                   aligned16(value_target) && (reinterpret_cast<uintptr_t>(terminated) & 3u) == 0;
  const int grid = elementwise_grid(n);
  int st = vec ? launch_pdl(delta_kernel<true>, grid, kThreads, 0, stream, reward, value, next_value, terminated,
                            gamma, n, value_target)
               : launch_pdl(delta_kernel<false>, grid, kThreads, 0, stream, reward, value, next_value, terminated,
                            gamma, n, value_target);
  if (st != kOk) return st;
  // gamma * lambda rounded once to fp32 (the scan's coefficient); the scan composes it in fp64.
  const float gl = float(double(gamma) * double(lmbda));
  st = rtg::run(value_target, done, gl, B, T, advantage, stream);
  if (st != kOk) return st;
  return vec ? launch_pdl(target_kernel<true>, grid, kThreads, 0, stream, static_cast<const float*>(advantage),
                          value, n, value_target)
             : launch_pdl(target_kernel<false>, grid, kThreads, 0, stream, static_cast<const float*>(advantage),
                          value, n, value_target);
}

}  // namespace gae
}  // namespace b200
