// Leaky integrate-and-fire layer: T sequential steps, B*H independent neurons.
//
// For each step t, in fp32 and in this order (tasks/leaky/reference.py:26-37, the oracle itself,
// and tasks/leaky/prompt.md "The operation"):
//   reset = mem >= th ? 1 : 0;  mem = beta*mem + x[t] - reset*th;  spikes[t] = mem >= th ? 1 : 0
// with beta clamped to [0, 1].  Every product and sum is rounded separately (no FMA contraction),
// so spikes and final_mem are bit-identical to the fp32 reference.  The drop-in boundary it
// replaces is `void reference(const float* input_current, const float* mem0, const float* beta,
// const float* threshold, int32_t T, int32_t B, int32_t H, float* spikes, float* final_mem)`
// (tasks/leaky/tests/task.json:3; expert launcher reference/leaky/solution.cu:106-138).
//
// B200 design: the membrane state lives in registers for the whole time loop; a thread owns 4
// consecutive neurons of the flattened (B*H) neuron axis (one 128-bit load of x[t] and one
// 128-bit streaming store of spikes[t] per step, coalesced across the warp), and keeps kDepth
// future time steps of x in flight in a register ring, so each SM always has loads outstanding.
// Unaligned pointers or B*H not a multiple of 4 take the one-neuron-per-thread form of the same
// loop.  8 bytes of HBM traffic per neuron-step (read x, write spike).
#pragma once

#include "../common/b200_common.cuh"

namespace b200 {
namespace lif {

constexpr int kThreads = 128;
constexpr int kDepth = 8;   // time steps of x in flight per thread

__device__ __forceinline__ float clamp01(float b) { return fminf(fmaxf(b, 0.0f), 1.0f); }

__device__ __forceinline__ float step(float& mem, float x, float beta, float th) {
  const float reset = mem >= th ? 1.0f : 0.0f;
  mem = __fsub_rn(__fadd_rn(__fmul_rn(beta, mem), x), __fmul_rn(reset, th));
  return mem >= th ? 1.0f : 0.0f;
}

// Vector form: thread owns neurons [4v, 4v+4) of the flattened neuron axis (NB = B*H, NB % 4 == 0).
__global__ void __launch_bounds__(kThreads) lif_vec_kernel(const float* __restrict__ x, const float* __restrict__ mem0,
                                                           const float* __restrict__ beta,
                                                           const float* __restrict__ th, int T, int64_t NB, int H,
                                                           float* __restrict__ spikes, float* __restrict__ final_mem) {
  const int64_t v = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  if (v * 4 >= NB) return;
  const int64_t i0 = v * 4;
  float4 m = *reinterpret_cast<const float4*>(mem0 + i0);
  float bq[4], tq[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int h = int((i0 + j) % H);
    bq[j] = clamp01(beta[h]);
    tq[j] = th[h];
  }
  const float* xp = x + i0;
  float* sp = spikes + i0;
  float4 ring[kDepth];
#pragma unroll
  for (int d = 0; d < kDepth; ++d)
    if (d < T) ring[d] = ld_stream_f4(xp + int64_t(d) * NB);
  for (int t0 = 0; t0 < T; t0 += kDepth) {
#pragma unroll
    for (int d = 0; d < kDepth; ++d) {
      const int t = t0 + d;
      if (t < T) {
        const float4 xv = ring[d];
        if (t + kDepth < T) ring[d] = ld_stream_f4(xp + int64_t(t + kDepth) * NB);
        float4 s;
        s.x = step(m.x, xv.x, bq[0], tq[0]);
        s.y = step(m.y, xv.y, bq[1], tq[1]);
        s.z = step(m.z, xv.z, bq[2], tq[2]);
        s.w = step(m.w, xv.w, bq[3], tq[3]);
        st_stream_f4(sp + int64_t(t) * NB, s);
      }
    }
  }
  *reinterpret_cast<float4*>(final_mem + i0) = m;
}

// Scalar form: one neuron per thread, same per-neuron arithmetic.
__global__ void __launch_bounds__(kThreads) lif_scalar_kernel(const float* __restrict__ x,
                                                              const float* __restrict__ mem0,
                                                              const float* __restrict__ beta,
                                                              const float* __restrict__ th, int T, int64_t NB, int H,
                                                              float* __restrict__ spikes,
                                                              float* __restrict__ final_mem) {
  const int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  if (i >= NB) return;
  float m = mem0[i];
  const int h = int(i % H);
  const float b = clamp01(beta[h]);
  const float tt = th[h];
  float ring[kDepth];
#pragma unroll
  for (int d = 0; d < kDepth; ++d)
    if (d < T) ring[d] = ld_stream_f1(x + i + int64_t(d) * NB);
  for (int t0 = 0; t0 < T; t0 += kDepth) {
#pragma unroll
    for (int d = 0; d < kDepth; ++d) {
      const int t = t0 + d;
      if (t < T) {
        const float xv = ring[d];
        if (t + kDepth < T) ring[d] = ld_stream_f1(x + i + int64_t(t + kDepth) * NB);
        st_stream_f1(spikes + i + int64_t(t) * NB, step(m, xv, b, tt));
      }
    }
  }
  final_mem[i] = m;
}

inline int run(const float* x, const float* mem0, const float* beta, const float* th, int32_t T, int32_t B, int32_t H,
               float* spikes, float* final_mem, cudaStream_t stream) {
  if (T < 0 || B < 0 || H < 0) return kInvalidArgument;
  const int64_t NB = int64_t(B) * int64_t(H);
  if (NB == 0) return kOk;
  if (mem0 == nullptr || beta == nullptr || th == nullptr || final_mem == nullptr) return kInvalidArgument;
  if (T > 0 && (x == nullptr || spikes == nullptr)) return kInvalidArgument;
  const bool vec = (NB % 4 == 0) && aligned16(mem0) && aligned16(final_mem) && (T == 0 || (aligned16(x) && aligned16(spikes)));
  if (vec) {
    const int64_t threads = NB / 4;
    const int64_t grid = (threads + kThreads - 1) / kThreads;
    lif_vec_kernel<<<unsigned(grid), kThreads, 0, stream>>>(x, mem0, beta, th, T, NB, H, spikes, final_mem);
  } else {
    const int64_t grid = (NB + kThreads - 1) / kThreads;
    lif_scalar_kernel<<<unsigned(grid), kThreads, 0, stream>>>(x, mem0, beta, th, T, NB, H, spikes, final_mem);
  }
  return launch_status();
}

}  // namespace lif
}  // namespace b200
