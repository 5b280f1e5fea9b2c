// Discounted reward-to-go with done flags: a reverse segmented scan along T for every row.
//
//   out[b, t] = reward[b, t] + gamma * (t == T-1 or done[b, t] ? 0 : out[b, t+1])
//
// Reference semantics: tasks/reward_to_go/prompt.md "The operation"; fp64 oracle
// tasks/reward_to_go/reference.py:34-42 (backward loop).  The drop-in boundary it replaces is
// `void reference(const float* reward, const bool* done, float gamma, int32_t B, int32_t T,
// float* output)` (tasks/reward_to_go/tests/task.json:3; expert launcher
// reference/reward_to_go/solution.cu:237-264).
//
// B200 design.  The recurrence is an affine map per step, y -> r[t] + a[t] * y with
// a[t] = done[t] ? 0 : gamma, so a run of steps composes to y -> B + A * y.  One warp owns one row
// at a time and walks it from the end in passes of kSeg = 32 * kLane elements:
//   1. the warp stages the pass's rewards and done bytes in shared memory with 128-bit loads
//      (the shared copy keeps the global 16-byte phase, so every full group is one vector
//      load and one vector shared store; edge groups use scalar loads);
//   2. lane l composes its contiguous run of kLane steps (kLane is odd, so the 32 lanes' strided
//      shared reads fall in 32 distinct banks);
//   3. a 5-step warp suffix scan of the lanes' (A, B) maps gives every lane its incoming value;
//   4. lane l re-runs its steps from that value and writes the outputs over the rewards in
//      shared memory, and the warp streams them out with 128-bit stores.
// The recurrence runs in fp64 (one fp32->fp64 conversion per read, one rounding per output), so
// the result is the fp64 oracle rounded once, independent of how rows are split into passes.
#pragma once

#include "../common/b200_common.cuh"

namespace b200 {
namespace rtg {

constexpr int kLane = 33;                    // steps per lane per pass (odd: conflict-free banks)
constexpr int kSeg = 32 * kLane;             // steps per warp pass
constexpr int kWarps = 4;                    // warps (rows in flight) per CTA
constexpr int kThreads = 32 * kWarps;
constexpr int kCtasPerSm = 10;
// Per-warp shared memory: kSeg floats (+16 B phase slack) and kSeg done bytes (+16 B slack).
constexpr int kRewardBytes = ((kSeg * 4 + 16) + 15) / 16 * 16;
constexpr int kDoneBytes = ((kSeg + 16) + 15) / 16 * 16;
constexpr int kWarpSmem = kRewardBytes + kDoneBytes;
constexpr int kSmemBytes = kWarps * kWarpSmem;

// Stage src[0..len) (floats) into shared memory at sdst[phase .. phase+len), where phase is the
// float offset of src within its 16-byte group.  Returns the phase.
__device__ __forceinline__ int stage_floats(const float* __restrict__ src, int len, float* sdst, int lane) {
  const int phase = int((reinterpret_cast<uintptr_t>(src) >> 2) & 3);
  const float* base = src - phase;  // 16-byte aligned; only in-range elements are dereferenced
  const int groups = (phase + len + 3) >> 2;
  for (int q = lane; q < groups; q += 32) {
    const int e0 = q * 4 - phase;
    if (e0 >= 0 && e0 + 4 <= len) {
      const float4 v = ld_stream_f4(base + q * 4);
      *reinterpret_cast<float4*>(sdst + q * 4) = v;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int e = e0 + j;
        if (e >= 0 && e < len) sdst[q * 4 + j] = ld_stream_f1(src + e);
      }
    }
  }
  return phase;
}

__device__ __forceinline__ unsigned char ld_stream_u8(const unsigned char* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u8 %0, [%1];" : "=h"(v) : "l"(p));
  return (unsigned char)v;
}

// Same for bytes: phase is the byte offset of src within its 16-byte group.
__device__ __forceinline__ int stage_bytes(const unsigned char* __restrict__ src, int len, unsigned char* sdst,
                                           int lane) {
  const int phase = int(reinterpret_cast<uintptr_t>(src) & 15);
  const unsigned char* base = src - phase;
  const int groups = (phase + len + 15) >> 4;
  for (int q = lane; q < groups; q += 32) {
    const int e0 = q * 16 - phase;
    if (e0 >= 0 && e0 + 16 <= len) {
      const uint4 v = ld_stream_u4(base + q * 16);
      *reinterpret_cast<uint4*>(sdst + q * 16) = v;
    } else {
      for (int j = 0; j < 16; ++j) {
        const int e = e0 + j;
        if (e >= 0 && e < len) sdst[q * 16 + j] = ld_stream_u8(src + e);
      }
    }
  }
  return phase;
}

// Write sfrom[phase .. phase+len) to dst[0..len).  When dst has the same 16-byte phase as the
// staged data, full groups go out as 128-bit streaming stores; otherwise lane-strided scalars.
__device__ __forceinline__ void drain_floats(float* __restrict__ dst, int len, const float* sfrom, int phase,
                                             int lane) {
  const int dphase = int((reinterpret_cast<uintptr_t>(dst) >> 2) & 3);
  if (dphase == phase) {
    float* base = dst - phase;
    const int groups = (phase + len + 3) >> 2;
    for (int q = lane; q < groups; q += 32) {
      const int e0 = q * 4 - phase;
      if (e0 >= 0 && e0 + 4 <= len) {
        st_stream_f4(base + q * 4, *reinterpret_cast<const float4*>(sfrom + q * 4));
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int e = e0 + j;
          if (e >= 0 && e < len) st_stream_f1(dst + e, sfrom[q * 4 + j]);
        }
      }
    }
  } else {
    for (int e = lane; e < len; e += 32) st_stream_f1(dst + e, sfrom[phase + e]);
  }
}

// One warp, one row: walks [0, T) from the end in passes of kSeg steps.
__device__ __forceinline__ void scan_row(const float* __restrict__ rrow, const unsigned char* __restrict__ drow,
                                         float* __restrict__ orow, int T, double gamma, float* s_r,
                                         unsigned char* s_d, int lane) {
  double carry = 0.0;  // value of out[t1] for the pass [t0, t1); 0 past the row end
  for (int t1 = T; t1 > 0; t1 -= kSeg) {
    const int t0 = t1 > kSeg ? t1 - kSeg : 0;
    const int len = t1 - t0;
    const int pr = stage_floats(rrow + t0, len, s_r, lane);
    const int pd = stage_bytes(drow + t0, len, s_d, lane);
    __syncwarp();

    // Lane l owns steps [l*kLane, min((l+1)*kLane, len)) of the pass.
    const int lo = lane * kLane;
    const int hi = min(lo + kLane, len);
    double A = 1.0, Bv = 0.0;
    for (int e = hi - 1; e >= lo; --e) {
      const double a = s_d[pd + e] ? 0.0 : gamma;
      Bv = fma(a, Bv, double(s_r[pr + e]));
      A *= a;
    }
    // Inclusive suffix composition over lanes: lane l gets f_l o f_{l+1} o ... o f_31.
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const double A2 = __shfl_down_sync(0xffffffffu, A, d);
      const double B2 = __shfl_down_sync(0xffffffffu, Bv, d);
      if (lane + d < 32) {
        Bv = fma(A, B2, Bv);
        A *= A2;
      }
    }
    const double start = fma(A, carry, Bv);                  // out[t0 + lo]
    double y = __shfl_down_sync(0xffffffffu, start, 1);      // out[t0 + hi] for lanes < 31
    if (lane == 31) y = carry;
    const double next_carry = __shfl_sync(0xffffffffu, start, 0);
    for (int e = hi - 1; e >= lo; --e) {
      const double a = s_d[pd + e] ? 0.0 : gamma;
      y = fma(a, y, double(s_r[pr + e]));
      s_r[pr + e] = float(y);
    }
    __syncwarp();
    drain_floats(orow + t0, len, s_r, pr, lane);
    __syncwarp();
    carry = next_carry;
  }
}

__global__ void __launch_bounds__(kThreads) rtg_kernel(const float* __restrict__ reward,
                                                       const unsigned char* __restrict__ done, float gamma,
                                                       int B, int T, float* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* s_r = reinterpret_cast<float*>(smem + warp * kWarpSmem);
  unsigned char* s_d = smem + warp * kWarpSmem + kRewardBytes;
  const double g = double(gamma);
  for (int64_t row = int64_t(blockIdx.x) * kWarps + warp; row < B; row += int64_t(gridDim.x) * kWarps) {
    const int64_t off = row * int64_t(T);
    scan_row(reward + off, done + off, out + off, T, g, s_r, s_d, lane);
  }
}

inline int run(const float* reward, const unsigned char* done, float gamma, int32_t B, int32_t T, float* out,
               cudaStream_t stream) {
  if (B < 0 || T < 0) return kInvalidArgument;
  if (B == 0 || T == 0) return kOk;
  if (reward == nullptr || done == nullptr || out == nullptr) return kInvalidArgument;
  const int64_t ctas_needed = (int64_t(B) + kWarps - 1) / kWarps;
  const int64_t cap = int64_t(sm_count()) * kCtasPerSm;
  const int grid = int(ctas_needed < cap ? ctas_needed : cap);
  rtg_kernel<<<grid, kThreads, kSmemBytes, stream>>>(reward, done, gamma, B, T, out);
  return launch_status();
}

}  // namespace rtg
}  // namespace b200
