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
//   1. lane 0 moves the 16-byte aligned interior of the pass's rewards and done bytes into
//      shared memory with one cp.async.bulk each (counted on the warp's mbarrier); the lanes
//      load the ragged ends (the shared copy keeps the global 16-byte phase);
//   2. lane l composes its contiguous run of kLane steps in fp64 (kLane is odd, so the 32 lanes'
//      strided shared reads fall in 32 distinct banks);
//   3. a 5-step warp suffix scan of the lanes' (A, B) maps, in fp64, gives every lane the exact
//      value entering its run;
//   4. lane l re-runs its steps from that value in fp32 (at most kLane roundings per output, no
//      error carried between runs) and writes the outputs over the rewards in shared memory,
//      and the warp streams them out with 128-bit stores.
// One warp per row and 40 warps per SM put every row of the BASELINE batch in flight at once.
#pragma once

#include "../common/b200_common.cuh"
#include "../common/bulk.cuh"

namespace b200 {
namespace rtg {

constexpr int kLane = 33;                    // steps per lane per pass (odd: conflict-free banks)
constexpr int kSeg = 32 * kLane;             // steps per warp pass
constexpr int kWarps = 4;                    // warps (rows in flight) per CTA
constexpr int kThreads = 32 * kWarps;
// Per-warp shared memory: kSeg floats (+16 B phase slack) and kSeg done bytes (+16 B slack).
constexpr int kRewardBytes = ((kSeg * 4 + 16) + 15) / 16 * 16;
constexpr int kDoneBytes = ((kSeg + 16) + 15) / 16 * 16;
constexpr int kWarpSmem = kRewardBytes + kDoneBytes;
constexpr int kSmemBytes = kWarps * kWarpSmem;

// Stage src[0..len) (floats) into shared memory at sdst[phase .. phase+len), where phase is the
// float offset of src within its 16-byte group (so the 16-byte aligned interior of the range maps
// to 16-byte aligned shared addresses).  Lane 0 moves the aligned interior with one bulk copy
// counted on `bar`; the lanes load the ragged head and tail (< 4 elements each) themselves.
// Returns the number of bytes the bulk copy will deliver (0 when there is no interior).
__device__ __forceinline__ uint32_t stage_floats(const float* __restrict__ src, int len, float* sdst, int phase,
                                                 uint64_t* bar, int lane) {
  const int ea = (4 - phase) & 3;                       // first element on a 16-byte boundary
  const int eb = len > ea ? ea + ((len - ea) & ~3) : ea;  // end of the aligned interior
  const uint32_t bytes = len > ea ? uint32_t(eb - ea) * 4u : 0u;
  if (lane == 0 && bytes) bulk_g2s(sdst + phase + ea, src + ea, bytes, bar);
  const int head = len < ea ? len : ea;
  if (lane < head) sdst[phase + lane] = ld_stream_f1(src + lane);
  if (lane < len - eb && eb < len) sdst[phase + eb + lane] = ld_stream_f1(src + eb + lane);
  return bytes;
}

__device__ __forceinline__ unsigned char ld_stream_u8(const unsigned char* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u8 %0, [%1];" : "=h"(v) : "l"(p));
  return (unsigned char)v;
}

// Same for bytes (16-byte phase; head and tail up to 15 bytes each).
__device__ __forceinline__ uint32_t stage_bytes(const unsigned char* __restrict__ src, int len, unsigned char* sdst,
                                                int phase, uint64_t* bar, int lane) {
  const int ea = (16 - phase) & 15;
  const int eb = len > ea ? ea + ((len - ea) & ~15) : ea;
  const uint32_t bytes = len > ea ? uint32_t(eb - ea) : 0u;
  if (lane == 0 && bytes) bulk_g2s(sdst + phase + ea, src + ea, bytes, bar);
  const int head = len < ea ? len : ea;
  if (lane < head) sdst[phase + lane] = ld_stream_u8(src + lane);
  if (lane < len - eb && eb < len) sdst[phase + eb + lane] = ld_stream_u8(src + eb + lane);
  return bytes;
}

// Write sfrom[phase .. phase+len) to dst[0..len).  When dst has the same 16-byte phase as the
// staged data, full groups go out as 128-bit streaming stores; otherwise lane-strided scalars.
__device__ __forceinline__ void drain_floats(float* __restrict__ dst, int len, const float* sfrom, int phase,
                                             int lane) {
  const int dphase = int((reinterpret_cast<uintptr_t>(dst) >> 2) & 3);
  if (dphase == phase) {
    float* base = dst - phase;
    const int groups = (phase + len + 3) >> 2;
#pragma unroll 4
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
#pragma unroll 4
    for (int e = lane; e < len; e += 32) st_stream_f1(dst + e, sfrom[phase + e]);
  }
}

// One warp, one row: walks [0, T) from the end in passes of kSeg steps.  `bar` is this warp's
// mbarrier and `uses` counts its completed phases (carried across rows).
__device__ __forceinline__ void scan_row(const float* __restrict__ rrow, const unsigned char* __restrict__ drow,
                                         float* __restrict__ orow, int T, double gamma, float gamma_f, float* s_r,
                                         unsigned char* s_d, uint64_t* bar, uint32_t& uses, int lane) {
  double carry = 0.0;  // value of out[t1] for the pass [t0, t1); 0 past the row end
  for (int t1 = T; t1 > 0; t1 -= kSeg) {
    const int t0 = t1 > kSeg ? t1 - kSeg : 0;
    const int len = t1 - t0;
    const float* rs = rrow + t0;
    const unsigned char* ds = drow + t0;
    const int pr = int((reinterpret_cast<uintptr_t>(rs) >> 2) & 3);
    const int pd = int(reinterpret_cast<uintptr_t>(ds) & 15);
    // Shared memory written by the previous pass through ordinary stores is about to be
    // overwritten by the bulk-copy engine: order the two.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    // Byte counts are known before either copy is issued, so the expect_tx arrive goes first.
    const int ear = (4 - pr) & 3, ead = (16 - pd) & 15;
    const uint32_t rb = len > ear ? uint32_t((len - ear) & ~3) * 4u : 0u;
    const uint32_t db = len > ead ? uint32_t((len - ead) & ~15) : 0u;
    if (lane == 0) mbar_arrive_expect_tx(bar, rb + db);
    stage_floats(rs, len, s_r, pr, bar, lane);
    stage_bytes(ds, len, s_d, pd, bar, lane);
    mbar_wait(bar, uses & 1u);
    ++uses;
    __syncwarp();

    // Lane l owns steps [l*kLane, min((l+1)*kLane, len)) of the pass.
    const int lo = lane * kLane;
    const int hi = min(lo + kLane, len);
    double A = 1.0, Bv = 0.0;
    unsigned long long dmask = 0;  // bit (e - lo) set when done[t0 + e]
    for (int e = hi - 1; e >= lo; --e) {
      const bool d = s_d[pd + e] != 0;
      dmask |= (unsigned long long)d << (e - lo);
      const double a = d ? 0.0 : gamma;
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
    double yin = __shfl_down_sync(0xffffffffu, start, 1);    // out[t0 + hi] for lanes < 31
    if (lane == 31) yin = carry;
    const double next_carry = __shfl_sync(0xffffffffu, start, 0);
    // Second pass from the exact incoming value, in fp32: at most kLane roundings per output.
    float y = float(yin);
    for (int e = hi - 1; e >= lo; --e) {
      const float a = (dmask >> (e - lo)) & 1ull ? 0.0f : gamma_f;
      y = __fmaf_rn(a, y, s_r[pr + e]);
      s_r[pr + e] = y;
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
  __shared__ uint64_t bars[kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* s_r = reinterpret_cast<float*>(smem + warp * kWarpSmem);
  unsigned char* s_d = smem + warp * kWarpSmem + kRewardBytes;
  if (lane == 0) {
    mbar_init(&bars[warp], 1);
    fence_barrier_init();
  }
  __syncwarp();
  uint32_t uses = 0;
  const double g = double(gamma);
  for (int64_t row = int64_t(blockIdx.x) * kWarps + warp; row < B; row += int64_t(gridDim.x) * kWarps) {
    const int64_t off = row * int64_t(T);
    scan_row(reward + off, done + off, out + off, T, g, gamma, s_r, s_d, &bars[warp], uses, lane);
  }
}

inline int run(const float* reward, const unsigned char* done, float gamma, int32_t B, int32_t T, float* out,
               cudaStream_t stream) {
  if (B < 0 || T < 0) return kInvalidArgument;
  if (B == 0 || T == 0) return kOk;
  if (reward == nullptr || done == nullptr || out == nullptr) return kInvalidArgument;
  const int64_t ctas_needed = (int64_t(B) + kWarps - 1) / kWarps;
  const int64_t cap = int64_t(sm_count()) * resident_ctas_per_sm(rtg_kernel, kThreads, kSmemBytes);
  const int grid = int(ctas_needed < cap ? ctas_needed : cap);
  rtg_kernel<<<grid, kThreads, kSmemBytes, stream>>>(reward, done, gamma, B, T, out);
  return launch_status();
}

}  // namespace rtg
}  // namespace b200
