// Reward-to-go over long rows: parallel along T within a row, and sharded along T across GPUs.
//
// reward_to_go.cuh gives every row to one warp, so a batch of few, long rows (T >> B: one long
// episode stream, or the reference's B1_T8000 case at larger T) runs on a handful of warps.  Here a
// row is cut into chunks of rtg::kSeg steps, aligned from its end exactly like the passes of the
// one-warp scan, and every chunk gets its own warp:
//   1. map_kernel: each chunk's affine map y_left = B + A * y_right in fp64 (the lane runs and the
//      warp composition of rtg::scan_pass, with the slots before a short chunk's start as
//      identities);
//   2. carry_kernel: per row, one CTA composes the chunk maps from the end of the row (a thread
//      owns a block of consecutive chunks; a CTA scan of the blocks' maps, then each thread walks
//      its block) and writes the value entering every chunk from the right, starting from y0 = 0, or
//      from this rank's carry-in when the row's steps are sharded over ranks; it can also write the
//      map of the whole row slice;
//   3. scan_kernel: each chunk re-runs rtg::scan_pass from its exact fp64 carry, so every output
//      takes at most kLane fp32 roundings, as in the one-warp scan.
// 14 bytes per element of HBM traffic (reward and done read twice, output written once) instead
// of 9, in exchange for B * ceil(T / kSeg) warps instead of B.
//
// Multi-GPU over time: rank r holds steps [r * T_loc, (r + 1) * T_loc) of every row.  Step 1 and
// the slice map of step 2 run first (slice_maps); the ranks all-gather the [B] slice maps (16
// bytes per row per rank); then each rank's carry-in is the composition of the slices of the
// ranks after it applied to 0, and steps 2 and 3 finish its slice (slice_scan).  The outputs equal
// the one-GPU chunked scan's up to the fp64 association of the carries (the oracle's tolerance).
#pragma once

#include "../common/b200_common.cuh"
#include "reward_to_go.cuh"

namespace b200 {
namespace rtgc {

constexpr int kWarps = 4;  // chunks in flight per CTA, one staging buffer each
constexpr int kThreads = 32 * kWarps;
constexpr int kCarryThreads = 256;  // one row per CTA in carry_kernel

struct Map {
  double a, b;  // y_left = b + a * y_right
};

inline int64_t chunk_count(int32_t T) { return T <= 0 ? 0 : (int64_t(T) + rtg::kSeg - 1) / rtg::kSeg; }

inline int64_t workspace_bytes(int32_t B, int32_t T) {
  if (B <= 0 || T <= 0) return 0;
  return int64_t(B) * chunk_count(T) * int64_t(sizeof(Map) + sizeof(double));
}

// Chunk k of a row (k = 0 is the last chunk in time): steps [t0, t1).
__device__ __forceinline__ void chunk_range(int T, int64_t k, int& t0, int& t1) {
  t1 = T - int(k) * rtg::kSeg;
  t0 = t1 > rtg::kSeg ? t1 - rtg::kSeg : 0;
}

// The staged pass's map over its valid slots (slots before the pass start act as identities).
// Returns the map on every lane.
template <bool kBits>
__device__ __forceinline__ Map compose_pass(const rtg::Pass& p, const rtg::Edges& ed, const float* s_r,
                                            const unsigned char* s_d, double gamma, int lane) {
  const int lo = lane * rtg::kLane;
  unsigned long long dmask;
  if (kBits) {
    const unsigned long long w2 = (unsigned long long)ed.dt << 32 | ed.dh;
    dmask = (w2 >> ((p.tg + lo) & 31)) & ((1ull << rtg::kLane) - 1ull);
  } else {
    dmask = rtg::done_mask(s_d, p.gd + lo);
  }
  const float* rl = s_r + p.gr + lo;
  const int pad = rtg::kSeg - p.len;
  double A = 1.0, Bv = 0.0;
#pragma unroll
  for (int e = rtg::kLane - 1; e >= 0; --e) {
    const bool valid = lo + e >= pad;
    const double a = valid ? (((dmask >> e) & 1ull) ? 0.0 : gamma) : 1.0;
    Bv = fma(a, Bv, valid ? double(rl[e]) : 0.0);
    A *= a;
  }
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const double A2 = __shfl_down_sync(0xffffffffu, A, d);
    const double B2 = __shfl_down_sync(0xffffffffu, Bv, d);
    if (lane + d < 32) {
      Bv = fma(A, B2, Bv);
      A *= A2;
    }
  }
  return Map{__shfl_sync(0xffffffffu, A, 0), __shfl_sync(0xffffffffu, Bv, 0)};
}

// Row r's done flags: bytes from r * T, or words from r * nw.
template <bool kBits>
__device__ __forceinline__ const void* done_row(const void* done, int64_t r, int T) {
  return kBits ? static_cast<const void*>(static_cast<const uint32_t*>(done) + r * int64_t((T + 31) >> 5))
               : static_cast<const void*>(static_cast<const unsigned char*>(done) + r * int64_t(T));
}

// Steps 1 and 3: warp w handles items (row, chunk) = w, w + #warps, ...; kScan = false writes the
// chunk maps to maps[row * nch + k], kScan = true rescans the chunk from carries[row * nch + k].
template <bool kBits, bool kScan>
__global__ void __launch_bounds__(kThreads) chunk_kernel(const float* __restrict__ reward,
                                                         const void* __restrict__ done, float gamma, int64_t B,
                                                         int T, Map* __restrict__ maps,
                                                         const double* __restrict__ carries,
                                                         float* __restrict__ out) {
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint64_t bars[kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned char* wbase = smem + warp * rtg::kWarpSmem;
  float* s_r = reinterpret_cast<float*>(wbase);
  unsigned char* s_d = wbase + rtg::kRewardBytes;
  if (lane == 0) {
    mbar_init(&bars[warp], 1);
    fence_barrier_init();
  }
  __syncwarp();
  const int64_t nch = (int64_t(T) + rtg::kSeg - 1) / rtg::kSeg;
  const int nw = (T + 31) >> 5;
  const double g = double(gamma), g_run = rtg::gamma_run(g);
  uint32_t phase = 0;
  const int64_t items = B * nch;
  for (int64_t it = int64_t(blockIdx.x) * kWarps + warp; it < items; it += int64_t(gridDim.x) * kWarps) {
    const int64_t row = it / nch, k = it - row * nch;
    int t0, t1;
    chunk_range(T, k, t0, t1);
    const rtg::Pass p = rtg::make_pass<kBits>(reward + row * int64_t(T), done_row<kBits>(done, row, T), t0, t1 - t0, nw);
    const rtg::Edges e = rtg::issue_pass<kBits>(p, s_r, s_d, &bars[warp], lane);
    rtg::land_pass<kBits>(p, e, s_r, s_d, &bars[warp], phase & 1u, lane);
    ++phase;
    if (!kScan) {
      const Map m = compose_pass<kBits>(p, e, s_r, s_d, g, lane);
      if (lane == 0) maps[it] = m;
    } else {
      rtg::scan_pass<kBits>(p, e, s_r, s_d, carries[it], g, g_run, gamma, lane);
      rtg::drain_floats(out + row * int64_t(T) + t0, p.len, s_r + (p.sr - p.pr), p.pr, lane);
    }
    __syncwarp();
  }
}

// Step 2, one warp per row.  maps [B, nch] (chunk 0 = last in time).  carries [B, nch] (or null):
// the value entering each chunk from the right, starting from y0 = the composition of the slice
// maps of ranks rank+1 .. world-1 (slices [world, B]) applied to 0, or 0 without slices.  slice_out
// [B] (or null): the map of the row's whole slice.
__global__ void __launch_bounds__(kCarryThreads) carry_kernel(const Map* __restrict__ maps, int64_t B, int64_t nch,
                                                              const Map* __restrict__ slices, int world, int rank,
                                                              double* __restrict__ carries,
                                                              Map* __restrict__ slice_out) {
  pdl_begin();
  __shared__ Map s_warp[kCarryThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = blockIdx.x;
  const Map* m = maps + row * nch;
  const int64_t per = (nch + kCarryThreads - 1) / kCarryThreads;  // chunks per thread block
  const int64_t k0 = threadIdx.x * per < nch ? threadIdx.x * per : nch, k1 = k0 + per < nch ? k0 + per : nch;
  // Block map: M_{k1-1} o ... o M_{k0} (later k applied after earlier k: y moves leftwards).  The
  // maps are loaded kUnroll at a time so their loads are in flight together.
  constexpr int kUnroll = 8;
  double A = 1.0, Bv = 0.0;
  for (int64_t k = k0; k < k1; k += kUnroll) {
    Map q[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) q[u] = k + u < k1 ? m[k + u] : Map{1.0, 0.0};
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      Bv = fma(q[u].a, Bv, q[u].b);
      A *= q[u].a;
    }
  }
  // Inclusive prefix over the CTA's threads: thread t gets G_t o ... o G_0 (a warp scan, then the
  // warp totals' exclusive prefix applied first).
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const double A2 = __shfl_up_sync(0xffffffffu, A, d);
    const double B2 = __shfl_up_sync(0xffffffffu, Bv, d);
    if (lane >= d) {
      Bv = fma(A, B2, Bv);
      A *= A2;
    }
  }
  if (lane == 31) s_warp[warp] = Map{A, Bv};
  __syncthreads();
  double Pa = 1.0, Pb = 0.0;  // W_{warp-1} o ... o W_0
  for (int w = 0; w < warp; ++w) {
    const Map q = s_warp[w];
    Pb = fma(q.a, Pb, q.b);
    Pa *= q.a;
  }
  Bv = fma(A, Pb, Bv);
  A *= Pa;
  if (slice_out != nullptr && threadIdx.x == kCarryThreads - 1) slice_out[row] = Map{A, Bv};
  if (carries == nullptr) return;
  double y0 = 0.0;
  if (slices != nullptr)
    for (int r = world - 1; r > rank; --r) {
      const Map q = slices[int64_t(r) * B + row];
      y0 = fma(q.a, y0, q.b);
    }
  // Exclusive prefix applied to y0: the value entering chunk k0.
  double Ae = __shfl_up_sync(0xffffffffu, A, 1), Be = __shfl_up_sync(0xffffffffu, Bv, 1);
  if (lane == 0) {
    Ae = Pa;
    Be = Pb;
  }
  double y = fma(Ae, y0, Be);
  double* c = carries + row * nch;
  for (int64_t k = k0; k < k1; k += kUnroll) {
    Map q[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) q[u] = k + u < k1 ? m[k + u] : Map{1.0, 0.0};
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (k + u < k1) c[k + u] = y;
      y = fma(q[u].a, y, q[u].b);
    }
  }
}

template <bool kBits>
inline int launch_chunks(bool scan, const float* reward, const void* done, float gamma, int32_t B, int32_t T, Map* maps,
                         const double* carries, float* out, cudaStream_t stream) {
  const int64_t items = int64_t(B) * chunk_count(T);
  const int64_t want = (items + kWarps - 1) / kWarps;
  const int64_t cap = int64_t(sm_count()) * 16;
  const int grid = int(want < cap ? want : cap);
  const int smem = kWarps * rtg::kWarpSmem;
  if (scan) {
    auto kern = chunk_kernel<kBits, true>;
    if (!ensure_dyn_smem(kern, smem)) return kCudaError;
    return launch_pdl(kern, grid, kThreads, smem, stream, reward, done, gamma, int64_t(B), T, maps, carries, out);
  }
  auto kern = chunk_kernel<kBits, false>;
  if (!ensure_dyn_smem(kern, smem)) return kCudaError;
  return launch_pdl(kern, grid, kThreads, smem, stream, reward, done, gamma, int64_t(B), T, maps, carries, out);
}

inline int launch_carries(const Map* maps, int32_t B, int32_t T, const Map* slices, int world, int rank,
                          double* carries, Map* slice_out, cudaStream_t stream) {
  return launch_pdl(carry_kernel, unsigned(B), kCarryThreads, 0, stream, maps, int64_t(B), chunk_count(T), slices,
                    world, rank, carries, slice_out);
}

struct Ws {
  Map* maps;
  double* carries;
};

inline bool split_ws(void* ws, int64_t ws_bytes, int32_t B, int32_t T, Ws* w) {
  if (ws == nullptr || ws_bytes < workspace_bytes(B, T)) return false;
  const int64_t n = int64_t(B) * chunk_count(T);
  w->maps = static_cast<Map*>(ws);
  w->carries = reinterpret_cast<double*>(w->maps + n);
  return true;
}

inline int check_args(const float* reward, const void* done, int32_t B, int32_t T, bool need_out, const float* out) {
  if (B < 0 || T < 0) return kInvalidArgument;
  if (B == 0 || T == 0) return kOk;
  if (reward == nullptr || done == nullptr || (need_out && out == nullptr)) return kInvalidArgument;
  return -1;  // proceed
}

// One GPU: the chunked scan of [B, T] rows.  done: bytes, or with done_bits the rtg::pack_done words.
inline int run(const float* reward, const void* done, bool done_bits, float gamma, int32_t B, int32_t T, float* out,
               void* ws, int64_t ws_bytes, cudaStream_t stream) {
  const int c = check_args(reward, done, B, T, true, out);
  if (c >= 0) return c;
  Ws w;
  if (!split_ws(ws, ws_bytes, B, T, &w)) return kWorkspaceTooSmall;
  int st = done_bits ? launch_chunks<true>(false, reward, done, gamma, B, T, w.maps, nullptr, nullptr, stream)
                     : launch_chunks<false>(false, reward, done, gamma, B, T, w.maps, nullptr, nullptr, stream);
  if (st != kOk) return st;
  st = launch_carries(w.maps, B, T, nullptr, 1, 0, w.carries, nullptr, stream);
  if (st != kOk) return st;
  return done_bits ? launch_chunks<true>(true, reward, done, gamma, B, T, nullptr, w.carries, out, stream)
                   : launch_chunks<false>(true, reward, done, gamma, B, T, nullptr, w.carries, out, stream);
}

// Multi-GPU over time, first half: this rank's slice maps [B] (Map = two doubles: a, then b).
inline int slice_maps(const float* reward, const void* done, bool done_bits, float gamma, int32_t B, int32_t T_loc,
                      Map* slice_out, void* ws, int64_t ws_bytes, cudaStream_t stream) {
  if (B < 0 || T_loc <= 0) return kInvalidArgument;  // every rank holds at least one step
  if (B == 0) return kOk;
  if (reward == nullptr || done == nullptr || slice_out == nullptr) return kInvalidArgument;
  Ws w;
  if (!split_ws(ws, ws_bytes, B, T_loc, &w)) return kWorkspaceTooSmall;
  const int st = done_bits
                     ? launch_chunks<true>(false, reward, done, gamma, B, T_loc, w.maps, nullptr, nullptr, stream)
                     : launch_chunks<false>(false, reward, done, gamma, B, T_loc, w.maps, nullptr, nullptr, stream);
  if (st != kOk) return st;
  return launch_carries(w.maps, B, T_loc, nullptr, 1, 0, nullptr, slice_out, stream);
}

// Second half, after the all-gather of every rank's slice maps into slices [world, B]: this
// rank's outputs.  The workspace must still hold this rank's chunk maps from slice_maps.
inline int slice_scan(const float* reward, const void* done, bool done_bits, float gamma, int32_t B, int32_t T_loc,
                      const Map* slices, int world, int rank, float* out, void* ws, int64_t ws_bytes,
                      cudaStream_t stream) {
  if (B < 0 || T_loc <= 0 || world < 1 || rank < 0 || rank >= world) return kInvalidArgument;
  if (B == 0) return kOk;
  if (reward == nullptr || done == nullptr || slices == nullptr || out == nullptr) return kInvalidArgument;
  Ws w;
  if (!split_ws(ws, ws_bytes, B, T_loc, &w)) return kWorkspaceTooSmall;
  int st = launch_carries(w.maps, B, T_loc, slices, world, rank, w.carries, nullptr, stream);
  if (st != kOk) return st;
  return done_bits ? launch_chunks<true>(true, reward, done, gamma, B, T_loc, nullptr, w.carries, out, stream)
                   : launch_chunks<false>(true, reward, done, gamma, B, T_loc, nullptr, w.carries, out, stream);
}

}  // namespace rtgc
}  // namespace b200
