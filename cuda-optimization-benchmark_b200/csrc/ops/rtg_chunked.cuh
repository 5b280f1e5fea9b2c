// Reward-to-go over long rows: parallel along T within a row, and sharded along T across GPUs.
//
// reward_to_go.cuh gives every row to one warp, so a batch of few, long rows (T >> B: one long
// episode stream, or the reference's B1_T8000 case at larger T) runs on a handful of warps.  Here a
// row is cut into chunks of rtg::kSeg steps, aligned from its end exactly like the passes of the
// one-warp scan, and every chunk gets its own warp.  Three steps:
//   1. each chunk's affine map y_left = B + A * y_right in fp64 (the lane runs and the warp
//      composition of rtg::scan_pass, with the slots before a short chunk's start as identities);
//   2. the value entering every chunk from the right, composed from the chunk maps after it,
//      starting from y0 = 0, or from this rank's carry-in when the row's steps are sharded over
//      ranks;
//   3. each chunk rescanned from its fp64 carry, so every output takes at most kLane fp32
//      roundings, as in the one-warp scan.
// On one GPU the three steps are one cooperative launch (stream_kernel, described before it): the
// chunks are read from HBM once, and their second read (step 3) is served in part from L2.
//
// Multi-GPU over time: rank r holds steps [r * T_loc, (r + 1) * T_loc) of every row.  The steps run
// as separate launches: chunk_kernel (step 1) and the slice map of carry_kernel first
// (slice_maps); the ranks all-gather the [B] slice maps (16 bytes per row per rank); then each
// rank's carry-in is the composition of the slices of the ranks after it applied to 0, and
// carry_kernel and chunk_kernel (step 3) finish its slice (slice_scan), reading each chunk twice
// from HBM.  The outputs equal the one-GPU scan's up to the fp64 association of the carries (the
// oracle's tolerance).
#pragma once

#include "../common/b200_common.cuh"
#include "reward_to_go.cuh"

namespace b200 {
namespace rtgc {

constexpr int kWarps = 4;  // chunks in flight per CTA, one staging buffer each
constexpr int kThreads = 32 * kWarps;
constexpr int kCarryThreads = 256;  // one row per CTA in carry_kernel
constexpr int kBlk = 8;              // chunks per block (one-launch form)
constexpr int kSup = 32;             // blocks per superblock (one-launch form; a lane each)
constexpr int64_t kCtlBytes = 256;   // control words at the workspace start

struct Map {
  double a, b;  // y_left = b + a * y_right
};

inline int64_t chunk_count(int32_t T) { return T <= 0 ? 0 : (int64_t(T) + rtg::kSeg - 1) / rtg::kSeg; }

inline int64_t block_count(int32_t T) { return (chunk_count(T) + kBlk - 1) / kBlk; }

// Workspace: kCtlBytes of control words (the one-launch form's grid-barrier count; zero before the
// first launch on the buffer, then advanced by a whole number of grids by every launch), then the
// chunk maps [B, nch], the block maps [B, nblk], the lane suffix maps [B, nch, 32], the chunk
// carries [B, nch] and the block carries [B, nblk].
inline int64_t workspace_bytes(int32_t B, int32_t T) {
  if (B <= 0 || T <= 0) return 0;
  const int64_t n = int64_t(B) * chunk_count(T), nb = int64_t(B) * block_count(T);
  return kCtlBytes + (n + nb) * int64_t(sizeof(Map) + sizeof(double)) + n * 32 * int64_t(sizeof(Map));
}

// Chunk k of a row (k = 0 is the last chunk in time): steps [t0, t1).
__device__ __forceinline__ void chunk_range(int T, int64_t k, int& t0, int& t1) {
  t1 = T - int(k) * rtg::kSeg;
  t0 = t1 > rtg::kSeg ? t1 - rtg::kSeg : 0;
}

// The staged pass's lane runs composed over its valid slots (slots before the pass start act as
// identities): lane l returns f_l o f_(l+1) o ... o f_31, the map from the value entering the pass
// on the right to the value at lane l's first slot; lane 0's is the chunk map.
template <bool kBits>
__device__ __forceinline__ Map compose_lanes(const rtg::Pass& p, const rtg::Edges& ed, const float* s_r,
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
  return Map{A, Bv};
}

// The staged pass's map over its valid slots, on every lane.
template <bool kBits>
__device__ __forceinline__ Map compose_pass(const rtg::Pass& p, const rtg::Edges& ed, const float* s_r,
                                            const unsigned char* s_d, double gamma, int lane) {
  const Map m = compose_lanes<kBits>(p, ed, s_r, s_d, gamma, lane);
  return Map{__shfl_sync(0xffffffffu, m.a, 0), __shfl_sync(0xffffffffu, m.b, 0)};
}

// Rescan of a staged pass from the value entering it on the right (carry), given each lane's
// suffix map from compose_lanes: the lane's incoming value in fp64, then its run in fp32 (at most
// kLane roundings per output, as rtg::scan_pass), the outputs written over the rewards.
template <bool kBits>
__device__ __forceinline__ void rescan_pass(const rtg::Pass& p, const rtg::Edges& ed, float* s_r,
                                            const unsigned char* s_d, const Map& suffix, double carry,
                                            float gamma_f, int lane) {
  const int lo = lane * rtg::kLane;
  unsigned long long dmask;
  if (kBits) {
    const unsigned long long w2 = (unsigned long long)ed.dt << 32 | ed.dh;
    dmask = (w2 >> ((p.tg + lo) & 31)) & ((1ull << rtg::kLane) - 1ull);
  } else {
    dmask = rtg::done_mask(s_d, p.gd + lo);
  }
  const double start = fma(suffix.a, carry, suffix.b);   // value at this lane's first slot
  double yin = __shfl_down_sync(0xffffffffu, start, 1);  // value entering this lane's run
  if (lane == 31) yin = carry;
  float* rl = s_r + p.gr + lo;
  float y = float(yin);
#pragma unroll
  for (int e = rtg::kLane - 1; e >= 0; --e) {
    const float rv = rl[e];
    y = ((dmask >> e) & 1ull) ? rv : __fmaf_rn(gamma_f, y, rv);
    rl[e] = y;
  }
  __syncwarp();
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

// ---------------------------------------------------------------------------------------------
// One-launch form of steps 1-3 on one GPU.  The three launches above move the rewards and done
// flags through HBM twice and put the carries of a row on one CTA between two grid-wide kernel
// boundaries.  Here one cooperative launch of one CTA per SM does all of it:
//   A. the CTA owns a contiguous range of whole blocks (kBlk consecutive chunks of a row) and
//      streams its chunks (two staging buffers per warp: the next chunk lands while the current
//      one is composed), writing every chunk's map and every lane's suffix map (the composition
//      of its run and the runs after it in the chunk), then every block's map;
//   -- grid barrier --
//   B. the CTA derives the value entering each of its blocks (the warps scan the superblocks it
//      needs in parallel, one thread per row folds the superblock maps), each thread the values
//      entering the chunks of one block, and the warps stream the range again from its last chunk
//      (the chunks read last in A are the likeliest to be in L2 still; each warp's first one is
//      read before the barrier): a lane's incoming value is its suffix map applied to the chunk's
//      carry, and only the fp32 rescan of its run remains.
// The association of the carries depends on (B, T) only, not on the grid: the value entering
// chunk k of a row is the composition, applied to 0, of the superblock maps before k's superblock
// (kSup blocks each), then the exclusive prefix of k's block within its superblock (both from one
// fixed 32-lane scan of the superblock's block maps), then the chunk maps before k within its
// block.
// Traffic: 9 bytes per step from HBM plus the second read of the rewards and flags, which L2
// serves in part, and 528 bytes of maps per 1056-step chunk.
// ---------------------------------------------------------------------------------------------
constexpr int kStreamWarps = 16;
constexpr int kStreamThreads = 32 * kStreamWarps;
constexpr int kStreamSmem = kStreamWarps * 2 * rtg::kWarpSmem;  // 171,520 B: one CTA per SM
constexpr int kSupWin = 256;             // superblock maps staged in shared memory (the fast carry path)
constexpr int kBlkWin = kStreamThreads;  // own blocks staged in shared memory (the fast carry path)
constexpr int kItemWin = 1024;           // own chunk maps kept in shared memory (when they fit)

struct GridBar {
  unsigned long long count;  // CTA arrivals at grid barriers over all launches on the workspace
};

// acc := m o acc (acc applied first).
__device__ __forceinline__ void fold(Map& acc, const Map& m) {
  acc.b = fma(m.a, acc.b, m.b);
  acc.a *= m.a;
}

// A map written by another CTA (or another warp) of this grid, read through L2.
__device__ __forceinline__ Map ld_map(const Map* p) { return Map{ld_cg_f64(&p->a), ld_cg_f64(&p->b)}; }

// Grid-wide barrier of a cooperative launch whose grid size is the same in every launch on the
// workspace: each CTA adds 1 to a 64-bit count that is never reset (zero before the first launch,
// so a multiple of the grid size whenever a launch starts), and the barrier completes when the
// count reaches the next multiple.  The CTA barrier orders the CTA's writes before thread 0's
// release-acquire add; thread 0's acquire orders the reads after the next CTA barrier.  A CTA that
// waits longer than kWaitLimitNs records kFaultWaitTimeout and goes on.
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void grid_sync(GridBar* gb) {
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long old;
    asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], 1;" : "=l"(old) : "l"(&gb->count) : "memory");
    const unsigned long long target = (old / gridDim.x + 1) * gridDim.x;
    if (old + 1 != target) {
      const unsigned long long t0 = global_ns();
      for (uint32_t i = 1; ld_acquire_u64(&gb->count) < target; ++i) {
        if ((i & 255u) == 0 && global_ns() - t0 > kWaitLimitNs) {
          atomicOr(&g_b200_fault, kFaultWaitTimeout);
          break;
        }
      }
    }
  }
  __syncthreads();
}

// Chunk `it` (flat index row * nch + k) as a staged pass.
template <bool kBits>
__device__ __forceinline__ rtg::Pass chunk_pass(const float* reward, const void* done, int T, int64_t nch, int64_t it) {
  const int64_t row = it / nch, k = it - row * nch;
  int t0, t1;
  chunk_range(T, k, t0, t1);
  return rtg::make_pass<kBits>(reward + row * int64_t(T), done_row<kBits>(done, row, T), t0, t1 - t0,
                               (T + 31) >> 5);
}

// The chunks of [i0, i1) that belong to warp w: i0 + w, i0 + w + W, ... in step A (chunk maps to
// maps and, when s_cm is not null, to s_cm[it - i0]; lane suffix maps to lanes), i1 - 1 - w,
// i1 - 1 - w - W, ... in step B (rescans from carries[item] and the lane suffix maps).  Two staging
// buffers with one mbarrier each; phbits holds their parities and is returned updated.  With
// `pre`, the warp's first chunk was already issued into buffer 0 (its edges in e0).
template <bool kBits, bool kScan>
__device__ __forceinline__ uint32_t walk(const float* __restrict__ reward, const void* __restrict__ done, float gamma,
                                         int T, int64_t nch, int64_t i0, int64_t i1, Map* __restrict__ maps,
                                         Map* s_cm, Map* __restrict__ lanes, const double* __restrict__ carries,
                                         float* __restrict__ out, unsigned char* wbase, uint64_t* bars,
                                         uint32_t phbits, bool pre, const rtg::Edges& e0, int w, int lane) {
  const int64_t n = i1 - i0;
  if (n <= w) return phbits;
  const int64_t cnt = (n - w + kStreamWarps - 1) / kStreamWarps;
  auto item = [&](int64_t q) { return kScan ? i1 - 1 - (w + q * kStreamWarps) : i0 + w + q * kStreamWarps; };
  auto s_r = [&](uint32_t b) { return reinterpret_cast<float*>(wbase + b * rtg::kWarpSmem); };
  auto s_d = [&](uint32_t b) { return wbase + b * rtg::kWarpSmem + rtg::kRewardBytes; };
  auto pass_of = [&](int64_t it) { return chunk_pass<kBits>(reward, done, T, nch, it); };
  const double g = double(gamma);
  int64_t it = item(0);
  rtg::Pass cur = pass_of(it);
  rtg::Edges ecur = pre ? e0 : rtg::issue_pass<kBits>(cur, s_r(0), s_d(0), &bars[0], lane);
  for (int64_t q = 0; q < cnt; ++q) {
    const uint32_t cb = uint32_t(q) & 1u, nb = cb ^ 1u;
    int64_t itn = it;
    rtg::Pass nxt = cur;
    rtg::Edges enxt = ecur;
    if (q + 1 < cnt) {
      itn = item(q + 1);
      nxt = pass_of(itn);
      if (kScan) rtg::outputs_read(lane);  // buffer nb holds the previous chunk: its outputs are read
      enxt = rtg::issue_pass<kBits>(nxt, s_r(nb), s_d(nb), &bars[nb], lane);
    }
    double carry = 0.0;
    Map suffix{1.0, 0.0};
    if (kScan) {
      carry = ld_cg_f64(carries + it);
      suffix = ld_map(lanes + it * 32 + lane);
    }
    rtg::land_pass<kBits>(cur, ecur, s_r(cb), s_d(cb), &bars[cb], (phbits >> cb) & 1u, lane);
    phbits ^= 1u << cb;
    if (!kScan) {
      const Map m = compose_lanes<kBits>(cur, ecur, s_r(cb), s_d(cb), g, lane);
      lanes[it * 32 + lane] = m;
      if (lane == 0) {
        maps[it] = m;
        if (s_cm != nullptr) s_cm[it - i0] = m;
      }
    } else {
      rescan_pass<kBits>(cur, ecur, s_r(cb), s_d(cb), suffix, carry, gamma, lane);
      rtg::store_pass(cur, s_r(cb), out + (cur.rs - reward), lane);
    }
    __syncwarp();
    cur = nxt;
    ecur = enxt;
    it = itn;
  }
  if (kScan) rtg::outputs_done(lane);  // the outputs are written before the CTA ends
  return phbits;
}

// Inclusive scan of the 32 lanes' maps (lane l: block l of a superblock, identities past the
// row's end) by doubling: lane l returns block l's map o ... o block 0's, with the same bits in
// every CTA that scans the same superblock; lane 31's is the superblock map.
__device__ __forceinline__ Map scan32(Map m, int lane) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const double a2 = __shfl_up_sync(0xffffffffu, m.a, d), b2 = __shfl_up_sync(0xffffffffu, m.b, d);
    if (lane >= d) {
      m.b = fma(m.a, b2, m.b);
      m.a *= a2;
    }
  }
  return m;
}

// Exclusive form on every lane: the map entering block l of the superblock from its start.
__device__ __forceinline__ Map exclusive32(const Map& incl, int lane) {
  Map e{__shfl_up_sync(0xffffffffu, incl.a, 1), __shfl_up_sync(0xffffffffu, incl.b, 1)};
  if (lane == 0) e = Map{1.0, 0.0};
  return e;
}

// The (row, superblock) pairs a CTA with blocks [b0, b1) needs, in order: for each row it touches,
// superblocks 0 .. (its last block there) / kSup.
struct Pairs {
  int64_t nblk, r0, r1;  // rows r0 .. r1 - 1
  int64_t c0, cm, c1;    // pairs of the first row, of each middle row, of the last row
  int64_t n;             // all pairs
  __device__ __forceinline__ Pairs(int64_t nblk_, int64_t b0, int64_t b1) : nblk(nblk_) {
    r0 = b0 / nblk;
    r1 = (b1 - 1) / nblk + 1;
    const int64_t jl = b1 - 1 - (r1 - 1) * nblk;  // last block, in the last row
    cm = (nblk - 1) / kSup + 1;
    c1 = jl / kSup + 1;
    c0 = r1 - r0 == 1 ? c1 : cm;
    n = r1 - r0 == 1 ? c0 : c0 + (r1 - r0 - 2) * cm + c1;
  }
  // Pair p -> row and superblock.
  __device__ __forceinline__ void at(int64_t p, int64_t& r, int64_t& s) const {
    if (p < c0) {
      r = r0;
      s = p;
      return;
    }
    const int64_t q = p - c0;
    r = r0 + 1 + q / cm;
    s = q - (q / cm) * cm;
  }
  // First pair of row r.
  __device__ __forceinline__ int64_t first(int64_t r) const { return r == r0 ? 0 : c0 + (r - r0 - 1) * cm; }
};

// The value entering each block of [b0, b1), by the whole CTA: the warps scan the superblocks the
// CTA needs (s_sup <- superblock maps; s_exc <- the exclusive maps of the CTA's own blocks), one
// thread per row folds the superblock maps in order (s_z <- the value entering each superblock),
// then the value entering own block b is s_exc[b - b0] applied to its superblock's s_z.  Needs
// Pairs::n <= kSupWin and b1 - b0 <= kBlkWin; block_carries_global is the same arithmetic
// otherwise.
__device__ __forceinline__ void block_carries_smem(const Map* blk, const Pairs& pr, int64_t b0, int64_t b1,
                                                   Map* s_sup, Map* s_exc, double* s_z, int warp, int lane) {
  const int64_t nblk = pr.nblk;
  for (int64_t p = warp; p < pr.n; p += 4 * kStreamWarps) {
    Map m[4];
    int64_t jb[4], rb[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t pu = p + u * kStreamWarps;
      m[u] = Map{1.0, 0.0};
      jb[u] = -1;
      rb[u] = 0;
      if (pu < pr.n) {
        int64_t s;
        pr.at(pu, rb[u], s);
        jb[u] = s * kSup + lane;
        if (jb[u] < nblk) m[u] = ld_map(blk + rb[u] * nblk + jb[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t pu = p + u * kStreamWarps;
      if (pu < pr.n) {
        const Map inc = scan32(m[u], lane);
        const Map exc = exclusive32(inc, lane);
        if (lane == 31) s_sup[pu] = inc;
        const int64_t b = rb[u] * nblk + jb[u];
        if (jb[u] < nblk && b >= b0 && b < b1) s_exc[b - b0] = exc;
      }
    }
  }
  __syncthreads();
  for (int64_t r = pr.r0 + threadIdx.x; r < pr.r1; r += blockDim.x) {
    const int64_t p0 = pr.first(r), p1 = r + 1 < pr.r1 ? pr.first(r + 1) : pr.n;
    double z = 0.0;
    for (int64_t p = p0; p < p1; ++p) {
      s_z[p] = z;
      z = fma(s_sup[p].a, z, s_sup[p].b);
    }
  }
  __syncthreads();
}

// The same values by one warp through global memory -> yblk[b] (a superblock scan per load round
// trip): the general path.
__device__ __forceinline__ void block_carries_global(const Map* blk, double* yblk, const Pairs& pr, int64_t b0,
                                                     int64_t b1, int lane) {
  const int64_t nblk = pr.nblk;
  for (int64_t r = pr.r0; r < pr.r1; ++r) {
    const int64_t p0 = pr.first(r), p1 = r + 1 < pr.r1 ? pr.first(r + 1) : pr.n;
    double z = 0.0;
    for (int64_t s = 0; s < p1 - p0; ++s) {
      const int64_t j = s * kSup + lane, b = r * nblk + j;
      const Map inc = scan32(j < nblk ? ld_map(blk + b) : Map{1.0, 0.0}, lane);
      const Map exc = exclusive32(inc, lane);
      if (j < nblk && b >= b0 && b < b1) yblk[b] = fma(exc.a, z, exc.b);
      z = fma(__shfl_sync(0xffffffffu, inc.a, 31), z, __shfl_sync(0xffffffffu, inc.b, 31));
    }
  }
}

// Chunk maps [k0, k0 + kn) of a row into q (the rest identities): from shared memory (s_cm, the
// chunks from i0 on) when this CTA kept them there, else through L2.
__device__ __forceinline__ void load_block(const Map* maps, const Map* s_cm, int64_t i0, int64_t rk0, int kn,
                                           Map (&q)[kBlk]) {
#pragma unroll
  for (int u = 0; u < kBlk; ++u)
    q[u] = u >= kn ? Map{1.0, 0.0} : s_cm != nullptr ? s_cm[rk0 - i0 + u] : ld_map(maps + rk0 + u);
}

template <bool kBits>
__global__ void __launch_bounds__(kStreamThreads, 1) stream_kernel(const float* __restrict__ reward,
                                                                   const void* __restrict__ done, float gamma,
                                                                   int64_t B, int T, Map* __restrict__ maps,
                                                                   Map* __restrict__ blk, Map* __restrict__ lanes,
                                                                   double* __restrict__ carries,
                                                                   double* __restrict__ yblk, GridBar* gb,
                                                                   float* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint64_t s_bars[kStreamWarps][2];
  __shared__ Map s_sup[kSupWin];
  __shared__ Map s_exc[kBlkWin];
  __shared__ double s_z[kSupWin];
  __shared__ Map s_cmap[kItemWin];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    mbar_init(&s_bars[warp][0], 1);
    mbar_init(&s_bars[warp][1], 1);
    fence_barrier_init();
  }
  __syncwarp();
  const int64_t nch = (int64_t(T) + rtg::kSeg - 1) / rtg::kSeg, nblk = (nch + kBlk - 1) / kBlk, nb = B * nblk;
  const int64_t b0 = nb * blockIdx.x / gridDim.x, b1 = nb * (blockIdx.x + 1) / gridDim.x;
  auto first_item = [&](int64_t b) {
    const int64_t r = b / nblk;
    return r * nch + (b - r * nblk) * kBlk;
  };
  const int64_t i0 = first_item(b0), i1 = first_item(b1);
  Map* s_cm = i1 - i0 <= kItemWin ? s_cmap : nullptr;
  unsigned char* wbase = smem + warp * 2 * rtg::kWarpSmem;
  // A: chunk and lane maps, then block maps (a thread per block; its first block's chunk maps stay
  // in registers for the chunk carries).
  const rtg::Edges e_none{0.f, 0.f, 0u, 0u};
  uint32_t ph = walk<kBits, false>(reward, done, gamma, T, nch, i0, i1, maps, s_cm, lanes, nullptr, nullptr, wbase,
                                   s_bars[warp], 0u, false, e_none, warp, lane);
  __syncthreads();
  auto block_of = [&](int64_t b, int64_t& r, int64_t& k0, int& kn) {
    r = b / nblk;
    k0 = (b - r * nblk) * kBlk;
    kn = int(nch - k0 < kBlk ? nch - k0 : kBlk);
  };
  const int64_t bt = b0 + threadIdx.x;
  Map q[kBlk];
  for (int64_t b = bt; b < b1; b += blockDim.x) {
    int64_t r, k0;
    int kn;
    block_of(b, r, k0, kn);
    load_block(maps, s_cm, i0, r * nch + k0, kn, q);
    Map acc{1.0, 0.0};
#pragma unroll
    for (int u = 0; u < kBlk; ++u)
      if (u < kn) fold(acc, q[u]);
    blk[b] = acc;
  }
  if (bt < b1 && bt + blockDim.x < b1) {  // several blocks per thread: back to the first one's maps
    int64_t r, k0;
    int kn;
    block_of(bt, r, k0, kn);
    load_block(maps, s_cm, i0, r * nch + k0, kn, q);
  }
  // The warp's first chunk of step B is read before the barrier: it needs no carry until it lands.
  const bool pre = i1 - i0 > warp;
  rtg::Edges e0 = e_none;
  if (pre) e0 = rtg::issue_pass<kBits>(chunk_pass<kBits>(reward, done, T, nch, i1 - 1 - warp),
                                       reinterpret_cast<float*>(wbase), wbase + rtg::kRewardBytes, &s_bars[warp][0],
                                       lane);
  grid_sync(gb);
  // B: block carries, chunk carries, rescans.
  const bool any = b1 > b0;
  const Pairs pr(nblk, any ? b0 : 0, any ? b1 : 1);
  const bool smem_path = any && pr.n <= kSupWin && b1 - b0 <= kBlkWin;
  if (smem_path) {
    block_carries_smem(blk, pr, b0, b1, s_sup, s_exc, s_z, warp, lane);
  } else if (any) {
    if (warp == 0) block_carries_global(blk, yblk, pr, b0, b1, lane);
    __syncthreads();
  }
  for (int64_t b = bt; b < b1; b += blockDim.x) {
    int64_t r, k0;
    int kn;
    block_of(b, r, k0, kn);
    if (b != bt) load_block(maps, s_cm, i0, r * nch + k0, kn, q);
    double y;
    if (smem_path) {
      const Map e = s_exc[b - b0];
      y = fma(e.a, s_z[pr.first(r) + (b - r * nblk) / kSup], e.b);
    } else {
      y = ld_cg_f64(yblk + b);
    }
    double* c = carries + r * nch + k0;
#pragma unroll
    for (int u = 0; u < kBlk; ++u)
      if (u < kn) {
        c[u] = y;
        y = fma(q[u].a, y, q[u].b);
      }
  }
  __syncthreads();
  walk<kBits, true>(reward, done, gamma, T, nch, i0, i1, nullptr, nullptr, lanes, carries, out, wbase, s_bars[warp], ph,
                    pre, e0, warp, lane);
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
  GridBar* ctl;
  Map* maps;
  Map* blk;
  Map* lanes;
  double* carries;
  double* yblk;
};

inline bool split_ws(void* ws, int64_t ws_bytes, int32_t B, int32_t T, Ws* w) {
  if (ws == nullptr || ws_bytes < workspace_bytes(B, T)) return false;
  const int64_t n = int64_t(B) * chunk_count(T), nb = int64_t(B) * block_count(T);
  w->ctl = static_cast<GridBar*>(ws);
  w->maps = reinterpret_cast<Map*>(static_cast<char*>(ws) + kCtlBytes);
  w->blk = w->maps + n;
  w->lanes = w->blk + nb;
  w->carries = reinterpret_cast<double*>(w->lanes + n * 32);
  w->yblk = w->carries + n;
  return true;
}

// The one-launch form: a cooperative launch (every CTA resident, as the grid barrier needs) of one
// CTA per SM, whatever the size (the barrier's count needs the same grid in every launch; CTAs
// without blocks only take part in the barrier).
template <bool kBits>
inline int launch_stream(const float* reward, const void* done, float gamma, int32_t B, int32_t T, const Ws& w,
                         float* out, cudaStream_t stream) {
  auto kern = stream_kernel<kBits>;
  if (!ensure_dyn_smem(kern, kStreamSmem)) return kCudaError;
  const int64_t grid = int64_t(sm_count()) * resident_ctas_per_sm(kern, kStreamThreads, kStreamSmem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kStreamThreads);
  cfg.dynamicSmemBytes = kStreamSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, reward, done, gamma, int64_t(B), T, w.maps, w.blk, w.lanes, w.carries, w.yblk,
                            w.ctl, out) == cudaSuccess
             ? kOk
             : kCudaError;
}

inline int check_args(const float* reward, const void* done, int32_t B, int32_t T, bool need_out, const float* out) {
  if (B < 0 || T < 0) return kInvalidArgument;
  if (B == 0 || T == 0) return kOk;
  if (reward == nullptr || done == nullptr || (need_out && out == nullptr)) return kInvalidArgument;
  return -1;  // proceed
}

// One GPU: the chunked scan of [B, T] rows in one launch.  done: bytes, or with done_bits the
// rtg::pack_done words.  ws: 8-byte aligned; its control words zero before the first call.
inline int run(const float* reward, const void* done, bool done_bits, float gamma, int32_t B, int32_t T, float* out,
               void* ws, int64_t ws_bytes, cudaStream_t stream) {
  const int c = check_args(reward, done, B, T, true, out);
  if (c >= 0) return c;
  Ws w;
  if (!split_ws(ws, ws_bytes, B, T, &w)) return kWorkspaceTooSmall;
  if (reinterpret_cast<uintptr_t>(ws) % 8 != 0) return kInvalidArgument;
  return done_bits ? launch_stream<true>(reward, done, gamma, B, T, w, out, stream)
                   : launch_stream<false>(reward, done, gamma, B, T, w, out, stream);
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
