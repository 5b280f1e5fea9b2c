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
// at a time and walks it from the end in passes of at most kSeg = 32 * kLane elements:
//   1. lane 0 moves the 16-byte aligned interior of the pass's rewards and done bytes into
//      shared memory with one cp.async.bulk each (counted on the warp's mbarrier, waited on with a
//      sleeping try_wait so a waiting warp takes no issue slots); the lanes load the ragged ends;
//   2. the pass is laid out right-aligned on a grid of 32 runs of kLane slots: lane l owns slots
//      [l*kLane, (l+1)*kLane), and a pass shorter than kSeg leaves its unused slots at the front.
//      Values flow only from later to earlier steps, so those slots (whatever they hold) reach no
//      valid output, and every lane runs exactly kLane steps with no per-step bounds checks;
//   3. lane l composes its run in fp64 (kLane is odd, so the 32 lanes' strided shared reads fall
//      in 32 distinct banks); A is gamma^kLane, or 0 when the run holds a done flag;
//   4. a 5-step warp suffix scan of the lanes' (A, B) maps, in fp64, gives every lane the exact
//      value entering its run;
//   5. lane l re-runs its steps from that value in fp32 (at most kLane roundings per output, no
//      error carried between runs) and writes the outputs over the rewards in shared memory,
//      and lane 0 writes them out with one bulk copy (store_pass).
// One warp per row and 40 warps per SM put every row of the BASELINE batch in flight at once.
//
// Done flags come as one byte per step (the reference layout) or, with kBits, as bits: uint32 words
// [B, ceil(T / 32)], bit t % 32 of word [b, t / 32] set when done[b, t] (pack_kernel makes them).
// Bits cut the flags' traffic from 1 byte to 1/8 byte per step and need no staging: kSeg is a
// multiple of 32, so a lane's kLane-step run spans at most two words of its row, which the lane
// loads when the pass is issued and funnels into its run mask.
#pragma once

#include "../common/b200_common.cuh"
#include "../common/bulk.cuh"

namespace b200 {
namespace rtg {

constexpr int kLane = 33;                    // steps per lane per pass (odd: conflict-free banks)
constexpr int kSeg = 32 * kLane;             // steps per warp pass
constexpr int kWarps = 4;                    // warps (rows in flight) per CTA
constexpr int kThreads = 32 * kWarps;
// Per-warp staging buffer: the lane grid of kSeg floats starts at float 0..3 (so the copy keeps the
// rows' 16-byte phase), the done grid at byte 0..15, and done_mask reads up to 40 bytes past the
// start of a lane's 33-byte window.
constexpr int kRewardBytes = (kSeg + 4) * 4;
constexpr int kDoneBytes = ((kSeg + 16 + 40) + 15) / 16 * 16;
constexpr int kWarpSmem = kRewardBytes + kDoneBytes;
constexpr int kSmemPerBuffer = kWarps * kWarpSmem;  // one staging buffer per warp
static_assert(kRewardBytes % 16 == 0 && kWarpSmem % 16 == 0, "staging buffers stay 16-byte aligned");

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

// Bit e (e < kLane) set when byte sd[at + e] is non-zero.  Reads the ten aligned 32-bit words that
// cover [at, at + 40) and folds each word's four "byte is non-zero" bits into a nibble: 0x80 marks
// every non-zero byte, and one multiply gathers the four marks into the top nibble.
__device__ __forceinline__ unsigned long long done_mask(const unsigned char* sd, int at) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(sd) + (at >> 2);
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const uint32_t v = w[i];
    const uint32_t marks = (((v & 0x7f7f7f7fu) + 0x7f7f7f7fu) | v) & 0x80808080u;  // bit 7 of each byte
    const uint32_t nib = (marks * 0x00204081u) >> 28;                              // bytes 0..3 -> bits 0..3
    if (i < 8) lo |= nib << (4 * i);
    else hi |= nib << (4 * (i - 8));
  }
  const unsigned long long m = ((unsigned long long)hi << 32 | lo) >> (at & 3);
  return m & ((1ull << kLane) - 1ull);
}

// Ragged-edge values a lane loaded for a prefetched pass; written to shared memory when the
// pass's bulk copy has landed, so issuing a pass never waits on its own plain loads.  With done
// bits, dh and dt are instead the two words that cover the lane's run.
struct Edges {
  float rh, rt;
  uint32_t dh, dt;
};

// Geometry of the pass [t0, t0 + len) of one row (1 <= len <= kSeg).  Element i sits at float
// sr + i of the reward buffer and byte sd + i of the done buffer; the lane grid starts gr floats
// and gd bytes into them (sr = gr + kSeg - len).  gr and gd are chosen so that the aligned
// interiors [ear, ebr) and [ead, ebd) land on 16-byte boundaries, as cp.async.bulk requires.
// With done bits: dw is the row's first word, nw its word count, and slot 0 of the lane grid is
// step tg = t0 - (kSeg - len) of the row (negative in the row's first pass: those slots reach no
// output).
struct Pass {
  const float* rs;
  const unsigned char* ds;
  const uint32_t* dw;
  int len, pr, gr, gd, sr, sd, ear, ebr, ead, ebd, tg, nw;
};

template <bool kBits>
__device__ __forceinline__ Pass make_pass(const float* rrow, const void* drow, int t0, int len, int nw) {
  Pass p;
  p.rs = rrow + t0;
  p.ds = kBits ? nullptr : static_cast<const unsigned char*>(drow) + t0;
  p.dw = kBits ? static_cast<const uint32_t*>(drow) : nullptr;
  p.len = len;
  const int pad = kSeg - len;
  p.tg = t0 - pad;
  p.nw = nw;
  p.pr = int((reinterpret_cast<uintptr_t>(p.rs) >> 2) & 3);
  const int pd = int(reinterpret_cast<uintptr_t>(p.ds) & 15);
  p.gr = (p.pr - pad) & 3;
  p.gd = (pd - pad) & 15;
  p.sr = p.gr + pad;
  p.sd = p.gd + pad;
  p.ear = (4 - p.pr) & 3;
  p.ebr = len > p.ear ? p.ear + ((len - p.ear) & ~3) : p.ear;
  p.ead = (16 - pd) & 15;
  p.ebd = len > p.ead ? p.ead + ((len - p.ead) & ~15) : p.ead;
  if (kBits) {  // no done bytes to stage
    p.ead = 0;
    p.ebd = 0;
  }
  return p;
}

__device__ __forceinline__ unsigned char ld_u8(const unsigned char* p) {
  unsigned short v;
  asm volatile("ld.global.nc.L1::no_allocate.u8 %0, [%1];" : "=h"(v) : "l"(p));
  return (unsigned char)v;
}

__device__ __forceinline__ uint32_t ld_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Start moving a pass into a staging buffer: lane 0 arms the buffer's barrier and issues one bulk
// copy per stream for the aligned interiors; every lane issues its ragged-edge loads (and, with
// done bits, the two words covering its run: words before the row's start read as 0).
template <bool kBits>
__device__ __forceinline__ Edges issue_pass(const Pass& p, float* s_r, unsigned char* s_d, uint64_t* bar, int lane) {
  fence_proxy_async_smem();  // earlier ordinary accesses of this buffer come before the copy
  __syncwarp();
  const uint32_t rb = uint32_t(p.ebr - p.ear) * 4u * (p.len > p.ear);
  const uint32_t db = uint32_t(p.ebd - p.ead) * (p.len > p.ead);
  if (lane == 0) {
    mbar_arrive_expect_tx(bar, rb + db);
    if (rb) bulk_g2s(s_r + p.sr + p.ear, p.rs + p.ear, rb, bar);
    if (db) bulk_g2s(s_d + p.sd + p.ead, p.ds + p.ead, db, bar);
  }
  Edges e{0.f, 0.f, 0u, 0u};
  const int hr = min(p.len, p.ear), tr = p.len - p.ebr;
  const int hd = min(p.len, p.ead), td = p.len - p.ebd;
  if (lane < hr) e.rh = ld_stream_f1(p.rs + lane);
  if (lane < tr) e.rt = ld_stream_f1(p.rs + p.ebr + lane);
  if (kBits) {
    const int w = (p.tg + lane * kLane) >> 5;  // arithmetic shift: floor for negative steps
    if (w >= 0 && w < p.nw) e.dh = ld_u32(p.dw + w);
    if (w + 1 >= 0 && w + 1 < p.nw) e.dt = ld_u32(p.dw + w + 1);
  } else {
    if (lane < hd) e.dh = ld_u8(p.ds + lane);
    if (lane < td) e.dt = ld_u8(p.ds + p.ebd + lane);
  }
  return e;
}

// Finish staging a pass: write the ragged edges, wait for the bulk copies (phase `parity`).
template <bool kBits>
__device__ __forceinline__ void land_pass(const Pass& p, const Edges& e, float* s_r, unsigned char* s_d,
                                          uint64_t* bar, uint32_t parity, int lane) {
  const int hr = min(p.len, p.ear), tr = p.len - p.ebr;
  if (lane < hr) s_r[p.sr + lane] = e.rh;
  if (lane < tr) s_r[p.sr + p.ebr + lane] = e.rt;
  if (!kBits) {
    const int hd = min(p.len, p.ead), td = p.len - p.ebd;
    if (lane < hd) s_d[p.sd + lane] = (unsigned char)e.dh;
    if (lane < td) s_d[p.sd + p.ebd + lane] = (unsigned char)e.dt;
  }
  mbar_wait_sleep(bar, parity);
  __syncwarp();
}

// A rescanned pass's outputs (staged over its rewards in shared memory) to dst, the pass's first
// output.  When dst has the rewards' 16-byte phase, lane 0 writes the aligned interior with one
// bulk copy and the lanes store the ragged ends; otherwise drain_floats.  The bulk copy may still
// be reading the buffer when this returns: outputs_read before the buffer is refilled,
// outputs_done before the warp is finished with its buffers.  One bulk copy per pass instead of
// 128-bit stores from every lane: reward-to-go B4096 T1000 7.7 -> 7.3 us, the fused RL step
// 17.1 -> 16.9 us.
__device__ __forceinline__ void store_pass(const Pass& p, const float* s_r, float* dst, int lane) {
  const float* src = s_r + p.sr;
  const int dphase = int((reinterpret_cast<uintptr_t>(dst) >> 2) & 3);
  if (dphase != p.pr || p.ebr <= p.ear) {
    drain_floats(dst, p.len, s_r + (p.sr - p.pr), p.pr, lane);
    return;
  }
  fence_proxy_async_smem();  // the rescan's shared-memory writes come before the copy's reads
  __syncwarp();
  if (lane == 0) {
    bulk_s2g(dst + p.ear, src + p.ear, uint32_t(p.ebr - p.ear) * 4u);
    bulk_commit();
  }
  const int hr = min(p.len, p.ear), tr = p.len - p.ebr;
  if (lane < hr) dst[lane] = src[lane];
  if (lane < tr) dst[p.ebr + lane] = src[p.ebr + lane];
}
__device__ __forceinline__ void outputs_read(int lane) {
  if (lane == 0) bulk_wait_read<0>();
  __syncwarp();
}
__device__ __forceinline__ void outputs_done(int lane) {
  if (lane == 0) bulk_wait_all();
  __syncwarp();
}

// gamma^kLane in fp64 (the composed factor of a run of kLane steps without a done flag).
__device__ __forceinline__ double gamma_run(double gamma) {
  double a = 1.0, q = gamma;
#pragma unroll
  for (int b = 0; b < 6; ++b) {
    if ((kLane >> b) & 1) a *= q;
    q *= q;
  }
  return a;
}

// Scan one staged pass given the value entering it from the right (`carry`); writes the outputs
// into the staging buffer and returns the value at the pass's first step (meaningful only for a
// full pass, len == kSeg: a shorter pass is the first of its row, whose value is not needed).
// gamma is the fp32 discount widened to fp64; g_run = gamma_run(gamma).  e: the lane's edges (its
// run's done words with kBits).
template <bool kBits>
__device__ __forceinline__ double scan_pass(const Pass& p, const Edges& ed, float* s_r, const unsigned char* s_d,
                                            double carry, double gamma, double g_run, float gamma_f, int lane) {
  const int lo = lane * kLane;
  unsigned long long dmask;  // bit e: done at slot lo + e
  if (kBits) {
    const unsigned long long w2 = (unsigned long long)ed.dt << 32 | ed.dh;
    dmask = (w2 >> ((p.tg + lo) & 31)) & ((1ull << kLane) - 1ull);
  } else {
    dmask = done_mask(s_d, p.gd + lo);
  }
  float* rl = s_r + p.gr + lo;
  // Composition of the run in fp64: y -> Bv + A*y (the factor of slot e is 0 at a done flag, else
  // gamma; Bv stays finite, so 0 * Bv is an exact zero).
  double Bv = 0.0;
#pragma unroll
  for (int e = kLane - 1; e >= 0; --e) {
    const double a = ((dmask >> e) & 1ull) ? 0.0 : gamma;
    Bv = fma(a, Bv, double(rl[e]));
  }
  double A = dmask == 0 ? g_run : 0.0;
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
  const double start = fma(A, carry, Bv);                // value at this lane's first slot
  double yin = __shfl_down_sync(0xffffffffu, start, 1);  // value entering this lane's run
  if (lane == 31) yin = carry;
  const double first = __shfl_sync(0xffffffffu, start, 0);
  // Second pass from the exact incoming value, in fp32: at most kLane roundings per output.
  float y = float(yin);
#pragma unroll
  for (int e = kLane - 1; e >= 0; --e) {
    const float rv = rl[e];
    y = ((dmask >> e) & 1ull) ? rv : __fmaf_rn(gamma_f, y, rv);
    rl[e] = y;
  }
  __syncwarp();
  return first;
}

// One warp streams rows first_row, first_row + row_stride, ... pass by pass, from the end of a row
// to its start.  wbase: the warp's staging memory (nbuf buffers of kWarpSmem bytes); bars: its two
// mbarriers (initialised here).  With nbuf = 2 the next pass is in flight in the second buffer
// while the current one is scanned and written out; with nbuf = 1 passes are staged one after the
// other (a smaller footprint, so more warps share an SM).
template <bool kBits>
__device__ __forceinline__ void warp_rows(const float* __restrict__ reward, const void* __restrict__ done,
                                          float gamma, int64_t B, int T, float* __restrict__ out, int64_t first_row,
                                          int64_t row_stride, unsigned char* wbase, uint64_t* bars, int nbuf,
                                          int lane) {
  auto s_rb = [&](uint32_t b) { return reinterpret_cast<float*>(wbase + b * kWarpSmem); };
  auto s_db = [&](uint32_t b) { return wbase + b * kWarpSmem + kRewardBytes; };
  if (lane == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_barrier_init();
  }
  __syncwarp();
  const double g = double(gamma), g_run = gamma_run(g);
  int64_t row = first_row;
  if (row >= B) return;
  int t1 = T;
  const int nw = (T + 31) >> 5;
  // Row r's done flags: bytes from r * T, or words from r * nw.
  auto drow = [&](int64_t r) -> const void* {
    return kBits ? static_cast<const void*>(static_cast<const uint32_t*>(done) + r * int64_t(nw))
                 : static_cast<const void*>(static_cast<const unsigned char*>(done) + r * int64_t(T));
  };
  // Current pass and its staging state.
  Pass cur = make_pass<kBits>(reward + row * int64_t(T), drow(row), t1 > kSeg ? t1 - kSeg : 0,
                              t1 > kSeg ? kSeg : t1, nw);
  Edges ecur = issue_pass<kBits>(cur, s_rb(0), s_db(0), &bars[0], lane);
  uint32_t k = 0;
  double carry = 0.0;
  for (;;) {
    // Work out and prefetch the next pass (next pass of this row, or the last pass of the next row).
    int64_t nrow = row;
    int nt1 = t1 - kSeg;
    if (nt1 <= 0) {
      nrow = row + row_stride;
      nt1 = T;
    }
    const bool has_next = nrow < B;
    Pass nxt{};
    Edges enxt{0.f, 0.f, 0u, 0u};
    const uint32_t nb = (k + 1) & 1u;
    if (has_next && nbuf == 2) {
      const int nt0 = nt1 > kSeg ? nt1 - kSeg : 0;
      nxt = make_pass<kBits>(reward + nrow * int64_t(T), drow(nrow), nt0, nt1 - nt0, nw);
      outputs_read(lane);  // buffer nb's outputs (the previous pass) have left shared memory
      enxt = issue_pass<kBits>(nxt, s_rb(nb), s_db(nb), &bars[nb], lane);
    }
    const uint32_t cb = nbuf == 2 ? (k & 1u) : 0u;
    const uint32_t par = nbuf == 2 ? ((k >> 1) & 1u) : (k & 1u);
    land_pass<kBits>(cur, ecur, s_rb(cb), s_db(cb), &bars[cb], par, lane);
    const double first = scan_pass<kBits>(cur, ecur, s_rb(cb), s_db(cb), carry, g, g_run, gamma, lane);
    const int t0 = t1 > kSeg ? t1 - kSeg : 0;
    if (k == 0) pdl_wait();  // first global write of this warp (no-op without PDL)
    store_pass(cur, s_rb(cb), out + row * int64_t(T) + t0, lane);
    __syncwarp();
    if (!has_next) break;
    if (nbuf == 1) {
      const int nt0 = nt1 > kSeg ? nt1 - kSeg : 0;
      nxt = make_pass<kBits>(reward + nrow * int64_t(T), drow(nrow), nt0, nt1 - nt0, nw);
      outputs_read(lane);
      enxt = issue_pass<kBits>(nxt, s_rb(0), s_db(0), &bars[0], lane);
    }
    carry = (nrow == row) ? first : 0.0;
    row = nrow;
    t1 = nt1;
    cur = nxt;
    ecur = enxt;
    ++k;
  }
  outputs_done(lane);
}

// Warp w of CTA c handles rows c*kWarps + w, + gridDim.x*kWarps, ...
template <bool kBits>
__global__ void __launch_bounds__(kThreads, 8) rtg_kernel(const float* __restrict__ reward,
                                                       const void* __restrict__ done, float gamma,
                                                       int B, int T, int nbuf, float* __restrict__ out) {
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint64_t bars[kWarps][2];  // one barrier per staging buffer
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  warp_rows<kBits>(reward, done, gamma, B, T, out, int64_t(blockIdx.x) * kWarps + warp,
                   int64_t(gridDim.x) * kWarps, smem + warp * nbuf * kWarpSmem, bars[warp], nbuf, lane);
}

// Done bytes -> bits: word [b, w] of `bits` holds done[b, 32w .. 32w + 31] (bits past T zero).
// One warp builds one word per step with a ballot over 32 consecutive flags of a row.
constexpr int kPackThreads = 256;
__global__ void __launch_bounds__(kPackThreads) pack_kernel(const unsigned char* __restrict__ done, int64_t B, int T,
                                                            uint32_t* __restrict__ bits) {
  pdl_begin();
  const int nw = (T + 31) >> 5;
  const int64_t words = B * int64_t(nw);
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (kPackThreads / 32);
  for (int64_t q = int64_t(blockIdx.x) * (kPackThreads / 32) + (threadIdx.x >> 5); q < words; q += warps) {
    const int64_t b = q / nw;
    const int t = int(q - b * nw) * 32 + lane;
    const bool d = t < T && done[b * int64_t(T) + t] != 0;
    const uint32_t w = __ballot_sync(0xffffffffu, d);
    if (lane == 0) bits[q] = w;
  }
}

inline int pack_done(const unsigned char* done, int32_t B, int32_t T, uint32_t* bits, cudaStream_t stream) {
  if (B < 0 || T < 0) return kInvalidArgument;
  if (B == 0 || T == 0) return kOk;
  if (done == nullptr || bits == nullptr) return kInvalidArgument;
  const int64_t words = int64_t(B) * ((int64_t(T) + 31) / 32);
  const int64_t want = (words + kPackThreads / 32 - 1) / (kPackThreads / 32);
  const int64_t cap = int64_t(sm_count()) * 8;
  return launch_pdl(pack_kernel, unsigned(want < cap ? want : cap), kPackThreads, 0, stream, done, int64_t(B), T,
                    bits);
}

template <bool kBits>
inline int run_impl(const float* reward, const void* done, float gamma, int32_t B, int32_t T, float* out,
                    cudaStream_t stream) {
  if (B < 0 || T < 0) return kInvalidArgument;
  if (B == 0 || T == 0) return kOk;
  if (reward == nullptr || done == nullptr || out == nullptr) return kInvalidArgument;
  // One row per warp in a single wave when the batch fits (10 CTAs = 40 warps per SM, one staging
  // buffer each); otherwise about 8 warps per SM streaming several rows through two buffers.
  const int64_t ctas_needed = (int64_t(B) + kWarps - 1) / kWarps;
  const int64_t one_wave = int64_t(sm_count()) * resident_ctas_per_sm(rtg_kernel<kBits>, kThreads, kSmemPerBuffer);
  const bool single = ctas_needed <= one_wave && T <= kSeg;
  const int nbuf = single ? 1 : 2;
  const int64_t cap = single ? one_wave : int64_t(sm_count()) * 2;
  const int grid = int(ctas_needed < cap ? ctas_needed : cap);
  return launch_pdl(rtg_kernel<kBits>, grid, kThreads, nbuf * kSmemPerBuffer, stream, reward, done, gamma, B, T, nbuf,
                    out);
}

// done: one byte per step, [B, T].
inline int run(const float* reward, const unsigned char* done, float gamma, int32_t B, int32_t T, float* out,
               cudaStream_t stream) {
  return run_impl<false>(reward, done, gamma, B, T, out, stream);
}

// done_bits: uint32 [B, ceil(T / 32)] from pack_done.
inline int run_bits(const float* reward, const uint32_t* done_bits, float gamma, int32_t B, int32_t T, float* out,
                    cudaStream_t stream) {
  return run_impl<true>(reward, done_bits, gamma, B, T, out, stream);
}

}  // namespace rtg
}  // namespace b200
