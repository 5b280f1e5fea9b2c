// PPO clipped surrogate loss and its diagnostics, in one HBM pass.
//
// Reference semantics: tasks/ppo_clip/reference.py:27-35 (fp64 oracle :42-45, where eps is first
// rounded to fp32 at :43).  Output order [loss, clip_fraction, approx_kl, ess, max_ratio,
// mean_ratio] (tasks/ppo_clip/tests/task.json:3-9).  The drop-in boundary it replaces is
// `void reference(const int32_t B, const int32_t T, const int32_t H, const float*
// current_log_prob, const float* old_log_prob, const float* advantage, const float clip_epsilon,
// float* output)` (task.json:3; expert host launcher reference/ppo_clip/solution.cu:165-182).
// The extended form adds a per-sample entropy stream and a 7th output, its mean (the
// BASELINE.json RL-pipeline configuration asks for the mean entropy diagnostic).
//
// Per element (lw = cur - old):
//   ratio r = exp(lw); clipped = lw < log1p(-eps) or lw > log1p(eps);
//   gain = min(r*adv, exp(clamp(lw))*adv)  (exp(clamp(lw)) is 1-eps / 1+eps when clipped, else r)
//   kl   = (r - 1) - lw, whose mean is (sum r - sum lw) / N - 1
// Reductions: sum gain, count clipped, sum lw, sum r, sum r^2, max r, [sum entropy].
// ESS = exp(2 lse(lw) - lse(2 lw)) / N = (sum r)^2 / (sum r^2) / N.
//
// B200 design.  12 (16 with entropy) bytes per element.  The element range is cut into fixed
// chunks of kChunk elements, each reduced by one CTA in a fixed order into a 48-byte partial
// (fp32 per thread, fp64 above), and the last CTA to finish combines the partials in chunk order:
// the result is bit-identical for any grid, any pointer alignment, and any chunk-aligned split of
// the range across GPUs (the multi-GPU path gathers the same partials and runs the same finish).
// Aligned inputs stream through a TMA bulk-copy pipeline: a producer warp keeps kStages chunks
// (48-64 KB each) in flight into shared memory with cp.async.bulk while 8 consumer warps reduce
// the resident chunk, so loads never wait for compute.  The clip decision matches the fp64
// oracle exactly: it is taken in fp32 and re-taken in fp64 for elements within 1e-6 of a clip
// boundary.  Elements with lw > 30 (outside the reference's stated input range, where r^2 could
// overflow fp32 sums) take an fp64 path.
#pragma once

#include <math.h>

#include "../common/b200_common.cuh"
#include "../common/bulk.cuh"
#include "../common/workspace.cuh"

namespace b200 {
namespace ppo {

constexpr int kThreads = 512;                                       // consumer threads
constexpr int kVecPerThread = 2;                                    // float4 per input per thread
constexpr int64_t kChunk = int64_t(kThreads) * kVecPerThread * 4;  // 4096 elements per chunk
constexpr int kPipeThreads = kThreads + 64;                         // + producer and reducer warps
constexpr uint32_t kRedBar = 1;                                     // named barrier of the consumers
constexpr int kOutputs = 6;
constexpr int kOutputsExt = 7;

template <bool kEnt>
struct Pipe {
  static constexpr int kArrays = kEnt ? 4 : 3;
  static constexpr int kArrayBytes = int(kChunk) * 4;
  static constexpr int kStageBytes = kArrays * kArrayBytes;
  static constexpr int kStages = kEnt ? 3 : 4;
  static constexpr int kSmem = kStages * kStageBytes;
};

struct __align__(16) Partial {
  double gain, lw, r, r2, ent;
  float rmax;
  unsigned clipped;
};
static_assert(sizeof(Partial) == 48, "partial layout");

// Clip constants derived on the host from the fp32 epsilon, in fp64 like the oracle.
struct Clip {
  double lo_d, hi_d;   // log1p(-eps), log1p(eps)
  float mid, hw;       // centre and half-width of [lo, hi] in fp32 (fast decision)
  float down, up;      // exp(log1p(-eps)), exp(log1p(eps)) rounded to fp32
};

inline Clip make_clip(float eps) {
  Clip c;
  const double e = double(eps);
  c.lo_d = log1p(-e);
  c.hi_d = log1p(e);
  c.mid = float(0.5 * (c.lo_d + c.hi_d));
  c.hw = float(0.5 * (c.hi_d - c.lo_d));
  c.down = float(exp(c.lo_d));
  c.up = float(exp(c.hi_d));
  return c;
}

inline int64_t num_chunks(int64_t n) { return (n + kChunk - 1) / kChunk; }
inline size_t workspace_bytes(int64_t n) { return 256 + align256(size_t(num_chunks(n)) * sizeof(Partial)); }

struct Acc {
  float gain = 0.f, lw = 0.f, r = 0.f, r2 = 0.f, ent = 0.f, rmax = 0.f;
  unsigned clipped = 0;
  double big_gain = 0.0, big_lw = 0.0, big_r = 0.0, big_r2 = 0.0;  // lw > 30 only
};

// Rare elements (within 1e-6 of a clip boundary, or lw > 30) leave the fast path: the clip
// decision is re-taken in fp64 and, for lw > 30, the element is accumulated in fp64.
__device__ __forceinline__ void add_element_slow(Acc& acc, float cur, float old, float adv, const Clip& c) {
  const double lwd = double(cur) - double(old);
  const bool below = lwd < c.lo_d;
  const bool clipped = below || lwd > c.hi_d;
  acc.clipped += clipped ? 1u : 0u;
  const float lw = __fsub_rn(cur, old);
  if (lw <= 30.0f) {
    const float r = __expf(lw);
    const float rc = clipped ? (below ? c.down : c.up) : r;
    acc.gain = __fadd_rn(acc.gain, fminf(__fmul_rn(r, adv), __fmul_rn(rc, adv)));
    acc.lw = __fadd_rn(acc.lw, lw);
    acc.r = __fadd_rn(acc.r, r);
    acc.r2 = __fmaf_rn(r, r, acc.r2);
    acc.rmax = fmaxf(acc.rmax, r);
  } else {
    const double r = exp(lwd);
    const double rc = exp(c.hi_d);
    acc.big_gain += fmin(r * double(adv), rc * double(adv));
    acc.big_lw += lwd;
    acc.big_r += r;
    acc.big_r2 += r * r;
    acc.rmax = fmaxf(acc.rmax, float(r));
  }
}

__device__ __forceinline__ void add_element(Acc& acc, float cur, float old, float adv, const Clip& c) {
  const float lw = __fsub_rn(cur, old);
  const float dm = __fsub_rn(lw, c.mid);
  const float adm = fabsf(dm);
  if (fabsf(__fsub_rn(adm, c.hw)) < 1e-6f || lw > 30.0f) {
    add_element_slow(acc, cur, old, adv, c);
    return;
  }
  const bool clipped = adm > c.hw;
  acc.clipped += clipped ? 1u : 0u;
  const float r = __expf(lw);
  const float rc = clipped ? (dm < 0.0f ? c.down : c.up) : r;
  acc.gain = __fadd_rn(acc.gain, fminf(__fmul_rn(r, adv), __fmul_rn(rc, adv)));
  acc.lw = __fadd_rn(acc.lw, lw);
  acc.r = __fadd_rn(acc.r, r);
  acc.r2 = __fmaf_rn(r, r, acc.r2);
  acc.rmax = fmaxf(acc.rmax, r);
}

template <bool kEnt>
__device__ __forceinline__ void add4(Acc& acc, float4 c4, float4 o4, float4 a4, float4 e4, const Clip& c) {
  add_element(acc, c4.x, o4.x, a4.x, c);
  add_element(acc, c4.y, o4.y, a4.y, c);
  add_element(acc, c4.z, o4.z, a4.z, c);
  add_element(acc, c4.w, o4.w, a4.w, c);
  if (kEnt) {
    acc.ent = __fadd_rn(acc.ent, e4.x);
    acc.ent = __fadd_rn(acc.ent, e4.y);
    acc.ent = __fadd_rn(acc.ent, e4.z);
    acc.ent = __fadd_rn(acc.ent, e4.w);
  }
}

// Per-thread pass over elements (k*kThreads + t)*4 + j of one chunk straight from global memory
// (k outer, j inner: the same order as the pipelined path), skipping elements past n.
template <bool kVec, bool kEnt>
__device__ __forceinline__ void thread_chunk_global(Acc& acc, const float* __restrict__ cur,
                                                    const float* __restrict__ old, const float* __restrict__ adv,
                                                    const float* __restrict__ ent, int64_t base, int64_t n,
                                                    const Clip& c) {
  const int t = threadIdx.x;
  if (kVec && base + kChunk <= n) {
    float4 vc[kVecPerThread], vo[kVecPerThread], va[kVecPerThread], ve[kVecPerThread];
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) {
      const int64_t i = base + int64_t(k * kThreads + t) * 4;
      vc[k] = ld_stream_f4(cur + i);
      vo[k] = ld_stream_f4(old + i);
      va[k] = ld_stream_f4(adv + i);
      ve[k] = kEnt ? ld_stream_f4(ent + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) add4<kEnt>(acc, vc[k], vo[k], va[k], ve[k], c);
  } else {
#pragma unroll 1
    for (int k = 0; k < kVecPerThread; ++k) {
      const int64_t i0 = base + int64_t(k * kThreads + t) * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t i = i0 + j;
        if (i < n) {
          add_element(acc, ld_stream_f1(cur + i), ld_stream_f1(old + i), ld_stream_f1(adv + i), c);
          if (kEnt) acc.ent = __fadd_rn(acc.ent, ld_stream_f1(ent + i));
        }
      }
    }
  }
}

// Warp-level record of one chunk (fp32 sums of the warp's 256 samples; the fp64 sums of the rare
// lw > 30 samples).  The reducer warp combines a chunk's 16 records in a fixed order.
struct WarpPart {
  float gain, lw, r, r2, ent, rmax;
  unsigned clipped, pad;
  double big_gain, big_lw, big_r, big_r2;
};
constexpr int kSlots = 4;                       // chunks in flight between consumers and reducer
constexpr int kConsumerWarps = kThreads / 32;   // 16

__device__ __forceinline__ void warp_record(const Acc& acc, WarpPart* slot, int lane) {
  float v[5] = {acc.gain, acc.lw, acc.r, acc.r2, acc.ent};
#pragma unroll
  for (int q = 0; q < 5; ++q)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[q] += __shfl_xor_sync(0xffffffffu, v[q], o);
  const float m = warp_max(acc.rmax);
  const unsigned cnt = warp_sum_u32(acc.clipped);
  const bool any_big = __any_sync(0xffffffffu, acc.big_r != 0.0);
  double bg = acc.big_gain, bl = acc.big_lw, br = acc.big_r, br2 = acc.big_r2;
  if (any_big) {
    bg = warp_sum(bg);
    bl = warp_sum(bl);
    br = warp_sum(br);
    br2 = warp_sum(br2);
  }
  if (lane == 0) {
    WarpPart w;
    w.gain = v[0];
    w.lw = v[1];
    w.r = v[2];
    w.r2 = v[3];
    w.ent = v[4];
    w.rmax = m;
    w.clipped = cnt;
    w.pad = 0;
    w.big_gain = any_big ? bg : 0.0;
    w.big_lw = any_big ? bl : 0.0;
    w.big_r = any_big ? br : 0.0;
    w.big_r2 = any_big ? br2 : 0.0;
    *slot = w;
  }
}

// Combine a chunk's kConsumerWarps warp records (lane w holds record w) into the chunk partial,
// valid in lane 0: fp64, fixed butterfly order.  Shared by every path, so all give the same bits.
__device__ __forceinline__ Partial combine_records(const WarpPart* recs, int lane) {
  double v[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
  float m = 0.f;
  unsigned cnt = 0;
  if (lane < kConsumerWarps) {
    const WarpPart& w = recs[lane];
    v[0] = double(w.gain);
    v[1] = double(w.lw);
    v[2] = double(w.r);
    v[3] = double(w.r2);
    v[4] = double(w.ent);
    v[5] = w.big_gain;
    v[6] = w.big_lw;
    v[7] = w.big_r;
    v[8] = w.big_r2;
    m = w.rmax;
    cnt = w.clipped;
  }
#pragma unroll
  for (int q = 0; q < 9; ++q) v[q] = warp_sum(v[q]);
  m = warp_max(m);
  cnt = warp_sum_u32(cnt);
  Partial p;
  p.gain = v[0] + v[5];
  p.lw = v[1] + v[6];
  p.r = v[2] + v[7];
  p.r2 = v[3] + v[8];
  p.ent = v[4];
  p.rmax = m;
  p.clipped = cnt;
  return p;
}

// Chunk partial of the kThreads consumer threads' accumulators (valid in thread 0), through the
// same warp records and combine as the pipelined path.  Uses a named barrier over the consumers.
__device__ __forceinline__ Partial cta_reduce(const Acc& acc) {
  __shared__ WarpPart s_rec[kConsumerWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  warp_record(acc, &s_rec[warp], lane);
  named_sync(kRedBar, kThreads);
  Partial p{};
  if (warp == 0) p = combine_records(s_rec, lane);
  named_sync(kRedBar, kThreads);
  return p;
}

// Final combination of partials[0..n_parts) in a fixed order by the kThreads consumer threads;
// writes 6 (or 7) outputs.  Every ratio is > 0, so 0 is the identity of the max.
__device__ __forceinline__ void finish(const Partial* parts, int64_t n_parts, int64_t n_total, bool ext, float* out) {
  __shared__ double s_d[5][kThreads / 32];
  __shared__ float s_max[kThreads / 32];
  __shared__ unsigned long long s_cnt[kThreads / 32];
  double v[5] = {0, 0, 0, 0, 0};
  float m = 0.f;
  unsigned long long cnt = 0;
  for (int64_t i = threadIdx.x; i < n_parts; i += kThreads) {
    const double* pd = reinterpret_cast<const double*>(parts + i);
#pragma unroll
    for (int q = 0; q < 5; ++q) v[q] += ld_cg_f64(pd + q);
    m = fmaxf(m, ld_cg_f32(reinterpret_cast<const float*>(pd + 5)));
    cnt += ld_cg_u32(reinterpret_cast<const unsigned*>(pd + 5) + 1);
  }
#pragma unroll
  for (int q = 0; q < 5; ++q) v[q] = warp_sum(v[q]);
  m = warp_max(m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
#pragma unroll
    for (int q = 0; q < 5; ++q) s_d[q][w] = v[q];
    s_max[w] = m;
    s_cnt[w] = cnt;
  }
  named_sync(kRedBar, kThreads);
  if (threadIdx.x == 0) {
    double t[5] = {0, 0, 0, 0, 0};
    float mx = 0.f;
    unsigned long long c = 0;
    for (int i = 0; i < kThreads / 32; ++i) {
#pragma unroll
      for (int q = 0; q < 5; ++q) t[q] += s_d[q][i];
      mx = fmaxf(mx, s_max[i]);
      c += s_cnt[i];
    }
    const double N = double(n_total);
    out[0] = float(-t[0] / N);
    out[1] = float(double(c) / N);
    out[2] = float((t[2] - t[1]) / N - 1.0);
    out[3] = float((t[2] / N) * (t[2] / t[3]));
    out[4] = n_total > 0 ? mx : __int_as_float(0x7fc00000);
    out[5] = float(t[2] / N);
    if (ext) out[6] = float(t[4] / N);
  }
}

// Direct form (unaligned inputs): CTA c handles chunks c, c + gridDim.x, ... from global memory.
template <bool kVec, bool kEnt, bool kFinish>
__global__ void __launch_bounds__(kThreads) chunk_kernel(const float* __restrict__ cur, const float* __restrict__ old,
                                                         const float* __restrict__ adv, const float* __restrict__ ent,
                                                         int64_t n, Clip clip, Partial* __restrict__ partials,
                                                         unsigned* __restrict__ ticket, float* __restrict__ out) {
  const int64_t n_chunks = (n + kChunk - 1) / kChunk;
  for (int64_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    Acc acc;
    thread_chunk_global<kVec, kEnt>(acc, cur, old, adv, ent, c * kChunk, n, clip);
    const Partial p = cta_reduce(acc);
    if (threadIdx.x == 0) partials[c] = p;
  }
  if (kFinish) {
    if (elect_last_cta(ticket)) finish(partials, n_chunks, n, kEnt, out);
  }
}

// Pipelined form (16-byte aligned inputs).  Warps 0-15 consume, warp 16 produces (bulk-copy ring),
// warp 17 reduces (16 warp records -> one chunk partial, fixed order, fp64).  A trailing partial
// chunk is read from global memory by the consumers of the CTA that owns it, in the same element
// order, and reduced the same way.  No CTA-wide barrier inside the loop.
template <bool kEnt, bool kFinish>
__global__ void __launch_bounds__(kPipeThreads, 1)
    pipe_kernel(const float* __restrict__ cur, const float* __restrict__ old, const float* __restrict__ adv,
                const float* __restrict__ ent, int64_t n, Clip clip, Partial* __restrict__ partials,
                unsigned* __restrict__ ticket, float* __restrict__ out) {
  using P = Pipe<kEnt>;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t full[P::kStages], empty[P::kStages], rec_full[kSlots], rec_free[kSlots];
  __shared__ WarpPart recs[kSlots][kConsumerWarps];
  const int64_t n_chunks = (n + kChunk - 1) / kChunk;
  const int64_t n_full = n / kChunk;
  const bool own_tail = n_full < n_chunks && (n_chunks - 1) % gridDim.x == blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < P::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&rec_full[s], kConsumerWarps);
      mbar_init(&rec_free[s], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // Producer: one lane keeps the ring full.
    if (lane == 0) {
      const float* src[4] = {cur, old, adv, ent};
      uint32_t i = 0;
      for (int64_t c = blockIdx.x; c < n_full; c += gridDim.x, ++i) {
        const uint32_t s = i % P::kStages, ph = (i / P::kStages) & 1u;
        mbar_wait(&empty[s], ph ^ 1u);
        mbar_arrive_expect_tx(&full[s], P::kStageBytes);
        unsigned char* dst = smem + s * P::kStageBytes;
#pragma unroll
        for (int a = 0; a < P::kArrays; ++a)
          bulk_g2s(dst + a * P::kArrayBytes, src[a] + c * kChunk, P::kArrayBytes, &full[s]);
      }
    }
  } else if (warp == kConsumerWarps + 1) {
    // Reducer: chunk i's 16 warp records, lane w holds record w; fixed-order fp64 tree.
    uint32_t i = 0;
    auto reduce_chunk = [&](int64_t c) {
      const uint32_t s = i % kSlots, ph = (i / kSlots) & 1u;
      mbar_wait(&rec_full[s], ph);
      const Partial p = combine_records(recs[s], lane);
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&rec_free[s]);
        partials[c] = p;
      }
      ++i;
    };
    for (int64_t c = blockIdx.x; c < n_full; c += gridDim.x) reduce_chunk(c);
    if (own_tail) reduce_chunk(n_chunks - 1);
  } else {
    uint32_t i = 0;
    auto record = [&](const Acc& acc) {
      const uint32_t s = i % kSlots, ph = (i / kSlots) & 1u;
      mbar_wait(&rec_free[s], ph ^ 1u);
      warp_record(acc, &recs[s][warp], lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&rec_full[s]);
      ++i;
    };
    uint32_t k = 0;
    for (int64_t c = blockIdx.x; c < n_full; c += gridDim.x, ++k) {
      const uint32_t s = k % P::kStages, ph = (k / P::kStages) & 1u;
      mbar_wait(&full[s], ph);
      const float* st = reinterpret_cast<const float*>(smem + s * P::kStageBytes);
      Acc acc;
#pragma unroll
      for (int kk = 0; kk < kVecPerThread; ++kk) {
        const int e = (kk * kThreads + threadIdx.x) * 4;
        const float4 c4 = *reinterpret_cast<const float4*>(st + e);
        const float4 o4 = *reinterpret_cast<const float4*>(st + kChunk + e);
        const float4 a4 = *reinterpret_cast<const float4*>(st + 2 * kChunk + e);
        const float4 e4 =
            kEnt ? *reinterpret_cast<const float4*>(st + 3 * kChunk + e) : make_float4(0.f, 0.f, 0.f, 0.f);
        add4<kEnt>(acc, c4, o4, a4, e4, clip);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      record(acc);
    }
    if (own_tail) {
      Acc acc;
      thread_chunk_global<true, kEnt>(acc, cur, old, adv, ent, (n_chunks - 1) * kChunk, n, clip);
      record(acc);
    }
  }
  if (kFinish) {
    const bool last = elect_last_cta(ticket);
    if (last && threadIdx.x < kThreads) finish(partials, n_chunks, n, kEnt, out);
  }
}

__global__ void __launch_bounds__(kThreads) finish_kernel(const Partial* __restrict__ partials, int64_t n_parts,
                                                          int64_t n_total, int ext, float* __restrict__ out) {
  finish(partials, n_parts, n_total, ext != 0, out);
}

template <bool kEnt, bool kFinish>
inline void launch_pipe(const float* cur, const float* old, const float* adv, const float* ent, int64_t n,
                        const Clip& clip, Partial* partials, unsigned* ticket, float* out, cudaStream_t stream) {
  auto kern = pipe_kernel<kEnt, kFinish>;
  ensure_dyn_smem(kern, Pipe<kEnt>::kSmem);
  const int grid = balanced_grid(num_chunks(n), 1);
  kern<<<grid, kPipeThreads, Pipe<kEnt>::kSmem, stream>>>(cur, old, adv, ent, n, clip, partials, ticket, out);
}

template <bool kEnt, bool kFinish>
inline void launch_direct(const float* cur, const float* old, const float* adv, const float* ent, int64_t n,
                          const Clip& clip, Partial* partials, unsigned* ticket, float* out, cudaStream_t stream) {
  auto kern = chunk_kernel<false, kEnt, kFinish>;
  const int grid = balanced_grid(num_chunks(n), resident_ctas_per_sm(kern, kThreads, 0));
  kern<<<grid, kThreads, 0, stream>>>(cur, old, adv, ent, n, clip, partials, ticket, out);
}

template <bool kFinish>
inline void launch_chunks(const float* cur, const float* old, const float* adv, const float* ent, int64_t n,
                          const Clip& clip, Partial* partials, unsigned* ticket, float* out, cudaStream_t stream) {
  const bool vec = aligned16(cur) && aligned16(old) && aligned16(adv) && (ent == nullptr || aligned16(ent));
  if (ent != nullptr) {
    if (vec) launch_pipe<true, kFinish>(cur, old, adv, ent, n, clip, partials, ticket, out, stream);
    else launch_direct<true, kFinish>(cur, old, adv, ent, n, clip, partials, ticket, out, stream);
  } else {
    if (vec) launch_pipe<false, kFinish>(cur, old, adv, ent, n, clip, partials, ticket, out, stream);
    else launch_direct<false, kFinish>(cur, old, adv, ent, n, clip, partials, ticket, out, stream);
  }
}

// Full op with a caller workspace (workspace_bytes(n), first 4 bytes zero before the first call).
// `ent` may be null (6 outputs) or an entropy stream (7 outputs).
inline int run(const float* cur, const float* old, const float* adv, const float* ent, int64_t n, float eps,
               float* out, void* workspace, size_t ws_bytes, cudaStream_t stream) {
  if (n < 0 || out == nullptr || (n > 0 && (cur == nullptr || old == nullptr || adv == nullptr)))
    return kInvalidArgument;
  if (workspace == nullptr || ws_bytes < workspace_bytes(n)) return kWorkspaceTooSmall;
  unsigned* ticket = static_cast<unsigned*>(workspace);
  Partial* partials = reinterpret_cast<Partial*>(static_cast<char*>(workspace) + 256);
  launch_chunks<true>(cur, old, adv, ent, n, make_clip(eps), partials, ticket, out, stream);
  return launch_status();
}

inline int shard_partials(const float* cur, const float* old, const float* adv, const float* ent, int64_t n,
                          float eps, Partial* partials, cudaStream_t stream) {
  if (n < 0 || (n > 0 && (cur == nullptr || old == nullptr || adv == nullptr || partials == nullptr)))
    return kInvalidArgument;
  if (n == 0) return kOk;
  launch_chunks<false>(cur, old, adv, ent, n, make_clip(eps), partials, nullptr, nullptr, stream);
  return launch_status();
}

inline int shard_finish(const Partial* partials, int64_t n_parts, int64_t n_total, bool ext, float* out,
                        cudaStream_t stream) {
  if (n_parts < 0 || n_total < 0 || out == nullptr || (n_parts > 0 && partials == nullptr)) return kInvalidArgument;
  finish_kernel<<<1, kThreads, 0, stream>>>(partials, n_parts, n_total, ext ? 1 : 0, out);
  return launch_status();
}

// B*T*H of the reference ABI, or -1 when a dimension is negative.
inline int64_t abi_count(int32_t B, int32_t T, int32_t H) {
  if (B < 0 || T < 0 || H < 0) return -1;
  return int64_t(B) * int64_t(T) * int64_t(H);
}

}  // namespace ppo
}  // namespace b200
