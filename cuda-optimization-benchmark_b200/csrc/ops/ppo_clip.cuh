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
// chunks of kChunk = 4096 samples, each reduced by one 256-thread CTA in a fixed order: each
// thread streams 4 float4 of every input (one of each at a time, 64 registers, 4 CTAs per SM)
// with 128-bit non-allocating loads, accumulates in fp32,
// each warp folds its lanes into one fp32 record, and the 8 records are combined in fp64 into a
// 48-byte chunk partial.  In the one-launch form of the PPO entry points each chunk partial is
// stored in LL form (every word with the launch's epoch) and the first CTA to reach its last chunk
// becomes the reducer: it folds the partials in chunk order as they arrive, so when the last chunk
// lands only about one L2 round trip remains.  (The fused RL step, where it measured slower, keeps
// plain partials and lets the last CTA to finish combine them, in the same order.)  The result is bit-identical for any grid, any pointer alignment, and any
// chunk-aligned split of the range across GPUs (the multi-GPU path gathers the same partials and
// runs the same combination), and the fused reward-to-go + PPO step kernel reuses the same
// per-chunk routine.  The clip decision
// matches the fp64 oracle exactly: it is taken in fp32 and re-taken in fp64 for elements within
// a few ulps of a clip boundary (Clip::margin).  Elements with lw > 30 (outside the reference's stated input range,
// where r^2 could overflow fp32 sums) take an fp64 path.
#pragma once

#include <math.h>

#include "../common/b200_common.cuh"
#include "../common/bulk.cuh"
#include "../common/ll.cuh"
#include "../common/workspace.cuh"

namespace b200 {
namespace ppo {

constexpr int kThreads = 256;                                       // threads per chunk
constexpr int kVecPerThread = 4;                                    // float4 per input per thread
constexpr int64_t kChunk = int64_t(kThreads) * kVecPerThread * 4;  // 4096 elements per chunk
constexpr uint32_t kRedBar = 1;                                     // named barrier of a chunk's threads
constexpr int kOutputs = 6;
constexpr int kOutputsExt = 7;

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
  float margin;        // |adm - hw| below which the fp32 decision may differ from the fp64 one
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
  // The fp32 test |fl(lw - mid)| > hw can disagree with the exact lw < lo or lw > hi only when
  // |lw - mid| is within the roundings of mid, hw and lw - mid of hw (lw itself is exact, or off by
  // at most half an ulp of |lw|, near a bound): a few ulps of hw + |mid|.  Eight ulps leave room;
  // samples inside the margin take the fp64 decision.
  const float span = c.hw + fabsf(c.mid);
  c.margin = 8.0f * (nextafterf(span, INFINITY) - span);
  return c;
}

__host__ __device__ inline int64_t num_chunks(int64_t n) { return (n + kChunk - 1) / kChunk; }

// Workspace of the one-launch forms: a 256-byte control block, then one plain 48-byte partial per
// chunk, then one 96-byte LL chunk record per chunk.  The control block must be zero before the
// first launch on it.
//   - ticket: completion counter of the last-CTA election (the fused RL step); left zero.
//   - claim, gen: the reducer claim and last epoch of the LL form (the PPO entry points); each
//     launch leaves `claim` zero and `gen` at its epoch, and the next launch's records carry
//     gen + 1, so no record of an earlier launch reads as fresh until the 32-bit counter wraps,
//     2^32 launches later.
// The two forms keep their records apart: a stale plain partial never meets an LL reader.
struct Control {
  unsigned ticket;
  unsigned claim;  // 1 once a CTA has become this launch's reducer
  unsigned gen;    // epoch of the last completed launch
};
constexpr int kPartWords = int(sizeof(Partial) / 4);          // 12
constexpr size_t kLLPartBytes = size_t(kPartWords) * 8;        // 96
inline size_t plain_region_bytes(int64_t n) { return align256(size_t(num_chunks(n)) * sizeof(Partial)); }
inline Partial* ws_partials(void* ws) { return reinterpret_cast<Partial*>(static_cast<char*>(ws) + 256); }
inline ulonglong2* ws_records(void* ws, int64_t n) {
  return reinterpret_cast<ulonglong2*>(static_cast<char*>(ws) + 256 + plain_region_bytes(n));
}
inline size_t workspace_bytes(int64_t n) {
  return 256 + plain_region_bytes(n) + align256(size_t(num_chunks(n)) * kLLPartBytes);
}

struct Acc {
  float gain = 0.f, lw = 0.f, r = 0.f, r2 = 0.f, ent = 0.f, rmax = 0.f;
  unsigned clipped = 0;
  double big_gain = 0.0, big_lw = 0.0, big_r = 0.0, big_r2 = 0.0;  // lw > 30 only
};

// Rare elements (within Clip::margin of a clip boundary, or lw > 30) leave the fast path: the clip
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
  if (fabsf(__fsub_rn(adm, c.hw)) < c.margin || lw > 30.0f) {
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

// Fast form of add_element: no rare-case branch.  It tracks what the rare cases test (the smallest
// |adm - hw| and the largest lw); when the tracked values show that some sample needed
// add_element_slow, the caller discards the accumulator and recomputes the same samples with
// add_element.  Otherwise every operation and its order equals add_element's, so the result has
// the same bits either way.
__device__ __forceinline__ void add_fast(Acc& acc, float cur, float old, float adv, const Clip& c, float& near,
                                         float& lw_max) {
  const float lw = __fsub_rn(cur, old);
  const float dm = __fsub_rn(lw, c.mid);
  const float adm = fabsf(dm);
  near = fminf(near, fabsf(__fsub_rn(adm, c.hw)));
  lw_max = fmaxf(lw_max, lw);
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
__device__ __forceinline__ void add4_fast(Acc& acc, float4 c4, float4 o4, float4 a4, float4 e4, const Clip& c,
                                          float& near, float& lw_max) {
  add_fast(acc, c4.x, o4.x, a4.x, c, near, lw_max);
  add_fast(acc, c4.y, o4.y, a4.y, c, near, lw_max);
  add_fast(acc, c4.z, o4.z, a4.z, c, near, lw_max);
  add_fast(acc, c4.w, o4.w, a4.w, c, near, lw_max);
  if (kEnt) {
    acc.ent = __fadd_rn(acc.ent, e4.x);
    acc.ent = __fadd_rn(acc.ent, e4.y);
    acc.ent = __fadd_rn(acc.ent, e4.z);
    acc.ent = __fadd_rn(acc.ent, e4.w);
  }
}

// Per-thread pass over elements (k*kThreads + t)*4 + j of one chunk straight from global memory
// (k outer, j inner), skipping elements past n; the vector and scalar forms give the same bits.
template <bool kVec, bool kEnt>
__device__ __forceinline__ void thread_chunk_global(Acc& acc, const float* __restrict__ cur,
                                                    const float* __restrict__ old, const float* __restrict__ adv,
                                                    const float* __restrict__ ent, int64_t base, int64_t n,
                                                    const Clip& c) {
  const int t = threadIdx.x;
  if (kVec && base + kChunk <= n) {
    // One float4 of each stream at a time: few live registers, so more CTAs share an SM.
    float near = __int_as_float(0x7f800000), lw_max = -__int_as_float(0x7f800000);
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) {
      const int64_t i = base + int64_t(k * kThreads + t) * 4;
      const float4 vc = ld_stream_f4(cur + i);
      const float4 vo = ld_stream_f4(old + i);
      const float4 va = ld_stream_f4(adv + i);
      const float4 ve = kEnt ? ld_stream_f4(ent + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      add4_fast<kEnt>(acc, vc, vo, va, ve, c, near, lw_max);
    }
    if (near < c.margin || lw_max > 30.0f) {  // rare: some sample needs add_element_slow
      acc = Acc();
#pragma unroll 1
      for (int k = 0; k < kVecPerThread; ++k) {
        const int64_t i = base + int64_t(k * kThreads + t) * 4;
        const float4 ve = kEnt ? ld_stream_f4(ent + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        add4<kEnt>(acc, ld_stream_f4(cur + i), ld_stream_f4(old + i), ld_stream_f4(adv + i), ve, c);
      }
    }
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

constexpr int kConsumerWarps = kThreads / 32;   // 8

// bar.red.or over the `count` threads of named barrier `id`: a barrier that also returns whether
// any arriving thread passed true.
__device__ __forceinline__ bool named_sync_or(uint32_t id, uint32_t count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %3, 0;\n\t"
      "barrier.red.or.pred q, %1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(count), "r"(v ? 1u : 0u)
      : "memory");
  return r != 0;
}

// Shared scratch of one 256-thread reduction group.
struct RedScratch {
  float v[5][kThreads];  // per-thread gain, lw, r, r2, ent
  float m[kThreads];     // per-thread max ratio
  unsigned c[kThreads];  // per-thread clip count
  double sum[5];
  double big[kConsumerWarps][4];
  float mx;
  unsigned cnt;
};

// Chunk partial of a group's 256 accumulators (tid = thread index in the group, `bar` its named
// barrier), valid in tid 0.  Each thread parks its fp32 sums in shared memory; warp q < 5 then
// adds quantity q over the 256 threads in fp64 (lane l takes threads l, l+32, ..., l+224 in that
// order, then a fixed butterfly), warp 5 takes the max and warp 6 the count.  The fp64 sums of the
// rare lw > 30 samples are added per warp, then over warps in order, only when a thread has some.
// Every path (one launch, fused step, multi-GPU shards) reduces a chunk through this routine, so all
// give the same bits.
__device__ __forceinline__ Partial group_reduce(const Acc& acc, RedScratch& s, int tid, uint32_t bar) {
  s.v[0][tid] = acc.gain;
  s.v[1][tid] = acc.lw;
  s.v[2][tid] = acc.r;
  s.v[3][tid] = acc.r2;
  s.v[4][tid] = acc.ent;
  s.m[tid] = acc.rmax;
  s.c[tid] = acc.clipped;
  const bool any_big = named_sync_or(bar, kThreads, acc.big_r != 0.0);
  const int w = tid >> 5, lane = tid & 31;
  if (w < 5) {
    double x = 0.0;
#pragma unroll
    for (int j = 0; j < kConsumerWarps; ++j) x += double(s.v[w][lane + 32 * j]);
    x = warp_sum(x);
    if (lane == 0) s.sum[w] = x;
  } else if (w == 5) {
    float x = 0.f;
#pragma unroll
    for (int j = 0; j < kConsumerWarps; ++j) x = fmaxf(x, s.m[lane + 32 * j]);
    x = warp_max(x);
    if (lane == 0) s.mx = x;
  } else if (w == 6) {
    unsigned x = 0;
#pragma unroll
    for (int j = 0; j < kConsumerWarps; ++j) x += s.c[lane + 32 * j];
    x = warp_sum_u32(x);
    if (lane == 0) s.cnt = x;
  }
  if (any_big) {
    const double b0 = warp_sum(acc.big_gain), b1 = warp_sum(acc.big_lw);
    const double b2 = warp_sum(acc.big_r), b3 = warp_sum(acc.big_r2);
    if (lane == 0) {
      s.big[w][0] = b0;
      s.big[w][1] = b1;
      s.big[w][2] = b2;
      s.big[w][3] = b3;
    }
  }
  named_sync(bar, kThreads);
  Partial p{};
  if (tid == 0) {
    double bg[4] = {0.0, 0.0, 0.0, 0.0};
    if (any_big) {
      for (int i = 0; i < kConsumerWarps; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) bg[q] += s.big[i][q];
    }
    p.gain = s.sum[0] + bg[0];
    p.lw = s.sum[1] + bg[1];
    p.r = s.sum[2] + bg[2];
    p.r2 = s.sum[3] + bg[3];
    p.ent = s.sum[4];
    p.rmax = s.mx;
    p.clipped = s.cnt;
  }
  return p;
}

// group_reduce over the kThreads threads of a chunk CTA (named barrier kRedBar).
__device__ __forceinline__ Partial cta_reduce(const Acc& acc) {
  __shared__ RedScratch s_red;
  return group_reduce(acc, s_red, threadIdx.x, kRedBar);
}

// Totals of a set of partials: the five sums, the ratio max and the clipped count.
struct Sums {
  double t[5];  // gain, lw, r, r2, ent
  float mx;
  unsigned long long c;
};

// Thread t accumulates records t, t + kThreads, ... in order (kU per round, loads issued before the
// adds); combine_threads then adds each warp's lanes by a butterfly and the 8 warps in order.  The
// totals are valid in thread 0.  Every ratio is > 0, so 0 is the identity of the max.
struct ThreadSums {
  double v[5] = {0, 0, 0, 0, 0};
  float m = 0.f;
  unsigned long long cnt = 0;
  __device__ __forceinline__ void add(const double (&d)[6]) {
#pragma unroll
    for (int q = 0; q < 5; ++q) v[q] += d[q];
    const unsigned long long w = __double_as_longlong(d[5]);
    m = fmaxf(m, __uint_as_float(unsigned(w & 0xffffffffull)));
    cnt += unsigned(w >> 32);
  }
};

__device__ __forceinline__ Sums combine_threads(ThreadSums a) {
  __shared__ double s_d[5][kThreads / 32];
  __shared__ float s_max[kThreads / 32];
  __shared__ unsigned long long s_cnt[kThreads / 32];
#pragma unroll
  for (int q = 0; q < 5; ++q) a.v[q] = warp_sum(a.v[q]);
  a.m = warp_max(a.m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a.cnt += __shfl_xor_sync(0xffffffffu, a.cnt, o);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
#pragma unroll
    for (int q = 0; q < 5; ++q) s_d[q][w] = a.v[q];
    s_max[w] = a.m;
    s_cnt[w] = a.cnt;
  }
  named_sync(kRedBar, kThreads);
  Sums t{{0, 0, 0, 0, 0}, 0.f, 0ull};
  if (threadIdx.x == 0) {
    for (int i = 0; i < kThreads / 32; ++i) {
#pragma unroll
      for (int q = 0; q < 5; ++q) t.t[q] += s_d[q][i];
      t.mx = fmaxf(t.mx, s_max[i]);
      t.c += s_cnt[i];
    }
  }
  return t;
}

__device__ __forceinline__ void partial_words(const Partial& p, uint32_t (&w)[kPartWords]) { memcpy(w, &p, sizeof(p)); }
__device__ __forceinline__ void words_to_doubles(const uint32_t (&w)[kPartWords], double (&d)[6]) {
#pragma unroll
  for (int q = 0; q < 6; ++q) d[q] = __hiloint2double(int(w[2 * q + 1]), int(w[2 * q]));
}

// Combination of partials[0..n_parts) (all written before this launch or by CTAs that have
// finished) by the kThreads threads of one CTA.
__device__ __forceinline__ Sums reduce_partials(const Partial* parts, int64_t n_parts) {
  ThreadSums a;
  for (int64_t i0 = threadIdx.x; i0 < n_parts; i0 += 4 * kThreads) {
    double d[4][6];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t i = i0 + int64_t(u) * kThreads;
      const double* pd = reinterpret_cast<const double*>(parts + (i < n_parts ? i : 0));
#pragma unroll
      for (int q = 0; q < 6; ++q) d[u][q] = i < n_parts ? ld_cg_f64(pd + q) : 0.0;  // L2: other CTAs wrote them
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (i0 + int64_t(u) * kThreads < n_parts) a.add(d[u]);
  }
  return combine_threads(a);
}

// The same combination over LL chunk records of this launch's epoch that are still arriving: each
// thread waits (bounded) for the records it adds, in its fixed order.
// kU records in flight per thread (24 registers of loads each).
template <int kU>
__device__ __forceinline__ Sums reduce_arriving(const ulonglong2* recs, int64_t n_parts, unsigned epoch) {
  ThreadSums a;
  LLReader<kPartWords, LLScope::kGpu> rd{recs, epoch};  // records of this grid's CTAs
  for (int64_t i0 = threadIdx.x; i0 < n_parts; i0 += kU * kThreads) {
    int64_t idx[kU];
    bool use[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      idx[u] = i0 + int64_t(u) * kThreads;
      use[u] = idx[u] < n_parts;
    }
    uint32_t w[kU][kPartWords];
    rd.read<kU>(idx, use, w);
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (use[u]) {
        double d[6];
        words_to_doubles(w[u], d);
        a.add(d);
      }
    }
  }
  return combine_threads(a);
}

// The 6 (or 7) outputs from the totals over n_total samples (one thread).  inv_n = 1 / n_total
// from the host (infinite for an empty batch, which makes every mean NaN, as the mean of nothing
// is).  Means by that 1/N (an fp64 divide takes hundreds of cycles on this tail); the ESS ratio
// sum(r) / sum(r^2) by one correctly rounded fp32 divide (relative error ~1e-7).
__device__ __forceinline__ void write_outputs(const Sums& s, int64_t n_total, double inv_n, bool ext, float* out) {
  out[0] = float(-s.t[0] * inv_n);
  out[1] = float(double(s.c) * inv_n);
  out[2] = float((s.t[2] - s.t[1]) * inv_n - 1.0);
  out[3] = float((s.t[2] * inv_n) * double(__fdiv_rn(float(s.t[2]), float(s.t[3]))));
  out[4] = n_total > 0 ? s.mx : __int_as_float(0x7fc00000);
  out[5] = float(s.t[2] * inv_n);
  if (ext) out[6] = float(s.t[4] * inv_n);
}

// Final combination of partials[0..n_parts) by the kThreads threads of one CTA; writes the outputs.
__device__ __forceinline__ void finish(const Partial* parts, int64_t n_parts, int64_t n_total, double inv_n, bool ext,
                                       float* out) {
  const Sums s = reduce_partials(parts, n_parts);
  if (threadIdx.x == 0) write_outputs(s, n_total, inv_n, ext, out);
}

// Chunk partials of chunks cta, cta + n_ctas, ... (all kThreads threads of the CTA take part);
// thread 0 hands chunk c's partial to `store(c, p)`, the first time after pdl_wait().
template <bool kVec, bool kEnt, class Store>
__device__ __forceinline__ void chunk_partials_to(const float* __restrict__ cur, const float* __restrict__ old,
                                                  const float* __restrict__ adv, const float* __restrict__ ent,
                                                  int64_t n, const Clip& clip, const Store& store, int64_t cta,
                                                  int64_t n_ctas) {
  const int64_t n_chunks = (n + kChunk - 1) / kChunk;
  for (int64_t c = cta; c < n_chunks; c += n_ctas) {
    Acc acc;
    thread_chunk_global<kVec, kEnt>(acc, cur, old, adv, ent, c * kChunk, n, clip);
    const Partial p = cta_reduce(acc);
    if (threadIdx.x == 0) {
      if (c == cta) pdl_wait();  // first global write of this CTA (no-op without PDL)
      store(c, p);
    }
  }
}

struct PlainStore {
  Partial* partials;
  __device__ __forceinline__ void operator()(int64_t c, const Partial& p) const { partials[c] = p; }
};

template <bool kVec, bool kEnt>
__device__ __forceinline__ void chunk_partials(const float* __restrict__ cur, const float* __restrict__ old,
                                               const float* __restrict__ adv, const float* __restrict__ ent, int64_t n,
                                               const Clip& clip, Partial* __restrict__ partials, int64_t cta,
                                               int64_t n_ctas) {
  chunk_partials_to<kVec, kEnt>(cur, old, adv, ent, n, clip, PlainStore{partials}, cta, n_ctas);
}

// The one-launch form's epoch: once the previous kernel on the stream has completed (so the last
// launch's `gen` is visible and its claim reset), gen + 1, skipping 0.  By thread 0.
__device__ __forceinline__ unsigned open_epoch(Control* ctl) {
  pdl_wait();
  const unsigned e = *reinterpret_cast<volatile unsigned*>(&ctl->gen) + 1u;
  return e == 0u ? 1u : e;
}

// By the reducer's thread 0 when the launch's outputs are written: the control block is ready for
// the next launch (which reads it only after this one has completed).
__device__ __forceinline__ void close_epoch(Control* ctl, unsigned epoch) {
  *reinterpret_cast<volatile unsigned*>(&ctl->claim) = 0u;
  *reinterpret_cast<volatile unsigned*>(&ctl->gen) = epoch;
}

// One-launch form of chunk_partials: the partials of chunks cta, cta + n_ctas, ... go to `recs` in
// LL form with the launch's epoch.  Thread 0 claims the reduction before it stores its CTA's last
// chunk (a CTA without a chunk, only the single CTA of an empty batch, claims at once), so the
// claim is taken exactly once, and before the reducer can have seen every record.  Returns true
// in the claiming CTA; *epoch receives the launch's epoch (all threads).
template <bool kVec, bool kEnt>
__device__ __forceinline__ bool chunk_records(const float* __restrict__ cur, const float* __restrict__ old,
                                              const float* __restrict__ adv, const float* __restrict__ ent, int64_t n,
                                              const Clip& clip, ulonglong2* __restrict__ recs, Control* ctl,
                                              int64_t cta, int64_t n_ctas, unsigned* epoch) {
  __shared__ unsigned s_epoch, s_claim;
  const int64_t n_chunks = num_chunks(n);
  unsigned e = 0;
  bool claimed = false;
  for (int64_t c = cta; c < n_chunks; c += n_ctas) {
    Acc acc;
    thread_chunk_global<kVec, kEnt>(acc, cur, old, adv, ent, c * kChunk, n, clip);
    const Partial p = cta_reduce(acc);
    if (threadIdx.x == 0) {
      if (e == 0) e = open_epoch(ctl);
      if (c + n_ctas >= n_chunks) claimed = atomicCAS(&ctl->claim, 0u, 1u) == 0u;
      uint32_t w[kPartWords];
      partial_words(p, w);
      ll_store_record<kPartWords, LLScope::kGpu>(recs + c * (kPartWords / 2), w, e);
    }
  }
  if (threadIdx.x == 0) {
    if (e == 0) {
      e = open_epoch(ctl);
      claimed = atomicCAS(&ctl->claim, 0u, 1u) == 0u;
    }
    s_epoch = e;
    s_claim = claimed ? 1u : 0u;
  }
  __syncthreads();
  *epoch = s_epoch;
  return s_claim != 0u;
}

// Before waiting for the previous kernel, thread 0 asks L2 for this CTA's chunks of every input
// stream (16 KB bulk prefetches, 16-byte aligned inputs only): the batch starts streaming from HBM
// at once, overlapping the previous kernel's tail, instead of as each thread's first loads are
// issued.  L2 is the point of coherence, so this is safe even if that kernel writes the inputs.
// One launch prefetches at most kPrefetchBudget bytes (the CTAs' first chunks, then their second
// ones, ...): under PDL the next launch's CTAs start, and prefetch, while this launch still reads,
// and two launches' prefetches beyond L2's capacity evict each other's lines before they are read.
// PPO with entropy (65.5 MB a call, four input sets rotating): 17.1 us a call with every chunk
// prefetched, 14.1 us with the budget (first chunks only); without entropy (49 MB) the budget
// covers every chunk, as before.
constexpr int64_t kPrefetchBudget = int64_t(48) << 20;

template <bool kEnt>
__device__ __forceinline__ void prefetch_chunks(const float* cur, const float* old, const float* adv,
                                                const float* ent, int64_t n, int64_t cta, int64_t n_ctas) {
  const int64_t n_chunks = num_chunks(n);
  const int64_t chunk_bytes = kChunk * 4 * (kEnt ? 4 : 3);
  for (int64_t c = cta, q = 1; c < n_chunks && q * n_ctas * chunk_bytes <= kPrefetchBudget; c += n_ctas, ++q) {
    const int64_t e0 = c * kChunk, cnt = (n - e0 < kChunk ? n - e0 : kChunk);
    const uint32_t bytes = uint32_t(cnt * 4) & ~15u;
    if (bytes == 0) continue;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(cur + e0), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(old + e0), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(adv + e0), "r"(bytes) : "memory");
    if (kEnt) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ent + e0), "r"(bytes) : "memory");
  }
}

// One launch of the whole op (CTA c handles chunks c, c + gridDim.x, ...; the grid is one resident
// wave, so the reducer's waits always end).  kVec: 128-bit loads for full chunks (16-byte aligned
// inputs).
template <bool kVec, bool kEnt>
__global__ void __launch_bounds__(kThreads, 4) loss_kernel(const float* __restrict__ cur, const float* __restrict__ old,
                                                        const float* __restrict__ adv, const float* __restrict__ ent,
                                                        int64_t n, Clip clip, ulonglong2* __restrict__ recs,
                                                        Control* __restrict__ ctl, double inv_n,
                                                        float* __restrict__ out) {
  if (kVec && threadIdx.x == 0) prefetch_chunks<kEnt>(cur, old, adv, ent, n, blockIdx.x, gridDim.x);
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  unsigned epoch;
  if (!chunk_records<kVec, kEnt>(cur, old, adv, ent, n, clip, recs, ctl, blockIdx.x, gridDim.x, &epoch)) return;
  const Sums s = reduce_arriving<1>(recs, num_chunks(n), epoch);  // 64 registers at 4 CTAs per SM
  if (threadIdx.x == 0) {
    write_outputs(s, n, inv_n, kEnt, out);
    close_epoch(ctl, epoch);
  }
}

// Chunk partials only (the multi-GPU shard form), plain 48-byte records.
template <bool kVec, bool kEnt>
__global__ void __launch_bounds__(kThreads, 4) partials_kernel(const float* __restrict__ cur,
                                                            const float* __restrict__ old,
                                                            const float* __restrict__ adv,
                                                            const float* __restrict__ ent, int64_t n, Clip clip,
                                                            Partial* __restrict__ partials) {
  if (kVec && threadIdx.x == 0) prefetch_chunks<kEnt>(cur, old, adv, ent, n, blockIdx.x, gridDim.x);
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  chunk_partials<kVec, kEnt>(cur, old, adv, ent, n, clip, partials, blockIdx.x, gridDim.x);
}

__global__ void __launch_bounds__(kThreads) finish_kernel(const Partial* __restrict__ partials, int64_t n_parts,
                                                          int64_t n_total, double inv_n, int ext,
                                                          float* __restrict__ out) {
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  finish(partials, n_parts, n_total, inv_n, ext != 0, out);
}

inline double inv_count(int64_t n) { return 1.0 / double(n); }

template <bool kVec, bool kEnt>
inline void launch_loss(const float* cur, const float* old, const float* adv, const float* ent, int64_t n,
                        const Clip& clip, ulonglong2* recs, Control* ctl, float* out, cudaStream_t stream) {
  auto kern = loss_kernel<kVec, kEnt>;
  const int grid = balanced_grid(num_chunks(n), resident_ctas_per_sm(kern, kThreads, 0));
  launch_pdl(kern, grid, kThreads, 0, stream, cur, old, adv, ent, n, clip, recs, ctl, inv_count(n), out);
}

template <bool kVec, bool kEnt>
inline void launch_partials(const float* cur, const float* old, const float* adv, const float* ent, int64_t n,
                            const Clip& clip, Partial* partials, cudaStream_t stream) {
  auto kern = partials_kernel<kVec, kEnt>;
  const int grid = balanced_grid(num_chunks(n), resident_ctas_per_sm(kern, kThreads, 0));
  launch_pdl(kern, grid, kThreads, 0, stream, cur, old, adv, ent, n, clip, partials);
}

inline bool vec_ok(const float* cur, const float* old, const float* adv, const float* ent) {
  return aligned16(cur) && aligned16(old) && aligned16(adv) && (ent == nullptr || aligned16(ent));
}

// Full op with a caller workspace (workspace_bytes(n); its control block zero before the first
// call, as every call leaves it ready for the next), in one launch with the progressive reducer.  `ent` may be null (6 outputs) or an entropy
// stream (7 outputs).
inline int run(const float* cur, const float* old, const float* adv, const float* ent, int64_t n, float eps,
               float* out, void* workspace, size_t ws_bytes, cudaStream_t stream) {
  if (n < 0 || out == nullptr || (n > 0 && (cur == nullptr || old == nullptr || adv == nullptr)))
    return kInvalidArgument;
  if (workspace == nullptr || ws_bytes < workspace_bytes(n)) return kWorkspaceTooSmall;
  Control* ctl = static_cast<Control*>(workspace);
  ulonglong2* recs = ws_records(workspace, n);
  const Clip clip = make_clip(eps);
  const bool vec = vec_ok(cur, old, adv, ent);
  if (ent != nullptr) {
    if (vec) launch_loss<true, true>(cur, old, adv, ent, n, clip, recs, ctl, out, stream);
    else launch_loss<false, true>(cur, old, adv, ent, n, clip, recs, ctl, out, stream);
  } else {
    if (vec) launch_loss<true, false>(cur, old, adv, ent, n, clip, recs, ctl, out, stream);
    else launch_loss<false, false>(cur, old, adv, ent, n, clip, recs, ctl, out, stream);
  }
  return launch_status();
}

inline int shard_partials(const float* cur, const float* old, const float* adv, const float* ent, int64_t n,
                          float eps, Partial* partials, cudaStream_t stream) {
  if (n < 0 || (n > 0 && (cur == nullptr || old == nullptr || adv == nullptr || partials == nullptr)))
    return kInvalidArgument;
  if (n == 0) return kOk;
  const Clip clip = make_clip(eps);
  const bool vec = vec_ok(cur, old, adv, ent);
  if (ent != nullptr) {
    if (vec) launch_partials<true, true>(cur, old, adv, ent, n, clip, partials, stream);
    else launch_partials<false, true>(cur, old, adv, ent, n, clip, partials, stream);
  } else {
    if (vec) launch_partials<true, false>(cur, old, adv, ent, n, clip, partials, stream);
    else launch_partials<false, false>(cur, old, adv, ent, n, clip, partials, stream);
  }
  return launch_status();
}

inline int shard_finish(const Partial* partials, int64_t n_parts, int64_t n_total, bool ext, float* out,
                        cudaStream_t stream) {
  if (n_parts < 0 || n_total < 0 || out == nullptr || (n_parts > 0 && partials == nullptr)) return kInvalidArgument;
  return launch_pdl(finish_kernel, 1, kThreads, 0, stream, partials, n_parts, n_total, inv_count(n_total), ext ? 1 : 0,
                    out);
}

// B*T*H of the reference ABI, or -1 when a dimension is negative.
inline int64_t abi_count(int32_t B, int32_t T, int32_t H) {
  if (B < 0 || T < 0 || H < 0) return -1;
  return int64_t(B) * int64_t(T) * int64_t(H);
}

}  // namespace ppo
}  // namespace b200
