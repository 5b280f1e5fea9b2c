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
//   kl   = (r - 1) - lw  (evaluated as expm1(lw) - lw to avoid cancellation)
// Reductions: sum gain, count clipped, sum kl, sum r, sum r^2, max r, [sum entropy].
// ESS = exp(2 lse(lw) - lse(2 lw)) / N = (sum r)^2 / (sum r^2) / N.
//
// B200 design: 12 (16 with entropy) bytes per element streamed with 128-bit loads; fixed global
// chunking with one 48-byte partial per chunk, fp32 per-thread accumulation and fp64 above it;
// single-launch finish by the last CTA.  Deterministic for any grid and any chunk-aligned split
// across GPUs.  The clip decision matches the fp64 oracle exactly: lw is formed in fp32 and only
// elements within 1e-6 of a clip boundary are re-decided in fp64.  Elements with lw > 30 (outside
// the reference's stated input range, where r^2 could overflow fp32 sums) take an fp64 path.
#pragma once

#include <math.h>

#include "../common/b200_common.cuh"
#include "../common/workspace.cuh"

namespace b200 {
namespace ppo {

constexpr int kThreads = 256;
constexpr int kVecPerThread = 4;                                    // float4 per input per thread
constexpr int64_t kChunk = int64_t(kThreads) * kVecPerThread * 4;  // 4096 elements per chunk
constexpr int kOutputs = 6;
constexpr int kOutputsExt = 7;

struct __align__(16) Partial {
  double gain, kl, r, r2, ent;
  float rmax;
  unsigned clipped;
};
static_assert(sizeof(Partial) == 48, "partial layout");

// Clip constants derived on the host from the fp32 epsilon, in fp64 like the oracle.
struct Clip {
  double lo_d, hi_d;   // log1p(-eps), log1p(eps)
  float lo_f, hi_f;    // the same rounded to fp32 (fast decision away from the boundary)
  float down, up;      // exp(log1p(-eps)), exp(log1p(eps)) rounded to fp32
};

inline Clip make_clip(float eps) {
  Clip c;
  const double e = double(eps);
  c.lo_d = log1p(-e);
  c.hi_d = log1p(e);
  c.lo_f = float(c.lo_d);
  c.hi_f = float(c.hi_d);
  c.down = float(exp(c.lo_d));
  c.up = float(exp(c.hi_d));
  return c;
}

inline int64_t num_chunks(int64_t n) { return (n + kChunk - 1) / kChunk; }
inline size_t workspace_bytes(int64_t n) { return 256 + align256(size_t(num_chunks(n)) * sizeof(Partial)); }

struct Acc {
  float gain = 0.f, kl = 0.f, r = 0.f, r2 = 0.f, ent = 0.f, rmax = 0.f;
  unsigned clipped = 0;
  double big_gain = 0.0, big_kl = 0.0, big_r = 0.0, big_r2 = 0.0;  // lw > 30 only
};

__device__ __forceinline__ void add_element(Acc& acc, float cur, float old, float adv, const Clip& c) {
  const float lw = __fsub_rn(cur, old);
  bool lo = lw < c.lo_f, hi = lw > c.hi_f;
  // Near a boundary the fp32 difference may sit on the other side of the fp64 one: redo it in fp64.
  if (fabsf(__fsub_rn(lw, c.hi_f)) < 1e-6f || fabsf(__fsub_rn(lw, c.lo_f)) < 1e-6f) {
    const double lwd = double(cur) - double(old);
    lo = lwd < c.lo_d;
    hi = lwd > c.hi_d;
  }
  acc.clipped += (lo || hi) ? 1u : 0u;
  if (lw <= 30.0f) {
    const float em1 = expm1f(lw);
    const float r = __fadd_rn(em1, 1.0f);
    const float rc = lo ? c.down : (hi ? c.up : r);
    const float g = fminf(__fmul_rn(r, adv), __fmul_rn(rc, adv));
    acc.gain = __fadd_rn(acc.gain, g);
    acc.kl = __fadd_rn(acc.kl, __fsub_rn(em1, lw));
    acc.r = __fadd_rn(acc.r, r);
    acc.r2 = __fmaf_rn(r, r, acc.r2);
    acc.rmax = fmaxf(acc.rmax, r);
  } else {
    const double lwd = double(cur) - double(old);
    const double r = exp(lwd);
    const double rc = hi ? exp(c.hi_d) : r;
    acc.big_gain += fmin(r * double(adv), rc * double(adv));
    acc.big_kl += (r - 1.0) - lwd;
    acc.big_r += r;
    acc.big_r2 += r * r;
    acc.rmax = fmaxf(acc.rmax, float(r));
  }
}

// Per-thread pass over elements (k*kThreads + t)*4 + j of one chunk, same order on every path.
template <bool kVec, bool kEnt>
__device__ __forceinline__ void thread_chunk(Acc& acc, const float* __restrict__ cur, const float* __restrict__ old,
                                             const float* __restrict__ adv, const float* __restrict__ ent,
                                             int64_t base, int64_t n, const Clip& c) {
  const int t = threadIdx.x;
  if (kVec && base + kChunk <= n) {
    float4 vc[kVecPerThread], vo[kVecPerThread], va[kVecPerThread], ve[kVecPerThread];
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) {
      const int64_t i = base + int64_t(k * kThreads + t) * 4;
      vc[k] = ld_stream_f4(cur + i);
      vo[k] = ld_stream_f4(old + i);
      va[k] = ld_stream_f4(adv + i);
      if (kEnt) ve[k] = ld_stream_f4(ent + i);
    }
#pragma unroll
    for (int k = 0; k < kVecPerThread; ++k) {
      add_element(acc, vc[k].x, vo[k].x, va[k].x, c);
      add_element(acc, vc[k].y, vo[k].y, va[k].y, c);
      add_element(acc, vc[k].z, vo[k].z, va[k].z, c);
      add_element(acc, vc[k].w, vo[k].w, va[k].w, c);
      if (kEnt) {
        acc.ent = __fadd_rn(acc.ent, ve[k].x);
        acc.ent = __fadd_rn(acc.ent, ve[k].y);
        acc.ent = __fadd_rn(acc.ent, ve[k].z);
        acc.ent = __fadd_rn(acc.ent, ve[k].w);
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

// Fixed-order CTA reduction of the per-thread accumulators into one chunk partial (thread 0).
__device__ __forceinline__ Partial cta_reduce(const Acc& acc) {
  __shared__ double s_d[5][kThreads / 32];
  __shared__ float s_max[kThreads / 32];
  __shared__ unsigned s_cnt[kThreads / 32];
  double v[5] = {double(acc.gain) + acc.big_gain, double(acc.kl) + acc.big_kl, double(acc.r) + acc.big_r,
                 double(acc.r2) + acc.big_r2, double(acc.ent)};
#pragma unroll
  for (int q = 0; q < 5; ++q) v[q] = warp_sum(v[q]);
  const float m = warp_max(acc.rmax);
  const unsigned cnt = warp_sum_u32(acc.clipped);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
#pragma unroll
    for (int q = 0; q < 5; ++q) s_d[q][w] = v[q];
    s_max[w] = m;
    s_cnt[w] = cnt;
  }
  __syncthreads();
  Partial p{};
  if (threadIdx.x == 0) {
    p.gain = p.kl = p.r = p.r2 = p.ent = 0.0;
    p.rmax = 0.f;
    p.clipped = 0;
#pragma unroll
    for (int i = 0; i < kThreads / 32; ++i) {
      p.gain += s_d[0][i];
      p.kl += s_d[1][i];
      p.r += s_d[2][i];
      p.r2 += s_d[3][i];
      p.ent += s_d[4][i];
      p.rmax = fmaxf(p.rmax, s_max[i]);
      p.clipped += s_cnt[i];
    }
  }
  __syncthreads();
  return p;
}

// Final combination of partials[0..n_parts) in a fixed order; writes 6 (or 7) outputs.
// Every ratio is > 0, so 0 is the identity of the max.
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
  __syncthreads();
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
    out[2] = float(t[1] / N);
    out[3] = float((t[2] / N) * (t[2] / t[3]));
    out[4] = n_total > 0 ? mx : __int_as_float(0x7fc00000);
    out[5] = float(t[2] / N);
    if (ext) out[6] = float(t[4] / N);
  }
}

template <bool kVec, bool kEnt, bool kFinish>
__global__ void __launch_bounds__(kThreads) chunk_kernel(const float* __restrict__ cur, const float* __restrict__ old,
                                                         const float* __restrict__ adv, const float* __restrict__ ent,
                                                         int64_t n, Clip clip, Partial* __restrict__ partials,
                                                         unsigned* __restrict__ ticket, float* __restrict__ out) {
  const int64_t n_chunks = (n + kChunk - 1) / kChunk;
  for (int64_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    Acc acc;
    thread_chunk<kVec, kEnt>(acc, cur, old, adv, ent, c * kChunk, n, clip);
    const Partial p = cta_reduce(acc);
    if (threadIdx.x == 0) partials[c] = p;
  }
  if (kFinish) {
    if (elect_last_cta(ticket)) finish(partials, n_chunks, n, kEnt, out);
  }
}

__global__ void __launch_bounds__(kThreads) finish_kernel(const Partial* __restrict__ partials, int64_t n_parts,
                                                          int64_t n_total, int ext, float* __restrict__ out) {
  finish(partials, n_parts, n_total, ext != 0, out);
}

template <bool kVec, bool kEnt, bool kFinish>
inline void launch_one(const float* cur, const float* old, const float* adv, const float* ent, int64_t n,
                       const Clip& clip, Partial* partials, unsigned* ticket, float* out, cudaStream_t stream) {
  auto kern = chunk_kernel<kVec, kEnt, kFinish>;
  const int grid = balanced_grid(num_chunks(n), resident_ctas_per_sm(kern, kThreads, 0));
  kern<<<grid, kThreads, 0, stream>>>(cur, old, adv, ent, n, clip, partials, ticket, out);
}

template <bool kFinish>
inline void launch_chunks(const float* cur, const float* old, const float* adv, const float* ent, int64_t n,
                          const Clip& clip, Partial* partials, unsigned* ticket, float* out, cudaStream_t stream) {
  const bool vec = aligned16(cur) && aligned16(old) && aligned16(adv) && (ent == nullptr || aligned16(ent));
  if (ent != nullptr) {
    if (vec) launch_one<true, true, kFinish>(cur, old, adv, ent, n, clip, partials, ticket, out, stream);
    else launch_one<false, true, kFinish>(cur, old, adv, ent, n, clip, partials, ticket, out, stream);
  } else {
    if (vec) launch_one<true, false, kFinish>(cur, old, adv, ent, n, clip, partials, ticket, out, stream);
    else launch_one<false, false, kFinish>(cur, old, adv, ent, n, clip, partials, ticket, out, stream);
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
