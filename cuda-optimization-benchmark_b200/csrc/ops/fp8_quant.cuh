// Per-tensor max-abs E4M3 quantisation: the step that feeds fp8_linear its operands.
//
// Reference semantics: tasks/fp8_linear/reference.py:15-18 (`_quantize`):
//   amax  = max |x| (fp32), taken as at least 1e-9;
//   scale = fp32(448 / amax), the division in fp64;
//   q     = e4m3fn(clamp(fp32(x * scale), -448, 448)), rounded to nearest even; NaN stays NaN.
// BASELINE.json's fp8 configuration quantises bf16 sources; a bf16 value widens to fp32 exactly, so
// both source types share the arithmetic.  The E4M3 byte of a NaN is 0x7F with the input's sign,
// as torch's float8_e4m3fn conversion makes it; every other value goes through the hardware
// round-to-nearest-even converter.
//
// B200 design: two HBM passes, both grid-stride over 16-element groups (one 16-byte store of 16
// E4M3 bytes per group), four groups in flight per thread.  amax_kernel: per-thread max of |x| and
// a NaN flag, one partial per CTA, the last CTA to finish combines the partials (max is order-free,
// so the result is exact) and writes scale (and, for the fused linear layer, the GEMM epilogue
// factor) to device memory.
// cast_kernel waits for it through programmatic dependent launch and writes the bytes, walking the
// groups in the reverse of amax_kernel's order so that the part of x still in L2 after the amax
// pass is read first.  Traffic: 2 reads of x (less what the second finds in L2) and 1 byte written
// per element.
#pragma once

#include <cuda_fp8.h>
#include <math.h>
#include <stdint.h>

#include "../common/b200_common.cuh"
#include "../common/workspace.cuh"

namespace b200 {
namespace fp8q {

constexpr int kThreads = 256;
constexpr int kGroup = 16;       // elements per group (16 bytes of output)
constexpr int kMaxGrid = 1024;   // amax partials
constexpr int kUnroll = 4;       // groups in flight per thread
constexpr float kE4M3Max = 448.0f;

// Workspace: a 256-byte header (completion ticket, scale, epilogue factor), then kMaxGrid partials.
struct Header {
  unsigned ticket;
  float scale;
  float epi;
};
inline size_t workspace_bytes() { return 256 + size_t(kMaxGrid) * sizeof(float); }

template <bool kBf16>
__device__ __forceinline__ float load1(const void* x, int64_t i) {
  if (kBf16) return __uint_as_float(uint32_t(__ldg(static_cast<const uint16_t*>(x) + i)) << 16);
  return __ldg(static_cast<const float*>(x) + i);
}

// The 16 values of group g (16-byte aligned source).
template <bool kBf16>
__device__ __forceinline__ void load16(const void* x, int64_t g, float (&v)[kGroup]) {
  if (kBf16) {
    const uint4* p = static_cast<const uint4*>(x) + 2 * g;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 u = __ldg(p + h);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[8 * h + 2 * j] = __uint_as_float(w[j] << 16);
        v[8 * h + 2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
      }
    }
  } else {
    const float4* p = static_cast<const float4*>(x) + 4 * g;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float4 f = ld_stream_f4(reinterpret_cast<const float*>(p + h));
      v[4 * h] = f.x;
      v[4 * h + 1] = f.y;
      v[4 * h + 2] = f.z;
      v[4 * h + 3] = f.w;
    }
  }
}

__device__ __forceinline__ float scale_clamp(float x, float scale) {
  const float v = __fmul_rn(x, scale);
  return v > kE4M3Max ? kE4M3Max : (v < -kE4M3Max ? -kE4M3Max : v);  // NaN passes through
}

// E4M3 byte of a NaN: 0x7F with its sign.
__device__ __forceinline__ uint32_t nan_byte(float v) { return 0x7Fu | ((__float_as_uint(v) >> 24) & 0x80u); }

__device__ __forceinline__ uint8_t to_e4m3(float x, float scale) {
  const float v = scale_clamp(x, scale);
  if (isnan(v)) return uint8_t(nan_byte(v));
  return uint8_t(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

// Four values to four E4M3 bytes (little-endian in the word), two per hardware conversion.
__device__ __forceinline__ uint32_t to_e4m3x4(float a, float b, float c, float d, float scale) {
  const float v[4] = {scale_clamp(a, scale), scale_clamp(b, scale), scale_clamp(c, scale), scale_clamp(d, scale)};
  uint32_t w = uint32_t(__nv_cvt_float2_to_fp8x2(make_float2(v[0], v[1]), __NV_SATFINITE, __NV_E4M3)) |
               (uint32_t(__nv_cvt_float2_to_fp8x2(make_float2(v[2], v[3]), __NV_SATFINITE, __NV_E4M3)) << 16);
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (isnan(v[k])) w = (w & ~(0xFFu << (8 * k))) | (nan_byte(v[k]) << (8 * k));
  return w;
}

template <bool kBf16, bool kVec>
__global__ void __launch_bounds__(kThreads) amax_kernel(const void* __restrict__ x, int64_t n,
                                                        float* __restrict__ partials, Header* __restrict__ hdr,
                                                        float scale_w, float* __restrict__ scale_out) {
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  __shared__ float s_m[kThreads / 32];
  __shared__ unsigned s_nan[kThreads / 32];
  float m = 0.f;
  unsigned nan = 0;
  const int64_t stride = int64_t(gridDim.x) * kThreads, t0 = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t groups = kVec ? n / kGroup : 0;
  int64_t g = t0;
  for (; g + (kUnroll - 1) * stride < groups; g += kUnroll * stride) {  // kUnroll groups in flight
    float v[kUnroll][kGroup];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) load16<kBf16>(x, g + u * stride, v[u]);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
#pragma unroll
      for (int j = 0; j < kGroup; ++j) {
        m = fmaxf(m, fabsf(v[u][j]));
        nan |= isnan(v[u][j]) ? 1u : 0u;
      }
  }
  for (; g < groups; g += stride) {
    float v[kGroup];
    load16<kBf16>(x, g, v);
#pragma unroll
    for (int j = 0; j < kGroup; ++j) {
      m = fmaxf(m, fabsf(v[j]));
      nan |= isnan(v[j]) ? 1u : 0u;
    }
  }
  for (int64_t i = groups * kGroup + t0; i < n; i += stride) {
    const float v = load1<kBf16>(x, i);
    m = fmaxf(m, fabsf(v));
    nan |= isnan(v) ? 1u : 0u;
  }
  m = warp_max(m);
  nan = __reduce_or_sync(0xffffffffu, nan);
  if ((threadIdx.x & 31) == 0) {
    s_m[threadIdx.x >> 5] = m;
    s_nan[threadIdx.x >> 5] = nan;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float bm = 0.f;
    unsigned bn = 0;
    for (int w = 0; w < kThreads / 32; ++w) {
      bm = fmaxf(bm, s_m[w]);
      bn |= s_nan[w];
    }
    partials[blockIdx.x] = bn ? __int_as_float(0x7fc00000) : bm;
  }
  if (!elect_last_cta(&hdr->ticket)) return;
  // The last CTA combines the partials, all its threads in parallel (one L2 round trip).
  float pm = 0.f;
  unsigned pn = 0;
  for (unsigned b = threadIdx.x; b < gridDim.x; b += kThreads) {
    const float p = __ldcg(partials + b);
    pn |= isnan(p) ? 1u : 0u;
    pm = fmaxf(pm, p);
  }
  pm = warp_max(pm);
  pn = __reduce_or_sync(0xffffffffu, pn);
  __syncthreads();  // s_m / s_nan are reused
  if ((threadIdx.x & 31) == 0) {
    s_m[threadIdx.x >> 5] = pm;
    s_nan[threadIdx.x >> 5] = pn;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float amax = 0.f;
    bool any_nan = false;
    for (int w = 0; w < kThreads / 32; ++w) {
      amax = fmaxf(amax, s_m[w]);
      any_nan |= s_nan[w] != 0u;
    }
    // scale = fp32(448 / max(amax, 1e-9)) with the division in fp64; NaN when x holds a NaN.
    const double a = double(amax) > 1e-9 ? double(amax) : 1e-9;
    const float scale = any_nan ? __int_as_float(0x7fc00000) : float(448.0 / a);
    hdr->scale = scale;
    // Epilogue factor of the fused linear layer: 1 / (scale_x * scale_w) in fp64, as fp8_linear
    // computes it on the host for given scales.
    hdr->epi = float(1.0 / (double(scale) * double(scale_w)));
    if (scale_out != nullptr) *scale_out = scale;
  }
}

template <bool kBf16, bool kVec>
__global__ void __launch_bounds__(kThreads) cast_kernel(const void* __restrict__ x, int64_t n,
                                                        const Header* __restrict__ hdr, uint8_t* __restrict__ q) {
  pdl_begin();  // the scale is written by the amax kernel just before this one
  const float scale = hdr->scale;
  const int64_t stride = int64_t(gridDim.x) * kThreads, t0 = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  const int64_t groups = kVec ? n / kGroup : 0;
  auto put = [&](int64_t gi, const float (&v)[kGroup]) {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = to_e4m3x4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3], scale);
    *reinterpret_cast<uint4*>(q + gi * kGroup) = make_uint4(w[0], w[1], w[2], w[3]);
  };
  // Groups in reverse order (group groups-1-g at step g): the amax pass read x front to back, so
  // its last-read lines, still in L2, are the first ones read here.
  int64_t g = t0;
  for (; g + (kUnroll - 1) * stride < groups; g += kUnroll * stride) {  // kUnroll groups in flight
    float v[kUnroll][kGroup];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) load16<kBf16>(x, groups - 1 - (g + u * stride), v[u]);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) put(groups - 1 - (g + u * stride), v[u]);
  }
  for (; g < groups; g += stride) {
    float v[kGroup];
    load16<kBf16>(x, groups - 1 - g, v);
    put(groups - 1 - g, v);
  }
  for (int64_t i = groups * kGroup + t0; i < n; i += stride) q[i] = to_e4m3(load1<kBf16>(x, i), scale);
}

inline int grid_for(int64_t n) {
  const int64_t want = (n / kGroup + kThreads - 1) / kThreads;
  const int64_t cap = int64_t(sm_count()) * 8 < kMaxGrid ? int64_t(sm_count()) * 8 : kMaxGrid;
  return int(want < 1 ? 1 : (want < cap ? want : cap));
}

template <bool kBf16, bool kVec>
inline int launch(const void* x, int64_t n, uint8_t* q, float scale_w, float* scale_out, void* ws,
                  cudaStream_t stream) {
  Header* hdr = static_cast<Header*>(ws);
  float* partials = reinterpret_cast<float*>(static_cast<char*>(ws) + 256);
  const int grid = grid_for(n);
  if (launch_pdl(amax_kernel<kBf16, kVec>, grid, kThreads, 0, stream, x, n, partials, hdr, scale_w, scale_out) !=
      kOk)
    return kCudaError;
  if (q == nullptr) return kOk;
  return launch_pdl(cast_kernel<kBf16, kVec>, grid, kThreads, 0, stream, x, n, static_cast<const Header*>(hdr), q);
}

// x: n values of fp32 (bf16 == false) or bf16; q: n bytes (may be null: amax and scale only);
// scale_out: one device float (may be null).  workspace: workspace_bytes(), its first 4 bytes zero
// before the first call (left zero).  scale_w only shapes the epilogue factor kept in the
// workspace header for fp8_linear (1 when unused).
inline int run(const void* x, bool bf16, int64_t n, uint8_t* q, float* scale_out, float scale_w, void* workspace,
               size_t ws_bytes, cudaStream_t stream) {
  if (n < 0 || (n > 0 && x == nullptr)) return kInvalidArgument;
  if (workspace == nullptr || ws_bytes < workspace_bytes()) return kWorkspaceTooSmall;
  const bool vec = aligned16(x) && (q == nullptr || aligned16(q));
  if (bf16) return vec ? launch<true, true>(x, n, q, scale_w, scale_out, workspace, stream)
                       : launch<true, false>(x, n, q, scale_w, scale_out, workspace, stream);
  return vec ? launch<false, true>(x, n, q, scale_w, scale_out, workspace, stream)
             : launch<false, false>(x, n, q, scale_w, scale_out, workspace, stream);
}

}  // namespace fp8q
}  // namespace b200
