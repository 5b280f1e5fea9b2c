// KAN linear layer (efficient-kan KANLinear forward):
//   out[b, o] = sum_i silu(x[b,i]) * W_base[o,i] + sum_i sum_c basis_c(x[b,i]) * sw[o,i,c] * scaler[o,i]
// with the C = G + K cubic (order K) B-spline bases of x on each input's knot grid (Cox-de Boor).
//
// Reference semantics: tasks/efficient_kan/reference.py:33-46 (fp64 oracle :54-57), tolerance
// 1e-5/1e-5 (tasks/efficient_kan/tests/task.json).  The drop-in boundary it replaces is
// `void reference(const float* x, const float* grid, const float* base_weight, const float*
// spline_weight, const float* spline_scaler, int32_t grid_size, int32_t spline_order, int32_t B,
// int32_t I, int32_t O, float* out)` (task.json:3; expert launcher
// reference/efficient_kan/solution.cu:177-288, which builds A and W and calls cuBLAS).
//
// B200 design.  The op is one GEMM out = A . W'^T over K' = I*(1+C): A[b, p*I + i] holds silu(x)
// (p = 0) and basis p-1 (p >= 1), W'[o, p*I + i] holds W_base (p = 0) and sw*scaler (p >= 1).
// The 1e-5 tolerance against fp64 rules out a single fp16/bf16/tf32 pass, so every operand value
// v is split into fp16 v_hi = fp16(v) and v_lo = fp16((v - v_hi) * 2^11) (22 significant bits
// together), and the tensor cores form
//   D0 = A_hi . W_hi^T      D1 = A_hi . W_lo^T + A_lo . W_hi^T      out = D0 + D1 * 2^-11
// in fp32 TMEM accumulators (the dropped A_lo . W_lo term is 2^-22 relative).  The tensor cores'
// fp32 accumulation is not round-to-nearest, so its error grows with the number of chained MMAs;
// D0 is therefore spread round-robin by k-block over three accumulators (a third of the chain
// each) and summed in the epilogue, which keeps K' = 9216 well inside 1e-5.  Rows of A and of W'
// are scaled by powers of two so every value fits fp16; the epilogue undoes them.
//   1. prep_wr_kernel: W' hi/lo planes (one CTA per output row), in the same launch the row scales
//      of the cubic cases (row_scale_rows);
//   2. silu + Cox-de Boor bases of x in fp32, hi/lo planes: for the cubic cases
//      prep_a3_kernel (a thread per two inputs down a block of rows, only the four non-zero bases
//      of each input formed), otherwise prep_a_kernel (one CTA per batch row);
//   3. gemm_kernel: persistent warp-specialised tcgen05 GEMM (kind::f16, 128 x 128 tiles, TMEM
//      = [D0a | D0b | D0c | D1], 128-byte-swizzled TMA loads of the four planes in a 3-stage ring,
//      12 MMAs per stage), fused combine/rescale epilogue writing fp32 rows.
// Planes are K-padded to a multiple of 64 with zeros so every TMA row pitch is 16-byte aligned.
#pragma once

#include <cuda_fp16.h>
#include <math.h>

#include "../common/b200_common.cuh"
#include "../common/bulk.cuh"
#include "../common/tcgen05.cuh"
#include "../common/workspace.cuh"

namespace b200 {
namespace kan {

constexpr int kMaxKnots = 64;  // G + 2K + 1 knots per input at most
constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kBKe = 64;       // fp16 elements of K per stage (one 128-byte swizzle row)
constexpr int kUmmaK = 16;     // K per tcgen05.mma for 16-bit operands
constexpr int kThreads = 320;  // warp 0 loads, warp 1 issues MMAs, warps 2-9 epilogue
constexpr int kGroupM = 8;
constexpr float kLoScale = 2048.0f;      // 2^11
constexpr float kLoUnscale = 1.0f / 2048.0f;
constexpr float kFp16Safe = 16384.0f;    // rows are scaled so |value| < 2^14

constexpr int kATile = kBM * kBKe * 2;   // 16 KB per A plane per stage
constexpr int kWTile = kBN * kBKe * 2;   // 16 KB per W plane per stage
constexpr int kStage = 2 * kATile + 2 * kWTile;  // 64 KB
constexpr int kStages = 3;
constexpr int kSmem = kStages * kStage + 1024;
constexpr int kD0Parts = 3;               // D0 accumulators (k-block round-robin)
constexpr int kTmemCols = 4 * kBN;       // D0a, D0b, D0c, D1

inline int64_t padded_k(int I, int C) { return (int64_t(I) * (1 + C) + kBKe - 1) / kBKe * kBKe; }

// Workspace layout (all 256-byte aligned): A_hi, A_lo [B][Kp] fp16; W_hi, W_lo [O][Kp] fp16;
// row scales rs[B], col scales cs[O] (fp32 powers of two).
struct Layout {
  size_t a_hi, a_lo, w_hi, w_lo, rs, cs, part, cnt, total;
};

// The GEMM's last, partial round of tiles is split in two K halves when that evens out the CTAs'
// work (split_tiles); each half leaves a 128 x 128 fp32 partial tile, and one counter per
// (split tile, epilogue warp) tells the second half to add the first's.
constexpr int kEpiWarps = 8;
inline int max_split_tiles() { return sm_count() / 2; }

inline Layout layout(int B, int I, int O, int C) {
  const int64_t kp = padded_k(I, C);
  Layout L;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += align256(bytes);
    return at;
  };
  L.a_hi = take(size_t(B) * kp * 2);
  L.a_lo = take(size_t(B) * kp * 2);
  L.w_hi = take(size_t(O) * kp * 2);
  L.w_lo = take(size_t(O) * kp * 2);
  L.rs = take(size_t(B) * 4);
  L.cs = take(size_t(O) * 4);
  L.part = take(size_t(2) * max_split_tiles() * kBM * kBN * 4);
  L.cnt = take(size_t(max_split_tiles()) * kEpiWarps * 4);
  L.total = off;
  return L;
}

// Power-of-two factor f (f <= 1) with amax * f < 2^14.
__device__ __forceinline__ float fp16_row_factor(float amax) {
  float f = 1.0f;
  while (amax * f >= kFp16Safe && f > 1e-30f) f *= 0.5f;
  return f;
}

__device__ __forceinline__ void split_store(float v, __half* hi, __half* lo) {
  const __half h = __float2half_rn(v);
  *hi = h;
  *lo = __float2half_rn((v - __half2float(h)) * kLoScale);
}

__device__ __forceinline__ float block_max(float v, float* s_red) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float m = threadIdx.x < (blockDim.x >> 5) ? s_red[threadIdx.x] : 0.0f;
    m = warp_max(m);
    if (threadIdx.x == 0) s_red[32] = m;
  }
  __syncthreads();
  const float r = s_red[32];
  __syncthreads();
  return r;
}

// ---------------------------------------------------------------------------------- W' planes
// One CTA per output row o, one thread per input i at a time (input-major, so each thread reads
// its C contiguous spline weights and the warp's reads are contiguous).  w'(p=0, i) = W_base[o,i];
// w'(p=1+c, i) = sw[o,i,c] * scaler[o,i] (the fp32 product the reference forms,
// tasks/efficient_kan/reference.py:45).  Pass 1 finds the row's max |w'|, pass 2 writes the planes.
__device__ __forceinline__ void prep_w_row(int o, const float* __restrict__ wb, const float* __restrict__ sw,
                                           const float* __restrict__ sc, int I, int C, int64_t kp,
                                           __half* __restrict__ w_hi, __half* __restrict__ w_lo,
                                           float* __restrict__ cs, float* s_red) {
  const float* wbr = wb + int64_t(o) * I;
  const float* swr = sw + int64_t(o) * I * C;
  const float* scr = sc + int64_t(o) * I;
  float amax = 0.0f;
  for (int i = threadIdx.x; i < I; i += blockDim.x) {
    amax = fmaxf(amax, fabsf(__ldg(wbr + i)));
    const float sv = __ldg(scr + i);
    for (int c = 0; c < C; ++c) amax = fmaxf(amax, fabsf(__fmul_rn(__ldg(swr + int64_t(i) * C + c), sv)));
  }
  const float f = fp16_row_factor(block_max(amax, s_red));
  if (threadIdx.x == 0) cs[o] = 1.0f / f;
  __half* hr = w_hi + int64_t(o) * kp;
  __half* lr = w_lo + int64_t(o) * kp;
  for (int i = threadIdx.x; i < I; i += blockDim.x) {
    split_store(__ldg(wbr + i) * f, hr + i, lr + i);
    const float sv = __ldg(scr + i);
    for (int c = 0; c < C; ++c)
      split_store(__fmul_rn(__ldg(swr + int64_t(i) * C + c), sv) * f, hr + int64_t(1 + c) * I + i,
                  lr + int64_t(1 + c) * I + i);
  }
  const int64_t kk = int64_t(I) * (1 + C);
  for (int64_t q = kk + threadIdx.x; q < kp; q += blockDim.x) {
    hr[q] = __float2half_rn(0.0f);
    lr[q] = __float2half_rn(0.0f);
  }
}

// -------------------------------------------------------------------------------- A planes
// silu(x) and the C bases of x on knots g[0..nk) (nk = G + 2K + 1) by the Cox-de Boor recurrence
// of tasks/efficient_kan/reference.py:33-39: order-0 indicators g[j] <= x < g[j+1], then K rounds
// b[j] = (x - g[j]) / (g[j+k] - g[j]) * b[j] + (g[j+k+1] - x) / (g[j+k+1] - g[j+1]) * b[j+1].
__device__ __forceinline__ void bases_of(float x, const float* g, int nk, int K, float* b) {
  for (int j = 0; j < nk - 1; ++j) b[j] = (x >= g[j] && x < g[j + 1]) ? 1.0f : 0.0f;
  for (int k = 1; k <= K; ++k) {
    for (int j = 0; j < nk - 1 - k; ++j) {
      const float l = __fdiv_rn(__fsub_rn(x, g[j]), __fsub_rn(g[j + k], g[j]));
      const float r = __fdiv_rn(__fsub_rn(g[j + k + 1], x), __fsub_rn(g[j + k + 1], g[j + 1]));
      b[j] = __fadd_rn(__fmul_rn(l, b[j]), __fmul_rn(r, b[j + 1]));
    }
  }
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// Same recurrence with the knot count NK and order KO known at compile time: fully unrolled, the
// knot and basis arrays stay in registers.
template <int NK, int KO>
__device__ __forceinline__ void bases_fixed(float x, const float* __restrict__ gsrc, float* b) {
  float g[NK];
#pragma unroll
  for (int j = 0; j < NK; ++j) g[j] = __ldg(gsrc + j);
#pragma unroll
  for (int j = 0; j < NK - 1; ++j) b[j] = (x >= g[j] && x < g[j + 1]) ? 1.0f : 0.0f;
#pragma unroll
  for (int k = 1; k <= KO; ++k) {
#pragma unroll
    for (int j = 0; j < NK - 1 - k; ++j) {
      const float l = __fdiv_rn(__fsub_rn(x, g[j]), __fsub_rn(g[j + k], g[j]));
      const float r = __fdiv_rn(__fsub_rn(g[j + k + 1], x), __fsub_rn(g[j + k + 1], g[j + 1]));
      b[j] = __fadd_rn(__fmul_rn(l, b[j]), __fmul_rn(r, b[j + 1]));
    }
  }
}

// Only the non-zero bases, for strictly increasing knots g[0..NK): if g[j0] <= x < g[j0+1], the
// order-k bases that can be non-zero are j0-k .. j0, and each is formed by the same two-term
// expression as in the full recurrence (the terms skipped are exact zeros), so the values equal
// the full recurrence's.  out[0..NK-KO-1) receives every order-KO basis (zero outside j0-KO..j0).
// Returns false (out untouched) when the knots are not strictly increasing.
template <int NK, int KO>
__device__ __forceinline__ bool bases_local(float x, const float* __restrict__ gsrc, float* out) {
  constexpr int C = NK - KO - 1;
  float g[NK];
#pragma unroll
  for (int j = 0; j < NK; ++j) g[j] = __ldg(gsrc + j);
  bool inc = true;
  int j0 = -1;
#pragma unroll
  for (int j = 0; j < NK - 1; ++j) {
    inc = inc && (g[j] < g[j + 1]);
    if (x >= g[j] && x < g[j + 1]) j0 = j;
  }
  if (!inc) return false;
#pragma unroll
  for (int c = 0; c < C; ++c) out[c] = 0.0f;
  if (j0 < 0) return true;
  float nb[KO + 1];  // nb[m]: basis j0-k+m of the current order k
  nb[0] = 1.0f;
#pragma unroll
  for (int k = 1; k <= KO; ++k) {
    float nn[KO + 1];
#pragma unroll
    for (int m = 0; m <= k; ++m) {
      const int j = j0 - k + m;
      float v = 0.0f;
      if (j >= 0 && j <= NK - 2 - k) {
        // b_k[j] = L * b_{k-1}[j] + R * b_{k-1}[j+1]; b_{k-1}[j] is nb[m-1], b_{k-1}[j+1] is nb[m].
        const float lt = m >= 1 ? __fmul_rn(__fdiv_rn(__fsub_rn(x, g[j]), __fsub_rn(g[j + k], g[j])), nb[m - 1])
                                : 0.0f;
        const float rt = m <= k - 1 ? __fmul_rn(__fdiv_rn(__fsub_rn(g[j + k + 1], x), __fsub_rn(g[j + k + 1], g[j + 1])),
                                                nb[m])
                                    : 0.0f;
        v = __fadd_rn(lt, rt);
      }
      nn[m] = v;
    }
#pragma unroll
    for (int m = 0; m <= k; ++m) nb[m] = nn[m];
  }
#pragma unroll
  for (int m = 0; m <= KO; ++m) {
    const int j = j0 - KO + m;
#pragma unroll
    for (int c = 0; c < C; ++c)
      if (c == j) out[c] = nb[m];
  }
  return true;
}

// One CTA per batch row b; the knots of input i are grid[i*nk .. i*nk + nk).  NK/KO > 0 select the
// unrolled form for that (knot count, order); 0 selects the general loop.
template <int NK, int KO>
__global__ void __launch_bounds__(256) prep_a_kernel(const float* __restrict__ x, const float* __restrict__ grid,
                                                     int I, int C, int K, int64_t kp, __half* __restrict__ a_hi,
                                                     __half* __restrict__ a_lo, float* __restrict__ rs) {
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  __shared__ float s_red[33];
  const int bi = blockIdx.x;
  const int nk = NK > 0 ? NK : C + K + 1;
  const int nc = NK > 0 ? NK - KO - 1 : C;
  const float* xr = x + int64_t(bi) * I;
  float amax = 0.0f;
  for (int i = threadIdx.x; i < I; i += blockDim.x) amax = fmaxf(amax, fabsf(silu(xr[i])));
  // B-spline bases on a non-decreasing grid lie in [0, 1].
  const float f = fp16_row_factor(fmaxf(block_max(amax, s_red), 1.0f));
  if (threadIdx.x == 0) rs[bi] = 1.0f / f;
  __half* hr = a_hi + int64_t(bi) * kp;
  __half* lr = a_lo + int64_t(bi) * kp;
  for (int i = threadIdx.x; i < I; i += blockDim.x) {
    const float xv = xr[i];
    split_store(silu(xv) * f, hr + i, lr + i);
    if (NK > 0) {
      float b[NK > 0 ? NK : 1];
      if (!bases_local<(NK > 0 ? NK : 2), KO>(xv, grid + int64_t(i) * nk, b))
        bases_fixed<(NK > 0 ? NK : 2), KO>(xv, grid + int64_t(i) * nk, b);
#pragma unroll
      for (int c = 0; c < (NK > 0 ? NK - KO - 1 : 1); ++c)
        split_store(b[c] * f, hr + int64_t(1 + c) * I + i, lr + int64_t(1 + c) * I + i);
    } else {
      float g[kMaxKnots], b[kMaxKnots];
      for (int j = 0; j < nk; ++j) g[j] = grid[int64_t(i) * nk + j];
      bases_of(xv, g, nk, K, b);
      for (int c = 0; c < nc; ++c) split_store(b[c] * f, hr + int64_t(1 + c) * I + i, lr + int64_t(1 + c) * I + i);
    }
  }
  const int64_t kk = int64_t(I) * (1 + C);
  for (int64_t q = kk + threadIdx.x; q < kp; q += blockDim.x) {
    hr[q] = __float2half_rn(0.0f);
    lr[q] = __float2half_rn(0.0f);
  }
}

// ----------------------------------------------------------------- A planes, column-major form
// prep_a_kernel gives each batch row to one CTA.  For the cubic cases the column-major form instead
// gives each thread two adjacent inputs down a block of rows (prep_a3_kernel below), after
//   row_scale_rows: per row the power-of-two factor that keeps silu and the bases inside fp16
//     (the same rule as prep_a_kernel), and the row's zero K padding.

// One warp per row.  The amax takes silu with fast intrinsics: the factor is a power of two chosen
// with a 4x margin below the fp16 maximum (kFp16Safe), so an amax a few ulps low can at most double
// the factor and every scaled value still fits fp16.
constexpr int kScaleRowsPerCta = 8;
__device__ __forceinline__ void row_scale_rows(int blk, const float* __restrict__ x, int B, int I, int C, int64_t kp,
                                               float* __restrict__ rs, __half* __restrict__ a_hi,
                                               __half* __restrict__ a_lo) {
  const int lane = threadIdx.x & 31;
  const int bi = blk * kScaleRowsPerCta + int(threadIdx.x >> 5);
  if (bi >= B) return;
  const float* xr = x + int64_t(bi) * I;
  float amax = 0.0f;
  auto silu_fast = [](float v) { return __fdividef(v, 1.0f + __expf(-v)); };
  if ((I & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
    for (int q = lane; q < I / 4; q += 32) {
      const float4 v = ld_stream_f4(xr + 4 * q);
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(silu_fast(v.x)), fabsf(silu_fast(v.y))),
                               fmaxf(fabsf(silu_fast(v.z)), fabsf(silu_fast(v.w)))));
    }
  } else {
    for (int i = lane; i < I; i += 32) amax = fmaxf(amax, fabsf(silu_fast(xr[i])));
  }
  amax = warp_max(amax);
  // B-spline bases on a non-decreasing grid lie in [0, 1].
  const float f = fp16_row_factor(fmaxf(amax, 1.0f));
  if (lane == 0) rs[bi] = 1.0f / f;
  const int64_t kk = int64_t(I) * (1 + C);
  for (int64_t q = kk + lane; q < kp; q += 32) {
    a_hi[int64_t(bi) * kp + q] = __float2half_rn(0.0f);
    a_lo[int64_t(bi) * kp + q] = __float2half_rn(0.0f);
  }
}

// The W' planes and, for the column-major A path, the row scales in one launch (the two are
// independent): CTAs [0, O) each prepare one output row of W', the scale_ctas CTAs after them
// kScaleRowsPerCta batch rows' scales each.
constexpr int kPrepThreads = 256;
static_assert(kPrepThreads == 32 * kScaleRowsPerCta, "a row-scale CTA is one warp per row");
__global__ void __launch_bounds__(kPrepThreads) prep_wr_kernel(const float* __restrict__ wb,
                                                               const float* __restrict__ sw,
                                                               const float* __restrict__ sc, int I, int O, int C,
                                                               int64_t kp, __half* __restrict__ w_hi,
                                                               __half* __restrict__ w_lo, float* __restrict__ cs,
                                                               const float* __restrict__ x, int B,
                                                               float* __restrict__ rs, __half* __restrict__ a_hi,
                                                               __half* __restrict__ a_lo, unsigned* __restrict__ cnt,
                                                               int n_cnt) {
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  __shared__ float s_red[33];
  if (blockIdx.x == 0)  // the GEMM's split-tile counters start each call at zero
    for (int q = threadIdx.x; q < n_cnt; q += blockDim.x) cnt[q] = 0u;
  if (int(blockIdx.x) < O) prep_w_row(int(blockIdx.x), wb, sw, sc, I, C, kp, w_hi, w_lo, cs, s_red);
  else row_scale_rows(int(blockIdx.x) - O, x, B, I, C, kp, rs, a_hi, a_lo);
}

__device__ __forceinline__ void split_store2(float v0, float v1, __half* hi, __half* lo) {
  const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
  *reinterpret_cast<__half2*>(hi) = __halves2half2(h0, h1);
  *reinterpret_cast<__half2*>(lo) = __halves2half2(__float2half_rn((v0 - __half2float(h0)) * kLoScale),
                                                   __float2half_rn((v1 - __half2float(h1)) * kLoScale));
}

// ------------------------------------------------------------ A planes, sparse cubic form
// For strictly increasing knots and g[s] <= x < g[s+1], only the cubic bases s-3 .. s can be
// non-zero, and each is the same two-term expression as in the full recurrence with the exact-zero
// terms left out (tasks/efficient_kan/reference.py:33-39).  prep_a3_kernel forms those four from
// the six knots g[s-2 .. s+3] (9 recurrence terms instead of 36, 6 reciprocals instead of 42
// register-held ones), so a thread needs few registers and the grid can fill the SMs.  The knot
// values are bit-identical to the full recurrence's with reciprocal knot differences (the same
// reciprocals, products and sums); only the sign of a zero basis can differ.  A thread owns inputs (i, i + 1); their knots are staged in
// shared memory as s_g[j][u][t] (input i0 + 2t + u), so the dynamic knot reads of a warp hit 32
// distinct banks.  The four bases go to their planes through a per-thread shared-memory row
// (a register array cannot take the dynamic plane index), so the global stores stay one
// contiguous 128-byte half2 row per warp and plane.
// A non-finite x gives NaN bases, as the full recurrence does; a column whose knots are not
// strictly increasing takes the full recurrence (bases_fixed).
constexpr int kPrep3Threads = 128;

// Rows per CTA: the fewest that fit the whole grid in one wave of resident CTAs (a second, partial
// wave would run at a fraction of the occupancy).
inline int prep3_rows(int B, int I, int ctas_per_sm) {
  const int64_t xblocks = (I + 2 * kPrep3Threads - 1) / (2 * kPrep3Threads);
  const int64_t wave = int64_t(sm_count()) * (ctas_per_sm > 0 ? ctas_per_sm : 1);
  const int64_t row_blocks = wave / xblocks > 0 ? wave / xblocks : 1;
  return int((B + row_blocks - 1) / row_blocks);
}

__device__ __forceinline__ void split_half(float v, __half* hi, __half* lo) {
  const __half h = __float2half_rn(v);
  *hi = h;
  *lo = __float2half_rn((v - __half2float(h)) * kLoScale);
}

__device__ __forceinline__ float rcp_approx(float v) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}

// The four cubic bases s-3 .. s of x (g[s] <= x < g[s+1]) from the knots gm2..g3 = g[s-2 .. s+3]:
// the terms of the Cox-de Boor recurrence with reciprocal knot differences (hardware reciprocal,
// within an ulp of the rounded one), in its order of products and sums.
__device__ __forceinline__ void cubic_local(float x, float gm2, float gm1, float g0, float g1, float g2, float g3,
                                            float (&n)[4]) {
  const float d0 = rcp_approx(__fsub_rn(g1, g0));
  const float a1 = __fmul_rn(__fsub_rn(g1, x), d0);  // order 1, basis s-1
  const float b1 = __fmul_rn(__fsub_rn(x, g0), d0);  // order 1, basis s
  const float e1 = rcp_approx(__fsub_rn(g1, gm1)), e2 = rcp_approx(__fsub_rn(g2, g0));
  const float c0 = __fmul_rn(__fmul_rn(__fsub_rn(g1, x), e1), a1);  // order 2, basis s-2
  const float c1 = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x, gm1), e1), a1),
                             __fmul_rn(__fmul_rn(__fsub_rn(g2, x), e2), b1));
  const float c2 = __fmul_rn(__fmul_rn(__fsub_rn(x, g0), e2), b1);
  const float f1 = rcp_approx(__fsub_rn(g1, gm2)), f2 = rcp_approx(__fsub_rn(g2, gm1)),
              f3 = rcp_approx(__fsub_rn(g3, g0));
  n[0] = __fmul_rn(__fmul_rn(__fsub_rn(g1, x), f1), c0);
  n[1] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x, gm2), f1), c0), __fmul_rn(__fmul_rn(__fsub_rn(g2, x), f2), c1));
  n[2] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x, gm1), f2), c1), __fmul_rn(__fmul_rn(__fsub_rn(g3, x), f3), c2));
  n[3] = __fmul_rn(__fmul_rn(__fsub_rn(x, g0), f3), c2);
}

// grid = (ceil(I / (2 * kPrep3Threads)), ceil(B / rows)); I even, x and grid 8-byte aligned.  rs
// from prep_wr_kernel.
template <int NK>
__global__ void __launch_bounds__(kPrep3Threads, 6) prep_a3_kernel(const float* __restrict__ x,
                                                                const float* __restrict__ grid, int B, int I,
                                                                int64_t kp, const float* __restrict__ rs,
                                                                __half* __restrict__ a_hi,
                                                                __half* __restrict__ a_lo, int rows) {
  constexpr int C = NK - 4;
  static_assert(NK >= 5 && NK <= 16, "the binary search below covers up to 16 knots");
  __shared__ float s_g[NK][2][kPrep3Threads];
  __shared__ uint2 s_w[NK - 4][kPrep3Threads];  // per-thread plane words {hi half2, lo half2}
  const int t = threadIdx.x;
  const int i = 2 * (int(blockIdx.x) * kPrep3Threads + t);
  pdl_begin();  // the row scales are written by prep_wr_kernel just before this kernel
  if (i >= I) return;
  // The thread's 2 * NK knots are contiguous (grid 8-byte aligned, i even): NK float2 loads.  Only
  // this thread reads its s_g column, so no block barrier is needed.
  bool inc = true;
  {
    float gv[2 * NK];
    const float2* gp = reinterpret_cast<const float2*>(grid + int64_t(i) * NK);
#pragma unroll
    for (int e = 0; e < NK; ++e) {
      const float2 v = __ldg(gp + e);
      gv[2 * e] = v.x;
      gv[2 * e + 1] = v.y;
    }
#pragma unroll
    for (int e = 0; e < 2 * NK; ++e) {
      s_g[e % NK][e / NK][t] = gv[e];
      if (e % NK != 0) inc = inc && gv[e - 1] < gv[e];
    }
  }
  const int b0 = int(blockIdx.y) * rows;
#pragma unroll 1
  for (int bb = 0; bb < rows; ++bb) {
    const int b = b0 + bb;
    if (b >= B) break;
    const float f = 1.0f / __ldg(rs + b);  // a power of two: exact
    const float2 xv = *reinterpret_cast<const float2*>(x + int64_t(b) * I + i);
    __half* hr = a_hi + int64_t(b) * kp + i;
    __half* lr = a_lo + int64_t(b) * kp + i;
    split_store2(silu(xv.x) * f, silu(xv.y) * f, hr, lr);
    if (inc) {
      // The thread's own C plane words in shared memory (a register array cannot take the
      // dynamic plane index): zeros (NaN for a non-finite x, as the full recurrence gives), then
      // the split halves of the four non-zero bases of each input at their plane, then read back
      // for coalesced half2 plane stores.
      const float za = fabsf(xv.x) <= 3.402823466e38f ? 0.0f : __int_as_float(0x7fc00000);
      const float zb = fabsf(xv.y) <= 3.402823466e38f ? 0.0f : __int_as_float(0x7fc00000);
      const __half2 z2 = __halves2half2(__float2half_rn(za), __float2half_rn(zb));
      const uint32_t zw = *reinterpret_cast<const uint32_t*>(&z2);
#pragma unroll
      for (int c = 0; c < C; ++c) s_w[c][t] = make_uint2(zw, zw);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const float xu = u == 0 ? xv.x : xv.y;
        // cnt = #{j : g[j] <= x} by binary search (the knots increase strictly); NaN gives 0.
        int cnt = 0;
#pragma unroll
        for (int step = 8; step >= 1; step >>= 1)
          if (cnt + step <= NK && s_g[min(cnt + step - 1, NK - 1)][u][t] <= xu) cnt += step;
        if (cnt < 1 || cnt > NK - 1) continue;  // outside [g0, g[NK-1]) or NaN: zero (or NaN) bases
        const int sj = cnt - 1;
        auto kn = [&](int m) { return s_g[min(max(sj + m, 0), NK - 1)][u][t]; };
        float n[4];
        cubic_local(xu, kn(-2), kn(-1), kn(0), kn(1), kn(2), kn(3), n);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int p = sj - 3 + m;  // basis index; invalid ones (outside 0 .. C-1) use clamped knots
          if (p >= 0 && p < C) {
            const float v = n[m] * f;
            const __half h = __float2half_rn(v);
            __half* w = reinterpret_cast<__half*>(&s_w[p][t]);
            w[u] = h;
            w[2 + u] = __float2half_rn((v - __half2float(h)) * kLoScale);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const uint2 w = s_w[c][t];
        *reinterpret_cast<uint32_t*>(hr + int64_t(1 + c) * I) = w.x;
        *reinterpret_cast<uint32_t*>(lr + int64_t(1 + c) * I) = w.y;
      }
    } else {
#pragma unroll 1
      for (int u = 0; u < 2; ++u) {
        float bsv[NK - 1];
        bases_fixed<NK, 3>(u == 0 ? xv.x : xv.y, grid + int64_t(i + u) * NK, bsv);
#pragma unroll
        for (int c = 0; c < C; ++c) split_half(bsv[c] * f, hr + int64_t(1 + c) * I + u, lr + int64_t(1 + c) * I + u);
      }
    }
  }
}

// ------------------------------------------------------------------------------------- GEMM
__device__ __forceinline__ void tile_coords(int tile, int n_m, int n_n, int& mb, int& nb) {
  const int group = kGroupM * n_n;
  const int g = tile / group;
  const int first = g * kGroupM;
  const int gm = min(n_m - first, kGroupM);
  const int r = tile - g * group;
  mb = first + r % gm;
  nb = r / gm;
}

// Work unit u of the persistent schedule: tiles 0 .. n_tiles - n_split - 1 whole, then each of the
// last n_split tiles as two halves of its K blocks (units n_tiles - n_split + 2s + h).
struct Unit {
  int tile, kb0, kb1, split, half;  // split: index among the split tiles, -1 for a whole tile
};

__device__ __forceinline__ Unit unit_of(int u, int n_tiles, int n_split, int nkb) {
  const int whole = n_tiles - n_split;
  if (u < whole) return Unit{u, 0, nkb, -1, 0};
  const int v = u - whole, sp = v >> 1, h = v & 1;
  return Unit{whole + sp, h ? nkb / 2 : 0, h ? nkb : nkb / 2, sp, h};
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_alo,
                const __grid_constant__ CUtensorMap tm_whi, const __grid_constant__ CUtensorMap tm_wlo, int M, int N,
                int64_t kp, const float* __restrict__ rs, const float* __restrict__ cs, float* __restrict__ out,
                float* __restrict__ part, unsigned* __restrict__ cnt, int n_split, int vec_ok) {
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
#if !B200_TCGEN05
  if (threadIdx.x == 0) atomicOr(&g_b200_fault, kFaultNoTensorCore);
  return;
#else
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[kStages], empty[kStages], tfull, tempty;
  __shared__ uint32_t tmem_base_s;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_m = (M + kBM - 1) / kBM, n_n = (N + kBN - 1) / kBN, n_tiles = n_m * n_n;
  const int nkb = int(kp / kBKe);
  const int n_units = n_tiles + n_split;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&tfull, 1);
    mbar_init(&tempty, kEpiWarps);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tensormap(&tm_ahi);
    tc::prefetch_tensormap(&tm_alo);
    tc::prefetch_tensormap(&tm_whi);
    tc::prefetch_tensormap(&tm_wlo);
  }
  if (warp == 1) {
    tc::tmem_alloc(&tmem_base_s, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t kb_all = 0;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
        const Unit un = unit_of(u, n_tiles, n_split, nkb);
        int mb, nb;
        tile_coords(un.tile, n_m, n_n, mb, nb);
        for (int kb = un.kb0; kb < un.kb1; ++kb, ++kb_all) {
          const uint32_t s = kb_all % kStages, ph = (kb_all / kStages) & 1u;
          mbar_wait(&empty[s], ph ^ 1u);
          mbar_arrive_expect_tx(&full[s], kStage);
          uint8_t* st = smem + s * kStage;
          const int kc = kb * kBKe;
          tc::tma_load_2d(st, &tm_ahi, kc, mb * kBM, &full[s]);
          tc::tma_load_2d(st + kATile, &tm_alo, kc, mb * kBM, &full[s]);
          tc::tma_load_2d(st + 2 * kATile, &tm_whi, kc, nb * kBN, &full[s]);
          tc::tma_load_2d(st + 2 * kATile + kWTile, &tm_wlo, kc, nb * kBN, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id = tc::idesc(kBM, kBN, 0);  // F16 x F16 -> F32
      uint32_t kb_all = 0, it = 0;
      const uint32_t d1 = tmem + kD0Parts * kBN;
      for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++it) {
        const Unit un = unit_of(u, n_tiles, n_split, nkb);
        mbar_wait(&tempty, (it & 1u) ^ 1u);
        tc::fence_after_sync();
        for (int kb = un.kb0; kb < un.kb1; ++kb, ++kb_all) {
          const uint32_t s = kb_all % kStages, ph = (kb_all / kStages) & 1u;
          mbar_wait(&full[s], ph);
          tc::fence_after_sync();
          const uint32_t base = smem_addr(smem + s * kStage);
          const uint64_t ahi = tc::sdesc_kmajor_sw128(base);
          const uint64_t alo = tc::sdesc_kmajor_sw128(base + kATile);
          const uint64_t whi = tc::sdesc_kmajor_sw128(base + 2 * kATile);
          const uint64_t wlo = tc::sdesc_kmajor_sw128(base + 2 * kATile + kWTile);
          const int kr = kb - un.kb0;  // k block within the unit
          const uint32_t d0 = tmem + uint32_t(kr % kD0Parts) * kBN;
#pragma unroll
          for (int k = 0; k < kBKe / kUmmaK; ++k) {
            const uint64_t adv = uint64_t((k * kUmmaK * 2) >> 4);
            tc::mma_f16(d0, ahi + adv, whi + adv, id, (kr >= kD0Parts || k != 0) ? 1u : 0u);
            tc::mma_f16(d1, ahi + adv, wlo + adv, id, (kr | k) != 0 ? 1u : 0u);
            tc::mma_f16(d1, alo + adv, whi + adv, id, 1u);
          }
          tc::mma_commit(&empty[s]);
        }
        tc::mma_commit(&tfull);
      }
    }
  } else {  // epilogue: warp w reads TMEM lanes [32*(w%4), 32*(w%4)+32), column half (w-2)/4
    const int q = warp & 3, h = (warp - 2) >> 2;
    const uint32_t lane_off = uint32_t(q * 32) << 16;
    uint32_t it = 0;
    for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++it) {
      const Unit un = unit_of(u, n_tiles, n_split, nkb);
      int mb, nb;
      tile_coords(un.tile, n_m, n_n, mb, nb);
      mbar_wait(&tfull, it & 1u);
      tc::fence_after_sync();
      const int row = mb * kBM + q * 32 + lane;
      const float rsc = row < M ? rs[row] : 0.0f;  // vec_ok: N % 4 == 0 and out 16-byte aligned
      const int nkb_u = un.kb1 - un.kb0;
      const int parts = nkb_u < kD0Parts ? nkb_u : kD0Parts;  // D0 accumulators written this unit
      // The unscaled value D0 + D1 * 2^-11 of this lane's row, columns cc*32 .. cc*32+31.
      auto combine = [&](int cc, float (&v)[32]) {
        uint32_t a[32], c[32], t[32];
        tc::tmem_ld32(tmem + lane_off + uint32_t(cc * 32), a);
        tc::tmem_ld32(tmem + lane_off + uint32_t(kD0Parts * kBN + cc * 32), c);
        tc::tmem_ld_wait();
        for (int p = 1; p < parts; ++p) {
          tc::tmem_ld32(tmem + lane_off + uint32_t(p * kBN + cc * 32), t);
          tc::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) a[j] = __float_as_uint(__uint_as_float(a[j]) + __uint_as_float(t[j]));
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = fmaf(__uint_as_float(c[j]), kLoUnscale, __uint_as_float(a[j]));
      };
      auto store = [&](int cc, const float (&v)[32]) {
        const int n0 = nb * kBN + cc * 32;
        if (row >= M) return;
        float* o = out + int64_t(row) * N + n0;
        if (vec_ok && n0 + 32 <= N) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            float4 w;
            w.x = v[j + 0] * rsc * cs[n0 + j + 0];
            w.y = v[j + 1] * rsc * cs[n0 + j + 1];
            w.z = v[j + 2] * rsc * cs[n0 + j + 2];
            w.w = v[j + 3] * rsc * cs[n0 + j + 3];
            *reinterpret_cast<float4*>(o + j) = w;
          }
        } else {
          for (int j = 0; j < 32; ++j)
            if (n0 + j < N) o[j] = v[j] * rsc * cs[n0 + j];
        }
      };
      if (un.split < 0) {
#pragma unroll 1
        for (int cc = h * (kBN / 64); cc < (h + 1) * (kBN / 64); ++cc) {
          float v[32];
          combine(cc, v);
          store(cc, v);
        }
      } else {
        // Half of a split tile: leave this half's unscaled values in its partial tile; the half
        // that counts second adds the other's (fp32 addition commutes, so the bits do not depend
        // on which half finishes first) and writes the output.
        float* mine = part + (size_t(2 * un.split + un.half) * kBM + q * 32 + lane) * kBN;
        const float* other = part + (size_t(2 * un.split + (un.half ^ 1)) * kBM + q * 32 + lane) * kBN;
#pragma unroll 1
        for (int cc = h * (kBN / 64); cc < (h + 1) * (kBN / 64); ++cc) {
          float v[32];
          combine(cc, v);
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(mine + cc * 32 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
        __threadfence();
        __syncwarp();
        unsigned prev = 0;
        if (lane == 0) prev = atomicAdd(&cnt[un.split * kEpiWarps + (warp - 2)], 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == 1u) {
          __threadfence();
#pragma unroll 1
          for (int cc = h * (kBN / 64); cc < (h + 1) * (kBN / 64); ++cc) {
            float v[32];
            combine(cc, v);
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 w = __ldcg(reinterpret_cast<const float4*>(other + cc * 32 + j));
              v[j] += w.x;
              v[j + 1] += w.y;
              v[j + 2] += w.z;
              v[j + 3] += w.w;
            }
            store(cc, v);
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
#endif
}

inline size_t workspace_bytes(int B, int I, int O, int C) { return layout(B, I, O, C).total; }

// Tiles of the last round split into K halves: the rem = n_tiles mod grid tiles of a partial last
// round, when their 2 * rem halves fit one round (the CTAs' work then differs by half a tile
// instead of a whole one) and each half keeps enough K blocks.
inline int split_tiles(int n_tiles, int grid, int nkb) {
  if (n_tiles <= grid) return 0;
  const int rem = n_tiles % grid;
  if (rem == 0 || 2 * rem > grid || rem > max_split_tiles() || nkb < 4 * kD0Parts) return 0;
  return rem;
}

// Full op with a caller workspace of workspace_bytes() bytes (no initialisation needed).
inline int run(const float* x, const float* grid, const float* wb, const float* sw, const float* sc, int32_t G,
               int32_t K, int32_t B, int32_t I, int32_t O, float* out, void* workspace, size_t ws_bytes,
               cudaStream_t stream) {
  if (B < 0 || I < 0 || O < 0 || G < 1 || K < 0) return kInvalidArgument;
  const int C = G + K;
  if (C + K + 1 > kMaxKnots) return kUnsupported;
  if (B == 0 || O == 0) return kOk;
  if (x == nullptr || grid == nullptr || wb == nullptr || sw == nullptr || sc == nullptr || out == nullptr)
    return kInvalidArgument;
  if (I == 0) {
    cudaMemsetAsync(out, 0, size_t(B) * O * 4, stream);
    return launch_status();
  }
  const Layout L = layout(B, I, O, C);
  if (workspace == nullptr || ws_bytes < L.total) return kWorkspaceTooSmall;
  char* w = static_cast<char*>(workspace);
  __half* a_hi = reinterpret_cast<__half*>(w + L.a_hi);
  __half* a_lo = reinterpret_cast<__half*>(w + L.a_lo);
  __half* w_hi = reinterpret_cast<__half*>(w + L.w_hi);
  __half* w_lo = reinterpret_cast<__half*>(w + L.w_lo);
  float* rs = reinterpret_cast<float*>(w + L.rs);
  float* cs = reinterpret_cast<float*>(w + L.cs);
  const int64_t kp = padded_k(I, C);
  // Column-major form for the cubic cases; its float2 loads of x need I even and x 8-byte aligned.
  const bool columns = K == 3 && (G == 5 || G == 8) && I % 2 == 0 && (reinterpret_cast<uintptr_t>(x) & 7u) == 0 &&
                       (reinterpret_cast<uintptr_t>(grid) & 7u) == 0;
  const int scale_ctas = columns ? (B + kScaleRowsPerCta - 1) / kScaleRowsPerCta : 0;
  unsigned* cnt = reinterpret_cast<unsigned*>(w + L.cnt);
  launch_pdl(prep_wr_kernel, unsigned(O + scale_ctas), kPrepThreads, 0, stream, wb, sw, sc, I, O, C, kp, w_hi, w_lo,
             cs, x, B, rs, a_hi, a_lo, cnt, max_split_tiles() * kEpiWarps);
  if (columns) {
    auto pk = G == 5 ? prep_a3_kernel<12> : prep_a3_kernel<15>;
    const int rows = prep3_rows(B, I, resident_ctas_per_sm(pk, kPrep3Threads, 0));
    const dim3 pg(unsigned((I + 2 * kPrep3Threads - 1) / (2 * kPrep3Threads)), unsigned((B + rows - 1) / rows));
    launch_pdl(pk, pg, kPrep3Threads, 0, stream, x, grid, B, I, kp, static_cast<const float*>(rs), a_hi, a_lo,
               rows);
  } else if (G == 5 && K == 3) {
    launch_pdl(prep_a_kernel<12, 3>, B, 256, 0, stream, x, grid, I, C, K, kp, a_hi, a_lo, rs);
  } else if (G == 8 && K == 3) {
    launch_pdl(prep_a_kernel<15, 3>, B, 256, 0, stream, x, grid, I, C, K, kp, a_hi, a_lo, rs);
  } else {
    launch_pdl(prep_a_kernel<0, 0>, B, 256, 0, stream, x, grid, I, C, K, kp, a_hi, a_lo, rs);
  }
  CUtensorMap m_ahi, m_alo, m_whi, m_wlo;
  if (!tc::make_map_sw128(&m_ahi, a_hi, uint64_t(B), uint64_t(kp), 2, kBM) ||
      !tc::make_map_sw128(&m_alo, a_lo, uint64_t(B), uint64_t(kp), 2, kBM) ||
      !tc::make_map_sw128(&m_whi, w_hi, uint64_t(O), uint64_t(kp), 2, kBN) ||
      !tc::make_map_sw128(&m_wlo, w_lo, uint64_t(O), uint64_t(kp), 2, kBN))
    return kUnsupported;
  if (!ensure_dyn_smem(gemm_kernel, kSmem)) return kCudaError;
  const int n_tiles = ((B + kBM - 1) / kBM) * ((O + kBN - 1) / kBN);
  const int grid_ctas = n_tiles < sm_count() ? n_tiles : sm_count();
  const int n_split = split_tiles(n_tiles, grid_ctas, int(kp / kBKe));
  launch_pdl(gemm_kernel, grid_ctas, kThreads, kSmem, stream, m_ahi, m_alo, m_whi, m_wlo, B, O, kp, rs, cs, out,
             reinterpret_cast<float*>(w + L.part), cnt, n_split, (O % 4 == 0 && aligned16(out)) ? 1 : 0);
  return launch_status();
}

}  // namespace kan
}  // namespace b200
