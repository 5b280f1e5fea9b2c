// Backward of the KAN linear layer (kan.cuh): the gradients torch autograd forms through the
// reference forward (tasks/efficient_kan/reference.py:33-46), for an incoming gradient G [B, O]:
//
//   grad_A = G . W'            [B, I(1+C)]   (W' = [W_base | sw * scaler], as in the forward)
//   grad_W = G^T . A           [O, I(1+C)]   (A = [silu(x) | bases(x)], as in the forward)
//   grad_x[b,i] = silu'(x) grad_A[b, i] + sum_c B'_c(x) grad_A[b, (1+c)I + i]
//   grad_W_base = grad_W[:, 0:I];  grad_sw[o,i,c] = grad_W[o, (1+c)I + i] * scaler[o,i];
//   grad_scaler[o,i] = sum_c grad_W[o, (1+c)I + i] * sw[o,i,c]
//
// with B'_c the derivative of the Cox-de Boor recurrence carried alongside it (forward-mode, the
// same two-term steps).  The two products are GEMMs of the forward's size (2 B O I (1+C) flop
// each) and run on the forward's split-fp16 tcgen05 kernel (kan::gemm_kernel: hi/lo fp16 planes,
// fp32 TMEM accumulators, power-of-two row and column scales), on operands laid out K-major for it:
//   GEMM 1: M = B, N = I(1+C), K = O: rows of G [B, O], and W' transposed ([I(1+C), O] planes,
//           built from W_base, sw and scaler through 32 x 32 shared-memory tiles);
//   GEMM 2: M = O, N = I(1+C), K = B: G transposed ([O, B] planes) and A transposed ([I(1+C), B]
//           planes: silu and the bases evaluated once per (b, i) into a tile, written row by row).
// Each plane row gets its own power-of-two scale from the row's max |value| (a column-max pass for
// the transposed operands; bases lie in [0, 1] and need none), as the forward's planes do.
// K padding (to a multiple of 64) is written as zeros.
#pragma once

#include "kan.cuh"

namespace b200 {
namespace kanb {

using kan::kMaxKnots;

constexpr int kTile = 32;              // transpose tiles: 32 x 32, 32 x 8 threads
constexpr int kTileRows = 8;
constexpr int kSplitThreads = 256;
constexpr int kColThreads = 256;
constexpr int kColChunk = 32;          // rows per CTA of the column-max pass
constexpr int kGradThreads = 256;
constexpr int kMaxTileSmem = 200 * 1024;

inline int64_t pad64(int64_t v) { return (v + 63) / 64 * 64; }

struct Layout {
  size_t g_hi, g_lo, rg, wt_hi, wt_lo, cwt, gt_hi, gt_lo, rgt, at_hi, at_lo, cat, amax_wt, amax_gt, amax_x, grad_a,
      grad_w, total;
};

inline Layout layout(int B, int I, int O, int C) {
  const int64_t nk = int64_t(I) * (1 + C), op = pad64(O), bp = pad64(B);
  Layout L;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += align256(bytes);
    return at;
  };
  L.g_hi = take(size_t(B) * op * 2);
  L.g_lo = take(size_t(B) * op * 2);
  L.rg = take(size_t(B) * 4);
  L.wt_hi = take(size_t(nk) * op * 2);
  L.wt_lo = take(size_t(nk) * op * 2);
  L.cwt = take(size_t(nk) * 4);
  L.gt_hi = take(size_t(O) * bp * 2);
  L.gt_lo = take(size_t(O) * bp * 2);
  L.rgt = take(size_t(O) * 4);
  L.at_hi = take(size_t(nk) * bp * 2);
  L.at_lo = take(size_t(nk) * bp * 2);
  L.cat = take(size_t(nk) * 4);
  L.amax_wt = take(size_t(nk) * 4);
  L.amax_gt = take(size_t(O) * 4);
  L.amax_x = take(size_t(I) * 4);
  L.grad_a = take(size_t(B) * nk * 4);
  L.grad_w = take(size_t(O) * nk * 4);
  L.total = off;
  return L;
}

inline size_t tile_smem(int C) { return size_t(1 + C) * kTile * (kTile + 1) * sizeof(float); }

// Rows of a row-major [R, kd] matrix into hi/lo planes [R, kp] (one CTA per row; unscale = 1/f).
__global__ void __launch_bounds__(kSplitThreads) split_rows_kernel(const float* __restrict__ src, int kd, int64_t kp,
                                                                   __half* __restrict__ hi, __half* __restrict__ lo,
                                                                   float* __restrict__ unscale) {
  pdl_begin();
  __shared__ float s_red[33];
  const int64_t r = blockIdx.x;
  const float* row = src + r * kd;
  float amax = 0.0f;
  for (int k = threadIdx.x; k < kd; k += kSplitThreads) amax = fmaxf(amax, fabsf(row[k]));
  const float f = kan::fp16_row_factor(kan::block_max(amax, s_red));
  if (threadIdx.x == 0) unscale[r] = 1.0f / f;
  for (int64_t k = threadIdx.x; k < kp; k += kSplitThreads) {
    const float v = k < kd ? row[k] * f : 0.0f;
    kan::split_store(v, hi + r * kp + k, lo + r * kp + k);
  }
}

// amax[c] = max over rows of |src[row, c]|: a thread per column, a block of kColChunk rows per CTA
// row, combined with atomicMax on the non-negative float bits.
__global__ void __launch_bounds__(kColThreads) colmax_kernel(const float* __restrict__ src, int64_t rows, int cols,
                                                             uint32_t* __restrict__ amax) {
  pdl_begin();
  const int c = blockIdx.x * kColThreads + threadIdx.x;
  if (c >= cols) return;
  const int64_t r0 = int64_t(blockIdx.y) * kColChunk;
  const int64_t r1 = r0 + kColChunk < rows ? r0 + kColChunk : rows;
  float m = 0.0f;
  for (int64_t r = r0; r < r1; ++r) m = fmaxf(m, fabsf(src[r * cols + c]));
  atomicMax(amax + c, __float_as_uint(m));
}

// Columns of a row-major [kd, R] matrix into hi/lo planes [R, kp]: plane row r = source column r.
// 32 x 32 tiles through shared memory; blockIdx.x walks kp (padding written as zeros).
__global__ void __launch_bounds__(kTile * kTileRows) split_cols_kernel(const float* __restrict__ src, int kd, int R,
                                                                       int64_t kp, const uint32_t* __restrict__ amax,
                                                                       __half* __restrict__ hi,
                                                                       __half* __restrict__ lo,
                                                                       float* __restrict__ unscale) {
  pdl_begin();
  __shared__ float t[kTile][kTile + 1];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t k0 = int64_t(blockIdx.x) * kTile;
  const int r0 = blockIdx.y * kTile;
  for (int y = ty; y < kTile; y += kTileRows) {
    const int64_t k = k0 + y;
    const int r = r0 + tx;
    t[y][tx] = (k < kd && r < R) ? src[k * R + r] : 0.0f;
  }
  __syncthreads();
  for (int y = ty; y < kTile; y += kTileRows) {
    const int r = r0 + y;
    if (r >= R) continue;
    const float f = kan::fp16_row_factor(__uint_as_float(amax[r]));
    if (blockIdx.x == 0 && tx == 0) unscale[r] = 1.0f / f;
    const int64_t k = k0 + tx;
    if (k < kp) kan::split_store(t[tx][y] * f, hi + int64_t(r) * kp + k, lo + int64_t(r) * kp + k);
  }
}

// W'[o, p*I + i] (p = 0: W_base; p = 1 + c: sw[o,i,c] * scaler[o,i], the forward's fp32 product).
__device__ __forceinline__ float wfull(const float* wb, const float* sw, const float* sc, int I, int C, int o, int i,
                                       int p) {
  const int64_t oi = int64_t(o) * I + i;
  return p == 0 ? wb[oi] : __fmul_rn(sw[oi * C + (p - 1)], sc[oi]);
}

// amax over o of |W'[o, p*I + i]| for every (p, i): a tile of 32 inputs x 64 outputs per CTA,
// reduced over the CTA's outputs in shared memory, then one atomicMax per (p, i).
__global__ void __launch_bounds__(kTile * kTileRows) wt_amax_kernel(const float* __restrict__ wb,
                                                                    const float* __restrict__ sw,
                                                                    const float* __restrict__ sc, int I, int O, int C,
                                                                    uint32_t* __restrict__ amax) {
  pdl_begin();
  __shared__ float s[kTileRows][kTile];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int i = blockIdx.x * kTile + tx;
  const int o0 = blockIdx.y * 64;
  for (int p = 0; p <= C; ++p) {
    float m = 0.0f;
    if (i < I)
      for (int o = o0 + ty; o < o0 + 64 && o < O; o += kTileRows) m = fmaxf(m, fabsf(wfull(wb, sw, sc, I, C, o, i, p)));
    s[ty][tx] = m;
    __syncthreads();
    if (ty == 0 && i < I) {
#pragma unroll
      for (int y = 1; y < kTileRows; ++y) m = fmaxf(m, s[y][tx]);
      atomicMax(amax + int64_t(p) * I + i, __float_as_uint(m));
    }
    __syncthreads();
  }
}

// W' transposed into planes [I(1+C), kp = pad64(O)]: a tile of 32 inputs x 32 outputs holds every
// p of W' (shared [1+C][32][33]); plane rows p*I + i are then written 32 outputs at a time.
__global__ void __launch_bounds__(kTile * kTileRows) wt_split_kernel(const float* __restrict__ wb,
                                                                     const float* __restrict__ sw,
                                                                     const float* __restrict__ sc, int I, int O,
                                                                     int C, int64_t kp,
                                                                     const uint32_t* __restrict__ amax,
                                                                     __half* __restrict__ hi, __half* __restrict__ lo,
                                                                     float* __restrict__ unscale) {
  pdl_begin();
  extern __shared__ float s_t[];  // [1 + C][kTile][kTile + 1]
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int i0 = blockIdx.x * kTile, o0 = blockIdx.y * kTile;
  const int i = i0 + tx;
  for (int y = ty; y < kTile; y += kTileRows) {
    const int o = o0 + y;
    for (int p = 0; p <= C; ++p)
      s_t[(p * kTile + tx) * (kTile + 1) + y] = (i < I && o < O) ? wfull(wb, sw, sc, I, C, o, i, p) : 0.0f;
  }
  __syncthreads();
  const int rows = (1 + C) * kTile;
  for (int rr = ty; rr < rows; rr += kTileRows) {
    const int p = rr / kTile, ii = rr - p * kTile;
    if (i0 + ii >= I) continue;
    const int64_t kr = int64_t(p) * I + i0 + ii;
    const float f = kan::fp16_row_factor(__uint_as_float(amax[kr]));
    if (blockIdx.y == 0 && tx == 0) unscale[kr] = 1.0f / f;
    const int64_t o = o0 + tx;
    if (o < kp) kan::split_store(s_t[(p * kTile + ii) * (kTile + 1) + tx] * f, hi + kr * kp + o, lo + kr * kp + o);
  }
}

// One input's knots g[0..NK) and reciprocal knot differences rk[k-1][j] = 1 / (g[j+k] - g[j])
// (j < NK - k), in registers: the same input's recurrence then runs on multiplies for every row a
// thread handles.
template <int NK, int KO>
__device__ __forceinline__ void load_knots(const float* __restrict__ gsrc, float (&g)[NK], float (&rk)[KO][NK]) {
#pragma unroll
  for (int j = 0; j < NK; ++j) g[j] = __ldg(gsrc + j);
#pragma unroll
  for (int k = 1; k <= KO; ++k)
#pragma unroll
    for (int j = 0; j < NK - k; ++j) rk[k - 1][j] = 1.0f / (g[j + k] - g[j]);
}

// The Cox-de Boor recurrence (every basis, unrolled) on the reciprocals; with kDeriv the
// derivatives d/dx ride along (b'[j] = l' b[j] + l b'[j] + r' b[j+1] + r b'[j+1]).
template <int NK, int KO, bool kDeriv>
__device__ __forceinline__ void bases_recip(float x, const float (&g)[NK], const float (&rk)[KO][NK], float* b,
                                            float* db) {
#pragma unroll
  for (int j = 0; j < NK - 1; ++j) {
    b[j] = (x >= g[j] && x < g[j + 1]) ? 1.0f : 0.0f;
    if (kDeriv) db[j] = 0.0f;
  }
#pragma unroll
  for (int k = 1; k <= KO; ++k) {
#pragma unroll
    for (int j = 0; j < NK - 1 - k; ++j) {
      const float il = rk[k - 1][j], ir = rk[k - 1][j + 1];
      const float l = (x - g[j]) * il, r = (g[j + k + 1] - x) * ir;
      const float nb = l * b[j] + r * b[j + 1];
      if (kDeriv) db[j] = il * b[j] + l * db[j] - ir * b[j + 1] + r * db[j + 1];
      b[j] = nb;
    }
  }
}

// The four cubic bases s-3 .. s of x (g[s] <= x < g[s+1]) and, with kDeriv, their derivatives,
// from the knots kn[0..6) = g[s-2 .. s+3]: the two-term steps of the recurrence (and of its
// derivative, as bases_recip carries it) restricted to the bases that can be non-zero, on hardware
// reciprocals of the knot differences.
template <bool kDeriv>
__device__ __forceinline__ void cubic_dual(float x, const float (&kn)[6], float (&n)[4], float (&dn)[4]) {
  float N[4] = {1.0f, 0.0f, 0.0f, 0.0f}, D[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int k = 1; k <= 3; ++k) {
    float Nn[4] = {0.0f, 0.0f, 0.0f, 0.0f}, Dn[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int m = 0; m <= k; ++m) {  // basis s - k + m of order k
      float v = 0.0f, dv = 0.0f;
      if (m >= 1) {  // (x - g[j]) / (g[j+k] - g[j]) * b[j],  j = s - k + m
        const float il = kan::rcp_approx(kn[m + 2] - kn[m - k + 2]);
        const float l = (x - kn[m - k + 2]) * il;
        v = l * N[m - 1];
        if (kDeriv) dv = il * N[m - 1] + l * D[m - 1];
      }
      if (m <= k - 1) {  // (g[j+k+1] - x) / (g[j+k+1] - g[j+1]) * b[j+1]
        const float ir = kan::rcp_approx(kn[m + 3] - kn[m - k + 3]);
        const float r = (kn[m + 3] - x) * ir;
        v = m >= 1 ? v + r * N[m] : r * N[m];
        if (kDeriv) dv = dv - ir * N[m] + r * D[m];
      }
      Nn[m] = v;
      Dn[m] = dv;
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      N[m] = Nn[m];
      D[m] = Dn[m];
    }
  }
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    n[m] = N[m];
    dn[m] = D[m];
  }
}

// Knot interval of x in a thread's knot column col[j * stride] (strictly increasing knots): the
// count of knots <= x, by binary search (NaN gives 0).
template <int NK>
__device__ __forceinline__ int knots_le(float x, const float* col, int stride) {
  static_assert(NK <= 16, "the binary search covers up to 16 knots");
  int cnt = 0;
#pragma unroll
  for (int step = 8; step >= 1; step >>= 1)
    if (cnt + step <= NK && col[min(cnt + step - 1, NK - 1) * stride] <= x) cnt += step;
  return cnt;
}

__host__ __device__ constexpr int at_tile_rows(int nk) { return nk > 0 ? 64 : kTile; }
inline size_t at_tile_smem(int C, int nk) {
  return size_t(1 + C) * kTile * (at_tile_rows(nk) + 1) * sizeof(float);
}

// A transposed into planes [I(1+C), kp = pad64(B)]: a tile of 32 inputs x 32 (or 64) batch rows; each
// thread evaluates silu and the bases of one x (the forward's recurrence) into shared memory.
// Plane rows p = 0 take the factor of the input's max |x| over the batch (|silu(x)| <= |x|); bases
// lie in [0, 1].  Only the K + 1 bases that can be non-zero are formed (kan::bases_local).
// NK, KO > 0: knot count and order known at compile time (the recurrence unrolled in registers).
template <int NK, int KO>
__global__ void __launch_bounds__(kTile * kTileRows) at_split_kernel(const float* __restrict__ x,
                                                                     const float* __restrict__ grid, int B, int I,
                                                                     int C, int K, int64_t kp,
                                                                     const uint32_t* __restrict__ amax_x,
                                                                     __half* __restrict__ hi, __half* __restrict__ lo,
                                                                     float* __restrict__ unscale) {
  pdl_begin();
  // The cubic forms take 64 batch rows per tile (each input's reciprocals serve 8 rows per thread;
  // a plane row's 64 values go out as two 64-byte warp stores of lanes' consecutive words, which
  // reads the tile row without bank conflicts); the general form 32.
  constexpr int kW = at_tile_rows(NK);
  extern __shared__ float s_t[];  // [1 + C][kTile][kW + 1]
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int i0 = blockIdx.x * kTile, b0 = blockIdx.y * kW;
  const int i = i0 + tx;
  const int nk = C + K + 1;
  constexpr int NKr = NK > 0 ? NK : 2;
  // Cubic forms: the tile's knots in shared memory, column tx = input i0 + tx (the tile's 8 thread
  // rows read the same column: broadcasts); only the four non-zero bases of each x are formed.
  __shared__ float s_kn[NKr][kTile];
  __shared__ int s_inc[kTile];
  if (NK > 0 && ty == 0) {
    bool inc = true;
    float prev = 0.0f;
#pragma unroll
    for (int j = 0; j < NKr; ++j) {
      const float g = i < I ? __ldg(grid + int64_t(i) * nk + j) : 0.0f;
      s_kn[j][tx] = g;
      if (j > 0) inc = inc && prev < g;
      prev = g;
    }
    s_inc[tx] = inc ? 1 : 0;
  }
  if (NK > 0) __syncthreads();
  for (int y = ty; y < kW; y += kTileRows) {
    const int b = b0 + y;
    const bool ok = i < I && b < B;
    const float xv = ok ? x[int64_t(b) * I + i] : 0.0f;
    s_t[(0 * kTile + tx) * (kW + 1) + y] = ok ? kan::silu(xv) : 0.0f;
    if (NK > 0) {
      constexpr int Cc = NK > 0 ? NK - 4 : 1;
      if (!ok || s_inc[tx]) {
        // Zeros (NaN for a non-finite x, as the full recurrence gives), then the four bases.
        const float z = fabsf(xv) <= 3.402823466e38f ? 0.0f : __int_as_float(0x7fc00000);
#pragma unroll
        for (int c = 0; c < Cc; ++c) s_t[((1 + c) * kTile + tx) * (kW + 1) + y] = z;
        const int cnt = ok ? knots_le<NKr>(xv, &s_kn[0][tx], kTile) : 0;
        if (cnt >= 1 && cnt <= NK - 1) {
          const int sj = cnt - 1;
          float kv[6], nb[4], dnb[4];
#pragma unroll
          for (int o = 0; o < 6; ++o) kv[o] = s_kn[min(max(sj - 2 + o, 0), NK - 1)][tx];
          cubic_dual<false>(xv, kv, nb, dnb);
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const int c = sj - 3 + m;  // invalid ones (outside 0 .. C-1) used clamped knots
            if (c >= 0 && c < Cc) s_t[((1 + c) * kTile + tx) * (kW + 1) + y] = nb[m];
          }
        }
      } else {  // knots not strictly increasing: the full recurrence
        float bs[NKr];
        kan::bases_fixed<NKr, 3>(xv, grid + int64_t(i) * nk, bs);
#pragma unroll
        for (int c = 0; c < Cc; ++c) s_t[((1 + c) * kTile + tx) * (kW + 1) + y] = bs[c];
      }
    } else {
      float g[kMaxKnots], bs[kMaxKnots];
      if (ok) {
        for (int j = 0; j < nk; ++j) g[j] = grid[int64_t(i) * nk + j];
        kan::bases_of(xv, g, nk, K, bs);
      }
      for (int c = 0; c < C; ++c) s_t[((1 + c) * kTile + tx) * (kW + 1) + y] = ok ? bs[c] : 0.0f;
    }
  }
  __syncthreads();
  const int rows = (1 + C) * kTile;
  for (int rr = ty; rr < rows; rr += kTileRows) {
    const int p = rr / kTile, ii = rr - p * kTile;
    if (i0 + ii >= I) continue;
    const int64_t kr = int64_t(p) * I + i0 + ii;
    const float f = p == 0 ? kan::fp16_row_factor(__uint_as_float(amax_x[i0 + ii])) : 1.0f;
    if (blockIdx.y == 0 && tx == 0) unscale[kr] = 1.0f / f;
    const float* srow = s_t + (p * kTile + ii) * (kW + 1);
    if (kW == 64) {  // b0 + 64 <= kp (kp is a multiple of 64); consecutive lanes read consecutive words
      const int64_t b = b0 + tx;
      kan::split_store(srow[tx] * f, hi + kr * kp + b, lo + kr * kp + b);
      kan::split_store(srow[tx + 32] * f, hi + kr * kp + b + 32, lo + kr * kp + b + 32);
    } else {
      const int64_t b = b0 + tx;
      if (b < kp) kan::split_store(srow[tx] * f, hi + kr * kp + b, lo + kr * kp + b);
    }
  }
}

// The bases of x and their derivatives d/dx: the forward's recurrence with each two-term step
// differentiated alongside (b'[j] = l' b[j] + l b'[j] + r' b[j+1] + r b'[j+1]).
__device__ __forceinline__ void bases_dual(float x, const float* g, int nk, int K, float* b, float* db) {
  for (int j = 0; j < nk - 1; ++j) {
    b[j] = (x >= g[j] && x < g[j + 1]) ? 1.0f : 0.0f;
    db[j] = 0.0f;
  }
  for (int k = 1; k <= K; ++k) {
    for (int j = 0; j < nk - 1 - k; ++j) {
      const float dl = 1.0f / (g[j + k] - g[j]);
      const float dr = -1.0f / (g[j + k + 1] - g[j + 1]);
      const float l = (x - g[j]) * dl;
      const float r = (g[j + k + 1] - x) * -dr;
      const float nb = l * b[j] + r * b[j + 1];
      db[j] = dl * b[j] + l * db[j] + dr * b[j + 1] + r * db[j + 1];
      b[j] = nb;
    }
  }
}

// grad_x[b, i] from grad_A [B, I(1+C)]: a thread per input i (i fastest across the CTA) and
// kGradRows batch rows, so each input's knots and reciprocals are set up once.  NK, KO as
// at_split_kernel.
constexpr int kGradRows = 8;
template <int NK, int KO>
__global__ void __launch_bounds__(kGradThreads) grad_x_kernel(const float* __restrict__ x,
                                                              const float* __restrict__ grid,
                                                              const float* __restrict__ ga, int64_t B, int I, int C,
                                                              int K, float* __restrict__ gx) {
  pdl_begin();
  const int i = blockIdx.x * kGradThreads + threadIdx.x;
  if (i >= I) return;
  const int nk = C + K + 1;
  const int64_t nkp = int64_t(I) * (1 + C);
  constexpr int NKr = NK > 0 ? NK : 2, KOr = KO > 0 ? KO : 1;
  // Cubic forms: this thread's knot column in shared memory (only this thread reads it, so no
  // barrier), and only the four non-zero bases' derivatives of each x.
  __shared__ float s_kn[NKr][kGradThreads];
  bool inc = true;
  float g[NK > 0 ? 1 : kMaxKnots];
  if (NK > 0) {
    float prev = 0.0f;
#pragma unroll
    for (int j = 0; j < NKr; ++j) {
      const float v = __ldg(grid + int64_t(i) * nk + j);
      s_kn[j][threadIdx.x] = v;
      if (j > 0) inc = inc && prev < v;
      prev = v;
    }
  } else {
    for (int j = 0; j < nk; ++j) g[j] = grid[int64_t(i) * nk + j];
  }
  const int64_t b0 = int64_t(blockIdx.y) * kGradRows;
  for (int r = 0; r < kGradRows; ++r) {
    const int64_t b = b0 + r;
    if (b >= B) break;
    const float xv = x[b * I + i];
    const float s = 1.0f / (1.0f + expf(-xv));
    const float dsilu = s * (1.0f + xv * (1.0f - s));
    const float* row = ga + b * nkp + i;
    float acc = row[0] * dsilu;
    if (NK > 0 && inc) {
      // Zero derivative outside [g0, g[NK-1]); NaN for a non-finite x, as the full recurrence.
      if (!(fabsf(xv) <= 3.402823466e38f)) acc = __int_as_float(0x7fc00000);
      const int cnt = knots_le<NKr>(xv, &s_kn[0][threadIdx.x], kGradThreads);
      if (cnt >= 1 && cnt <= NK - 1) {
        const int sj = cnt - 1;
        float kv[6], nb[4], dnb[4];
#pragma unroll
        for (int o = 0; o < 6; ++o) kv[o] = s_kn[min(max(sj - 2 + o, 0), NK - 1)][threadIdx.x];
        cubic_dual<true>(xv, kv, nb, dnb);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int c = sj - 3 + m;
          if (c >= 0 && c < NKr - KOr - 1) acc = fmaf(row[int64_t(1 + c) * I], dnb[m], acc);
        }
      }
    } else if (NK > 0) {  // knots not strictly increasing: the full recurrence (rare; local arrays)
      float gk[NKr], bs[NKr], dbs[NKr];
      for (int j = 0; j < NKr; ++j) gk[j] = s_kn[j][threadIdx.x];
      bases_dual(xv, gk, NKr, KOr, bs, dbs);
      for (int c = 0; c < NKr - KOr - 1; ++c) acc = fmaf(row[int64_t(1 + c) * I], dbs[c], acc);
    } else {
      float bs[kMaxKnots], dbs[kMaxKnots];
      bases_dual(xv, g, nk, K, bs, dbs);
      for (int c = 0; c < C; ++c) acc = fmaf(row[int64_t(1 + c) * I], dbs[c], acc);
    }
    gx[b * I + i] = acc;
  }
}

// Weight gradients from grad_W [O, I(1+C)]: a thread per (o, i), i fastest.
__global__ void __launch_bounds__(kGradThreads) grad_w_kernel(const float* __restrict__ gw,
                                                              const float* __restrict__ sw,
                                                              const float* __restrict__ sc, int64_t O, int I, int C,
                                                              float* __restrict__ g_wb, float* __restrict__ g_sw,
                                                              float* __restrict__ g_sc) {
  pdl_begin();
  const int64_t q = int64_t(blockIdx.x) * kGradThreads + threadIdx.x;
  if (q >= O * I) return;
  const int64_t o = q / I;
  const int i = int(q - o * I);
  const float* row = gw + o * (int64_t(I) * (1 + C)) + i;
  if (g_wb != nullptr) g_wb[q] = row[0];
  const float scv = sc[q];
  float acc = 0.0f;
  for (int c = 0; c < C; ++c) {
    const float v = row[int64_t(1 + c) * I];
    if (g_sw != nullptr) g_sw[q * C + c] = v * scv;
    acc = fmaf(v, sw[q * C + c], acc);
  }
  if (g_sc != nullptr) g_sc[q] = acc;
}

// out[M, N] = (A planes [M, kp]) . (W planes [N, kp])^T * rs[m] * cs[n] on kan::gemm_kernel.
inline int gemm(const __half* a_hi, const __half* a_lo, int M, const __half* w_hi, const __half* w_lo, int N,
                int64_t kp, const float* rs, const float* cs, float* out, cudaStream_t stream) {
  CUtensorMap m_ahi, m_alo, m_whi, m_wlo;
  if (!tc::make_map_sw128(&m_ahi, a_hi, uint64_t(M), uint64_t(kp), 2, kan::kBM) ||
      !tc::make_map_sw128(&m_alo, a_lo, uint64_t(M), uint64_t(kp), 2, kan::kBM) ||
      !tc::make_map_sw128(&m_whi, w_hi, uint64_t(N), uint64_t(kp), 2, kan::kBN) ||
      !tc::make_map_sw128(&m_wlo, w_lo, uint64_t(N), uint64_t(kp), 2, kan::kBN))
    return kUnsupported;
  if (!ensure_dyn_smem(kan::gemm_kernel, kan::kSmem)) return kCudaError;
  const int n_tiles = ((M + kan::kBM - 1) / kan::kBM) * ((N + kan::kBN - 1) / kan::kBN);
  const int grid = n_tiles < sm_count() ? n_tiles : sm_count();
  return launch_pdl(kan::gemm_kernel, grid, kan::kThreads, kan::kSmem, stream, m_ahi, m_alo, m_whi, m_wlo, M, N, kp,
                    rs, cs, out, static_cast<float*>(nullptr), static_cast<unsigned*>(nullptr), 0,
                    (N % 4 == 0 && aligned16(out)) ? 1 : 0);
}

inline size_t workspace_bytes(int B, int I, int O, int C) { return layout(B, I, O, C).total; }

// Gradients for grad_out [B, O]; any of grad_x, grad_wb, grad_sw, grad_sc may be null (not
// computed).  Shapes and knots as kan::run.
inline int backward(const float* x, const float* grid, const float* wb, const float* sw, const float* sc, int32_t G,
                    int32_t K, int32_t B, int32_t I, int32_t O, const float* grad_out, float* grad_x, float* grad_wb,
                    float* grad_sw, float* grad_sc, void* workspace, size_t ws_bytes, cudaStream_t stream) {
  if (B < 0 || I < 0 || O < 0 || G < 1 || K < 0) return kInvalidArgument;
  const int C = G + K;
  if (C + K + 1 > kMaxKnots || tile_smem(C) > size_t(kMaxTileSmem)) return kUnsupported;
  const bool need_x = grad_x != nullptr;
  const bool need_w = grad_wb != nullptr || grad_sw != nullptr || grad_sc != nullptr;
  if (int64_t(B) * I == 0 && int64_t(O) * I == 0) return kOk;
  if (x == nullptr || grid == nullptr || wb == nullptr || sw == nullptr || sc == nullptr ||
      (int64_t(B) * O > 0 && grad_out == nullptr))
    return kInvalidArgument;
  if (B == 0 || O == 0 || I == 0) {  // every gradient is an empty sum
    if (need_x && B > 0 && I > 0) cudaMemsetAsync(grad_x, 0, size_t(B) * I * 4, stream);
    if (O > 0 && I > 0) {
      if (grad_wb) cudaMemsetAsync(grad_wb, 0, size_t(O) * I * 4, stream);
      if (grad_sw) cudaMemsetAsync(grad_sw, 0, size_t(O) * I * C * 4, stream);
      if (grad_sc) cudaMemsetAsync(grad_sc, 0, size_t(O) * I * 4, stream);
    }
    return launch_status();
  }
  const Layout L = layout(B, I, O, C);
  if (workspace == nullptr || ws_bytes < L.total) return kWorkspaceTooSmall;
  char* w = static_cast<char*>(workspace);
  auto half_at = [&](size_t off) { return reinterpret_cast<__half*>(w + off); };
  auto float_at = [&](size_t off) { return reinterpret_cast<float*>(w + off); };
  auto u32_at = [&](size_t off) { return reinterpret_cast<uint32_t*>(w + off); };
  const int64_t nkp = int64_t(I) * (1 + C), op = pad64(O), bp = pad64(B);
  if (nkp > 0x7fffffff) return kUnsupported;
  const size_t tsm = tile_smem(C);
  // The cubic cases of the reference (G = 5 and G = 8) take the unrolled recurrences.
  const int form = K == 3 && G == 5 ? 1 : (K == 3 && G == 8 ? 2 : 0);
  auto at_kern = form == 1 ? at_split_kernel<12, 3> : (form == 2 ? at_split_kernel<15, 3> : at_split_kernel<0, 0>);
  auto gx_kern = form == 1 ? grad_x_kernel<12, 3> : (form == 2 ? grad_x_kernel<15, 3> : grad_x_kernel<0, 0>);
  const int at_nk = form == 1 ? 12 : (form == 2 ? 15 : 0);
  const size_t at_sm = at_tile_smem(C, at_nk);
  if (!ensure_dyn_smem(wt_split_kernel, int(tsm)) || !ensure_dyn_smem(at_kern, int(at_sm))) return kCudaError;
  const dim3 tb(kTile, kTileRows);
  int st = kOk;
  if (need_x) {
    cudaMemsetAsync(u32_at(L.amax_wt), 0, size_t(nkp) * 4, stream);
    st = launch_pdl(split_rows_kernel, unsigned(B), kSplitThreads, 0, stream, grad_out, O, op, half_at(L.g_hi),
                    half_at(L.g_lo), float_at(L.rg));
    if (st != kOk) return st;
    st = launch_pdl(wt_amax_kernel, dim3(unsigned((I + kTile - 1) / kTile), unsigned((O + 63) / 64)), tb, 0, stream,
                    wb, sw, sc, I, O, C, u32_at(L.amax_wt));
    if (st != kOk) return st;
    st = launch_pdl(wt_split_kernel, dim3(unsigned((I + kTile - 1) / kTile), unsigned(op / kTile)), tb, tsm, stream,
                    wb, sw, sc, I, O, C, op, static_cast<const uint32_t*>(u32_at(L.amax_wt)), half_at(L.wt_hi),
                    half_at(L.wt_lo), float_at(L.cwt));
    if (st != kOk) return st;
    st = gemm(half_at(L.g_hi), half_at(L.g_lo), B, half_at(L.wt_hi), half_at(L.wt_lo), int(nkp), op, float_at(L.rg),
              float_at(L.cwt), float_at(L.grad_a), stream);
    if (st != kOk) return st;
    st = launch_pdl(gx_kern, dim3(unsigned((I + kGradThreads - 1) / kGradThreads),
                                  unsigned((int64_t(B) + kGradRows - 1) / kGradRows)),
                    kGradThreads, 0, stream, x, grid, static_cast<const float*>(float_at(L.grad_a)), int64_t(B), I, C,
                    K, grad_x);
    if (st != kOk) return st;
  }
  if (need_w) {
    cudaMemsetAsync(u32_at(L.amax_gt), 0, size_t(O) * 4, stream);
    cudaMemsetAsync(u32_at(L.amax_x), 0, size_t(I) * 4, stream);
    const unsigned chunks = unsigned((int64_t(B) + kColChunk - 1) / kColChunk);
    st = launch_pdl(colmax_kernel, dim3(unsigned((O + kColThreads - 1) / kColThreads), chunks), kColThreads,
                    0, stream, grad_out, int64_t(B), O, u32_at(L.amax_gt));
    if (st != kOk) return st;
    st = launch_pdl(split_cols_kernel, dim3(unsigned(bp / kTile), unsigned((O + kTile - 1) / kTile)), tb, 0, stream,
                    grad_out, B, O, bp, static_cast<const uint32_t*>(u32_at(L.amax_gt)), half_at(L.gt_hi),
                    half_at(L.gt_lo), float_at(L.rgt));
    if (st != kOk) return st;
    st = launch_pdl(colmax_kernel, dim3(unsigned((I + kColThreads - 1) / kColThreads), chunks), kColThreads, 0,
                    stream, x, int64_t(B), I, u32_at(L.amax_x));
    if (st != kOk) return st;
    st = launch_pdl(at_kern, dim3(unsigned((I + kTile - 1) / kTile), unsigned(bp / at_tile_rows(at_nk))), tb, at_sm, stream,
                    x, grid, B, I, C, K, bp, static_cast<const uint32_t*>(u32_at(L.amax_x)), half_at(L.at_hi),
                    half_at(L.at_lo), float_at(L.cat));
    if (st != kOk) return st;
    st = gemm(half_at(L.gt_hi), half_at(L.gt_lo), O, half_at(L.at_hi), half_at(L.at_lo), int(nkp), bp,
              float_at(L.rgt), float_at(L.cat), float_at(L.grad_w), stream);
    if (st != kOk) return st;
    st = launch_pdl(grad_w_kernel, unsigned((int64_t(O) * I + kGradThreads - 1) / kGradThreads), kGradThreads, 0,
                    stream, static_cast<const float*>(float_at(L.grad_w)), sw, sc, int64_t(O), I, C, grad_wb,
                    grad_sw, grad_sc);
  }
  return st;
}

}  // namespace kanb
}  // namespace b200
