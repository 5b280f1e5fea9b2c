// FP8 E4M3 linear layer: out[M, N] (bf16) = (x_q[M, K] . w_q[N, K]^T) / (scale_x * scale_w) + bias.
//
// Reference semantics: tasks/fp8_linear/reference.py:34-37 (fp64 oracle :44-45: dequantise by
// dividing by the per-tensor scales, fp64 matmul plus bias, one rounding to bf16) and
// tasks/fp8_linear/prompt.md "Computation".  The drop-in boundary it replaces is
// `void reference(const int32_t M, const int32_t K, const int32_t N, const __nv_fp8_e4m3* x_fp8,
// float scale_x, const __nv_fp8_e4m3* w_fp8, float scale_w, const __nv_bfloat16* bias,
// __nv_bfloat16* output)` (tasks/fp8_linear/tests/task.json:3; expert launcher
// reference/fp8_linear/solution.cu:276-320, which calls cuBLASLt).
//
// B200 design (tensor path, K a multiple of 16 and 16-byte aligned operands):
//   - one persistent CTA per SM walks output tiles of 128 x BN in grouped order (kGroupM row
//     blocks share each sweep over column blocks, so both operands stay L2-resident);
//   - warp 0: one thread issues 128-byte-swizzled TMA tile loads of x and w (both K-major) into a
//     STAGES-deep shared-memory ring (every CTA loads its own tiles);
//   - warp 1: allocates 2*BN TMEM columns (two fp32 accumulators) and one thread issues
//     tcgen05.mma kind::f8f6f4 (E4M3 x E4M3 -> fp32, 128 x BN x 32 per instruction), committing
//     each stage back to the loader and each finished accumulator to the epilogue;
//   - warps 2-9: epilogue; tcgen05.ld the accumulator (one TMEM lane quarter and one half of the
//     columns per warp, one output row per thread), fused acc * (1/(sx*sw)) + bias, round to
//     bf16; it drains one accumulator while the MMAs fill the other.  For BN >= 128 each warp
//     stages 32 rows x 64 columns through a bank-conflict-free 4 KB shared-memory block so a
//     128-bit store instruction writes four whole 128-byte row segments (store_packed64_staged);
//     stored from registers, each instruction touched 32 rows.  The bias of a tile's columns is
//     loaded before its accumulator is ready.  Measured on M = 2048, N = 4096, K = 1024 (one or
//     two tiles per CTA): 16.1 us with four epilogue warps storing from registers, 8.7 us with the
//     stores removed, 14.9 us with eight warps, 13.9 us staged, 11.3 us with the bias loaded early.
// Small problems take BN = 128 or 64 so more SMs get tiles; M <= 64 swaps the operands and splits
// K over a cluster (gemv_kernel).  Other shapes (K not a multiple of 16, unaligned operands) take a
// shared-memory tiled CUDA-core kernel with the same arithmetic.
#pragma once

#include <cuda_bf16.h>
#include <math.h>

#include <mutex>

#include "../common/b200_common.cuh"
#include "../common/bulk.cuh"
#include "../common/tcgen05.cuh"

namespace b200 {
namespace fp8 {

constexpr int kBM = 128;       // rows of x per tile (UMMA M)
constexpr int kBK = 128;       // bytes (= elements) of K per stage: one 128-byte swizzle row
constexpr int kUmmaK = 32;     // K per tcgen05.mma for 8-bit operands
constexpr int kThreads = 192;  // small-M kernel: warp 0 loads, warp 1 issues MMAs, warps 2-5 epilogue
constexpr int kThreadsG = 320; // 128-row tiles: warp 0 loads, warp 1 issues MMAs, warps 2-9 epilogue
constexpr int kGroupM = 8;

template <int BN>
struct Cfg {
  static constexpr int kATile = kBM * kBK;
  static constexpr int kBTile = BN * kBK;
  static constexpr int kStage = kATile + kBTile;
  static constexpr int kStages = (192 * 1024) / kStage;
  static constexpr int kTmemCols = 2 * BN;
  // Per-epilogue-warp staging of 32 rows x 64 bf16 columns (4 KB each, eight warps) for BN >= 128.
  static constexpr int kStageOut = BN >= 128 ? 8 * 4096 : 0;
  static constexpr int kSmem = kStages * kStage + kStageOut + 1024;  // + alignment slack for the 1024 B atoms
};

__device__ __forceinline__ void tile_coords(int tile, int n_m, int n_n, int& mb, int& nb) {
  const int group = kGroupM * n_n;
  const int g = tile / group;
  const int first = g * kGroupM;
  const int gm = min(n_m - first, kGroupM);
  const int r = tile - g * group;
  mb = first + r % gm;
  nb = r / gm;
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Epilogue of 32 consecutive columns n0..n0+31 of one output row.
__device__ __forceinline__ void store_row32(const uint32_t (&r)[32], int row, int n0, int M, int N, float scale,
                                            const uint16_t* __restrict__ bias, uint16_t* __restrict__ out,
                                            bool vec_ok) {
  if (row >= M) return;
  uint16_t* o = out + int64_t(row) * N + n0;
  if (vec_ok && n0 + 32 <= N) {
    uint32_t p[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float v0 = fmaf(__uint_as_float(r[2 * j]), scale, bf16_bits_to_float(__ldg(bias + n0 + 2 * j)));
      const float v1 = fmaf(__uint_as_float(r[2 * j + 1]), scale, bf16_bits_to_float(__ldg(bias + n0 + 2 * j + 1)));
      p[j] = pack_bf16x2(v0, v1);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4*>(o + 8 * j) = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (n0 + j < N) {
        const float v = fmaf(__uint_as_float(r[j]), scale, bf16_bits_to_float(__ldg(bias + n0 + j)));
        o[j] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
      }
    }
  }
}

// The bias of the 64 columns n0 .. n0+63 as 32 bf16 pairs (zero past N); bias_vec: bias 16-byte
// aligned.  Loaded before the accumulator is ready, so its latency hides behind the MMAs (at
// M = 2048 N = 4096 K = 1024: 13.9 -> 11.3 us, the epilogue having waited on it after every
// accumulator read).
__device__ __forceinline__ void load_bias64(const uint16_t* __restrict__ bias, int n0, int N, bool bias_vec,
                                            uint32_t (&bw)[32]) {
  const int nb = N - n0 < 64 ? N - n0 : 64;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
#pragma unroll
    for (int j = 0; j < 4; ++j) bw[4 * c + j] = 0u;
    if (8 * c < nb) {
      if (bias_vec) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(bias + n0) + c);
        bw[4 * c] = v.x;
        bw[4 * c + 1] = v.y;
        bw[4 * c + 2] = v.z;
        bw[4 * c + 3] = v.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          bw[4 * c + j] = uint32_t(__ldg(bias + n0 + 8 * c + 2 * j)) |
                          (uint32_t(__ldg(bias + n0 + 8 * c + 2 * j + 1)) << 16);
      }
    }
  }
}

// Epilogue of 64 consecutive columns n0..n0+63 for a warp's 32 rows row0..row0+31 (this lane's
// accumulator row is row0 + lane: r0 holds its columns 0-31, r1 columns 32-63).  pack_row64
// scales, biases and rounds the lane's row to bf16 pairs (store_row32's arithmetic; bw from
// load_bias64); store_packed64_staged writes the warp's rows through its 4 KB staging area so that
// each 128-bit global store instruction writes four whole 128-byte row segments instead of 32
// scattered 16-byte pieces.  Staging layout: row r at byte 128 r, its 16-byte chunk c at
// ((c ^ (r & 7)) * 16), so the writes (a lane's 8 chunks of its row) and the reads (8 lanes per
// row) are both free of bank conflicts.  N % 8 == 0 and out 16-byte aligned.
__device__ __forceinline__ void pack_row64(const uint32_t (&r0)[32], const uint32_t (&r1)[32], float scale,
                                           const uint32_t (&bw)[32], uint32_t (&p)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int e = 2 * j;  // column within the block
    const uint32_t a0 = e < 32 ? r0[e] : r1[e - 32], a1 = e < 32 ? r0[e + 1] : r1[e - 31];
    p[j] = pack_bf16x2(fmaf(__uint_as_float(a0), scale, __uint_as_float(bw[j] << 16)),
                       fmaf(__uint_as_float(a1), scale, __uint_as_float(bw[j] & 0xffff0000u)));
  }
}

__device__ __forceinline__ void store_packed64_staged(const uint32_t (&p)[32], int row0, int lane, int n0, int M,
                                                      int N, uint16_t* __restrict__ out, uint8_t* stage) {
  const int nb = N - n0 < 64 ? N - n0 : 64;  // columns of this block inside the output (multiple of 8)
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<uint4*>(stage + lane * 128 + ((c ^ (lane & 7)) << 4)) =
        make_uint4(p[4 * c], p[4 * c + 1], p[4 * c + 2], p[4 * c + 3]);
  __syncwarp();
  const int c = lane & 7;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int rr = 4 * k + (lane >> 3);
    const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * 128 + ((c ^ (rr & 7)) << 4));
    const int row = row0 + rr;
    if (row < M && 8 * c < nb) *reinterpret_cast<uint4*>(out + int64_t(row) * N + n0 + 8 * c) = v;
  }
  __syncwarp();
}

// Operands of at most kPrefetchBytes together are brought into L2 at kernel start, before the
// wait for the previous kernel: each CTA asks for its 1/gridDim share of x and w (contiguous
// [M, K] and [N, K] bytes), so a call whose operands are not yet in L2 streams them from HBM at
// the full rate while the tile pipeline starts, instead of at the rate of the first tiles' TMA
// loads.  L2 is the point of coherence, so this is safe even when the previous kernel writes them.
constexpr int64_t kPrefetchBytes = int64_t(48) << 20;

__device__ __forceinline__ void prefetch_share(const uint8_t* x, int64_t xb, const uint8_t* w, int64_t wb) {
#if B200_TCGEN05
  const int64_t total = xb + wb;
  if (total == 0 || total > kPrefetchBytes) return;
  const int64_t share = ((total + gridDim.x - 1) / gridDim.x + 15) & ~int64_t(15);
  int64_t lo = int64_t(blockIdx.x) * share;
  const int64_t hi = lo + share < total ? lo + share : total;
  while (lo < hi) {
    const bool in_x = lo < xb;
    const int64_t seg_end = in_x ? (xb < hi ? xb : hi) : hi;
    const uint8_t* p = in_x ? x + lo : w + (lo - xb);
    const int64_t n = seg_end - lo;
    if (n >= 16) tc::prefetch_l2(p, uint32_t(n & ~int64_t(15)));
    lo = seg_end;
  }
#endif
}

template <int BN>
__global__ void __launch_bounds__(kThreadsG, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N, int K,
                float scale, const float* __restrict__ scale_ptr, const uint16_t* __restrict__ bias,
                uint16_t* __restrict__ out, int vec_ok, const uint8_t* pf_x, const uint8_t* pf_w) {
  if (threadIdx.x == 0) prefetch_share(pf_x, pf_x ? int64_t(M) * K : 0, pf_w, pf_w ? int64_t(N) * K : 0);
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  if (scale_ptr != nullptr) scale = *scale_ptr;  // written on the device by the quantisation kernels
  using C = Cfg<BN>;
  constexpr int S = C::kStages;
#if !B200_TCGEN05
  if (threadIdx.x == 0) atomicOr(&g_b200_fault, kFaultNoTensorCore);
  return;
#else
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[S], empty[S], tfull[2], tempty[2];
  __shared__ uint32_t tmem_base_s;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_m = (M + kBM - 1) / kBM, n_n = (N + BN - 1) / BN, n_tiles = n_m * n_n;
  const int nkb = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tensormap(&tmA);
    tc::prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tc::tmem_alloc(&tmem_base_s, C::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      uint32_t kb_all = 0;
      for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, n_m, n_n, mb, nb);
        for (int kb = 0; kb < nkb; ++kb, ++kb_all) {
          const uint32_t s = kb_all % S, ph = (kb_all / S) & 1u;
          mbar_wait(&empty[s], ph ^ 1u);
          mbar_arrive_expect_tx(&full[s], C::kStage);
          uint8_t* a = smem + s * C::kStage;
          tc::tma_load_2d(a, &tmA, kb * kBK, mb * kBM, &full[s]);
          tc::tma_load_2d(a + C::kATile, &tmB, kb * kBK, nb * BN, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      const uint32_t id = tc::idesc(kBM, BN, 0);
      uint32_t kb_all = 0, it = 0;
      for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
        const uint32_t acc = it & 1u, aph = (it >> 1) & 1u;
        mbar_wait(&tempty[acc], aph ^ 1u);
        tc::fence_after_sync();
        const uint32_t d = tmem + acc * BN;
        for (int kb = 0; kb < nkb; ++kb, ++kb_all) {
          const uint32_t s = kb_all % S, ph = (kb_all / S) & 1u;
          mbar_wait(&full[s], ph);
          tc::fence_after_sync();
          const uint32_t a_addr = smem_addr(smem + s * C::kStage);
          const uint64_t ad = tc::sdesc_kmajor_sw128(a_addr);
          const uint64_t bd = tc::sdesc_kmajor_sw128(a_addr + C::kATile);
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k)
            tc::mma_f8(d, ad + uint64_t((k * kUmmaK) >> 4), bd + uint64_t((k * kUmmaK) >> 4), id,
                       (kb | k) != 0 ? 1u : 0u);
          tc::mma_commit(&empty[s]);
        }
        tc::mma_commit(&tfull[acc]);
      }
    }
  } else {  // epilogue warps 2..9: warp w reads TMEM lanes [32*(w%4), 32*(w%4)+32), column half (w-2)/4
    const int q = warp & 3, h = (warp - 2) >> 2;
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      int mb, nb;
      tile_coords(tile, n_m, n_n, mb, nb);
      const uint32_t acc = it & 1u, aph = (it >> 1) & 1u;
      const int row = mb * kBM + q * 32 + lane;
      if (BN >= 128 && (vec_ok & 1)) {
        // The bias of this warp's columns, loaded while the MMAs still run (the staged epilogue
        // was otherwise waiting on it after every accumulator read).
        constexpr int kBlocks = BN >= 128 ? BN / 128 : 1;
        uint32_t bw[kBlocks][32];
#pragma unroll
        for (int c64 = 0; c64 < kBlocks; ++c64)
          load_bias64(bias, nb * BN + h * (BN / 2) + c64 * 64, N, (vec_ok & 2) != 0, bw[c64]);
        mbar_wait(&tfull[acc], aph);
        tc::fence_after_sync();
        uint8_t* stage = smem + S * C::kStage + (warp - 2) * 4096;
#pragma unroll
        for (int c64 = 0; c64 < kBlocks; ++c64) {
          const int col = h * (BN / 2) + c64 * 64;
          if (nb * BN + col >= N) break;
          uint32_t r0[32], r1[32], pk[32];
          tc::tmem_ld32(tmem + (uint32_t(q * 32) << 16) + acc * BN + uint32_t(col), r0);
          tc::tmem_ld32(tmem + (uint32_t(q * 32) << 16) + acc * BN + uint32_t(col + 32), r1);
          tc::tmem_ld_wait();
          pack_row64(r0, r1, scale, bw[c64], pk);
          store_packed64_staged(pk, mb * kBM + q * 32, lane, nb * BN + col, M, N, out, stage);
        }
      } else {
        mbar_wait(&tfull[acc], aph);
        tc::fence_after_sync();
#pragma unroll 1
        for (int cc = h * (BN / 64); cc < (h + 1) * (BN / 64); ++cc) {
          uint32_t r[32];
          tc::tmem_ld32(tmem + (uint32_t(q * 32) << 16) + acc * BN + uint32_t(cc * 32), r);
          tc::tmem_ld_wait();
          store_row32(r, row, nb * BN + cc * 32, M, N, scale, bias, out, (vec_ok & 1) != 0);
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, C::kTmemCols);
  }
#endif
}

// ------------------------------------------------------------- large shapes: 256 x 256 tiles
// A CTA's operand bandwidth from L2 (about 100 GB/s per SM here) caps a 128 x 256 tile at ~175
// flop per staged byte, below the E4M3 rate.  For large problems each CTA computes a 256 x 256
// tile as two M = 128 MMAs that share one 256-row B tile (262 flop per staged byte): A and B are
// each one 256-row TMA box per stage, the two fp32 accumulators fill all 512 TMEM columns (one
// tile at a time; the MMAs of the next tile wait for the epilogue), and eight epilogue warps
// drain them, two per TMEM lane quarter (warps 2-5 the upper 128 rows, warps 6-9 the lower).
// Each epilogue thread reads and rounds its whole 256-column row (bias from shared memory, staged
// there while the MMAs run), releases TMEM, and only then stores, through the staging area, while
// the next tile's MMAs run: the next tile waits for the accumulator reads, not for the stores
// (16384 x 28672 x 8192: about 8 % faster, interleaved runs on one box).
constexpr int kBM2 = 256;          // rows of x per tile (two UMMAs of 128)
constexpr int kBN2 = 256;          // columns (rows of w) per tile
constexpr int kThreads2 = 320;     // warp 0 loads, warp 1 issues MMAs, warps 2-9 epilogue
struct Cfg2 {
  static constexpr int kATile = kBM2 * kBK;
  static constexpr int kBTile = kBN2 * kBK;
  static constexpr int kStage = kATile + kBTile;  // 64 KB
  static constexpr int kStages = (200 * 1024) / kStage;
  static constexpr int kTmemCols = 512;
  static constexpr int kStageOut = 8 * 4096;  // per-epilogue-warp staging of 32 rows x 64 columns
  static constexpr int kSmem = kStages * kStage + kStageOut + 1024;
};

__global__ void __launch_bounds__(kThreads2, 1)
    gemm256_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
                   int K, float scale, const float* __restrict__ scale_ptr, const uint16_t* __restrict__ bias,
                   uint16_t* __restrict__ out, int vec_ok, const uint8_t* pf_x, const uint8_t* pf_w) {
  if (threadIdx.x == 0) prefetch_share(pf_x, pf_x ? int64_t(M) * K : 0, pf_w, pf_w ? int64_t(N) * K : 0);
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  if (scale_ptr != nullptr) scale = *scale_ptr;
  using C = Cfg2;
  constexpr int S = C::kStages;
#if !B200_TCGEN05
  if (threadIdx.x == 0) atomicOr(&g_b200_fault, kFaultNoTensorCore);
  return;
#else
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[S], empty[S], tfull, tempty;
  __shared__ uint32_t tmem_base_s;
  __shared__ uint32_t s_bias[2][kBN2 / 2];  // a tile's bias as bf16 pairs, by tile parity
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_m = (M + kBM2 - 1) / kBM2, n_n = (N + kBN2 - 1) / kBN2, n_tiles = n_m * n_n;
  const int nkb = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&tfull, 1);
    mbar_init(&tempty, 8);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tensormap(&tmA);
    tc::prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tc::tmem_alloc(&tmem_base_s, C::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer (a wait that gives up ends this role: no tile after it)
      uint32_t kb_all = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, n_m, n_n, mb, nb);
        for (int kb = 0; kb < nkb; ++kb, ++kb_all) {
          const uint32_t s = kb_all % S, ph = (kb_all / S) & 1u;
          if (!(ok = mbar_wait(&empty[s], ph ^ 1u))) break;
          mbar_arrive_expect_tx(&full[s], C::kStage);
          uint8_t* a = smem + s * C::kStage;
          tc::tma_load_2d(a, &tmA, kb * kBK, mb * kBM2, &full[s]);
          tc::tma_load_2d(a + C::kATile, &tmB, kb * kBK, nb * kBN2, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer: D0 (rows 0-127) at column 0, D1 (rows 128-255) at column 256
      const uint32_t id = tc::idesc(128, kBN2, 0);
      uint32_t kb_all = 0, it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++it) {
        ok = mbar_wait(&tempty, (it & 1u) ^ 1u);  // the epilogue has drained the previous tile
        tc::fence_after_sync();
        for (int kb = 0; kb < nkb && ok; ++kb, ++kb_all) {
          const uint32_t s = kb_all % S, ph = (kb_all / S) & 1u;
          if (!(ok = mbar_wait(&full[s], ph))) break;
          tc::fence_after_sync();
          const uint32_t a_addr = smem_addr(smem + s * C::kStage);
          const uint64_t a0 = tc::sdesc_kmajor_sw128(a_addr);
          const uint64_t a1 = tc::sdesc_kmajor_sw128(a_addr + 128 * kBK);
          const uint64_t bd = tc::sdesc_kmajor_sw128(a_addr + C::kATile);
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            const uint64_t ko = uint64_t((k * kUmmaK) >> 4);
            const uint32_t acc = (kb | k) != 0 ? 1u : 0u;
            tc::mma_f8(tmem, a0 + ko, bd + ko, id, acc);
            tc::mma_f8(tmem + 256u, a1 + ko, bd + ko, id, acc);
          }
          tc::mma_commit(&empty[s]);
        }
        tc::mma_commit(&tfull);
      }
    }
  } else {  // epilogue warps 2..9: warp w reads TMEM lanes of quarter w % 4; w < 6: D0, else D1
    const int q = warp & 3, half = warp < 6 ? 0 : 1;
    const bool staged = (vec_ok & 1) != 0;
    uint8_t* stage = smem + S * C::kStage + (warp - 2) * 4096;
    const int et = int(threadIdx.x) - 64;  // 0 .. 255 over the epilogue warps
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
      int mb, nb;
      tile_coords(tile, n_m, n_n, mb, nb);
      const int n0 = nb * kBN2;
      if (staged) {
        // The tile's bias into shared memory while its MMAs run (one pair per thread of the first
        // 128); the epilogue warps' barrier makes it visible, and the parity buffers keep a fast
        // warp's next tile from overwriting what a slow warp still reads.
        if (et < kBN2 / 2) {
          const int c = n0 + 2 * et;
          uint32_t v = 0u;
          if (c < N)
            v = (vec_ok & 2) ? __ldg(reinterpret_cast<const uint32_t*>(bias + c))
                             : uint32_t(__ldg(bias + c)) | (uint32_t(__ldg(bias + c + 1)) << 16);
          s_bias[it & 1u][et] = v;
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
      }
      if (!mbar_wait(&tfull, it & 1u)) break;
      tc::fence_after_sync();
      const int row = mb * kBM2 + half * 128 + q * 32 + lane;
      if (staged) {
        // Read and round the whole accumulator row first, then free TMEM for the next tile's MMAs,
        // then store through the staging area while they run.
        uint32_t pk[kBN2 / 2];
#pragma unroll
        for (int cc = 0; cc < kBN2 / 32; ++cc) {
          uint32_t r[32];
          tc::tmem_ld32(tmem + (uint32_t(q * 32) << 16) + uint32_t(half * 256 + cc * 32), r);
          tc::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const uint32_t bw = s_bias[it & 1u][cc * 16 + j];
            pk[cc * 16 + j] = pack_bf16x2(fmaf(__uint_as_float(r[2 * j]), scale, __uint_as_float(bw << 16)),
                                          fmaf(__uint_as_float(r[2 * j + 1]), scale, __uint_as_float(bw & 0xffff0000u)));
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty);
#pragma unroll
        for (int b = 0; b < kBN2 / 64; ++b) {
          uint32_t pb[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) pb[j] = pk[32 * b + j];
          if (n0 + 64 * b < N) store_packed64_staged(pb, mb * kBM2 + half * 128 + q * 32, lane, n0 + 64 * b, M, N, out, stage);
        }
      } else {
#pragma unroll 1
        for (int cc = 0; cc < kBN2 / 32; ++cc) {
          uint32_t r[32];
          tc::tmem_ld32(tmem + (uint32_t(q * 32) << 16) + uint32_t(half * 256 + cc * 32), r);
          tc::tmem_ld_wait();
          store_row32(r, row, n0 + cc * 32, M, N, scale, bias, out, false);
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, C::kTmemCols);
  }
#endif
}

// ------------------------------------------------------------------ small M: swap-AB, split-K
// For M <= 64 the W stream dominates and a 128-row tile of x would be mostly padding.  The MMA
// roles swap: a CTA computes D^T[128 rows of W, BNX >= M columns] = W_tile . x^T with
// tcgen05.mma M = 128, N = BNX, and a cluster of SK CTAs splits K between them.  Each CTA
// accumulates its K range in TMEM; the 128 rows are divided among the cluster's ranks, and each
// epilogue thread stores its row's fp32 partial straight into the owning rank's shared memory
// (distributed shared memory stores, one slot per source rank, beside the stage ring).  After one
// cluster barrier every rank adds its rows' SK partials in rank order, applies scale and bias and
// writes out[m][n].  Pushing instead of having one CTA pull the others' tiles removes the remote
// round trips and spreads the sums over the cluster (M = 16: 9.0 -> 7.7 us, M = 64: 15.8 -> 10.6 us
// with W streamed from HBM).  W is read once from HBM; the small x tile is read by every CTA (L2).
// No multicast.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_cluster_smem(uint32_t smem_byte_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_byte_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
__device__ __forceinline__ void st_cluster_f4(uint32_t cluster_addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}

constexpr int kMaxSplit = 8;  // CTAs per cluster of the small-M kernel (the portable cluster size)

template <int BNX>
struct SmallCfg {
  static constexpr int kATile = kBM * kBK;   // 128 rows of W x 128 bytes of K
  static constexpr int kBTile = BNX * kBK;   // BNX rows of x x 128 bytes of K
  static constexpr int kStage = kATile + kBTile;
  // Incoming partial rows from the cluster's CTAs: [kMaxSplit][rows per owner][BNX] fp32, beside
  // the stage ring (peers write it while this CTA's MMAs may still read the ring).
  static constexpr int kInBytes = ((kBM + kMaxSplit) * BNX * 4 + 1023) / 1024 * 1024;
  static constexpr int kStages = (192 * 1024 - kInBytes) / kStage;
  static constexpr int kTmemCols = BNX < 32 ? 32 : BNX;
  static constexpr int kSmem = kStages * kStage + kInBytes + 1024;
  static_assert(kStage % 1024 == 0, "stages keep the 1024-byte swizzle-atom alignment");
};

// grid = (SK, ceil(N / 128)), cluster (SK, 1, 1).  tmW: map over w [N, K], 128-row box; tmX: map
// over x [M, K], BNX-row box.
template <int BNX>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, int M, int N, int K,
                float scale, const float* __restrict__ scale_ptr, const uint16_t* __restrict__ bias,
                uint16_t* __restrict__ out) {
  using C = SmallCfg<BNX>;
  constexpr int S = C::kStages;
#if !B200_TCGEN05
  if (threadIdx.x == 0) atomicOr(&g_b200_fault, kFaultNoTensorCore);
  return;
#else
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full[S], empty[S], tfull;
  __shared__ uint32_t tmem_base_s;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* in_rows = reinterpret_cast<float*>(smem + S * C::kStage);  // incoming partial rows
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank(), SK = gridDim.x;
  const int nb = blockIdx.y;
  const int nkb = (K + kBK - 1) / kBK;
  const int kb0 = int((int64_t(nkb) * rank) / SK), kb1 = int((int64_t(nkb) * (rank + 1)) / SK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&tfull, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tensormap(&tmW);
    tc::prefetch_tensormap(&tmX);
  }
  if (warp == 1) {
    tc::tmem_alloc(&tmem_base_s, C::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_base_s;
  cluster_arrive_relaxed();  // waited on just before the first distributed shared memory store
  // The set-up above touches no global memory, so it runs before the wait for the previous kernel
  // (on an SM the previous call's CTA has left, while its other CTAs finish: M = 16 7.7 -> 7.2 us;
  // the same order in the large-tile kernels made M = 2048 K = 1024 slower, 13.8 -> 15.4 us).
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  if (scale_ptr != nullptr) scale = *scale_ptr;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer over this CTA's K range
      for (int kb = kb0, i = 0; kb < kb1; ++kb, ++i) {
        const uint32_t s = uint32_t(i) % S, ph = (uint32_t(i) / S) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u)) break;
        mbar_arrive_expect_tx(&full[s], C::kStage);
        uint8_t* a = smem + s * C::kStage;
        tc::tma_load_2d(a, &tmW, kb * kBK, nb * kBM, &full[s]);
        tc::tma_load_2d(a + C::kATile, &tmX, kb * kBK, 0, &full[s]);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      const uint32_t id = tc::idesc(kBM, BNX, 0);
      for (int kb = kb0, i = 0; kb < kb1; ++kb, ++i) {
        const uint32_t s = uint32_t(i) % S, ph = (uint32_t(i) / S) & 1u;
        if (!mbar_wait(&full[s], ph)) break;
        tc::fence_after_sync();
        const uint32_t a_addr = smem_addr(smem + s * C::kStage);
        const uint64_t ad = tc::sdesc_kmajor_sw128(a_addr);
        const uint64_t bd = tc::sdesc_kmajor_sw128(a_addr + C::kATile);
#pragma unroll
        for (int k = 0; k < kBK / kUmmaK; ++k)
          tc::mma_f8(tmem, ad + uint64_t((k * kUmmaK) >> 4), bd + uint64_t((k * kUmmaK) >> 4), id,
                     (i | k) != 0 ? 1u : 0u);
        tc::mma_commit(&empty[s]);
      }
      tc::mma_commit(&tfull);  // also when this CTA's K range is empty (then nothing is added)
    }
    __syncwarp();
  } else {  // epilogue warps 2..5: warp w holds TMEM lanes (W rows) [32*(w%4), 32*(w%4)+32)
    const int q = warp & 3, r = q * 32 + lane;
    const bool have_k = kb1 > kb0;
    if (have_k) {
      mbar_wait(&tfull, 0u);
      tc::fence_after_sync();
    }
    float v[BNX];
#pragma unroll
    for (int c0 = 0; c0 < BNX; c0 += 32) {
      uint32_t t[32];
      if (have_k) {
        tc::tmem_ld32(tmem + (uint32_t(q * 32) << 16) + uint32_t(c0), t);
        tc::tmem_ld_wait();
      }
#pragma unroll
      for (int j = 0; j < 32 && c0 + j < BNX; ++j) v[c0 + j] = have_k ? __uint_as_float(t[j]) : 0.f;
    }
    // Push this row's partial to the CTA that owns the row (rows [o * RP, (o + 1) * RP) belong to
    // cluster rank o), into slot `rank` of its incoming rows: remote stores, no round trip.
    cluster_wait();  // every CTA of the cluster has started (the arrive is at the end of set-up)
    const int RP = (kBM + int(SK) - 1) / int(SK), owner = r / RP;
    const uint32_t dst = map_cluster_smem(smem_addr(in_rows + (int(rank) * RP + (r - owner * RP)) * BNX),
                                          uint32_t(owner));
#pragma unroll
    for (int j = 0; j < BNX; j += 4) st_cluster_f4(dst + uint32_t(j) * 4u, make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
  }
  if (warp < 2) cluster_wait();
  cluster_sync_all();  // every CTA's pushes have landed in their owners' shared memory
  if (warp >= 2) {
    // This CTA's rows: the ranks' partials added in rank order (the same sum on every call), then
    // scale, bias and bf16.  Thread t takes rows t, t + 128, ... of its RP x ceil(BNX/4) items,
    // rows fastest so the output stores of a column run along n.
    const int RP = (kBM + int(SK) - 1) / int(SK);
    const int r0 = int(rank) * RP, rows = min(RP, kBM - r0);
    const int t = threadIdx.x - 64;
    for (int it = t; it < rows * (BNX / 4); it += 128) {
      const int rl = it % rows, c4 = it / rows;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (uint32_t k = 0; k < SK; ++k) {
        const float4 p = *reinterpret_cast<const float4*>(in_rows + (int(k) * RP + rl) * BNX + 4 * c4);
        acc.x += p.x;
        acc.y += p.y;
        acc.z += p.z;
        acc.w += p.w;
      }
      const int n = nb * kBM + r0 + rl;
      if (n < N) {
        const float bv = bf16_bits_to_float(__ldg(bias + n));
        const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = 4 * c4 + e;
          if (j < M) out[int64_t(j) * N + n] = __bfloat16_as_ushort(__float2bfloat16_rn(fmaf(a4[e], scale, bv)));
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, C::kTmemCols);
  }
#endif
}

// ------------------------------------------------------------------------ CUDA-core fallback
// 64 x 64 output tiles, 256 threads, each thread a 4 x 4 block; K in steps of 32 through shared
// memory, E4M3 bytes decoded with a 256-entry table built from the format definition (sign,
// 4 exponent bits with bias 7, 3 mantissa bits; exponent 0 subnormal; S.1111.111 NaN).
__device__ __forceinline__ float e4m3_value(unsigned b) {
  const unsigned e = (b >> 3) & 15u, m = b & 7u;
  float v;
  if (e == 15u && m == 7u) v = __int_as_float(0x7fc00000);
  else if (e == 0u) v = float(m) * 0.001953125f;  // m/8 * 2^-6
  else v = __uint_as_float(((e + 120u) << 23) | (m << 20));  // (1 + m/8) * 2^(e-7)
  return (b & 0x80u) ? -v : v;
}

__global__ void __launch_bounds__(256) simt_kernel(int M, int N, int K, const uint8_t* __restrict__ x,
                                                   const uint8_t* __restrict__ w, float scale,
                                                   const float* __restrict__ scale_ptr,
                                                   const uint16_t* __restrict__ bias, uint16_t* __restrict__ out) {
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  if (scale_ptr != nullptr) scale = *scale_ptr;
  __shared__ float lut[256];
  __shared__ float xs[32][65], ws[32][65];
  lut[threadIdx.x] = e4m3_value(threadIdx.x);
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  __syncthreads();
  for (int k0 = 0; k0 < K; k0 += 32) {
    for (int i = threadIdx.x; i < 64 * 32; i += 256) {
      const int r = i >> 5, kk = i & 31;
      const int gm = m0 + r, gn = n0 + r, gk = k0 + kk;
      xs[kk][r] = (gm < M && gk < K) ? lut[x[int64_t(gm) * K + gk]] : 0.f;
      ws[kk][r] = (gn < N && gk < K) ? lut[w[int64_t(gn) * K + gk]] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = xs[kk][ty * 4 + i];
        b[i] = ws[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn < N) {
        const float v = fmaf(acc[i][j], scale, bf16_bits_to_float(bias[gn]));
        out[int64_t(gm) * N + gn] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
      }
    }
  }
}

// ------------------------------------------------------------------------------------- host
struct MapKey {
  const void* a;
  const void* b;
  int rows_a, rows_b, K, box_a, box_b;
};

struct MapEntry {
  MapKey key;
  CUtensorMap a, b;
  int dev;
  bool used = false;
};

// A few recently used tensor-map pairs (operand A [rows_a, K] with box_a-row boxes, operand B
// [rows_b, K] with box_b-row boxes): a repeated call at the same pointers skips the host-side
// encoding.
inline bool get_maps(const void* pa, const void* pb, int rows_a, int rows_b, int K, int box_a, int box_b,
                     CUtensorMap* a, CUtensorMap* b) {
  static MapEntry cache[8];
  static int next = 0;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  const MapKey k{pa, pb, rows_a, rows_b, K, box_a, box_b};
  std::lock_guard<std::mutex> lock(mu);
  for (auto& e : cache) {
    if (e.used && e.dev == dev && e.key.a == k.a && e.key.b == k.b && e.key.rows_a == k.rows_a &&
        e.key.rows_b == k.rows_b && e.key.K == k.K && e.key.box_a == k.box_a && e.key.box_b == k.box_b) {
      *a = e.a;
      *b = e.b;
      return true;
    }
  }
  MapEntry& e = cache[next];
  next = (next + 1) % 8;
  e.used = false;
  if (!tc::make_map_sw128(&e.a, pa, uint64_t(rows_a), uint64_t(K), 1, uint32_t(box_a))) return false;
  if (!tc::make_map_sw128(&e.b, pb, uint64_t(rows_b), uint64_t(K), 1, uint32_t(box_b))) return false;
  e.key = k;
  e.dev = dev;
  e.used = true;
  *a = e.a;
  *b = e.b;
  return true;
}

template <int BN>
inline int launch_tc(int M, int N, int K, const uint8_t* x, const uint8_t* w, float scale, const float* scale_ptr,
                     const uint16_t* bias, uint16_t* out, cudaStream_t stream) {
  CUtensorMap a, b;
  if (!get_maps(x, w, M, N, K, kBM, BN, &a, &b)) return kUnsupported;
  auto kern = gemm_kernel<BN>;
  if (!ensure_dyn_smem(kern, Cfg<BN>::kSmem)) return kCudaError;
  const int n_tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  const int grid = n_tiles < sm_count() ? n_tiles : sm_count();
  const int vec_ok = ((N % 8 == 0) && aligned16(out) ? 1 : 0) | (aligned16(bias) ? 2 : 0);
  launch_pdl(kern, grid, kThreadsG, Cfg<BN>::kSmem, stream, a, b, M, N, K, scale, scale_ptr, bias, out, vec_ok, x, w);
  return launch_status();
}

inline int launch_tc256(int M, int N, int K, const uint8_t* x, const uint8_t* w, float scale, const float* scale_ptr,
                        const uint16_t* bias, uint16_t* out, cudaStream_t stream) {
  CUtensorMap a, b;
  if (!get_maps(x, w, M, N, K, kBM2, kBN2, &a, &b)) return kUnsupported;
  if (!ensure_dyn_smem(gemm256_kernel, Cfg2::kSmem)) return kCudaError;
  const int n_tiles = ((M + kBM2 - 1) / kBM2) * ((N + kBN2 - 1) / kBN2);
  const int grid = n_tiles < sm_count() ? n_tiles : sm_count();
  const int vec_ok = ((N % 8 == 0) && aligned16(out) ? 1 : 0) | (aligned16(bias) ? 2 : 0);
  launch_pdl(gemm256_kernel, grid, kThreads2, Cfg2::kSmem, stream, a, b, M, N, K, scale, scale_ptr, bias, out,
             vec_ok, x, w);
  return launch_status();
}

// Split-K factor of the small-M kernel: enough clusters x CTAs to cover the SMs, at most 8 (the
// portable cluster size) and at most one CTA per 128-byte K block.
inline int small_split(int N, int K) {
  const int n_tiles = (N + kBM - 1) / kBM, nkb = (K + kBK - 1) / kBK;
  int sk = sm_count() / n_tiles;
  if (sk > kMaxSplit) sk = kMaxSplit;
  if (sk > nkb) sk = nkb;
  return sk < 1 ? 1 : sk;
}

template <int BNX>
inline int launch_small(int M, int N, int K, const uint8_t* x, const uint8_t* w, float scale, const float* scale_ptr,
                        const uint16_t* bias, uint16_t* out, cudaStream_t stream) {
  CUtensorMap mw, mx;
  if (!get_maps(w, x, N, M, K, kBM, BNX, &mw, &mx)) return kUnsupported;
  auto kern = gemv_kernel<BNX>;
  if (!ensure_dyn_smem(kern, SmallCfg<BNX>::kSmem)) return kCudaError;
  const int sk = small_split(N, K);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(sk), unsigned((N + kBM - 1) / kBM));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = SmallCfg<BNX>::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(sk);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, kern, mw, mx, M, N, K, scale, scale_ptr, bias, out) != cudaSuccess) return kCudaError;
  return launch_status();
}

// Which tensor-core tile width a shape uses (0 = CUDA-core fallback).
// 512 = the 256 x 256 tiles of gemm256_kernel, for problems with at least four waves of them.
inline int plan_bn(int M, int N, int K, const void* x, const void* w) {
  if (K % 16 != 0 || !aligned16(x) || !aligned16(w)) return 0;
#ifdef B200_FP8_FORCE_BN  // tuning builds only: one tile width for every tensor-core shape with M > 64
  if (M > 64) return B200_FP8_FORCE_BN;
#endif
  const int n_m = (M + kBM - 1) / kBM;
  const int sms = sm_count();
  if (((M + kBM2 - 1) / kBM2) * ((N + kBN2 - 1) / kBN2) >= 4 * sms) return 512;
  if (n_m * ((N + 255) / 256) >= (sms * 4) / 5) return 256;
  if (n_m * ((N + 127) / 128) >= sms / 2) return 128;
  return 64;
}

// scale_ptr (may be null): a device float holding 1 / (sx * sw), read by the kernel in place of the
// host-computed factor (the fused bf16 entry, whose activation scale is computed on the device).
inline int run(int32_t M, int32_t K, int32_t N, const uint8_t* x, float sx, const uint8_t* w, float sw,
               const uint16_t* bias, uint16_t* out, cudaStream_t stream, const float* scale_ptr = nullptr) {
  if (M < 0 || K < 0 || N < 0) return kInvalidArgument;
  if (M == 0 || N == 0) return kOk;
  if (out == nullptr || bias == nullptr || (K > 0 && (x == nullptr || w == nullptr))) return kInvalidArgument;
  const float scale = float(1.0 / (double(sx) * double(sw)));
  const int bn = K > 0 ? plan_bn(M, N, K, x, w) : 0;
  if (bn != 0 && M <= 64) {  // W-stream bound: swap-AB with split-K over a cluster
    if (M <= 16) return launch_small<16>(M, N, K, x, w, scale, scale_ptr, bias, out, stream);
    if (M <= 32) return launch_small<32>(M, N, K, x, w, scale, scale_ptr, bias, out, stream);
    return launch_small<64>(M, N, K, x, w, scale, scale_ptr, bias, out, stream);
  }
  if (bn == 512) return launch_tc256(M, N, K, x, w, scale, scale_ptr, bias, out, stream);
  if (bn == 256) return launch_tc<256>(M, N, K, x, w, scale, scale_ptr, bias, out, stream);
  if (bn == 128) return launch_tc<128>(M, N, K, x, w, scale, scale_ptr, bias, out, stream);
  if (bn == 64) return launch_tc<64>(M, N, K, x, w, scale, scale_ptr, bias, out, stream);
  dim3 grid((N + 63) / 64, (M + 63) / 64);
  launch_pdl(simt_kernel, grid, 256, 0, stream, M, N, K, x, w, scale, scale_ptr, bias, out);
  return launch_status();
}

// CUDA-core path only (used by tests to cross-check the tensor path on the same inputs).
inline int run_simt(int32_t M, int32_t K, int32_t N, const uint8_t* x, float sx, const uint8_t* w, float sw,
                    const uint16_t* bias, uint16_t* out, cudaStream_t stream) {
  if (M < 0 || K < 0 || N < 0) return kInvalidArgument;
  if (M == 0 || N == 0) return kOk;
  const float scale = float(1.0 / (double(sx) * double(sw)));
  dim3 grid((N + 63) / 64, (M + 63) / 64);
  launch_pdl(simt_kernel, grid, 256, 0, stream, M, N, K, x, w, scale, static_cast<const float*>(nullptr), bias, out);
  return launch_status();
}

}  // namespace fp8
}  // namespace b200
