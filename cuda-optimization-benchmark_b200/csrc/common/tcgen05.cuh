// Blackwell (sm_100a) tensor-core building blocks: TMA tensor loads, tensor memory (TMEM)
// allocation, UMMA shared-memory / instruction descriptors, tcgen05.mma issue and commit, and
// tcgen05.ld for epilogues.  Hand-written PTX; every encoding below follows the PTX ISA
// descriptions of the tcgen05 family (instruction descriptor: D format at bits 4-5, A/B formats
// at 7-9 / 10-12, K-major flags at 15/16, N>>3 at 17-22, M>>4 at 24-28; shared-memory
// descriptor: start>>4 at 0-13, leading byte offset>>4 at 16-29, stride byte offset>>4 at 32-45,
// version 1 at 46-47, swizzle mode at 61-63).
//
// Every TMA load here is issued by the CTA that uses the tile, for itself alone.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "bulk.cuh"

// tcgen05 instructions exist only in the architecture-specific sm_100a target.  A build such as
// `nvcc -arch=sm_100a` also emits generic compute_100 PTX for the same source; in that pass the
// wrappers below compile to nothing and the tensor-core kernels only record kFaultNoTensorCore.
// On a B200 the driver runs the sm_100a code, never that PTX.
#if defined(__CUDA_ARCH__) && !defined(__CUDA_ARCH_FEAT_SM100_ALL)
#define B200_TCGEN05 0
#else
#define B200_TCGEN05 1
#endif

namespace b200 {
namespace tc {

// ------------------------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor for a K-major operand tile stored the way a 128-byte-swizzled
// TMA load writes it: rows of 128 bytes, 8-row swizzle atoms of 1024 bytes stacked along M/N
// (stride byte offset 1024), tile base 1024-byte aligned.  Advancing along K inside the 128-byte
// row is done by adding (bytes >> 4) to the start-address field.
__device__ __forceinline__ uint64_t sdesc_kmajor_sw128(uint32_t smem_byte_addr) {
  return uint64_t((smem_byte_addr >> 4) & 0x3FFFu)  // start address
         | (uint64_t(1) << 16)                       // leading byte offset (unused for this mode)
         | (uint64_t(1024 >> 4) << 32)               // stride byte offset: 8 rows x 128 B
         | (uint64_t(1) << 46)                       // descriptor version (sm_100)
         | (uint64_t(2) << 61);                      // 128-byte swizzle
}

// Instruction descriptor: fp32 accumulator, A and B K-major, A/B format code `ab_fmt`
// (kind::f8f6f4: 0 = E4M3; kind::f16: 0 = F16, 1 = BF16), tile M x N.
__host__ __device__ constexpr uint32_t idesc(int M, int N, uint32_t ab_fmt) {
  return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// ------------------------------------------------------------------------------------- TMEM
// Warp-wide: allocate `ncols` (power of two >= 32) TMEM columns; the base address is written to
// *smem_dst.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
#if B200_TCGEN05
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(smem_dst)),
               "r"(ncols)
               : "memory");
#endif
}
__device__ __forceinline__ void tmem_relinquish() {
#if B200_TCGEN05
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
#endif
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
#if B200_TCGEN05
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
#endif
}

__device__ __forceinline__ void fence_before_sync() {
#if B200_TCGEN05
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
#endif
}
__device__ __forceinline__ void fence_after_sync() {
#if B200_TCGEN05
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#endif
}

// --------------------------------------------------------------------------------------- MMA
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, issued by one thread.
__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t id,
                                       uint32_t accumulate) {
#if B200_TCGEN05
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(id), "r"(accumulate)
      : "memory");
#endif
}
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t id,
                                        uint32_t accumulate) {
#if B200_TCGEN05
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(id), "r"(accumulate)
      : "memory");
#endif
}

// Arrive on `bar` once every MMA previously issued by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
#if B200_TCGEN05
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
#endif
}

// ------------------------------------------------------------------------------ TMEM -> regs
// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (base lane + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
#if B200_TCGEN05
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#endif
}
__device__ __forceinline__ void tmem_ld_wait() {
#if B200_TCGEN05
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#endif
}

// ---------------------------------------------------------------------------------------- TMA
// 2-D tiled load of the box at (c0 = innermost coordinate, c1) into shared memory, completing on
// `bar`.  c0 * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Bring `bytes` of global memory into L2 (no shared memory, no completion to wait for).  L2 is
// the device's point of coherence, so this is safe to issue before the kernel has waited for the
// previous one: a line that kernel writes later is updated in L2.
// `bytes` is a multiple of 16 and the address 16-byte aligned.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------------------- host: encoding
// cuTensorMapEncodeTiled fetched through the runtime (no -lcuda link needed).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D map over a row-major [rows, cols] matrix of `elem_bytes`-byte elements (row pitch
// cols*elem_bytes, a multiple of 16), box = [box_rows, 128 bytes of columns], 128-byte swizzle,
// zero fill outside the matrix.  Returns false when the encoding is refused.
inline bool make_map_sw128(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t elem_bytes,
                           uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const CUtensorMapDataType dt = elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {cols * elem_bytes};
  cuuint32_t box[2] = {128u / elem_bytes, box_rows};
  cuuint32_t estride[2] = {1, 1};
  return fn(map, dt, 2, const_cast<void*>(base), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc
}  // namespace b200
