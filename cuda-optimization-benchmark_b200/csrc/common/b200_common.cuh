// Common device and host helpers shared by every op of the B200 (sm_100a) kernel set.
//
// Everything here is header-only so that a single op can be amalgamated into one
// self-contained `solution.cu` translation unit, which is the build unit the
// reference grader compiles (graders/grade.py:92-113 copies only solution.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

namespace b200 {

// Status codes returned by every stream form of the C ABI (include/b200ops.h).
enum Status : int {
  kOk = 0,
  kInvalidArgument = 1,   // negative or overflowing size, null pointer with non-empty data
  kCudaError = 2,         // a CUDA runtime call or a launch failed
  kUnsupported = 3,       // shape or alignment outside what the entry point handles
  kWorkspaceTooSmall = 4, // caller-provided workspace is smaller than required
  kTimeout = 5,           // a bounded device-side wait gave up
};

inline const char* status_string(int s) {
  switch (s) {
    case kOk: return "ok";
    case kInvalidArgument: return "invalid argument";
    case kCudaError: return "CUDA error";
    case kUnsupported: return "unsupported shape or alignment";
    case kWorkspaceTooSmall: return "workspace too small";
    case kTimeout: return "device-side wait timed out";
    default: return "unknown status";
  }
}

// Launch check: returns kCudaError when the last launch failed to start.
inline int launch_status() {
  return cudaGetLastError() == cudaSuccess ? kOk : kCudaError;
}

// ---------------------------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched by launch_pdl may begin while the kernel
// before it on the stream is still running, as soon as every CTA of that kernel has called
// pdl_trigger() or exited.  Before its first global write (consecutive launches share output
// buffers, partial slots and counters) each writing thread calls pdl_wait(), which returns once
// the previous kernel has completed and its writes are visible.  Reads of inputs no kernel of the
// sequence writes can go ahead before it.  Both are no-ops in a kernel launched without PDL.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// First statement of a kernel that reads its inputs only after the previous kernel has completed:
// wait for it, then let the next launch queue up behind this one (its CTAs take SM slots as this
// kernel's free up and wait there), which hides the launch latency between back-to-back calls.
__device__ __forceinline__ void pdl_begin() {
  pdl_wait();
  pdl_trigger();
}

template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      const Args&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...) == cudaSuccess ? kOk : kCudaError;
}

// ---------------------------------------------------------------------------------------------
// Device properties, cached per device (the SM count sizes persistent grids).
// ---------------------------------------------------------------------------------------------
inline int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

// Resident CTAs per SM of one kernel instantiation at a given block size and dynamic shared
// memory (queried once per process and instantiation; used to size single-wave grids).
// Keyed by kernel address, block size and shared memory; a small fixed table suffices because
// the library has a few dozen kernel instantiations.
template <typename Kernel>
inline int resident_ctas_per_sm(Kernel kernel, int threads, size_t dyn_smem) {
  struct Entry {
    const void* fn;
    int threads;
    size_t smem;
    int ctas;
  };
  static Entry table[128];
  static int used = 0;
  static std::mutex mu;
  const void* key = reinterpret_cast<const void*>(kernel);
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (table[i].fn == key && table[i].threads == threads && table[i].smem == dyn_smem) return table[i].ctas;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, dyn_smem) != cudaSuccess || n <= 0) n = 1;
  if (used < 128) table[used++] = Entry{key, threads, dyn_smem, n};
  return n;
}

// Make sure a kernel may use `bytes` of dynamic shared memory on the current device: the limit
// recorded per (kernel, device) is raised whenever a launch needs more than any earlier one.
// Returns false when the runtime refuses.
template <typename Kernel>
inline bool ensure_dyn_smem(Kernel kernel, int bytes) {
  struct Entry {
    const void* fn;
    int dev;
    int bytes;
  };
  static Entry done[256];
  static int used = 0;
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const void* key = reinterpret_cast<const void*>(kernel);
  std::lock_guard<std::mutex> lock(mu);
  Entry* e = nullptr;
  for (int i = 0; i < used; ++i)
    if (done[i].fn == key && done[i].dev == dev) e = &done[i];
  if (e != nullptr && e->bytes >= bytes) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  if (e != nullptr) e->bytes = bytes;
  else if (used < 256) done[used++] = Entry{key, dev, bytes};
  return true;
}

// CTAs for a single-wave grid over `units` equal work units: at most the resident capacity, and
// sized so every CTA gets the same number of units (up to one).
inline int balanced_grid(int64_t units, int ctas_per_sm) {
  const int64_t cap = int64_t(sm_count()) * (ctas_per_sm > 0 ? ctas_per_sm : 1);
  if (units <= 0) return 1;
  const int64_t per = (units + cap - 1) / cap;
  return int((units + per - 1) / per);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------------------------
// Memory access wrappers.
// ---------------------------------------------------------------------------------------------
// 128-bit read-only streaming load: no L1 allocation (each byte is read once).
__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float ld_stream_f1(const float* p) {
  float v;
  asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 128-bit streaming store (evict-first in L2: the output is not re-read by this op).
__device__ __forceinline__ void st_stream_f4(float* p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ void st_stream_f1(float* p, float v) {
  asm volatile("st.global.cs.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// L2-coherent load (bypasses L1): used to read values written by other CTAs of the same grid.
__device__ __forceinline__ double ld_cg_f64(const double* p) {
  double v;
  asm volatile("ld.global.cg.f64 %0, [%1];" : "=d"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float ld_cg_f32(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ unsigned ld_cg_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// ---------------------------------------------------------------------------------------------
// Fixed-order warp / block reductions.  The butterfly order depends only on the lane index,
// so a given set of per-thread values always reduces to the same bits.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ unsigned warp_sum_u32(unsigned v) { return __reduce_add_sync(0xffffffffu, v); }

// Completion counting by amounts: a CTA that completed `add` of `total` work items (after writing
// their results) adds them to the counter once; returns true in the one CTA whose add reaches
// `total`, which then sees every other CTA's writes and resets the counter to zero.
__device__ __forceinline__ bool elect_last_add(unsigned* ticket, unsigned add, unsigned total) {
  __shared__ bool s_last_add;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(ticket, add);
    s_last_add = (prev + add == total);
    if (s_last_add) {
      __threadfence();
      *reinterpret_cast<volatile unsigned*>(ticket) = 0u;
    }
  }
  __syncthreads();
  return s_last_add;
}

// Last-CTA election for single-launch grid reductions.  Every CTA calls this once after
// writing its partial results; it returns true in exactly one CTA (the last to arrive), which
// then sees every other CTA's writes.  The winner resets the counter to zero, so the counter
// is ready for the next launch on the same stream.
__device__ __forceinline__ bool elect_last_cta(unsigned* ticket) {
  __shared__ bool s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(ticket, 1u);
    s_last = (prev == gridDim.x - 1);
    if (s_last) {
      __threadfence();
      *reinterpret_cast<volatile unsigned*>(ticket) = 0u;
    }
  }
  __syncthreads();
  return s_last;
}

}  // namespace b200
