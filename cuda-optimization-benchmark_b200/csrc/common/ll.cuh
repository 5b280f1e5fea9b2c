// "LL" records: payloads whose every 4-byte word travels with a 32-bit epoch in one 8-byte value.
//
// A reader that sees a word whose epoch field equals the epoch it expects knows the word belongs
// to that epoch: the 8-byte value is written and read as one single-copy-atomic access (each
// 64-bit element of a vector access is one), so no fence and no separate ready flag are needed
// between writer and reader.  Two words move per 16-byte access.  The accesses are relaxed (never
// kept in L1) at the scope that holds both sides: GPU scope between CTAs of one GPU, system scope
// for records that peers write over NVLink (system-scope accesses cost several microseconds more
// on B200, so they are kept to the cross-GPU records).
#pragma once

#include <stdint.h>

#include "bulk.cuh"

namespace b200 {

__device__ __forceinline__ unsigned long long ll_word(uint32_t word, uint32_t epoch) {
  return (static_cast<unsigned long long>(epoch) << 32) | word;
}

enum class LLScope { kGpu, kSys };

template <LLScope S>
__device__ __forceinline__ void ll_store2(ulonglong2* p, unsigned long long a, unsigned long long b) {
  if (S == LLScope::kGpu)
    asm volatile("st.relaxed.gpu.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
  else
    asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
template <LLScope S>
__device__ __forceinline__ ulonglong2 ll_load2(const ulonglong2* p) {
  ulonglong2 v;
  if (S == LLScope::kGpu)
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  else
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool ll_fresh(unsigned long long v, uint32_t epoch) { return uint32_t(v >> 32) == epoch; }
__device__ __forceinline__ bool ll_fresh2(const ulonglong2& v, uint32_t epoch) {
  return ll_fresh(v.x, epoch) & ll_fresh(v.y, epoch);
}

// Store kWords payload words as kWords / 2 16-byte LL pairs.
template <int kWords, LLScope S>
__device__ __forceinline__ void ll_store_record(ulonglong2* rec, const uint32_t (&w)[kWords], uint32_t epoch) {
  static_assert(kWords % 2 == 0, "records are whole 16-byte pairs of LL words");
#pragma unroll
  for (int q = 0; q < kWords / 2; ++q)
    ll_store2<S>(rec + q, ll_word(w[2 * q], epoch), ll_word(w[2 * q + 1], epoch));
}

// Waiting reader of LL records of kWords payload words (kWords even, records 16-byte aligned and
// kWords * 8 bytes apart).  One per thread: the thread waits at most kWaitLimitNs in all, from its
// first wait; past that it records kFaultWaitTimeout and takes whatever the words hold, so the
// kernel always ends and the host sees the fault.
template <int kWords, LLScope S>
struct LLReader {
  static_assert(kWords % 2 == 0, "records are whole 16-byte pairs of LL words");
  static constexpr int kPairs = kWords / 2;
  const ulonglong2* recs;  // record 0
  unsigned epoch;
  unsigned long long t0 = 0;
  bool dead = false;

  // Records idx[u] for the kU records with use[u]: all loads issued together, then the stale pairs
  // re-read until fresh (static indices, so everything stays in registers).
  template <int kU>
  __device__ __forceinline__ void read(const int64_t (&idx)[kU], const bool (&use)[kU], uint32_t (&w)[kU][kWords]) {
    ulonglong2 v[kU][kPairs];
    bool ok = true;
#pragma unroll
    for (int u = 0; u < kU; ++u) {
#pragma unroll
      for (int q = 0; q < kPairs; ++q) {
        v[u][q] = use[u] ? ll_load2<S>(recs + idx[u] * kPairs + q) : make_ulonglong2(0ull, 0ull);
        ok &= !use[u] || ll_fresh2(v[u][q], epoch);
      }
    }
    if (!ok && !dead) {
      if (t0 == 0) t0 = global_ns();
      do {
        if (global_ns() - t0 > kWaitLimitNs) {
          atomicOr(&g_b200_fault, kFaultWaitTimeout);
          dead = true;
          break;
        }
        ok = true;
#pragma unroll
        for (int u = 0; u < kU; ++u) {
#pragma unroll
          for (int q = 0; q < kPairs; ++q) {
            if (use[u] && !ll_fresh2(v[u][q], epoch)) v[u][q] = ll_load2<S>(recs + idx[u] * kPairs + q);
            ok &= !use[u] || ll_fresh2(v[u][q], epoch);
          }
        }
      } while (!ok);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
#pragma unroll
      for (int q = 0; q < kPairs; ++q) {
        w[u][2 * q] = uint32_t(v[u][q].x);
        w[u][2 * q + 1] = uint32_t(v[u][q].y);
      }
    }
  }

  __device__ __forceinline__ void read(int64_t i, uint32_t (&w)[kWords]) {
    const int64_t idx[1] = {i};
    const bool use[1] = {true};
    uint32_t ww[1][kWords];
    read<1>(idx, use, ww);
#pragma unroll
    for (int q = 0; q < kWords; ++q) w[q] = ww[0][q];
  }
};

}  // namespace b200
