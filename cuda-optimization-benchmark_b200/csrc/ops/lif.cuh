// Leaky integrate-and-fire layer: T sequential steps, B*H independent neurons.
//
// For each step t, in fp32 and in this order (tasks/leaky/reference.py:26-37, the oracle itself,
// and tasks/leaky/prompt.md "The operation"):
//   reset = mem >= th ? 1 : 0;  mem = beta*mem + x[t] - reset*th;  spikes[t] = mem >= th ? 1 : 0
// with beta clamped to [0, 1].  Every product and sum is rounded separately (no FMA contraction),
// so spikes and final_mem are bit-identical to the fp32 reference.  The drop-in boundary it
// replaces is `void reference(const float* input_current, const float* mem0, const float* beta,
// const float* threshold, int32_t T, int32_t B, int32_t H, float* spikes, float* final_mem)`
// (tasks/leaky/tests/task.json:3; expert launcher reference/leaky/solution.cu:106-138).
//
// B200 design: the membrane state lives in registers for the whole time loop.  Each CTA owns a
// contiguous slab of S neurons of the flattened (B*H) neuron axis (S ~ B*H / #SMs, one CTA per
// SM).  One producer thread keeps up to kMaxDepth future x[t] slab slices (S*4 contiguous bytes
// each) in flight into a shared-memory ring with cp.async.bulk, one "full" mbarrier per slot; the
// consumer warps (one thread per 4 neurons) wait on the slot, read their 4 inputs with one 128-bit
// shared load, store their 4 spikes straight to global memory with one 128-bit streaming store
// (each warp writes 512 contiguous bytes), and release the slot through its "empty" mbarrier, one
// arrive per warp.  No CTA-wide barrier is taken per step: warps drift apart by up to the ring
// depth, and the producer refills a slot as soon as every warp has read it.  8 bytes of HBM
// traffic per neuron-step (read x, write spike); 4 + 1/8 with bit-packed spikes (run_packed).  Shapes whose neuron count is not a multiple of
// 4, or unaligned pointers, take the one-neuron-per-thread form of the same loop.
//
// For training (lif_backward.cuh) the same loop also stores the membrane state every kSeg steps,
// checkpoint k being the state before step k * kSeg (checkpoint 0 = mem0): 1/4 byte per
// neuron-step, from which the backward recomputes each kSeg-step segment in registers.
#pragma once

#include "../common/b200_common.cuh"
#include "../common/bulk.cuh"

namespace b200 {
namespace lif {

constexpr int kThreads = 128;
constexpr int kDepth = 8;   // time steps of x in flight per thread (scalar form)

__device__ __forceinline__ float clamp01(float b) { return fminf(fmaxf(b, 0.0f), 1.0f); }

__device__ __forceinline__ bool step_bit(float& mem, float x, float beta, float th) {
  const float reset = mem >= th ? 1.0f : 0.0f;
  mem = __fsub_rn(__fadd_rn(__fmul_rn(beta, mem), x), __fmul_rn(reset, th));
  return mem >= th;
}
__device__ __forceinline__ float step(float& mem, float x, float beta, float th) {
  return step_bit(mem, x, beta, th) ? 1.0f : 0.0f;
}

constexpr int kSeg = 16;                    // time steps per membrane checkpoint
constexpr int kMaxDepth = 64;               // x slices in flight per CTA, at most
constexpr int kSmemBudget = 192 * 1024;      // bytes of the x ring
constexpr int kInFlight = 168 * 1024;        // bytes of x in flight per CTA the ring aims for
constexpr int kMaxSlab = (1024 - 32) * 4;    // neurons per CTA: consumer threads + one producer warp

// Spike outputs: fp32 [T, B*H] (the reference layout), bits (bit t % 32 of uint32 word
// [t / 32][neuron], written 32 steps at a time), or none (checkpoints only).
enum Out { kOutFloat = 0, kOutBits = 1, kOutNone = 2 };

// Slab form (NB % 4 == 0, 16-byte aligned pointers): CTA c owns neurons [c*S, c*S + cnt); warp 0
// produces, warps 1.. consume (thread 32 + i owns neurons 4i .. 4i + 3 of the slab).  kCkpt: store
// the checkpoints to ckpt [ceil(T / kSeg), B*H].
template <int kOut, bool kCkpt>
__global__ void __launch_bounds__(1024, 1) lif_slab_kernel(const float* __restrict__ x, const float* __restrict__ mem0,
                                                          const float* __restrict__ beta,
                                                          const float* __restrict__ th, int T, int64_t NB, int H,
                                                          int S, int depth, void* __restrict__ spikes,
                                                          float* __restrict__ final_mem, float* __restrict__ ckpt) {
  constexpr bool kPacked = kOut != kOutFloat;  // the lean loop (see the producer)
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  extern __shared__ __align__(128) float xr[];  // depth slices of S floats
  __shared__ uint64_t full[kMaxDepth], empty[kMaxDepth];
  const int64_t n0 = int64_t(blockIdx.x) * S;
  const int cnt = int(NB - n0 < S ? NB - n0 : S);
  const uint32_t bytes = uint32_t(cnt) * 4u;
  const int consumer_warps = int(blockDim.x / 32) - 1;
  if (threadIdx.x == 0) {
    for (int d = 0; d < depth; ++d) {
      mbar_init(&full[d], 1);
      mbar_init(&empty[d], uint32_t(consumer_warps));
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // Producer: slot d holds x[t] for t = d, d + depth, ...; it is refilled once every consumer
    // warp has released the previous use.
    if (threadIdx.x == 0) {
      int issued = 0;
      // Slot and use count from t each step for the fp32 layout, running counters for the packed
      // one: the paced producer measured 11% faster for fp32 (83 against 94 us; refills issued a
      // little sooner slow its read/write mix), the lean one 13% faster for packed (68 against
      // 78 us), at the BASELINE size in one process.
      int d = 0, k = 0;
      const float* src = x + n0;
      for (int t = 0; t < T; ++t) {
        if (!kPacked) {
          d = t % depth;
          k = t / depth;
          src = x + int64_t(t) * NB + n0;
        }
        if (k > 0 && !mbar_wait_sleep(&empty[d], uint32_t(k - 1) & 1u)) break;
        mbar_arrive_expect_tx(&full[d], bytes);
        bulk_g2s(xr + d * S, src, bytes, &full[d]);
        issued = t + 1;
        if (kPacked) {
          src += NB;
          if (++d == depth) {
            d = 0;
            ++k;
          }
        }
      }
      // No copy may still be writing this CTA's shared memory when it exits (the consumers wait
      // for every copy on the normal path; this covers a wait that gave up): the last use of each
      // slot has completed once its phase has.
      for (int t = issued > depth ? issued - depth : 0; t < issued; ++t)
        if (!mbar_wait_sleep(&full[t % depth], uint32_t(t / depth) & 1u)) break;
    }
    return;
  }
  const int i = threadIdx.x - 32, lane = threadIdx.x & 31;
  const bool mine = 4 * i < cnt;
  float4 m = make_float4(0.f, 0.f, 0.f, 0.f);
  float bq[4] = {0.f, 0.f, 0.f, 0.f}, tq[4] = {0.f, 0.f, 0.f, 0.f};
  if (mine) {
    m = *reinterpret_cast<const float4*>(mem0 + n0 + 4 * i);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int h = int((n0 + 4 * i + j) % H);
      bq[j] = clamp01(beta[h]);
      tq[j] = th[h];
    }
  }
  // The packed layout's loop is issue-bound: running slot, phase and pointers, no division or
  // 64-bit multiply per step, and waiting warps sleep.  The fp32 layout, bound by its read/write
  // mix, derives slot and phase from t each step and polls (see the producer).
  float* out = static_cast<float*>(spikes) + n0 + 4 * i;
  uint32_t* bits = static_cast<uint32_t*>(spikes) + n0 + 4 * i;
  const float* xs = xr + 4 * i;
  uint4 pk = make_uint4(0u, 0u, 0u, 0u);
  int d = 0;
  uint32_t ph = 0;
  for (int t = 0; t < T; ++t) {
    if (!kPacked) {
      d = t % depth;
      ph = uint32_t(t / depth) & 1u;
    }
    if (!(kPacked ? mbar_wait_sleep(&full[d], ph) : mbar_wait(&full[d], ph))) break;
    if (mine) {
      if (kCkpt && (t % kSeg) == 0) *reinterpret_cast<float4*>(ckpt + int64_t(t / kSeg) * NB + n0 + 4 * i) = m;
      const float4 xv = *reinterpret_cast<const float4*>(xs + d * S);
      if (kOut == kOutNone) {
        step_bit(m.x, xv.x, bq[0], tq[0]);
        step_bit(m.y, xv.y, bq[1], tq[1]);
        step_bit(m.z, xv.z, bq[2], tq[2]);
        step_bit(m.w, xv.w, bq[3], tq[3]);
      } else if (kPacked) {
        const uint32_t bit = 1u << (t & 31);
        pk.x |= step_bit(m.x, xv.x, bq[0], tq[0]) ? bit : 0u;
        pk.y |= step_bit(m.y, xv.y, bq[1], tq[1]) ? bit : 0u;
        pk.z |= step_bit(m.z, xv.z, bq[2], tq[2]) ? bit : 0u;
        pk.w |= step_bit(m.w, xv.w, bq[3], tq[3]) ? bit : 0u;
        if ((t & 31) == 31 || t == T - 1) {
          *reinterpret_cast<uint4*>(bits) = pk;
          bits += NB;
          pk = make_uint4(0u, 0u, 0u, 0u);
        }
      } else {
        float4 sp;
        sp.x = step(m.x, xv.x, bq[0], tq[0]);
        sp.y = step(m.y, xv.y, bq[1], tq[1]);
        sp.z = step(m.z, xv.z, bq[2], tq[2]);
        sp.w = step(m.w, xv.w, bq[3], tq[3]);
        st_stream_f4(out + int64_t(t) * NB, sp);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[d]);
    if (kPacked && ++d == depth) {
      d = 0;
      ph ^= 1u;
    }
  }
  if (mine && final_mem != nullptr) *reinterpret_cast<float4*>(final_mem + n0 + 4 * i) = m;
}

// Scalar form: one neuron per thread, same per-neuron arithmetic (kOut, kCkpt as the slab form).
template <int kOut, bool kCkpt>
__global__ void __launch_bounds__(kThreads) lif_scalar_kernel(const float* __restrict__ x,
                                                              const float* __restrict__ mem0,
                                                              const float* __restrict__ beta,
                                                              const float* __restrict__ th, int T, int64_t NB, int H,
                                                              void* __restrict__ spikes,
                                                              float* __restrict__ final_mem, float* __restrict__ ckpt) {
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  const int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x;
  if (i >= NB) return;
  float m = mem0[i];
  const int h = int(i % H);
  const float b = clamp01(beta[h]);
  const float tt = th[h];
  float ring[kDepth];
#pragma unroll
  for (int d = 0; d < kDepth; ++d)
    if (d < T) ring[d] = ld_stream_f1(x + i + int64_t(d) * NB);
  uint32_t pk = 0;
  for (int t0 = 0; t0 < T; t0 += kDepth) {
#pragma unroll
    for (int d = 0; d < kDepth; ++d) {
      const int t = t0 + d;
      if (t < T) {
        const float xv = ring[d];
        if (t + kDepth < T) ring[d] = ld_stream_f1(x + i + int64_t(t + kDepth) * NB);
        if (kCkpt && (t % kSeg) == 0) ckpt[int64_t(t / kSeg) * NB + i] = m;
        if (kOut == kOutNone) {
          step_bit(m, xv, b, tt);
        } else if (kOut == kOutBits) {
          pk |= step_bit(m, xv, b, tt) ? (1u << (t & 31)) : 0u;
          if ((t & 31) == 31 || t == T - 1) {
            static_cast<uint32_t*>(spikes)[int64_t(t >> 5) * NB + i] = pk;
            pk = 0;
          }
        } else {
          st_stream_f1(static_cast<float*>(spikes) + i + int64_t(t) * NB, step(m, xv, b, tt));
        }
      }
    }
  }
  if (final_mem != nullptr) final_mem[i] = m;
}

template <int kOut, bool kCkpt>
inline int run_impl(const float* x, const float* mem0, const float* beta, const float* th, int32_t T, int32_t B,
                    int32_t H, void* spikes, float* final_mem, float* ckpt, cudaStream_t stream) {
  if (T < 0 || B < 0 || H < 0) return kInvalidArgument;
  const int64_t NB = int64_t(B) * int64_t(H);
  if (NB == 0) return kOk;
  if (mem0 == nullptr || beta == nullptr || th == nullptr) return kInvalidArgument;
  if (kOut != kOutNone && final_mem == nullptr) return kInvalidArgument;
  if (T > 0 && (x == nullptr || (kOut != kOutNone && spikes == nullptr) || (kCkpt && ckpt == nullptr)))
    return kInvalidArgument;
  if (T == 0 && kOut == kOutNone) return kOk;
  const bool slab = T > 0 && (NB % 4 == 0) && aligned16(mem0) && aligned16(final_mem) && aligned16(x) &&
                    aligned16(spikes) && aligned16(ckpt);
  if (slab) {
    // Slab of S neurons per CTA: about one CTA per SM, S a multiple of 128 (whole consumer warps).
    const int sms = sm_count();
    int64_t S = (NB + sms - 1) / sms;
    S = (S + 127) / 128 * 128;
    if (S > kMaxSlab) S = kMaxSlab;
    const int64_t grid = (NB + S - 1) / S;
    // Ring depth: enough slices for about kInFlight bytes in flight (at least 24, the depth
    // measured best at the BASELINE size), within the shared-memory budget.  Narrow slabs (few
    // neurons per SM, e.g. one rank's share of a batch split over GPUs) get deeper rings, so the
    // bytes in flight per SM, and with them the HBM rate, do not shrink with the slab.
    const int64_t slice = S * 4;
    int depth = int(kSmemBudget / slice);
    const int64_t want = (kInFlight + slice - 1) / slice;
    const int cap = want > 24 ? int(want < kMaxDepth ? want : kMaxDepth) : 24;
    if (depth > cap) depth = cap;
    if (depth < 2) depth = 2;
    const size_t smem = size_t(depth) * size_t(S) * 4;
    auto kern = lif_slab_kernel<kOut, kCkpt>;
    if (!ensure_dyn_smem(kern, int(smem))) return kCudaError;
    return launch_pdl(kern, unsigned(grid), unsigned(S / 4 + 32), smem, stream, x, mem0, beta, th, T, NB, H, int(S),
                      depth, spikes, final_mem, ckpt);
  }
  const int64_t grid = (NB + kThreads - 1) / kThreads;
  return launch_pdl(lif_scalar_kernel<kOut, kCkpt>, unsigned(grid), kThreads, 0, stream, x, mem0, beta, th, T, NB,
                    H, spikes, final_mem, ckpt);
}

// spikes: fp32 [T, B*H], 0 or 1 (the reference layout).
inline int run(const float* x, const float* mem0, const float* beta, const float* th, int32_t T, int32_t B, int32_t H,
               float* spikes, float* final_mem, cudaStream_t stream) {
  return run_impl<kOutFloat, false>(x, mem0, beta, th, T, B, H, spikes, final_mem, nullptr, stream);
}

// spike_bits: uint32 [ceil(T / 32), B*H]; bit t % 32 of word [t / 32][n] is the spike of neuron n
// at step t (bits past T are zero).  1/32 of the fp32 layout's spike bytes.
inline int run_packed(const float* x, const float* mem0, const float* beta, const float* th, int32_t T, int32_t B,
                      int32_t H, uint32_t* spike_bits, float* final_mem, cudaStream_t stream) {
  return run_impl<kOutBits, false>(x, mem0, beta, th, T, B, H, spike_bits, final_mem, nullptr, stream);
}

inline int64_t checkpoint_count(int32_t T) { return T <= 0 ? 0 : (int64_t(T) + kSeg - 1) / kSeg; }

// The forward for training: run() plus the membrane checkpoints ckpt [ceil(T / kSeg), B*H].
inline int run_train(const float* x, const float* mem0, const float* beta, const float* th, int32_t T, int32_t B,
                     int32_t H, float* spikes, float* final_mem, float* ckpt, cudaStream_t stream) {
  return run_impl<kOutFloat, true>(x, mem0, beta, th, T, B, H, spikes, final_mem, ckpt, stream);
}

// The checkpoints alone (after a forward that did not store them): reads x, writes ckpt.
inline int run_checkpoints(const float* x, const float* mem0, const float* beta, const float* th, int32_t T,
                           int32_t B, int32_t H, float* ckpt, cudaStream_t stream) {
  return run_impl<kOutNone, true>(x, mem0, beta, th, T, B, H, nullptr, nullptr, ckpt, stream);
}

}  // namespace lif
}  // namespace b200
