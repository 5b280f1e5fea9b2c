// Surrogate-gradient backward of the leaky integrate-and-fire layer (lif.cuh), the step after it
// when the layer is trained (snnTorch's Leaky, which tasks/leaky restates, trained through its
// default arctangent surrogate with the reset detached; the surrogate is that of Fang et al.,
// "Incorporating Learnable Membrane Time Constant to Enhance Learning of Spiking Neural
// Networks", 2021).  With mem[t] the forward's fp32 state after step t (mem[-1] = mem0),
// u[t] = mem[t] - th and r[t] = (mem[t-1] >= th), per neuron, backwards in time:
//
//   s'[t]     = (alpha / 2) / (1 + (pi / 2 * alpha * u[t])^2)
//   g[t]      = grad_spikes[t] * s'[t] + beta * g[t+1]          (beta * g[T] := grad_final_mem)
//   grad_x[t] = g[t],  grad_mem0 = beta * g[0]
//   grad_beta[h]      = [0 <= beta_raw[h] <= 1] * sum over b, t of g[t] * mem[t-1]
//   grad_threshold[h] = -sum over b, t of (grad_spikes[t] * s'[t] + r[t] * g[t])
//
// B200 design.  The backward needs mem[t] for every step in reverse order; storing it would cost
// the forward 4 more bytes per neuron-step and the backward 4 more to read it back.  Instead the
// forward stores one checkpoint per kSeg steps (lif::run_train, 1/4 byte per neuron-step) and the
// backward recomputes each kSeg-step segment from its checkpoint in registers, with the forward's
// exact arithmetic (so every reset and spike decision is the forward's), then runs it backwards.
// 12 bytes of HBM traffic per neuron-step (x, grad_spikes, grad_x), the minimum for a backward
// that does not read a stored trajectory.  One neuron per thread: per segment a thread issues all
// kSeg loads of x and of grad_spikes at once (a warp's loads and stores are 128 contiguous bytes
// per step), runs the segment forwards with the states in registers, then backwards, streaming
// grad_x out.  kSeg = 16 keeps the kernel at 72 registers (28 warps per SM); with 32-step segments
// it needed 128 (16 warps) and reached 0.68 of the HBM roofline instead of 0.82.  Staging [kSeg x
// 128-neuron] tiles through shared memory (2-D TMA loads and stores, double-buffered) was slower
// still: 96 KB per 128 neurons leaves 8 warps per SM, too few for the serial recurrences.
//
// grad_beta and grad_threshold sum over the batch: each thread writes its neuron's two fp32 sums
// (over its T steps) to the workspace and reduce_kernel adds them over b in a fixed order in fp64,
// so the result does not depend on the launch shape.
#pragma once

#include "../common/b200_common.cuh"
#include "lif.cuh"

namespace b200 {
namespace lif {

constexpr int kBwdThreads = 128;
constexpr int kReduceThreads = 256;

// (alpha / 2) / (1 + (k u)^2) with k = pi / 2 * alpha: one multiply, one fma and the fast
// division (a hardware reciprocal and a multiply, within 2 ulp; the denominator is >= 1).  The
// IEEE division's extra checking instructions made the special-function pipe the kernel's limit.
__device__ __forceinline__ float atan_grad(float u, float half_alpha, float k) {
  const float z = k * u;
  return __fdividef(half_alpha, fmaf(z, z, 1.0f));
}

// One neuron per thread.  ckpt [ceil(T / kSeg), NB]; partials [2, NB] (beta, threshold) or null.
__global__ void __launch_bounds__(kBwdThreads) lif_backward_kernel(
    const float* __restrict__ x, const float* __restrict__ ckpt, const float* __restrict__ beta,
    const float* __restrict__ th, const float* __restrict__ gspk, const float* __restrict__ gfinal, float half_alpha,
    float k, int T, int64_t NB, int H, float* __restrict__ gx, float* __restrict__ gmem0,
    float* __restrict__ partials) {
  pdl_begin();  // launched with PDL: wait for the previous kernel, let the next one queue
  const int64_t n = int64_t(blockIdx.x) * kBwdThreads + threadIdx.x;
  if (n >= NB) return;
  const int h = int(n % H);
  const float b = clamp01(beta[h]);
  const float tt = th[h];
  float c = gfinal != nullptr ? gfinal[n] : 0.0f;  // beta * g[t+1], the gradient carried back
  float acc_b = 0.0f, acc_t = 0.0f;
  const int nseg = int((int64_t(T) + kSeg - 1) / kSeg);
  for (int s = nseg - 1; s >= 0; --s) {
    const int t0 = s * kSeg;
    const int len = T - t0 < kSeg ? T - t0 : kSeg;
    const float m0 = ckpt[int64_t(s) * NB + n];
    float mem[kSeg], gs[kSeg];
    {
      const float* xp = x + int64_t(t0) * NB + n;
      const float* gp = gspk + int64_t(t0) * NB + n;
#pragma unroll
      for (int j = 0; j < kSeg; ++j) {
        if (j < len) {
          mem[j] = ld_stream_f1(xp);
          gs[j] = ld_stream_f1(gp);
        }
        xp += NB;
        gp += NB;
      }
    }
    // Forward over the segment: mem[j] becomes the state after step t0 + j; bit j of rb is the
    // reset that step applied.
    uint32_t rb = 0;
    float p = m0;
#pragma unroll
    for (int j = 0; j < kSeg; ++j) {
      if (j < len) {
        rb |= (p >= tt ? 1u : 0u) << j;
        step_bit(p, mem[j], b, tt);
        mem[j] = p;
      }
    }
    // Backward over the segment.
    float* op = gx + int64_t(t0 + len - 1) * NB + n;
#pragma unroll
    for (int j = kSeg - 1; j >= 0; --j) {
      if (j < len) {
        const float gsp = gs[j] * atan_grad(mem[j] - tt, half_alpha, k);
        const float g = gsp + c;
        st_stream_f1(op, g);
        op -= NB;
        acc_b = fmaf(g, j > 0 ? mem[j - 1] : m0, acc_b);
        acc_t -= ((rb >> j) & 1u) ? gsp + g : gsp;
        c = b * g;
      }
    }
  }
  if (gmem0 != nullptr) gmem0[n] = c;
  if (partials != nullptr) {
    partials[n] = acc_b;
    partials[NB + n] = acc_t;
  }
}

// grad_beta[h] and grad_threshold[h]: the B per-neuron sums of column h added in order b = 0..B-1.
__global__ void __launch_bounds__(kReduceThreads) lif_reduce_kernel(const float* __restrict__ partials,
                                                                    const float* __restrict__ beta, int B, int H,
                                                                    float* __restrict__ gbeta,
                                                                    float* __restrict__ gth) {
  pdl_begin();
  const int h = blockIdx.x * kReduceThreads + threadIdx.x;
  if (h >= H) return;
  const int64_t NB = int64_t(B) * H;
  double sb = 0.0, st = 0.0;
  for (int b = 0; b < B; ++b) {
    sb += double(partials[int64_t(b) * H + h]);
    st += double(partials[NB + int64_t(b) * H + h]);
  }
  const float braw = beta[h];
  if (gbeta != nullptr) gbeta[h] = (braw >= 0.0f && braw <= 1.0f) ? float(sb) : 0.0f;
  if (gth != nullptr) gth[h] = float(st);
}

inline int64_t backward_workspace_bytes(int32_t B, int32_t H) {
  if (B <= 0 || H <= 0) return 0;
  return 2 * int64_t(B) * int64_t(H) * int64_t(sizeof(float));
}

// ckpt from run_train or run_checkpoints with the same x, mem0, beta, th.  grad_final_mem, grad_mem0,
// grad_beta and grad_threshold may be null (zero incoming gradient / not wanted); the workspace is
// needed only for grad_beta or grad_threshold.
inline int backward(const float* x, const float* ckpt, const float* beta, const float* th, int32_t T, int32_t B,
                    int32_t H, const float* grad_spikes, const float* grad_final_mem, float alpha, float* grad_x,
                    float* grad_mem0, float* grad_beta, float* grad_th, void* ws, int64_t ws_bytes,
                    cudaStream_t stream) {
  if (T < 0 || B < 0 || H < 0) return kInvalidArgument;
  const int64_t NB = int64_t(B) * int64_t(H);
  if (NB == 0) return kOk;
  if (beta == nullptr || th == nullptr) return kInvalidArgument;
  if (T > 0 && (x == nullptr || ckpt == nullptr || grad_spikes == nullptr || grad_x == nullptr))
    return kInvalidArgument;
  const bool sums = grad_beta != nullptr || grad_th != nullptr;
  if (sums && (ws == nullptr || ws_bytes < backward_workspace_bytes(B, H))) return kWorkspaceTooSmall;
  float* partials = sums ? static_cast<float*>(ws) : nullptr;
  const double pi = 3.14159265358979323846;
  const float half_alpha = float(0.5 * double(alpha));
  const float k = float(pi / 2.0 * double(alpha));
  const int64_t grid = (NB + kBwdThreads - 1) / kBwdThreads;
  const int st = launch_pdl(lif_backward_kernel, unsigned(grid), kBwdThreads, 0, stream, x, ckpt, beta, th,
                            grad_spikes, grad_final_mem, half_alpha, k, T, NB, H, grad_x, grad_mem0, partials);
  if (st != kOk || !sums) return st;
  return launch_pdl(lif_reduce_kernel, unsigned((H + kReduceThreads - 1) / kReduceThreads), kReduceThreads, 0, stream,
                    static_cast<const float*>(partials), beta, B, H, grad_beta, grad_th);
}

}  // namespace lif
}  // namespace b200
