// Fused RL loss step: discounted reward-to-go over a [B, T] batch and the PPO clipped loss with
// its diagnostics (optionally the mean entropy) over N samples, in one kernel launch.
//
// The two ops are independent (BASELINE.json configs[1] draws the PPO advantages independently of
// the returns), and each alone is too small to hide a kernel's ramp-up and drain.  One launch runs
// both: CTA b is a reward-to-go CTA or a PPO CTA, the two kinds interleaved evenly over the grid
// (Bresenham on the block index) so that every SM holds both at once and the latency-bound row
// scans overlap the PPO streams.
//   - reward-to-go CTAs: 8 warps, one row per warp at a time, exactly rtg::warp_rows (the same
//     passes and the same bits as the reward_to_go entry points);
//   - PPO CTAs: chunks of 4096 samples through ppo::chunk_partials (the same partials, hence the
//     same bits, as the ppo_clip entry points); the PPO CTA that finishes last combines the
//     partials, or, in the shard form, the partials are left for a cross-GPU gather and ppo finish.
// One resident wave of B200_RL_MIN_CTAS CTAs per SM is split between the roles so that the
// slowest CTA of either kind has the least work (see split_roles).
#pragma once

#include "../common/b200_common.cuh"
#include "ppo_clip.cuh"
#include "reward_to_go.cuh"

namespace b200 {
namespace rl {

#ifndef B200_RL_MIN_CTAS
#define B200_RL_MIN_CTAS 3  // resident CTAs per SM the register budget is sized for
#endif

constexpr int kThreads = ppo::kThreads;        // 256: the PPO chunk mapping
constexpr int kRows = kThreads / 32;           // reward-to-go rows in flight per CTA
constexpr int kSmem = kRows * rtg::kWarpSmem;  // one staging buffer per warp
static_assert(ppo::kThreads == 256, "the reward-to-go role uses the CTA's 8 warps");

struct Args {
  const float* reward;
  const unsigned char* done;
  float gamma;
  int64_t B;
  int T;
  float* rtg_out;
  const float* cur;
  const float* old;
  const float* adv;
  const float* ent;
  int64_t n;
  ppo::Clip clip;
  ppo::Partial* partials;
  unsigned* ticket;
  float* ppo_out;
  double inv_n;      // 1 / n for the PPO finish
  int64_t rtg_ctas;  // CTAs with the reward-to-go role (kRows rows each per round)
  int64_t ppo_ctas;  // CTAs with the PPO role
};

template <bool kVec, bool kEnt, bool kFinish>
__global__ void __launch_bounds__(kThreads, B200_RL_MIN_CTAS) step_kernel(const Args a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint64_t bars[kRows][2];
  const int64_t b = blockIdx.x, G = gridDim.x;
  const int64_t rtg_before = (b * a.rtg_ctas) / G;  // reward-to-go CTAs with a smaller index
  const bool is_rtg = ((b + 1) * a.rtg_ctas) / G > rtg_before;
  if (is_rtg) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    rtg::warp_rows(a.reward, a.done, a.gamma, a.B, a.T, a.rtg_out, rtg_before * kRows + warp, a.rtg_ctas * kRows,
                   smem + warp * rtg::kWarpSmem, bars[warp], 1, lane);
    return;
  }
  const int64_t pidx = b - rtg_before;  // index among the PPO CTAs
  ppo::chunk_partials<kVec, kEnt>(a.cur, a.old, a.adv, a.ent, a.n, a.clip, a.partials, pidx, a.ppo_ctas);
  if (kFinish) {
    if (elect_last_add(a.ticket, 1u, unsigned(a.ppo_ctas)))
      ppo::finish(a.partials, ppo::num_chunks(a.n), a.n, a.inv_n, kEnt, a.ppo_out);
  }
}

template <bool kVec, bool kEnt, bool kFinish>
inline int launch(const Args& a, cudaStream_t stream) {
  auto kern = step_kernel<kVec, kEnt, kFinish>;
  if (!ensure_dyn_smem(kern, kSmem)) return kCudaError;
  kern<<<unsigned(a.rtg_ctas + a.ppo_ctas), kThreads, kSmem, stream>>>(a);
  return launch_status();
}

// Split of `slots` CTAs into reward-to-go CTAs and PPO CTAs: the count r of reward-to-go CTAs
// minimising the larger per-CTA load, ceil(rows / (r*kRows)) rounds of kRows rows against
// ceil(chunks / (slots - r)) chunks, in bytes; each role keeps at least one CTA while it has work
// (and the finish form always one PPO CTA, which writes the outputs even for an empty batch).
// B200_RL_ROW_CTAS, when defined, fixes r (for tuning runs).
inline void split_roles(int64_t rows, int64_t row_bytes, int64_t chunks, int64_t chunk_bytes, int64_t slots,
                        bool finish, int64_t* r_out, int64_t* p_out) {
  const int64_t row_ctas = (rows + kRows - 1) / kRows;  // CTAs that have a row in the first round
  if (rows == 0 || chunks == 0) {
    *r_out = row_ctas < slots ? row_ctas : slots;
    *p_out = chunks > 0 ? (chunks < slots ? chunks : slots) : (finish ? 1 : 0);
    return;
  }
  int64_t best_r = 1;
  double best = -1.0;
  for (int64_t r = 1; r < slots; ++r) {
    const int64_t p = slots - r;
    const double t_rows = double((rows + r * kRows - 1) / (r * kRows)) * double(kRows * row_bytes);
    const double t_chunks = double((chunks + p - 1) / p) * double(chunk_bytes);
    const double t = t_rows > t_chunks ? t_rows : t_chunks;
    if (best < 0.0 || t < best) {
      best = t;
      best_r = r;
    }
  }
#ifdef B200_RL_ROW_CTAS
  best_r = B200_RL_ROW_CTAS;
#endif
  *r_out = best_r < row_ctas ? best_r : row_ctas;
  *p_out = slots - best_r < chunks ? slots - best_r : chunks;
}

// Both ops in one launch.  PPO workspace: ppo::workspace_bytes(n) (first 4 bytes zero before the
// first call; left zero).  With finish == false the PPO chunk partials are written to
// `partials_out` (one ppo::Partial per chunk) and ppo_out is untouched (the multi-GPU shard form).
inline int run(const float* reward, const unsigned char* done, float gamma, int32_t B, int32_t T, float* rtg_out,
               const float* cur, const float* old, const float* adv, const float* ent, int64_t n, float eps,
               float* ppo_out, void* workspace, size_t ws_bytes, bool finish, void* partials_out,
               cudaStream_t stream) {
  if (B < 0 || T < 0 || n < 0) return kInvalidArgument;
  if (int64_t(B) * T > 0 && (reward == nullptr || done == nullptr || rtg_out == nullptr)) return kInvalidArgument;
  if (n > 0 && (cur == nullptr || old == nullptr || adv == nullptr)) return kInvalidArgument;
  Args a;
  a.reward = reward;
  a.done = done;
  a.gamma = gamma;
  a.B = T > 0 ? int64_t(B) : 0;
  a.T = T;
  a.rtg_out = rtg_out;
  a.cur = cur;
  a.old = old;
  a.adv = adv;
  a.ent = ent;
  a.n = n;
  a.clip = ppo::make_clip(eps);
  if (finish) {
    if (ppo_out == nullptr) return kInvalidArgument;
    if (workspace == nullptr || ws_bytes < ppo::workspace_bytes(n)) return kWorkspaceTooSmall;
    a.ticket = static_cast<unsigned*>(workspace);
    a.partials = reinterpret_cast<ppo::Partial*>(static_cast<char*>(workspace) + 256);
  } else {
    if (n > 0 && partials_out == nullptr) return kInvalidArgument;
    a.ticket = nullptr;
    a.partials = static_cast<ppo::Partial*>(partials_out);
  }
  a.ppo_out = ppo_out;
  a.inv_n = ppo::inv_count(n);
  const int64_t slots = int64_t(sm_count()) * B200_RL_MIN_CTAS;
  split_roles(a.B, 9 * int64_t(T), ppo::num_chunks(n), (ent != nullptr ? 16 : 12) * ppo::kChunk, slots, finish,
              &a.rtg_ctas, &a.ppo_ctas);
  if (a.rtg_ctas + a.ppo_ctas == 0) return kOk;
  const bool vec = aligned16(cur) && aligned16(old) && aligned16(adv) && (ent == nullptr || aligned16(ent));
  if (finish) {
    if (ent != nullptr) return vec ? launch<true, true, true>(a, stream) : launch<false, true, true>(a, stream);
    return vec ? launch<true, false, true>(a, stream) : launch<false, false, true>(a, stream);
  }
  if (ent != nullptr) return vec ? launch<true, true, false>(a, stream) : launch<false, true, false>(a, stream);
  return vec ? launch<true, false, false>(a, stream) : launch<false, false, false>(a, stream);
}

}  // namespace rl
}  // namespace b200
