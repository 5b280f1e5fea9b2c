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
//   - PPO CTAs: chunks of 4096 samples through ppo::chunk_partials (the same partials, combined in
//     the same order, hence the same bits, as the ppo_clip entry points); the PPO CTA that finishes
//     last combines the partials, or, in the shard form, the partials are left for a cross-GPU
//     gather and ppo finish.
// One resident wave of B200_RL_MIN_CTAS CTAs per SM is split between the roles so that the
// slowest CTA of either kind has the least work (see split_roles).  Steps are launched with
// programmatic dependent launch, so back-to-back steps overlap the tail of one with the start of
// the next (step_prologue).
#pragma once

#include <cstdlib>

#include "../common/b200_common.cuh"
#include "../common/peer.cuh"
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
  const void* done;  // bytes [B, T], or with kBits uint32 words [B, ceil(T / 32)] (rtg::pack_done)
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
  ppo::Partial* partials;  // chunk partials (workspace, or the caller's buffer in the shard form)
  unsigned* ticket;        // completion counter of the last-CTA election (workspace)
  float* ppo_out;
  double inv_n;      // 1 / n for the PPO finish
  int64_t rtg_ctas;  // CTAs with the reward-to-go role (kRows rows each per round)
  int64_t ppo_ctas;  // CTAs with the PPO role
  bool early_reads;  // read the inputs before the previous kernel on the stream completes
};

// Under PDL the launch may begin before the previous kernel on the stream has finished.  Unless
// the caller has declared that the kernel launched just before writes none of the inputs
// (early_reads), every thread first waits for it, so only the launch latency overlaps; otherwise
// the loads go ahead and each thread waits just before its first global write.  Either way the
// next launch is released at once: its CTAs take the SM slots this step's CTAs free as they finish
// (every CTA of this step is resident by then, so none of them can be starved of a slot).
__device__ __forceinline__ void step_prologue(const Args& a) {
  if (!a.early_reads) pdl_wait();
  pdl_trigger();
}

template <bool kVec, bool kEnt, bool kFinish, bool kBits>
__global__ void __launch_bounds__(kThreads, B200_RL_MIN_CTAS) step_kernel(const Args a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint64_t bars[kRows][2];
  step_prologue(a);
  const int64_t b = blockIdx.x, G = gridDim.x;
  const int64_t rtg_before = (b * a.rtg_ctas) / G;  // reward-to-go CTAs with a smaller index
  const bool is_rtg = ((b + 1) * a.rtg_ctas) / G > rtg_before;
  if (is_rtg) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    rtg::warp_rows<kBits>(a.reward, a.done, a.gamma, a.B, a.T, a.rtg_out, rtg_before * kRows + warp,
                          a.rtg_ctas * kRows, smem + warp * rtg::kWarpSmem, bars[warp], 1, lane);
    return;
  }
  const int64_t pidx = b - rtg_before;  // index among the PPO CTAs
  ppo::chunk_partials<kVec, kEnt>(a.cur, a.old, a.adv, a.ent, a.n, a.clip, a.partials, pidx, a.ppo_ctas);
  if (kFinish) {
    if (threadIdx.x == 0) pdl_wait();  // the ticket (also when this CTA had no chunk)
    if (elect_last_add(a.ticket, 1u, unsigned(a.ppo_ctas)))
      ppo::finish(a.partials, ppo::num_chunks(a.n), a.n, a.inv_n, kEnt, a.ppo_out);
  }
}

// The rank record of the multi-GPU step: this rank's PPO totals (ppo::Sums) as 14 words, each
// stored with the epoch (LL form, 112 bytes).
constexpr int kRankWords = 14;
constexpr size_t kExchangeRecordBytes = size_t(kRankWords) * 8;

__device__ __forceinline__ void pack_sums(const ppo::Sums& s, uint32_t (&w)[kRankWords]) {
#pragma unroll
  for (int q = 0; q < 5; ++q) {
    const unsigned long long b = __double_as_longlong(s.t[q]);
    w[2 * q] = uint32_t(b);
    w[2 * q + 1] = uint32_t(b >> 32);
  }
  w[10] = __float_as_uint(s.mx);
  w[11] = 0u;
  w[12] = uint32_t(s.c);
  w[13] = uint32_t(s.c >> 32);
}

__device__ __forceinline__ ppo::Sums unpack_sums(const uint32_t (&w)[kRankWords]) {
  ppo::Sums s;
#pragma unroll
  for (int q = 0; q < 5; ++q) s.t[q] = __hiloint2double(int(w[2 * q + 1]), int(w[2 * q]));
  s.mx = __uint_as_float(w[10]);
  s.c = (static_cast<unsigned long long>(w[13]) << 32) | w[12];
  return s;
}

// Multi-GPU step with the PPO exchange fused in (one launch per rank per step).  Each rank reduces
// its own chunk partials exactly as the one-GPU step does; the CTA that does so (the last PPO CTA
// to finish) stores the rank's totals, in LL form, into slot `rank` of every other rank's buffer
// (16-byte stores of two {word, epoch} pairs over NVLink; no fence, no flag), reads the other
// ranks' totals from its own buffer (one thread per rank, each waiting until its record's epoch
// has arrived) and adds all ranks' totals in rank order.  Every rank writes the same outputs; with
// one rank they are bit-identical to the one-GPU step.
template <bool kVec, bool kEnt, bool kBits>
__global__ void __launch_bounds__(kThreads, B200_RL_MIN_CTAS) step_exchange_kernel(const Args a, const PeerView pv) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint64_t bars[kRows][2];
  __shared__ ppo::Sums s_rank[kMaxPeers];
  step_prologue(a);
  const int64_t b = blockIdx.x, G = gridDim.x;
  const int64_t rtg_before = (b * a.rtg_ctas) / G;
  const bool is_rtg = ((b + 1) * a.rtg_ctas) / G > rtg_before;
  if (is_rtg) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    rtg::warp_rows<kBits>(a.reward, a.done, a.gamma, a.B, a.T, a.rtg_out, rtg_before * kRows + warp,
                          a.rtg_ctas * kRows, smem + warp * rtg::kWarpSmem, bars[warp], 1, lane);
    return;
  }
  const int64_t pidx = b - rtg_before;
  ppo::chunk_partials<kVec, kEnt>(a.cur, a.old, a.adv, a.ent, a.n, a.clip, a.partials, pidx, a.ppo_ctas);
  if (threadIdx.x == 0) pdl_wait();  // the ticket (also when this CTA had no chunk)
  if (!elect_last_add(a.ticket, 1u, unsigned(a.ppo_ctas))) return;
  const ppo::Sums mine = ppo::reduce_partials(a.partials, ppo::num_chunks(a.n));
  if (threadIdx.x == 0) {
    uint32_t w[kRankWords];
    pack_sums(mine, w);
    for (int r = 0; r < pv.world; ++r) {
      if (r == pv.rank) continue;
      ulonglong2* rec = peer_record(pv, r, pv.rank, 0);
#pragma unroll
      for (int q = 0; q < kRankWords / 2; ++q)
        ll_store2<LLScope::kSys>(rec + q, ll_word(w[2 * q], pv.epoch), ll_word(w[2 * q + 1], pv.epoch));
    }
  }
  if (threadIdx.x == 0) {
    s_rank[pv.rank] = mine;  // this rank's own totals need no round trip through memory
  } else if (threadIdx.x < pv.world) {
    const int r = threadIdx.x - 1 < pv.rank ? threadIdx.x - 1 : threadIdx.x;  // threads 1.. take the other ranks
    LLReader<kRankWords, LLScope::kSys> rd{peer_record(pv, pv.rank, 0, 0), pv.epoch};
    uint32_t w[kRankWords];
    rd.read(r, w);
    s_rank[r] = unpack_sums(w);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    ppo::Sums t = s_rank[0];
    for (int r = 1; r < pv.world; ++r) {
#pragma unroll
      for (int q = 0; q < 5; ++q) t.t[q] += s_rank[r].t[q];
      t.mx = fmaxf(t.mx, s_rank[r].mx);
      t.c += s_rank[r].c;
    }
    ppo::write_outputs(t, int64_t(pv.world) * a.n, a.inv_n, kEnt, a.ppo_out);
  }
}

template <bool kVec, bool kEnt, bool kFinish, bool kBits>
inline int launch(const Args& a, cudaStream_t stream) {
  auto kern = step_kernel<kVec, kEnt, kFinish, kBits>;
  if (!ensure_dyn_smem(kern, kSmem)) return kCudaError;
  return launch_pdl(kern, unsigned(a.rtg_ctas + a.ppo_ctas), kThreads, kSmem, stream, a);
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
// early_reads: the caller declares that the kernel launched just before on the stream writes none
// of the inputs, so they may be read before it completes.  done_bits: `done` holds the flags as
// bits (rtg::pack_done), 1/8 byte per step instead of 1.
inline int64_t row_bytes(int32_t T, bool done_bits) {
  return done_bits ? 8 * int64_t(T) + 4 * ((int64_t(T) + 31) / 32) : 9 * int64_t(T);
}

inline int run(const float* reward, const void* done, float gamma, int32_t B, int32_t T, float* rtg_out,
               const float* cur, const float* old, const float* adv, const float* ent, int64_t n, float eps,
               float* ppo_out, void* workspace, size_t ws_bytes, bool finish, void* partials_out,
               bool early_reads, bool done_bits, cudaStream_t stream) {
  if (B < 0 || T < 0 || n < 0) return kInvalidArgument;
  if (int64_t(B) * T > 0 && (reward == nullptr || done == nullptr || rtg_out == nullptr)) return kInvalidArgument;
  if (n > 0 && (cur == nullptr || old == nullptr || adv == nullptr)) return kInvalidArgument;
  Args a;
  a.early_reads = early_reads;
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
    a.ticket = &static_cast<ppo::Control*>(workspace)->ticket;
    a.partials = ppo::ws_partials(workspace);
  } else {
    if (n > 0 && partials_out == nullptr) return kInvalidArgument;
    a.ticket = nullptr;
    a.partials = static_cast<ppo::Partial*>(partials_out);
  }
  a.ppo_out = ppo_out;
  a.inv_n = ppo::inv_count(n);
  const int64_t slots = int64_t(sm_count()) * B200_RL_MIN_CTAS;
  split_roles(a.B, row_bytes(T, done_bits), ppo::num_chunks(n), (ent != nullptr ? 16 : 12) * ppo::kChunk, slots,
              finish, &a.rtg_ctas, &a.ppo_ctas);
  if (a.rtg_ctas + a.ppo_ctas == 0) return kOk;
  const bool vec = aligned16(cur) && aligned16(old) && aligned16(adv) && (ent == nullptr || aligned16(ent));
  if (done_bits) {
    if (!finish) return ent != nullptr ? (vec ? launch<true, true, false, true>(a, stream)
                                              : launch<false, true, false, true>(a, stream))
                                       : (vec ? launch<true, false, false, true>(a, stream)
                                              : launch<false, false, false, true>(a, stream));
    return ent != nullptr ? (vec ? launch<true, true, true, true>(a, stream) : launch<false, true, true, true>(a, stream))
                          : (vec ? launch<true, false, true, true>(a, stream)
                                 : launch<false, false, true, true>(a, stream));
  }
  if (finish) {
    if (ent != nullptr)
      return vec ? launch<true, true, true, false>(a, stream) : launch<false, true, true, false>(a, stream);
    return vec ? launch<true, false, true, false>(a, stream) : launch<false, false, true, false>(a, stream);
  }
  if (ent != nullptr)
    return vec ? launch<true, true, false, false>(a, stream) : launch<false, true, false, false>(a, stream);
  return vec ? launch<true, false, false, false>(a, stream) : launch<false, false, false, false>(a, stream);
}

// Lead of the PPO role in the multi-GPU step's CTA split (see run_exchange): 0.25 measured best
// at N = 2 (22.1 us per step against 22.5 us with none and 24.2 us with 0.5); B200_RL_PPO_LEAD in
// the environment overrides it for tuning runs.
inline double ppo_lead() {
  static const double v = [] {
    const char* e = std::getenv("B200_RL_PPO_LEAD");
    return e != nullptr ? std::atof(e) : 0.25;
  }();
  return v;
}

// The fused multi-GPU step: every rank calls this with its own batch (the same B, T and n on
// every rank) and the same `epoch` (1 on the first step, peer_next_epoch() of the previous one
// after); ppo_out receives the PPO outputs of all ranks' samples on every rank.  The exchange must
// have been created with one slot of kExchangeRecordBytes bytes, and opened.  workspace as for run().
inline int run_exchange(const float* reward, const void* done, float gamma, int32_t B, int32_t T,
                        float* rtg_out, const float* cur, const float* old, const float* adv, const float* ent,
                        int64_t n, float eps, float* ppo_out, void* workspace, size_t ws_bytes,
                        const PeerExchange* x, unsigned epoch, bool early_reads, bool done_bits,
                        cudaStream_t stream) {
  if (B < 0 || T < 0 || n < 0 || x == nullptr || ppo_out == nullptr || epoch == 0) return kInvalidArgument;
  if (int64_t(B) * T > 0 && (reward == nullptr || done == nullptr || rtg_out == nullptr)) return kInvalidArgument;
  if (n > 0 && (cur == nullptr || old == nullptr || adv == nullptr)) return kInvalidArgument;
  if (x->slots != 1 || x->rec_bytes != kExchangeRecordBytes || x->world > kMaxPeers) return kInvalidArgument;
  for (int r = 0; r < x->world; ++r)
    if (x->base[r] == nullptr) return kInvalidArgument;  // not opened
  if (workspace == nullptr || ws_bytes < ppo::workspace_bytes(n)) return kWorkspaceTooSmall;
  Args a;
  a.early_reads = early_reads;
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
  a.ticket = &static_cast<ppo::Control*>(workspace)->ticket;
  a.partials = ppo::ws_partials(workspace);
  a.ppo_out = ppo_out;
  a.inv_n = ppo::inv_count(int64_t(x->world) * n);
  const int64_t slots = int64_t(sm_count()) * B200_RL_MIN_CTAS;
  // The exchange starts when the rank's PPO chunks are done, so the PPO role gets a share of the
  // CTAs as if its chunks were (1 + lead) times their bytes: it finishes first and the peer
  // records travel while the reward-to-go rows finish.
  const double lead = ppo_lead();
  const int64_t cb = int64_t(double((ent != nullptr ? 16 : 12) * ppo::kChunk) * (1.0 + lead));
  split_roles(a.B, row_bytes(T, done_bits), ppo::num_chunks(n), cb, slots, true, &a.rtg_ctas, &a.ppo_ctas);
  const PeerView pv = peer_view(*x, epoch);
  const bool vec = aligned16(cur) && aligned16(old) && aligned16(adv) && (ent == nullptr || aligned16(ent));
  auto go = [&](auto kern) {
    if (!ensure_dyn_smem(kern, kSmem)) return int(kCudaError);
    return launch_pdl(kern, unsigned(a.rtg_ctas + a.ppo_ctas), kThreads, kSmem, stream, a, pv);
  };
  if (done_bits) {
    if (ent != nullptr)
      return vec ? go(step_exchange_kernel<true, true, true>) : go(step_exchange_kernel<false, true, true>);
    return vec ? go(step_exchange_kernel<true, false, true>) : go(step_exchange_kernel<false, false, true>);
  }
  if (ent != nullptr)
    return vec ? go(step_exchange_kernel<true, true, false>) : go(step_exchange_kernel<false, true, false>);
  return vec ? go(step_exchange_kernel<true, false, false>) : go(step_exchange_kernel<false, false, false>);
}

}  // namespace rl
}  // namespace b200
