// C ABI of libb200ops.so: the declarations live in include/b200ops.h.
//
// Each drop-in entry point has the argument list of the reference's `void reference(...)` for its
// task and runs on the legacy default stream, as the reference grader expects
// (tasks/*/prompt.md "Launch your work on the default stream").  The stream forms return a
// status and take the stream (and, for reductions, the workspace) from the caller.
#include <cuda_runtime.h>

#include "../../include/b200ops.h"
#include "dropin/efficient_kan.cuh"
#include "dropin/fp8_linear.cuh"
#include "dropin/leaky.cuh"
#include "dropin/pow_abs_sqrt_mean.cuh"
#include "dropin/ppo_clip.cuh"
#include "dropin/reward_to_go.cuh"
#include "ops/fp8_pipeline.cuh"
#include "ops/gae.cuh"
#include "ops/kan_backward.cuh"
#include "ops/lif_backward.cuh"
#include "ops/rl_step.cuh"
#include "ops/rtg_chunked.cuh"

namespace {
thread_local int g_last_status = 0;

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline void record(int s) { g_last_status = s; }
}  // namespace

extern "C" {

const char* b200_status_string(int status) { return b200::status_string(status); }
int b200_last_status(void) { return g_last_status; }

int b200_device_fault(void) {
  unsigned v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&v, b200::g_b200_fault, sizeof(v)) != cudaSuccess) return -1;
  const unsigned zero = 0;
  if (cudaMemcpyToSymbol(b200::g_b200_fault, &zero, sizeof(zero)) != cudaSuccess) return -1;
  return int(v);
}

// ---------------------------------------------------------------------------------- robust-L1
void b200_pow_abs_sqrt_mean(const float* inp, const float* target, int64_t batch_size, int64_t height,
                            int64_t width, float* output) {
  record(b200::dropin::pow_abs_sqrt_mean(inp, target, batch_size, height, width, output));
}

size_t b200_robust_l1_workspace_bytes(int64_t n) { return n < 0 ? 0 : b200::robust_l1::workspace_bytes(n); }

int b200_robust_l1_async(const float* inp, const float* target, int64_t n, float* output, void* workspace,
                         size_t workspace_bytes, void* stream) {
  return b200::robust_l1::run(inp, target, n, output, workspace, workspace_bytes, as_stream(stream));
}

int64_t b200_robust_l1_chunk_elems(void) { return b200::robust_l1::kChunk; }

int b200_robust_l1_shard_partials(const float* inp, const float* target, int64_t n, double* partials,
                                  void* stream) {
  return b200::robust_l1::shard_partials(inp, target, n, partials, as_stream(stream));
}

int b200_robust_l1_finish(const double* partials, int64_t n_partials, int64_t n_total, float* output,
                          void* stream) {
  return b200::robust_l1::shard_finish(partials, n_partials, n_total, output, as_stream(stream));
}

// ---------------------------------------------------------------------------------------- PPO
void b200_ppo_clip(const int32_t B, const int32_t T, const int32_t H, const float* current_log_prob,
                   const float* old_log_prob, const float* advantage, const float clip_epsilon, float* output) {
  record(b200::dropin::ppo_clip(B, T, H, current_log_prob, old_log_prob, advantage, nullptr, clip_epsilon, output));
}

void b200_ppo_clip_ext(const int32_t B, const int32_t T, const int32_t H, const float* current_log_prob,
                       const float* old_log_prob, const float* advantage, const float* entropy,
                       const float clip_epsilon, float* output) {
  if (entropy == nullptr) return record(b200::kInvalidArgument);
  record(b200::dropin::ppo_clip(B, T, H, current_log_prob, old_log_prob, advantage, entropy, clip_epsilon, output));
}

size_t b200_ppo_workspace_bytes(int64_t n) { return n < 0 ? 0 : b200::ppo::workspace_bytes(n); }

int b200_ppo_async(const float* current_log_prob, const float* old_log_prob, const float* advantage,
                   const float* entropy, int64_t n, float clip_epsilon, float* output, void* workspace,
                   size_t workspace_bytes, void* stream) {
  return b200::ppo::run(current_log_prob, old_log_prob, advantage, entropy, n, clip_epsilon, output, workspace,
                        workspace_bytes, as_stream(stream));
}

int64_t b200_ppo_chunk_elems(void) { return b200::ppo::kChunk; }
size_t b200_ppo_partial_bytes(void) { return sizeof(b200::ppo::Partial); }

int b200_ppo_shard_partials(const float* current_log_prob, const float* old_log_prob, const float* advantage,
                            const float* entropy, int64_t n, float clip_epsilon, void* partials, void* stream) {
  return b200::ppo::shard_partials(current_log_prob, old_log_prob, advantage, entropy, n, clip_epsilon,
                                   static_cast<b200::ppo::Partial*>(partials), as_stream(stream));
}

int b200_ppo_finish(const void* partials, int64_t n_partials, int64_t n_total, int with_entropy, float* output,
                    void* stream) {
  return b200::ppo::shard_finish(static_cast<const b200::ppo::Partial*>(partials), n_partials, n_total,
                                 with_entropy != 0, output, as_stream(stream));
}

// ------------------------------------------------------------------------------- reward-to-go
void b200_reward_to_go(const float* reward, const bool* done, float gamma, int32_t B, int32_t T, float* output) {
  record(b200::dropin::reward_to_go(reward, done, gamma, B, T, output));
}

int b200_reward_to_go_async(const float* reward, const uint8_t* done, float gamma, int32_t B, int32_t T,
                            float* output, void* stream) {
  return b200::rtg::run(reward, done, gamma, B, T, output, as_stream(stream));
}

int b200_pack_done_async(const uint8_t* done, int32_t B, int32_t T, uint32_t* done_bits, void* stream) {
  return b200::rtg::pack_done(done, B, T, done_bits, as_stream(stream));
}

int b200_reward_to_go_bits_async(const float* reward, const uint32_t* done_bits, float gamma, int32_t B, int32_t T,
                                 float* output, void* stream) {
  return b200::rtg::run_bits(reward, done_bits, gamma, B, T, output, as_stream(stream));
}

int64_t b200_reward_to_go_chunked_workspace_bytes(int32_t B, int32_t T) {
  if (B < 0 || T < 0) return -1;
  return b200::rtgc::workspace_bytes(B, T);
}

int b200_reward_to_go_chunked_async(const float* reward, const void* done, int done_is_bits, float gamma, int32_t B,
                                    int32_t T, float* output, void* workspace, int64_t workspace_bytes,
                                    void* stream) {
  return b200::rtgc::run(reward, done, done_is_bits != 0, gamma, B, T, output, workspace, workspace_bytes,
                         as_stream(stream));
}

int b200_reward_to_go_slice_maps_async(const float* reward, const void* done, int done_is_bits, float gamma,
                                       int32_t B, int32_t T_local, double* slice_maps, void* workspace,
                                       int64_t workspace_bytes, void* stream) {
  return b200::rtgc::slice_maps(reward, done, done_is_bits != 0, gamma, B, T_local,
                                reinterpret_cast<b200::rtgc::Map*>(slice_maps), workspace, workspace_bytes,
                                as_stream(stream));
}

int b200_reward_to_go_slice_scan_async(const float* reward, const void* done, int done_is_bits, float gamma,
                                       int32_t B, int32_t T_local, const double* all_slice_maps, int world,
                                       int rank, float* output, void* workspace, int64_t workspace_bytes,
                                       void* stream) {
  return b200::rtgc::slice_scan(reward, done, done_is_bits != 0, gamma, B, T_local,
                                reinterpret_cast<const b200::rtgc::Map*>(all_slice_maps), world, rank, output,
                                workspace, workspace_bytes, as_stream(stream));
}

// ------------------------------------------------------------------------------ fused RL step
int b200_rl_step_async(const float* reward, const uint8_t* done, float gamma, int32_t B, int32_t T, float* rtg_out,
                       const float* current_log_prob, const float* old_log_prob, const float* advantage,
                       const float* entropy, int64_t n, float clip_epsilon, float* ppo_out, void* workspace,
                       size_t workspace_bytes, void* stream) {
  return b200_rl_step_ex_async(reward, done, gamma, B, T, rtg_out, current_log_prob, old_log_prob, advantage, entropy,
                               n, clip_epsilon, ppo_out, workspace, workspace_bytes, 0u, stream);
}

int b200_rl_step_ex_async(const float* reward, const uint8_t* done, float gamma, int32_t B, int32_t T,
                          float* rtg_out, const float* current_log_prob, const float* old_log_prob,
                          const float* advantage, const float* entropy, int64_t n, float clip_epsilon, float* ppo_out,
                          void* workspace, size_t workspace_bytes, unsigned flags, void* stream) {
  if (flags & ~unsigned(B200_STEP_INPUTS_READY | B200_STEP_DONE_BITS)) return b200::kInvalidArgument;
  return b200::rl::run(reward, done, gamma, B, T, rtg_out, current_log_prob, old_log_prob, advantage, entropy, n,
                       clip_epsilon, ppo_out, workspace, workspace_bytes, true, nullptr,
                       (flags & B200_STEP_INPUTS_READY) != 0, (flags & B200_STEP_DONE_BITS) != 0, as_stream(stream));
}

int b200_rl_step_shard_async(const float* reward, const uint8_t* done, float gamma, int32_t B, int32_t T,
                             float* rtg_out, const float* current_log_prob, const float* old_log_prob,
                             const float* advantage, const float* entropy, int64_t n, float clip_epsilon,
                             void* partials, void* stream) {
  return b200::rl::run(reward, done, gamma, B, T, rtg_out, current_log_prob, old_log_prob, advantage, entropy, n,
                       clip_epsilon, nullptr, nullptr, 0, false, partials, false, false, as_stream(stream));
}

// ------------------------------------------------------------- multi-GPU peer exchange (NVLink)
size_t b200_peer_handle_bytes(void) { return b200::kPeerHandleBytes; }
size_t b200_rl_step_exchange_record_bytes(void) { return b200::rl::kExchangeRecordBytes; }
unsigned b200_peer_next_epoch(unsigned epoch) { return b200::peer_next_epoch(epoch); }

int b200_peer_exchange_create(int world, int rank, int64_t slots, size_t record_bytes, void** exchange,
                              void* handle) {
  b200::PeerExchange* x = nullptr;
  const int st = b200::peer_create(world, rank, slots, record_bytes, &x, handle);
  if (exchange) *exchange = x;
  return st;
}

int b200_peer_exchange_open(void* exchange, const void* handles) {
  return b200::peer_open(static_cast<b200::PeerExchange*>(exchange), handles);
}

int b200_peer_exchange_destroy(void* exchange) { return b200::peer_destroy(static_cast<b200::PeerExchange*>(exchange)); }

int b200_rl_step_exchange_async(const float* reward, const uint8_t* done, float gamma, int32_t B, int32_t T,
                                float* rtg_out, const float* current_log_prob, const float* old_log_prob,
                                const float* advantage, const float* entropy, int64_t n, float clip_epsilon,
                                float* ppo_out, void* workspace, size_t workspace_bytes, void* exchange,
                                unsigned epoch, unsigned flags, void* stream) {
  if (flags & ~unsigned(B200_STEP_INPUTS_READY | B200_STEP_DONE_BITS)) return b200::kInvalidArgument;
  return b200::rl::run_exchange(reward, done, gamma, B, T, rtg_out, current_log_prob, old_log_prob, advantage, entropy,
                                n, clip_epsilon, ppo_out, workspace, workspace_bytes,
                                static_cast<const b200::PeerExchange*>(exchange), epoch,
                                (flags & B200_STEP_INPUTS_READY) != 0, (flags & B200_STEP_DONE_BITS) != 0,
                                as_stream(stream));
}

size_t b200_robust_l1_exchange_record_bytes(void) { return b200::robust_l1::kExchangeRecordBytes; }
int64_t b200_robust_l1_exchange_slots(int64_t n_total, int world) {
  if (n_total < 0 || world < 1) return -1;
  return b200::robust_l1::exchange_slots(n_total, world);
}
int b200_robust_l1_exchange_async(const float* inp, const float* target, int64_t n_total, float* output,
                                  void* workspace, size_t workspace_bytes, void* exchange, unsigned epoch,
                                  void* stream) {
  return b200::robust_l1::run_exchange(inp, target, n_total, output, workspace, workspace_bytes,
                                       static_cast<const b200::PeerExchange*>(exchange), epoch, as_stream(stream));
}

// ----------------------------------------------------------------------------------------- GAE
int b200_gae_async(const float* reward, const float* value, const float* next_value, const uint8_t* done,
                   const uint8_t* terminated, float gamma, float lmbda, int32_t B, int32_t T, float* advantage,
                   float* value_target, void* stream) {
  return b200::gae::run(reward, value, next_value, done, terminated, gamma, lmbda, B, T, advantage, value_target,
                        as_stream(stream));
}

// ---------------------------------------------------------------------------------------- LIF
void b200_leaky(const float* input_current, const float* mem0, const float* beta, const float* threshold,
                int32_t T, int32_t B, int32_t H, float* spikes, float* final_mem) {
  record(b200::dropin::leaky(input_current, mem0, beta, threshold, T, B, H, spikes, final_mem));
}

int b200_leaky_async(const float* input_current, const float* mem0, const float* beta, const float* threshold,
                     int32_t T, int32_t B, int32_t H, float* spikes, float* final_mem, void* stream) {
  return b200::lif::run(input_current, mem0, beta, threshold, T, B, H, spikes, final_mem, as_stream(stream));
}

int b200_leaky_packed_async(const float* input_current, const float* mem0, const float* beta, const float* threshold,
                            int32_t T, int32_t B, int32_t H, uint32_t* spike_bits, float* final_mem, void* stream) {
  return b200::lif::run_packed(input_current, mem0, beta, threshold, T, B, H, spike_bits, final_mem,
                               as_stream(stream));
}

int64_t b200_leaky_checkpoint_bytes(int32_t T, int32_t B, int32_t H) {
  if (T < 0 || B < 0 || H < 0) return -1;
  return b200::lif::checkpoint_count(T) * int64_t(B) * int64_t(H) * int64_t(sizeof(float));
}

int b200_leaky_train_async(const float* input_current, const float* mem0, const float* beta, const float* threshold,
                           int32_t T, int32_t B, int32_t H, float* spikes, float* final_mem, float* checkpoints,
                           void* stream) {
  return b200::lif::run_train(input_current, mem0, beta, threshold, T, B, H, spikes, final_mem, checkpoints,
                              as_stream(stream));
}

int b200_leaky_checkpoints_async(const float* input_current, const float* mem0, const float* beta,
                                 const float* threshold, int32_t T, int32_t B, int32_t H, float* checkpoints,
                                 void* stream) {
  return b200::lif::run_checkpoints(input_current, mem0, beta, threshold, T, B, H, checkpoints, as_stream(stream));
}

int64_t b200_leaky_backward_workspace_bytes(int32_t B, int32_t H) {
  if (B < 0 || H < 0) return -1;
  return b200::lif::backward_workspace_bytes(B, H);
}

int b200_leaky_backward_async(const float* input_current, const float* checkpoints, const float* beta,
                              const float* threshold, int32_t T, int32_t B, int32_t H, const float* grad_spikes,
                              const float* grad_final_mem, float alpha, float* grad_input, float* grad_mem0,
                              float* grad_beta, float* grad_threshold, void* workspace, int64_t workspace_bytes,
                              void* stream) {
  return b200::lif::backward(input_current, checkpoints, beta, threshold, T, B, H, grad_spikes, grad_final_mem, alpha,
                             grad_input, grad_mem0, grad_beta, grad_threshold, workspace, workspace_bytes,
                             as_stream(stream));
}

// --------------------------------------------------------------------------------- FP8 linear
void b200_fp8_linear(const int32_t M, const int32_t K, const int32_t N, const uint8_t* x_fp8, float scale_x,
                     const uint8_t* w_fp8, float scale_w, const uint16_t* bias, uint16_t* output) {
  record(b200::dropin::fp8_linear(M, K, N, x_fp8, scale_x, w_fp8, scale_w, bias, output));
}

int b200_fp8_linear_async(const int32_t M, const int32_t K, const int32_t N, const uint8_t* x_fp8, float scale_x,
                          const uint8_t* w_fp8, float scale_w, const uint16_t* bias, uint16_t* output,
                          void* stream) {
  return b200::fp8::run(M, K, N, x_fp8, scale_x, w_fp8, scale_w, bias, output, as_stream(stream));
}

int b200_fp8_linear_cuda_core_async(const int32_t M, const int32_t K, const int32_t N, const uint8_t* x_fp8,
                                    float scale_x, const uint8_t* w_fp8, float scale_w, const uint16_t* bias,
                                    uint16_t* output, void* stream) {
  return b200::fp8::run_simt(M, K, N, x_fp8, scale_x, w_fp8, scale_w, bias, output, as_stream(stream));
}

int b200_fp8_linear_plan(const int32_t M, const int32_t K, const int32_t N, const uint8_t* x_fp8,
                         const uint8_t* w_fp8) {
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  return b200::fp8::plan_bn(M, N, K, x_fp8, w_fp8);
}

// ------------------------------------------------------------------- E4M3 quantisation (fp8)
size_t b200_fp8_quantize_workspace_bytes(void) { return b200::fp8q::workspace_bytes(); }

int b200_fp8_quantize_async(const void* x, int32_t x_is_bf16, int64_t n, uint8_t* q, float* scale, void* workspace,
                            size_t workspace_bytes, void* stream) {
  return b200::fp8q::run(x, x_is_bf16 != 0, n, q, scale, 1.0f, workspace, workspace_bytes, as_stream(stream));
}

size_t b200_fp8_linear_bf16_workspace_bytes(int32_t M, int32_t K) {
  return M < 0 || K < 0 ? 0 : b200::fp8q::linear_workspace_bytes(M, K);
}

int b200_fp8_linear_bf16_async(const int32_t M, const int32_t K, const int32_t N, const uint16_t* x_bf16,
                               const uint8_t* w_fp8, float scale_w, const uint16_t* bias, uint16_t* output,
                               float* scale_x, void* workspace, size_t workspace_bytes, void* stream) {
  return b200::fp8q::linear_bf16(M, K, N, x_bf16, w_fp8, scale_w, bias, output, scale_x, workspace, workspace_bytes,
                                 as_stream(stream));
}

// ----------------------------------------------------------------------------------------- KAN
void b200_efficient_kan(const float* x, const float* grid, const float* base_weight, const float* spline_weight,
                        const float* spline_scaler, int32_t grid_size, int32_t spline_order, int32_t B, int32_t I,
                        int32_t O, float* out) {
  record(b200::dropin::efficient_kan(x, grid, base_weight, spline_weight, spline_scaler, grid_size, spline_order, B,
                                     I, O, out));
}

size_t b200_efficient_kan_workspace_bytes(int32_t grid_size, int32_t spline_order, int32_t B, int32_t I, int32_t O) {
  if (B < 0 || I < 0 || O < 0 || grid_size < 1 || spline_order < 0) return 0;
  return b200::kan::workspace_bytes(B, I, O, grid_size + spline_order);
}

int b200_efficient_kan_async(const float* x, const float* grid, const float* base_weight, const float* spline_weight,
                             const float* spline_scaler, int32_t grid_size, int32_t spline_order, int32_t B,
                             int32_t I, int32_t O, float* out, void* workspace, size_t workspace_bytes,
                             void* stream) {
  return b200::kan::run(x, grid, base_weight, spline_weight, spline_scaler, grid_size, spline_order, B, I, O, out,
                        workspace, workspace_bytes, as_stream(stream));
}

size_t b200_efficient_kan_backward_workspace_bytes(int32_t grid_size, int32_t spline_order, int32_t B, int32_t I,
                                                   int32_t O) {
  if (grid_size < 1 || spline_order < 0 || B < 0 || I < 0 || O < 0) return 0;
  return b200::kanb::workspace_bytes(B, I, O, grid_size + spline_order);
}

int b200_efficient_kan_backward_async(const float* x, const float* grid, const float* base_weight,
                                      const float* spline_weight, const float* spline_scaler, int32_t grid_size,
                                      int32_t spline_order, int32_t B, int32_t I, int32_t O, const float* grad_out,
                                      float* grad_x, float* grad_base_weight, float* grad_spline_weight,
                                      float* grad_spline_scaler, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  return b200::kanb::backward(x, grid, base_weight, spline_weight, spline_scaler, grid_size, spline_order, B, I, O,
                              grad_out, grad_x, grad_base_weight, grad_spline_weight, grad_spline_scaler, workspace,
                              workspace_bytes, as_stream(stream));
}

}  // extern "C"

// ----------------------------------------------------------------- robust-L1 without allocating
// b200_pow_abs_sqrt_mean_noalloc: the robust-L1 mean for callers that must not allocate device
// memory at all.  Such callers exist: a serving engine or framework that reserves the whole GPU
// for its own pool (a stray cudaMalloc then fails or fragments that pool), a plugin host whose
// contract forbids plugins from allocating, or a latency-critical loop that cannot take the
// implicit device synchronisation and unpredictable latency of cudaMalloc/cudaFree.  The regular
// entry points take their scratch from an arena that cudaMalloc fills on first use; this one uses
// a fixed array of device memory compiled into the library instead.
//
// The array is kNoAllocScratchBytes (131,328 bytes) per GPU: a 256-byte counter block plus one
// fp64 partial per 8192-element chunk, enough for kNoAllocMaxElems = 2^27 elements; larger calls
// are refused with B200_WORKSPACE_TOO_SMALL before anything is launched.  Every GPU that loads the
// library holds the array until the process exits.  All calls on a device share it, so calls that
// overlap on the GPU (different streams, no ordering) race on it; calls on one stream are safe.
// The first call on each device looks up the array's device address (cudaGetSymbolAddress with
// that device current) and caches it with the context's id; make that first call before any
// stream capture begins.  A later call in another context of the device (after cudaDeviceReset)
// looks the address up again.
// Each call clears the counter block on its stream before launching, so a call never depends on
// what an earlier call left there; the partials are fully rewritten by every call.
namespace {
constexpr int64_t kNoAllocMaxElems = int64_t(1) << 27;
constexpr size_t kNoAllocScratchBytes =
    256 + size_t(kNoAllocMaxElems / b200::robust_l1::kChunk) * sizeof(double);  // 131,328 bytes
}  // namespace

// In host code this name is only a stand-in for the array, not a device address: the kernel must
// be given the address returned by cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
// The unique id of the calling thread's current context (cuCtxGetCurrent + cuCtxGetId, fetched
// through the runtime so the library needs no -lcuda link), or 0 when there is none yet.  Ids are
// never reused within a process, so a context re-created after cudaDeviceReset has a new one.
typedef int (*CtxGetCurrentFn)(void**);
typedef int (*CtxGetIdFn)(void*, unsigned long long*);

unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool looked_up = false;
  if (!looked_up) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
    looked_up = true;
  }
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != 0 || ctx == nullptr) return 0;
  return get_id(ctx, &id) == 0 ? id : 0;
}

// Device address of g_noalloc_scratch on the current device: looked up once per device and
// context (cudaGetSymbolAddress with that device current), and looked up again when the device's
// context has changed since (a primary context re-created after cudaDeviceReset may map the
// library's module at another address).
void* noalloc_scratch(int* status) {
  static void* addr[64] = {nullptr};
  static unsigned long long ctx_id[64] = {0};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *status = b200::kCudaError;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  const unsigned long long id = current_context_id();
  if (addr[dev] == nullptr || id == 0 || id != ctx_id[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      *status = b200::kCudaError;
      return nullptr;
    }
    addr[dev] = p;
    ctx_id[dev] = current_context_id();  // the lookup has made the device's context current
  }
  *status = b200::kOk;
  return addr[dev];
}
}  // namespace

extern "C" int b200_pow_abs_sqrt_mean_noalloc(const float* inp, const float* target, int64_t batch_size,
                                              int64_t height, int64_t width, float* output, void* stream) {
  const int64_t n = b200::robust_l1::abi_count(batch_size, height, width);
  if (n < 0) return b200::kInvalidArgument;
  if (n > kNoAllocMaxElems) return b200::kWorkspaceTooSmall;
  int st = 0;
  void* scratch = noalloc_scratch(&st);
  if (st != b200::kOk) return st;
  if (cudaMemsetAsync(scratch, 0, 256, as_stream(stream)) != cudaSuccess) return b200::kCudaError;
  return b200::robust_l1::run(inp, target, n, output, scratch, kNoAllocScratchBytes, as_stream(stream));
}
