/*
 * b200ops.h - C ABI of the B200 (sm_100a) kernels for the six ops of
 * Mohamed-Alaboudi/cuda-optimization-benchmark.
 *
 * Two forms per op:
 *
 *  - Drop-in form, b200_<task>(...): the exact argument list and meaning of the reference's
 *    `void reference(...)` for that task (tasks/<task>/tests/task.json:3), with C linkage so a
 *    ctypes/cffi/dlsym caller can bind it by name.  Device pointers, work on the legacy default
 *    stream, nothing returned; errors surface at the caller's next synchronize, as with the
 *    reference.  b200_last_status() reports the status of the calling thread's last drop-in call.
 *    Ops that need scratch take it from a per-device arena allocated on first use.
 *
 *  - Stream form, b200_<op>_async(...): the same work on a caller stream (a cudaStream_t passed
 *    as void*), returning a b200 status code (0 = ok).  Reductions also take a caller workspace
 *    and expose shard/finish halves for multi-GPU use.
 *
 * All pointers are device pointers to contiguous row-major data.  `bool` is one byte (0 or 1);
 * fp8 E4M3 and bf16 buffers are passed as uint8_t / uint16_t.
 */
#ifndef B200OPS_H
#define B200OPS_H

#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes of the stream forms and of b200_last_status(). */
#define B200_OK 0
#define B200_INVALID_ARGUMENT 1
#define B200_CUDA_ERROR 2
#define B200_UNSUPPORTED 3
#define B200_WORKSPACE_TOO_SMALL 4
#define B200_TIMEOUT 5

const char* b200_status_string(int status);
int b200_last_status(void);

/* Device-side fault word of the current device: bit 0 = a bounded wait inside a kernel gave up
 * (its results are then unreliable).  Synchronizes the device, returns the word (or -1 when the
 * read itself fails) and clears it.  No reference counterpart: the reference's kernels have no
 * waits. */
int b200_device_fault(void);

/* ---------------------------------------------------------------------------------------------
 * Robust-L1 mean (task pow_abs_sqrt_mean): output[0] = mean(sqrt((inp - target)^2 + 1e-6)).
 * Replaces `void reference(const float* inp, const float* target, int64_t batch_size,
 * int64_t height, int64_t width, float* output)`: tasks/pow_abs_sqrt_mean/tests/task.json:3,
 * reference/pow_abs_sqrt_mean/solution.cu:99.
 * ------------------------------------------------------------------------------------------- */
void b200_pow_abs_sqrt_mean(const float* inp, const float* target, int64_t batch_size, int64_t height,
                            int64_t width, float* output);

/* Stream form over n elements.  workspace: b200_robust_l1_workspace_bytes(n) bytes, zero-filled
 * once before its first use (every call leaves it ready for the next). */
size_t b200_robust_l1_workspace_bytes(int64_t n);
int b200_robust_l1_async(const float* inp, const float* target, int64_t n, float* output, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Robust-L1 mean that allocates nothing, for callers that may not allocate device memory: a
 * framework or serving engine that owns the whole GPU through its own memory pool, a plugin host
 * whose contract forbids allocation, or a latency-critical loop that cannot take cudaMalloc's
 * implicit synchronisation.  This entry point has no counterpart in the reference.  Scratch is a
 * 131,328-byte device array inside the library, held by every GPU that loads it until exit, so a
 * call may cover at most B200_NOALLOC_MAX_ELEMS elements (batch_size*4*height*width); larger calls
 * return B200_WORKSPACE_TOO_SMALL without launching.  The first call on a device looks up the
 * array's device address; make it before any stream capture begins (the lookup is repeated once
 * when the device's context changes, e.g. after cudaDeviceReset).  All calls on a device share
 * the array: calls that overlap on the GPU race, calls ordered on one stream do not. */
#define B200_NOALLOC_MAX_ELEMS 134217728LL
int b200_pow_abs_sqrt_mean_noalloc(const float* inp, const float* target, int64_t batch_size, int64_t height,
                                   int64_t width, float* output, void* stream);

/* Multi-GPU halves.  The global element range is cut into chunks of b200_robust_l1_chunk_elems();
 * a shard must start on a chunk boundary.  shard_partials writes one double per local chunk;
 * finish sums the gathered partials of all shards (in chunk order) and divides by n_total.  The
 * result is bit-identical to b200_robust_l1_async on the whole range. */
int64_t b200_robust_l1_chunk_elems(void);
int b200_robust_l1_shard_partials(const float* inp, const float* target, int64_t n, double* partials,
                                  void* stream);
int b200_robust_l1_finish(const double* partials, int64_t n_partials, int64_t n_total, float* output,
                          void* stream);

/* ---------------------------------------------------------------------------------------------
 * PPO clipped loss + diagnostics (task ppo_clip): output[0..6) = [loss, clip_fraction,
 * approx_kl, ess, max_ratio, mean_ratio].
 * Replaces `void reference(const int32_t B, const int32_t T, const int32_t H,
 * const float* current_log_prob, const float* old_log_prob, const float* advantage,
 * const float clip_epsilon, float* output)`: tasks/ppo_clip/tests/task.json:3,
 * reference/ppo_clip/solution.cu:165.
 * ------------------------------------------------------------------------------------------- */
void b200_ppo_clip(const int32_t B, const int32_t T, const int32_t H, const float* current_log_prob,
                   const float* old_log_prob, const float* advantage, const float clip_epsilon, float* output);

/* Extended form (no reference counterpart; the BASELINE RL-pipeline metric set): also reads a
 * per-sample entropy stream and writes a 7th output, its mean. */
void b200_ppo_clip_ext(const int32_t B, const int32_t T, const int32_t H, const float* current_log_prob,
                       const float* old_log_prob, const float* advantage, const float* entropy,
                       const float clip_epsilon, float* output);

/* Stream form over n samples; entropy may be NULL (6 outputs) or a stream (7 outputs).
 * workspace: b200_ppo_workspace_bytes(n) bytes, zero-filled once before first use. */
size_t b200_ppo_workspace_bytes(int64_t n);
int b200_ppo_async(const float* current_log_prob, const float* old_log_prob, const float* advantage,
                   const float* entropy, int64_t n, float clip_epsilon, float* output, void* workspace,
                   size_t workspace_bytes, void* stream);

/* Multi-GPU halves: one b200_ppo_partial_bytes() record per chunk of b200_ppo_chunk_elems()
 * samples; shards start on chunk boundaries; finish is bit-identical to the one-device form. */
int64_t b200_ppo_chunk_elems(void);
size_t b200_ppo_partial_bytes(void);
int b200_ppo_shard_partials(const float* current_log_prob, const float* old_log_prob, const float* advantage,
                            const float* entropy, int64_t n, float clip_epsilon, void* partials, void* stream);
int b200_ppo_finish(const void* partials, int64_t n_partials, int64_t n_total, int with_entropy, float* output,
                    void* stream);

/* ---------------------------------------------------------------------------------------------
 * Discounted reward-to-go with done flags (task reward_to_go).
 * Replaces `void reference(const float* reward, const bool* done, float gamma, int32_t B,
 * int32_t T, float* output)`: tasks/reward_to_go/tests/task.json:3,
 * reference/reward_to_go/solution.cu:237.
 * ------------------------------------------------------------------------------------------- */
void b200_reward_to_go(const float* reward, const bool* done, float gamma, int32_t B, int32_t T, float* output);
int b200_reward_to_go_async(const float* reward, const uint8_t* done, float gamma, int32_t B, int32_t T,
                            float* output, void* stream);

/* Done flags as bits (no reference counterpart; the ABI fixes one bool per step): word [b, w] of
 * done_bits (uint32 [B, ceil(T/32)]) holds done[b, 32w .. 32w + 31], bit t % 32 for step t, bits
 * past T zero.  b200_pack_done_async packs the bool layout; b200_reward_to_go_bits_async is
 * b200_reward_to_go_async reading the bits (the same output bits, 8 1/8 instead of 9 bytes moved
 * per step). */
int b200_pack_done_async(const uint8_t* done, int32_t B, int32_t T, uint32_t* done_bits, void* stream);
int b200_reward_to_go_bits_async(const float* reward, const uint32_t* done_bits, float gamma, int32_t B, int32_t T,
                                 float* output, void* stream);

/* Long rows (no reference counterpart): reward-to-go parallel along T.  The row is cut into
 * 1056-step chunks, each on its own warp (chunk maps in fp64, the carries composed from them, then
 * each chunk rescanned from its carry), so a batch of few long rows fills the GPU.  One cooperative
 * launch of one CTA per SM: 9 bytes per step from HBM, plus the second read of the chunks that L2
 * does not serve.  done is bytes [B, T], or with done_is_bits != 0 the words of
 * b200_pack_done_async.  Outputs within the reward-to-go tolerance of the oracle (the carries'
 * fp64 association differs from b200_reward_to_go_async's) and the same bits on every call.
 * Workspace: b200_reward_to_go_chunked_workspace_bytes(B, T) bytes (-1 for negative sizes),
 * 8-byte aligned, zero-filled once before first use (its first 8 bytes count grid-barrier
 * arrivals), used on one stream at a time.
 *
 * Sharded over time across GPUs: rank r holds steps [offset_r, offset_r + T_local) of every row
 * (any T_local >= 1 per rank; the same B everywhere).  Each rank calls
 * b200_reward_to_go_slice_maps_async (writes its [B] slice maps, two doubles per row), the ranks
 * all-gather them into [world, B, 2] doubles in rank order, and each rank calls
 * b200_reward_to_go_slice_scan_async with the same workspace (it still holds the chunk maps) to
 * write its [B, T_local] outputs (these two read each chunk twice from HBM: 14 bytes per step). */
int64_t b200_reward_to_go_chunked_workspace_bytes(int32_t B, int32_t T);
int b200_reward_to_go_chunked_async(const float* reward, const void* done, int done_is_bits, float gamma, int32_t B,
                                    int32_t T, float* output, void* workspace, int64_t workspace_bytes,
                                    void* stream);
int b200_reward_to_go_slice_maps_async(const float* reward, const void* done, int done_is_bits, float gamma,
                                       int32_t B, int32_t T_local, double* slice_maps, void* workspace,
                                       int64_t workspace_bytes, void* stream);
int b200_reward_to_go_slice_scan_async(const float* reward, const void* done, int done_is_bits, float gamma,
                                       int32_t B, int32_t T_local, const double* all_slice_maps, int world,
                                       int rank, float* output, void* workspace, int64_t workspace_bytes,
                                       void* stream);

/* ---------------------------------------------------------------------------------------------
 * Fused RL loss step (no reference counterpart: the BASELINE RL pipeline, configs[1], runs
 * reward_to_go and ppo_clip back to back on independent inputs).  One launch computes both;
 * rtg_out is bit-identical to b200_reward_to_go_async and ppo_out to b200_ppo_async on the same
 * inputs.  entropy may be NULL (6 PPO outputs) or a stream (7).  workspace as b200_ppo_async
 * (b200_ppo_workspace_bytes(n), zero-filled once; the same buffer may serve both entry points).
 * ------------------------------------------------------------------------------------------- */
int b200_rl_step_async(const float* reward, const uint8_t* done, float gamma, int32_t B, int32_t T, float* rtg_out,
                       const float* current_log_prob, const float* old_log_prob, const float* advantage,
                       const float* entropy, int64_t n, float clip_epsilon, float* ppo_out, void* workspace,
                       size_t workspace_bytes, void* stream);
/* The step kernels are launched with programmatic dependent launch: a step may begin while the
 * kernel before it on the stream is finishing.  By default it waits for that kernel before reading
 * anything, so only the launch latency overlaps.  With B200_STEP_INPUTS_READY in `flags` the caller
 * declares that the kernel launched just before on the stream writes none of this step's inputs
 * (they were written by copies, or by kernels launched earlier): the inputs are then read while
 * that kernel finishes, and the step waits only before its own writes.  Steps over resident
 * batches issued back to back qualify; a step right after the kernel producing its log-probs does
 * not.  With B200_STEP_DONE_BITS, `done` points to the flags as bits (uint32 words [B, ceil(T/32)],
 * b200_pack_done_async) instead of bytes: same results, 1/8 of the flags' bytes.  Other flag bits
 * are rejected. */
#define B200_STEP_INPUTS_READY 1u
#define B200_STEP_DONE_BITS 2u
int b200_rl_step_ex_async(const float* reward, const uint8_t* done, float gamma, int32_t B, int32_t T,
                          float* rtg_out, const float* current_log_prob, const float* old_log_prob,
                          const float* advantage, const float* entropy, int64_t n, float clip_epsilon, float* ppo_out,
                          void* workspace, size_t workspace_bytes, unsigned flags, void* stream);
/* Multi-GPU shard form: the PPO half writes its per-chunk partials (as b200_ppo_shard_partials)
 * for a cross-GPU gather and b200_ppo_finish. */
int b200_rl_step_shard_async(const float* reward, const uint8_t* done, float gamma, int32_t B, int32_t T,
                             float* rtg_out, const float* current_log_prob, const float* old_log_prob,
                             const float* advantage, const float* entropy, int64_t n, float clip_epsilon,
                             void* partials, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Multi-GPU RL step with the PPO exchange fused into the kernel (one process per GPU of one node,
 * NVLink / NVSwitch peer memory through CUDA IPC; no collective library on the step's path).
 * Each rank creates an exchange (its 64-byte IPC handle comes back in `handle`), the ranks swap
 * handles over their own channel, and each opens the others' (`handles`: world x 64 bytes in rank
 * order).  b200_rl_step_exchange_async then runs one rank's step: its own reward-to-go batch and
 * PPO samples (the same B, T, n on every rank; the exchange created with slots = 1 and
 * record_bytes = b200_rl_step_exchange_record_bytes()); `epoch` is the same on every rank, 1 on the
 * first step and b200_peer_next_epoch(previous) after; `flags` as b200_rl_step_ex_async.  Each rank
 * reduces its own PPO chunk partials exactly as b200_rl_step_async does, stores its totals into
 * every rank's buffer as 8-byte {word, epoch} values (no fence or flag needed), and adds all ranks'
 * totals in rank order: every rank's ppo_out receives the same bits, the outputs over all ranks'
 * samples (with one rank, bit-identical to b200_rl_step_async).  A rank whose totals do not arrive
 * within 2 s makes the others set bit 0 of the device fault word (b200_last_status after a
 * synchronize) instead of hanging.
 * ------------------------------------------------------------------------------------------- */
size_t b200_peer_handle_bytes(void);
size_t b200_rl_step_exchange_record_bytes(void);
unsigned b200_peer_next_epoch(unsigned epoch);
int b200_peer_exchange_create(int world, int rank, int64_t slots, size_t record_bytes, void** exchange,
                              void* handle);
int b200_peer_exchange_open(void* exchange, const void* handles);
int b200_peer_exchange_destroy(void* exchange);
int b200_rl_step_exchange_async(const float* reward, const uint8_t* done, float gamma, int32_t B, int32_t T,
                                float* rtg_out, const float* current_log_prob, const float* old_log_prob,
                                const float* advantage, const float* entropy, int64_t n, float clip_epsilon,
                                float* ppo_out, void* workspace, size_t workspace_bytes, void* exchange,
                                unsigned epoch, unsigned flags, void* stream);

/* Robust-L1 over GPUs with the partial exchange fused into the kernel (one process per GPU of one
 * node; no counterpart in the reference, whose op runs on one device: it is
 * reference/pow_abs_sqrt_mean/solution.cu:99-118's reduction split over ranks).  Rank r holds the
 * elements of global chunks [floor(C r / world), floor(C (r + 1) / world)) of the n_total-element
 * range, C = ceil(n_total / b200_robust_l1_chunk_elems()) (inp / target point at the first of them).
 * Each rank creates an exchange with b200_peer_exchange_create(world, rank,
 * b200_robust_l1_exchange_slots(n_total, world), b200_robust_l1_exchange_record_bytes(), ...),
 * the ranks swap handles and open them as for the RL step, and every call passes the same `epoch` on
 * every rank (1 first, then b200_peer_next_epoch(previous)).  Each rank's kernel pushes its chunk
 * partials to every rank over NVLink as they are computed and every rank reduces all of them in
 * chunk order: every rank's output[0] is bit-identical to b200_robust_l1_async over the whole range
 * on one GPU, for any number of ranks.  workspace: 256 bytes, the first 4 zero before the first
 * call (left zero).  A rank whose partials do not arrive within 2 s makes the others set bit 0 of
 * the device fault word instead of hanging. */
size_t b200_robust_l1_exchange_record_bytes(void);
int64_t b200_robust_l1_exchange_slots(int64_t n_total, int world);
int b200_robust_l1_exchange_async(const float* inp, const float* target, int64_t n_total, float* output,
                                  void* workspace, size_t workspace_bytes, void* exchange, unsigned epoch,
                                  void* stream);

/* ---------------------------------------------------------------------------------------------
 * Generalised advantage estimation (no reference counterpart: the step between reward_to_go and
 * ppo_clip in the reference's source library, TorchRL's generalized_advantage_estimate; Schulman
 * et al. 2016).  Per row of [B, T] (time along T), with done / terminated one byte per element:
 *   delta[t] = reward[t] + gamma * next_value[t] * (1 - terminated[t]) - value[t]
 *   advantage[t] = delta[t] + gamma * lambda * (1 - done[t]) * advantage[t + 1]  (0 past T - 1)
 *   value_target[t] = advantage[t] + value[t]
 * With value = next_value = 0, terminated = done and lmbda = 1 the advantages are bit-identical to
 * b200_reward_to_go_async.
 * ------------------------------------------------------------------------------------------- */
int b200_gae_async(const float* reward, const float* value, const float* next_value, const uint8_t* done,
                   const uint8_t* terminated, float gamma, float lmbda, int32_t B, int32_t T, float* advantage,
                   float* value_target, void* stream);

/* ---------------------------------------------------------------------------------------------
 * Leaky integrate-and-fire layer (task leaky).
 * Replaces `void reference(const float* input_current, const float* mem0, const float* beta,
 * const float* threshold, int32_t T, int32_t B, int32_t H, float* spikes, float* final_mem)`:
 * tasks/leaky/tests/task.json:3, reference/leaky/solution.cu:106.
 * ------------------------------------------------------------------------------------------- */
void b200_leaky(const float* input_current, const float* mem0, const float* beta, const float* threshold,
                int32_t T, int32_t B, int32_t H, float* spikes, float* final_mem);
int b200_leaky_async(const float* input_current, const float* mem0, const float* beta, const float* threshold,
                     int32_t T, int32_t B, int32_t H, float* spikes, float* final_mem, void* stream);
/* Bit-packed spikes: spike_bits is uint32 [ceil(T / 32), B*H]; bit t % 32 of word [t / 32][n] is
 * the spike of neuron n (n = b*H + h) at step t, bits past T zero.  The same arithmetic as
 * b200_leaky_async (so the same spikes and final_mem bits); 1/32 of its spike bytes. */
int b200_leaky_packed_async(const float* input_current, const float* mem0, const float* beta, const float* threshold,
                            int32_t T, int32_t B, int32_t H, uint32_t* spike_bits, float* final_mem, void* stream);

/* Training (no reference counterpart: the backward of snnTorch's Leaky, the layer the task
 * restates, through its default arctangent spike surrogate with the reset detached).
 *
 * b200_leaky_train_async: b200_leaky_async (same spikes and final_mem bits) that also stores the
 * membrane checkpoints [ceil(T / 16), B, H] fp32: checkpoint k is the state before step 16k
 * (checkpoint 0 = mem0); b200_leaky_checkpoint_bytes gives their size (-1 for negative sizes).
 * b200_leaky_checkpoints_async stores the checkpoints alone (after a forward that did not).
 *
 * b200_leaky_backward_async: from the checkpoints, the incoming grad_spikes [T, B, H] and
 * grad_final_mem [B, H] (may be NULL: zero), with u[t] = mem[t] - threshold, r[t] = the reset at
 * step t, s'(u) = (alpha / 2) / (1 + (pi / 2 * alpha * u)^2) and g[t] = grad_spikes[t] * s'(u[t])
 * + beta * g[t + 1] (beta * g[T] := grad_final_mem):
 *   grad_input[t] = g[t];  grad_mem0 = beta * g[0];
 *   grad_beta[h] = [0 <= beta[h] <= 1] * sum_{b,t} g[t] * mem[t - 1];
 *   grad_threshold[h] = -sum_{b,t} (grad_spikes[t] * s'(u[t]) + r[t] * g[t]).
 * grad_mem0, grad_beta and grad_threshold may be NULL (not computed); grad_beta or grad_threshold
 * need a workspace of b200_leaky_backward_workspace_bytes(B, H) bytes (status 4 if smaller).  The
 * sums over b are taken in a fixed order: results do not depend on the launch shape. */
int64_t b200_leaky_checkpoint_bytes(int32_t T, int32_t B, int32_t H);
int b200_leaky_train_async(const float* input_current, const float* mem0, const float* beta, const float* threshold,
                           int32_t T, int32_t B, int32_t H, float* spikes, float* final_mem, float* checkpoints,
                           void* stream);
int b200_leaky_checkpoints_async(const float* input_current, const float* mem0, const float* beta,
                                 const float* threshold, int32_t T, int32_t B, int32_t H, float* checkpoints,
                                 void* stream);
int64_t b200_leaky_backward_workspace_bytes(int32_t B, int32_t H);
int b200_leaky_backward_async(const float* input_current, const float* checkpoints, const float* beta,
                              const float* threshold, int32_t T, int32_t B, int32_t H, const float* grad_spikes,
                              const float* grad_final_mem, float alpha, float* grad_input, float* grad_mem0,
                              float* grad_beta, float* grad_threshold, void* workspace, int64_t workspace_bytes,
                              void* stream);

/* ---------------------------------------------------------------------------------------------
 * KAN linear layer (task efficient_kan): out[B, O] = silu(x) . base_weight^T + bases(x) .
 * (spline_weight * spline_scaler)^T, with the G + K B-spline bases of order K on each input's
 * knot grid[I, G + 2K + 1].
 * Replaces `void reference(const float* x, const float* grid, const float* base_weight,
 * const float* spline_weight, const float* spline_scaler, int32_t grid_size, int32_t spline_order,
 * int32_t B, int32_t I, int32_t O, float* out)`: tasks/efficient_kan/tests/task.json:3,
 * reference/efficient_kan/solution.cu:177.
 * ------------------------------------------------------------------------------------------- */
void b200_efficient_kan(const float* x, const float* grid, const float* base_weight, const float* spline_weight,
                        const float* spline_scaler, int32_t grid_size, int32_t spline_order, int32_t B, int32_t I,
                        int32_t O, float* out);
/* Stream form; workspace: b200_efficient_kan_workspace_bytes(...) bytes (no initialisation). */
size_t b200_efficient_kan_workspace_bytes(int32_t grid_size, int32_t spline_order, int32_t B, int32_t I, int32_t O);
int b200_efficient_kan_async(const float* x, const float* grid, const float* base_weight, const float* spline_weight,
                             const float* spline_scaler, int32_t grid_size, int32_t spline_order, int32_t B,
                             int32_t I, int32_t O, float* out, void* workspace, size_t workspace_bytes,
                             void* stream);

/* Backward of the layer (no reference counterpart: the gradients torch autograd forms through
 * tasks/efficient_kan/reference.py:33-46) for grad_out [B, O]: grad_x [B, I], grad_base_weight
 * [O, I], grad_spline_weight [O, I, G+K], grad_spline_scaler [O, I]; any of them may be NULL (not
 * computed).  The two GEMMs (grad_out . W' and grad_out^T . A) run on the forward's split-fp16
 * tensor-core kernel.  Workspace: b200_efficient_kan_backward_workspace_bytes(...) bytes (no
 * initialisation); status 5 when G + 2K + 1 > 64 or the (1 + G + K)-row tiles exceed shared memory. */
size_t b200_efficient_kan_backward_workspace_bytes(int32_t grid_size, int32_t spline_order, int32_t B, int32_t I,
                                                   int32_t O);
int b200_efficient_kan_backward_async(const float* x, const float* grid, const float* base_weight,
                                      const float* spline_weight, const float* spline_scaler, int32_t grid_size,
                                      int32_t spline_order, int32_t B, int32_t I, int32_t O, const float* grad_out,
                                      float* grad_x, float* grad_base_weight, float* grad_spline_weight,
                                      float* grad_spline_scaler, void* workspace, size_t workspace_bytes,
                                      void* stream);

/* ---------------------------------------------------------------------------------------------
 * FP8 E4M3 linear layer (task fp8_linear): output[M, N] (bf16) =
 * (x_fp8[M, K] . w_fp8[N, K]^T) / (scale_x * scale_w) + bias[N].
 * Replaces `void reference(const int32_t M, const int32_t K, const int32_t N,
 * const __nv_fp8_e4m3* x_fp8, float scale_x, const __nv_fp8_e4m3* w_fp8, float scale_w,
 * const __nv_bfloat16* bias, __nv_bfloat16* output)`: tasks/fp8_linear/tests/task.json:3,
 * reference/fp8_linear/solution.cu:276.  x_fp8 / w_fp8 are E4M3 bytes, bias / output bf16 bits.
 * ------------------------------------------------------------------------------------------- */
void b200_fp8_linear(const int32_t M, const int32_t K, const int32_t N, const uint8_t* x_fp8, float scale_x,
                     const uint8_t* w_fp8, float scale_w, const uint16_t* bias, uint16_t* output);
int b200_fp8_linear_async(const int32_t M, const int32_t K, const int32_t N, const uint8_t* x_fp8, float scale_x,
                          const uint8_t* w_fp8, float scale_w, const uint16_t* bias, uint16_t* output,
                          void* stream);
/* The CUDA-core path alone (any shape and alignment), for cross-checking the tensor-core path. */
int b200_fp8_linear_cuda_core_async(const int32_t M, const int32_t K, const int32_t N, const uint8_t* x_fp8,
                                    float scale_x, const uint8_t* w_fp8, float scale_w, const uint16_t* bias,
                                    uint16_t* output, void* stream);
/* Tile width the tensor-core path would use for this call (256, 128 or 64), or 0 when the call
 * takes the CUDA-core path (K not a multiple of 16, or an operand not 16-byte aligned). */
int b200_fp8_linear_plan(const int32_t M, const int32_t K, const int32_t N, const uint8_t* x_fp8,
                         const uint8_t* w_fp8);

/* ---------------------------------------------------------------------------------------------
 * Per-tensor E4M3 quantisation, the step before fp8_linear (tasks/fp8_linear/reference.py:15-18,
 * `_quantize`): scale = fp32(448 / max(max|x|, 1e-9)) (division in fp64), q = e4m3(clamp(x * scale,
 * -448, 448)), round to nearest even, NaN kept (0x7F with the input's sign).  x holds n fp32
 * values, or bf16 values when x_is_bf16 != 0; q receives n bytes (may be NULL: amax and scale
 * only); scale (device, may be NULL) receives the scale.  workspace:
 * b200_fp8_quantize_workspace_bytes() bytes, zero-filled once before first use.
 * ------------------------------------------------------------------------------------------- */
size_t b200_fp8_quantize_workspace_bytes(void);
int b200_fp8_quantize_async(const void* x, int32_t x_is_bf16, int64_t n, uint8_t* q, float* scale, void* workspace,
                            size_t workspace_bytes, void* stream);
/* The linear layer from a bf16 activation: quantise x [M, K] on the device and run the E4M3 GEMM
 * with it; output bit-identical to b200_fp8_quantize_async followed by b200_fp8_linear_async with
 * the computed scale.  scale_x (device, may be NULL) receives the activation scale.  workspace:
 * b200_fp8_linear_bf16_workspace_bytes(M, K) bytes, zero-filled once before first use. */
size_t b200_fp8_linear_bf16_workspace_bytes(int32_t M, int32_t K);
int b200_fp8_linear_bf16_async(const int32_t M, const int32_t K, const int32_t N, const uint16_t* x_bf16,
                               const uint8_t* w_fp8, float scale_w, const uint16_t* bias, uint16_t* output,
                               float* scale_x, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200OPS_H */
