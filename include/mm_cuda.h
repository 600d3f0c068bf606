/*
 * mm_cuda.h -- C ABI of the sm_100a backend for the mini-MLA engine's online GRPO step.
 *
 * This is the boundary a `backend = "cuda"` Execution binds to. Each entry point names
 * the reference interface it replaces (paths and lines are in the reference engine):
 *
 *   class Execution             include/mini_mla/execution.hpp:28-61
 *   make_execution(...)         src/infer/inference.cpp:314-329
 *   CpuDecoder prefill/decode   src/infer/inference.cpp:47-174
 *   sample_token                src/infer/inference.cpp:345-426
 *   rollout()                   src/train/trainer.cpp:187-213
 *   GRPO update body            src/train/trainer.cpp:814-891
 *   Optimizer::step (AdamW)     src/train/optimizer.cpp:105-161
 *
 * Conventions (mirroring the reference's Result/ErrorCode, include/mini_mla/result.hpp:9-16):
 *   - every call returns 0 on success or 1 + ErrorCode:
 *       MM_INVALID_ARGUMENT 1, MM_IO_ERROR 2, MM_UNSUPPORTED 3, MM_OUT_OF_MEMORY 4,
 *       MM_GPU_ERROR 5, MM_NUMERICAL_ERROR 6;
 *     mm_cuda_last_error() returns the message of the last failure on that context;
 *   - inputs are validated before anything is mutated; a failed update leaves weights,
 *     moments and the step count unchanged (tests/test_training.cpp:192-206, 256-263);
 *   - host buffers are caller-owned and borrowed for the call only; device memory is
 *     owned by the context; one context per GPU; every call returns completed results;
 *   - parameters cross the boundary as one flat float32 array in the reference's
 *     registry order and [in, out] row-major layout (src/model/model.cpp:40-63);
 *   - token ids are uint16 (vocabulary <= 65535, src/model/config.cpp:35).
 * A context is not thread-safe; the reference never shares an Execution across threads.
 */
#ifndef MM_CUDA_H
#define MM_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    MM_OK = 0,
    MM_INVALID_ARGUMENT = 1,
    MM_IO_ERROR = 2,
    MM_UNSUPPORTED = 3,
    MM_OUT_OF_MEMORY = 4,
    MM_GPU_ERROR = 5,
    MM_NUMERICAL_ERROR = 6
};

/* ModelConfig (include/mini_mla/model_config.hpp:5-19). */
typedef struct mm_model_desc {
    int32_t vocab_size, max_sequence_length, n_layers, d_model, n_heads;
    int32_t head_dim_nope, head_dim_rope, head_dim_value, q_lora_rank, kv_lora_rank, d_ff;
    float norm_epsilon, rope_theta;
} mm_model_desc;

/* OptimizerConfig, AdamW fields (include/mini_mla/optimizer.hpp:5-14). */
typedef struct mm_adamw_desc {
    float beta1, beta2, epsilon, weight_decay, clip_norm;
} mm_adamw_desc;

/* StepResult (include/mini_mla/execution.hpp:21-23) plus the GRPO host sums
 * (trainer.cpp:840-841) and the skip rule (trainer.cpp:818-820). */
typedef struct mm_step_result {
    double loss;          /* sum over tokens of objective / (n_total * supervised_i) */
    double kl;            /* same for the k3 KL term */
    double grad_norm;     /* pre-clip global gradient norm (optimizer.cpp:128) */
    int32_t skipped;      /* 1 when every advantage of the update is zero */
    int32_t reserved;
} mm_step_result;

typedef struct mm_cuda_ctx mm_cuda_ctx;

/* ---------------------------------------------------------------- host helpers */

/* ModelConfig::parameter_count (src/model/config.cpp:7-19); -1 if the config is invalid. */
int64_t mm_model_parameter_count(const mm_model_desc* desc);

/* Model::create's seeded initialisation (src/model/model.cpp:20-75), on the host, into a
 * caller buffer of mm_model_parameter_count() floats. Same float arithmetic as the
 * reference, so the weights are identical. */
int mm_model_init_params(const mm_model_desc* desc, uint64_t seed, float* out);

/* cosine_learning_rate (src/train/optimizer.cpp:162-173). */
float mm_cosine_learning_rate(uint64_t completed, uint64_t total, uint64_t warmup, float peak,
                              float minimum_fraction);

/* ---------------------------------------------------------------- context */

/* make_execution(model, optimizer, "cuda", ...): allocates device state on `device`.
 * trainable != 0 allocates gradients and AdamW moments (optimizer may then be NULL for the
 * reference defaults). The weights start at zero until mm_cuda_upload_params. */
int mm_cuda_create(const mm_model_desc* desc, int device, int trainable,
                   const mm_adamw_desc* optimizer, mm_cuda_ctx** out);
void mm_cuda_destroy(mm_cuda_ctx* ctx);
/* Copies the last error message (NUL-terminated, truncated to cap); returns its length. */
size_t mm_cuda_last_error(const mm_cuda_ctx* ctx, char* buf, size_t cap);

/* Uploads weights (and optionally moments, NULL = zero) in registry order, sets the
 * optimizer's completed-step count, refreshes every derived fp16 copy.
 * Equivalent of constructing an Execution over an existing Model/Optimizer. */
int mm_cuda_upload_params(mm_cuda_ctx* ctx, const float* params, const float* first_moment,
                          const float* second_moment, uint64_t steps);
/* Execution::synchronize_to_host (execution.hpp:58): any pointer may be NULL. */
int mm_cuda_download(mm_cuda_ctx* ctx, float* params, float* grads, float* first_moment,
                     float* second_moment, uint64_t* steps);

/* ---------------------------------------------------------------- Execution methods */

/* Execution::forward (execution.hpp:37-38): logits [batch*seq][vocab], FP32-accurate head. */
int mm_cuda_forward_logits(mm_cuda_ctx* ctx, const uint16_t* tokens, int batch, int seq,
                           float* logits);
/* Execution::log_probabilities (execution.hpp:39, inference.cpp:197-207): out [batch*seq]. */
int mm_cuda_log_probs(mm_cuda_ctx* ctx, const uint16_t* input, const uint16_t* target, int batch,
                      int seq, float* out);
/* Execution::zero_grad. */
int mm_cuda_zero_grad(mm_cuda_ctx* ctx);
/* Execution::accumulate (inference.cpp:208-222): forward, weighted NLL with the given
 * per-token coefficients, backward into the gradient accumulator. `loss` receives
 * sum(coef * nll) (may be NULL). */
int mm_cuda_accumulate(mm_cuda_ctx* ctx, const uint16_t* input, const uint16_t* target,
                       const float* coefficients, int batch, int seq, double* loss);
/* Execution::update (inference.cpp:227-232): all-reduce of the gradients when a
 * communicator is attached, then AdamW with global-norm clipping. grad_norm receives the
 * pre-clip norm. */
int mm_cuda_update(mm_cuda_ctx* ctx, float learning_rate, double* grad_norm);

/* ---------------------------------------------------------------- batched decode sessions */

/* CpuDecoder::prefill for `batch` independent prompts of equal length (the batched form of
 * Execution::prefill): fills the latent cache of rows [0, batch) and returns the
 * last-position logits [batch][vocab] (logits may be NULL). */
int mm_cuda_prefill_batch(mm_cuda_ctx* ctx, const uint16_t* prompts, int batch, int prompt_len,
                          float* logits);
/* CpuDecoder::decode for every row of the current session: appends tokens[b] at the
 * row's next position and returns logits [batch][vocab] (may be NULL). */
int mm_cuda_decode_batch(mm_cuda_ctx* ctx, const uint16_t* tokens, int batch, float* logits);

/* ---------------------------------------------------------------- serving (continuous batching) */

/* InferenceEngine::generate_tokens (inference.cpp:469-579) for many requests at once: `slots`
 * independent latent-cache rows of max_context positions, each holding one request between
 * admit and release; requests join and leave while the others keep decoding. Opening a
 * session replaces the batched decode/rollout state (and a later prefill_batch or rollout
 * replaces the session). */
int mm_cuda_serve_open(mm_cuda_ctx* ctx, int slots, int max_context);
/* Prefills `prompt` into a free slot (that slot's cache rows only) and samples the request's
 * first token, draw 0 of Rng(seed) at `temperature` (0 = greedy), into *first; logits (may be
 * NULL) receives the last prompt position's logits [vocab]. len + max_new must fit the
 * model's context and the session's. */
int mm_cuda_serve_admit(mm_cuda_ctx* ctx, int slot, const uint16_t* prompt, int len, int max_new,
                        float temperature, uint64_t seed, uint16_t* first, float* logits);
/* One decode step of every active slot (active[s] != 0): appends tokens[s] at the slot's next
 * position and samples next[s] with draw draw_index[s] of Rng(seeds[s]); logits (may be NULL)
 * receives [slots][vocab]. Inactive slots are left as they are. */
int mm_cuda_serve_step(mm_cuda_ctx* ctx, const uint16_t* tokens, const int32_t* active, float temperature,
                       const uint64_t* seeds, const int32_t* draw_index, uint16_t* next, float* logits);
/* Frees a slot for the next request. */
int mm_cuda_serve_release(mm_cuda_ctx* ctx, int slot);

/* sample_token with top_p = 1, top_k = 0, repetition penalty 1, no bans
 * (inference.cpp:345-426) on host logits [batch][vocab]: row b uses draw `draw_index[b]`
 * of Rng(seeds[b]) (temperature 0 = greedy, no draw). */
int mm_cuda_sample(mm_cuda_ctx* ctx, const float* logits, int batch, float temperature,
                   const uint64_t* seeds, const int32_t* draw_index, uint16_t* out);

/* rollout() (trainer.cpp:187-213) for n prompts at once: prefill, then sampling with
 * Rng(seeds[i]) at `temperature`, stopping a row after eos or after
 * length = min(completion_tokens, sequence + 1 - prompt_len) tokens. Outputs:
 *   out_tokens [n][completion_tokens] (entries past out_len are eos-padded),
 *   out_len [n], and when out_old_lp != NULL the completion_batch (trainer.cpp:386-408)
 *   rows and old-policy log-probabilities [n][sequence]: out_input, out_target, out_mask
 *   may then also be non-NULL. */
int mm_cuda_rollout(mm_cuda_ctx* ctx, const uint16_t* prompts, int n, int prompt_len,
                    int completion_tokens, int sequence, uint16_t eos, uint16_t pad,
                    const uint64_t* seeds, float temperature, uint16_t* out_tokens,
                    int32_t* out_len, uint16_t* out_input, uint16_t* out_target, float* out_mask,
                    float* out_old_lp);

/* ---------------------------------------------------------------- GRPO */

/* grpo_objective + group_advantages + coefficient assembly (trainer.cpp:351-385, 827-846)
 * on host arrays, on the device: lp/old/ref/mask [n][seq], rewards [n] in groups of
 * group_size. n_total is the number of rollouts in the whole update (all ranks).
 * Outputs coefficients [n][seq], advantages [n], loss and kl sums. Returns
 * MM_NUMERICAL_ERROR when a token is rejected (|lp-old| > 80, |ref-lp| > 80, non-finite). */
int mm_cuda_grpo_coefficients(mm_cuda_ctx* ctx, const float* lp, const float* old_lp,
                              const float* ref_lp, const float* mask, const float* rewards,
                              int n, int seq, int group_size, int64_t n_total, float clip,
                              float kl_coefficient, float* coefficients, float* advantages,
                              double* loss, double* kl);

/* One GRPO update (trainer.cpp:814-891 with gradient_epochs = 1) over n local rollouts:
 * advantages per group, the global skip rule, the policy forward (its log-probs are the
 * "current" ones), the frozen reference forward on `reference` (same device), the fused
 * objective/coefficients, the backward, the gradient all-reduce and AdamW at
 * learning_rate. old_lp [n][seq] are the rollout-time log-probs. n_total = rollouts over
 * all ranks. */
int mm_cuda_grpo_step(mm_cuda_ctx* policy, mm_cuda_ctx* reference, const uint16_t* input,
                      const uint16_t* target, const float* mask, const float* old_lp,
                      const float* rewards, int n, int seq, int group_size, int64_t n_total,
                      float clip, float kl_coefficient, float learning_rate,
                      mm_step_result* out);

/* One DPO update (trainer.cpp:765-783: preference_objective :107-121 and dpo_objective
 * :345-350 per pair, then Execution::step) over n local preference pairs: rows 2p (chosen)
 * and 2p + 1 (rejected) of input/target/mask [2n][seq] (completion_batch layout, mask 1 on
 * completion tokens). The frozen reference forward on `reference`, the policy forward, the
 * per-pair objective and signed coefficients (+-scale / n_total), the backward, the gradient
 * all-reduce and AdamW at learning_rate. out->loss = sum of pair losses / n_total,
 * out->kl = mean margin over the n_total pairs, out->grad_norm = pre-clip norm. margins
 * (host [n], may be NULL) receives each local pair's margin. n_total = pairs over all ranks. */
int mm_cuda_dpo_step(mm_cuda_ctx* policy, mm_cuda_ctx* reference, const uint16_t* input,
                     const uint16_t* target, const float* mask, int n, int seq, int64_t n_total,
                     float beta, float learning_rate, mm_step_result* out, double* margins);

/* ---------------------------------------------------------------- data parallel */

/* NCCL bootstrap: rank 0 creates the id (128 bytes), every rank attaches with it. The
 * communicator is formed without blocking and polled: when the other ranks have not joined
 * within MM_NCCL_INIT_TIMEOUT seconds (default 300) it is aborted and the call returns
 * MM_GPU_ERROR instead of hanging. */
int mm_cuda_nccl_unique_id(char out[128]);
int mm_cuda_init_comm(mm_cuda_ctx* ctx, int rank, int world, const char id[128]);

/* ---------------------------------------------------------------- statistics */

/* ExecutionStats (execution.hpp:24-26): kernels launched by this context so far. */
int64_t mm_cuda_kernel_launches(const mm_cuda_ctx* ctx);

#ifdef __cplusplus
}
#endif
#endif /* MM_CUDA_H */
