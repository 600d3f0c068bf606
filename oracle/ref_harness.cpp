// Test infrastructure, never shipped: a C ABI over the reference engine's own public
// C++ API (Model, Optimizer, make_execution("cpu"), sample_token, grpo_objective,
// group_advantages, completion_batch, cosine_learning_rate), compiled together with the
// unmodified reference CPU sources into oracle/_ref/libmini_mla_ref.so by oracle/Makefile.
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it, as the
// checker and as the timed CPU baseline.
//
// Three functions restate file-local reference code that is not reachable through a
// public symbol:
//   * ref_rollout     <- rollout()             src/train/trainer.cpp:187-213
//   * ref_grpo_update <- the GRPO update body src/train/trainer.cpp:814-847 + 848-883
//   * ref_dpo_update  <- the DPO update body  src/train/trainer.cpp:765-783 (+ :107-121)
// Both call only the reference's public API, step for step as those lines do.
#include "mini_mla/execution.hpp"
#include "mini_mla/inference.hpp"
#include "mini_mla/optimizer.hpp"
#include "mini_mla/trainer.hpp"

#include <cstdint>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

using namespace mini_mla;

#ifdef MM_REF_EXECUTION_CUDA
// Built a second time (libmini_mla_ref_cuda.so) with sessions on the sm_100a backend through
// its reference-side adapter (cpp_inference_train_engine_b200/reference_adapter), so the
// drivers below run the reference's own Execution-API sequences on the GPU.
namespace mini_mla {
Result<std::unique_ptr<Execution>> make_cuda_execution(Model&, Optimizer*, int device);
}
#endif

namespace {
thread_local std::string g_last_error;

int fail(const Error& e) {
    g_last_error = e.message;
    return 1 + static_cast<int>(e.code);
}
int fail_msg(const char* m) {
    g_last_error = m;
    return 1;
}

struct Session {
    std::unique_ptr<Model> model;
    std::unique_ptr<Optimizer> optimizer;
    std::unique_ptr<Execution> execution;
};

ModelConfig make_config(const int* c, float eps, float theta) {
    ModelConfig cfg;
    cfg.vocab_size = c[0];
    cfg.max_sequence_length = c[1];
    cfg.n_layers = c[2];
    cfg.d_model = c[3];
    cfg.n_heads = c[4];
    cfg.head_dim_nope = c[5];
    cfg.head_dim_rope = c[6];
    cfg.head_dim_value = c[7];
    cfg.q_lora_rank = c[8];
    cfg.kv_lora_rank = c[9];
    cfg.d_ff = c[10];
    cfg.norm_epsilon = eps;
    cfg.rope_theta = theta;
    return cfg;
}

Batch make_batch(const std::uint16_t* input, const std::uint16_t* target, const float* mask,
                 int batch, int seq) {
    Batch b;
    b.batch = batch;
    b.sequence = seq;
    auto n = static_cast<std::size_t>(batch) * static_cast<std::size_t>(seq);
    b.input.assign(input, input + n);
    b.target.assign(target, target + n);
    b.mask.assign(mask, mask + n);
    return b;
}
} // namespace

extern "C" {

const char* ref_last_error() { return g_last_error.c_str(); }

// cfg: vocab, max_seq, layers, d_model, heads, nope, rope, value, q_rank, kv_rank, d_ff.
// opt: beta1, beta2, epsilon, weight_decay, clip_norm (ignored when with_optimizer == 0).
void* ref_session_create(const int* cfg, float eps, float theta, std::uint64_t seed,
                         int with_optimizer, const float* opt) {
    auto made = Model::create(make_config(cfg, eps, theta), seed, with_optimizer != 0);
    if (!made) {
        fail(made.error());
        return nullptr;
    }
    auto s = new Session;
    s->model = std::move(made.value());
    if (with_optimizer) {
        OptimizerConfig oc;
        oc.beta1 = opt[0];
        oc.beta2 = opt[1];
        oc.epsilon = opt[2];
        oc.weight_decay = opt[3];
        oc.clip_norm = opt[4];
        s->optimizer = std::make_unique<Optimizer>(oc);
        auto init = s->optimizer->initialize(*s->model);
        if (!init) {
            fail(init.error());
            delete s;
            return nullptr;
        }
    }
#ifdef MM_REF_EXECUTION_CUDA
    auto e = make_cuda_execution(*s->model, s->optimizer.get(), 0);
#else
    auto e = make_execution(*s->model, s->optimizer.get(), "cpu", "fp32");
#endif
    if (!e) {
        fail(e.error());
        delete s;
        return nullptr;
    }
    s->execution = std::move(e.value());
    return s;
}

void ref_session_destroy(void* h) { delete static_cast<Session*>(h); }

std::int64_t ref_session_param_count(void* h) {
    return static_cast<std::int64_t>(static_cast<Session*>(h)->model->config().parameter_count());
}

// which: 0 weights, 1 gradients, 2 first moments, 3 second moments. Registry order.
int ref_session_read(void* h, int which, float* out) {
    auto* s = static_cast<Session*>(h);
    if (auto st = s->execution->synchronize_to_host(); !st)  // device results to the host Model
        return fail(st.error());
    std::size_t off = 0;
    for (std::size_t i = 0; i < s->model->parameters().size(); ++i) {
        const auto& p = s->model->parameters()[i];
        const Matrix* m = nullptr;
        if (which == 0)
            m = &p.value;
        else if (which == 1)
            m = &p.gradient;
        else {
            if (!s->optimizer)
                return fail_msg("session has no optimizer");
            const auto& st = s->optimizer->states()[i];
            m = which == 2 ? &st.first : &st.second;
        }
        if (m->size() != p.value.size())
            return fail_msg("tensor not allocated");
        std::memcpy(out + off, m->data(), m->size() * sizeof(float));
        off += p.value.size();
    }
    return 0;
}

int ref_session_write(void* h, int which, const float* in) {
    auto* s = static_cast<Session*>(h);
    std::size_t off = 0;
    for (std::size_t i = 0; i < s->model->parameters().size(); ++i) {
        auto& p = s->model->parameters()[i];
        Matrix* m = nullptr;
        if (which == 0)
            m = &p.value;
        else if (which == 1)
            m = &p.gradient;
        else {
            if (!s->optimizer)
                return fail_msg("session has no optimizer");
            auto& st = s->optimizer->states()[i];
            m = which == 2 ? &st.first : &st.second;
        }
        std::memcpy(m->data(), in + off, p.value.size() * sizeof(float));
        off += p.value.size();
    }
    if (which == 0)
        s->model->mark_weights_changed();
    return 0;
}

std::uint64_t ref_session_steps(void* h) {
    auto* s = static_cast<Session*>(h);
    return s->optimizer ? s->optimizer->steps() : 0;
}
void ref_session_set_steps(void* h, std::uint64_t steps) {
    auto* s = static_cast<Session*>(h);
    if (s->optimizer)
        s->optimizer->set_steps(steps);
}

// Model::forward logits [batch*seq, vocab] (src/model/model.cpp:76-155).
int ref_forward(void* h, const std::uint16_t* tokens, int batch, int seq, float* logits) {
    auto* s = static_cast<Session*>(h);
    auto n = static_cast<std::size_t>(batch) * static_cast<std::size_t>(seq);
    auto r = s->execution->forward(std::span<const std::uint16_t>(tokens, n), batch, seq);
    if (!r)
        return fail(r.error());
    std::memcpy(logits, r.value()->data(), r.value()->size() * sizeof(float));
    return 0;
}

// Execution::log_probabilities (src/infer/inference.cpp:197-207).
int ref_log_probs(void* h, const std::uint16_t* input, const std::uint16_t* target,
                  const float* mask, int batch, int seq, float* out) {
    auto* s = static_cast<Session*>(h);
    auto b = make_batch(input, target, mask, batch, seq);
    auto r = s->execution->log_probabilities(b);
    if (!r)
        return fail(r.error());
    std::memcpy(out, r.value().data(), r.value().size() * sizeof(float));
    return 0;
}

int ref_zero_grad(void* h) {
    auto st = static_cast<Session*>(h)->execution->zero_grad();
    return st ? 0 : fail(st.error());
}

// Execution::accumulate (src/infer/inference.cpp:208-222).
int ref_accumulate(void* h, const std::uint16_t* input, const std::uint16_t* target,
                   const float* mask, const float* coefficients, int batch, int seq,
                   double* loss) {
    auto* s = static_cast<Session*>(h);
    auto b = make_batch(input, target, mask, batch, seq);
    auto r = s->execution->accumulate(
        b, std::span<const float>(coefficients, b.target.size()));
    if (!r)
        return fail(r.error());
    *loss = r.value();
    return 0;
}

// Execution::update -> Optimizer::step (src/train/optimizer.cpp:105-161). Returns the
// pre-clip global gradient norm.
int ref_update(void* h, float lr, double* norm) {
    auto r = static_cast<Session*>(h)->execution->update(lr);
    if (!r)
        return fail(r.error());
    *norm = r.value();
    return 0;
}

// CpuDecoder::prefill / decode through the Execution interface
// (src/infer/inference.cpp:47-174).
int ref_prefill(void* h, const std::uint16_t* ids, int n, float* logits) {
    auto* s = static_cast<Session*>(h);
    auto r = s->execution->prefill(std::span<const std::uint16_t>(ids, static_cast<std::size_t>(n)));
    if (!r)
        return fail(r.error());
    std::memcpy(logits, r.value().data(), r.value().size() * sizeof(float));
    return 0;
}
int ref_decode(void* h, std::uint16_t token, float* logits) {
    auto r = static_cast<Session*>(h)->execution->decode(token);
    if (!r)
        return fail(r.error());
    std::memcpy(logits, r.value().data(), r.value().size() * sizeof(float));
    return 0;
}

// sample_token (src/infer/inference.cpp:345-426). rng_state is the Rng state before the
// call and receives the state after it.
int ref_sample_token(const float* logits, int n, const std::uint16_t* history, int n_history,
                     float temperature, float top_p, int top_k, float repetition_penalty,
                     const std::uint16_t* banned, int n_banned, std::uint64_t* rng_state,
                     std::uint16_t* out) {
    GenerationConfig c;
    c.temperature = temperature;
    c.top_p = top_p;
    c.top_k = top_k;
    c.repetition_penalty = repetition_penalty;
    Rng rng(0);
    rng.restore(*rng_state);
    auto r = sample_token(
        std::span<const float>(logits, static_cast<std::size_t>(n)),
        std::span<const std::uint16_t>(history, static_cast<std::size_t>(n_history)), c, rng,
        std::span<const std::uint16_t>(banned, static_cast<std::size_t>(n_banned)));
    *rng_state = rng.state();
    if (!r)
        return fail(r.error());
    *out = r.value();
    return 0;
}

// grpo_objective (src/train/trainer.cpp:351-370).
int ref_grpo_objective(float lp, float old, float ref, float advantage, float clip, float klc,
                       double* loss, double* kl, float* coefficient) {
    auto r = grpo_objective(lp, old, ref, advantage, clip, klc);
    if (!r)
        return fail(r.error());
    *loss = r.value().loss;
    *kl = r.value().kl;
    *coefficient = r.value().nll_coefficient;
    return 0;
}

// group_advantages (src/train/trainer.cpp:371-385).
int ref_group_advantages(const float* rewards, int n, float eps, float* out) {
    auto r = group_advantages(std::span<const float>(rewards, static_cast<std::size_t>(n)), eps);
    if (!r)
        return fail(r.error());
    std::memcpy(out, r.value().data(), r.value().size() * sizeof(float));
    return 0;
}

// completion_batch (src/train/trainer.cpp:386-408).
int ref_completion_batch(const std::uint16_t* prompt, int np, const std::uint16_t* response,
                         int nr, int seq, std::uint16_t pad, std::uint16_t* input,
                         std::uint16_t* target, float* mask) {
    auto r = completion_batch(std::span<const std::uint16_t>(prompt, static_cast<std::size_t>(np)),
                              std::span<const std::uint16_t>(response, static_cast<std::size_t>(nr)),
                              seq, pad);
    if (!r)
        return fail(r.error());
    std::memcpy(input, r.value().input.data(), r.value().input.size() * 2);
    std::memcpy(target, r.value().target.data(), r.value().target.size() * 2);
    std::memcpy(mask, r.value().mask.data(), r.value().mask.size() * 4);
    return 0;
}

// cosine_learning_rate (src/train/optimizer.cpp:162-173).
float ref_cosine_lr(std::uint64_t done, std::uint64_t total, std::uint64_t warmup, float peak,
                    float minimum) {
    return cosine_learning_rate(done, total, warmup, peak, minimum);
}

// Rng (include/mini_mla/rng.hpp:7-35): one call per draw kind, state in/out.
std::uint64_t ref_rng_next(std::uint64_t* state) {
    Rng r(*state);
    auto v = r.next();
    *state = r.state();
    return v;
}
float ref_rng_uniform(std::uint64_t* state) {
    Rng r(*state);
    auto v = r.uniform();
    *state = r.state();
    return v;
}
std::uint64_t ref_rng_bounded(std::uint64_t* state, std::uint64_t bound) {
    Rng r(*state);
    auto v = r.bounded(bound);
    *state = r.state();
    return v;
}
float ref_rng_normal(std::uint64_t* state) {
    Rng r(*state);
    auto v = r.normal();
    *state = r.state();
    return v;
}

// rollout() restated from src/train/trainer.cpp:187-213 over the public API: prefill,
// then temperature-1 / top-p-1 sampling with Rng(seed), stopping after eos or `length`
// tokens, decoding every sampled token but the last; then completion_batch and the
// old-policy log-probabilities. out_tokens holds up to completion_tokens ids,
// out_input/out_target/out_mask/out_old_lp hold `sequence` entries each.
int ref_rollout(void* h, const std::uint16_t* prompt, int prompt_len, int completion_tokens,
                int sequence, std::uint16_t eos, std::uint16_t pad, std::uint64_t seed,
                float temperature, std::uint16_t* out_tokens, int* out_len,
                std::uint16_t* out_input, std::uint16_t* out_target, float* out_mask,
                float* out_old_lp) {
    auto* s = static_cast<Session*>(h);
    auto& e = *s->execution;
    std::span<const std::uint16_t> p(prompt, static_cast<std::size_t>(prompt_len));
    auto logits = e.prefill(p);
    if (!logits)
        return fail(logits.error());
    std::vector<float> current(logits.value().begin(), logits.value().end());
    std::vector<std::uint16_t> response, history(p.begin(), p.end());
    Rng rng(seed);
    GenerationConfig gc;
    gc.temperature = temperature;
    gc.top_p = 1;
    gc.max_new_tokens = completion_tokens;
    int length = std::min(completion_tokens, sequence + 1 - prompt_len);
    if (length < 1)
        return fail_msg("GRPO prompt leaves no room for a response");
    for (int i = 0; i < length; ++i) {
        auto token = sample_token(current, history, gc, rng);
        if (!token)
            return fail(token.error());
        response.push_back(token.value());
        history.push_back(token.value());
        if (token.value() == eos)
            break;
        if (i + 1 < length) {
            auto next = e.decode(token.value());
            if (!next)
                return fail(next.error());
            current.assign(next.value().begin(), next.value().end());
        }
    }
    auto b = completion_batch(p, response, sequence, pad);
    if (!b)
        return fail(b.error());
    auto old = e.log_probabilities(b.value());
    if (!old)
        return fail(old.error());
    std::memcpy(out_tokens, response.data(), response.size() * 2);
    *out_len = static_cast<int>(response.size());
    std::memcpy(out_input, b.value().input.data(), b.value().input.size() * 2);
    std::memcpy(out_target, b.value().target.data(), b.value().target.size() * 2);
    std::memcpy(out_mask, b.value().mask.data(), b.value().mask.size() * 4);
    std::memcpy(out_old_lp, old.value().data(), old.value().size() * 4);
    return 0;
}

// The GRPO update restated from src/train/trainer.cpp:814-847 (advantages per group,
// skip when all are zero, per-token coefficients over the whole update) and :848-883
// (Execution::step with the cosine learning rate supplied by the caller).
// Rollout i occupies rows [i*sequence, (i+1)*sequence) of the flat arrays; groups are
// consecutive runs of group_size rollouts. Outputs: loss and kl (the host objective
// sums), grad_norm (pre-clip), skipped (1 when every advantage is zero), and the
// advantages and per-token coefficients that were used.
int ref_grpo_update(void* policy, void* reference, int n_rollouts, int group_size, int sequence,
                    const std::uint16_t* input, const std::uint16_t* target, const float* mask,
                    const float* old_lp, const float* rewards, float clip, float klc, float lr,
                    double* loss, double* kl, double* grad_norm, int* skipped,
                    float* out_advantages, float* out_coefficients) {
    auto* ps = static_cast<Session*>(policy);
    auto* rs = static_cast<Session*>(reference);
    if (n_rollouts < 1 || group_size < 2 || n_rollouts % group_size)
        return fail_msg("rollouts must form whole groups");
    auto S = static_cast<std::size_t>(sequence);
    std::vector<Batch> batches;
    for (int i = 0; i < n_rollouts; ++i)
        batches.push_back(make_batch(input + i * S, target + i * S, mask + i * S, 1, sequence));
    std::vector<float> advantages;
    for (int g = 0; g < n_rollouts / group_size; ++g) {
        auto a = group_advantages(std::span<const float>(rewards + g * group_size,
                                                         static_cast<std::size_t>(group_size)));
        if (!a)
            return fail(a.error());
        advantages.insert(advantages.end(), a.value().begin(), a.value().end());
    }
    std::memcpy(out_advantages, advantages.data(), advantages.size() * 4);
    *loss = 0;
    *kl = 0;
    *grad_norm = 0;
    *skipped = 0;
    if (std::all_of(advantages.begin(), advantages.end(), [](float a) { return a == 0; })) {
        *skipped = 1;
        return 0;
    }
    auto z = ps->execution->zero_grad();
    if (!z)
        return fail(z.error());
    std::vector<std::vector<float>> coefficients;
    for (std::size_t i = 0; i < batches.size(); ++i) {
        auto current = ps->execution->log_probabilities(batches[i]);
        if (!current)
            return fail(current.error());
        auto ref = rs->execution->log_probabilities(batches[i]);
        if (!ref)
            return fail(ref.error());
        auto c = batches[i].mask;
        double denominator =
            static_cast<double>(batches.size() * batches[i].supervised_tokens());
        for (std::size_t t = 0; t < c.size(); ++t) {
            if (c[t] == 0)
                continue;
            auto objective = grpo_objective(current.value()[t], old_lp[i * S + t], ref.value()[t],
                                            advantages[i], clip, klc);
            if (!objective)
                return fail(objective.error());
            *loss += objective.value().loss / denominator;
            *kl += objective.value().kl / denominator;
            c[t] = static_cast<float>(objective.value().nll_coefficient / denominator);
        }
        coefficients.push_back(std::move(c));
    }
    for (std::size_t i = 0; i < coefficients.size(); ++i)
        std::memcpy(out_coefficients + i * S, coefficients[i].data(), S * 4);
    std::vector<GradientBatch> jobs;
    for (std::size_t i = 0; i < batches.size(); ++i)
        jobs.push_back({&batches[i], coefficients[i]});
    auto r = ps->execution->step(jobs, lr);
    if (!r)
        return fail(r.error());
    *grad_norm = r.value().gradient_norm;
    return 0;
}

// dpo_objective (src/train/trainer.cpp:345-350).
int ref_dpo_objective(double chosen, double rejected, double ref_chosen, double ref_rejected, float beta,
                      double* loss, double* margin, float* chosen_coef, float* rejected_coef) {
    auto o = dpo_objective(chosen, rejected, ref_chosen, ref_rejected, beta);
    *loss = o.loss;
    *margin = o.margin;
    *chosen_coef = o.chosen_nll_coefficient;
    *rejected_coef = o.rejected_nll_coefficient;
    return 0;
}

// The DPO update body restated from src/train/trainer.cpp:765-783 over the public API:
// per pair preference_objective (:107-121: both executions' log-probabilities, masked sums in
// double, dpo_objective), loss += objective.loss / pairs, coefficients = mask * (+-scale) /
// pairs; then Execution::step (:848-883). Pair p is rows 2p (chosen) and 2p + 1 (rejected)
// of the flat [2 n_pairs][sequence] arrays. margins receives each pair's margin.
int ref_dpo_update(void* policy, void* reference, int n_pairs, int sequence, const std::uint16_t* input,
                   const std::uint16_t* target, const float* mask, float beta, float lr, double* loss,
                   double* grad_norm, double* margins) {
    auto* ps = static_cast<Session*>(policy);
    auto* rs = static_cast<Session*>(reference);
    if (n_pairs < 1)
        return fail_msg("no preference pairs");
    auto S = static_cast<std::size_t>(sequence);
    std::vector<Batch> batches;
    std::vector<std::vector<float>> coefficients;
    *loss = 0;
    for (int p = 0; p < n_pairs; ++p) {
        const std::size_t off = 2 * static_cast<std::size_t>(p) * S;
        auto b = make_batch(input + off, target + off, mask + off, 2, sequence);
        auto pl = ps->execution->log_probabilities(b);
        if (!pl)
            return fail(pl.error());
        auto rl = rs->execution->log_probabilities(b);
        if (!rl)
            return fail(rl.error());
        double chosen = 0, rejected = 0, ref_chosen = 0, ref_rejected = 0;
        for (std::size_t t = 0; t < b.target.size(); ++t)
            if (b.mask[t] != 0) {
                if (t < S) {
                    chosen += pl.value()[t];
                    ref_chosen += rl.value()[t];
                } else {
                    rejected += pl.value()[t];
                    ref_rejected += rl.value()[t];
                }
            }
        auto objective = dpo_objective(chosen, rejected, ref_chosen, ref_rejected, beta);
        *loss += objective.loss / n_pairs;
        margins[p] = objective.margin;
        auto c = b.mask;
        for (std::size_t t = 0; t < c.size(); ++t)
            c[t] *= (t < S ? objective.chosen_nll_coefficient : objective.rejected_nll_coefficient) /
                    static_cast<float>(n_pairs);
        batches.push_back(std::move(b));
        coefficients.push_back(std::move(c));
    }
    std::vector<GradientBatch> jobs;
    for (std::size_t i = 0; i < batches.size(); ++i)
        jobs.push_back({&batches[i], coefficients[i]});
    auto r = ps->execution->step(jobs, lr);
    if (!r)
        return fail(r.error());
    *grad_norm = r.value().gradient_norm;
    return 0;
}

} // extern "C"
