// CudaExecution: the reference engine's `class Execution` (include/mini_mla/execution.hpp:28-61)
// over the sm_100a backend's C ABI (include/mm_cuda.h). This is the translation unit a
// maintainer adds to the reference as src/backends/cuda_execution.cpp; `make_execution`
// (src/infer/inference.cpp:314-329) then dispatches backend "cuda" to make_cuda_execution.
// It compiles against the reference's own headers and links libmm_cuda.so; oracle/Makefile
// builds it with the reference's CPU sources for tests/test_gpu_reference_adapter.py.
//
// Ownership follows the reference (architecture.md:37): the Model owns host FP32 weights and
// gradients, the Optimizer the moments; the execution holds device copies. Device results
// reach the host on synchronize_to_host. A host edit of the weights (mark_weights_changed,
// model.hpp:56-59) is uploaded before the next device call, the way the MPS backend keys its
// device copy on Model::revision (mps_backend.mm:1063-1065).
#include "mini_mla/execution.hpp"
#include "mini_mla/model.hpp"
#include "mini_mla/optimizer.hpp"

#include "mm_cuda.h"

#include <algorithm>
#include <memory>
#include <optional>
#include <span>
#include <vector>

namespace mini_mla {

Result<std::unique_ptr<Execution>> make_cuda_execution(Model& model, Optimizer* optimizer, int device);

namespace {

Error cuda_error(mm_cuda_ctx* c, int rc) {
    char msg[1024] = {};
    if (c) mm_cuda_last_error(c, msg, sizeof msg);
    return make_error(static_cast<ErrorCode>(rc - 1), msg);  // 1 + ErrorCode across the ABI
}

std::vector<float> flat(const Model& m) {
    std::vector<float> v;
    for (const auto& p : m.parameters()) v.insert(v.end(), p.value.values.begin(), p.value.values.end());
    return v;
}

mm_model_desc desc(const ModelConfig& c) {
    return {c.vocab_size, c.max_sequence_length, c.n_layers, c.d_model, c.n_heads, c.head_dim_nope,
            c.head_dim_rope, c.head_dim_value, c.q_lora_rank, c.kv_lora_rank, c.d_ff,
            c.norm_epsilon, c.rope_theta};
}

// Weights (and, with an optimizer whose state is allocated, its moments and step count)
// from host to device.
int upload(mm_cuda_ctx* c, const Model& m, const Optimizer* o) {
    const std::vector<float> w = flat(m);
    std::vector<float> mo, vo;
    const bool moments = o && o->states().size() == m.parameters().size();
    if (moments)
        for (const auto& s : o->states()) {
            mo.insert(mo.end(), s.first.values.begin(), s.first.values.end());
            vo.insert(vo.end(), s.second.values.begin(), s.second.values.end());
        }
    return mm_cuda_upload_params(c, w.data(), moments ? mo.data() : nullptr, moments ? vo.data() : nullptr,
                                 o ? o->steps() : 0);
}

class CudaExecution final : public Execution {
  public:
    CudaExecution(Model& m, Optimizer* o, mm_cuda_ctx* c) : model_(m), opt_(o), c_(c), rev_(m.revision()) {}
    ~CudaExecution() override { mm_cuda_destroy(c_); }
    CudaExecution(const CudaExecution&) = delete;
    CudaExecution& operator=(const CudaExecution&) = delete;

    std::string device_name() const override { return "NVIDIA B200 (sm_100a)"; }
    std::string attention_name() const override { return "tcgen05 / latent decode"; }

    Result<const Matrix*> forward(std::span<const std::uint16_t> ids, int b, int t) override {
        if (auto e = refresh()) return Result<const Matrix*>::failure(*e);
        if (b < 1 || t < 1 || ids.size() != static_cast<std::size_t>(b) * static_cast<std::size_t>(t))
            return Result<const Matrix*>::failure(ErrorCode::invalid_argument, "Token count does not match shape");
        out_.resize(b * t, model_.config().vocab_size);
        if (int rc = mm_cuda_forward_logits(c_, ids.data(), b, t, out_.data()))
            return Result<const Matrix*>::failure(cuda_error(c_, rc));
        return Result<const Matrix*>::success(&out_);
    }
    Result<std::vector<float>> log_probabilities(const Batch& b) override {
        if (auto e = refresh()) return Result<std::vector<float>>::failure(*e);
        std::vector<float> lp(b.target.size());
        if (int rc = mm_cuda_log_probs(c_, b.input.data(), b.target.data(), b.batch, b.sequence, lp.data()))
            return Result<std::vector<float>>::failure(cuda_error(c_, rc));
        return Result<std::vector<float>>::success(std::move(lp));
    }
    Result<double> accumulate(const Batch& b, std::span<const float> coef) override {
        if (auto e = refresh()) return Result<double>::failure(*e);
        if (coef.size() != b.target.size())
            return Result<double>::failure(ErrorCode::invalid_argument, "Coefficient count does not match batch");
        double loss = 0;
        if (int rc = mm_cuda_accumulate(c_, b.input.data(), b.target.data(), coef.data(), b.batch, b.sequence, &loss))
            return Result<double>::failure(cuda_error(c_, rc));
        return Result<double>::success(loss);
    }
    Status zero_grad() override {
        if (auto e = refresh()) return Status::failure(*e);
        if (int rc = mm_cuda_zero_grad(c_)) return Status::failure(cuda_error(c_, rc));
        return ok();
    }
    Result<double> update(float lr) override {
        if (auto e = refresh()) return Result<double>::failure(*e);
        if (!opt_) return Result<double>::failure(ErrorCode::invalid_argument, "Inference execution has no optimizer");
        double norm = 0;
        if (int rc = mm_cuda_update(c_, lr, &norm)) return Result<double>::failure(cuda_error(c_, rc));
        opt_->set_steps(opt_->steps() + 1);
        // the device copy is now newer than the host's: flag the change without re-uploading
        model_.mark_weights_changed();
        rev_ = model_.revision();
        return Result<double>::success(norm);
    }
    Status synchronize_to_host() override {
        if (opt_ && opt_->states().size() != model_.parameters().size())
            if (auto st = opt_->initialize(model_); !st) return st;
        const std::size_t n = flat_size();
        // gradients and moments live on the device only for a training execution
        std::vector<float> w(n), g(opt_ ? n : 0), m(opt_ ? n : 0), v(opt_ ? n : 0);
        std::uint64_t steps = 0;
        if (int rc = mm_cuda_download(c_, w.data(), opt_ ? g.data() : nullptr, opt_ ? m.data() : nullptr,
                                      opt_ ? v.data() : nullptr, &steps))
            return Status::failure(cuda_error(c_, rc));
        std::size_t off = 0;
        for (std::size_t i = 0; i < model_.parameters().size(); ++i) {
            auto& p = model_.parameters()[i];
            const std::size_t k = p.value.size();
            std::copy_n(w.data() + off, k, p.value.values.begin());
            if (opt_ && p.gradient.size() == k) std::copy_n(g.data() + off, k, p.gradient.values.begin());
            if (opt_) {
                std::copy_n(m.data() + off, k, opt_->states()[i].first.values.begin());
                std::copy_n(v.data() + off, k, opt_->states()[i].second.values.begin());
            }
            off += k;
        }
        if (opt_) opt_->set_steps(steps);
        return ok();
    }
    Result<std::span<const float>> prefill(std::span<const std::uint16_t> ids) override {
        if (auto e = refresh()) return Result<std::span<const float>>::failure(*e);
        logits_.resize(static_cast<std::size_t>(model_.config().vocab_size));
        if (int rc = mm_cuda_prefill_batch(c_, ids.data(), 1, static_cast<int>(ids.size()), logits_.data()))
            return Result<std::span<const float>>::failure(cuda_error(c_, rc));
        return Result<std::span<const float>>::success(logits_);
    }
    Result<std::span<const float>> decode(std::uint16_t token) override {
        if (auto e = refresh()) return Result<std::span<const float>>::failure(*e);
        if (int rc = mm_cuda_decode_batch(c_, &token, 1, logits_.data()))
            return Result<std::span<const float>>::failure(cuda_error(c_, rc));
        return Result<std::span<const float>>::success(logits_);
    }

  private:
    std::size_t flat_size() const {
        std::size_t n = 0;
        for (const auto& p : model_.parameters()) n += p.value.size();
        return n;
    }
    // Host weights edited since the last transfer go to the device first.
    std::optional<Error> refresh() {
        if (model_.revision() == rev_) return std::nullopt;
        if (int rc = upload(c_, model_, opt_)) return cuda_error(c_, rc);
        rev_ = model_.revision();
        return std::nullopt;
    }

    Model& model_;
    Optimizer* opt_;
    mm_cuda_ctx* c_;
    std::uint64_t rev_;
    Matrix out_;
    std::vector<float> logits_;
};

} // namespace

Result<std::unique_ptr<Execution>> make_cuda_execution(Model& m, Optimizer* o, int device) {
    using R = Result<std::unique_ptr<Execution>>;
    if (o && o->config().kind != "adamw")
        return R::failure(ErrorCode::unsupported, "The cuda backend implements the AdamW optimizer only");
    mm_adamw_desc opt{0.9F, 0.95F, 1e-8F, 0.1F, 1.0F};
    if (o) opt = {o->config().beta1, o->config().beta2, o->config().epsilon, o->config().weight_decay,
                  o->config().clip_norm};
    const mm_model_desc d = desc(m.config());
    mm_cuda_ctx* c = nullptr;
    if (int rc = mm_cuda_create(&d, device, o != nullptr, &opt, &c)) {
        auto e = cuda_error(c, rc);
        mm_cuda_destroy(c);
        return R::failure(e);
    }
    if (int rc = upload(c, m, o)) {
        auto e = cuda_error(c, rc);
        mm_cuda_destroy(c);
        return R::failure(e);
    }
    return R::success(std::make_unique<CudaExecution>(m, o, c));
}

} // namespace mini_mla
