// C ABI of the sm_100a backend (include/mm_cuda.h, include/mm_cuda_kernels.h). Every
// entry point validates its arguments, runs on the context's stream, waits for completion
// and maps failures to 1 + ErrorCode with a message, as the reference's Result does.
#include <mutex>
#include <new>

#include "train.cuh"

#include "../../include/mm_cuda_kernels.h"

struct mm_cuda_ctx {
    mm::Context cx;
};

namespace {

template <class F> int guarded(mm_cuda_ctx* h, F&& f) {
    if (!h) return MM_INVALID_ARGUMENT;
    try {
        if (h->cx.unusable) mm::fail(MM_GPU_ERROR, "Execution is unusable after a device failure");
        MM_CUDA_CHECK(cudaSetDevice(h->cx.device));
        f(h->cx);
        return MM_OK;
    } catch (const mm::Failure& e) {
        h->cx.last_error = e.what();
        return e.code;
    } catch (const std::bad_alloc&) {
        h->cx.last_error = "host allocation failed";
        return MM_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        h->cx.last_error = e.what();
        return MM_INVALID_ARGUMENT;
    }
}

mm::Dims checked_dims(const mm_model_desc* d) {
    if (!d) mm::fail(MM_INVALID_ARGUMENT, "null model description");
    mm::Dims c = mm::dims_from(*d);
    const int v[] = {c.V, c.maxS, c.L, c.d, c.H, c.nope, c.rope, c.dv, c.qr, c.kvr, c.dff};
    for (int x : v)
        if (x < 1 || x > 65535) mm::fail(MM_INVALID_ARGUMENT, "model dimensions must be in [1, 65535]");
    return c;
}

// Rng of include/mini_mla/rng.hpp:7-35 (splitmix64; float uniform; Box-Muller normal).
struct HostRng {
    uint64_t s;
    uint64_t next() {
        uint64_t z = (s += 0x9e3779b97f4a7c15ULL);
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
        return z ^ (z >> 31);
    }
    float uniform() { return (static_cast<float>(next() >> 40) + 0.5F) / 16777216.0F; }
    float normal() {
        const float u1 = uniform();  // first draw feeds the logarithm, as the reference build does
        const float u2 = uniform();
        return std::sqrt(-2.0F * std::log(u1)) * std::cos(2.0F * 3.14159265358979323846F * u2);
    }
};

void check_tokens(const mm::Context& cx, const uint16_t* t, long long n) {
    for (long long i = 0; i < n; ++i)
        if (t[i] >= cx.c.V) mm::fail(MM_INVALID_ARGUMENT, "Input token exceeds vocabulary");
}

// Scratch of mm_decode_attention_noalloc: partials (max, sum, 128-wide context) of 8 heads
// for up to 256 (row, split) pairs, in a static device array instead of an allocation.
// In host code the symbol is only a handle; the kernel gets the device address resolved by
// cudaGetSymbolAddress once per device, with that device current.
constexpr int kStaticPartialSlots = 256;
__device__ __align__(256) float g_static_partials[kStaticPartialSlots * mm::dec::H * (mm::dec::KV + 2)];
constexpr int kMaxDevices = 64;
float* g_static_partials_addr[kMaxDevices] = {};
std::mutex g_static_partials_mu;

float* static_partials_address() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_static_partials_mu);
    if (!g_static_partials_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_static_partials) != cudaSuccess || !p) return nullptr;
        g_static_partials_addr[dev] = static_cast<float*>(p);
    }
    return g_static_partials_addr[dev];
}

} // namespace

extern "C" {

int64_t mm_model_parameter_count(const mm_model_desc* desc) {
    try {
        return mm::parameter_count(checked_dims(desc));
    } catch (...) {
        return -1;
    }
}

int mm_model_init_params(const mm_model_desc* desc, uint64_t seed, float* out) {
    try {
        const mm::Dims c = checked_dims(desc);
        if (!out) return MM_INVALID_ARGUMENT;
        HostRng rng{seed};
        auto reg = mm::registry(c);
        long long off = 0;
        for (size_t i = 0; i < reg.size(); ++i) {
            auto [rows, cols, role] = reg[i];
            // w_o and w_down (registry slots 8 and 12 of a layer) carry the residual scale.
            bool residual = false;
            if (i >= 2) {
                const int slot = static_cast<int>((i - 2) % mm::kLayerParams);
                residual = slot == mm::kWo || slot == mm::kWdown;
            }
            const float scale = residual ? 0.02F / std::sqrt(static_cast<float>(2 * c.L)) : 0.02F;
            for (long long j = 0; j < static_cast<long long>(rows) * cols; ++j)
                out[off + j] = role == 2 ? 1.0F : rng.normal() * scale;
            off += static_cast<long long>(rows) * cols;
        }
        return MM_OK;
    } catch (const mm::Failure& e) {
        return e.code;
    }
}

float mm_cosine_learning_rate(uint64_t done, uint64_t total, uint64_t warmup, float peak, float minimum) {
    if (warmup && done < warmup) return peak * static_cast<float>(done + 1) / static_cast<float>(warmup);
    if (total <= warmup) return peak;
    double t = static_cast<double>(done - std::min(done, warmup)) / static_cast<double>(total - warmup);
    t = std::min(std::max(t, 0.0), 1.0);
    return peak * static_cast<float>(minimum + (1 - minimum) * 0.5 * (1 + std::cos(3.14159265358979323846 * t)));
}

int mm_cuda_create(const mm_model_desc* desc, int device, int trainable, const mm_adamw_desc* optimizer,
                   mm_cuda_ctx** out) {
    if (!desc || !out) return MM_INVALID_ARGUMENT;
    *out = nullptr;
    auto* h = new (std::nothrow) mm_cuda_ctx;
    if (!h) return MM_OUT_OF_MEMORY;
    int rc = guarded(h, [&](mm::Context& cx) { mm::create_context(cx, *desc, device, trainable != 0, optimizer); });
    *out = h;  // returned even on failure so the caller can read the message
    return rc;
}

void mm_cuda_destroy(mm_cuda_ctx* h) {
    if (!h) return;
    cudaSetDevice(h->cx.device);
    if (h->cx.stream) cudaStreamSynchronize(h->cx.stream);
    if (h->cx.nccl_comm) {
        try {
            ncclComm_t comm = static_cast<ncclComm_t>(h->cx.nccl_comm);
            const ncclResult_t r = mm::nccl().commDestroy(comm);
            if (r == ncclInProgress && h->cx.nccl_nonblocking) mm::nccl_settle(comm, 30.0, "ncclCommDestroy");
        } catch (...) {
        }
    }
    if (h->cx.ev0) cudaEventDestroy(h->cx.ev0);
    if (h->cx.ev1) cudaEventDestroy(h->cx.ev1);
    cudaStream_t s = h->cx.stream;
    delete h;
    if (s) cudaStreamDestroy(s);
}

size_t mm_cuda_last_error(const mm_cuda_ctx* h, char* buf, size_t cap) {
    if (!h) return 0;
    const std::string& m = h->cx.last_error;
    if (buf && cap) {
        const size_t n = std::min(cap - 1, m.size());
        std::memcpy(buf, m.data(), n);
        buf[n] = 0;
    }
    return m.size();
}

int mm_cuda_upload_params(mm_cuda_ctx* h, const float* params, const float* m, const float* v, uint64_t steps) {
    return guarded(h, [&](mm::Context& cx) {
        if (!params) mm::fail(MM_INVALID_ARGUMENT, "null parameters");
        mm::upload_params(cx, params, m, v, steps);
    });
}

int mm_cuda_download(mm_cuda_ctx* h, float* params, float* grads, float* m, float* v, uint64_t* steps) {
    return guarded(h, [&](mm::Context& cx) {
        mm::download(cx, params, grads, m, v);
        if (steps) *steps = cx.steps;
    });
}

int mm_cuda_forward_logits(mm_cuda_ctx* h, const uint16_t* tokens, int batch, int seq, float* logits) {
    return guarded(h, [&](mm::Context& cx) {
        if (!tokens || !logits || batch < 1 || seq < 1 || seq > cx.c.maxS)
            mm::fail(MM_INVALID_ARGUMENT, "Input batch or sequence shape is invalid");
        check_tokens(cx, tokens, static_cast<long long>(batch) * seq);
        const int per = std::max(1, mm::chunk_tokens(cx) / seq);
        mm::ensure_workspace(cx, std::min(batch, per) * seq, false);
        for (int r0 = 0; r0 < batch; r0 += per) {
            const int bc = std::min(per, batch - r0);
            const long long T = static_cast<long long>(bc) * seq;
            MM_CUDA_CHECK(cudaMemcpyAsync(cx.ws.tokens, tokens + static_cast<long long>(r0) * seq, T * 2,
                                          cudaMemcpyHostToDevice, cx.stream));
            mm::forward_chunk(cx, bc, seq, false, mm::kVocabAll, false, nullptr, 0, 0, nullptr);
            MM_CUDA_CHECK(cudaMemcpyAsync(logits + static_cast<long long>(r0) * seq * cx.c.V, cx.ws.logits,
                                          T * cx.c.V * 4, cudaMemcpyDeviceToHost, cx.stream));
        }
        mm::check_device(cx, "forward");
    });
}

int mm_cuda_log_probs(mm_cuda_ctx* h, const uint16_t* input, const uint16_t* target, int batch, int seq, float* out) {
    return guarded(h, [&](mm::Context& cx) {
        if (!input || !target || !out || batch < 1 || seq < 1 || seq > cx.c.maxS)
            mm::fail(MM_INVALID_ARGUMENT, "Input batch or sequence shape is invalid");
        check_tokens(cx, input, static_cast<long long>(batch) * seq);
        check_tokens(cx, target, static_cast<long long>(batch) * seq);
        mm::log_probs_host(cx, input, target, batch, seq, out);
    });
}

int mm_cuda_zero_grad(mm_cuda_ctx* h) {
    return guarded(h, [&](mm::Context& cx) {
        if (!cx.trainable) mm::fail(MM_INVALID_ARGUMENT, "Inference execution has no optimizer");
        MM_CUDA_CHECK(cudaMemsetAsync(cx.g, 0, sizeof(float) * cx.P_dev, cx.stream));
        MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
    });
}

int mm_cuda_accumulate(mm_cuda_ctx* h, const uint16_t* input, const uint16_t* target, const float* coef, int batch,
                       int seq, double* loss) {
    return guarded(h, [&](mm::Context& cx) {
        if (!cx.trainable) mm::fail(MM_INVALID_ARGUMENT, "Inference execution has no optimizer");
        if (!input || !target || !coef || batch < 1 || seq < 1 || seq > cx.c.maxS)
            mm::fail(MM_INVALID_ARGUMENT, "Input batch or sequence shape is invalid");
        const long long N = static_cast<long long>(batch) * seq;
        check_tokens(cx, input, N);
        check_tokens(cx, target, N);
        for (long long i = 0; i < N; ++i)
            if (!std::isfinite(coef[i])) mm::fail(MM_INVALID_ARGUMENT, "Invalid target or loss coefficient");
        const int per = std::max(1, mm::chunk_tokens(cx) / seq);
        mm::ensure_workspace(cx, std::min(batch, per) * seq, true);
        mm::Workspace& w = cx.ws;
        double total = 0;
        std::vector<float> lp;
        for (int r0 = 0; r0 < batch; r0 += per) {
            const int bc = std::min(per, batch - r0);
            const long long T = static_cast<long long>(bc) * seq, off = static_cast<long long>(r0) * seq;
            MM_CUDA_CHECK(cudaMemcpyAsync(w.tokens, input + off, T * 2, cudaMemcpyHostToDevice, cx.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(w.targets, target + off, T * 2, cudaMemcpyHostToDevice, cx.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(w.coef, coef + off, T * 4, cudaMemcpyHostToDevice, cx.stream));
            mm::forward_chunk(cx, bc, seq, true, mm::kVocabAll, true, nullptr, 0, 0, nullptr);
            lp.resize(static_cast<size_t>(T));
            MM_CUDA_CHECK(cudaMemcpyAsync(lp.data(), w.lp, T * 4, cudaMemcpyDeviceToHost, cx.stream));
            MM_CUDA_CHECK(cudaMemsetAsync(&cx.d_sums->max_coef_bits, 0, 4, cx.stream));
            MM_LAUNCH(mm::absmax_kernel, std::min<unsigned>(mm::blocks_for(T, 1024), mm::sm_count() * 4), 256, 0, w.coef, T,
                      &cx.d_sums->max_coef_bits);
            MM_LAUNCH(mm::grad_scale_kernel, 1, 1, 0, cx.d_sums, cx.d_scale);
            mm::backward_chunk(cx, bc, seq);
            MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
            for (long long i = 0; i < T; ++i) total += static_cast<double>(coef[off + i]) * -static_cast<double>(lp[i]);
        }
        mm::check_device(cx, "accumulate");
        if (!std::isfinite(total)) mm::fail(MM_NUMERICAL_ERROR, "Nonfinite logits or loss");
        if (loss) *loss = total;
    });
}

int mm_cuda_update(mm_cuda_ctx* h, float lr, double* grad_norm) {
    return guarded(h, [&](mm::Context& cx) {
        const double n = mm::adamw_update(cx, lr);
        if (grad_norm) *grad_norm = n;
    });
}

int mm_cuda_prefill_batch(mm_cuda_ctx* h, const uint16_t* prompts, int batch, int prompt_len, float* logits) {
    return guarded(h, [&](mm::Context& cx) {
        if (!prompts || batch < 1 || prompt_len < 1 || prompt_len > cx.c.maxS)
            mm::fail(MM_INVALID_ARGUMENT, "Prompt exceeds context or is empty");
        check_tokens(cx, prompts, static_cast<long long>(batch) * prompt_len);
        mm::ensure_decode(cx, batch, cx.c.maxS, 1);
        cx.serving = false;  // the decode state now holds this batch
        uint16_t* d = static_cast<uint16_t*>(cx.stage.get(static_cast<size_t>(batch) * prompt_len * 2));
        MM_CUDA_CHECK(cudaMemcpyAsync(d, prompts, static_cast<size_t>(batch) * prompt_len * 2, cudaMemcpyHostToDevice, cx.stream));
        mm::prefill_rows(cx, d, batch, prompt_len, mm::chunk_tokens(cx));
        if (logits)
            MM_CUDA_CHECK(cudaMemcpyAsync(logits, cx.dec.logits, sizeof(float) * batch * cx.c.V, cudaMemcpyDeviceToHost, cx.stream));
        cx.dec_len = prompt_len;
        mm::check_device(cx, "prefill");
    });
}

int mm_cuda_decode_batch(mm_cuda_ctx* h, const uint16_t* tokens, int batch, float* logits) {
    return guarded(h, [&](mm::Context& cx) {
        if (!tokens || batch != cx.dec.B || cx.dec_len < 1)
            mm::fail(MM_INVALID_ARGUMENT, "Decode requires current-weight prefill, available context, and a valid token");
        if (cx.dec_len >= cx.c.maxS) mm::fail(MM_INVALID_ARGUMENT, "Decode requires available context");
        check_tokens(cx, tokens, batch);
        MM_CUDA_CHECK(cudaMemcpyAsync(cx.dec.tok, tokens, static_cast<size_t>(batch) * 2, cudaMemcpyHostToDevice, cx.stream));
        mm::decode_step(cx);
        if (logits)
            MM_CUDA_CHECK(cudaMemcpyAsync(logits, cx.dec.logits, sizeof(float) * batch * cx.c.V, cudaMemcpyDeviceToHost, cx.stream));
        cx.dec_len += 1;
        mm::check_device(cx, "decode");
    });
}

int mm_cuda_serve_open(mm_cuda_ctx* h, int slots, int max_context) {
    return guarded(h, [&](mm::Context& cx) {
        if (slots < 1 || max_context < 2 || max_context > cx.c.maxS)
            mm::fail(MM_INVALID_ARGUMENT, "Invalid serving slots or context");
        mm::ensure_decode(cx, slots, max_context, 1);
        MM_CUDA_CHECK(cudaMemsetAsync(cx.dec.pos, 0, sizeof(int) * slots, cx.stream));
        cx.serve_pos.assign(static_cast<size_t>(slots), -1);
        cx.serving = true;
        cx.dec_len = 1;
        mm::check_device(cx, "serve_open");
    });
}

int mm_cuda_serve_admit(mm_cuda_ctx* h, int slot, const uint16_t* prompt, int len, int max_new, float temperature,
                        uint64_t seed, uint16_t* first, float* logits) {
    return guarded(h, [&](mm::Context& cx) {
        mm::DecodeState& d = cx.dec;
        if (!cx.serving) mm::fail(MM_INVALID_ARGUMENT, "No serving session");
        if (slot < 0 || slot >= d.B || cx.serve_pos[slot] >= 0) mm::fail(MM_INVALID_ARGUMENT, "Slot is not free");
        if (!prompt || !first || len < 1 || max_new < 1 || len + max_new > cx.c.maxS || len + max_new - 1 > d.Sc)
            mm::fail(MM_INVALID_ARGUMENT, "Prompt plus requested tokens exceeds context");
        if (!std::isfinite(temperature) || temperature < 0) mm::fail(MM_INVALID_ARGUMENT, "Invalid generation settings");
        check_tokens(cx, prompt, len);
        char* base = static_cast<char*>(cx.stage.get(mm::round_up(len * 2LL, 256) + 256));
        uint16_t* d_prompt = reinterpret_cast<uint16_t*>(base);
        uint64_t* d_seed = reinterpret_cast<uint64_t*>(base + mm::round_up(len * 2LL, 256));
        int* d_draw = reinterpret_cast<int*>(d_seed + 1);
        int* d_len = d_draw + 1;
        uint16_t* d_first = reinterpret_cast<uint16_t*>(d_len + 1);
        const int zero = 0;
        MM_CUDA_CHECK(cudaMemcpyAsync(d_prompt, prompt, len * 2LL, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(d_seed, &seed, 8, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(d_draw, &zero, 4, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(d_len, &len, 4, cudaMemcpyHostToDevice, cx.stream));
        // the prompt's cache rows of this slot only, and its last-position logits
        mm::ensure_workspace(cx, len, cx.ws.tape);
        MM_CUDA_CHECK(cudaMemcpyAsync(cx.ws.tokens, d_prompt, len * 2LL, cudaMemcpyDeviceToDevice, cx.stream));
        float* row_logits = d.logits + static_cast<long long>(slot) * cx.c.V;
        mm::forward_chunk(cx, 1, len, false, mm::kVocabLast, false, d.cache, d.Sc, slot, row_logits);
        MM_CUDA_CHECK(cudaMemcpyAsync(d.pos + slot, d_len, 4, cudaMemcpyDeviceToDevice, cx.stream));
        // first token: draw 0 of Rng(seed) (generate_tokens, inference.cpp:469-579)
        mm::launch_sample(cx, row_logits, 1, temperature, d_seed, d_draw, 0, nullptr, d_first, 1);
        MM_CUDA_CHECK(cudaMemcpyAsync(first, d_first, 2, cudaMemcpyDeviceToHost, cx.stream));
        if (logits)
            MM_CUDA_CHECK(cudaMemcpyAsync(logits, row_logits, sizeof(float) * cx.c.V, cudaMemcpyDeviceToHost, cx.stream));
        mm::check_device(cx, "serve_admit");
        cx.serve_pos[slot] = len;
    });
}

int mm_cuda_serve_step(mm_cuda_ctx* h, const uint16_t* tokens, const int32_t* active, float temperature,
                       const uint64_t* seeds, const int32_t* draw_index, uint16_t* next, float* logits) {
    return guarded(h, [&](mm::Context& cx) {
        mm::DecodeState& d = cx.dec;
        if (!cx.serving) mm::fail(MM_INVALID_ARGUMENT, "No serving session");
        if (!tokens || !active || !seeds || !draw_index || !next) mm::fail(MM_INVALID_ARGUMENT, "null serving buffer");
        if (!std::isfinite(temperature) || temperature < 0) mm::fail(MM_INVALID_ARGUMENT, "Invalid generation settings");
        const int B = d.B;
        int longest = 1;
        for (int b = 0; b < B; ++b) {
            if (!active[b]) continue;
            if (cx.serve_pos[b] < 1) mm::fail(MM_INVALID_ARGUMENT, "Active slot holds no request");
            if (cx.serve_pos[b] >= d.Sc || cx.serve_pos[b] >= cx.c.maxS)
                mm::fail(MM_INVALID_ARGUMENT, "Decode requires available context");
            if (tokens[b] >= cx.c.V) mm::fail(MM_INVALID_ARGUMENT, "Input token exceeds vocabulary");
            longest = std::max(longest, cx.serve_pos[b] + 1);
        }
        std::vector<int> act(static_cast<size_t>(B));
        for (int b = 0; b < B; ++b) act[b] = active[b] ? 1 : 0;
        MM_CUDA_CHECK(cudaMemcpyAsync(d.tok, tokens, sizeof(uint16_t) * B, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(d.active, act.data(), sizeof(int) * B, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(d.seeds, seeds, sizeof(uint64_t) * B, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(d.draw, draw_index, sizeof(int) * B, cudaMemcpyHostToDevice, cx.stream));
        MM_LAUNCH(mm::serve_prepare_kernel, mm::blocks_for(B, 256), 256, 0, d.pos, d.tok, d.active, B);
        cx.dec_len = longest - 1;  // cache entries before this step's write (the split heuristic)
        mm::decode_step(cx);
        mm::launch_sample(cx, d.logits, B, temperature, d.seeds, d.draw, 0, d.active, d.out_tok, 1);
        MM_CUDA_CHECK(cudaMemcpyAsync(next, d.out_tok, sizeof(uint16_t) * B, cudaMemcpyDeviceToHost, cx.stream));
        if (logits)
            MM_CUDA_CHECK(cudaMemcpyAsync(logits, d.logits, sizeof(float) * B * cx.c.V, cudaMemcpyDeviceToHost, cx.stream));
        mm::check_device(cx, "serve_step");
        for (int b = 0; b < B; ++b)
            if (act[b]) cx.serve_pos[b] += 1;
    });
}

int mm_cuda_serve_release(mm_cuda_ctx* h, int slot) {
    return guarded(h, [&](mm::Context& cx) {
        if (!cx.serving || slot < 0 || slot >= cx.dec.B) mm::fail(MM_INVALID_ARGUMENT, "No such serving slot");
        cx.serve_pos[slot] = -1;
    });
}

int mm_cuda_sample(mm_cuda_ctx* h, const float* logits, int batch, float temperature, const uint64_t* seeds,
                   const int32_t* draw_index, uint16_t* out) {
    return guarded(h, [&](mm::Context& cx) {
        if (!logits || !seeds || !out || batch < 1 || !std::isfinite(temperature) || temperature < 0)
            mm::fail(MM_INVALID_ARGUMENT, "Invalid generation settings");
        for (long long i = 0; i < static_cast<long long>(batch) * cx.c.V; ++i)
            if (!std::isfinite(logits[i])) mm::fail(MM_NUMERICAL_ERROR, "Invalid sampler logits");
        const size_t lb = sizeof(float) * batch * cx.c.V;
        char* base = static_cast<char*>(cx.stage.get(lb + static_cast<size_t>(batch) * 16 + 1024));
        float* d_log = reinterpret_cast<float*>(base);
        uint64_t* d_seed = reinterpret_cast<uint64_t*>(base + mm::round_up(static_cast<long long>(lb), 256));
        int* d_draw = reinterpret_cast<int*>(reinterpret_cast<char*>(d_seed) + mm::round_up(batch * 8LL, 256));
        uint16_t* d_out = reinterpret_cast<uint16_t*>(reinterpret_cast<char*>(d_draw) + mm::round_up(batch * 4LL, 256));
        MM_CUDA_CHECK(cudaMemcpyAsync(d_log, logits, lb, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(d_seed, seeds, batch * 8, cudaMemcpyHostToDevice, cx.stream));
        if (draw_index) MM_CUDA_CHECK(cudaMemcpyAsync(d_draw, draw_index, batch * 4, cudaMemcpyHostToDevice, cx.stream));
        mm::launch_sample(cx, d_log, batch, temperature, d_seed, draw_index ? d_draw : nullptr, 0, nullptr, d_out, 1);
        MM_CUDA_CHECK(cudaMemcpyAsync(out, d_out, batch * 2, cudaMemcpyDeviceToHost, cx.stream));
        mm::check_device(cx, "sample");
    });
}

int mm_cuda_rollout(mm_cuda_ctx* h, const uint16_t* prompts, int n, int prompt_len, int completion_tokens, int sequence,
                    uint16_t eos, uint16_t pad, const uint64_t* seeds, float temperature, uint16_t* out_tokens,
                    int32_t* out_len, uint16_t* out_input, uint16_t* out_target, float* out_mask, float* out_old_lp) {
    return guarded(h, [&](mm::Context& cx) {
        if (!prompts || !seeds || !out_tokens || !out_len) mm::fail(MM_INVALID_ARGUMENT, "null rollout buffer");
        mm::rollout(cx, prompts, n, prompt_len, completion_tokens, sequence, eos, pad, seeds, temperature, out_tokens,
                    out_len, out_input, out_target, out_mask, out_old_lp);
        cx.dec_len = 0;
    });
}

int mm_cuda_grpo_coefficients(mm_cuda_ctx* h, const float* lp, const float* old_lp, const float* ref_lp,
                              const float* mask, const float* rewards, int n, int seq, int group_size, int64_t n_total,
                              float clip, float klc, float* coefficients, float* advantages, double* loss, double* kl) {
    return guarded(h, [&](mm::Context& cx) {
        if (!lp || !old_lp || !ref_lp || !mask || !rewards || !coefficients || n < 1 || seq < 1 || group_size < 2 ||
            n % group_size || n_total < n)
            mm::fail(MM_INVALID_ARGUMENT, "Invalid reward group");
        if (!std::isfinite(clip) || clip <= 0 || clip >= 1 || !std::isfinite(klc) || klc < 0)
            mm::fail(MM_NUMERICAL_ERROR, "Invalid or unbounded GRPO token statistics");
        const long long T = static_cast<long long>(n) * seq;
        std::vector<int> sup(n, 0);
        for (int i = 0; i < n; ++i)
            for (int t = 0; t < seq; ++t) sup[i] += mask[static_cast<long long>(i) * seq + t] == 1.f ? 1 : 0;
        const long long fb = mm::round_up(T * 4, 256);
        char* base = static_cast<char*>(cx.stage.get(static_cast<size_t>(fb * 5 + mm::round_up(n * 4LL, 256) * 3 + 1024)));
        float* d_lp = reinterpret_cast<float*>(base);
        float* d_old = reinterpret_cast<float*>(base + fb);
        float* d_ref = reinterpret_cast<float*>(base + 2 * fb);
        float* d_mask = reinterpret_cast<float*>(base + 3 * fb);
        float* d_coef = reinterpret_cast<float*>(base + 4 * fb);
        float* d_rew = reinterpret_cast<float*>(base + 5 * fb);
        float* d_adv = d_rew + mm::round_up(n, 64);
        int* d_sup = reinterpret_cast<int*>(d_adv + mm::round_up(n, 64));
        MM_CUDA_CHECK(cudaMemcpyAsync(d_lp, lp, T * 4, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(d_old, old_lp, T * 4, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(d_ref, ref_lp, T * 4, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(d_mask, mask, T * 4, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(d_rew, rewards, n * 4, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(d_sup, sup.data(), n * 4, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemsetAsync(cx.d_any, 0, 4, cx.stream));
        MM_CUDA_CHECK(cudaMemsetAsync(cx.d_sums, 0, sizeof(mm::GrpoSums), cx.stream));
        MM_LAUNCH(mm::advantages_kernel, mm::blocks_for(n / group_size, 128), 128, 0, d_rew, n / group_size, group_size,
                  1e-6f, d_adv, cx.d_any);
        const unsigned nb = mm::blocks_for(T, 256);
        double2* part = static_cast<double2*>(cx.sums_part.get(sizeof(double2) * nb));
        MM_LAUNCH(mm::grpo_coef_kernel, nb, 256, 0, d_lp, d_old, d_ref, d_mask, d_adv, d_sup,
                  static_cast<int>(T), seq, static_cast<double>(n_total), clip, klc, d_coef, cx.d_sums, part);
        MM_LAUNCH(mm::grpo_sums_kernel, 1, 32, 0, part, static_cast<int>(nb), cx.d_sums);
        mm::GrpoSums sums{};
        MM_CUDA_CHECK(cudaMemcpyAsync(coefficients, d_coef, T * 4, cudaMemcpyDeviceToHost, cx.stream));
        if (advantages) MM_CUDA_CHECK(cudaMemcpyAsync(advantages, d_adv, n * 4, cudaMemcpyDeviceToHost, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(&sums, cx.d_sums, sizeof(sums), cudaMemcpyDeviceToHost, cx.stream));
        mm::check_device(cx, "grpo_coefficients");
        if (sums.rejected) mm::fail(MM_NUMERICAL_ERROR, "Invalid or unbounded GRPO token statistics");
        if (loss) *loss = sums.loss;
        if (kl) *kl = sums.kl;
    });
}

int mm_cuda_grpo_step(mm_cuda_ctx* policy, mm_cuda_ctx* reference, const uint16_t* input, const uint16_t* target,
                      const float* mask, const float* old_lp, const float* rewards, int n, int seq, int group_size,
                      int64_t n_total, float clip, float klc, float lr, mm_step_result* out) {
    if (!reference) return MM_INVALID_ARGUMENT;
    return guarded(policy, [&](mm::Context& cx) {
        if (!input || !target || !mask || !old_lp || !rewards || !out) mm::fail(MM_INVALID_ARGUMENT, "null GRPO buffer");
        if (reference->cx.unusable) mm::fail(MM_GPU_ERROR, "reference execution is unusable");
        *out = mm::grpo_step(cx, reference->cx, input, target, mask, old_lp, rewards, n, seq, group_size, n_total, clip,
                             klc, lr);
    });
}

int mm_cuda_dpo_step(mm_cuda_ctx* policy, mm_cuda_ctx* reference, const uint16_t* input, const uint16_t* target,
                     const float* mask, int n, int seq, int64_t n_total, float beta, float lr, mm_step_result* out,
                     double* margins) {
    if (!reference) return MM_INVALID_ARGUMENT;
    return guarded(policy, [&](mm::Context& cx) {
        if (!input || !target || !mask || !out) mm::fail(MM_INVALID_ARGUMENT, "null DPO buffer");
        if (reference->cx.unusable) mm::fail(MM_GPU_ERROR, "reference execution is unusable");
        *out = mm::dpo_step(cx, reference->cx, input, target, mask, n, seq, n_total, beta, lr, margins);
    });
}

int mm_cuda_nccl_unique_id(char out[128]) {
    try {
        ncclUniqueId id;
        if (mm::nccl().getUniqueId(&id) != ncclSuccess) return MM_GPU_ERROR;
        std::memcpy(out, &id, sizeof(id) < 128 ? sizeof(id) : 128);
        return MM_OK;
    } catch (const mm::Failure& e) {
        return e.code;
    }
}

int mm_cuda_init_comm(mm_cuda_ctx* h, int rank, int world, const char id[128]) {
    return guarded(h, [&](mm::Context& cx) {
        if (world < 1 || rank < 0 || rank >= world || !id) mm::fail(MM_INVALID_ARGUMENT, "invalid rank/world");
        if (world == 1) return;
        ncclUniqueId uid;
        std::memcpy(&uid, id, sizeof(uid));
        mm::nccl_init(cx, world, uid, rank);
        cx.rank = rank;
        cx.world = world;
    });
}

int64_t mm_cuda_kernel_launches(const mm_cuda_ctx* h) { return h ? h->cx.launches : -1; }

namespace mm {
// Waits on an mbarrier nothing arrives at for at most `polls` polls, then records a wait
// timeout in the error word and returns: the same bounded-wait exit as a stalled GEMM pipeline.
__global__ void wait_probe_kernel(uint32_t polls, int* err) {
    MM_PDL_ENTRY();
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        bool ok = false;
        for (uint32_t i = 0; i < polls && !ok; ++i) {
            ok = mbar_try_wait(&bar, 0);
            if (i > 64) __nanosleep(32);
        }
        if (!ok) raise_error(err, kErrWaitTimeout);
    }
}
}  // namespace mm

int mm_cuda_selftest_wait_timeout(mm_cuda_ctx* h, uint32_t polls) {
    return guarded(h, [&](mm::Context& cx) {
        if (polls < 1 || polls > (1u << 22)) mm::fail(MM_INVALID_ARGUMENT, "polls must be in [1, 2^22]");
        MM_LAUNCH(mm::wait_probe_kernel, 1, 32, 0, polls, cx.d_err);
        mm::check_device(cx, "wait self-test");
    });
}

// ---------------------------------------------------------------- include/mm_cuda_kernels.h

int mm_cuda_profile(mm_cuda_ctx* h, int enable, double* ms, int64_t* calls, double* work) {
    return guarded(h, [&](mm::Context& cx) {
        cx.prof_resolve();
        for (int i = 0; i < mm::kProfTags; ++i) {
            if (ms) ms[i] = cx.prof.ms[i];
            if (calls) calls[i] = cx.prof.calls[i];
            if (work) work[i] = cx.prof.work[i];
        }
        if (enable >= 0) {
            cx.profiling = enable != 0;
            cx.prof = mm::Profile{};
            cx.evlog.shapes.clear();
        }
    });
}

int mm_cuda_gemm_f16(mm_cuda_ctx* h, int M, int N, int K, const void* a, int64_t lda, int a_mn, const void* b,
                     int64_t ldb, int b_mn, void* out, int64_t ldc, int out_kind, float alpha, const float* residual,
                     int64_t ldr, int bf16) {
    return guarded(h, [&](mm::Context& cx) {
        // inputs written on any stream (the caller's) are complete before this stream reads them
        MM_CUDA_CHECK(cudaDeviceSynchronize());
        if (M < 1 || N < 1 || K < 1 || !a || !b || !out || out_kind < 0 || out_kind > 3)
            mm::fail(MM_INVALID_ARGUMENT, "invalid GEMM arguments");
        mm::GemmOutSpec o{out, ldc, out_kind};
        o.alpha = alpha;
        o.residual = residual;
        o.ldr = ldr;
        mm::gemm(cx, M, N, K, {a, lda, a_mn != 0}, {b, ldb, b_mn != 0}, o, bf16 != 0);
        mm::check_device(cx, "gemm");
    });
}

int mm_cuda_bench_gemm(mm_cuda_ctx* h, int reps, int M, int N, int K, const void* a, int64_t lda, int a_mn,
                       const void* b, int64_t ldb, int b_mn, void* out, int64_t ldc, int out_kind,
                       float* ms_per_launch) {
    return guarded(h, [&](mm::Context& cx) {
        // inputs written on any stream (the caller's) are complete before this stream reads them
        MM_CUDA_CHECK(cudaDeviceSynchronize());
        if (reps < 1 || reps > 4096 || M < 1 || N < 1 || K < 1 || !a || !b || !out || out_kind < 0 ||
            out_kind > 5 || !ms_per_launch)
            mm::fail(MM_INVALID_ARGUMENT, "invalid GEMM arguments");
        mm::GemmOutSpec o{out, ldc, out_kind <= 3 ? out_kind : (out_kind == 4 ? mm::kOutF32 : mm::kOutF16)};
        // the vocabulary head's epilogues: per-row inputs and outputs in one scratch block
        struct Scratch {
            void* p = nullptr;
            ~Scratch() { if (p) cudaFree(p); }
        } scratch;
        if (out_kind >= 4) {
            const size_t parts = 2ull * ((N + 63) / 64) * M;  // float2 partials, any tile width
            const size_t bytes = parts * 8 + 4ull * M * 4 + 16;
            MM_CUDA_CHECK(cudaMalloc(&scratch.p, bytes));
            MM_CUDA_CHECK(cudaMemsetAsync(scratch.p, 0, bytes, cx.stream));
            char* q = static_cast<char*>(scratch.p);
            float2* lse_part = reinterpret_cast<float2*>(q);
            uint16_t* targets = reinterpret_cast<uint16_t*>(q + parts * 8);
            float* row_a = reinterpret_cast<float*>(q + parts * 8 + 4ull * M);      // tgt_logit / lse
            float* row_b = reinterpret_cast<float*>(q + parts * 8 + 8ull * M);      // coef
            float* scale = reinterpret_cast<float*>(q + parts * 8 + 12ull * M);
            std::vector<uint16_t> t(M);
            for (int r = 0; r < M; ++r) t[r] = static_cast<uint16_t>(r % std::min(N, 65536));
            const float one = 1.f;
            std::vector<float> ones(M, 1.f);
            MM_CUDA_CHECK(cudaMemcpyAsync(targets, t.data(), 2ull * M, cudaMemcpyHostToDevice, cx.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(row_b, ones.data(), 4ull * M, cudaMemcpyHostToDevice, cx.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(scale, &one, 4, cudaMemcpyHostToDevice, cx.stream));
            MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
            o.targets = targets;
            if (out_kind == 4) {
                o.lse_part = lse_part;
                o.tgt_logit = row_a;
                o.no_store = true;
            } else {
                o.vg_lse = row_a;
                o.vg_coef = row_b;
                o.vg_scale = scale;
            }
        }
        const mm::Opnd A{a, lda, a_mn != 0}, B{b, ldb, b_mn != 0};
        // one eager launch sets kernel attributes and sizes the split-K staging
        mm::gemm(cx, M, N, K, A, B, o);
        mm::check_device(cx, "gemm");
        const bool prof = cx.profiling;
        const long long before = cx.launches;
        cx.profiling = false;
        cudaGraph_t g = nullptr;
        cudaGraphExec_t ge = nullptr;
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        MM_CUDA_CHECK(cudaStreamBeginCapture(cx.stream, cudaStreamCaptureModeThreadLocal));
        try {
            for (int r = 0; r < reps; ++r) mm::gemm(cx, M, N, K, A, B, o);
        } catch (...) {
            cudaStreamEndCapture(cx.stream, &g);
            if (g) cudaGraphDestroy(g);
            cx.profiling = prof;
            throw;
        }
        const cudaError_t ce = cudaStreamEndCapture(cx.stream, &g);
        cx.profiling = prof;
        const long long per_replay = cx.launches - before;
        if (ce != cudaSuccess || !g) mm::fail(MM_GPU_ERROR, std::string("GEMM graph capture: ") + cudaGetErrorString(ce));
        const cudaError_t ie = cudaGraphInstantiate(&ge, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) mm::fail(MM_GPU_ERROR, std::string("GEMM graph instantiate: ") + cudaGetErrorString(ie));
        float ms = 0.f;
        cudaError_t e = cudaGraphLaunch(ge, cx.stream);  // warm replay
        if (e == cudaSuccess) e = cudaEventCreate(&e0);
        if (e == cudaSuccess) e = cudaEventCreate(&e1);
        if (e == cudaSuccess) e = cudaEventRecord(e0, cx.stream);
        if (e == cudaSuccess) e = cudaGraphLaunch(ge, cx.stream);
        if (e == cudaSuccess) e = cudaEventRecord(e1, cx.stream);
        if (e == cudaSuccess) e = cudaEventSynchronize(e1);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
        if (e0) cudaEventDestroy(e0);
        if (e1) cudaEventDestroy(e1);
        cudaGraphExecDestroy(ge);
        if (e != cudaSuccess) mm::fail(MM_GPU_ERROR, std::string("GEMM graph replay: ") + cudaGetErrorString(e));
        cx.launches = before + 2 * per_replay;
        mm::check_device(cx, "gemm");
        *ms_per_launch = ms / static_cast<float>(reps);
    });
}

int mm_cuda_decode_attention(mm_cuda_ctx* h, const float* q, const void* cache, int64_t cache_seq_stride,
                             const int32_t* pos, int batch, int splits, float scale, void* out) {
    return guarded(h, [&](mm::Context& cx) {
        // inputs written on any stream (the caller's) are complete before this stream reads them
        MM_CUDA_CHECK(cudaDeviceSynchronize());
        if (!q || !cache || !pos || !out || batch < 1 || splits < 1 || splits > mm::kMaxDecodeSplits ||
            cache_seq_stride < mm::dec::W)
            mm::fail(MM_INVALID_ARGUMENT, "invalid decode attention arguments");
        float* part = nullptr;
        if (splits > 1)
            part = static_cast<float*>(cx.stage.get(sizeof(float) * static_cast<size_t>(batch) * splits * mm::dec::H *
                                                    (mm::dec::KV + 2)));
        // device time of the launch(es) alone, for the profile (the synchronisation above is not in it)
        cudaEvent_t t0 = cx.prof_begin();
        mm::launch_decode_attention(cx, q, static_cast<const __half*>(cache), cache_seq_stride, pos, batch, splits, scale,
                                    static_cast<__half*>(out), part);
        cx.prof_end(mm::kKDecodeAttn, t0);
        mm::check_device(cx, "decode_attention");
    });
}

int mm_decode_attention_noalloc(const float* q, const void* cache, int64_t cache_seq_stride, const int32_t* pos,
                                int batch, int splits, float scale, void* out, void* stream) {
    if (!q || !cache || !pos || !out || batch < 1 || splits < 1 || splits > mm::kMaxDecodeSplits ||
        cache_seq_stride < mm::dec::W)
        return MM_INVALID_ARGUMENT;
    if (splits > 1 && static_cast<long long>(batch) * splits > kStaticPartialSlots) return MM_INVALID_ARGUMENT;
    // the static array is read only by the split combine; one split writes `out` directly
    float* part = nullptr;
    if (splits > 1 && !(part = static_partials_address())) return MM_GPU_ERROR;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    try {
        mm::set_dynamic_smem<mm::decode_attention_row_kernel>(mm::dec::kRowSmem);
    } catch (...) {
        return MM_GPU_ERROR;
    }
    // Launch errors are taken from the launches themselves, not cudaGetLastError, so an error
    // an earlier call left pending stays with its owner and does not fail this call.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(mm::blocks_for(static_cast<long long>(batch) * splits, mm::dec::kWarps));
    cfg.blockDim = dim3(32 * mm::dec::kWarps);
    cfg.dynamicSmemBytes = mm::dec::kRowSmem;
    cfg.stream = s;
    if (cudaLaunchKernelEx(&cfg, mm::decode_attention_row_kernel, q, static_cast<const __half*>(cache),
                           static_cast<long long>(cache_seq_stride), static_cast<const int*>(pos), batch, splits, scale,
                           static_cast<__half*>(out), part, static_cast<const float*>(nullptr),
                           static_cast<const float*>(nullptr)) != cudaSuccess)
        return MM_GPU_ERROR;
    if (splits > 1) {
        cudaLaunchConfig_t cc = {};
        cc.gridDim = dim3(mm::blocks_for(static_cast<long long>(batch) * mm::dec::H * 32, 128));
        cc.blockDim = dim3(128);
        cc.stream = s;
        if (cudaLaunchKernelEx(&cc, mm::decode_attention_combine_kernel, static_cast<const float*>(part), splits, batch,
                               static_cast<__half*>(out)) != cudaSuccess)
            return MM_GPU_ERROR;
    }
    if (cudaStreamSynchronize(s) != cudaSuccess) return MM_GPU_ERROR;
    return MM_OK;
}

int64_t mm_cuda_profile_gemm_shapes(mm_cuda_ctx* h, char* buf, int64_t cap) {
    std::string text;
    int rc = guarded(h, [&](mm::Context& cx) {
        cx.prof_resolve();
        for (const auto& [key, st] : cx.evlog.shapes) {
            char line[192];
            std::snprintf(line, sizeof line, "%s calls=%lld ms=%.4f tflops=%.2f\n", key.c_str(), st.calls, st.ms,
                          st.ms > 0 ? st.flops / (st.ms * 1e9) : 0.0);
            text += line;
        }
    });
    if (rc) return -rc;
    if (buf && cap > 0) {
        const size_t n = std::min(static_cast<size_t>(cap - 1), text.size());
        std::memcpy(buf, text.data(), n);
        buf[n] = 0;
    }
    return static_cast<int64_t>(text.size());
}

int mm_cuda_decode_trace(mm_cuda_ctx* h, int enable, uint64_t* out_ns, int cap, int* count) {
    return guarded(h, [&](mm::Context& cx) {
        if (enable >= 0) cx.dec.mk_trace_on = enable != 0;
        if (count) *count = 0;
        if (!out_ns || cap <= 0 || !cx.dec.mk_trace) return;
        const int n = std::min(cap, mm::kMkTraceSlots);
        MM_CUDA_CHECK(cudaMemcpyAsync(out_ns, cx.dec.mk_trace, sizeof(uint64_t) * n, cudaMemcpyDeviceToHost, cx.stream));
        MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
        if (count) *count = n;
    });
}

int mm_cuda_stream(mm_cuda_ctx* h, void** stream) {
    return guarded(h, [&](mm::Context& cx) { *stream = cx.stream; });
}

} // extern "C"
