// Optimizer step, gradient all-reduce (NCCL over NVLink), the GRPO update and the batched
// rollout driver.
#pragma once
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <thread>

#include "decode.cuh"

namespace mm {

// ------------------------------------------------------------------ NCCL, loaded on demand
// The library is opened at the first data-parallel call, so single-GPU use carries no
// NCCL dependency and a process that already loaded one (e.g. through torch) reuses it.
struct Nccl {
    void* lib = nullptr;
    ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    const char* (*getErrorString)(ncclResult_t) = nullptr;
    // non-blocking initialisation with a deadline (present in NCCL >= 2.14)
    ncclResult_t (*commInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
};
inline Nccl& nccl() {
    static Nccl n;
    if (!n.lib) {
        n.lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!n.lib) fail(MM_UNSUPPORTED, std::string("cannot load libnccl.so.2: ") + dlerror());
        n.getUniqueId = reinterpret_cast<decltype(n.getUniqueId)>(dlsym(n.lib, "ncclGetUniqueId"));
        n.commInitRank = reinterpret_cast<decltype(n.commInitRank)>(dlsym(n.lib, "ncclCommInitRank"));
        n.allReduce = reinterpret_cast<decltype(n.allReduce)>(dlsym(n.lib, "ncclAllReduce"));
        n.commDestroy = reinterpret_cast<decltype(n.commDestroy)>(dlsym(n.lib, "ncclCommDestroy"));
        n.getErrorString = reinterpret_cast<decltype(n.getErrorString)>(dlsym(n.lib, "ncclGetErrorString"));
        if (!n.getUniqueId || !n.commInitRank || !n.allReduce || !n.commDestroy || !n.getErrorString)
            fail(MM_UNSUPPORTED, "libnccl.so.2 lacks the expected symbols");
        n.commInitRankConfig = reinterpret_cast<decltype(n.commInitRankConfig)>(dlsym(n.lib, "ncclCommInitRankConfig"));
        n.commGetAsyncError = reinterpret_cast<decltype(n.commGetAsyncError)>(dlsym(n.lib, "ncclCommGetAsyncError"));
        n.commAbort = reinterpret_cast<decltype(n.commAbort)>(dlsym(n.lib, "ncclCommAbort"));
    }
    return n;
}
#define MM_NCCL_CHECK(x)                                                                     \
    do {                                                                                     \
        ncclResult_t r_ = (x);                                                               \
        if (r_ != ncclSuccess) ::mm::fail(MM_GPU_ERROR, std::string(#x) + ": " + ::mm::nccl().getErrorString(r_)); \
    } while (0)

// Seconds a communicator may take to form (MM_NCCL_INIT_TIMEOUT, default 300): a rank
// that never joins turns into a gpu_error instead of a hang.
inline double nccl_init_timeout() {
    const char* e = std::getenv("MM_NCCL_INIT_TIMEOUT");
    const double v = e ? std::atof(e) : 0.0;
    return v > 0 ? v : 300.0;
}

// Waits, up to `seconds`, for a non-blocking communicator's pending operation; false on
// timeout, fails on an NCCL error.
inline bool nccl_settle(ncclComm_t comm, double seconds, const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        ncclResult_t st = ncclSuccess;
        MM_NCCL_CHECK(nccl().commGetAsyncError(comm, &st));
        if (st == ncclSuccess) return true;
        if (st != ncclInProgress) fail(MM_GPU_ERROR, std::string(what) + ": " + nccl().getErrorString(st));
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > seconds) return false;
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
}

// ncclCommInitRank with a deadline: non-blocking initialisation polled until it completes,
// aborted (gpu_error) when the other ranks do not join in time. Blocking when the library
// lacks the non-blocking entry points.
inline void nccl_init(Context& cx, int world, const ncclUniqueId& uid, int rank) {
    Nccl& n = nccl();
    ncclComm_t comm = nullptr;
    if (!n.commInitRankConfig || !n.commGetAsyncError || !n.commAbort) {
        MM_NCCL_CHECK(n.commInitRank(&comm, world, uid, rank));
        cx.nccl_comm = comm;
        return;
    }
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    const ncclResult_t r = n.commInitRankConfig(&comm, world, uid, rank, &config);
    if (r != ncclSuccess && r != ncclInProgress)
        fail(MM_GPU_ERROR, std::string("ncclCommInitRankConfig: ") + n.getErrorString(r));
    const double limit = nccl_init_timeout();
    if (!nccl_settle(comm, limit, "ncclCommInitRankConfig")) {
        n.commAbort(comm);
        fail(MM_GPU_ERROR, "NCCL communicator did not form within " + std::to_string(static_cast<int>(limit)) +
                               " s (a rank did not join)");
    }
    cx.nccl_comm = comm;
    cx.nccl_nonblocking = true;
}

inline void allreduce(Context& cx, void* buf, size_t count, ncclDataType_t t, ncclRedOp_t op) {
    if (cx.world <= 1 || !cx.nccl_comm) return;
    ncclComm_t comm = static_cast<ncclComm_t>(cx.nccl_comm);
    const ncclResult_t r = nccl().allReduce(buf, buf, count, t, op, comm, cx.stream);
    if (r == ncclInProgress && cx.nccl_nonblocking) {
        if (!nccl_settle(comm, nccl_init_timeout(), "ncclAllReduce")) fail(MM_GPU_ERROR, "ncclAllReduce was not enqueued");
        return;
    }
    if (r != ncclSuccess) fail(MM_GPU_ERROR, std::string("ncclAllReduce: ") + nccl().getErrorString(r));
}

// Waits for the context stream once a collective has been enqueued on it. With several
// ranks on a non-blocking communicator the wait is bounded: the stream and the
// communicator's asynchronous error are polled, and a collective that has not completed
// within MM_NCCL_INIT_TIMEOUT seconds (a peer stopped, or took a different path) aborts the
// communicator, marks the context unusable and fails with gpu_error instead of hanging.
inline void sync_collective(Context& cx) {
    if (cx.world <= 1 || !cx.nccl_comm || !cx.nccl_nonblocking) {
        MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
        return;
    }
    ncclComm_t comm = static_cast<ncclComm_t>(cx.nccl_comm);
    const double limit = nccl_init_timeout();
    const auto t0 = std::chrono::steady_clock::now();
    for (long long polls = 0;; ++polls) {
        const cudaError_t e = cudaStreamQuery(cx.stream);
        if (e == cudaSuccess) return;
        if (e != cudaErrorNotReady) MM_CUDA_CHECK(e);
        ncclResult_t st = ncclSuccess;
        nccl().commGetAsyncError(comm, &st);
        const double waited = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if ((st != ncclSuccess && st != ncclInProgress) || waited > limit) {
            nccl().commAbort(comm);
            cx.nccl_comm = nullptr;
            cx.unusable = true;
            if (st != ncclSuccess && st != ncclInProgress)
                fail(MM_GPU_ERROR, std::string("collective failed: ") + nccl().getErrorString(st));
            fail(MM_GPU_ERROR, "collective did not complete within " + std::to_string(static_cast<int>(limit)) +
                                   " s (a peer rank stopped or diverged); communicator aborted");
        }
        if (polls < 2000)
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// First failed host-side check of a batch: the code and message to report. On several ranks
// the status travels with the step's first collective, so every rank fails together instead
// of the others blocking in a collective the failing rank never joins.
struct BatchCheck {
    int code = 0;
    std::string msg;
    void set(int c, const char* m) {
        if (!code) {
            code = c;
            msg = m;
        }
    }
};

// Max-reduces [flag0, invalid] over the ranks (flag0 as computed on the device, invalid =
// this rank's BatchCheck) and fails on every rank when any rank's batch was invalid.
// Returns the reduced flag0.
inline int reduce_flag_and_check(Context& cx, int* d_flags, const BatchCheck& bad) {
    MM_CUDA_CHECK(cudaMemsetAsync(d_flags + 1, bad.code ? 1 : 0, 4, cx.stream));
    allreduce(cx, d_flags, 2, ncclInt32, ncclMax);
    int flags[2] = {0, 0};
    MM_CUDA_CHECK(cudaMemcpyAsync(flags, d_flags, 8, cudaMemcpyDeviceToHost, cx.stream));
    sync_collective(cx);
    if (bad.code) fail(bad.code, bad.msg);
    if (flags[1]) fail(MM_INVALID_ARGUMENT, "a peer rank rejected its batch");
    return flags[0];
}

// ------------------------------------------------------------------ timing
struct PhaseTimer {
    Context& cx;
    int ph;
    cudaEvent_t start;
    PhaseTimer(Context& c, int p) : cx(c), ph(p), start(c.prof_begin()) {}
    ~PhaseTimer() { cx.prof_end(ph, start); }
};

// ------------------------------------------------------------------ AdamW
// Execution::update: all-reduce, then Optimizer::step (optimizer.cpp:105-161).
inline double adamw_update(Context& cx, float lr) {
    if (!cx.trainable) fail(MM_INVALID_ARGUMENT, "Inference execution has no optimizer");
    if (!std::isfinite(lr) || lr < 0) fail(MM_INVALID_ARGUMENT, "Invalid learning rate or uninitialized optimizer");
    {
        PhaseTimer t(cx, kPhAllreduce);
        allreduce(cx, cx.g, static_cast<size_t>(cx.P_dev), ncclFloat32, ncclSum);
    }
    PhaseTimer t(cx, kPhAdamw);
    MM_CUDA_CHECK(cudaMemsetAsync(cx.d_nonfinite, 0, 4, cx.stream));
    MM_CUDA_CHECK(cudaMemsetAsync(cx.d_nonfinite_out, 0, 4, cx.stream));
    MM_LAUNCH(adamw_norm_partial_kernel, cx.n_partial, 256, 0, cx.g, cx.P_dev, cx.d_partial, cx.d_nonfinite);
    MM_LAUNCH(adamw_finalize_kernel, 1, 1024, 0, cx.d_partial, cx.n_partial, cx.opt.clip_norm, cx.d_norm, cx.d_gs);
    const uint64_t next = cx.steps + 1;
    const float bc1 = static_cast<float>(1.0 - std::pow(static_cast<double>(cx.opt.beta1), static_cast<double>(next)));
    const float bc2 = static_cast<float>(1.0 - std::pow(static_cast<double>(cx.opt.beta2), static_cast<double>(next)));
    dim3 grid(256, static_cast<unsigned>(cx.params.size()));
    // w, g, m, v read + w, m, v written in fp32 + the fp16 shadow (3 copies for the table)
    const double bytes = 28.0 * cx.P + 2.0 * cx.P + 4.0 * cx.c.V * cx.c.d;
    MM_LAUNCH_TIMED(kKAdamw, bytes, adamw_update_kernel, grid, 256, 0, cx.d_params, cx.w, cx.g, cx.m, cx.v, cx.shadow,
                    cx.d_gs, cx.d_nonfinite, lr, cx.opt.beta1, cx.opt.beta2, cx.opt.epsilon, bc1, bc2, cx.d_nonfinite_out);
    int flags[2] = {0, 0};
    double norm = 0;
    MM_CUDA_CHECK(cudaMemcpyAsync(&flags[0], cx.d_nonfinite, 4, cudaMemcpyDeviceToHost, cx.stream));
    MM_CUDA_CHECK(cudaMemcpyAsync(&flags[1], cx.d_nonfinite_out, 4, cudaMemcpyDeviceToHost, cx.stream));
    MM_CUDA_CHECK(cudaMemcpyAsync(&norm, cx.d_norm, 8, cudaMemcpyDeviceToHost, cx.stream));
    sync_collective(cx);
    if (flags[0]) fail(MM_NUMERICAL_ERROR, "Nonfinite gradient before optimizer update");
    cx.steps = next;
    refresh_derived(cx, false);
    if (flags[1]) fail(MM_NUMERICAL_ERROR, "Nonfinite optimizer output");
    check_device(cx, "update");
    return norm;
}

// Rollout decode steps replay a captured CUDA graph unless MM_DECODE_GRAPH=0 (then every
// kernel is launched and timed individually; same work, same results).
inline bool decode_graphs_enabled() {
    static int v = [] {
        const char* e = std::getenv("MM_DECODE_GRAPH");
        return (e && e[0] == '0') ? 0 : 1;
    }();
    return v != 0;
}

// The frozen reference's forward of one chunk. By default it runs on its own stream beside
// the policy's backward of the previous chunk, with single-CTA products (CTA pairs need both
// SMs of a TPC free at once and stall behind the other stream's CTAs); MM_REF_OVERLAP=0 runs
// it after that backward instead, on CTA pairs where they apply.
inline bool ref_overlap_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("MM_REF_OVERLAP");
        return !(e && e[0] == '0');
    }();
    return on;
}
inline void reference_forward(Context& pc, Context& rc, int rows, int S) {
    const bool overlap = ref_overlap_enabled();
    if (!overlap) MM_CUDA_CHECK(cudaStreamSynchronize(pc.stream));
    struct Restore {  // pair products allowed again however the forward ends
        Context& c;
        ~Restore() { c.pair_ok = true; }
    } restore{rc};
    rc.pair_ok = !overlap;
    forward_chunk(rc, rows, S, false, kVocabAll, true, nullptr, 0, 0, nullptr);
}

// Tokens per teacher-forced chunk (whole sequences). 196,608 = 512 sequences of 384: the
// policy's workspace with tape is ~340 KB per token (~67 GB), the frozen reference's ~100 KB
// per token, well inside 180 GB; per-chunk fixed costs (host synchronisation per chunk, the
// reference overlap's ramp, wave tails, split-K partials) fall with the chunk count. Measured
// GRPO step at 2,048 x 384: 1.199 s at 32,768, 1.161 at 49,152, 1.104 at 98,304, 1.083 at
// 196,608 tokens. MM_CHUNK_TOKENS overrides it.
inline int chunk_tokens_default() {
    static int v = [] {
        const char* e = std::getenv("MM_CHUNK_TOKENS");
        int x = e ? std::atoi(e) : 0;
        return x > 0 ? x : 196608;
    }();
    return v;
}

// Tokens per chunk for this model: the default, capped (unless MM_CHUNK_TOKENS is set) so
// that the policy's workspace with tape stays within 45 % of the device's memory. The cap
// depends only on the model and the device, never on what is free at the time, so the
// chunking (and with it the update's rounding) is the same on every run and rank. The 35.8M
// model (~360 KB per token) keeps 196,608; the 2,048-wide 1.1B model (~2.4 MB) gets ~34 K.
inline int chunk_tokens(Context& cx) {
    static const bool pinned = std::getenv("MM_CHUNK_TOKENS") != nullptr;
    if (pinned) return chunk_tokens_default();
    if (!cx.chunk_cap) {
        constexpr int kProbe = 4096;
        const int T0 = cx.ws.T;
        const bool tape0 = cx.ws.tape;
        Sizer a, b;
        plan_workspace(cx, a, kProbe, true);
        plan_workspace(cx, b, 2 * kProbe, true);
        const double per_token = static_cast<double>(b.used() - a.used()) / kProbe;
        size_t fr = 0, total = 0;
        MM_CUDA_CHECK(cudaMemGetInfo(&fr, &total));
        cx.chunk_cap = static_cast<int>(std::min(2.0e9, 0.45 * static_cast<double>(total) / per_token));
        // plan_workspace leaves the chunk's buffer table pointing nowhere: restore it
        if (cx.ws_arena.capacity()) {
            cx.ws_arena.reset();
            plan_workspace(cx, cx.ws_arena, T0, tape0);
        } else {
            cx.ws.T = 0;
            cx.ws.tape = tape0;
        }
    }
    return std::max(1, std::min(chunk_tokens_default(), cx.chunk_cap));
}

// Teacher-forced log-probabilities of host batches [B][S] (Execution::log_probabilities),
// chunked over whole sequences. Result into host `out` [B*S].
inline void log_probs_host(Context& cx, const uint16_t* input, const uint16_t* target, int B, int S, float* out) {
    PhaseTimer t(cx, kPhLogprob);
    const int per = std::max(1, chunk_tokens(cx) / S);
    ensure_workspace(cx, std::min(B, per) * S, false);  // reuses a larger workspace with tape
    Workspace& w = cx.ws;
    for (int r0 = 0; r0 < B; r0 += per) {
        const int bc = std::min(per, B - r0);
        const long long T = static_cast<long long>(bc) * S;
        MM_CUDA_CHECK(cudaMemcpyAsync(w.tokens, input + r0 * static_cast<long long>(S), T * 2, cudaMemcpyHostToDevice, cx.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(w.targets, target + r0 * static_cast<long long>(S), T * 2, cudaMemcpyHostToDevice, cx.stream));
        forward_chunk(cx, bc, S, false, kVocabAll, true, nullptr, 0, 0, nullptr);
        MM_CUDA_CHECK(cudaMemcpyAsync(out + r0 * static_cast<long long>(S), w.lp, T * 4, cudaMemcpyDeviceToHost, cx.stream));
    }
    check_device(cx, "log_probabilities");
}

// ------------------------------------------------------------------ GRPO update
// Records, on `from`, the point after which `to` may proceed (cudaStreamWaitEvent) — used
// so the frozen reference's next forward never overwrites log-probs a pending copy on the
// policy stream still reads.
struct StreamOrder {
    cudaEvent_t ev = nullptr;
    bool recorded = false;
    StreamOrder() { MM_CUDA_CHECK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming)); }
    ~StreamOrder() { cudaEventDestroy(ev); }
    void record(cudaStream_t from) {
        MM_CUDA_CHECK(cudaEventRecord(ev, from));
        recorded = true;
    }
    void wait(cudaStream_t to) {
        if (recorded) MM_CUDA_CHECK(cudaStreamWaitEvent(to, ev, 0));
    }
};

inline mm_step_result grpo_step(Context& pc, Context& rc, const uint16_t* input, const uint16_t* target,
                                const float* mask, const float* old_lp, const float* rewards, int n, int S, int G,
                                long long n_total, float clip, float klc, float lr) {
    if (!pc.trainable) fail(MM_INVALID_ARGUMENT, "policy context must be trainable");
    if (pc.device != rc.device) fail(MM_INVALID_ARGUMENT, "policy and reference must share a device");
    BatchCheck bad;
    if (n < 1 || G < 2 || n % G || S < 1 || S > pc.c.maxS || n_total < n)
        bad.set(MM_INVALID_ARGUMENT, "rollouts must form whole groups within the context");
    else if (!std::isfinite(clip) || clip <= 0 || clip >= 1 || !std::isfinite(klc) || klc < 0)
        bad.set(MM_NUMERICAL_ERROR, "Invalid or unbounded GRPO token statistics");
    std::vector<int> sup(std::max(n, 0), 0);
    if (!bad.code) {
        const long long NS = static_cast<long long>(n) * S;
        for (int i = 0; i < n && !bad.code; ++i) {
            for (int t = 0; t < S; ++t) {
                const float mv = mask[static_cast<long long>(i) * S + t];
                if (mv != 0.f && mv != 1.f) {
                    bad.set(MM_INVALID_ARGUMENT, "Loss mask must contain zero or one");
                    break;
                }
                sup[i] += mv == 1.f ? 1 : 0;
            }
            if (!bad.code && sup[i] == 0) bad.set(MM_INVALID_ARGUMENT, "Batch has no supervised tokens");
        }
        for (long long i = 0; i < NS && !bad.code; ++i)
            if (input[i] >= pc.c.V || target[i] >= pc.c.V) bad.set(MM_INVALID_ARGUMENT, "Input token exceeds vocabulary");
        for (int i = 0; i < n && !bad.code; ++i)
            if (!std::isfinite(rewards[i])) bad.set(MM_INVALID_ARGUMENT, "Invalid reward group");
    }
    if (bad.code && pc.world <= 1) fail(bad.code, bad.msg);
    char* base = static_cast<char*>(pc.stage.get(static_cast<size_t>(std::max(n, 1)) * 16 + 1024));
    float* d_rew = reinterpret_cast<float*>(base);
    float* d_adv = reinterpret_cast<float*>(base + round_up(n * 4LL, 256));
    int* d_sup = reinterpret_cast<int*>(base + 2 * round_up(n * 4LL, 256));
    MM_CUDA_CHECK(cudaMemsetAsync(pc.d_any, 0, 8, pc.stream));
    if (!bad.code) {
        MM_CUDA_CHECK(cudaMemcpyAsync(d_rew, rewards, n * 4, cudaMemcpyHostToDevice, pc.stream));
        MM_CUDA_CHECK(cudaMemcpyAsync(d_sup, sup.data(), n * 4, cudaMemcpyHostToDevice, pc.stream));
        MM_LAUNCH_CX(pc, advantages_kernel, blocks_for(n / G, 128), 128, 0, d_rew, n / G, G, 1e-6f, d_adv, pc.d_any);
    }
    // the global skip rule (trainer.cpp:818-820) and every rank's batch check in one collective
    const int any = reduce_flag_and_check(pc, pc.d_any, bad);
    mm_step_result res{};
    if (!any) {
        res.skipped = 1;
        return res;
    }
    MM_CUDA_CHECK(cudaMemsetAsync(pc.g, 0, sizeof(float) * pc.P_dev, pc.stream));
    MM_CUDA_CHECK(cudaMemsetAsync(pc.d_sums, 0, sizeof(GrpoSums), pc.stream));
    const int per = std::max(1, chunk_tokens(pc) / S);
    ensure_workspace(pc, std::min(n, per) * S, true);
    ensure_workspace(rc, std::min(n, per) * S, rc.ws.tape);
    Workspace& w = pc.ws;
    StreamOrder ref_lp_copied;
    // the rows whose log-probabilities the update uses (mask != 0), per chunk: both models'
    // vocabulary heads and the policy's vocabulary backward run on these only
    struct Selection {
        Context &p, &r;
        ~Selection() { p.ws.nsel = r.ws.nsel = -1; }
    } selection{pc, rc};
    for (int r0 = 0; r0 < n; r0 += per) {
        const int bc = std::min(per, n - r0);
        const long long T = static_cast<long long>(bc) * S, off = static_cast<long long>(r0) * S;
        int nsel = 0;  // the GEMMs' row count; the devices list the rows themselves
        for (long long i = 0; i < T; ++i) nsel += mask[off + i] != 0.f;
        {
            PhaseTimer t(pc, kPhLogprob);
            // the previous chunk's log-probs must have left rc.ws.lp before this forward
            // rewrites it (the copy is queued on the policy stream behind its backward)
            ref_lp_copied.wait(rc.stream);
            MM_CUDA_CHECK(cudaMemcpyAsync(rc.ws.tokens, input + off, T * 2, cudaMemcpyHostToDevice, rc.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(rc.ws.targets, target + off, T * 2, cudaMemcpyHostToDevice, rc.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(rc.ws.mask, mask + off, T * 4, cudaMemcpyHostToDevice, rc.stream));
            select_rows(rc, static_cast<int>(T), nsel);
            reference_forward(pc, rc, bc, S);
            MM_CUDA_CHECK(cudaMemcpyAsync(w.tokens, input + off, T * 2, cudaMemcpyHostToDevice, pc.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(w.targets, target + off, T * 2, cudaMemcpyHostToDevice, pc.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(w.mask, mask + off, T * 4, cudaMemcpyHostToDevice, pc.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(w.old_lp, old_lp + off, T * 4, cudaMemcpyHostToDevice, pc.stream));
            select_rows(pc, static_cast<int>(T), nsel);
            // the reference's log-probs reach the policy stream only after its forward completes
            MM_CUDA_CHECK(cudaStreamSynchronize(rc.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(w.ref_lp, rc.ws.lp, T * 4, cudaMemcpyDeviceToDevice, pc.stream));
            ref_lp_copied.record(pc.stream);
            forward_chunk(pc, bc, S, true, kVocabAll, true, nullptr, 0, 0, nullptr);
        }
        PhaseTimer t(pc, kPhBackward);
        MM_CUDA_CHECK(cudaMemsetAsync(&pc.d_sums->max_coef_bits, 0, 4, pc.stream));
        const unsigned nb = blocks_for(T, 256);
        double2* part = static_cast<double2*>(pc.sums_part.get(sizeof(double2) * nb));
        MM_LAUNCH_CX(pc, grpo_coef_kernel, nb, 256, 0, w.lp, w.old_lp, w.ref_lp, w.mask, d_adv + r0,
                     d_sup + r0, static_cast<int>(T), S, static_cast<double>(n_total), clip, klc, w.coef, pc.d_sums, part);
        MM_LAUNCH_CX(pc, grpo_sums_kernel, 1, 32, 0, part, static_cast<int>(nb), pc.d_sums);
        MM_LAUNCH_CX(pc, grad_scale_kernel, 1, 1, 0, pc.d_sums, pc.d_scale);
        backward_chunk(pc, bc, S);
    }
    check_device(rc, "reference log_probabilities");
    check_device(pc, "grpo backward");
    GrpoSums sums{};
    MM_CUDA_CHECK(cudaMemcpyAsync(&sums, pc.d_sums, sizeof(GrpoSums), cudaMemcpyDeviceToHost, pc.stream));
    MM_CUDA_CHECK(cudaStreamSynchronize(pc.stream));
    if (sums.rejected && pc.world <= 1) fail(MM_NUMERICAL_ERROR, "Invalid or unbounded GRPO token statistics");
    // loss and kl sums, and every rank's rejected-token count, in one collective: a rejection
    // anywhere fails the step on every rank before the gradient all-reduce
    const double rejected = sums.rejected ? 1.0 : 0.0;
    MM_CUDA_CHECK(cudaMemcpyAsync(&pc.d_sums->rejected_ranks, &rejected, 8, cudaMemcpyHostToDevice, pc.stream));
    allreduce(pc, pc.d_sums, 3, ncclFloat64, ncclSum);
    MM_CUDA_CHECK(cudaMemcpyAsync(&sums, pc.d_sums, sizeof(GrpoSums), cudaMemcpyDeviceToHost, pc.stream));
    sync_collective(pc);
    if (sums.rejected_ranks != 0) fail(MM_NUMERICAL_ERROR, "Invalid or unbounded GRPO token statistics");
    res.grad_norm = adamw_update(pc, lr);
    res.loss = sums.loss;
    res.kl = sums.kl;
    return res;
}

// ------------------------------------------------------------------ DPO update
// The DPO update (trainer.cpp:765-783 with preference_objective :107-121 and Execution::step)
// over n preference pairs: rows 2p (chosen) and 2p + 1 (rejected) of the [2n][S] batch. Per
// chunk of whole pairs: the frozen reference's log-probs, the policy's taped forward,
// dpo_coef_kernel (coefficients over the n_total pairs of the update across ranks), the
// backward; then the gradient all-reduce and AdamW. loss = sum of pair losses / n_total and
// kl = sum of pair margins / n_total, both summed over ranks; margins (host [n], may be null)
// receives each local pair's margin.
inline mm_step_result dpo_step(Context& pc, Context& rc, const uint16_t* input, const uint16_t* target,
                               const float* mask, int n, int S, long long n_total, float beta, float lr,
                               double* margins) {
    if (!pc.trainable) fail(MM_INVALID_ARGUMENT, "policy context must be trainable");
    if (pc.device != rc.device) fail(MM_INVALID_ARGUMENT, "policy and reference must share a device");
    BatchCheck bad;
    if (n < 1 || S < 1 || S > pc.c.maxS || n_total < n) bad.set(MM_INVALID_ARGUMENT, "Invalid preference batch");
    else if (!std::isfinite(beta) || beta <= 0) bad.set(MM_INVALID_ARGUMENT, "Invalid DPO beta");
    if (!bad.code) {
        const long long NS = 2LL * n * S;
        for (long long i = 0; i < NS && !bad.code; ++i) {
            if (mask[i] != 0.f && mask[i] != 1.f) bad.set(MM_INVALID_ARGUMENT, "Loss mask must contain zero or one");
            else if (input[i] >= pc.c.V || target[i] >= pc.c.V) bad.set(MM_INVALID_ARGUMENT, "Input token exceeds vocabulary");
        }
    }
    if (bad.code && pc.world <= 1) fail(bad.code, bad.msg);
    if (pc.world > 1) {  // every rank's batch check, before any rank starts the passes
        MM_CUDA_CHECK(cudaMemsetAsync(pc.d_any, 0, 8, pc.stream));
        reduce_flag_and_check(pc, pc.d_any, bad);
    }
    MM_CUDA_CHECK(cudaMemsetAsync(pc.g, 0, sizeof(float) * pc.P_dev, pc.stream));
    MM_CUDA_CHECK(cudaMemsetAsync(pc.d_sums, 0, sizeof(GrpoSums), pc.stream));
    double2* part = static_cast<double2*>(pc.sums_part.get(sizeof(double2) * static_cast<size_t>(n) +
                                                            sizeof(double) * static_cast<size_t>(n)));
    double* d_margins = reinterpret_cast<double*>(part + n);
    const int per = std::max(1, chunk_tokens(pc) / (2 * S));  // pairs per chunk
    ensure_workspace(pc, 2 * std::min(n, per) * S, true);
    ensure_workspace(rc, 2 * std::min(n, per) * S, rc.ws.tape);
    Workspace& w = pc.ws;
    StreamOrder ref_lp_copied;
    for (int p0 = 0; p0 < n; p0 += per) {
        const int bp = std::min(per, n - p0), rows = 2 * bp;
        const long long T = static_cast<long long>(rows) * S, off = 2LL * p0 * S;
        {
            PhaseTimer t(pc, kPhLogprob);
            ref_lp_copied.wait(rc.stream);  // the previous chunk's copy out of rc.ws.lp is done
            MM_CUDA_CHECK(cudaMemcpyAsync(rc.ws.tokens, input + off, T * 2, cudaMemcpyHostToDevice, rc.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(rc.ws.targets, target + off, T * 2, cudaMemcpyHostToDevice, rc.stream));
            reference_forward(pc, rc, rows, S);
            MM_CUDA_CHECK(cudaMemcpyAsync(w.tokens, input + off, T * 2, cudaMemcpyHostToDevice, pc.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(w.targets, target + off, T * 2, cudaMemcpyHostToDevice, pc.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(w.mask, mask + off, T * 4, cudaMemcpyHostToDevice, pc.stream));
            // the reference's log-probs reach the policy stream only after its forward completes
            MM_CUDA_CHECK(cudaStreamSynchronize(rc.stream));
            MM_CUDA_CHECK(cudaMemcpyAsync(w.ref_lp, rc.ws.lp, T * 4, cudaMemcpyDeviceToDevice, pc.stream));
            ref_lp_copied.record(pc.stream);
            forward_chunk(pc, rows, S, true, kVocabAll, true, nullptr, 0, 0, nullptr);
        }
        PhaseTimer t(pc, kPhBackward);
        MM_LAUNCH_CX(pc, dpo_coef_kernel, bp, 256, 0, w.lp, w.ref_lp, w.mask, S, beta, static_cast<float>(n_total),
                     static_cast<double>(n_total), w.coef, part + p0, d_margins + p0);
        MM_CUDA_CHECK(cudaMemsetAsync(&pc.d_sums->max_coef_bits, 0, 4, pc.stream));
        MM_LAUNCH_CX(pc, absmax_kernel, std::min<unsigned>(blocks_for(T, 1024), sm_count() * 4), 256, 0, w.coef, T,
                     &pc.d_sums->max_coef_bits);
        MM_LAUNCH_CX(pc, grad_scale_kernel, 1, 1, 0, pc.d_sums, pc.d_scale);
        backward_chunk(pc, rows, S);
    }
    check_device(rc, "reference log_probabilities");
    check_device(pc, "dpo backward");
    MM_LAUNCH_CX(pc, grpo_sums_kernel, 1, 32, 0, part, n, pc.d_sums);
    if (margins) MM_CUDA_CHECK(cudaMemcpyAsync(margins, d_margins, sizeof(double) * n, cudaMemcpyDeviceToHost, pc.stream));
    allreduce(pc, pc.d_sums, 2, ncclFloat64, ncclSum);
    GrpoSums sums{};
    MM_CUDA_CHECK(cudaMemcpyAsync(&sums, pc.d_sums, sizeof(GrpoSums), cudaMemcpyDeviceToHost, pc.stream));
    sync_collective(pc);
    if (!std::isfinite(sums.loss)) fail(MM_NUMERICAL_ERROR, "Nonfinite logits or loss");
    mm_step_result res{};
    res.grad_norm = adamw_update(pc, lr);
    res.loss = sums.loss;
    res.kl = sums.kl / static_cast<double>(n_total);
    return res;
}

__global__ void column_gather_kernel(const uint16_t* __restrict__ src, long long stride, int col, int B,
                                     uint16_t* __restrict__ dst) {
    MM_PDL_ENTRY();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) dst[b] = src[b * stride + col];
}

// rollout() for n prompts (trainer.cpp:187-213).
inline void rollout(Context& cx, const uint16_t* prompts, int n, int P, int completion, int S, uint16_t eos,
                    uint16_t pad, const uint64_t* seeds, float temperature, uint16_t* out_tokens, int32_t* out_len,
                    uint16_t* out_input, uint16_t* out_target, float* out_mask, float* out_old_lp) {
    const Dims& c = cx.c;
    if (n < 1 || P < 1 || P > c.maxS || completion < 1) fail(MM_INVALID_ARGUMENT, "Prompt exceeds context or is empty");
    if (!std::isfinite(temperature) || temperature < 0) fail(MM_INVALID_ARGUMENT, "Invalid generation settings");
    const int length = std::min(completion, S + 1 - P);
    if (length < 1) fail(MM_INVALID_ARGUMENT, "GRPO prompt leaves no room for a response");
    if (P + length - 1 > c.maxS) fail(MM_INVALID_ARGUMENT, "Decode requires available context");
    for (long long i = 0; i < static_cast<long long>(n) * P; ++i)
        if (prompts[i] >= c.V) fail(MM_INVALID_ARGUMENT, "Input token exceeds vocabulary");
    const int Sc = P + length - 1;
    ensure_decode(cx, n, Sc, completion);
    struct InUse {  // the cache is written from the prefill on: no workspace request may free it
        bool& f;
        explicit InUse(bool& x) : f(x) { f = true; }
        ~InUse() { f = false; }
    } in_use(cx.dec.in_use);
    cx.serving = false;  // the decode state now holds the rollout batch
    DecodeState& d = cx.dec;
    uint16_t* d_prompts = static_cast<uint16_t*>(cx.stage.get(static_cast<size_t>(n) * P * 2));
    MM_CUDA_CHECK(cudaMemcpyAsync(d_prompts, prompts, static_cast<size_t>(n) * P * 2, cudaMemcpyHostToDevice, cx.stream));
    MM_CUDA_CHECK(cudaMemcpyAsync(d.seeds, seeds, static_cast<size_t>(n) * 8, cudaMemcpyHostToDevice, cx.stream));
    {
        PhaseTimer t(cx, kPhPrefill);
        prefill_rows(cx, d_prompts, n, P, chunk_tokens(cx));
    }
    MM_CUDA_CHECK(cudaMemsetAsync(d.step, 0, sizeof(int), cx.stream));
    {
        PhaseTimer t(cx, kPhSample);
        launch_sample(cx, d.logits, n, temperature, d.seeds, nullptr, 0, nullptr, d.out_tok, completion, d.step);
    }
    // Steps 1..length-1: the first runs eagerly (it also initialises every kernel and
    // tensor map it uses); the rest replay one captured graph of a whole step, whose
    // arguments are all constant because the step index lives in device memory.
    for (int k = 1; k < length; ++k) {
        cx.dec_len = P + k - 1;  // cache entries before this step's write
        PhaseTimer t(cx, kPhDecode);
        if (k == 1 || !decode_graphs_enabled()) {
            decode_sample_step(cx, completion, temperature);
            continue;
        }
        if (!d.graph || d.graph_completion != completion || d.graph_temperature != temperature) {
            d.drop_graph();
            const bool prof = cx.profiling;
            const long long before = cx.launches;
            cx.profiling = false;
            cudaGraph_t g = nullptr;
            MM_CUDA_CHECK(cudaStreamBeginCapture(cx.stream, cudaStreamCaptureModeThreadLocal));
            try {
                decode_sample_step(cx, completion, temperature);
            } catch (...) {
                cudaStreamEndCapture(cx.stream, &g);  // leave the stream usable
                if (g) cudaGraphDestroy(g);
                cx.profiling = prof;
                throw;
            }
            const cudaError_t e = cudaStreamEndCapture(cx.stream, &g);
            cx.profiling = prof;
            if (e != cudaSuccess || !g) fail(MM_GPU_ERROR, std::string("decode graph capture: ") + cudaGetErrorString(e));
            const cudaError_t ie = cudaGraphInstantiate(&d.graph, g, 0);
            cudaGraphDestroy(g);
            if (ie != cudaSuccess) fail(MM_GPU_ERROR, std::string("decode graph instantiate: ") + cudaGetErrorString(ie));
            d.graph_completion = completion;
            d.graph_temperature = temperature;
            d.graph_launches = cx.launches - before;
            cx.launches = before;
        }
        MM_CUDA_CHECK(cudaGraphLaunch(d.graph, cx.stream));
        cx.launches += d.graph_launches;
    }
    std::vector<uint16_t> toks(static_cast<size_t>(n) * completion);
    MM_CUDA_CHECK(cudaMemcpyAsync(toks.data(), d.out_tok, toks.size() * 2, cudaMemcpyDeviceToHost, cx.stream));
    MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
    // The graph holds raw pointers (split-K staging, derived weights) that later calls may
    // reallocate, so it lives for one rollout only.
    d.drop_graph();
    check_device(cx, "rollout");
    for (int i = 0; i < n; ++i) {
        int len = length;
        for (int k = 0; k < length; ++k)
            if (toks[static_cast<size_t>(i) * completion + k] == eos) {
                len = k + 1;
                break;
            }
        out_len[i] = len;
        for (int k = 0; k < completion; ++k)
            out_tokens[static_cast<size_t>(i) * completion + k] = k < len ? toks[static_cast<size_t>(i) * completion + k] : eos;
    }
    if (!out_old_lp) return;
    // completion_batch (trainer.cpp:386-408) then the old-policy log-probabilities.
    std::vector<uint16_t> inp(static_cast<size_t>(n) * S, pad), tgt(static_cast<size_t>(n) * S, pad);
    std::vector<float> msk(static_cast<size_t>(n) * S, 0.f);
    for (int i = 0; i < n; ++i) {
        std::vector<uint16_t> ids(prompts + static_cast<size_t>(i) * P, prompts + static_cast<size_t>(i) * P + P);
        ids.insert(ids.end(), out_tokens + static_cast<size_t>(i) * completion,
                   out_tokens + static_cast<size_t>(i) * completion + out_len[i]);
        for (size_t t = 0; t + 1 < ids.size(); ++t) {
            inp[static_cast<size_t>(i) * S + t] = ids[t];
            tgt[static_cast<size_t>(i) * S + t] = ids[t + 1];
            msk[static_cast<size_t>(i) * S + t] = t + 1 >= static_cast<size_t>(P) ? 1.f : 0.f;
        }
    }
    log_probs_host(cx, inp.data(), tgt.data(), n, S, out_old_lp);
    if (out_input) std::memcpy(out_input, inp.data(), inp.size() * 2);
    if (out_target) std::memcpy(out_target, tgt.data(), tgt.size() * 2);
    if (out_mask) std::memcpy(out_mask, msk.data(), msk.size() * 4);
}

} // namespace mm
