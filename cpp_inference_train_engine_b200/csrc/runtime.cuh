// Host runtime of the backend: device context, parameter arenas, workspaces, the GEMM
// launcher and the launch helpers shared by the passes (passes.cu) and the C ABI (api.cu).
#pragma once
#include <cudaTypedefs.h>

#include <atomic>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "attention.cuh"
#include "common.cuh"
#include "flash_mma.cuh"
#include "gemm_tc.cuh"
#include "kernels_vec.cuh"
#include "optim.cuh"
#include "vocab_grpo.cuh"

#include "../../include/mm_cuda.h"

namespace mm {

// Error carried up to the C ABI as 1 + ErrorCode with a message.
struct Failure : std::runtime_error {
    int code;
    Failure(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};
[[noreturn]] inline void fail(int code, const std::string& m) { throw Failure(code, m); }

#define MM_CUDA_CHECK(x)                                                                  \
    do {                                                                                  \
        cudaError_t e_ = (x);                                                             \
        if (e_ != cudaSuccess)                                                            \
            ::mm::fail(e_ == cudaErrorMemoryAllocation ? MM_OUT_OF_MEMORY : MM_GPU_ERROR, \
                       std::string(#x) + ": " + cudaGetErrorString(e_));                  \
    } while (0)

inline long long round_up(long long x, long long a) { return (x + a - 1) / a * a; }

struct Dims {
    int V, maxS, L, d, H, nope, rope, dv, qr, kvr, dff;
    float eps, theta;
    int qk() const { return nope + rope; }
    int kvw() const { return kvr + rope; }
    int aw() const { return H * dv; }
};

// One device allocation with bump sub-allocation (256-byte aligned pieces).
class Arena {
  public:
    ~Arena() { release(); }
    void reserve(size_t bytes) {
        release();
        if (bytes == 0) return;
        MM_CUDA_CHECK(cudaMalloc(&base_, bytes));
        cap_ = bytes;
        used_ = 0;
    }
    template <class T> T* take(long long count) {
        size_t off = static_cast<size_t>(round_up(static_cast<long long>(used_), 256));
        size_t bytes = static_cast<size_t>(count) * sizeof(T);
        if (off + bytes > cap_) fail(MM_OUT_OF_MEMORY, "workspace arena exhausted");
        used_ = off + bytes;
        return reinterpret_cast<T*>(static_cast<char*>(base_) + off);
    }
    void reset() { used_ = 0; }
    // Whether `bytes` more fit on the device now (with 1 GB to spare), counting this arena's
    // own block as free when it is about to be replaced.
    bool fits(size_t bytes) const {
        size_t fr = 0, total = 0;
        if (cudaMemGetInfo(&fr, &total) != cudaSuccess) return true;
        return bytes + (1ull << 30) <= fr + cap_;
    }
    void release() {
        if (base_) cudaFree(base_);
        base_ = nullptr;
        cap_ = used_ = 0;
    }
    size_t capacity() const { return cap_; }

  private:
    void* base_ = nullptr;
    size_t cap_ = 0, used_ = 0;
};

// Byte counter used to size an Arena before allocating it: same take() sequence.
class Sizer {
  public:
    template <class T> T* take(long long count) {
        used_ = static_cast<size_t>(round_up(static_cast<long long>(used_), 256)) + static_cast<size_t>(count) * sizeof(T);
        return nullptr;
    }
    size_t used() const { return used_; }

  private:
    size_t used_ = 0;
};

// Reusable device staging buffer for host inputs of one call.
struct Staging {
    Arena a;
    size_t cap = 0;
    void* get(size_t bytes) {
        if (bytes > cap) {
            a.release();
            a.reserve(bytes + 1024);
            cap = bytes;
        }
        a.reset();
        return a.take<char>(static_cast<long long>(bytes));
    }
};

enum LayerParam { kAttnNorm, kWdq, kQNorm, kWuq, kWdkv, kKvNorm, kWuk, kWuv, kWo, kFfnNorm, kWgate, kWup, kWdown, kLayerParams };

// Per-layer activations of a teacher-forced pass (the reference's LayerTape,
// include/mini_mla/model.hpp:31-34, in the mixed-precision layout of this backend).
struct LayerBuf {
    float* x_in;      // [T][d]     layer input (residual stream)
    __half* h;        // [T][ld16(d)]
    float* raw_cq;    // [T][qr]
    __half* cq;       // [T][ld16(qr)]
    __half* q;        // [T][H*qk]  rotated
    float* kvp;       // [T][kvw]   raw latent | raw rope key
    __half* ckv;      // [T][ld16(kvr)]
    float* k_rope;    // [T][rope]  rotated
    __half* k;        // [T][H*qk]
    __half* v;        // [T][H*dv]
    __half* ao;       // [T][H*dv]
    float* lse;       // [T][H]
    float* res;       // [T][d]
    __half* h2;       // [T][ld16(d)]
    __half* gate;     // [T][ld16(dff)]
    __half* up;       // [T][ld16(dff)]
    __half* gated;    // [T][ld16(dff)]
};

struct Workspace {
    int T = 0;          // token capacity
    bool tape = false;  // one LayerBuf per layer (training) or one shared
    std::vector<LayerBuf> layers;
    float* x_out;       // [T][d] output of the last layer
    float* hf;          // [T][d] final norm output
    __half* h3;         // [T][ld16(3d)]
    float* logits;      // [T][V]
    float2* lse_part;   // [2 * ceil(V / 64)][T] per tile and epilogue half (max, sum exp)
    float* tgt_logit;   // [T]
    float* lp;          // [T]
    float* lse_v;       // [T]
    uint16_t* tokens;   // [T]
    uint16_t* targets;  // [T]
    float* mask;        // [T]
    float* coef;        // [T]
    float* old_lp;      // [T]
    float* ref_lp;      // [T]
    // scratch
    float* knope;       // [T][H*nope]
    // backward scratch (tape only)
    __half* dgated16;  // [T][ld16(dff)]
    float *dy, *dh2, *dres, *dao, *dk, *drope, *drope2, *dckv, *dkvraw, *dh, *dcq, *Dd;
    __half *dy16, *dg16, *du16, *dres16, *dq16, *dkn16, *dv16, *dkvp16, *draw16, *g16, *dao16;
    float* norm_part;   // [kNormBlocks][max(d, qr, kv_rank)] RMSNorm weight-gradient partials
    // Rows whose log-probabilities the update uses (mask != 0): with 0 < nsel < T the
    // vocabulary head and its backward run on these rows only (h3, logits, lse partials and
    // the vocabulary gradient hold nsel compacted rows). nsel < 0: every row.
    int nsel = -1;
    int* sel;            // [T] row of compacted row i
    int* sel_counts;     // [ceil(T / 1024)] selected rows per 1024-row block
    uint16_t* sel_tgt;   // [T] target of compacted row i
    float *sel_lp, *sel_lse, *sel_coef;  // [T] per compacted row
};

// Blocks of the RMSNorm backward (2 per SM): one weight-gradient partial row each.
constexpr int kNormBlocks = 296;

struct DecodeState {
    int B = 0, Sc = 0;  // rows, cache positions per row
    __half* cache = nullptr;  // [L][B][Sc][kvw]
    int* pos = nullptr;       // [B] next position to write
    float* x;                 // [B][d]
    __half* h16;              // [B][ld16(d)]
    float* y;                 // [B][qr + kvw]
    __half* cq16;             // [B][ld16(qr)]
    __half* lat16;            // [B][ld16(kvr)]
    float* k_rope;            // [B][rope]
    float* qf;                // [B][H*kvw]
    float* qf2;               // [B][H*kvw]
    __half* ctx16;            // [B][H*kvr]
    float* res;               // [B][d]
    __half* h2;               // [B][ld16(d)]
    __half* gu;               // [B][ld16(2 dff)]
    __half* gated;            // [B][ld16(dff)]
    float* hf;                // [B][d]
    __half* h3;               // [B][ld16(3d)]
    float* logits;            // [B][V]
    uint16_t* tok;            // [B]
    uint64_t* seeds;          // [B]
    int* draw;                // [B]
    uint16_t* out_tok;        // [B][max_new]
    float* part;              // [B][splits][H][kv_rank + 2] decode-attention partials
    int* step;                // device step counter of the rollout loop
    int* active;              // [B] serving: 1 for slots holding a request
    // fused decode step (decode_mk_kernel): split-K partials [6][B][d], per-row attention
    // arrival counters [B] (zero between uses) and the grid barrier's arrival counter
    float* mk_qs = nullptr;   // [B] the fused step's query row factor (q-latent RMSNorm scale)
    float* mk_part = nullptr;
    int* mk_cnt = nullptr;
    unsigned* mk_bar = nullptr;
    unsigned long long* mk_trace = nullptr;  // [kMkTraceSlots] phase timestamps when tracing
    bool mk_trace_on = false;
    int max_new = 0;
    Arena arena;
    // set for the whole of a rollout: a workspace request inside it never takes the arena
    bool in_use = false;
    // one captured rollout decode step (decode_sample_step), valid for the buffers above
    cudaGraphExec_t graph = nullptr;
    long long graph_launches = 0;  // kernels per replay
    int graph_completion = 0;
    float graph_temperature = 0.f;
    void drop_graph() {
        if (graph) cudaGraphExecDestroy(graph);
        graph = nullptr;
    }
    ~DecodeState() { drop_graph(); }
};

struct PrepLayer {
    __half *Wa, *Wq, *Wo, *Wgu;
    int lda, ldq, ldo, ldgu;
    // the fused decode step's query weights W_dq . diag(g_q) . Wq [d][ldf] (its shape only)
    __half* Wf = nullptr;
    int ldf = 0;
};

// Device-time accounting while profiling is on: event pairs recorded on the context's
// stream around each phase and around every launch of a kernel class, resolved only when
// read, so the timed region gains no host synchronisation. Each kernel-class launch also
// adds its algorithmic work (bytes moved or flops) as computed from the launch shape.
enum Phase { kPhPrefill, kPhDecode, kPhSample, kPhLogprob, kPhBackward, kPhAdamw, kPhAllreduce, kPhPrep };
enum KernelClass { kKGemm = 8, kKDecodeAttn, kKFlashFwd, kKFlashBwd, kKSample, kKLogsoftmax, kKAdamw, kKOther };
constexpr int kProfTags = 16;
struct Profile {
    double ms[kProfTags] = {0};
    long long calls[kProfTags] = {0};
    double work[kProfTags] = {0};  // flops (GEMM, attention) or bytes (the rest)
};
struct ShapeStat {
    long long calls = 0;
    double ms = 0, flops = 0;
};
struct EventLog {
    std::vector<cudaEvent_t> free_events;
    std::vector<std::tuple<int, cudaEvent_t, cudaEvent_t>> pending;
    // GEMM intervals by launch shape: (shape key, start, end)
    std::vector<std::tuple<std::string, cudaEvent_t, cudaEvent_t>> pending_shapes;
    std::map<std::string, ShapeStat> shapes;
    cudaEvent_t take() {
        if (free_events.empty()) {
            cudaEvent_t e;
            cudaEventCreate(&e);
            return e;
        }
        cudaEvent_t e = free_events.back();
        free_events.pop_back();
        return e;
    }
};

class Context {
  public:
    Dims c{};
    int device = 0;
    bool trainable = false;
    mm_adamw_desc opt{0.9f, 0.95f, 1e-8f, 0.1f, 1.0f};
    uint64_t steps = 0;
    cudaStream_t stream = nullptr;
    float* wq32 = nullptr;  // [qr][H * kvw] scratch of the query-weight fold (fused decode shape only)
    std::string last_error;
    bool unusable = false;
    long long launches = 0;

    // parameters
    std::vector<ParamDesc> params;      // registry order
    std::vector<long long> flat_off;    // offsets in the caller's flat array
    long long P = 0, P_dev = 0;         // logical and padded element counts
    long long shadow_elems = 0;
    ParamDesc* d_params = nullptr;
    Arena weights;                      // master, grad, m, v, shadow, rope tables, prep
    float *w = nullptr, *g = nullptr, *m = nullptr, *v = nullptr;
    __half* shadow = nullptr;
    float *cos_t = nullptr, *sin_t = nullptr;
    std::vector<PrepLayer> prep;

    // scalars on device
    int* d_err = nullptr;
    double* d_partial = nullptr;  // AdamW norm partials
    int n_partial = 0;
    double* d_norm = nullptr;
    float* d_gs = nullptr;
    int* d_nonfinite = nullptr;
    int* d_nonfinite_out = nullptr;
    GrpoSums* d_sums = nullptr;
    float* d_scale = nullptr;     // [2] gradient scale, inverse
    int* d_any = nullptr;
    float* d_one = nullptr;       // constant 1.0f
    Arena scalars;

    Workspace ws;
    Arena ws_arena;
    int chunk_cap = 0;  // tokens per chunk this model's workspace allows (chunk_tokens)
    Staging stage;
    Staging splitk;  // split-K partials of the GEMM
    Staging emb_acc; // fixed-point embedding-gather gradient [V][d] (+ max |dy|, non-finite flag)
    Staging sums_part;  // per-block GRPO loss/kl partials (double2)
    DecodeState dec;
    int dec_len = 0;  // positions filled in the decode session (0: no session)
    // continuous-batching serving session over dec (mm_cuda_serve_*): next position of
    // each slot on the host, -1 for a free slot
    bool serving = false;
    // false while this context's products run beside another stream's (the frozen
    // reference's forward overlapping the policy's backward): CTA-pair products need two free
    // SMs of one TPC at once and stall behind the other stream's CTAs, so they stay single
    bool pair_ok = true;
    std::vector<int> serve_pos;

    // NCCL
    void* nccl_comm = nullptr;
    bool nccl_nonblocking = false;  // communicator created with blocking = 0
    int rank = 0, world = 1;

    // timing
    bool profiling = false;
    Profile prof;
    EventLog evlog;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;

    // Opens a timed interval for `tag` (no-op unless profiling); close with prof_end.
    cudaEvent_t prof_begin() {
        if (!profiling) return nullptr;
        cudaEvent_t e = evlog.take();
        cudaEventRecord(e, stream);
        return e;
    }
    void prof_end(int tag, cudaEvent_t start, double work = 0) {
        if (!start) return;
        cudaEvent_t e = evlog.take();
        cudaEventRecord(e, stream);
        evlog.pending.emplace_back(tag, start, e);
        prof.work[tag] += work;
        prof.calls[tag] += 1;
    }
    // Also files the interval opened by `start` (owned by the class log) under a GEMM shape;
    // the shape log records its own end event.
    void prof_shape(const std::string& key, cudaEvent_t start, double flops) {
        if (!start) return;
        cudaEvent_t b = evlog.take();
        cudaEventRecord(b, stream);
        evlog.pending_shapes.emplace_back(key, start, b);
        evlog.shapes[key].calls += 1;
        evlog.shapes[key].flops += flops;
    }
    // Waits for the stream and folds every pending interval into prof.ms.
    void prof_resolve() {
        if (evlog.pending.empty() && evlog.pending_shapes.empty()) return;
        cudaStreamSynchronize(stream);
        for (auto& [key, a, b] : evlog.pending_shapes) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, a, b);
            evlog.shapes[key].ms += ms;
            evlog.free_events.push_back(b);
        }
        evlog.pending_shapes.clear();
        for (auto& [tag, a, b] : evlog.pending) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, a, b);
            prof.ms[tag] += ms;
            evlog.free_events.push_back(a);
            evlog.free_events.push_back(b);
        }
        evlog.pending.clear();
    }

    int d16(int n) const { return static_cast<int>(round_up(n, 8)); }
    int param_index(int l, int which) const { return 2 + l * kLayerParams + which; }
    float* W(int l, int which) const { return w + params[param_index(l, which)].off; }
    float* G(int l, int which) const { return g + params[param_index(l, which)].off; }
    __half* S(int l, int which) const { return shadow + params[param_index(l, which)].shadow_off; }
    int SL(int l, int which) const { return params[param_index(l, which)].shadow_ld; }
    float* E() const { return w + params[0].off; }
    float* GE() const { return g + params[0].off; }
    __half* E3() const { return shadow + params[0].shadow_off; }
    int E3L() const { return params[0].shadow_ld; }
    float* FinalNorm() const { return w + params[1].off; }
    float* GFinalNorm() const { return g + params[1].off; }
};

// ------------------------------------------------------------------ tensor maps
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        MM_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !p) fail(MM_GPU_ERROR, "cuTensorMapEncodeTiled unavailable");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2-D fp16/bf16 tensor map, 128-byte swizzle, zero fill out of bounds. Cached by
// (address, shape, pitch, box): buffers are long-lived, so the encode runs once per view.
enum MapType : int { kMapF16 = 0, kMapBF16 = 1, kMapF32 = 2 };

inline const CUtensorMap& tensor_map_t(const void* base, int type, long long dim0, long long dim1,
                                       long long pitch_elems, int box0, int box1) {
    using Key = std::tuple<const void*, int, long long, long long, long long, int, int>;
    static std::map<Key, CUtensorMap> cache;
    Key k{base, type, dim0, dim1, pitch_elems, box0, box1};
    auto it = cache.find(k);
    if (it != cache.end()) return it->second;
    const int esize = type == kMapF32 ? 4 : 2;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (pitch_elems * esize) % 16)
        fail(MM_INVALID_ARGUMENT, "tensor map needs 16-byte aligned base and pitch");
    CUtensorMap map;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(dim0), static_cast<cuuint64_t>(dim1)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch_elems * esize)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(box0), static_cast<cuuint32_t>(box1)};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = type == kMapF32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : type == kMapBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = tensor_map_encoder()(&map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(MM_GPU_ERROR, "cuTensorMapEncodeTiled failed: " + std::to_string(static_cast<int>(r)));
    return cache.emplace(k, map).first->second;
}
inline const CUtensorMap& tensor_map(const void* base, bool bf16, long long dim0, long long dim1,
                                     long long pitch_elems, int box0, int box1) {
    return tensor_map_t(base, bf16 ? kMapBF16 : kMapF16, dim0, dim1, pitch_elems, box0, box1);
}

// ------------------------------------------------------------------ GEMM launcher
// Operand views. K-major A: [M][K] rows; MN-major A: [K][M] rows. K-major B: [N][K];
// MN-major B: [K][N]. `ld` is the row pitch in elements (a multiple of 8).
struct Opnd {
    const void* p;
    long long ld;
    bool mn;
};

struct GemmOutSpec {
    void* out;
    long long ldc;
    int kind;
    const float* residual = nullptr;
    long long ldr = 0;
    float alpha = 1.f;
    const float* alpha_ptr = nullptr;
    // row log-sum-exp partials of an fp32 product (GemmArgs::lse_part); gemm() returns the
    // tile width, so the partials are [2 * ceil(N / width)][M]
    float2* lse_part = nullptr;
    const uint16_t* targets = nullptr;
    float* tgt_logit = nullptr;
    bool no_store = false;
    // SwiGLU output (GemmArgs::glu_n): N = output columns, B holds [gate | up] with the up
    // half glu_n columns after the gate half; fp16 output, B MN-major
    int glu_n = 0;
    // RoPE on an fp16 output (GemmArgs::rope_cos): position = row % rope_seq
    const float* rope_cos = nullptr;
    const float* rope_sin = nullptr;
    int rope_seq = 1, rope_period = 1, rope_begin = 0, rope_len = 0;
    // with glu_n: also store the fp16 pre-activations, gate at pre_gate[r][c] and up at
    // pre_gate[r][glu_n + c] (row pitch pre_ld)
    __half* pre_gate = nullptr;
    long long pre_ld = 0;
    // SwiGLU backward of dH (fp16 product, N = d_ff): out receives d gate and dglu_up d up
    // (both row pitch ldc), from gate / up at dglu_gu[r][c] / dglu_gu[r][N + c] (pitch dglu_ld)
    const __half* dglu_gu = nullptr;
    long long dglu_ld = 0;
    __half* dglu_up = nullptr;
    // split A (GemmArgs::b_k_wrap, b_k3): two-term, B (MN-major) has b_k_wrap rows and
    // K = 2 b_k_wrap; three-term, B holds [hi; lo] of b_k_wrap rows each and K = 3 b_k_wrap
    int b_k_wrap = 0;
    bool b_k3 = false;
    // weighted-NLL gradient of the recomputed logits (GemmArgs::vg_lse): fp16 product, per row
    // log-sum-exp, coefficient and target (targets), device scale vg_scale[0]
    const float* vg_lse = nullptr;
    const float* vg_coef = nullptr;
    const float* vg_scale = nullptr;
};

inline int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// Programmatic dependent launch for every kernel (MM_PDL=0 turns it off).
inline bool pdl_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("MM_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Launches `kernel` on stream s with programmatic stream serialization (the kernel enters
// through MM_PDL_ENTRY, so it touches no memory before its predecessor completes).
template <typename... KArgs, typename... Args>
inline void launch_k(cudaStream_t s, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    MM_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) for a kernel, once per device.
template <auto Kernel>
inline void set_dynamic_smem(int bytes) {
    static std::atomic<unsigned long long> done{0};
    int dev = 0;
    MM_CUDA_CHECK(cudaGetDevice(&dev));
    const unsigned long long bit = 1ull << (dev & 63);
    if (done.load() & bit) return;
    MM_CUDA_CHECK(cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.fetch_or(bit);
}

template <int BN, int STAGES, int EPI = kEpiPlain>
inline void launch_gemm_bn(Context& cx, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                           const CUtensorMap& td, const CUtensorMap& te, const GemmArgs& ga) {
    using C = GemmCfg<BN, STAGES>;
    set_dynamic_smem<gemm_tc_kernel<BN, STAGES, EPI>>(C::SMEM);
    const long long num_k = (ga.K + kGemmBK - 1) / kGemmBK;
    const long long per = ga.k_tiles_per_split > 0 ? ga.k_tiles_per_split : num_k;
    const int tw = ga.glu_n ? BN / 2 : BN;
    const long long tiles = static_cast<long long>((ga.N + tw - 1) / tw) * ((ga.M + kGemmBM - 1) / kGemmBM) *
                            ((num_k + per - 1) / per);
    // resident CTAs per SM: two TMEM accumulators of BN columns each out of 512, and smem
    const int per_sm = std::max(1, std::min(512 / (2 * BN), (227 * 1024) / C::SMEM));
    dim3 grid(static_cast<unsigned>(std::min<long long>(tiles, static_cast<long long>(sm_count()) * per_sm)));
    cudaEvent_t t0 = cx.prof_begin();
    launch_k(cx.stream, gemm_tc_kernel<BN, STAGES, EPI>, grid, dim3(C::THREADS), C::SMEM, ta, tb, tc, td, te, ga);
    const double flops = 2.0 * ga.M * static_cast<double>(ga.N) * ga.K;
    if (t0) {
        char key[96];
        std::snprintf(key, sizeof key, "M%d N%d K%d a%s b%s bn%d out%d", ga.M, ga.N, ga.K, ga.a_mn ? "mn" : "k",
                      ga.b_mn ? "mn" : "k", BN, ga.out_kind);
        cx.prof_shape(key, t0, flops);
    }
    cx.prof_end(kKGemm, t0, flops);
    ++cx.launches;
}

// MM_GEMM_PAIR=0 keeps every product on the single-CTA kernel (for comparison).
inline bool pair_gemm_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("MM_GEMM_PAIR");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Smallest M (rows) a product needs to run on CTA pairs (the 2,048-row decode step's
// vocabulary head and SwiGLU products gain ~1% of the step); MM_GEMM_PAIR_MIN_M overrides it.
inline int pair_gemm_min_m() {
    static const int m = [] {
        const char* e = std::getenv("MM_GEMM_PAIR_MIN_M");
        const int v = e ? std::atoi(e) : 0;
        return v > 0 ? v : 2048;
    }();
    return m;
}

// CTA pairs of gemm_tc_pair_kernel that can be resident at once on this device (0 when the
// cluster launch does not fit).
inline int pair_gemm_slots() {
    static int slots = -1;
    if (slots < 0) {
        set_dynamic_smem<gemm_tc_pair_kernel<kEpiPlain>>(PairCfg::SMEM);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * 74);
        cfg.blockDim = dim3(PairCfg::THREADS);
        cfg.dynamicSmemBytes = PairCfg::SMEM;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_pair_kernel<kEpiPlain>, &cfg) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        slots = n;
    }
    return slots;
}

// The CTA-pair product: one persistent cluster per resident pair slot, 256-row tiles.
template <int EPI>
inline void launch_gemm_pair(Context& cx, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                             const CUtensorMap& td, const CUtensorMap& te, const GemmArgs& ga) {
    set_dynamic_smem<gemm_tc_pair_kernel<EPI>>(PairCfg::SMEM);
    const int tw = ga.glu_n ? 128 : 256;
    const long long tiles = static_cast<long long>((ga.N + tw - 1) / tw) * ((ga.M + 255) / 256);
    dim3 grid(static_cast<unsigned>(2 * std::min<long long>(tiles, pair_gemm_slots())));
    cudaEvent_t t0 = cx.prof_begin();
    launch_k(cx.stream, gemm_tc_pair_kernel<EPI>, grid, dim3(PairCfg::THREADS), PairCfg::SMEM, ta, tb, tc, td, te, ga);
    const double flops = 2.0 * ga.M * static_cast<double>(ga.N) * ga.K;
    if (t0) {
        char key[96];
        std::snprintf(key, sizeof key, "M%d N%d K%d a%s b%s pair out%d", ga.M, ga.N, ga.K, ga.a_mn ? "mn" : "k",
                      ga.b_mn ? "mn" : "k", ga.out_kind);
        cx.prof_shape(key, t0, flops);
    }
    cx.prof_end(kKGemm, t0, flops);
    ++cx.launches;
}

// D[M,N] = alpha * A * B (+ residual | += D). bf16 selects bf16 operands.
int gemm(Context& cx, int M, int N, int K, Opnd A, Opnd B, const GemmOutSpec& o, bool bf16 = false);

// ------------------------------------------------------------------ small launch helpers
inline unsigned blocks_for(long long n, int threads) {
    return static_cast<unsigned>((n + threads - 1) / threads);
}

} // namespace mm
