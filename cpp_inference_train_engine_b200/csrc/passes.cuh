// Teacher-forced forward and backward passes over a chunk of whole sequences
// (Model::forward / Model::backward, src/model/model.cpp:76-245), tensor-core GEMMs with
// fp16 operands and fp32 accumulation, fp32 residual stream and norms, an FP32-accurate
// tied vocabulary head.
#pragma once
#include "setup.cuh"
#include "flash_tc.cuh"

namespace mm {

// Writes the normalised latent and rotated rope key of token rows into the decode cache:
// row t -> sequence row0 + t / S at position (pos ? pos[t / S] : 0) + t % S.
__global__ void cache_write_kernel(const __half* __restrict__ ckv, long long ldckv,
                                   const float* __restrict__ k_rope, int T, int S,
                                   const int* __restrict__ pos, int row0, __half* __restrict__ cache,
                                   int Sc, int kvr, int rope) {
    MM_PDL_ENTRY();
    const int kvw = kvr + rope;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(T) * kvw) return;
    const int t = static_cast<int>(idx / kvw), j = static_cast<int>(idx % kvw);
    const int seq = t / S;
    const int p = (pos ? pos[seq] : 0) + t % S;
    if (p >= Sc) return;
    __half* dst = cache + (static_cast<long long>(row0 + seq) * Sc + p) * kvw;
    dst[j] = j < kvr ? ckv[t * ldckv + j] : __float2half_rn(k_rope[t * rope + (j - kvr)]);
}

// After the [W_dq | W_dkv] product, per token row t of y = [raw_cq (qr) | raw latent (kvr)
// | raw rope key (rope)]: cq16 = RMSNorm(raw_cq) (fp16); the normalised latent (fp16) into
// ckv16 and/or the cache; the rope key rotated to its position into k_rope32 (fp32) and/or
// the cache. Row t belongs to sequence t / S at position (pos_base ? pos_base[t / S] : 0) +
// t % S; its cache row is row0 + t / S (positions >= Sc are not stored). This is the
// rmsnorm_kernel / rope_key_kernel / cache_write_kernel sequence in one pass with the same
// float expressions. One warp per row; qr, kvr, rope multiples of 4, 16-byte aligned y rows,
// qr + kvr + rope <= 512.
__global__ void latent_kernel(const float* __restrict__ y, long long ldy, int qr, int kvr, int rope,
                              const float* __restrict__ w_q, const float* __restrict__ w_kv, float eps, int T, int S,
                              const int* __restrict__ pos_base, int row0, const float* __restrict__ cos_t,
                              const float* __restrict__ sin_t, __half* __restrict__ cq16, long long ld_cq,
                              __half* __restrict__ ckv16, long long ld_ckv, float* __restrict__ k_rope32,
                              __half* __restrict__ cache, int Sc) {
    MM_PDL_ENTRY();
    const int t = warp_row(), lane = threadIdx.x & 31;
    if (t >= T) return;
    const float* row = y + t * ldy;
    const int n4 = (qr + kvr + rope) >> 2;
    constexpr int MAXV = 4;  // up to 512 values per row
    float4 v[MAXV];
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int k = 0; k < MAXV; ++k) {
        const int q = k * 32 + lane;
        if (q < n4) {
            v[k] = *reinterpret_cast<const float4*>(row + 4 * q);
            const float s = v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
            if (4 * q < qr) sq += s;
            else if (4 * q < qr + kvr) sk += s;
        }
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    const float iq = 1.0f / sqrtf(sq / static_cast<float>(qr) + eps);
    const float ik = 1.0f / sqrtf(sk / static_cast<float>(kvr) + eps);
    const int seq = t / S;
    const int p = (pos_base ? pos_base[seq] : 0) + t % S;
    const bool to_cache = cache && p < Sc;
    __half* crow = to_cache ? cache + (static_cast<long long>(row0 + seq) * Sc + p) * (kvr + rope) : nullptr;
    const int half_r = rope / 2;
#pragma unroll
    for (int k = 0; k < MAXV; ++k) {
        const int q = k * 32 + lane, c = 4 * q;
        if (q >= n4) continue;
        float f[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
        if (c < qr) {
            const float4 wv = *reinterpret_cast<const float4*>(w_q + c);
            *reinterpret_cast<uint2*>(cq16 + t * ld_cq + c) =
                pack_h4(f[0] * iq * wv.x, f[1] * iq * wv.y, f[2] * iq * wv.z, f[3] * iq * wv.w);
        } else if (c < qr + kvr) {
            const float4 wv = *reinterpret_cast<const float4*>(w_kv + (c - qr));
            const uint2 h = pack_h4(f[0] * ik * wv.x, f[1] * ik * wv.y, f[2] * ik * wv.z, f[3] * ik * wv.w);
            if (ckv16) *reinterpret_cast<uint2*>(ckv16 + t * ld_ckv + (c - qr)) = h;
            if (to_cache) *reinterpret_cast<uint2*>(crow + (c - qr)) = h;
        } else {
            const int j = c - qr - kvr;  // even: two rotation pairs
#pragma unroll
            for (int e = 0; e < 4; e += 2) {
                const int pair = (j + e) >> 1;
                const float cs = cos_t[p * half_r + pair], sn = sin_t[p * half_r + pair];
                const float a = f[e], bb = f[e + 1];
                f[e] = a * cs - bb * sn;
                f[e + 1] = a * sn + bb * cs;
            }
            if (k_rope32) *reinterpret_cast<float4*>(k_rope32 + t * rope + j) = make_float4(f[0], f[1], f[2], f[3]);
            if (to_cache) *reinterpret_cast<uint2*>(crow + kvr + j) = pack_h4(f[0], f[1], f[2], f[3]);
        }
    }
}

// h3 rows for the vocabulary head from fp32 rows in[t * mul + add].
__global__ void split3_gather_kernel(const float* __restrict__ h, int d, int T, int mul, int add,
                                     __half* __restrict__ h3, long long ld3) {
    MM_PDL_ENTRY();
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(T) * d) return;
    const int t = static_cast<int>(idx / d), j = static_cast<int>(idx % d);
    const float v = h[(static_cast<long long>(t) * mul + add) * d + j];
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(v - __half2float(hi));
    h3[t * ld3 + j] = hi;
    h3[t * ld3 + d + j] = lo;
    h3[t * ld3 + 2 * d + j] = hi;
}

// The vocabulary head's rows of an update, compacted: h3 row i = the three-term split of hf
// row sel[i] ([hi | lo | hi], as split3_gather_v4_kernel) and sel_tgt[i] its target.
// 4 columns per thread (d % 4 == 0, 8-byte aligned h3 rows).
__global__ void split3_select_v4_kernel(const float* __restrict__ h, int d, const int* __restrict__ sel, int n,
                                        const uint16_t* __restrict__ targets, __half* __restrict__ h3, long long ld3,
                                        uint16_t* __restrict__ sel_tgt) {
    MM_PDL_ENTRY();
    const int nv = d >> 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * nv) return;
    const int t = i / nv, j = (i - t * nv) << 2;
    const int src = sel[t];
    if (j == 0) sel_tgt[t] = targets[src];
    const float4 v = *reinterpret_cast<const float4*>(h + static_cast<long long>(src) * d + j);
    const float f[4] = {v.x, v.y, v.z, v.w};
    __half hi[4], lo[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        hi[k] = __float2half_rn(f[k]);
        lo[k] = __float2half_rn(f[k] - __half2float(hi[k]));
    }
    __half* row = h3 + t * ld3;
    const uint2 H = *reinterpret_cast<const uint2*>(hi), L = *reinterpret_cast<const uint2*>(lo);
    *reinterpret_cast<uint2*>(row + j) = H;
    *reinterpret_cast<uint2*>(row + d + j) = L;
    *reinterpret_cast<uint2*>(row + 2 * d + j) = H;
}

// Row selection (mask != 0) in ascending order, in two launches of 1024-row blocks:
// select_count_kernel counts each block's rows, select_write_kernel writes each block's
// selected rows after the rows of the blocks before it.
constexpr int kSelectBlock = 1024;
__global__ void __launch_bounds__(kSelectBlock) select_count_kernel(const float* __restrict__ mask, int T,
                                                                    int* __restrict__ counts) {
    MM_PDL_ENTRY();
    const int t = blockIdx.x * kSelectBlock + threadIdx.x;
    const int c = __syncthreads_count(t < T && mask[t] != 0.f);
    if (threadIdx.x == 0) counts[blockIdx.x] = c;
}
__global__ void __launch_bounds__(kSelectBlock) select_write_kernel(const float* __restrict__ mask, int T,
                                                                    const int* __restrict__ counts,
                                                                    int* __restrict__ sel) {
    MM_PDL_ENTRY();
    __shared__ int part[32], wcnt[32], woff[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int before = 0;  // rows selected by the blocks before this one
    for (int b = threadIdx.x; b < static_cast<int>(blockIdx.x); b += kSelectBlock) before += counts[b];
    before = __reduce_add_sync(0xffffffffu, before);
    const int t = blockIdx.x * kSelectBlock + threadIdx.x;
    const bool f = t < T && mask[t] != 0.f;
    const unsigned bal = __ballot_sync(0xffffffffu, f);
    if (lane == 0) {
        part[warp] = before;
        wcnt[warp] = __popc(bal);
    }
    __syncthreads();
    if (warp == 0) {
        const int base = __reduce_add_sync(0xffffffffu, part[lane]);
        int c = wcnt[lane], x = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        woff[lane] = base + x - c;  // exclusive prefix of the warps' counts
    }
    __syncthreads();
    if (f) sel[woff[warp] + __popc(bal & ((1u << lane) - 1u))] = t;
}

// lp / lse of compacted row i to row sel[i] (the other rows were cleared).
__global__ void scatter_lp_kernel(const int* __restrict__ sel, int n, const float* __restrict__ lp_c,
                                  const float* __restrict__ lse_c, float* __restrict__ lp, float* __restrict__ lse) {
    MM_PDL_ENTRY();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    lp[sel[i]] = lp_c[i];
    lse[sel[i]] = lse_c[i];
}

// coef of row sel[i] into compacted row i.
__global__ void gather_coef_kernel(const int* __restrict__ sel, int n, const float* __restrict__ coef,
                                   float* __restrict__ coef_c) {
    MM_PDL_ENTRY();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) coef_c[i] = coef[sel[i]];
}

// fp32 rows [n][d] to rows sel[i] of a [T][d] array whose other rows were cleared; 4 columns
// per thread (d % 4 == 0, 16-byte aligned rows).
__global__ void scatter_rows_v4_kernel(const float* __restrict__ src, const int* __restrict__ sel, int n, int d,
                                       float* __restrict__ dst) {
    MM_PDL_ENTRY();
    const int nv = d >> 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * nv) return;
    const int t = i / nv, j = (i - t * nv) << 2;
    *reinterpret_cast<float4*>(dst + static_cast<long long>(sel[t]) * d + j) =
        *reinterpret_cast<const float4*>(src + static_cast<long long>(t) * d + j);
}

// split3_gather_kernel, 4 columns per thread (d % 4 == 0, 8-byte aligned h3 rows).
__global__ void split3_gather_v4_kernel(const float* __restrict__ h, int d, int T, int mul, int add,
                                        __half* __restrict__ h3, long long ld3) {
    MM_PDL_ENTRY();
    const int nv = d >> 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * nv) return;
    const int t = i / nv, j = (i - t * nv) << 2;
    const float4 v = *reinterpret_cast<const float4*>(h + (static_cast<long long>(t) * mul + add) * d + j);
    const float f[4] = {v.x, v.y, v.z, v.w};
    __half hi[4], lo[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        hi[k] = __float2half_rn(f[k]);
        lo[k] = __float2half_rn(f[k] - __half2float(hi[k]));
    }
    __half* row = h3 + t * ld3;
    const uint2 H = *reinterpret_cast<const uint2*>(hi), L = *reinterpret_cast<const uint2*>(lo);
    *reinterpret_cast<uint2*>(row + j) = H;
    *reinterpret_cast<uint2*>(row + d + j) = L;
    *reinterpret_cast<uint2*>(row + 2 * d + j) = H;
}

template <class A> void plan_workspace(Context& cx, A& a, int T, bool tape) {
    Workspace& w = cx.ws;
    const Dims& c = cx.c;
    const long long t = T;
    const int nl = tape ? c.L : 1;
    w.T = T;
    w.tape = tape;
    w.layers.assign(nl, LayerBuf{});
    for (int l = 0; l < nl; ++l) {
        LayerBuf& b = w.layers[l];
        b.x_in = a.template take<float>(t * c.d);
        b.h = a.template take<__half>(t * cx.d16(c.d));
        // [raw_cq | kv_pack] from one product with [W_dq | W_dkv], row pitch qr + kvw
        b.raw_cq = a.template take<float>(t * (c.qr + c.kvw()));
        b.kvp = b.raw_cq ? b.raw_cq + c.qr : nullptr;
        b.cq = a.template take<__half>(t * cx.d16(c.qr));
        b.q = a.template take<__half>(t * c.H * c.qk());
        b.ckv = a.template take<__half>(t * cx.d16(c.kvr));
        b.k_rope = a.template take<float>(t * c.rope);
        b.k = a.template take<__half>(t * c.H * c.qk());
        b.v = a.template take<__half>(t * c.aw());
        b.ao = a.template take<__half>(t * c.aw());
        b.lse = a.template take<float>(t * c.H);
        b.res = a.template take<float>(t * c.d);
        b.h2 = a.template take<__half>(t * 3 * cx.d16(c.d));  // [hi | lo | hi] rows (ffn_terms)
        // [gate | up] from one product with [W_gate | W_up], row pitch ld16(2 d_ff)
        b.gate = a.template take<__half>(t * cx.d16(2 * c.dff));
        b.up = b.gate ? b.gate + c.dff : nullptr;
        b.gated = a.template take<__half>(t * cx.d16(c.dff));
    }
    w.x_out = a.template take<float>(t * c.d);
    w.hf = a.template take<float>(t * c.d);
    w.h3 = a.template take<__half>(t * cx.d16(3 * c.d));
    w.logits = a.template take<float>(t * c.V);
    w.lse_part = a.template take<float2>(t * 2 * ((c.V + 63) / 64));
    w.tgt_logit = a.template take<float>(t);
    w.lp = a.template take<float>(t);
    w.lse_v = a.template take<float>(t);
    w.tokens = a.template take<uint16_t>(t);
    w.targets = a.template take<uint16_t>(t);
    w.mask = a.template take<float>(t);
    w.coef = a.template take<float>(t);
    w.old_lp = a.template take<float>(t);
    w.ref_lp = a.template take<float>(t);
    w.sel = a.template take<int>(t);
    w.sel_counts = a.template take<int>((t + kSelectBlock - 1) / kSelectBlock);
    w.sel_tgt = a.template take<uint16_t>(t);
    w.sel_lp = a.template take<float>(t);
    w.sel_lse = a.template take<float>(t);
    w.sel_coef = a.template take<float>(t);
    w.knope = a.template take<float>(t * c.H * c.nope);
    if (tape) {
        w.dy = a.template take<float>(t * c.d);
        w.dgated16 = a.template take<__half>(t * cx.d16(c.dff));
        w.dh2 = a.template take<float>(t * c.d);
        w.dres = a.template take<float>(t * c.d);
        w.dao = a.template take<float>(t * c.aw());
        w.dk = a.template take<float>(t * c.H * c.qk());
        w.drope = a.template take<float>(t * c.rope);
        w.drope2 = a.template take<float>(t * c.rope);
        w.dckv = a.template take<float>(t * c.kvr);
        w.dkvraw = a.template take<float>(t * c.kvr);
        w.dh = a.template take<float>(t * c.d);
        w.dcq = a.template take<float>(t * c.qr);
        w.Dd = a.template take<float>(t * c.H);
        w.dy16 = a.template take<__half>(t * cx.d16(c.d));
        // [d gate | d up], pitch ld16(2 d_ff)
        w.dg16 = a.template take<__half>(t * cx.d16(2 * c.dff));
        w.du16 = w.dg16 ? w.dg16 + c.dff : nullptr;
        w.dres16 = a.template take<__half>(t * cx.d16(c.d));
        w.dq16 = a.template take<__half>(t * cx.d16(c.H * c.qk()));
        w.dkn16 = a.template take<__half>(t * cx.d16(c.H * c.nope));
        w.dv16 = a.template take<__half>(t * cx.d16(c.aw()));
        // [d raw_cq | d kv_pack], pitch ld16(qr + kvw)
        w.draw16 = a.template take<__half>(t * cx.d16(c.qr + c.kvw()));
        w.dkvp16 = w.draw16 ? w.draw16 + c.qr : nullptr;
        w.g16 = a.template take<__half>(t * c.V);
        w.dao16 = a.template take<__half>(t * c.aw());
        w.norm_part = a.template take<float>(static_cast<long long>(kNormBlocks) * std::max(c.d, std::max(c.qr, c.kvr)));
    }
}

// Ensures the chunk workspace holds T tokens (and a tape when requested).
inline void ensure_workspace(Context& cx, int T, bool tape) {
    if (cx.ws.T >= T && (cx.ws.tape || !tape) && cx.ws_arena.capacity()) return;
    if (tape && !cx.trainable) fail(MM_INVALID_ARGUMENT, "backward needs a trainable context");
    MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
    Sizer sz;
    plan_workspace(cx, sz, T, tape);
    // the rollout's latent cache makes room for a training chunk (tape) when both do not
    // fit: 109 GB of cache for 2,048 rows of the 2,048-context 1.1B model. Never while a
    // rollout or a serving session holds the cache.
    if (tape && !cx.ws_arena.fits(sz.used() + 4096) && !cx.serving && !cx.dec.in_use && cx.dec.arena.capacity()) {
        cx.dec.drop_graph();
        cx.dec.arena.release();
        cx.dec.B = 0;
        cx.dec_len = 0;  // a later decode without a new prefill fails cleanly
    }
    cx.ws_arena.release();
    cx.ws_arena.reserve(sz.used() + 4096);
    plan_workspace(cx, cx.ws_arena, T, tape);
}

#define MM_LAUNCH_CX(ctx, kernel, grid, block, smem, ...)                 \
    do {                                                                 \
        ::mm::launch_k((ctx).stream, kernel, dim3(grid), dim3(block), (smem), __VA_ARGS__); \
        ++(ctx).launches;                                                \
    } while (0)
#define MM_LAUNCH(kernel, grid, block, smem, ...) MM_LAUNCH_CX(cx, kernel, grid, block, smem, __VA_ARGS__)
// Launch recorded under a kernel class with its algorithmic work.
#define MM_LAUNCH_TIMED(tag, work, kernel, grid, block, smem, ...)       \
    do {                                                                 \
        cudaEvent_t t0_ = cx.prof_begin();                               \
        MM_LAUNCH(kernel, grid, block, smem, __VA_ARGS__);               \
        cx.prof_end(tag, t0_, work);                                     \
    } while (0)

inline unsigned warp_rows_grid(int rows) { return blocks_for(static_cast<long long>(rows) * 32, 256); }

// ------------------------------------------------------------------ elementwise dispatch
// Vector kernels (kernels_vec.cuh) when pitches and addresses allow 16-byte accesses.
inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
inline bool al8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }

// Terms of the teacher-forced passes' [W_gate | W_up] product (MM_FFN_EXACT): 3 (default)
// hi(x).hi(W) + lo(x).hi(W) + hi(x).lo(W), 2 without the weights' residual, 1 = plain fp16.
// The FFN's input and weights in fp16 are the largest sources of the teacher-forced
// log-probabilities' deviation from the fp32 reference (about a third of it). Needs d % 64 == 0
// (the weight-row wrap falls on whole 64-wide k-blocks).
inline int ffn_terms(const Context& cx) {
    static const int v = [] {
        const char* e = std::getenv("MM_FFN_EXACT");
        if (!e) return 3;
        const int x = std::atoi(e);
        return x <= 0 ? 1 : std::min(x, 3);
    }();
    return cx.c.d % 64 == 0 ? v : 1;
}

// split16: the fp16 output is the two-term [hi | lo] row (lo = fp16(y - hi) at column n of
// the same row), or with split16 == 2 the three-term [hi | lo | hi] row, so a product over
// K = 2n or 3n against the weights (and their residual) reads y to about 2^-22 relative
// instead of fp16's 2^-11.
inline void launch_rmsnorm(Context& cx, const float* x, long long ldx, const float* w, int T, int n, float* y32,
                           long long ld32, __half* y16, long long ld16, int split16 = 0) {
    const float eps = cx.c.eps;
    const bool vec = n % 4 == 0 && n <= 1024 && ldx % 4 == 0 && al16(x) && al16(w) &&
                     (!y32 || (ld32 % 4 == 0 && al16(y32))) && (!y16 || (ld16 % 4 == 0 && al8(y16)));
    const int sp = split16;
    if (vec && n <= 512)
        MM_LAUNCH(rmsnorm_v4_kernel<4>, warp_rows_grid(T), 256, 0, x, ldx, w, T, n, eps, y32, ld32, y16, ld16,
                  (float*)nullptr, sp);
    else if (vec)
        MM_LAUNCH(rmsnorm_v4_kernel<8>, warp_rows_grid(T), 256, 0, x, ldx, w, T, n, eps, y32, ld32, y16, ld16,
                  (float*)nullptr, sp);
    else
        MM_LAUNCH(rmsnorm_kernel, warp_rows_grid(T), 256, 0, x, ldx, w, T, n, eps, y32, ld32, y16, ld16, (float*)nullptr,
                  sp);
}

// dx = RMSNorm backward (+ add); dw += scale * sum over rows (fixed-order reduction when
// vectorised).
inline void launch_rmsnorm_backward(Context& cx, const float* x, long long ldx, const float* w, const float* dy,
                                    long long lddy, const float* add, long long ldadd, int T, int n, float* dx32,
                                    long long lddx, __half* dx16, long long lddx16, float* dw, const float* scale) {
    const float eps = cx.c.eps;
    const bool vec = n % 4 == 0 && n <= 1024 && cx.ws.norm_part && ldx % 4 == 0 && lddy % 4 == 0 && al16(x) &&
                     al16(w) && al16(dy) && (!add || (ldadd % 4 == 0 && al16(add))) &&
                     (!dx32 || (lddx % 4 == 0 && al16(dx32))) && (!dx16 || (lddx16 % 4 == 0 && al8(dx16)));
    if (!vec) {
        MM_LAUNCH(rmsnorm_backward_kernel, 148 * 4, 256, n * 4, x, ldx, w, dy, lddy, add, ldadd, T, n, eps, dx32, lddx,
                  dx16, lddx16, dw, scale);
        return;
    }
    const size_t smem = sizeof(float) * 8 * n;
    if (n <= 512)
        MM_LAUNCH(rmsnorm_backward_v4_kernel<4>, kNormBlocks, 256, smem, x, ldx, w, dy, lddy, add, ldadd, T, n, eps,
                  dx32, lddx, dx16, lddx16, cx.ws.norm_part);
    else
        MM_LAUNCH(rmsnorm_backward_v4_kernel<8>, kNormBlocks, 256, smem, x, ldx, w, dy, lddy, add, ldadd, T, n, eps,
                  dx32, lddx, dx16, lddx16, cx.ws.norm_part);
    MM_LAUNCH(colsum_kernel, (n + 31) / 32, dim3(32, kColsumGroups), 0, cx.ws.norm_part, kNormBlocks, n, scale, dw);
}

inline void launch_swiglu(Context& cx, const __half* gate, const __half* up, long long ld, int T, int n, __half* out,
                          long long ldo) {
    if (n % 8 == 0 && ld % 8 == 0 && ldo % 8 == 0 && al16(gate) && al16(up) && al16(out))
        MM_LAUNCH(swiglu_v8_kernel, blocks_for(static_cast<long long>(T) * (n / 8), 256), 256, 0, gate, up, ld, T, n,
                  out, ldo);
    else
        MM_LAUNCH(swiglu_kernel, blocks_for(static_cast<long long>(T) * n, 256), 256, 0, gate, up, ld, T, n, out, ldo);
}

inline void launch_swiglu_backward(Context& cx, const __half* gate, const __half* up, long long ld, const float* dy,
                                   long long lddy, int T, int n, __half* dg, __half* du, long long ldo) {
    if (n % 8 == 0 && ld % 8 == 0 && ldo % 8 == 0 && lddy % 4 == 0 && al16(gate) && al16(up) && al16(dy) && al16(dg) &&
        al16(du))
        MM_LAUNCH(swiglu_backward_v8_kernel, blocks_for(static_cast<long long>(T) * (n / 8), 256), 256, 0, gate, up,
                  ld, dy, lddy, T, n, dg, du, ldo);
    else
        MM_LAUNCH(swiglu_backward_kernel<float>, blocks_for(static_cast<long long>(T) * n, 256), 256, 0, gate, up, ld, dy,
                  lddy, T, n, dg, du, ldo);
}
inline void launch_swiglu_backward(Context& cx, const __half* gate, const __half* up, long long ld, const __half* dy,
                                   long long lddy, int T, int n, __half* dg, __half* du, long long ldo) {
    if (n % 8 == 0 && ld % 8 == 0 && ldo % 8 == 0 && lddy % 8 == 0 && al16(gate) && al16(up) && al16(dy) && al16(dg) &&
        al16(du))
        MM_LAUNCH(swiglu_backward_h8_kernel, blocks_for(static_cast<long long>(T) * (n / 8), 256), 256, 0, gate, up,
                  ld, dy, lddy, T, n, dg, du, ldo);
    else
        MM_LAUNCH(swiglu_backward_kernel<__half>, blocks_for(static_cast<long long>(T) * n, 256), 256, 0, gate, up, ld,
                  dy, lddy, T, n, dg, du, ldo);
}

inline void launch_to_half(Context& cx, const float* in, long long ldin, int T, int n, __half* out, long long ldo) {
    if (n % 4 == 0 && ldin % 4 == 0 && ldo % 4 == 0 && al16(in) && al8(out))
        MM_LAUNCH(to_half_v4_kernel, blocks_for(static_cast<long long>(T) * (n / 4), 256), 256, 0, in, ldin, T, n, out,
                  ldo);
    else
        MM_LAUNCH(to_half_kernel, blocks_for(static_cast<long long>(T) * n, 256), 256, 0, in, ldin, T, n, out, ldo);
}

inline void launch_assemble_k(Context& cx, const float* k_nope, long long ldn, const float* k_rope, int T,
                              __half* k, long long ldk) {
    const Dims& c = cx.c;
    const int qk = c.qk();
    if (c.nope % 8 == 0 && c.rope % 8 == 0 && ldn % 4 == 0 && ldk % 8 == 0 && al16(k_nope) && al16(k_rope) && al16(k))
        MM_LAUNCH(assemble_k_v8_kernel, blocks_for(static_cast<long long>(T) * c.H * qk / 8, 256), 256, 0, k_nope, ldn,
                  k_rope, T, c.H, c.nope, c.rope, k, ldk);
    else
        MM_LAUNCH(assemble_k_kernel, blocks_for(static_cast<long long>(T) * c.H * qk, 256), 256, 0, k_nope, ldn, k_rope,
                  T, c.H, c.nope, c.rope, k, ldk);
}

inline void launch_split3(Context& cx, const float* h, int d, int T, int mul, int add, __half* h3, long long ld3) {
    if (d % 4 == 0 && ld3 % 4 == 0 && al16(h) && al8(h3))
        MM_LAUNCH(split3_gather_v4_kernel, blocks_for(static_cast<long long>(T) * (d / 4), 256), 256, 0, h, d, T, mul,
                  add, h3, ld3);
    else
        MM_LAUNCH(split3_gather_kernel, blocks_for(static_cast<long long>(T) * d, 256), 256, 0, h, d, T, mul, add, h3,
                  ld3);
}

// The workspace's row selection from its mask (already on cx.stream), nsel = the caller's
// count of the same rows.
inline void select_rows(Context& cx, int T, int nsel) {
    Workspace& w = cx.ws;
    w.nsel = nsel;
    if (nsel <= 0 || nsel >= T) return;
    const int nb = (T + kSelectBlock - 1) / kSelectBlock;
    MM_LAUNCH(select_count_kernel, nb, kSelectBlock, 0, w.mask, T, w.sel_counts);
    MM_LAUNCH(select_write_kernel, nb, kSelectBlock, 0, w.mask, T, w.sel_counts, w.sel);
}

inline void launch_rowdot(Context& cx, const __half* dout, const __half* out, int T, int H, int DV, float* Dd) {
    if (DV % 8 == 0 && al16(dout) && al16(out))
        MM_LAUNCH(attn_rowdot_v8_kernel, blocks_for(static_cast<long long>(T) * H, 256), 256, 0, dout, out, T, H, DV, Dd);
    else
        MM_LAUNCH(attn_rowdot_kernel, blocks_for(static_cast<long long>(T) * H, 256), 256, 0, dout, out, T, H, DV, Dd);
}

inline void launch_vocab_grad(Context& cx, const float* logits, long long ld, int V, const uint16_t* target,
                              const float* lse, const float* coef, const float* scale, int T, __half* g, long long ldg) {
    if (V % 4 == 0 && ld % 4 == 0 && ldg % 4 == 0 && al16(logits) && al8(g))
        MM_LAUNCH(vocab_grad_v4_kernel, blocks_for(static_cast<long long>(T) * (V / 4), 256), 256, 0, logits, ld, V,
                  target, lse, coef, scale, T, g, ldg);
    else
        MM_LAUNCH(vocab_grad_kernel, T, 256, 0, logits, ld, V, target, lse, coef, scale, T, g, ldg);
}

inline void launch_rope_rows(Context& cx,const float* in, long long ldin, int T, int seq, const int* pos_base, int heads,
                             int width, int begin, int rope, int inverse, float* out32, long long ld32, __half* out16,
                             long long ld16) {
    if ((heads * width) % 4 == 0 && width % 2 == 0 && begin % 2 == 0 && rope % 2 == 0 && ldin % 4 == 0 && al16(in) &&
        (!out32 || (ld32 % 4 == 0 && al16(out32))) && (!out16 || (ld16 % 4 == 0 && al8(out16))))
        MM_LAUNCH(rope_rows_v4_kernel, blocks_for(static_cast<long long>(T) * heads * width / 4, 256), 256, 0, in, ldin,
                  T, seq, pos_base, heads, width, begin, rope, cx.cos_t, cx.sin_t, inverse, out32, ld32, out16, ld16);
    else
        MM_LAUNCH(rope_rows_kernel, warp_rows_grid(T), 256, 0, in, ldin, T, seq, pos_base, heads, width, begin, rope,
                  cx.cos_t, cx.sin_t, inverse, out32, ld32, out16, ld16);
}

// MM_FLASH_TC=0 keeps the 64- and 128-wide forward on the mma.sync kernels (for comparison).
inline bool flash_tc_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("MM_FLASH_TC");
        return !(e && e[0] == '0');
    }();
    return on;
}

// MM_FUSED_SWIGLU=0 keeps the training SwiGLU (forward with tape, backward) as separate
// elementwise kernels around plain products (for comparison).
inline bool swiglu_fused_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("MM_FUSED_SWIGLU");
        return !(e && e[0] == '0');
    }();
    return on;
}

inline void launch_flash_fwd(Context& cx, const LayerBuf& b, int Bc, int S) {
    const Dims& c = cx.c;
    dim3 grid(c.H, Bc, (S + fa::kTile - 1) / fa::kTile);
    const float scale = 1.0f / std::sqrt(static_cast<float>(c.qk()));
    // causal pairs x (qk + dv) multiply-adds
    const double work = 2.0 * Bc * c.H * (S * (S + 1.0) / 2.0) * (c.qk() + c.dv);
    if ((c.qk() == 64 || c.qk() == 128) && c.dv == c.qk() && flash_tc_enabled()) {
        // tcgen05 forward: Q, K, V tiles of 128 rows x qk through TMA (boxes of 64 columns)
        const int D = c.qk();
        const long long T = static_cast<long long>(Bc) * S, wd = static_cast<long long>(c.H) * D;
        const CUtensorMap& tq = tensor_map(b.q, false, wd, T, wd, 64, fatc::kRows);
        const CUtensorMap& tk = tensor_map(b.k, false, wd, T, wd, 64, fatc::kRows);
        const CUtensorMap& tv = tensor_map(b.v, false, wd, T, wd, 64, fatc::kRows);
        // persistent: the resident CTAs walk every (query tile, sequence, head) item
        const long long items = static_cast<long long>(c.H) * Bc * ((S + fatc::kRows - 1) / fatc::kRows);
        const int resident = sm_count() * (D == 64 ? 2 : 1);
        static const bool persistent = [] {
            const char* e = std::getenv("MM_FLASH_PERSISTENT");  // 0: one item per CTA (comparison)
            return !(e && e[0] == '0');
        }();
        const int gt = static_cast<int>(persistent ? std::min<long long>(items, resident) : items);
        if (D == 64) {
            set_dynamic_smem<flash_fwd_tc_kernel<64>>(fatc::smem_bytes<64>());
            MM_LAUNCH_TIMED(kKFlashFwd, work, flash_fwd_tc_kernel<64>, gt, fatc::kThreads, fatc::smem_bytes<64>(), tq, tk,
                            tv, S, c.H, Bc, scale, b.ao, b.lse, cx.d_err);
        } else {
            set_dynamic_smem<flash_fwd_tc_kernel<128>>(fatc::smem_bytes<128>());
            MM_LAUNCH_TIMED(kKFlashFwd, work, flash_fwd_tc_kernel<128>, gt, fatc::kThreads, fatc::smem_bytes<128>(), tq,
                            tk, tv, S, c.H, Bc, scale, b.ao, b.lse, cx.d_err);
        }
    } else if (c.qk() == 64) {
        MM_LAUNCH_TIMED(kKFlashFwd, work, flash_fwd_mma_kernel<64>, grid, 128, flash_fwd_smem<64>(), b.q, b.k, b.v, S,
                        c.H, scale, b.ao, b.lse);
    } else if (c.qk() == 128) {
        set_dynamic_smem<flash_fwd_mma_kernel<128>>(flash_fwd_smem<128>());
        MM_LAUNCH_TIMED(kKFlashFwd, work, flash_fwd_mma_kernel<128>, grid, 128, flash_fwd_smem<128>(), b.q, b.k, b.v, S,
                        c.H, scale, b.ao, b.lse);
    } else {
        MM_LAUNCH_TIMED(kKFlashFwd, work, flash_fwd_mma_kernel<16>, grid, 128, flash_fwd_smem<16>(), b.q, b.k, b.v, S,
                        c.H, scale, b.ao, b.lse);
    }
}

enum VocabMode { kVocabNone, kVocabAll, kVocabLast };

// The vocabulary backward recomputes the logit tiles (the same three-term product as the
// forward, hence the same values) with the weighted-NLL gradient in the product's epilogue,
// so no [T][V] logits are ever stored. MM_VOCAB_RECOMPUTE=0: the tape pass stores fp32
// logits and vocab_grad_v4_kernel reads them (for comparison).
inline bool vocab_recompute_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("MM_VOCAB_RECOMPUTE");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Whether the vocabulary head of a T-row chunk runs on its nsel selected rows only (set by
// the GRPO update for the rows with mask != 0; needs d % 4 == 0 for the row kernels).
// MM_VOCAB_ROWS=all keeps every row (for comparison).
inline bool vocab_rows_compact(const Context& cx, long long T) {
    static const bool on = [] {
        const char* e = std::getenv("MM_VOCAB_ROWS");
        return !(e && std::strcmp(e, "all") == 0);
    }();
    return on && cx.ws.nsel > 0 && cx.ws.nsel < T && cx.c.d % 4 == 0;
}

// Forward over ws.tokens [Bc*S]. tape: keep every layer's activations. cache: write the
// latent/rope cache of rows [row0, row0 + Bc) (prefill). Vocabulary head:
//   kVocabAll  logits [T][V] into ws.logits and, with targets, lp/lse into ws.lp/ws.lse_v;
//   kVocabLast logits of each sequence's last position into last_logits [Bc][V].
inline void forward_chunk(Context& cx, int Bc, int S, bool tape, VocabMode vm, bool with_targets,
                          __half* cache, int Sc, int row0, float* last_logits) {
    const Dims& c = cx.c;
    Workspace& w = cx.ws;
    const int T = Bc * S;
    const int qk = c.qk(), kvw = c.kvw();
    const int ld_d = cx.d16(c.d), ld_qr = cx.d16(c.qr), ld_kvr = cx.d16(c.kvr), ld_ff = cx.d16(c.dff);
    MM_LAUNCH(embed_kernel, warp_rows_grid(T), 256, 0, w.tokens, cx.E(), w.layers[0].x_in, T, c.d, c.V, cx.d_err);
    for (int l = 0; l < c.L; ++l) {
        LayerBuf& b = w.layers[tape ? l : 0];
        // tape: every layer keeps its input and mid-block residual; otherwise the residual
        // stream is one buffer updated in place by the reduce-add epilogues
        float* x_next = tape ? (l + 1 < c.L ? w.layers[l + 1].x_in : w.x_out) : b.x_in;
        float* res = tape ? b.res : b.x_in;
        // attention block
        launch_rmsnorm(cx, b.x_in, c.d, cx.W(l, kAttnNorm), T, c.d, (float*)nullptr, 0LL, b.h, ld_d);
        const PrepLayer& pw = cx.prep[l];
        const int qkv = c.qr + kvw;
        gemm(cx, T, qkv, c.d, {b.h, ld_d, false}, {pw.Wa, pw.lda, true}, {b.raw_cq, qkv, kOutF32});
        // both latent norms, the rope key and the prefill cache rows in one pass when the
        // widths allow 16-byte rows
        const bool fused_latent = c.qr % 4 == 0 && c.kvr % 4 == 0 && c.rope % 4 == 0 && qkv % 4 == 0 && qkv <= 512 &&
                                  ld_qr % 4 == 0 && ld_kvr % 4 == 0;
        __half* cache_l = cache ? cache + (long long)l * cx.dec.B * Sc * kvw : nullptr;
        if (fused_latent)
            MM_LAUNCH(latent_kernel, warp_rows_grid(T), 256, 0, b.raw_cq, (long long)qkv, c.qr, c.kvr, c.rope,
                      cx.W(l, kQNorm), cx.W(l, kKvNorm), c.eps, T, S, (const int*)nullptr, row0, cx.cos_t, cx.sin_t,
                      b.cq, (long long)ld_qr, b.ckv, (long long)ld_kvr, b.k_rope, cache_l, Sc);
        else
            launch_rmsnorm(cx, b.raw_cq, qkv, cx.W(l, kQNorm), T, c.qr, (float*)nullptr, 0LL, b.cq, ld_qr);
        {
            // q = cq . W_uq with the rope part of every head rotated in the epilogue (fp16)
            GemmOutSpec o{b.q, c.H * qk, kOutF16};
            o.rope_cos = cx.cos_t;
            o.rope_sin = cx.sin_t;
            o.rope_seq = S;
            o.rope_period = qk;
            o.rope_begin = c.nope;
            o.rope_len = c.rope;
            gemm(cx, T, c.H * qk, c.qr, {b.cq, ld_qr, false}, {cx.S(l, kWuq), cx.SL(l, kWuq), true}, o);
        }
        if (!fused_latent) {
            launch_rmsnorm(cx, b.kvp, qkv, cx.W(l, kKvNorm), T, c.kvr, (float*)nullptr, 0LL, b.ckv, ld_kvr);
            MM_LAUNCH(rope_key_kernel, blocks_for((long long)T * (c.rope / 2), 256), 256, 0, b.kvp, (long long)qkv,
                      c.kvr, c.rope, T, S, (const int*)nullptr, cx.cos_t, cx.sin_t, b.k_rope, (__half*)nullptr, 0LL);
            if (cache)
                MM_LAUNCH(cache_write_kernel, blocks_for((long long)T * kvw, 256), 256, 0, b.ckv, (long long)ld_kvr,
                          b.k_rope, T, S, (const int*)nullptr, row0, cache_l, Sc, c.kvr, c.rope);
        }
        gemm(cx, T, c.H * c.nope, c.kvr, {b.ckv, ld_kvr, false}, {cx.S(l, kWuk), cx.SL(l, kWuk), true},
             {w.knope, c.H * c.nope, kOutF32});
        launch_assemble_k(cx, w.knope, (c.H * c.nope), b.k_rope, T, b.k, (c.H * qk));
        gemm(cx, T, c.aw(), c.kvr, {b.ckv, ld_kvr, false}, {cx.S(l, kWuv), cx.SL(l, kWuv), true}, {b.v, c.aw(), kOutF16});
        launch_flash_fwd(cx, b, Bc, S);
        {
            GemmOutSpec o{res, c.d, tape ? kOutF32 : kOutF32Acc};
            if (tape) o.residual = b.x_in;
            o.ldr = c.d;
            gemm(cx, T, c.d, c.aw(), {b.ao, c.aw(), false}, {cx.S(l, kWo), cx.SL(l, kWo), true}, o);
        }
        // feed-forward block: the [W_gate | W_up] product in ffn_terms(cx) fp16 terms, its input
        // written by the norm as [hi | lo | hi] and the weight rows wrapped onto [W_hi; W_lo]
        // (the rollout prefill, kVocabLast, yields no log-probabilities: one term)
        const int nt = vm == kVocabLast ? 1 : ffn_terms(cx);
        const long long ld_h2 = nt * static_cast<long long>(ld_d);
        launch_rmsnorm(cx, res, c.d, cx.W(l, kFfnNorm), T, c.d, (float*)nullptr, 0LL, b.h2, ld_h2, nt - 1);
        const int ld_gu = cx.d16(2 * c.dff);
        const int k_gu = nt * c.d;
        if (c.dff % 8 || (tape && !swiglu_fused_enabled())) {
            // the backward needs gate and up themselves
            GemmOutSpec o{b.gate, ld_gu, kOutF16};
            if (nt > 1) o.b_k_wrap = c.d;
            o.b_k3 = nt == 3;
            gemm(cx, T, 2 * c.dff, k_gu, {b.h2, ld_h2, false}, {pw.Wgu, pw.ldgu, true}, o);
            launch_swiglu(cx, b.gate, b.up, ld_gu, T, c.dff, b.gated, ld_ff);
        } else {
            // SwiGLU in the product's epilogue; with tape it also stores gate and up for the backward
            GemmOutSpec o{b.gated, ld_ff, kOutF16};
            o.glu_n = c.dff;
            if (nt > 1) o.b_k_wrap = c.d;
            o.b_k3 = nt == 3;
            if (tape) {
                o.pre_gate = b.gate;
                o.pre_ld = ld_gu;
            }
            gemm(cx, T, c.dff, k_gu, {b.h2, ld_h2, false}, {pw.Wgu, pw.ldgu, true}, o);
        }
        {
            GemmOutSpec o{x_next, c.d, tape ? kOutF32 : kOutF32Acc};
            if (tape) o.residual = b.res;
            o.ldr = c.d;
            gemm(cx, T, c.d, c.dff, {b.gated, ld_ff, false}, {cx.S(l, kWdown), cx.SL(l, kWdown), true}, o);
        }
    }
    if (vm == kVocabNone) return;
    launch_rmsnorm(cx, tape ? w.x_out : w.layers[0].x_in, c.d, cx.FinalNorm(), T, c.d, w.hf, c.d, (__half*)nullptr, 0LL);
    const int ld3 = cx.d16(3 * c.d);
    GemmOutSpec lo{nullptr, c.V, kOutF32};
    lo.alpha = 1.0f / kVocabScale;
    if (vm == kVocabAll) {
        // an update's passes (nsel set) run the head on the rows it uses only
        const bool compact = with_targets && vocab_rows_compact(cx, T);
        const int M = compact ? w.nsel : T;
        if (compact)
            MM_LAUNCH(split3_select_v4_kernel, blocks_for(static_cast<long long>(M) * (c.d / 4), 256), 256, 0, w.hf, c.d,
                      w.sel, M, w.targets, w.h3, (long long)ld3, w.sel_tgt);
        else
            launch_split3(cx, w.hf, c.d, T, 1, 0, w.h3, ld3);
        lo.out = w.logits;
        if (with_targets) {
            // log-softmax fused into the product: per-tile row partials, then one combine;
            // the logits are never stored (the backward recomputes them), except for the
            // backward with stored logits (MM_VOCAB_RECOMPUTE=0)
            lo.lse_part = w.lse_part;
            lo.targets = compact ? w.sel_tgt : w.targets;
            lo.tgt_logit = w.tgt_logit;
            lo.no_store = !tape || vocab_recompute_enabled();
        }
        const int bn = gemm(cx, M, c.V, 3 * c.d, {w.h3, ld3, false}, {cx.E3(), cx.E3L(), false}, lo);
        if (with_targets) {
            MM_LAUNCH_TIMED(kKLogsoftmax, 16.0 * M * ((c.V + bn - 1) / bn), lse_combine_kernel, blocks_for(M, kLseRows), 256,
                            0, w.lse_part, 2 * ((c.V + bn - 1) / bn), M, w.tgt_logit, compact ? w.sel_lp : w.lp,
                            compact ? w.sel_lse : w.lse_v, cx.d_err);
            if (compact) {  // rows outside the selection (mask 0) are never read: zero
                MM_CUDA_CHECK(cudaMemsetAsync(w.lp, 0, sizeof(float) * T, cx.stream));
                MM_CUDA_CHECK(cudaMemsetAsync(w.lse_v, 0, sizeof(float) * T, cx.stream));
                MM_LAUNCH(scatter_lp_kernel, blocks_for(M, 256), 256, 0, w.sel, M, w.sel_lp, w.sel_lse, w.lp, w.lse_v);
            }
        }
    } else {
        MM_LAUNCH(split3_gather_kernel, blocks_for((long long)Bc * c.d, 256), 256, 0, w.hf, c.d, Bc, S, S - 1, w.h3,
                  (long long)ld3);
        lo.out = last_logits;
        gemm(cx, Bc, c.V, 3 * c.d, {w.h3, ld3, false}, {cx.E3(), cx.E3L(), false}, lo);
    }
}

// Backward of the chunk most recently run forward with tape = true and kVocabAll.
// ws.coef holds the per-token weighted-NLL coefficients; d_scale[0] is the power-of-two
// gradient scale for the fp16 operands and d_scale[1] its inverse, applied when a
// gradient lands in the fp32 accumulator.
inline void backward_chunk(Context& cx, int Bc, int S) {
    const Dims& c = cx.c;
    Workspace& w = cx.ws;
    const int T = Bc * S;
    const int qk = c.qk(), kvw = c.kvw(), aw = c.aw();
    const int ld_d = cx.d16(c.d), ld_qr = cx.d16(c.qr), ld_kvr = cx.d16(c.kvr), ld_ff = cx.d16(c.dff);
    const int ld3 = cx.d16(3 * c.d);
    const float* inv_s = cx.d_scale + 1;
    // vocabulary head: g = s * coef * (softmax - onehot), on the forward's selected rows when
    // it ran on those only (the other rows' coef is 0: their g, dH and dE terms are zero)
    const bool compact = vocab_rows_compact(cx, T);
    const int M = compact ? w.nsel : T;
    if (compact) MM_LAUNCH(gather_coef_kernel, blocks_for(M, 256), 256, 0, w.sel, M, w.coef, w.sel_coef);
    const uint16_t* tgt = compact ? w.sel_tgt : w.targets;
    const float* lse = compact ? w.sel_lse : w.lse_v;
    const float* cf = compact ? w.sel_coef : w.coef;
    if (vocab_recompute_enabled()) {
        // the forward's logit tiles again (h3 still holds its rows), gradient in the epilogue
        GemmOutSpec o{w.g16, c.V, kOutF16};
        o.alpha = 1.0f / kVocabScale;
        o.targets = tgt;
        o.vg_lse = lse;
        o.vg_coef = cf;
        o.vg_scale = cx.d_scale;
        gemm(cx, M, c.V, 3 * c.d, {w.h3, ld3, false}, {cx.E3(), cx.E3L(), false}, o);
    } else {
        launch_vocab_grad(cx, w.logits, c.V, c.V, tgt, lse, cf, cx.d_scale, M, w.g16, c.V);
    }
    {
        // dH of the selected rows into dy (free until the final norm's backward writes it),
        // then scattered into the cleared dH
        GemmOutSpec o{compact ? w.dy : w.dh, c.d, kOutF32};
        o.alpha = 1.0f / kVocabScale;  // E3's hi part holds 64 * E
        gemm(cx, M, c.d, c.V, {w.g16, c.V, false}, {cx.E3(), cx.E3L(), true}, o);
        if (compact) {
            MM_CUDA_CHECK(cudaMemsetAsync(w.dh, 0, sizeof(float) * T * c.d, cx.stream));
            MM_LAUNCH(scatter_rows_v4_kernel, blocks_for(static_cast<long long>(M) * (c.d / 4), 256), 256, 0, w.dy, w.sel,
                      M, c.d, w.dh);
        }
    }
    {
        GemmOutSpec o{cx.GE(), c.d, kOutF32Acc};
        o.alpha_ptr = inv_s;
        gemm(cx, c.V, c.d, M, {w.g16, c.V, true}, {w.h3, ld3, true}, o);  // h_hi = h3[:, :d]
    }
    // dy (fp32, the residual gradient) and its fp16 copy for the layer's products
    launch_rmsnorm_backward(cx, w.x_out, c.d, cx.FinalNorm(), w.dh, c.d, (const float*)nullptr, 0LL, T, c.d, w.dy, c.d,
                            w.dy16, ld_d, cx.GFinalNorm(), inv_s);
    for (int l = c.L - 1; l >= 0; --l) {
        LayerBuf& b = w.layers[l];
        // feed-forward block
        {
            GemmOutSpec o{cx.G(l, kWdown), c.d, kOutF32Acc};
            o.alpha_ptr = inv_s;
            gemm(cx, c.dff, c.d, T, {b.gated, ld_ff, true}, {w.dy16, ld_d, true}, o);
        }
        const int ld_gu = cx.d16(2 * c.dff);
        const PrepLayer& pw = cx.prep[l];
        if (c.dff % 8 == 0 && swiglu_fused_enabled()) {
            // dH = dY W_down^T with the SwiGLU backward in its epilogue: [d gate | d up] in fp16
            // (scaled like every backward operand) straight from the fp32 accumulator
            GemmOutSpec o{w.dg16, ld_gu, kOutF16};
            o.dglu_gu = b.gate;
            o.dglu_ld = ld_gu;
            o.dglu_up = w.du16;
            gemm(cx, T, c.dff, c.d, {w.dy16, ld_d, false}, {cx.S(l, kWdown), cx.SL(l, kWdown), false}, o);
        } else {
            // dH in fp16, read once by the SwiGLU backward
            gemm(cx, T, c.dff, c.d, {w.dy16, ld_d, false}, {cx.S(l, kWdown), cx.SL(l, kWdown), false},
                 {w.dgated16, ld_ff, kOutF16});
            launch_swiglu_backward(cx, b.gate, b.up, ld_gu, w.dgated16, ld_ff, T, c.dff, w.dg16, w.du16, ld_gu);
        }
        {
            // the weight gradients read the fp16 high part of the FFN input
            const long long ld_h2 = ffn_terms(cx) * static_cast<long long>(ld_d);
            GemmOutSpec o{cx.G(l, kWgate), c.dff, kOutF32Acc};
            o.alpha_ptr = inv_s;
            gemm(cx, c.d, c.dff, T, {b.h2, ld_h2, true}, {w.dg16, ld_gu, true}, o);
            o.out = cx.G(l, kWup);
            gemm(cx, c.d, c.dff, T, {b.h2, ld_h2, true}, {w.du16, ld_gu, true}, o);
        }
        // dh2 = [dg | du] . [W_gate | W_up]^T, one product over K = 2 d_ff
        gemm(cx, T, c.d, 2 * c.dff, {w.dg16, ld_gu, false}, {pw.Wgu, pw.ldgu, false}, {w.dh2, c.d, kOutF32});
        launch_rmsnorm_backward(cx, b.res, c.d, cx.W(l, kFfnNorm), w.dh2, c.d, w.dy, c.d, T, c.d, w.dres, c.d, w.dres16, ld_d, cx.G(l, kFfnNorm), inv_s);
        // attention output projection
        {
            GemmOutSpec o{cx.G(l, kWo), c.d, kOutF32Acc};
            o.alpha_ptr = inv_s;
            gemm(cx, aw, c.d, T, {b.ao, aw, true}, {w.dres16, ld_d, true}, o);
        }
        gemm(cx, T, aw, c.d, {w.dres16, ld_d, false}, {cx.S(l, kWo), cx.SL(l, kWo), false}, {w.dao16, aw, kOutF16});
        // attention
        launch_rowdot(cx, w.dao16, b.ao, T, c.H, c.dv, w.Dd);
        {
            dim3 grid(c.H, Bc, (S + fa::kTile - 1) / fa::kTile);
            const float scale = 1.0f / std::sqrt(static_cast<float>(qk));
            const double pairs = static_cast<double>(Bc) * c.H * (S * (S + 1.0) / 2.0);
            // dK/dV: S^T, dP^T, dV, dK products; dQ: S, dP, dQ products (2 flops per MAC)
            const double w_kv = pairs * 2.0 * (2 * qk + 2 * c.dv), w_q = pairs * 2.0 * (2 * qk + c.dv);
            const int ld_q16 = cx.d16(c.H * qk), ld_v16 = cx.d16(aw);
            if (qk == 64) {
                set_dynamic_smem<flash_bwd_dkdv_mma_kernel<64>>(flash_dkdv_smem<64>());
                set_dynamic_smem<flash_bwd_dq_mma_kernel<64>>(flash_dq_smem<64>());
                MM_LAUNCH_TIMED(kKFlashBwd, w_kv, flash_bwd_dkdv_mma_kernel<64>, grid, 128, flash_dkdv_smem<64>(), b.q, b.k,
                                b.v, w.dao16, b.lse, w.Dd, S, c.H, scale, w.dk, w.dv16, (long long)ld_v16);
                if (c.dv == 64 && flash_tc_enabled()) {
                    // tcgen05 dQ: Q/dO tiles of 128 rows, K/V tiles of 64 keys through TMA
                    const long long T64 = static_cast<long long>(Bc) * S, wd = static_cast<long long>(c.H) * 64;
                    const CUtensorMap& tq = tensor_map(b.q, false, wd, T64, wd, 64, fadq::kRows);
                    const CUtensorMap& tg = tensor_map(w.dao16, false, wd, T64, wd, 64, fadq::kRows);
                    const CUtensorMap& tk = tensor_map(b.k, false, wd, T64, wd, 64, fadq::kKeys);
                    const CUtensorMap& tv = tensor_map(b.v, false, wd, T64, wd, 64, fadq::kKeys);
                    set_dynamic_smem<flash_bwd_dq_tc_kernel>(fadq::kSmem);
                    dim3 gq(c.H, Bc, (S + fadq::kRows - 1) / fadq::kRows);
                    MM_LAUNCH_TIMED(kKFlashBwd, w_q, flash_bwd_dq_tc_kernel, gq, fadq::kThreads, fadq::kSmem, tq, tg, tk,
                                    tv, b.lse, w.Dd, S, c.H, scale, w.dq16, (long long)ld_q16, cx.cos_t, cx.sin_t,
                                    c.nope, c.rope, cx.d_err);
                } else {
                    MM_LAUNCH_TIMED(kKFlashBwd, w_q, flash_bwd_dq_mma_kernel<64>, grid, 128, flash_dq_smem<64>(), b.q, b.k,
                                    b.v, w.dao16, b.lse, w.Dd, S, c.H, scale, w.dq16, (long long)ld_q16, cx.cos_t,
                                    cx.sin_t, c.nope, c.rope);
                }
            } else if (qk == 128) {
                set_dynamic_smem<flash_bwd_dkdv_mma_kernel<128>>(flash_dkdv_smem<128>());
                set_dynamic_smem<flash_bwd_dq_mma_kernel<128>>(flash_dq_smem<128>());
                MM_LAUNCH_TIMED(kKFlashBwd, w_kv, flash_bwd_dkdv_mma_kernel<128>, grid, 128, flash_dkdv_smem<128>(), b.q,
                                b.k, b.v, w.dao16, b.lse, w.Dd, S, c.H, scale, w.dk, w.dv16, (long long)ld_v16);
                MM_LAUNCH_TIMED(kKFlashBwd, w_q, flash_bwd_dq_mma_kernel<128>, grid, 128, flash_dq_smem<128>(), b.q, b.k,
                                b.v, w.dao16, b.lse, w.Dd, S, c.H, scale, w.dq16, (long long)ld_q16, cx.cos_t, cx.sin_t,
                                c.nope, c.rope);
            } else {
                MM_LAUNCH_TIMED(kKFlashBwd, w_kv, flash_bwd_dkdv_mma_kernel<16>, grid, 128, flash_dkdv_smem<16>(), b.q, b.k,
                                b.v, w.dao16, b.lse, w.Dd, S, c.H, scale, w.dk, w.dv16, (long long)ld_v16);
                MM_LAUNCH_TIMED(kKFlashBwd, w_q, flash_bwd_dq_mma_kernel<16>, grid, 128, flash_dq_smem<16>(), b.q, b.k, b.v,
                                w.dao16, b.lse, w.Dd, S, c.H, scale, w.dq16, (long long)ld_q16, cx.cos_t, cx.sin_t,
                                c.nope, c.rope);
            }
        }
        const int ld_q16 = cx.d16(c.H * qk);
        const int ld_kn16 = cx.d16(c.H * c.nope);
        MM_LAUNCH(split_dk_kernel, warp_rows_grid(T), 256, 0, w.dk, T, c.H, c.nope, c.rope, w.dkn16, (long long)ld_kn16, w.drope);
        launch_rope_rows(cx, w.drope, c.rope, T, S, (const int*)nullptr, 1, c.rope, 0, c.rope, 1, w.drope2, c.rope, (__half*)nullptr, 0LL);
        const int ld_v16 = cx.d16(aw);
        {
            GemmOutSpec o{cx.G(l, kWuk), c.H * c.nope, kOutF32Acc};
            o.alpha_ptr = inv_s;
            gemm(cx, c.kvr, c.H * c.nope, T, {b.ckv, ld_kvr, true}, {w.dkn16, ld_kn16, true}, o);
            o.out = cx.G(l, kWuv);
            o.ldc = aw;
            gemm(cx, c.kvr, aw, T, {b.ckv, ld_kvr, true}, {w.dv16, ld_v16, true}, o);
        }
        gemm(cx, T, c.kvr, c.H * c.nope, {w.dkn16, ld_kn16, false}, {cx.S(l, kWuk), cx.SL(l, kWuk), false}, {w.dckv, c.kvr, kOutF32});
        gemm(cx, T, c.kvr, aw, {w.dv16, ld_v16, false}, {cx.S(l, kWuv), cx.SL(l, kWuv), false}, {w.dckv, c.kvr, kOutF32Acc});
        const int qkv = c.qr + kvw, ld_qkv16 = cx.d16(qkv);
        launch_rmsnorm_backward(cx, b.kvp, qkv, cx.W(l, kKvNorm), w.dckv, c.kvr, (const float*)nullptr, 0LL, T, c.kvr, w.dkvraw, c.kvr, (__half*)nullptr, 0LL, cx.G(l, kKvNorm), inv_s);
        MM_LAUNCH(pack_dkv_kernel, blocks_for((long long)T * kvw, 256), 256, 0, w.dkvraw, w.drope2, T, c.kvr, c.rope, w.dkvp16,
                  (long long)ld_qkv16);
        {
            GemmOutSpec o{cx.G(l, kWdkv), kvw, kOutF32Acc};
            o.alpha_ptr = inv_s;
            gemm(cx, c.d, kvw, T, {b.h, ld_d, true}, {w.dkvp16, ld_qkv16, true}, o);
        }
        {
            GemmOutSpec o{cx.G(l, kWuq), c.H * qk, kOutF32Acc};
            o.alpha_ptr = inv_s;
            gemm(cx, c.qr, c.H * qk, T, {b.cq, ld_qr, true}, {w.dq16, ld_q16, true}, o);
        }
        gemm(cx, T, c.qr, c.H * qk, {w.dq16, ld_q16, false}, {cx.S(l, kWuq), cx.SL(l, kWuq), false}, {w.dcq, c.qr, kOutF32});
        launch_rmsnorm_backward(cx, b.raw_cq, qkv, cx.W(l, kQNorm), w.dcq, c.qr, (const float*)nullptr, 0LL, T, c.qr, (float*)nullptr, 0LL, w.draw16, ld_qkv16, cx.G(l, kQNorm), inv_s);
        {
            GemmOutSpec o{cx.G(l, kWdq), c.qr, kOutF32Acc};
            o.alpha_ptr = inv_s;
            gemm(cx, c.d, c.qr, T, {b.h, ld_d, true}, {w.draw16, ld_qkv16, true}, o);
        }
        // dh = [d raw_cq | d kv_pack] . [W_dq | W_dkv]^T, one product over K = qr + kvw
        gemm(cx, T, c.d, qkv, {w.draw16, ld_qkv16, false}, {cx.prep[l].Wa, cx.prep[l].lda, false}, {w.dh, c.d, kOutF32});
        launch_rmsnorm_backward(cx, b.x_in, c.d, cx.W(l, kAttnNorm), w.dh, c.d, w.dres, c.d, T, c.d, w.dy, c.d, w.dy16,
                                ld_d, cx.G(l, kAttnNorm), inv_s);
    }
    // embedding-gather gradient, summed per vocabulary row in 64-bit fixed point (the
    // accumulator is zero between chunks: the conversion clears what it consumes)
    const long long nE = static_cast<long long>(c.V) * c.d;
    const size_t acc_bytes = sizeof(unsigned long long) * static_cast<size_t>(nE);
    const bool fresh = cx.emb_acc.cap < acc_bytes + 256;
    char* eb = static_cast<char*>(cx.emb_acc.get(acc_bytes + 256));
    auto* acc = reinterpret_cast<unsigned long long*>(eb);
    auto* max_bits = reinterpret_cast<unsigned int*>(eb + acc_bytes);
    int* nonfinite = reinterpret_cast<int*>(eb + acc_bytes + 4);
    if (fresh) MM_CUDA_CHECK(cudaMemsetAsync(acc, 0, acc_bytes, cx.stream));
    MM_CUDA_CHECK(cudaMemsetAsync(max_bits, 0, 8, cx.stream));
    MM_LAUNCH(absmax_kernel, static_cast<unsigned>(sm_count() * 4), 256, 0, w.dy, static_cast<long long>(T) * c.d, max_bits);
    MM_LAUNCH(embed_grad_fixed_kernel, warp_rows_grid(T), 256, 0, w.tokens, w.dy, T, c.d, acc, max_bits, nonfinite);
    MM_LAUNCH(embed_grad_convert_kernel, static_cast<unsigned>(sm_count() * 8), 256, 0, acc, nE, T, max_bits, nonfinite,
              inv_s, cx.GE());
}

} // namespace mm
