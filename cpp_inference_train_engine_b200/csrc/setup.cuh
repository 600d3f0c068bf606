// Context construction, GEMM dispatch, parameter upload/download and the derived fp16
// weight copies.
#pragma once
#include "runtime.cuh"
#include "decode_mk.cuh"

namespace mm {

// The model shape the fused decode step (decode_mk_kernel) is built for: the 35.8M model.
inline bool mk_shape(const Dims& c) {
    return c.d == mk::D && c.qr == mk::QR && c.kvr == mk::KVR && c.rope == mk::ROPE && c.H == mk::H &&
           c.dff == mk::DFF && c.L <= mk::kMaxLayers && c.nope + c.rope == 64;
}


// out[r][c] += alpha * (*alpha_ptr) * sum_z part[z][r][c], z in order (deterministic
// split-K); split z's partial starts at part + z * split_stride.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, long long split_stride, int M, int N,
                                     float* __restrict__ out, long long ldc, float alpha,
                                     const float* __restrict__ alpha_ptr) {
    MM_PDL_ENTRY();
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long long MN = static_cast<long long>(M) * N;
    if (idx >= MN) return;
    float s = 0.f;
    for (int z = 0; z < splits; ++z) s += part[z * split_stride + idx];
    const float a = alpha * (alpha_ptr ? *alpha_ptr : 1.0f);
    const int r = static_cast<int>(idx / N), c = static_cast<int>(idx % N);
    out[r * ldc + c] += a * s;
}

inline int gemm(Context& cx, int M, int N, int K, Opnd A, Opnd B, const GemmOutSpec& o_in, bool bf16) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    GemmOutSpec o = o_in;
    if (o.lse_part && (o.kind != kOutF32 || o.residual || !o.targets || !o.tgt_logit))
        fail(MM_INVALID_ARGUMENT, "log-sum-exp epilogue needs a plain fp32 product with targets");
    if (o.rope_cos && (o.kind != kOutF16 || o.glu_n || o.rope_len % 2 || o.rope_begin % 2 || o.rope_period < 1 ||
                       o.rope_seq < 1))
        fail(MM_INVALID_ARGUMENT, "RoPE epilogue needs a plain fp16 product");
    if (o.glu_n && (o.kind != kOutF16 || o.residual || o.lse_part || !B.mn || o.glu_n < N))
        fail(MM_INVALID_ARGUMENT, "SwiGLU epilogue needs an fp16 product with [gate | up] MN-major weights");
    if (o.pre_gate && (!o.glu_n || o.glu_n != N || N % 8 || o.pre_ld % 8 || o.pre_ld < 2 * N))
        fail(MM_INVALID_ARGUMENT, "pre-activation stores need the SwiGLU epilogue over all d_ff columns");
    if (o.dglu_gu && (o.kind != kOutF16 || o.residual || o.lse_part || o.glu_n || o.rope_cos || !o.dglu_up ||
                      N % 8 || o.ldc % 8 || o.dglu_ld % 8 || o.dglu_ld < 2 * N))
        fail(MM_INVALID_ARGUMENT, "SwiGLU-backward epilogue needs a plain fp16 product, N % 8 == 0");
    if (o.vg_lse && (o.kind != kOutF16 || o.residual || o.lse_part || o.glu_n || o.dglu_gu || o.rope_cos ||
                     !o.targets || !o.vg_coef || !o.vg_scale))
        fail(MM_INVALID_ARGUMENT, "vocabulary-gradient epilogue needs a plain fp16 product with targets");
    if (o.residual) {
        // out = alpha * A B + residual  ==  out := residual, then out += alpha * A B through the
        // TMA reduce-add epilogue (the residual moves as one coalesced device copy).
        if (o.kind != kOutF32) fail(MM_INVALID_ARGUMENT, "residual epilogue needs fp32 output");
        MM_CUDA_CHECK(cudaMemcpy2DAsync(o.out, o.ldc * 4, o.residual, o.ldr * 4, static_cast<size_t>(N) * 4, M,
                                        cudaMemcpyDeviceToDevice, cx.stream));
        o.residual = nullptr;
        o.kind = kOutF32Acc;
    }
    const long long tiles_m = (M + kGemmBM - 1) / kGemmBM;
    const int num_k_all = (K + kGemmBK - 1) / kGemmBK;
    // products that will be split over K (few output tiles, long K) use the widest tile
    const bool split_candidate = o.kind == kOutF32Acc && num_k_all >= 32 && N % 4 == 0 &&
                                 tiles_m * ((N + 63) / 64) < sm_count();
    int BN = 64;
    if (o.glu_n || o.dglu_gu) BN = 256;  // SwiGLU: 128 gate + 128 up columns per tile; both on 256-wide tiles only
    else if (N >= 256 && (split_candidate || tiles_m * ((N + 255) / 256) >= 148)) BN = 256;
    else if (tiles_m * ((N + 127) / 128) >= 120 && N > 64) BN = 128;
    // MM_GEMM_BN (64, 128 or 256) pins the tile width of every plain product, for tuning.
    static const int forced_bn = [] {
        const char* e = std::getenv("MM_GEMM_BN");
        const int v = e ? std::atoi(e) : 0;
        return v == 64 || v == 128 || v == 256 ? v : 0;
    }();
    if (forced_bn && !o.glu_n && !o.dglu_gu) BN = forced_bn;
    if (o.b_k_wrap && (!B.mn || o.b_k_wrap % kGemmBK || K != (o.b_k3 ? 3 : 2) * o.b_k_wrap))
        fail(MM_INVALID_ARGUMENT, "split A needs MN-major B and K = 2 or 3 times the 64-aligned wrap");
    const int nb = o.glu_n ? o.glu_n + N : N;  // columns of B
    const int kb_rows = o.b_k_wrap ? (o.b_k3 ? 2 : 1) * o.b_k_wrap : K;  // rows of B
    const CUtensorMap& ta = A.mn ? tensor_map(A.p, bf16, M, K, A.ld, 64, 64)
                                 : tensor_map(A.p, bf16, K, M, A.ld, 64, kGemmBM);
    const CUtensorMap& tb = B.mn ? tensor_map(B.p, bf16, nb, kb_rows, B.ld, 64, 64)
                                 : tensor_map(B.p, bf16, K, nb, B.ld, 64, BN);
    GemmArgs ga{M, N, K, A.mn ? 1 : 0, B.mn ? 1 : 0, bf16 ? 1 : 0, o.kind,
                o.residual, o.ldr, o.alpha, o.alpha_ptr, cx.d_err, 0, 0,
                o.lse_part, o.targets, o.tgt_logit, (o.lse_part && o.no_store) ? 1 : 0, o.glu_n,
                o.rope_cos, o.rope_sin, o.rope_seq, o.rope_period, o.rope_begin, o.rope_len,
                o.pre_gate ? 1 : 0, o.dglu_gu, o.dglu_ld, o.dglu_gu ? N : 0, o.b_k_wrap, o.b_k3 ? 1 : 0,
                o.vg_lse, o.vg_coef, o.vg_scale};
    // Split-K for accumulating products with few output tiles over a long K (the weight
    // gradients, K = tokens): each K slice stores its fp32 partial, then one reduction adds
    // them in order into the destination.
    const long long tiles = tiles_m * ((N + BN - 1) / BN);
    const int num_k = (K + kGemmBK - 1) / kGemmBK;
    int splits = 1;
    if (!o.glu_n && o.kind == kOutF32Acc && !o.residual && tiles < sm_count() && num_k >= 32 && N % 4 == 0) {
        // the split count whose waves of (tile, split) units cost least per split: time ~
        // ceil(tiles * s / SMs) / s (a nearly empty last wave costs as much as a full one);
        // ties go to fewer splits (less partial traffic)
        const int cap = static_cast<int>(std::min<long long>(32, num_k / 8));
        double best = 2.0;
        for (int s = 1; s <= cap; ++s) {
            const double cost = static_cast<double>((tiles * s + sm_count() - 1) / sm_count()) / s;
            if (cost < best - 1e-12) {
                best = cost;
                splits = s;
            }
        }
    }
    // Output map: 32-row x 128-byte boxes; fp32 partials of split z occupy rows
    // [z * Mp, z * Mp + M) with Mp = M rounded up to whole 128-row tiles, so a tile's
    // clipped edge never reaches the next split.
    const int map_type = (o.kind == kOutF16) ? kMapF16 : (o.kind == kOutBF16) ? kMapBF16 : kMapF32;
    const int ch = map_type == kMapF32 ? 32 : 64;
    float* part = nullptr;
    const CUtensorMap* tc = nullptr;
    if (splits > 1) {
        const int per = (num_k + splits - 1) / splits;
        splits = (num_k + per - 1) / per;
        const int Mp = static_cast<int>(tiles_m * kGemmBM);
        const long long n_pad = N;  // N % 4 == 0: 16-byte row pitch
        part = static_cast<float*>(cx.splitk.get(sizeof(float) * static_cast<size_t>(splits) * Mp * n_pad));
        ga.k_tiles_per_split = per;
        ga.split_rows = Mp;
        ga.out_kind = kOutF32;
        ga.alpha = 1.f;
        ga.alpha_ptr = nullptr;
        tc = &tensor_map_t(part, kMapF32, N, static_cast<long long>(splits) * Mp, n_pad, 32, 32);
    } else {
        tc = &tensor_map_t(o.out, map_type, N, M, o.ldc, ch, 32);
    }
    // A grid that fits one wave (the decode-time products, M = batch) has each CTA's whole
    // K loop on the critical path: a deeper TMA ring keeps more of it in flight.
    const bool one_wave = tiles * splits <= sm_count();
    // auxiliary fp16 outputs of the SwiGLU epilogues: 64-column x 32-row boxes like tc
    const CUtensorMap* td = tc;
    const CUtensorMap* te = tc;
    if (o.pre_gate) {
        td = &tensor_map_t(o.pre_gate, kMapF16, N, M, o.pre_ld, 64, 32);
        te = &tensor_map_t(o.pre_gate + o.glu_n, kMapF16, N, M, o.pre_ld, 64, 32);
    } else if (o.dglu_gu) {
        td = &tensor_map_t(o.dglu_up, kMapF16, N, M, o.ldc, 64, 32);
    }
    // Large 256-wide products run on CTA pairs: M >= pair_gemm_min_m(), at least one full
    // wave of 256 x 256 tiles, and no other stream's products running beside them.
    const long long pair_tiles = static_cast<long long>((M + 255) / 256) * ((N + (o.glu_n ? 127 : 255)) / (o.glu_n ? 128 : 256));
    if (BN == 256 && splits == 1 && M >= pair_gemm_min_m() && cx.pair_ok && pair_gemm_enabled() && pair_gemm_slots() > 0 &&
        pair_tiles >= pair_gemm_slots()) {
        // the B tile of each CTA is 128 columns: K-major B boxes are 128 rows high
        const CUtensorMap& tb2 = B.mn ? tb : tensor_map(B.p, bf16, K, nb, B.ld, 64, 128);
        if (o.glu_n) launch_gemm_pair<kEpiGlu>(cx, ta, tb2, *tc, *td, *te, ga);
        else if (o.dglu_gu) launch_gemm_pair<kEpiDglu>(cx, ta, tb2, *tc, *td, *te, ga);
        else launch_gemm_pair<kEpiPlain>(cx, ta, tb2, *tc, *td, *te, ga);
    } else if (o.glu_n) launch_gemm_bn<256, 4, kEpiGlu>(cx, ta, tb, *tc, *td, *te, ga);
    else if (o.dglu_gu) launch_gemm_bn<256, 4, kEpiDglu>(cx, ta, tb, *tc, *td, *te, ga);
    else if (BN == 256) launch_gemm_bn<256, 4>(cx, ta, tb, *tc, *td, *te, ga);
    else if (BN == 128) {
        if (one_wave && num_k > 3) launch_gemm_bn<128, 6>(cx, ta, tb, *tc, *td, *te, ga);
        else launch_gemm_bn<128, 3>(cx, ta, tb, *tc, *td, *te, ga);
    } else {
        if (one_wave && num_k > 4) launch_gemm_bn<64, 8>(cx, ta, tb, *tc, *td, *te, ga);
        else launch_gemm_bn<64, 4>(cx, ta, tb, *tc, *td, *te, ga);
    }
    if (splits > 1) {
        // partial of split z, row r: part[(z * Mp + r) * n_pad + c]; reduce over a dense view
        const int Mp = ga.split_rows;
        const long long n_pad = N;
        const long long MN = static_cast<long long>(M) * N;
        if (o.ldc % 4 == 0 && (reinterpret_cast<uintptr_t>(o.out) & 15) == 0)  // N % 4 == 0 here
            launch_k(cx.stream, splitk_reduce_v4_kernel, dim3(blocks_for(MN / 4, 256)), dim3(256), 0,
                part, splits, static_cast<long long>(Mp) * n_pad, M, N, static_cast<float*>(o.out), o.ldc, o.alpha,
                o.alpha_ptr);
        else
            launch_k(cx.stream, splitk_reduce_kernel, dim3(blocks_for(MN, 256)), dim3(256), 0,
                part, splits, static_cast<long long>(Mp) * n_pad, M, N, static_cast<float*>(o.out), o.ldc, o.alpha,
                o.alpha_ptr);
        ++cx.launches;
    }
    return BN;
}

inline Dims dims_from(const mm_model_desc& d) {
    Dims c;
    c.V = d.vocab_size; c.maxS = d.max_sequence_length; c.L = d.n_layers; c.d = d.d_model;
    c.H = d.n_heads; c.nope = d.head_dim_nope; c.rope = d.head_dim_rope; c.dv = d.head_dim_value;
    c.qr = d.q_lora_rank; c.kvr = d.kv_lora_rank; c.dff = d.d_ff;
    c.eps = d.norm_epsilon; c.theta = d.rope_theta;
    return c;
}

// ModelConfig::validate (src/model/config.cpp:20-48) minus the 1e9-parameter cap, plus
// the limits of this backend's kernels.
inline void validate_dims(const Dims& c) {
    const int v[] = {c.V, c.maxS, c.L, c.d, c.H, c.nope, c.rope, c.dv, c.qr, c.kvr, c.dff};
    for (int x : v)
        if (x < 1 || x > 65535) fail(MM_INVALID_ARGUMENT, "model dimensions must be in [1, 65535]");
    if (c.L > 128 || c.H > 256 || c.d % c.H || c.rope % 2)
        fail(MM_INVALID_ARGUMENT, "Invalid vocabulary/layer/head count, d_model divisibility, or odd RoPE dimension");
    if (!std::isfinite(c.eps) || c.eps <= 0 || !std::isfinite(c.theta) || c.theta <= 1)
        fail(MM_INVALID_ARGUMENT, "Invalid normalization epsilon or RoPE theta");
    const bool att_ok = c.qk() == c.dv && (c.qk() == 16 || c.qk() == 64 || c.qk() == 128);
    if (!att_ok) fail(MM_UNSUPPORTED, "attention kernels are built for qk = dv in {16, 64, 128}");
    const bool dec_ok = (c.kvr == 8 && c.rope == 4) || (c.kvr == 128 && c.rope == 16) || (c.kvr == 512 && c.rope == 32);
    if (!dec_ok) fail(MM_UNSUPPORTED, "decode attention is built for (kv_rank, rope) = (8, 4), (128, 16) or (512, 32)");
    if (c.H > kMaxDecodeHeads) fail(MM_UNSUPPORTED, "decode attention is built for at most 64 heads");
}

inline long long parameter_count(const Dims& c) {
    const long long d = c.d, h = c.H, q = c.qr, kv = c.kvr;
    return static_cast<long long>(c.V) * d + d +
           static_cast<long long>(c.L) *
               (d * q + q * h * c.qk() + d * c.kvw() + kv * h * (c.nope + c.dv) + h * c.dv * d +
                3 * d * c.dff + 2 * d + q + kv);
}

// Registry of Model::create (src/model/model.cpp:40-63): (rows, cols, role) per entry,
// role 0 hidden matrix, 1 token embedding, 2 norm scale.
inline std::vector<std::tuple<int, int, int>> registry(const Dims& c) {
    std::vector<std::tuple<int, int, int>> r;
    r.emplace_back(c.V, c.d, 1);
    r.emplace_back(1, c.d, 2);
    for (int l = 0; l < c.L; ++l) {
        r.emplace_back(1, c.d, 2);
        r.emplace_back(c.d, c.qr, 0);
        r.emplace_back(1, c.qr, 2);
        r.emplace_back(c.qr, c.H * c.qk(), 0);
        r.emplace_back(c.d, c.kvw(), 0);
        r.emplace_back(1, c.kvr, 2);
        r.emplace_back(c.kvr, c.H * c.nope, 0);
        r.emplace_back(c.kvr, c.aw(), 0);
        r.emplace_back(c.aw(), c.d, 0);
        r.emplace_back(1, c.d, 2);
        r.emplace_back(c.d, c.dff, 0);
        r.emplace_back(c.d, c.dff, 0);
        r.emplace_back(c.dff, c.d, 0);
    }
    return r;
}

// Rope cos/sin tables with the reference's float arithmetic (ops.cpp:92-96):
// angle = float(t) * pow(theta, -float(j) / float(rope)) for even j.
inline void rope_tables(const Dims& c, std::vector<float>& cs, std::vector<float>& sn) {
    const int half_r = c.rope / 2;
    cs.resize(static_cast<size_t>(c.maxS) * half_r);
    sn.resize(cs.size());
    for (int t = 0; t < c.maxS; ++t)
        for (int p = 0; p < half_r; ++p) {
            const int j = 2 * p;
            float angle = static_cast<float>(t) *
                          std::pow(c.theta, -static_cast<float>(j) / static_cast<float>(c.rope));
            cs[static_cast<size_t>(t) * half_r + p] = std::cos(angle);
            sn[static_cast<size_t>(t) * half_r + p] = std::sin(angle);
        }
}

inline void create_context(Context& cx, const mm_model_desc& desc, int device, bool trainable,
                           const mm_adamw_desc* opt) {
    cx.c = dims_from(desc);
    validate_dims(cx.c);
    cx.device = device;
    cx.trainable = trainable;
    if (opt) cx.opt = *opt;
    MM_CUDA_CHECK(cudaSetDevice(device));
    MM_CUDA_CHECK(cudaStreamCreateWithFlags(&cx.stream, cudaStreamNonBlocking));
    MM_CUDA_CHECK(cudaEventCreate(&cx.ev0));
    MM_CUDA_CHECK(cudaEventCreate(&cx.ev1));
    const Dims& c = cx.c;
    auto reg = registry(c);
    long long cur = 0, scur = 0, flat = 0;
    for (auto& [rows, cols, role] : reg) {
        ParamDesc p{};
        p.off = round_up(cur, 64);
        cur = p.off + static_cast<long long>(rows) * cols;
        p.rows = rows;
        p.cols = cols;
        p.decay = role == 2 ? 0.f : cx.opt.weight_decay;
        if (role == 0) {
            p.shadow_kind = kShadowHalf;
            p.shadow_ld = cx.d16(cols);
        } else if (role == 1) {
            p.shadow_kind = kShadowVocab3;
            p.shadow_ld = cx.d16(3 * cols);
        } else {
            p.shadow_kind = kShadowNone;
            p.shadow_ld = 0;
        }
        if (p.shadow_kind != kShadowNone) {
            p.shadow_off = round_up(scur, 64);
            scur = p.shadow_off + static_cast<long long>(rows) * p.shadow_ld;
        }
        cx.params.push_back(p);
        cx.flat_off.push_back(flat);
        flat += static_cast<long long>(rows) * cols;
    }
    cx.P = flat;
    cx.P_dev = round_up(cur, 64);
    cx.shadow_elems = round_up(scur, 64);
    // decode-derived weights
    const int lda = cx.d16(c.qr + c.kvw()), ldq = cx.d16(c.H * c.kvw()), ldo = cx.d16(c.d),
              ldgu = cx.d16(2 * c.dff);
    auto plan = [&](auto& a) {
        cx.w = a.template take<float>(cx.P_dev);
        if (trainable) {
            cx.g = a.template take<float>(cx.P_dev);
            cx.m = a.template take<float>(cx.P_dev);
            cx.v = a.template take<float>(cx.P_dev);
        }
        cx.shadow = a.template take<__half>(cx.shadow_elems);
        cx.cos_t = a.template take<float>(static_cast<long long>(c.maxS) * (c.rope / 2));
        cx.sin_t = a.template take<float>(static_cast<long long>(c.maxS) * (c.rope / 2));
        cx.d_params = a.template take<ParamDesc>(static_cast<long long>(cx.params.size()));
        cx.prep.resize(c.L);
        for (int l = 0; l < c.L; ++l) {
            PrepLayer& p = cx.prep[l];
            p.lda = lda; p.ldq = ldq; p.ldo = ldo; p.ldgu = ldgu;
            p.Wa = a.template take<__half>(static_cast<long long>(c.d) * lda);
            p.Wq = a.template take<__half>(static_cast<long long>(c.qr) * ldq);
            p.Wo = a.template take<__half>(static_cast<long long>(c.H) * c.kvr * ldo);
            p.Wgu = a.template take<__half>(2LL * c.d * ldgu);  // [hi; lo] rows
            if (mk_shape(c)) {
                p.ldf = static_cast<int>(round_up(static_cast<long long>(c.H) * c.kvw(), 8));
                p.Wf = a.template take<__half>(static_cast<long long>(c.d) * p.ldf);
            }
        }
        if (mk_shape(c)) cx.wq32 = a.template take<float>(static_cast<long long>(c.qr) * c.H * c.kvw());
    };
    Sizer sz;
    plan(sz);
    cx.weights.reserve(sz.used() + 4096);
    plan(cx.weights);
    MM_CUDA_CHECK(cudaMemsetAsync(cx.w, 0, sizeof(float) * cx.P_dev, cx.stream));
    if (trainable) {
        MM_CUDA_CHECK(cudaMemsetAsync(cx.g, 0, sizeof(float) * cx.P_dev, cx.stream));
        MM_CUDA_CHECK(cudaMemsetAsync(cx.m, 0, sizeof(float) * cx.P_dev, cx.stream));
        MM_CUDA_CHECK(cudaMemsetAsync(cx.v, 0, sizeof(float) * cx.P_dev, cx.stream));
    }
    MM_CUDA_CHECK(cudaMemsetAsync(cx.shadow, 0, sizeof(__half) * cx.shadow_elems, cx.stream));
    std::vector<float> cs, sn;
    rope_tables(c, cs, sn);
    MM_CUDA_CHECK(cudaMemcpyAsync(cx.cos_t, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, cx.stream));
    MM_CUDA_CHECK(cudaMemcpyAsync(cx.sin_t, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, cx.stream));
    MM_CUDA_CHECK(cudaMemcpyAsync(cx.d_params, cx.params.data(), cx.params.size() * sizeof(ParamDesc),
                                  cudaMemcpyHostToDevice, cx.stream));
    // device scalars
    cx.n_partial = 1184;  // 8 blocks per SM on 148 SMs
    auto plan_s = [&](auto& a) {
        cx.d_err = a.template take<int>(4);
        cx.d_partial = a.template take<double>(cx.n_partial);
        cx.d_norm = a.template take<double>(1);
        cx.d_gs = a.template take<float>(1);
        cx.d_nonfinite = a.template take<int>(1);
        cx.d_nonfinite_out = a.template take<int>(1);
        cx.d_sums = a.template take<GrpoSums>(1);
        cx.d_scale = a.template take<float>(2);
        cx.d_any = a.template take<int>(2);  // [flag, a rank's batch was invalid]
        cx.d_one = a.template take<float>(1);
    };
    Sizer s2;
    plan_s(s2);
    cx.scalars.reserve(s2.used() + 1024);
    plan_s(cx.scalars);
    MM_CUDA_CHECK(cudaMemsetAsync(cx.d_err, 0, 16, cx.stream));
    const float one = 1.f;
    MM_CUDA_CHECK(cudaMemcpyAsync(cx.d_one, &one, 4, cudaMemcpyHostToDevice, cx.stream));
    MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
}

// Reads and clears the device error word; raises gpu_error on anything recorded.
inline void check_device(Context& cx, const char* where) {
    MM_CUDA_CHECK(cudaGetLastError());
    int err = 0;
    MM_CUDA_CHECK(cudaMemcpyAsync(&err, cx.d_err, 4, cudaMemcpyDeviceToHost, cx.stream));
    MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
    if (err) {
        MM_CUDA_CHECK(cudaMemsetAsync(cx.d_err, 0, 4, cx.stream));
        if (err & kErrBadIndex) fail(MM_INVALID_ARGUMENT, std::string(where) + ": token id out of range");
        if (err & kErrNonfinite) fail(MM_NUMERICAL_ERROR, std::string(where) + ": nonfinite value");
        cx.unusable = true;
        fail(MM_GPU_ERROR, std::string(where) + ": device wait timed out (error word " + std::to_string(err) + ")");
    }
}

// fp16 shadow of every matrix and the absorbed decode weights, from the fp32 master.
inline void refresh_derived(Context& cx, bool shadows) {
    const Dims& c = cx.c;
    if (shadows) {
        dim3 grid(256, static_cast<unsigned>(cx.params.size()));
        launch_k(cx.stream, shadow_refresh_kernel, grid, dim3(256), 0, cx.d_params, cx.w, cx.shadow);
        ++cx.launches;
    }
    for (int l = 0; l < c.L; ++l) {
        PrepArgs a;
        a.w_dq = cx.W(l, kWdq); a.w_dkv = cx.W(l, kWdkv); a.w_uq = cx.W(l, kWuq); a.w_uk = cx.W(l, kWuk);
        a.w_uv = cx.W(l, kWuv); a.w_o = cx.W(l, kWo); a.w_gate = cx.W(l, kWgate); a.w_up = cx.W(l, kWup);
        const PrepLayer& p = cx.prep[l];
        a.Wa = p.Wa; a.Wq = p.Wq; a.Wo = p.Wo; a.Wgu = p.Wgu;
        a.lda = p.lda; a.ldq = p.ldq; a.ldo = p.ldo; a.ldgu = p.ldgu;
        a.d = c.d; a.qr = c.qr; a.kvr = c.kvr; a.rope = c.rope; a.nope = c.nope; a.dv = c.dv;
        a.H = c.H; a.dff = c.dff;
        launch_k(cx.stream, decode_prep_kernel, dim3(592), dim3(256), 0, a);
        ++cx.launches;
        if (p.Wf) {  // the fused decode step's query weights, from the fp32 sums
            const int n = c.H * c.kvw();
            launch_k(cx.stream, absorbed_wq32_kernel, dim3(148), dim3(256), 0, a, cx.wq32);
            launch_k(cx.stream, fold_wq_kernel, dim3((n + 15) / 16, (c.d + 15) / 16), dim3(256), 0,
                     (const float*)cx.W(l, kWdq), (const float*)cx.W(l, kQNorm), (const float*)cx.wq32, c.d, c.qr, n,
                     p.Wf, p.ldf);
            cx.launches += 2;
        }
    }
}

inline void upload_params(Context& cx, const float* params, const float* m, const float* v, uint64_t steps) {
    std::vector<float> buf(static_cast<size_t>(cx.P_dev), 0.f);
    auto scatter = [&](const float* src) {
        std::fill(buf.begin(), buf.end(), 0.f);
        for (size_t i = 0; i < cx.params.size(); ++i) {
            const auto& p = cx.params[i];
            std::memcpy(buf.data() + p.off, src + cx.flat_off[i], sizeof(float) * p.rows * p.cols);
        }
    };
    for (size_t i = 0; i < static_cast<size_t>(cx.P); ++i)
        if (!std::isfinite(params[i])) fail(MM_INVALID_ARGUMENT, "nonfinite parameter");
    scatter(params);
    MM_CUDA_CHECK(cudaMemcpyAsync(cx.w, buf.data(), sizeof(float) * cx.P_dev, cudaMemcpyHostToDevice, cx.stream));
    MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
    if (cx.trainable) {
        if (m) {
            scatter(m);
            MM_CUDA_CHECK(cudaMemcpyAsync(cx.m, buf.data(), sizeof(float) * cx.P_dev, cudaMemcpyHostToDevice, cx.stream));
            MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
        } else {
            MM_CUDA_CHECK(cudaMemsetAsync(cx.m, 0, sizeof(float) * cx.P_dev, cx.stream));
        }
        if (v) {
            scatter(v);
            MM_CUDA_CHECK(cudaMemcpyAsync(cx.v, buf.data(), sizeof(float) * cx.P_dev, cudaMemcpyHostToDevice, cx.stream));
            MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
        } else {
            MM_CUDA_CHECK(cudaMemsetAsync(cx.v, 0, sizeof(float) * cx.P_dev, cx.stream));
        }
        MM_CUDA_CHECK(cudaMemsetAsync(cx.g, 0, sizeof(float) * cx.P_dev, cx.stream));
    }
    cx.steps = steps;
    refresh_derived(cx, true);
    check_device(cx, "upload");
}

inline void download(Context& cx, float* params, float* grads, float* m, float* v) {
    std::vector<float> buf(static_cast<size_t>(cx.P_dev));
    auto gather = [&](const float* dev, float* dst) {
        MM_CUDA_CHECK(cudaMemcpyAsync(buf.data(), dev, sizeof(float) * cx.P_dev, cudaMemcpyDeviceToHost, cx.stream));
        MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
        for (size_t i = 0; i < cx.params.size(); ++i) {
            const auto& p = cx.params[i];
            std::memcpy(dst + cx.flat_off[i], buf.data() + p.off, sizeof(float) * p.rows * p.cols);
        }
    };
    if (params) gather(cx.w, params);
    if ((grads || m || v) && !cx.trainable) fail(MM_INVALID_ARGUMENT, "inference context has no gradients or moments");
    if (grads) gather(cx.g, grads);
    if (m) gather(cx.m, m);
    if (v) gather(cx.v, v);
}

} // namespace mm
