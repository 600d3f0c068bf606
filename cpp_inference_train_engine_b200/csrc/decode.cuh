// Batched rollout decoding over the compressed latent cache (CpuDecoder, inference.cpp:47-174,
// absorbed form), on-device sampling (sample_token, inference.cpp:345-426) and the batched
// rollout() of trainer.cpp:187-213.
#pragma once
#include "decode_mk.cuh"
#include "passes.cuh"

namespace mm {

// Timestamps one traced fused decode step can record (start, every barrier, end).
constexpr int kMkTraceSlots = 320;

// Context splits of the tensor-core decode attention: enough CTAs for ~2 per SM when the
// batch alone does not provide them, at least 4 tiles of 16 positions per split.
constexpr int kMaxDecodeSplits = 16;
// Context splits of the latent decode attention (one warp per row and split): enough warps
// for ~8 per SM when the batch alone does not provide them, at least 4 tiles of 16
// positions per split.
// Warps the split latent attention aims for per launch (MM_DECODE_TARGET_WARPS, for tuning).
inline int decode_target_warps() {
    static const int v = [] {
        const char* e = std::getenv("MM_DECODE_TARGET_WARPS");
        const int x = e ? std::atoi(e) : 0;
        return x > 0 ? x : dec::kTargetWarps;
    }();
    return v;
}

inline int decode_splits(int B, int ctx) {
    const int target = decode_target_warps();
    if (B >= target) return 1;
    const int want = (target + B - 1) / B;
    const int by_len = std::max(1, (ctx + 63) / 64);
    return std::max(1, std::min(std::min(want, by_len), kMaxDecodeSplits));
}

// Latent decode attention (+ split combine) on the context stream.
// cos_t/sin_t given: q holds the unrotated rope part, rotated to position pos[b] on load.
inline void launch_decode_attention(Context& cx, const float* q, const __half* cache, long long seq_stride,
                                    const int* pos, int B, int ns, float scale, __half* out, float* part,
                                    const float* cos_t = nullptr, const float* sin_t = nullptr) {
    set_dynamic_smem<decode_attention_row_kernel>(dec::kRowSmem);
    MM_LAUNCH(decode_attention_row_kernel, blocks_for(static_cast<long long>(B) * ns, dec::kWarps), 32 * dec::kWarps,
              dec::kRowSmem, q, cache, seq_stride, pos, B, ns, scale, out, part, cos_t, sin_t);
    if (ns > 1)
        MM_LAUNCH(decode_attention_combine_kernel, blocks_for(static_cast<long long>(B) * dec::H * 32, 128), 128, 0, part,
                  ns, B, out);
}

// Context splits of the 16-head tensor-core form: enough (row, split) work items for
// decw::kTargetItems CTAs, at least 4 tiles of 32 positions per split.
inline int decode_splits_wide(int B, int ctx) {
    if (B >= decw::kTargetItems) return 1;
    const int want = (decw::kTargetItems + B - 1) / B;
    const int by_len = std::max(1, (ctx + 127) / 128);
    return std::max(1, std::min(std::min(want, by_len), kMaxDecodeSplits));
}

// MM_WIDE_ATTENTION=0 keeps the 2,048-wide model's decode attention on the CUDA-core form
// (for comparison).
inline bool wide_attention_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("MM_WIDE_ATTENTION");
        return !(e && e[0] == '0');
    }();
    return on;
}

inline void ensure_decode(Context& cx, int B, int Sc, int max_new) {
    DecodeState& d = cx.dec;
    if (d.B == B && d.Sc >= Sc && d.max_new >= max_new && d.arena.capacity()) return;
    const Dims& c = cx.c;
    MM_CUDA_CHECK(cudaStreamSynchronize(cx.stream));
    auto plan = [&](auto& a) {
        d.cache = a.template take<__half>(static_cast<long long>(c.L) * B * Sc * c.kvw());
        d.pos = a.template take<int>(B);
        d.x = a.template take<float>(static_cast<long long>(B) * c.d);
        d.h16 = a.template take<__half>(static_cast<long long>(B) * cx.d16(c.d));
        d.y = a.template take<float>(static_cast<long long>(B) * (c.qr + c.kvw()));
        d.cq16 = a.template take<__half>(static_cast<long long>(B) * cx.d16(c.qr));
        d.lat16 = a.template take<__half>(static_cast<long long>(B) * cx.d16(c.kvr));
        d.k_rope = a.template take<float>(static_cast<long long>(B) * c.rope);
        d.qf = a.template take<float>(static_cast<long long>(B) * c.H * c.kvw());
        d.qf2 = a.template take<float>(static_cast<long long>(B) * c.H * c.kvw());
        d.ctx16 = a.template take<__half>(static_cast<long long>(B) * c.H * c.kvr);
        d.res = a.template take<float>(static_cast<long long>(B) * c.d);
        d.h2 = a.template take<__half>(static_cast<long long>(B) * cx.d16(c.d));
        d.gu = a.template take<__half>(static_cast<long long>(B) * cx.d16(2 * c.dff));
        d.gated = a.template take<__half>(static_cast<long long>(B) * cx.d16(c.dff));
        d.hf = a.template take<float>(static_cast<long long>(B) * c.d);
        d.h3 = a.template take<__half>(static_cast<long long>(B) * cx.d16(3 * c.d));
        d.logits = a.template take<float>(static_cast<long long>(B) * c.V);
        d.tok = a.template take<uint16_t>(B);
        d.seeds = a.template take<uint64_t>(B);
        d.draw = a.template take<int>(B);
        d.out_tok = a.template take<uint16_t>(static_cast<long long>(B) * std::max(max_new, 1));
        // flash-decoding partials (max, sum, O[kv_rank]) per split and head
        d.part = a.template take<float>(B >= std::max(decode_target_warps(), decw::kTargetItems)
                                            ? 1 : static_cast<long long>(B) * kMaxDecodeSplits * c.H * (c.kvr + 2));
        d.step = a.template take<int>(1);
        d.active = a.template take<int>(B);
        d.mk_part = a.template take<float>(static_cast<long long>(mk::kMaxKs) * B * c.d);
        d.mk_cnt = a.template take<int>(B);
        d.mk_qs = a.template take<float>(B);
        d.mk_bar = a.template take<unsigned>(1);
        d.mk_trace = a.template take<unsigned long long>(kMkTraceSlots);
    };
    d.drop_graph();
    d.B = B;
    d.Sc = Sc;
    d.max_new = max_new;
    Sizer sz;
    plan(sz);
    // and the teacher-forced workspace makes room for the cache (the next pass re-creates it)
    if (!d.arena.fits(sz.used() + 4096) && cx.ws_arena.capacity()) {
        cx.ws_arena.release();
        cx.ws.T = 0;
        cx.ws.tape = false;  // a released workspace holds no tape: the next request plans its own
    }
    d.arena.release();
    d.arena.reserve(sz.used() + 4096);
    plan(d.arena);
    MM_CUDA_CHECK(cudaMemsetAsync(d.mk_cnt, 0, sizeof(int) * B, cx.stream));
}

// The fused decode step (decode_mk_kernel) runs for the 35.8M model's shapes unless
// MM_DECODE_MK=0 (then every layer is its own chain of launches; same arithmetic up to the
// order of fp32 additions).
inline bool decode_mk_enabled(const Context& cx) {
    static const bool on = [] {
        const char* e = std::getenv("MM_DECODE_MK");
        return !(e && e[0] == '0');
    }();
    // rows up to which the fused step is used (MM_DECODE_MK_MAX_ROWS). Per step, fused vs one
    // launch chain per layer (decode_bench, 128 + 64 tokens): 768 rows 0.744 vs 0.897 ms,
    // 1,024 0.819 vs 0.965, 1,536 1.100 vs 1.144, 2,048 1.201 vs 1.251
    static const int max_rows = [] {
        const char* e = std::getenv("MM_DECODE_MK_MAX_ROWS");
        const int v = e ? std::atoi(e) : 0;
        return v > 0 ? v : 4096;
    }();
    // (the folded query weights exist for that shape only)
    return on && cx.dec.B <= max_rows && mk_shape(cx.c) && cx.prep[0].Wf;
}

// Launches decode_mk_kernel for the rows of cx.dec: embedding of dec.tok through the h3 rows
// of the vocabulary head, cache rows written at dec.pos, positions advanced. One CTA per SM
// (cooperative launch, so every CTA is resident for the grid barriers).
inline void launch_decode_mk(Context& cx) {
    const Dims& c = cx.c;
    DecodeState& d = cx.dec;
    const int B = d.B;
    const int G = sm_count();
    MkParams p{};
    p.a_h16 = tensor_map(d.h16, false, mk::D, B, cx.d16(c.d), 64, 128);
    p.a_ctx16 = tensor_map(d.ctx16, false, mk::HKV, B, mk::HKV, 64, 128);
    p.a_h2 = tensor_map(d.h2, false, mk::D, B, cx.d16(c.d), 64, 128);
    p.a_gated = tensor_map(d.gated, false, mk::DFF, B, cx.d16(c.dff), 64, 128);
    for (int l = 0; l < c.L; ++l) {
        const PrepLayer& w = cx.prep[l];
        p.wa[l] = tensor_map(w.Wa, false, mk::QKV, mk::D, w.lda, 64, 64);
        p.wf[l] = tensor_map(w.Wf, false, mk::QW, mk::D, w.ldf, 64, 64);
        p.wo[l] = tensor_map(w.Wo, false, mk::D, mk::HKV, w.ldo, 64, 64);
        p.wgu[l] = tensor_map(w.Wgu, false, 2 * mk::DFF, mk::D, w.ldgu, 64, 64);
        p.wdown[l] = tensor_map(cx.S(l, kWdown), false, mk::D, mk::DFF, cx.SL(l, kWdown), 64, 64);
        const void* wb[5] = {w.Wa, w.Wf, w.Wo, w.Wgu, cx.S(l, kWdown)};
        const long long wn[5] = {2LL * mk::D * w.lda, 2LL * mk::D * w.ldf, 2LL * mk::HKV * w.ldo,
                                 2LL * mk::D * w.ldgu, 2LL * mk::DFF * cx.SL(l, kWdown)};
        for (int k = 0; k < 5; ++k) {
            p.wbase[l][k] = wb[k];
            p.wbytes[l][k] = wn[k];
        }
        p.attn_norm[l] = cx.W(l, kAttnNorm);
        p.ffn_norm[l] = cx.W(l, kFfnNorm);
        p.q_norm[l] = cx.W(l, kQNorm);
        p.kv_norm[l] = cx.W(l, kKvNorm);
    }
    p.final_norm = cx.FinalNorm();
    p.E = cx.E();
    p.tok = d.tok;
    p.V = c.V;
    p.B = B;
    p.L = c.L;
    p.Sc = d.Sc;
    // context splits: as many as keep every (row, split) item within half the grid's warps (at
    // least two 16-position tiles per split): the merge of the splits costs more than the
    // longer per-item tile loop (512 rows, 128 + 64 tokens: 0.675 ms per step with 1 split per
    // row, 0.694 with 2; 64 and 256 rows unchanged)
    p.ns = std::max(1, std::min(std::min(kMaxDecodeSplits, G * mk::kWarps / (2 * B)), (cx.dec_len + 1 + 31) / 32));
    // K splits of the residual products: about one wave of (split, m-tile, n-tile) units
    const int MT = (B + 127) / 128;
    auto pick = [&](int nk, int maxks, int& ks, int& per) {
        const int want = std::max(1, std::min(maxks, G / (MT * (mk::D / 128))));
        per = (nk + want - 1) / want;
        ks = (nk + per - 1) / per;
    };
    pick(mk::HKV / 64, 4, p.ks_o, p.per_o);
    pick((mk::DFF + 63) / 64, mk::kMaxKs, p.ks_d, p.per_d);
    p.eps = c.eps;
    p.scale = 1.0f / std::sqrt(static_cast<float>(c.qk()));
    p.x = d.x;
    p.h16 = d.h16;
    p.qs = d.mk_qs;
    p.qf = d.qf;
    p.ctx16 = d.ctx16;
    p.h2 = d.h2;
    p.gated = d.gated;
    p.h3 = d.h3;
    p.ld3 = cx.d16(3 * c.d);
    p.part = d.mk_part;
    p.attn_part = d.part;
    p.attn_cnt = d.mk_cnt;
    p.cache = d.cache;
    p.pos = d.pos;
    p.cos_t = cx.cos_t;
    p.sin_t = cx.sin_t;
    p.bar = d.mk_bar;
    p.err = cx.d_err;
    p.trace = d.mk_trace_on ? d.mk_trace : nullptr;
    set_dynamic_smem<decode_mk_kernel>(mk::kSmem);
    MM_CUDA_CHECK(cudaMemsetAsync(d.mk_bar, 0, sizeof(unsigned), cx.stream));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(mk::kThreads);
    cfg.dynamicSmemBytes = mk::kSmem;
    cfg.stream = cx.stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaEvent_t t0 = cx.prof_begin();
    MM_CUDA_CHECK(cudaLaunchKernelEx(&cfg, decode_mk_kernel, p));
    cx.prof_end(kKOther, t0);
    ++cx.launches;
}

// Prefill of rows [0, B) from device prompts [B][P] (already in ws-independent storage):
// runs the teacher-forced forward in chunks that fit the workspace, writing the cache and
// the last-position logits into dec.logits.
inline void prefill_rows(Context& cx, const uint16_t* d_prompts, int B, int P, int chunk_tokens) {
    DecodeState& d = cx.dec;
    const int per = std::max(1, chunk_tokens / P);
    ensure_workspace(cx, std::min(B, per) * P, false);  // reuses a larger workspace with tape
    for (int r0 = 0; r0 < B; r0 += per) {
        const int bc = std::min(per, B - r0);
        MM_CUDA_CHECK(cudaMemcpyAsync(cx.ws.tokens, d_prompts + static_cast<long long>(r0) * P,
                                      sizeof(uint16_t) * bc * P, cudaMemcpyDeviceToDevice, cx.stream));
        forward_chunk(cx, bc, P, false, kVocabLast, false, d.cache, d.Sc, r0, d.logits + static_cast<long long>(r0) * cx.c.V);
    }
    std::vector<int> pos(B, P);
    MM_CUDA_CHECK(cudaMemcpyAsync(d.pos, pos.data(), sizeof(int) * B, cudaMemcpyHostToDevice, cx.stream));
}

// Serving: free slots decode a dummy token at position 0 of their own cache row, so their
// positions never run past the row (the step advances every row).
__global__ void serve_prepare_kernel(int* __restrict__ pos, uint16_t* __restrict__ tok, const int* __restrict__ active,
                                     int B) {
    MM_PDL_ENTRY();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B && !active[b]) {
        pos[b] = 0;
        tok[b] = 0;
    }
}

__global__ void advance_pos_kernel(int* pos, int B) {
    MM_PDL_ENTRY();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) pos[b] += 1;
}

// One decode step for every row: dec.tok holds the tokens to append at dec.pos.
inline void decode_step(Context& cx) {
    const Dims& c = cx.c;
    DecodeState& d = cx.dec;
    const int B = d.B, kvw = c.kvw(), qrk = c.qr + kvw;
    const int ld_d = cx.d16(c.d), ld_qr = cx.d16(c.qr), ld_kvr = cx.d16(c.kvr);
    if (decode_mk_enabled(cx)) {
        launch_decode_mk(cx);  // every layer, the final norm and the positions' advance
        GemmOutSpec lo{d.logits, c.V, kOutF32};
        lo.alpha = 1.0f / kVocabScale;
        gemm(cx, B, c.V, 3 * c.d, {d.h3, cx.d16(3 * c.d), false}, {cx.E3(), cx.E3L(), false}, lo);
        return;
    }
    MM_LAUNCH(embed_kernel, warp_rows_grid(B), 256, 0, d.tok, cx.E(), d.x, B, c.d, c.V, cx.d_err);
    for (int l = 0; l < c.L; ++l) {
        const PrepLayer& p = cx.prep[l];
        launch_rmsnorm(cx, d.x, c.d, cx.W(l, kAttnNorm), B, c.d, (float*)nullptr, 0LL, d.h16, ld_d);
        gemm(cx, B, qrk, c.d, {d.h16, ld_d, false}, {p.Wa, p.lda, true}, {d.y, qrk, kOutF32});
        const bool fused_latent = c.qr % 4 == 0 && c.kvr % 4 == 0 && c.rope % 4 == 0 && qrk % 4 == 0 && qrk <= 512 &&
                                  ld_qr % 4 == 0;
        __half* cache_l = d.cache + static_cast<long long>(l) * B * d.Sc * kvw;
        if (fused_latent) {
            MM_LAUNCH(latent_kernel, warp_rows_grid(B), 256, 0, d.y, (long long)qrk, c.qr, c.kvr, c.rope, cx.W(l, kQNorm),
                      cx.W(l, kKvNorm), c.eps, B, 1, (const int*)d.pos, 0, cx.cos_t, cx.sin_t, d.cq16, (long long)ld_qr,
                      (__half*)nullptr, 0LL, (float*)nullptr, cache_l, d.Sc);
        } else {
            launch_rmsnorm(cx, d.y, qrk, cx.W(l, kQNorm), B, c.qr, (float*)nullptr, 0LL, d.cq16, ld_qr);
            launch_rmsnorm(cx, d.y + c.qr, qrk, cx.W(l, kKvNorm), B, c.kvr, (float*)nullptr, 0LL, d.lat16, ld_kvr);
            MM_LAUNCH(rope_key_kernel, blocks_for((long long)B * (c.rope / 2), 256), 256, 0, d.y + c.qr, (long long)qrk, c.kvr,
                      c.rope, B, 1, d.pos, cx.cos_t, cx.sin_t, d.k_rope, (__half*)nullptr, 0LL);
            MM_LAUNCH(cache_write_kernel, blocks_for((long long)B * kvw, 256), 256, 0, d.lat16, (long long)ld_kvr, d.k_rope, B, 1,
                      d.pos, 0, cache_l, d.Sc, c.kvr, c.rope);
        }
        gemm(cx, B, c.H * kvw, c.qr, {d.cq16, ld_qr, false}, {p.Wq, p.ldq, true}, {d.qf, c.H * kvw, kOutF32});
        const bool mma_attn = c.kvr == dec::KV && c.rope == dec::R && c.H == dec::H;
        // the tensor-core attention rotates the rope part of q while loading it
        if (!mma_attn)
            launch_rope_rows(cx, d.qf, (c.H * kvw), B, 1, d.pos, c.H, kvw, c.kvr, c.rope, 0, d.qf2, (c.H * kvw),
                             (__half*)nullptr, 0LL);
        {
            const float scale = 1.0f / std::sqrt(static_cast<float>(c.qk()));
            // cache rows read once (fp16) + absorbed queries in (fp32) + context out (fp16)
            const double bytes = static_cast<double>(B) * ((cx.dec_len + 1.0) * kvw * 2 + c.H * kvw * 4.0 + c.H * c.kvr * 2.0);
            if (mma_attn) {
                const int ns = decode_splits(B, cx.dec_len + 1);
                cudaEvent_t t0 = cx.prof_begin();
                launch_decode_attention(cx, d.qf, cache_l, (long long)d.Sc * kvw, d.pos, B, ns, scale, d.ctx16, d.part,
                                        cx.cos_t, cx.sin_t);
                cx.prof_end(kKDecodeAttn, t0, bytes);
            } else if (c.kvr == decw::KV && c.rope == decw::R && c.H == decw::H && wide_attention_enabled()) {
                const int ns = decode_splits_wide(B, cx.dec_len + 1);
                cudaEvent_t t0 = cx.prof_begin();
                set_dynamic_smem<decode_attention_wide_kernel>(decw::kSmem);
                MM_LAUNCH(decode_attention_wide_kernel, B * ns, decw::kThreads, decw::kSmem, d.qf2, cache_l,
                          (long long)d.Sc * kvw, d.pos, B, ns, scale, d.ctx16, d.part);
                if (ns > 1)
                    MM_LAUNCH(decode_attention_wide_combine_kernel, blocks_for(static_cast<long long>(B) * decw::H * 32, 128),
                              128, 0, d.part, ns, B, d.ctx16);
                cx.prof_end(kKDecodeAttn, t0, bytes);
            } else if (c.kvr == 512) {
                set_dynamic_smem<decode_attention_kernel<512, 32>>(decode_attention_smem<512, 32>(kMaxDecodeHeads));
                MM_LAUNCH_TIMED(kKDecodeAttn, bytes, (decode_attention_kernel<512, 32>), B, 32 * c.H,
                                (decode_attention_smem<512, 32>(c.H)), d.qf2, cache_l, (long long)d.Sc * kvw, d.pos, c.H,
                                scale, d.ctx16);
            } else if (c.kvr == 128) {
                set_dynamic_smem<decode_attention_kernel<128, 16>>(decode_attention_smem<128, 16>(kMaxDecodeHeads));
                MM_LAUNCH_TIMED(kKDecodeAttn, bytes, (decode_attention_kernel<128, 16>), B, 32 * c.H,
                                (decode_attention_smem<128, 16>(c.H)), d.qf2, cache_l, (long long)d.Sc * kvw, d.pos, c.H,
                                scale, d.ctx16);
            } else {
                MM_LAUNCH_TIMED(kKDecodeAttn, bytes, (decode_attention_kernel<8, 4>), B, 32 * c.H,
                                (decode_attention_smem<8, 4>(c.H)), d.qf2, cache_l, (long long)d.Sc * kvw, d.pos, c.H,
                                scale, d.ctx16);
            }
        }
        {
            GemmOutSpec o{d.x, c.d, kOutF32Acc};  // residual stream updated in place
            o.ldr = c.d;
            gemm(cx, B, c.d, c.H * c.kvr, {d.ctx16, c.H * c.kvr, false}, {p.Wo, p.ldo, true}, o);
        }
        launch_rmsnorm(cx, d.x, c.d, cx.W(l, kFfnNorm), B, c.d, (float*)nullptr, 0LL, d.h2, ld_d);
        const int ld_gu = cx.d16(2 * c.dff), ld_ff = cx.d16(c.dff);
        if (c.dff % 8) {
            gemm(cx, B, 2 * c.dff, c.d, {d.h2, ld_d, false}, {p.Wgu, p.ldgu, true}, {d.gu, ld_gu, kOutF16});
            launch_swiglu(cx, d.gu, d.gu + c.dff, ld_gu, B, c.dff, d.gated, ld_ff);
        } else {
            GemmOutSpec o{d.gated, ld_ff, kOutF16};
            o.glu_n = c.dff;
            gemm(cx, B, c.dff, c.d, {d.h2, ld_d, false}, {p.Wgu, p.ldgu, true}, o);
        }
        {
            GemmOutSpec o{d.x, c.d, kOutF32Acc};
            o.ldr = c.d;
            gemm(cx, B, c.d, c.dff, {d.gated, ld_ff, false}, {cx.S(l, kWdown), cx.SL(l, kWdown), true}, o);
        }
    }
    launch_rmsnorm(cx, d.x, c.d, cx.FinalNorm(), B, c.d, d.hf, c.d, (__half*)nullptr, 0LL);
    const int ld3 = cx.d16(3 * c.d);
    launch_split3(cx, d.hf, c.d, B, 1, 0, d.h3, ld3);
    GemmOutSpec lo{d.logits, c.V, kOutF32};
    lo.alpha = 1.0f / kVocabScale;
    gemm(cx, B, c.V, 3 * c.d, {d.h3, ld3, false}, {cx.E3(), cx.E3L(), false}, lo);
    MM_LAUNCH(advance_pos_kernel, blocks_for(B, 256), 256, 0, d.pos, B);
}

inline void launch_sample(Context& cx, const float* logits, int B, float temperature, const uint64_t* seeds,
                          const int* draw, int draw_offset, const int* active, uint16_t* out, long long out_stride,
                          const int* counter = nullptr) {
    MM_LAUNCH_TIMED(kKSample, 4.0 * B * cx.c.V, sample_kernel, B, kSampleThreads, 0, logits, (long long)cx.c.V, cx.c.V,
                    temperature, seeds, draw, draw_offset, counter, active, out, out_stride);
}

__global__ void counter_add_kernel(int* c, int v) {
    MM_PDL_ENTRY(); *c += v; }

// out_tok column (*counter - 1) -> tok, for the token to append at this step.
__global__ void column_gather_counter_kernel(const uint16_t* __restrict__ src, long long stride,
                                             const int* __restrict__ counter, int B, uint16_t* __restrict__ dst) {
    MM_PDL_ENTRY();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b < B) dst[b] = src[b * stride + *counter - 1];
}

// One rollout decode step as a replayable unit: step += 1; append out_tok[:, step - 1] at
// every row's position; logits; sample draw `step` into out_tok[:, step].
inline void decode_sample_step(Context& cx, int completion, float temperature) {
    DecodeState& d = cx.dec;
    const int n = d.B;
    MM_LAUNCH(counter_add_kernel, 1, 1, 0, d.step, 1);
    MM_LAUNCH(column_gather_counter_kernel, blocks_for(n, 256), 256, 0, d.out_tok, (long long)completion, d.step, n, d.tok);
    decode_step(cx);
    launch_sample(cx, d.logits, n, temperature, d.seeds, nullptr, 0, nullptr, d.out_tok, completion, d.step);
}

} // namespace mm
