// Fused AdamW (Optimizer::step, optimizer.cpp:105-161; Metal adamw.metal:21-70) over the
// device parameter arena, and the derived fp16 weights the tensor-core passes read.
//
//   adamw_norm_partial_kernel  per-block sum of g^2 in double + non-finite flag
//   adamw_finalize_kernel      global norm (double), clip scale gs (float), in fixed order
//   adamw_update_kernel        m, v, w update in float with the reference's exact operation
//                              order (no fused multiply-add), then the fp16 shadow copy
//   decode_prep_kernel         absorbed decode projections (inference.cpp:28-46 and the
//                              W_uk absorption of inference.cpp:120-124)
#pragma once
#include "common.cuh"

namespace mm {

enum ShadowKind : int { kShadowNone = 0, kShadowHalf = 1, kShadowVocab3 = 2 };

struct ParamDesc {
    long long off;        // offset in the fp32 arenas (master, grad, m, v)
    int rows, cols;
    float decay;          // weight decay (0 for norm scales)
    int shadow_kind;
    long long shadow_off; // offset in the fp16 arena
    int shadow_ld;        // row pitch of the shadow (elements)
};

// Scale of the vocabulary table before its hi/lo fp16 split: keeps the low part of
// 0.02-sized weights out of the fp16 subnormal range. Logits are scaled back by 1/64.
constexpr float kVocabScale = 64.0f;

__global__ void adamw_norm_partial_kernel(const float* __restrict__ g, long long n,
                                          double* __restrict__ partial, int* __restrict__ nonfinite) {
    MM_PDL_ENTRY();
    __shared__ double red[32];
    double s = 0.0;
    bool bad = false;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float v = g[i];
        if (!isfinite(v)) bad = true;
        s += static_cast<double>(v) * static_cast<double>(v);
    }
    if (bad) atomicOr(nonfinite, 1);
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double a = 0.0;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) a += red[w];
        partial[blockIdx.x] = a;
    }
}

// out[0] = norm (double), gs (float) written to gs_out. clip <= 0 disables clipping.
__global__ void adamw_finalize_kernel(const double* __restrict__ partial, int nparts, float clip,
                                      double* __restrict__ norm_out, float* __restrict__ gs_out) {
    MM_PDL_ENTRY();
    __shared__ double red[32];
    double s = 0.0;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += partial[i];
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double a = 0.0;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) a += red[w];
        const double norm = sqrt(a);
        norm_out[0] = norm;
        gs_out[0] = clip > 0.f ? static_cast<float>(fmin(1.0, static_cast<double>(clip) / fmax(norm, 1e-30))) : 1.0f;
    }
}

// One block column per parameter (blockIdx.y). Skips every write when `skip` is set (a
// non-finite gradient: the reference fails before mutating anything).
__global__ void adamw_update_kernel(const ParamDesc* __restrict__ params, float* __restrict__ w,
                                    const float* __restrict__ g, float* __restrict__ m,
                                    float* __restrict__ v, __half* __restrict__ shadow,
                                    const float* __restrict__ gs_ptr, const int* __restrict__ skip,
                                    float lr, float beta1, float beta2, float eps, float bc1,
                                    float bc2, int* __restrict__ nonfinite_out) {
    MM_PDL_ENTRY();
    if (*skip) return;
    const ParamDesc p = params[blockIdx.y];
    const long long n = static_cast<long long>(p.rows) * p.cols;
    const float gs = *gs_ptr;
    const float one_b1 = __fsub_rn(1.f, beta1), one_b2 = __fsub_rn(1.f, beta2);
    const float keep = __fsub_rn(1.f, __fmul_rn(lr, p.decay));
    bool bad = false;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long k = p.off + i;
        const float gi = __fmul_rn(g[k], gs);
        const float mi = __fadd_rn(__fmul_rn(beta1, m[k]), __fmul_rn(one_b1, gi));
        const float vi = __fadd_rn(__fmul_rn(beta2, v[k]), __fmul_rn(__fmul_rn(one_b2, gi), gi));
        const float den = __fadd_rn(__fsqrt_rn(__fdiv_rn(vi, bc2)), eps);
        const float wi = __fsub_rn(__fmul_rn(w[k], keep), __fdiv_rn(__fmul_rn(lr, __fdiv_rn(mi, bc1)), den));
        m[k] = mi;
        v[k] = vi;
        w[k] = wi;
        if (!isfinite(wi)) bad = true;
        if (p.shadow_kind == kShadowHalf) {
            const int r = static_cast<int>(i / p.cols), c = static_cast<int>(i % p.cols);
            shadow[p.shadow_off + static_cast<long long>(r) * p.shadow_ld + c] = __float2half_rn(wi);
        } else if (p.shadow_kind == kShadowVocab3) {
            const int r = static_cast<int>(i / p.cols), c = static_cast<int>(i % p.cols);
            const float s = wi * kVocabScale;
            const __half hi = __float2half_rn(s);
            const __half lo = __float2half_rn(s - __half2float(hi));
            __half* row = shadow + p.shadow_off + static_cast<long long>(r) * p.shadow_ld;
            row[c] = hi;
            row[p.cols + c] = hi;
            row[2 * p.cols + c] = lo;
        }
    }
    if (bad) atomicOr(nonfinite_out, 1);
}

// Shadow refresh without an update (after an upload): same layout as the update writes.
__global__ void shadow_refresh_kernel(const ParamDesc* __restrict__ params, const float* __restrict__ w,
                                      __half* __restrict__ shadow) {
    MM_PDL_ENTRY();
    const ParamDesc p = params[blockIdx.y];
    const long long n = static_cast<long long>(p.rows) * p.cols;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float wi = w[p.off + i];
        const int r = static_cast<int>(i / p.cols), c = static_cast<int>(i % p.cols);
        if (p.shadow_kind == kShadowHalf) {
            shadow[p.shadow_off + static_cast<long long>(r) * p.shadow_ld + c] = __float2half_rn(wi);
        } else if (p.shadow_kind == kShadowVocab3) {
            const float s = wi * kVocabScale;
            const __half hi = __float2half_rn(s);
            const __half lo = __float2half_rn(s - __half2float(hi));
            __half* row = shadow + p.shadow_off + static_cast<long long>(r) * p.shadow_ld;
            row[c] = hi;
            row[p.cols + c] = hi;
            row[2 * p.cols + c] = lo;
        }
    }
}

// Decode-side derived weights of one layer, from the fp32 master:
//   Wa  [d][q_rank + kv_rank + rope]      = [W_dq | W_dkv]
//   Wq  [q_rank][H*(kv_rank + rope)]      per head: [W_uq_nope,h . W_uk,h^T | W_uq_rope,h]
//   Wo  [H*kv_rank][d]                    per head: W_uv,h . W_o,h
//   Wgu [2 d][2*d_ff]                     = [W_gate | W_up] in fp16 (rows [0, d)), then the
//                                           rounding residual fp16(W - fp16(W)) (rows [d, 2d)):
//                                           the teacher-forced FFN's three-term product reads both
struct PrepArgs {
    const float *w_dq, *w_dkv, *w_uq, *w_uk, *w_uv, *w_o, *w_gate, *w_up;
    __half *Wa, *Wq, *Wo, *Wgu;
    int lda, ldq, ldo, ldgu;
    int d, qr, kvr, rope, nope, dv, H, dff;
};

__global__ void decode_prep_kernel(PrepArgs a) {
    MM_PDL_ENTRY();
    const int qk = a.nope + a.rope;
    const int kvw = a.kvr + a.rope;
    const long long nWa = static_cast<long long>(a.d) * (a.qr + kvw);
    const long long nWq = static_cast<long long>(a.qr) * a.H * kvw;
    const long long nWo = static_cast<long long>(a.H) * a.kvr * a.d;
    const long long nWgu = static_cast<long long>(a.d) * 2 * a.dff;
    const long long total = nWa + nWq + nWo + nWgu;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        long long j = i;
        if (j < nWa) {
            const int r = static_cast<int>(j / (a.qr + kvw)), c = static_cast<int>(j % (a.qr + kvw));
            const float v = c < a.qr ? a.w_dq[r * a.qr + c] : a.w_dkv[r * kvw + (c - a.qr)];
            a.Wa[static_cast<long long>(r) * a.lda + c] = __float2half_rn(v);
            continue;
        }
        j -= nWa;
        if (j < nWq) {
            const int r = static_cast<int>(j / (a.H * kvw)), c = static_cast<int>(j % (a.H * kvw));
            const int h = c / kvw, e = c % kvw;
            float v;
            if (e < a.kvr) {
                float s = 0.f;
                for (int n = 0; n < a.nope; ++n)
                    s += a.w_uq[r * a.H * qk + h * qk + n] * a.w_uk[e * a.H * a.nope + h * a.nope + n];
                v = s;
            } else {
                v = a.w_uq[r * a.H * qk + h * qk + a.nope + (e - a.kvr)];
            }
            a.Wq[static_cast<long long>(r) * a.ldq + c] = __float2half_rn(v);
            continue;
        }
        j -= nWq;
        if (j < nWo) {
            const int r = static_cast<int>(j / a.d), c = static_cast<int>(j % a.d);
            const int h = r / a.kvr, e = r % a.kvr;
            float s = 0.f;
            for (int k = 0; k < a.dv; ++k)
                s += a.w_uv[e * a.H * a.dv + h * a.dv + k] * a.w_o[(h * a.dv + k) * a.d + c];
            a.Wo[static_cast<long long>(r) * a.ldo + c] = __float2half_rn(s);
            continue;
        }
        j -= nWo;
        {
            const int r = static_cast<int>(j / (2 * a.dff)), c = static_cast<int>(j % (2 * a.dff));
            const float v = c < a.dff ? a.w_gate[r * a.dff + c] : a.w_up[r * a.dff + (c - a.dff)];
            const __half hi = __float2half_rn(v);
            a.Wgu[static_cast<long long>(r) * a.ldgu + c] = hi;
            a.Wgu[static_cast<long long>(a.d + r) * a.ldgu + c] = __float2half_rn(v - __half2float(hi));
        }
    }
}

// The absorbed query weights in fp32, [qr][H * (kvr + rope)]: per head the nope query folded
// into the latent (W_uq,nope,h . W_uk,h^T) and the rope query columns, the sums of
// decode_prep_kernel's Wq before its fp16 rounding. Grid-stride over the entries.
__global__ void absorbed_wq32_kernel(PrepArgs a, float* __restrict__ wq32) {
    MM_PDL_ENTRY();
    const int qk = a.nope + a.rope, kvw = a.kvr + a.rope;
    const long long n = static_cast<long long>(a.qr) * a.H * kvw;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(i / (a.H * kvw)), c = static_cast<int>(i % (a.H * kvw));
        const int h = c / kvw, e = c % kvw;
        float v;
        if (e < a.kvr) {
            float s = 0.f;
            for (int k = 0; k < a.nope; ++k)
                s += a.w_uq[r * a.H * qk + h * qk + k] * a.w_uk[e * a.H * a.nope + h * a.nope + k];
            v = s;
        } else {
            v = a.w_uq[r * a.H * qk + h * qk + a.nope + (e - a.kvr)];
        }
        wq32[i] = v;
    }
}

// The fused decode step's query weights: Wf = W_dq . diag(g_q) . Wq, [d][n] fp16 (row pitch
// ldf), so that the absorbed query of a row is rms_q^-1 * (h . Wf) with rms_q the q latent's
// RMS (its RMSNorm is a per-row scalar times diag(g_q)). fp32 sums over k in order; 16 x 16
// output tiles with their operand tiles in shared memory. grid (ceil(n / 16), ceil(d / 16)).
__global__ void fold_wq_kernel(const float* __restrict__ w_dq, const float* __restrict__ g_q,
                               const float* __restrict__ wq32, int d, int qr, int n, __half* __restrict__ wf,
                               int ldf) {
    MM_PDL_ENTRY();
    __shared__ float sa[16][17], sb[16][17];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int row = blockIdx.y * 16 + ty, col = blockIdx.x * 16 + tx;
    float acc = 0.f;
    for (int k0 = 0; k0 < qr; k0 += 16) {
        const int ka = k0 + tx, kb = k0 + ty;
        sa[ty][tx] = (row < d && ka < qr) ? w_dq[static_cast<long long>(row) * qr + ka] * g_q[ka] : 0.f;
        sb[ty][tx] = (kb < qr && col < n) ? wq32[static_cast<long long>(kb) * n + col] : 0.f;
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; ++k) acc += sa[ty][k] * sb[k][tx];
        __syncthreads();
    }
    if (row < d && col < n) wf[static_cast<long long>(row) * ldf + col] = __float2half_rn(acc);
}

} // namespace mm
