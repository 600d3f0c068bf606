// Attention kernels.
//
// Teacher-forced passes (ops::attention / ops::attention_backward, ops.cpp:109-172):
// causal softmax attention per (sequence, head) with qk = nope + rope and value width dv,
// computed tile by tile with an online softmax so the [T, T] probability matrix of the
// reference is never written. Forward stores the output (fp16) and the row log-sum-exp;
// backward recomputes probabilities from them. Tiles of 64 keys/queries are staged in
// shared memory; each thread owns one query (forward, dq) or one key (dk, dv).
//
// Decode (CpuDecoder::decode, inference.cpp:116-153, absorbed form): every head of a
// sequence attends over the same compressed cache row [latent kv_rank | rope], so one CTA
// per sequence stages cache tiles once and its warps (one per head) all read them.
#pragma once
#include "common.cuh"

namespace mm {

constexpr int kAttTile = 64;

// Forward. q, k: fp16 [B*S][H*QK]; v: fp16 [B*S][H*DV]. out fp16 [B*S][H*DV],
// lse fp32 [B*S][H] (natural log). grid (ceil(S/64), H, B), block 64.
template <int QK, int DV>
__global__ void __launch_bounds__(64) flash_fwd_kernel(const __half* __restrict__ q,
                                                       const __half* __restrict__ k,
                                                       const __half* __restrict__ v, int S, int H,
                                                       float scale, __half* __restrict__ out,
                                                       float* __restrict__ lse) {
    __shared__ float Ks[kAttTile][QK + 1];
    __shared__ float Vs[kAttTile][DV + 1];
    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int i = qt * kAttTile + threadIdx.x;  // query position
    const long long base = static_cast<long long>(b) * S;
    const int ldq = H * QK, ldv = H * DV;
    float qr[QK], o[DV];
    if (i < S) {
#pragma unroll
        for (int c = 0; c < QK; ++c) qr[c] = __half2float(q[(base + i) * ldq + h * QK + c]) * scale;
    }
#pragma unroll
    for (int c = 0; c < DV; ++c) o[c] = 0.f;
    float m = -INFINITY, l = 0.f;
    for (int kt = 0; kt <= qt; ++kt) {
        __syncthreads();
        for (int e = threadIdx.x; e < kAttTile * QK; e += blockDim.x) {
            const int r = e / QK, c = e % QK, j = kt * kAttTile + r;
            Ks[r][c] = j < S ? __half2float(k[(base + j) * ldq + h * QK + c]) : 0.f;
        }
        for (int e = threadIdx.x; e < kAttTile * DV; e += blockDim.x) {
            const int r = e / DV, c = e % DV, j = kt * kAttTile + r;
            Vs[r][c] = j < S ? __half2float(v[(base + j) * ldv + h * DV + c]) : 0.f;
        }
        __syncthreads();
        if (i < S) {
            const int jmax = min(kAttTile, i - kt * kAttTile + 1);
            for (int r = 0; r < jmax; ++r) {
                float s = 0.f;
#pragma unroll
                for (int c = 0; c < QK; ++c) s += qr[c] * Ks[r][c];
                if (s > m) {
                    const float corr = __expf(m - s);
                    l *= corr;
#pragma unroll
                    for (int c = 0; c < DV; ++c) o[c] *= corr;
                    m = s;
                }
                const float p = __expf(s - m);
                l += p;
#pragma unroll
                for (int c = 0; c < DV; ++c) o[c] += p * Vs[r][c];
            }
        }
    }
    if (i < S) {
        const float inv = 1.0f / l;
#pragma unroll
        for (int c = 0; c < DV; ++c) out[(base + i) * ldv + h * DV + c] = __float2half_rn(o[c] * inv);
        lse[(base + i) * H + h] = m + logf(l);
    }
}

// D[t, h] = sum_c dO[t, h, c] * O[t, h, c] (the softmax-backward row term).
__global__ void attn_bwd_dot_kernel(const float* __restrict__ dout, const __half* __restrict__ out,
                                    int T, int H, int DV, float* __restrict__ D) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= T * H) return;
    const int t = idx / H, h = idx % H;
    const long long o = static_cast<long long>(t) * H * DV + h * DV;
    float s = 0.f;
    for (int c = 0; c < DV; ++c) s += dout[o + c] * __half2float(out[o + c]);
    D[idx] = s;
}

// dK, dV for one key tile. dout fp32 [B*S][H*DV]. dk fp32 [B*S][H*QK] (already scaled by
// `scale`), dv fp32 [B*S][H*DV]. grid (ceil(S/64), H, B), block 64 (one key per thread).
template <int QK, int DV>
__global__ void __launch_bounds__(64) flash_bwd_dkdv_kernel(
    const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
    const float* __restrict__ dout, const float* __restrict__ lse, const float* __restrict__ D,
    int S, int H, float scale, float* __restrict__ dk, float* __restrict__ dv) {
    __shared__ float Qs[kAttTile][QK + 1];
    __shared__ float Gs[kAttTile][DV + 1];
    __shared__ float Ls[kAttTile], Ds[kAttTile];
    const int kt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int j = kt * kAttTile + threadIdx.x;
    const long long base = static_cast<long long>(b) * S;
    const int ldq = H * QK, ldv = H * DV;
    float kr[QK], vr[DV], dkr[QK], dvr[DV];
#pragma unroll
    for (int c = 0; c < QK; ++c) {
        kr[c] = j < S ? __half2float(k[(base + j) * ldq + h * QK + c]) : 0.f;
        dkr[c] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < DV; ++c) {
        vr[c] = j < S ? __half2float(v[(base + j) * ldv + h * DV + c]) : 0.f;
        dvr[c] = 0.f;
    }
    const int ntiles = (S + kAttTile - 1) / kAttTile;
    for (int qt = kt; qt < ntiles; ++qt) {
        __syncthreads();
        for (int e = threadIdx.x; e < kAttTile * QK; e += blockDim.x) {
            const int r = e / QK, c = e % QK, i = qt * kAttTile + r;
            Qs[r][c] = i < S ? __half2float(q[(base + i) * ldq + h * QK + c]) : 0.f;
        }
        for (int e = threadIdx.x; e < kAttTile * DV; e += blockDim.x) {
            const int r = e / DV, c = e % DV, i = qt * kAttTile + r;
            Gs[r][c] = i < S ? dout[(base + i) * ldv + h * DV + c] : 0.f;
        }
        {
            const int i = qt * kAttTile + threadIdx.x;
            Ls[threadIdx.x] = i < S ? lse[(base + i) * H + h] : 0.f;
            Ds[threadIdx.x] = i < S ? D[(base + i) * H + h] : 0.f;
        }
        __syncthreads();
        if (j < S) {
            const int rmin = qt == kt ? threadIdx.x : 0;
            const int rmax = min(kAttTile, S - qt * kAttTile);
            for (int r = rmin; r < rmax; ++r) {
                float s = 0.f;
#pragma unroll
                for (int c = 0; c < QK; ++c) s += Qs[r][c] * kr[c];
                const float p = __expf(s * scale - Ls[r]);
                float dp = 0.f;
#pragma unroll
                for (int c = 0; c < DV; ++c) {
                    dp += Gs[r][c] * vr[c];
                    dvr[c] += p * Gs[r][c];
                }
                const float ds = p * (dp - Ds[r]) * scale;
#pragma unroll
                for (int c = 0; c < QK; ++c) dkr[c] += ds * Qs[r][c];
            }
        }
    }
    if (j < S) {
#pragma unroll
        for (int c = 0; c < QK; ++c) dk[(base + j) * ldq + h * QK + c] = dkr[c];
#pragma unroll
        for (int c = 0; c < DV; ++c) dv[(base + j) * ldv + h * DV + c] = dvr[c];
    }
}

// dQ for one query tile (one query per thread). dq fp32 [B*S][H*QK], scaled by `scale`.
template <int QK, int DV>
__global__ void __launch_bounds__(64) flash_bwd_dq_kernel(
    const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
    const float* __restrict__ dout, const float* __restrict__ lse, const float* __restrict__ D,
    int S, int H, float scale, float* __restrict__ dq) {
    __shared__ float Ks[kAttTile][QK + 1];
    __shared__ float Vs[kAttTile][DV + 1];
    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int i = qt * kAttTile + threadIdx.x;
    const long long base = static_cast<long long>(b) * S;
    const int ldq = H * QK, ldv = H * DV;
    float qr[QK], gr[DV], dqr[QK];
    float li = 0.f, di = 0.f;
    if (i < S) {
        li = lse[(base + i) * H + h];
        di = D[(base + i) * H + h];
    }
#pragma unroll
    for (int c = 0; c < QK; ++c) {
        qr[c] = i < S ? __half2float(q[(base + i) * ldq + h * QK + c]) : 0.f;
        dqr[c] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < DV; ++c) gr[c] = i < S ? dout[(base + i) * ldv + h * DV + c] : 0.f;
    for (int kt = 0; kt <= qt; ++kt) {
        __syncthreads();
        for (int e = threadIdx.x; e < kAttTile * QK; e += blockDim.x) {
            const int r = e / QK, c = e % QK, j = kt * kAttTile + r;
            Ks[r][c] = j < S ? __half2float(k[(base + j) * ldq + h * QK + c]) : 0.f;
        }
        for (int e = threadIdx.x; e < kAttTile * DV; e += blockDim.x) {
            const int r = e / DV, c = e % DV, j = kt * kAttTile + r;
            Vs[r][c] = j < S ? __half2float(v[(base + j) * ldv + h * DV + c]) : 0.f;
        }
        __syncthreads();
        if (i < S) {
            const int jmax = min(kAttTile, i - kt * kAttTile + 1);
            for (int r = 0; r < jmax; ++r) {
                float s = 0.f, dp = 0.f;
#pragma unroll
                for (int c = 0; c < QK; ++c) s += qr[c] * Ks[r][c];
#pragma unroll
                for (int c = 0; c < DV; ++c) dp += gr[c] * Vs[r][c];
                const float p = __expf(s * scale - li);
                const float ds = p * (dp - di) * scale;
#pragma unroll
                for (int c = 0; c < QK; ++c) dqr[c] += ds * Ks[r][c];
            }
        }
    }
    if (i < S) {
#pragma unroll
        for (int c = 0; c < QK; ++c) dq[(base + i) * ldq + h * QK + c] = dqr[c];
    }
}

// Absorbed latent decode attention for one new token per sequence.
// qf fp32 [B][H][KV + R]: per head the absorbed query (W_uk folded in) then the rotated
// rope query. Cache: fp16 [B][max_seq][KV + R] for this layer. Positions 0..pos[b]
// (inclusive) are attended. ctx out fp16 [B][H*KV]. grid B, block 32*H.
template <int KV, int R>
__global__ void decode_attention_kernel(const float* __restrict__ qf, const __half* __restrict__ cache,
                                        long long cache_seq_stride, const int* __restrict__ pos,
                                        int H, float scale, __half* __restrict__ ctx) {
    constexpr int W = KV + R;
    constexpr int TILE = 32;
    __shared__ float Cs[TILE][W + 1];
    extern __shared__ float qsm[];  // [H][W]
    const int b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = pos[b] + 1;
    for (int e = threadIdx.x; e < H * W; e += blockDim.x) qsm[e] = qf[static_cast<long long>(b) * H * W + e] * scale;
    const __half* cb = cache + static_cast<long long>(b) * cache_seq_stride;
    constexpr int PER = (KV + 31) / 32;
    float acc[PER];
#pragma unroll
    for (int u = 0; u < PER; ++u) acc[u] = 0.f;
    float m = -INFINITY, l = 0.f;
    for (int t0 = 0; t0 < n; t0 += TILE) {
        __syncthreads();
        for (int e = threadIdx.x; e < TILE * W; e += blockDim.x) {
            const int r = e / W, c = e % W;
            Cs[r][c] = t0 + r < n ? __half2float(cb[static_cast<long long>(t0 + r) * W + c]) : 0.f;
        }
        __syncthreads();
        if (warp < H) {
            const float* qh = qsm + warp * W;
            // lane r scores position t0 + r
            float s = -INFINITY;
            if (t0 + lane < n) {
                float a = 0.f;
#pragma unroll 8
                for (int c = 0; c < W; ++c) a += qh[c] * Cs[lane][c];
                s = a;
            }
            const float tmax = warp_max(s);
            const float mnew = fmaxf(m, tmax);
            const float corr = __expf(m - mnew);
            const float p = t0 + lane < n ? __expf(s - mnew) : 0.f;
            l = l * corr + warp_sum(p);
#pragma unroll
            for (int u = 0; u < PER; ++u) acc[u] *= corr;
            m = mnew;
            const int cnt = min(TILE, n - t0);
            for (int r = 0; r < cnt; ++r) {
                const float pr = __shfl_sync(0xffffffffu, p, r);
#pragma unroll
                for (int u = 0; u < PER; ++u) {
                    const int c = lane + 32 * u;
                    if (c < KV) acc[u] += pr * Cs[r][c];
                }
            }
        }
    }
    if (warp < H) {
        const float inv = 1.0f / l;
#pragma unroll
        for (int u = 0; u < PER; ++u) {
            const int c = lane + 32 * u;
            if (c < KV) ctx[static_cast<long long>(b) * H * KV + warp * KV + c] = __float2half_rn(acc[u] * inv);
        }
    }
}

} // namespace mm
