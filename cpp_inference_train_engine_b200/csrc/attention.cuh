// Decode attention.
//
// Decode (CpuDecoder::decode, inference.cpp:116-153, absorbed form): every head of a
// sequence attends over the same compressed cache row [latent kv_rank | rope], so one CTA
// per sequence stages cache tiles once and its warps (one per head) all read them.
#pragma once
#include "common.cuh"
#include "flash_mma.cuh"

namespace mm {

// Absorbed latent decode attention for one new token per sequence.
// qf fp32 [B][H][KV + R]: per head the absorbed query (W_uk folded in) then the rotated
// rope query. Cache: fp16 [B][max_seq][KV + R] for this layer. Positions 0..pos[b]
// (inclusive) are attended. ctx out fp16 [B][H*KV]. grid B, block 32*H, dynamic shared
// memory decode_attention_smem<KV, R>(H) bytes.
template <int KV, int R>
constexpr size_t decode_attention_smem(int H) {
    return sizeof(float) * (static_cast<size_t>(H) * (KV + R) + 32 * (KV + R + 1));
}
template <int KV, int R>
__global__ void decode_attention_kernel(const float* __restrict__ qf, const __half* __restrict__ cache,
                                        long long cache_seq_stride, const int* __restrict__ pos,
                                        int H, float scale, __half* __restrict__ ctx) {
    MM_PDL_ENTRY();
    constexpr int W = KV + R;
    constexpr int TILE = 32;
    extern __shared__ float qsm[];  // [H][W], then the cache tile [TILE][W + 1]
    float (*Cs)[W + 1] = reinterpret_cast<float (*)[W + 1]>(qsm + H * W);
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

// Tensor-core form for 8 heads over a [128 latent | 16 rope] cache row (the 35.8M model).
// The 8 heads are exactly the N = 8 of mma.sync m16n8k16, so per 16 cached positions a warp
// computes S^T = C[16 x 144] * Q^T (9 MMAs) and O^T += C^T[128 x 16] * P^T (8 MMAs, C^T via
// transposed ldmatrix). For few sequences the context is also split over several warps
// (flash-decoding): each writes a partial (max, sum, O) to `part` and
// decode_attention_combine_kernel merges them.
namespace dec {
constexpr int H = 8, KV = 128, R = 16, W = KV + R;
constexpr int LDQ = W + 8;    // padded rows: 16-byte aligned, conflict-free ldmatrix
constexpr int LDP = 16 + 8;
constexpr int kWarps = 4;
constexpr int kStages = 2;  // cache tiles per warp ring: one computing, one landing
// per warp: a tile ring, its row's query (fp16) and P
constexpr int kRingBytes = kStages * 16 * LDQ * 2;
constexpr int kWarpSmem = kRingBytes + H * LDQ * 2 + H * LDP * 2;
// the same with a STAGES-deep ring (the fused decode step gives its warps a deeper one)
template <int STAGES> constexpr int warp_smem() { return STAGES * 16 * LDQ * 2 + H * LDQ * 2 + H * LDP * 2; }
constexpr int kRowSmem = kWarps * kWarpSmem;
// warps wanted in flight for the whole batch (8 per SM) when choosing context splits
constexpr int kTargetWarps = 148 * 8;
}  // namespace dec

// Latent decode attention with one warp per (sequence row, context split): the warp
// streams its row's cache tiles through its own cp.async ring (kStages deep) and keeps
// one online-softmax state, so no cross-warp merge is needed. Work item
// blockIdx.x * kWarps + warp = b * nsplit + split covers tiles [split * per, ...) of row b.
// With nsplit == 1 the normalised context goes to ctx (fp16 [B][H * KV]); otherwise the
// partial (max, sum, O) of each split goes to part for decode_attention_combine_kernel.
// With cos_t/sin_t, the rope part of each head's query is rotated to position pos[b] as
// it is loaded (the step's query comes straight from the W_uq product).
// Launch: ceil(B * nsplit / kWarps) blocks of 128 threads, dec::kRowSmem dynamic smem.
// One work item of the split latent decode attention for one warp: row b, context split sp
// of nsplit. `mine` is the warp's kWarpSmem bytes of shared memory. With nsplit == 1 the
// normalised context goes to ctx; otherwise the split's partial (max, sum, O) goes to
// part[(b * nsplit + sp) * H * (KV + 2)]. STAGES cache tiles in the warp's ring (the
// standalone kernel: dec::kStages; `mine` holds dec::warp_smem<STAGES>() bytes). qrow
// (optional): a per-row factor of the queries (the fused step's q-latent RMSNorm scale).
template <int STAGES = dec::kStages>
__device__ __forceinline__ void decode_attention_item(const float* __restrict__ qf, const __half* __restrict__ cache,
                                                      long long cache_seq_stride, const int* __restrict__ pos, int b,
                                                      int sp, int nsplit, float scale, __half* __restrict__ ctx,
                                                      float* __restrict__ part, const float* __restrict__ cos_t,
                                                      const float* __restrict__ sin_t, unsigned char* mine,
                                                      const float* __restrict__ qrow = nullptr,
                                                      unsigned long long* stamps = nullptr) {
    using namespace dec;
    using fa::ldsm_x4;
    using fa::ldsm_x4_t;
    using fa::mma16816;
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const long long item = static_cast<long long>(b) * nsplit + sp;
    constexpr int kRing = STAGES * 16 * LDQ * 2;
    auto ring = reinterpret_cast<__half (*)[16][LDQ]>(mine);
    auto Qs = reinterpret_cast<__half (*)[LDQ]>(mine + kRing);
    auto Pw = reinterpret_cast<__half (*)[LDP]>(mine + kRing + H * LDQ * 2);
    const int n = __ldcg(pos + b) + 1;
    const int tiles = (n + 15) / 16;
    const int per = (tiles + nsplit - 1) / nsplit;
    const int t_begin = sp * per, t_end = min(tiles, t_begin + per);
    const __half* cb = cache + static_cast<long long>(b) * cache_seq_stride;
    auto issue = [&](int j) {
        const int tile = t_begin + j;
        if (tile < t_end) {
            const int p0 = tile * 16;
            for (int e = lane; e < 16 * (W / 8); e += 32) {
                const int r = e / (W / 8), cc = (e % (W / 8)) * 8;
                const bool ok = p0 + r < n;
                cp_async16(&ring[j % STAGES][r][cc], cb + static_cast<long long>(ok ? p0 + r : 0) * W + cc, ok);
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int j = 0; j < STAGES - 1; ++j) issue(j);
    // the row's absorbed queries, pre-scaled into the base-2 domain (and by the row factor
    // qrow[b] when the queries come unnormalised), as fp16
    const float4* q4 = reinterpret_cast<const float4*>(qf + static_cast<long long>(b) * H * W);
    const int p = n - 1;  // position of this step's token
    // every load first (the lane's 9 query float4s, the row factor and the rope tables its rope
    // float4 needs), so they are in flight together, then the rotation and the fp16 stores
    constexpr int NQ = H * W / 4 / 32;
    static_assert(H * W / 4 == NQ * 32, "whole float4s per lane");
    float4 v[NQ];
    float cs[NQ][2], sn[NQ][2];
#pragma unroll
    for (int i = 0; i < NQ; ++i) v[i] = __ldcg(q4 + lane + 32 * i);
    const float qscale = scale * fa::kLog2e * (qrow ? __ldcg(qrow + b) : 1.f);
#pragma unroll
    for (int i = 0; i < NQ; ++i) {
        const int c = (4 * (lane + 32 * i)) % W;
        const bool rope = cos_t && c >= KV;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int pair = rope ? (c - KV) / 2 + k : 0;
            cs[i][k] = rope ? cos_t[p * (R / 2) + pair] : 1.f;
            sn[i][k] = rope ? sin_t[p * (R / 2) + pair] : 0.f;
        }
    }
#pragma unroll
    for (int i = 0; i < NQ; ++i) {
        const int e = lane + 32 * i;
        const int hh = (4 * e) / W, c = (4 * e) % W;
        float* f = reinterpret_cast<float*>(&v[i]);
        if (cos_t && c >= KV) {  // adjacent-pair RoPE of the rope query (rope_rows_kernel's arithmetic)
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const float a = f[2 * k], bb = f[2 * k + 1];
                f[2 * k] = a * cs[i][k] - bb * sn[i][k];
                f[2 * k + 1] = a * sn[i][k] + bb * cs[i][k];
            }
        }
        *reinterpret_cast<__half2*>(&Qs[hh][c]) = __floats2half2_rn(f[0] * qscale, f[1] * qscale);
        *reinterpret_cast<__half2*>(&Qs[hh][c + 2]) = __floats2half2_rn(f[2] * qscale, f[3] * qscale);
    }
    __syncwarp();
    if (stamps && lane == 0) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(stamps[0]));
    uint32_t qb[W / 16][2];
#pragma unroll
    for (int kk = 0; kk < W / 16; ++kk) {
        uint32_t r[4];
        ldsm_x4(r, &Qs[lane & 7][kk * 16 + ((lane >> 3) & 1) * 8]);
        qb[kk][0] = r[0];
        qb[kk][1] = r[1];
    }
    float acc[KV / 16][4];
#pragma unroll
    for (int i = 0; i < KV / 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // heads 2t, 2t+1
    for (int j = 0;; ++j) {
        const int tile = t_begin + j;
        if (tile >= t_end) break;
        const int p0 = tile * 16;
        issue(j + STAGES - 1);
        cp_async_wait<STAGES - 1>();
        __syncwarp();
        __half (*Ct)[LDQ] = ring[j % STAGES];
        float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < W / 16; ++kk) {
            uint32_t a[4];
            ldsm_x4(a, &Ct[lane & 15][kk * 16 + (lane >> 4) * 8]);
            mma16816(s, a, qb[kk][0], qb[kk][1]);
        }
        if (p0 + g >= n) { s[0] = -INFINITY; s[1] = -INFINITY; }
        if (p0 + g + 8 >= n) { s[2] = -INFINITY; s[3] = -INFINITY; }
        float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
        }
        const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);  // finite: position p0 is valid
        const float c0 = exp2f(m0 - n0), c1 = exp2f(m1 - n1);
        m0 = n0;
        m1 = n1;
        l0 *= c0;
        l1 *= c1;
#pragma unroll
        for (int i = 0; i < KV / 16; ++i) {
            acc[i][0] *= c0; acc[i][2] *= c0;
            acc[i][1] *= c1; acc[i][3] *= c1;
        }
        const float p00 = exp2f(s[0] - n0), p01 = exp2f(s[1] - n1), p10 = exp2f(s[2] - n0), p11 = exp2f(s[3] - n1);
        l0 += p00 + p10;
        l1 += p01 + p11;
        Pw[2 * t][g] = __float2half_rn(p00);
        Pw[2 * t + 1][g] = __float2half_rn(p01);
        Pw[2 * t][g + 8] = __float2half_rn(p10);
        Pw[2 * t + 1][g + 8] = __float2half_rn(p11);
        __syncwarp();
        uint32_t bp[4];
        ldsm_x4(bp, &Pw[lane & 7][((lane >> 3) & 1) * 8]);
#pragma unroll
        for (int mt = 0; mt < KV / 16; ++mt) {
            uint32_t a[4];
            ldsm_x4_t(a, &Ct[(lane & 7) + ((lane >> 4) << 3)][mt * 16 + ((lane >> 3) & 1) * 8]);
            mma16816(acc[mt], a, bp[0], bp[1]);
        }
        __syncwarp();
    }
    cp_async_wait<0>();
    if (stamps && lane == 0) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(stamps[1]));
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    if (nsplit == 1) {
        const float i0 = 1.f / l0, i1 = 1.f / l1;
        __half* o0 = ctx + static_cast<long long>(b) * H * KV + (2 * t) * KV;
        __half* o1 = o0 + KV;
#pragma unroll
        for (int mt = 0; mt < KV / 16; ++mt) {
            o0[mt * 16 + g] = __float2half_rn(acc[mt][0] * i0);
            o1[mt * 16 + g] = __float2half_rn(acc[mt][1] * i1);
            o0[mt * 16 + g + 8] = __float2half_rn(acc[mt][2] * i0);
            o1[mt * 16 + g + 8] = __float2half_rn(acc[mt][3] * i1);
        }
    } else {
        float* pp = part + static_cast<long long>(item) * H * (KV + 2);
        float* q0 = pp + (2 * t) * (KV + 2);
        float* q1 = q0 + (KV + 2);
        if (g == 0) {
            q0[0] = m0; q0[1] = l0;
            q1[0] = m1; q1[1] = l1;
        }
#pragma unroll
        for (int mt = 0; mt < KV / 16; ++mt) {
            q0[2 + mt * 16 + g] = acc[mt][0];
            q1[2 + mt * 16 + g] = acc[mt][1];
            q0[2 + mt * 16 + g + 8] = acc[mt][2];
            q1[2 + mt * 16 + g + 8] = acc[mt][3];
        }
    }
}


__global__ void __launch_bounds__(128) decode_attention_row_kernel(
    const float* __restrict__ qf, const __half* __restrict__ cache, long long cache_seq_stride,
    const int* __restrict__ pos, int B, int nsplit, float scale, __half* __restrict__ ctx, float* __restrict__ part,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t) {
    MM_PDL_ENTRY();
    using namespace dec;
    extern __shared__ __align__(16) unsigned char row_smem[];
    const int warp = threadIdx.x >> 5;
    const int item = blockIdx.x * kWarps + warp;
    if (item >= B * nsplit) return;  // no block-wide barrier follows
    const int b = item / nsplit, sp = item - b * nsplit;
    decode_attention_item(qf, cache, cache_seq_stride, pos, b, sp, nsplit, scale, ctx, part, cos_t, sin_t,
                          row_smem + warp * kWarpSmem);
}

// Merges the nsplit partials of decode_attention_row_kernel: one warp per (row, head),
// 4 context columns per lane; grid ceil(B * H / 4), block 128.
__global__ void decode_attention_combine_kernel(const float* __restrict__ part, int nsplit, int B,
                                                __half* __restrict__ ctx) {
    MM_PDL_ENTRY();
    using namespace dec;
    const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (wid >= B * H) return;
    const int b = wid / H, hh = wid % H;
    const float* pb = part + static_cast<long long>(b) * nsplit * H * (KV + 2) + hh * (KV + 2);
    const long long stride = static_cast<long long>(H) * (KV + 2);
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, pb[s * stride]);
    float L = 0.f, o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
    for (int s = 0; s < nsplit; ++s) {
        const float* ps = pb + s * stride;
        const float m = ps[0];
        if (m == -INFINITY) continue;
        const float f = exp2f(m - M);
        L += f * ps[1];
        const float2 a = *reinterpret_cast<const float2*>(ps + 2 + 4 * lane);
        const float2 c = *reinterpret_cast<const float2*>(ps + 4 + 4 * lane);
        o0 += f * a.x;
        o1 += f * a.y;
        o2 += f * c.x;
        o3 += f * c.y;
    }
    const float inv = 1.f / L;
    __half* out = ctx + static_cast<long long>(b) * H * KV + hh * KV + 4 * lane;
    *reinterpret_cast<__half2*>(out) = __floats2half2_rn(o0 * inv, o1 * inv);
    *reinterpret_cast<__half2*>(out + 2) = __floats2half2_rn(o2 * inv, o3 * inv);
}

// Merges the nsplit partials of row b (all H heads) into ctx with one warp, in one pass over
// the splits with every head's state in registers (lane = 4 context columns of each head):
// the loads of one split, all heads, are independent and in flight together. Running
// maximum per head, sums rescaled when it rises (the same result as the combine kernel's
// two passes up to rounding). The partials were written by other warps (other CTAs), so
// they are read from L2.
__device__ __forceinline__ void decode_attention_merge_row(const float* __restrict__ part, int nsplit, int b,
                                                           __half* __restrict__ ctx) {
    using namespace dec;
    const int lane = threadIdx.x & 31;
    const long long stride = static_cast<long long>(H) * (KV + 2);
    const float* pb = part + static_cast<long long>(b) * nsplit * stride;
    float M[H], L[H], o[H][4];
#pragma unroll
    for (int hh = 0; hh < H; ++hh) {
        M[hh] = -INFINITY;
        L[hh] = 0.f;
        o[hh][0] = o[hh][1] = o[hh][2] = o[hh][3] = 0.f;
    }
    for (int sp = 0; sp < nsplit; ++sp) {
        const float* ps = pb + sp * stride;
        float2 ml[H];
        float4 ov[H];
#pragma unroll
        for (int hh = 0; hh < H; ++hh) {
            ml[hh] = __ldcg(reinterpret_cast<const float2*>(ps + hh * (KV + 2)));
            const float2 a = __ldcg(reinterpret_cast<const float2*>(ps + hh * (KV + 2) + 2 + 4 * lane));
            const float2 c = __ldcg(reinterpret_cast<const float2*>(ps + hh * (KV + 2) + 4 + 4 * lane));
            ov[hh] = make_float4(a.x, a.y, c.x, c.y);
        }
#pragma unroll
        for (int hh = 0; hh < H; ++hh) {
            const float m = ml[hh].x;
            if (m == -INFINITY) continue;
            const float nm = fmaxf(M[hh], m);
            const float fo = exp2f(M[hh] - nm), fn = exp2f(m - nm);  // fo = 0 while empty
            L[hh] = L[hh] * fo + fn * ml[hh].y;
            o[hh][0] = o[hh][0] * fo + fn * ov[hh].x;
            o[hh][1] = o[hh][1] * fo + fn * ov[hh].y;
            o[hh][2] = o[hh][2] * fo + fn * ov[hh].z;
            o[hh][3] = o[hh][3] * fo + fn * ov[hh].w;
            M[hh] = nm;
        }
    }
#pragma unroll
    for (int hh = 0; hh < H; ++hh) {
        const float inv = 1.f / L[hh];
        __half* out = ctx + static_cast<long long>(b) * H * KV + hh * KV + 4 * lane;
        *reinterpret_cast<__half2*>(out) = __floats2half2_rn(o[hh][0] * inv, o[hh][1] * inv);
        *reinterpret_cast<__half2*>(out + 2) = __floats2half2_rn(o[hh][2] * inv, o[hh][3] * inv);
    }
}

// Tensor-core form for 16 heads over a [512 latent | 32 rope] cache row (the 2,048-wide
// model). All heads of a row attend over the same cache rows (multi-query form), so one CTA
// of 4 warps takes a (row, context split) work item and streams 32-position tiles of the
// row's cache through a cp.async ring (zero-filled past the row's length):
//   scores  S[16 heads x 32 positions] = Q[16 x 544] C^T: warp w takes positions 8w..8w+7
//           (A = the row's queries from shared memory, B = the cache tile, 34 k-steps),
//   softmax thread i owns head i / 8 and 4 positions: running max and sum per head in the
//           base-2 domain, P in fp16, the per-head rescale factor shared,
//   output  O^T[512 x 16] += C^T[512 x 32] P^T: warp w accumulates latent columns
//           [128 w, 128 w + 128) for all 16 heads (8 x 2 m16n8 tiles in registers), A = the
//           cache tile through transposed ldmatrix, B = P.
// Arithmetic as the 8-head form: fp16 operands (queries pre-scaled by scale * log2 e),
// fp32 accumulation, fp16 probabilities. With nsplit == 1 the normalised context goes to ctx
// (fp16 [B][16 * 512]); otherwise (max, sum, O[512]) per head goes to part for
// decode_attention_wide_combine_kernel.
namespace decw {
constexpr int H = 16, KV = 512, R = 32, W = KV + R;
constexpr int kTile = 32;               // cached positions per tile
constexpr int LD = W + 8;               // padded rows: conflict-free ldmatrix
constexpr int LDP = kTile + 8;
constexpr int kStages = 2;
constexpr int kThreads = 128;
constexpr int kQBytes = H * LD * 2;
constexpr int kTileBytes = kTile * LD * 2;
constexpr int kSmem = kQBytes + kStages * kTileBytes + H * kTile * 4 + H * LDP * 2 + 3 * H * 4;
// work items (CTAs) wanted in flight for the whole batch when choosing context splits
constexpr int kTargetItems = 148 * 4;
}  // namespace decw

__global__ void __launch_bounds__(decw::kThreads, 2) decode_attention_wide_kernel(
    const float* __restrict__ qf, const __half* __restrict__ cache, long long cache_seq_stride,
    const int* __restrict__ pos, int B, int nsplit, float scale, __half* __restrict__ ctx, float* __restrict__ part) {
    MM_PDL_ENTRY();
    using namespace decw;
    using fa::ldsm_x4;
    using fa::ldsm_x4_t;
    using fa::mma16816;
    extern __shared__ __align__(16) unsigned char wide_smem[];
    auto Qs = reinterpret_cast<__half (*)[LD]>(wide_smem);
    auto ring = reinterpret_cast<__half (*)[kTile][LD]>(wide_smem + kQBytes);
    auto Ss = reinterpret_cast<float (*)[kTile]>(wide_smem + kQBytes + kStages * kTileBytes);
    auto Ps = reinterpret_cast<__half (*)[LDP]>(wide_smem + kQBytes + kStages * kTileBytes + H * kTile * 4);
    float* corr_s = reinterpret_cast<float*>(wide_smem + kQBytes + kStages * kTileBytes + H * kTile * 4 + H * LDP * 2);
    float* m_s = corr_s + H;
    float* l_s = m_s + H;
    const int item = blockIdx.x;
    if (item >= B * nsplit) return;
    const int b = item / nsplit, sp = item - b * nsplit;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int n = __ldcg(pos + b) + 1;
    const int tiles = (n + kTile - 1) / kTile;
    const int per = (tiles + nsplit - 1) / nsplit;
    const int t_begin = sp * per, t_end = min(tiles, t_begin + per);
    const __half* cb = cache + static_cast<long long>(b) * cache_seq_stride;
    auto issue = [&](int j) {
        const int tile = t_begin + j;
        if (tile < t_end) {
            const int p0 = tile * kTile;
            for (int e = tid; e < kTile * (W / 8); e += kThreads) {
                const int r = e / (W / 8), cc = (e % (W / 8)) * 8;
                const bool ok = p0 + r < n;
                cp_async16(&ring[j % kStages][r][cc], cb + static_cast<long long>(ok ? p0 + r : 0) * W + cc, ok);
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int j = 0; j < kStages - 1; ++j) issue(j);
    // the row's queries (rope part already rotated), pre-scaled into the base-2 domain
    const float qscale = scale * fa::kLog2e;
    const float4* q4 = reinterpret_cast<const float4*>(qf + static_cast<long long>(b) * H * W);
    for (int e = tid; e < H * W / 4; e += kThreads) {
        const float4 v = __ldcg(q4 + e);
        const int hh = (4 * e) / W, c = (4 * e) % W;
        *reinterpret_cast<__half2*>(&Qs[hh][c]) = __floats2half2_rn(v.x * qscale, v.y * qscale);
        *reinterpret_cast<__half2*>(&Qs[hh][c + 2]) = __floats2half2_rn(v.z * qscale, v.w * qscale);
    }
    float acc[8][2][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int k = 0; k < 2; ++k) acc[i][k][0] = acc[i][k][1] = acc[i][k][2] = acc[i][k][3] = 0.f;
    // softmax state of head tid / 8 (replicated over its 8 threads)
    const int sh = tid >> 3, sq = (tid & 7) * 4;
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0;; ++j) {
        const int tile = t_begin + j;
        if (tile >= t_end) break;
        const int p0 = tile * kTile;
        cp_async_wait<kStages - 2>();
        __syncthreads();  // tile j (and the queries) visible; every warp is done with tile j - 1
        issue(j + kStages - 1);
        __half (*Ct)[LD] = ring[j % kStages];
        // scores of positions 8 warp .. 8 warp + 7 for all 16 heads
        {
            float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int kk = 0; kk < W / 16; kk += 2) {
                uint32_t cbf[4];  // k-steps kk and kk + 1 of the 8 positions
                ldsm_x4(cbf, &Ct[8 * warp + (lane & 7)][kk * 16 + (lane >> 3) * 8]);
                uint32_t a[4];
                ldsm_x4(a, &Qs[lane & 15][kk * 16 + (lane >> 4) * 8]);
                mma16816(s, a, cbf[0], cbf[1]);
                ldsm_x4(a, &Qs[lane & 15][(kk + 1) * 16 + (lane >> 4) * 8]);
                mma16816(s, a, cbf[2], cbf[3]);
            }
            const int q0 = 8 * warp + 2 * t;
            const bool v0 = p0 + q0 < n, v1 = p0 + q0 + 1 < n;
            Ss[g][q0] = v0 ? s[0] : -INFINITY;
            Ss[g][q0 + 1] = v1 ? s[1] : -INFINITY;
            Ss[g + 8][q0] = v0 ? s[2] : -INFINITY;
            Ss[g + 8][q0 + 1] = v1 ? s[3] : -INFINITY;
        }
        __syncthreads();
        // online softmax: thread tid owns positions sq..sq+3 of head sh
        {
            const float4 sv = *reinterpret_cast<const float4*>(&Ss[sh][sq]);
            float mx = fmaxf(fmaxf(sv.x, sv.y), fmaxf(sv.z, sv.w));
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float mn = fmaxf(m_run, mx);  // finite: position p0 is valid
            const float cf = exp2f(m_run - mn);
            const float e0 = exp2f(sv.x - mn), e1 = exp2f(sv.y - mn), e2 = exp2f(sv.z - mn), e3 = exp2f(sv.w - mn);
            float ps = (e0 + e1) + (e2 + e3);
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            l_run = l_run * cf + ps;
            m_run = mn;
            *reinterpret_cast<__half2*>(&Ps[sh][sq]) = __floats2half2_rn(e0, e1);
            *reinterpret_cast<__half2*>(&Ps[sh][sq + 2]) = __floats2half2_rn(e2, e3);
            if ((tid & 7) == 0) corr_s[sh] = cf;
        }
        __syncthreads();
        // rescale this warp's accumulators, then O^T += C^T P^T over the tile's 32 positions
        {
            const float c00 = corr_s[2 * t], c01 = corr_s[2 * t + 1], c10 = corr_s[8 + 2 * t], c11 = corr_s[9 + 2 * t];
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                acc[mt][0][0] *= c00; acc[mt][0][1] *= c01; acc[mt][0][2] *= c00; acc[mt][0][3] *= c01;
                acc[mt][1][0] *= c10; acc[mt][1][1] *= c11; acc[mt][1][2] *= c10; acc[mt][1][3] *= c11;
            }
#pragma unroll
            for (int ks = 0; ks < kTile / 16; ++ks) {
                uint32_t bp[4];  // heads 0-7 (bp[0], bp[1]) and 8-15 (bp[2], bp[3])
                ldsm_x4(bp, &Ps[(lane & 7) + ((lane >> 4) << 3)][16 * ks + ((lane >> 3) & 1) * 8]);
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    uint32_t a[4];
                    ldsm_x4_t(a, &Ct[16 * ks + (lane & 7) + ((lane >> 4) << 3)][128 * warp + mt * 16 + ((lane >> 3) & 1) * 8]);
                    mma16816(acc[mt][0], a, bp[0], bp[1]);
                    mma16816(acc[mt][1], a, bp[2], bp[3]);
                }
            }
        }
    }
    cp_async_wait<0>();
    if ((tid & 7) == 0) {
        m_s[sh] = m_run;
        l_s[sh] = l_run;
    }
    __syncthreads();
    const int h0 = 2 * t, h1 = 2 * t + 1, h2 = 8 + 2 * t, h3 = 9 + 2 * t;
    if (nsplit == 1) {
        const float i0 = 1.f / l_s[h0], i1 = 1.f / l_s[h1], i2 = 1.f / l_s[h2], i3 = 1.f / l_s[h3];
        __half* o = ctx + static_cast<long long>(b) * H * KV + 128 * warp;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            const int c = mt * 16 + g;
            o[h0 * KV + c] = __float2half_rn(acc[mt][0][0] * i0);
            o[h1 * KV + c] = __float2half_rn(acc[mt][0][1] * i1);
            o[h0 * KV + c + 8] = __float2half_rn(acc[mt][0][2] * i0);
            o[h1 * KV + c + 8] = __float2half_rn(acc[mt][0][3] * i1);
            o[h2 * KV + c] = __float2half_rn(acc[mt][1][0] * i2);
            o[h3 * KV + c] = __float2half_rn(acc[mt][1][1] * i3);
            o[h2 * KV + c + 8] = __float2half_rn(acc[mt][1][2] * i2);
            o[h3 * KV + c + 8] = __float2half_rn(acc[mt][1][3] * i3);
        }
    } else {
        float* pp = part + static_cast<long long>(item) * H * (KV + 2);
        if (tid < H) {
            pp[tid * (KV + 2)] = m_s[tid];
            pp[tid * (KV + 2) + 1] = l_s[tid];
        }
        float* o = pp + 2 + 128 * warp;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            const int c = mt * 16 + g;
            o[h0 * (KV + 2) + c] = acc[mt][0][0];
            o[h1 * (KV + 2) + c] = acc[mt][0][1];
            o[h0 * (KV + 2) + c + 8] = acc[mt][0][2];
            o[h1 * (KV + 2) + c + 8] = acc[mt][0][3];
            o[h2 * (KV + 2) + c] = acc[mt][1][0];
            o[h3 * (KV + 2) + c] = acc[mt][1][1];
            o[h2 * (KV + 2) + c + 8] = acc[mt][1][2];
            o[h3 * (KV + 2) + c + 8] = acc[mt][1][3];
        }
    }
}

// Merges the nsplit partials of decode_attention_wide_kernel: one warp per (row, head),
// 16 context columns per lane; grid ceil(B * 16 / 4), block 128.
__global__ void decode_attention_wide_combine_kernel(const float* __restrict__ part, int nsplit, int B,
                                                     __half* __restrict__ ctx) {
    MM_PDL_ENTRY();
    using namespace decw;
    const int wid = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (wid >= B * H) return;
    const int b = wid / H, hh = wid % H;
    const float* pb = part + static_cast<long long>(b) * nsplit * H * (KV + 2) + hh * (KV + 2);
    const long long stride = static_cast<long long>(H) * (KV + 2);
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, pb[s * stride]);
    float L = 0.f, o[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = 0.f;
    for (int s = 0; s < nsplit; ++s) {
        const float* ps = pb + s * stride;
        const float m = ps[0];
        if (m == -INFINITY) continue;
        const float f = exp2f(m - M);
        L += f * ps[1];
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] += f * ps[2 + 32 * i + lane];
    }
    const float inv = 1.f / L;
    __half* out = ctx + static_cast<long long>(b) * H * KV + hh * KV + lane;
#pragma unroll
    for (int i = 0; i < 16; ++i) out[32 * i] = __float2half_rn(o[i] * inv);
}

} // namespace mm
