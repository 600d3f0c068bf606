// Vocabulary head, GRPO objective and sampling kernels.
//
//   logsoftmax_rows_kernel  weighted_nll's normaliser (ops.cpp:183-201): per row max,
//                           z = sum exp(l - max) accumulated in double, lp = l_t - max - log z.
//   vocab_grad_kernel       weighted_nll's gradient (ops.cpp:202-207), pre-scaled by the
//                           chunk's power-of-two gradient scale, fp16 for the GEMMs.
//   grpo_coef_kernel        grpo_objective + coefficient assembly (trainer.cpp:351-370,
//                           827-846) for every supervised token, in double.
//   advantages_kernel       group_advantages (trainer.cpp:371-385), one thread per group.
//   sample_kernel           sample_token at top_p = 1, no penalties (inference.cpp:345-426).
#pragma once
#include "common.cuh"

namespace mm {

// One block per row. logits fp32 [T][ld]; writes lp[t] (float) and lse[t] = max + log z.
__global__ void logsoftmax_rows_kernel(const float* __restrict__ logits, long long ld, int V,
                                       const uint16_t* __restrict__ target, int T,
                                       float* __restrict__ lp, float* __restrict__ lse, int* err) {
    MM_PDL_ENTRY();
    __shared__ float red_f[32];
    __shared__ double red_d[32];
    const int t = blockIdx.x;
    if (t >= T) return;
    const float* row = logits + t * ld;
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < V; j += blockDim.x) mx = fmaxf(mx, row[j]);
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) red_f[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red_f[threadIdx.x] : -INFINITY;
        v = warp_max(v);
        if (threadIdx.x == 0) red_f[0] = v;
    }
    __syncthreads();
    mx = red_f[0];
    double z = 0.0;
    for (int j = threadIdx.x; j < V; j += blockDim.x) z += static_cast<double>(__expf(row[j] - mx));
    z = warp_sum(z);
    if ((threadIdx.x & 31) == 0) red_d[threadIdx.x >> 5] = z;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) s += red_d[w];
        const int tg = target ? target[t] : 0;
        if (tg >= V) raise_error(err, kErrBadIndex);
        const double l = log(s) + static_cast<double>(mx);
        if (lse) lse[t] = static_cast<float>(l);
        if (lp) {
            const double v = static_cast<double>(row[min(tg, V - 1)]) - l;
            if (!isfinite(v)) raise_error(err, kErrNonfinite);
            lp[t] = static_cast<float>(v);
        }
    }
}

// Combines the per-tile (max, sum exp) partials of the vocabulary GEMM's log-sum-exp
// epilogue, part[j * T + t] for j < ntiles: lse[t] = M + log(sum_j s_j exp(m_j - M)) with the
// sum in double, lp[t] = target logit - lse[t]. One thread per row.
__global__ void lse_combine_kernel(const float2* __restrict__ part, int ntiles, int T,
                                   const float* __restrict__ tgt_logit, float* __restrict__ lp,
                                   float* __restrict__ lse, int* err) {
    MM_PDL_ENTRY();
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T) return;
    float mx = -INFINITY;
    for (int j = 0; j < ntiles; ++j) mx = fmaxf(mx, part[static_cast<long long>(j) * T + t].x);
    double z = 0.0;
    for (int j = 0; j < ntiles; ++j) {
        const float2 p = part[static_cast<long long>(j) * T + t];
        z += static_cast<double>(p.y) * static_cast<double>(__expf(p.x - mx));
    }
    const double l = log(z) + static_cast<double>(mx);
    if (lse) lse[t] = static_cast<float>(l);
    if (lp) {
        const double v = static_cast<double>(tgt_logit[t]) - l;
        if (!isfinite(v)) raise_error(err, kErrNonfinite);
        lp[t] = static_cast<float>(v);
    }
}

// g[t, j] = scale * coef[t] * (exp(l - lse) - [j == target]) in fp16, [T][ldg].
__global__ void vocab_grad_kernel(const float* __restrict__ logits, long long ld, int V,
                                  const uint16_t* __restrict__ target, const float* __restrict__ lse,
                                  const float* __restrict__ coef, const float* __restrict__ scale,
                                  int T, __half* __restrict__ g, long long ldg) {
    MM_PDL_ENTRY();
    const int t = blockIdx.x;
    if (t >= T) return;
    const float c = coef[t] * *scale;
    const float L = lse[t];
    const int tg = target[t];
    const float* row = logits + t * ld;
    __half* out = g + t * ldg;
    if (c == 0.f) {
        for (int j = threadIdx.x; j < V; j += blockDim.x) out[j] = __float2half_rn(0.f);
        return;
    }
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
        const float p = __expf(row[j] - L);
        out[j] = __float2half_rn(c * (p - (j == tg ? 1.f : 0.f)));
    }
}

struct GrpoSums {
    double loss, kl;
    unsigned int max_coef_bits;  // max |coef| of the current chunk, as float bits
    int rejected;
};

// Per token t of a chunk (rows t in [0, T), sequence = t / S): when mask[t] != 0,
// coef[t] = nll_coefficient / (n_total * supervised[seq]) in float, and loss/kl sums
// (objective/denominator) accumulate in double. Masked tokens get coef 0.
__global__ void grpo_coef_kernel(const float* __restrict__ lp, const float* __restrict__ old_lp,
                                 const float* __restrict__ ref_lp, const float* __restrict__ mask,
                                 const float* __restrict__ adv, const int* __restrict__ supervised,
                                 int T, int S, double n_total, float clip, float klc,
                                 float* __restrict__ coef, GrpoSums* __restrict__ sums) {
    MM_PDL_ENTRY();
    __shared__ double sl[32], sk[32];
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    double lo = 0.0, kl = 0.0;
    float cf = 0.f;
    if (t < T) {
        if (mask[t] != 0.f) {
            const float a = lp[t], o = old_lp[t], r = ref_lp[t], A = adv[t / S];
            if (!isfinite(a) || !isfinite(o) || !isfinite(r) || !isfinite(A) ||
                fabsf(a - o) > 80.f || fabsf(r - a) > 80.f) {
                atomicAdd(&sums->rejected, 1);
            } else {
                const double ratio = exp(static_cast<double>(a) - static_cast<double>(o));
                const double clipped = fmin(fmax(ratio, 1.0 - static_cast<double>(clip)), 1.0 + static_cast<double>(clip));
                const double delta = static_cast<double>(r) - static_cast<double>(a);
                const double ed = exp(delta);
                const double k3 = ed - delta - 1.0;
                const double obj = -fmin(ratio * A, clipped * A) + static_cast<double>(klc) * k3;
                // 1 + clip is float arithmetic in the reference (trainer.cpp:363).
                const bool active = A >= 0.f ? ratio <= static_cast<double>(1.f + clip)
                                             : ratio >= static_cast<double>(1.f - clip);
                const double c = (active ? ratio * A : 0.0) + static_cast<double>(klc) * (ed - 1.0);
                const double den = n_total * static_cast<double>(supervised[t / S]);
                lo = obj / den;
                kl = k3 / den;
                cf = static_cast<float>(c / den);
                if (!isfinite(obj) || !isfinite(c)) atomicAdd(&sums->rejected, 1);
            }
        }
        coef[t] = cf;
    }
    lo = warp_sum(lo);
    kl = warp_sum(kl);
    float am = fabsf(cf);
    am = warp_max(am);
    if ((threadIdx.x & 31) == 0) {
        sl[threadIdx.x >> 5] = lo;
        sk[threadIdx.x >> 5] = kl;
        if (am > 0.f) atomicMax(&sums->max_coef_bits, __float_as_uint(am));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double a = 0.0, b = 0.0;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
            a += sl[w];
            b += sk[w];
        }
        atomicAdd(&sums->loss, a);
        atomicAdd(&sums->kl, b);
    }
}

// scale = 2^-floor(log2(max|coef|)) so that the largest scaled coefficient lies in [1, 2);
// inv = 1 / scale. Exact powers of two: the backward pass is linear in the coefficients.
__global__ void grad_scale_kernel(const GrpoSums* __restrict__ sums, float* __restrict__ scale_inv) {
    MM_PDL_ENTRY();
    const float m = __uint_as_float(sums->max_coef_bits);
    float s = 1.f;
    if (m > 0.f && isfinite(m)) s = exp2f(-floorf(log2f(m)));
    scale_inv[0] = s;
    scale_inv[1] = 1.f / s;
}

// group_advantages for groups of G consecutive rewards.
__global__ void advantages_kernel(const float* __restrict__ rewards, int n_groups, int G, float eps,
                                  float* __restrict__ adv, int* __restrict__ any_nonzero) {
    MM_PDL_ENTRY();
    const int g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n_groups) return;
    const float* r = rewards + g * G;
    double mean = 0.0;
    for (int i = 0; i < G; ++i) mean += r[i];
    mean /= static_cast<double>(G);
    double sq = 0.0;
    for (int i = 0; i < G; ++i) sq += (r[i] - mean) * (r[i] - mean);
    const double scale = sqrt(sq / static_cast<double>(G)) + static_cast<double>(eps);
    for (int i = 0; i < G; ++i) {
        const float a = static_cast<float>((r[i] - mean) / scale);
        adv[g * G + i] = a;
        if (a != 0.f) atomicOr(any_nonzero, 1);
    }
}

// ------------------------------------------------------------------ sampling
__device__ __forceinline__ uint64_t splitmix_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
// Draw k (0-based) of Rng(seed).uniform() (rng.hpp:10-18): splitmix64 is a counter
// generator, state after k+1 calls is seed + (k+1) * golden gamma.
__device__ __forceinline__ float rng_uniform_at(uint64_t seed, uint32_t k) {
    const uint64_t x = splitmix_mix(seed + static_cast<uint64_t>(k + 1) * 0x9e3779b97f4a7c15ull);
    return (static_cast<float>(x >> 40) + 0.5f) / 16777216.0f;
}
// Order-preserving map of a float to uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kSampleThreads = 512;
constexpr int kSampleBuckets = 2048;
constexpr int kSampleCap = 1024;
constexpr int kSampleCache = 32;  // scores per thread held in registers (rows up to 16384)

// Block-wide inclusive prefix sum of one u64 per thread (blockDim.x = kSampleThreads).
__device__ __forceinline__ unsigned long long block_scan_incl(unsigned long long v, unsigned long long* warp_tot) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    if (lane == 31) warp_tot[warp] = v;
    __syncthreads();
    if (warp == 0) {
        unsigned long long t = lane < (kSampleThreads >> 5) ? warp_tot[lane] : 0ull;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long n = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += n;
        }
        if (lane < (kSampleThreads >> 5)) warp_tot[lane] = t;
    }
    __syncthreads();
    const unsigned long long before = warp > 0 ? warp_tot[warp - 1] : 0ull;
    __syncthreads();  // warp_tot is reused by the next scan
    return v + before;
}

// Sampling weight in 2^-48 fixed point: w = exp(double(s - s0) / T) <= 1 (s0 is the row
// maximum; the float difference and the double division are those of sample_token,
// inference.cpp:410-411), so a row of at most 65535 weights sums below 2^64 and every
// partial sum is exact and independent of the order of addition.
__device__ __forceinline__ unsigned long long sample_weight_q(float s, float s0, double T) {
    const double d = static_cast<double>(__fsub_rn(s, s0));
    return __double2ull_rn(exp(T == 1.0 ? d : d / T) * 281474976710656.0);  // d / 1 == d exactly
}

// The draw u * total in the same fixed point, with the reference's 24-bit uniform
// u = (x + 1/2) / 2^24 of draw k (rng.hpp:10-18): ((2x + 1) * total) >> 25, exact in 128 bits.
__device__ __forceinline__ unsigned long long sample_draw(uint64_t seed, int k, unsigned long long total) {
    const uint64_t x = splitmix_mix(seed + static_cast<uint64_t>(k + 1) * 0x9e3779b97f4a7c15ull) >> 40;
    const unsigned long long f = 2ull * x + 1ull;
    const unsigned long long lo = f * total, hi = __umul64hi(f, total);
    return (hi << 39) | (lo >> 25);
}

// Adds q to hist[bucket] and 1 to hcount[bucket], one atomic per distinct bucket of the
// warp (scores crowd into few key buckets, so per-lane atomics would serialise).
__device__ __forceinline__ void warp_bucket_add(unsigned long long* hist, int* hcount, int bucket,
                                                unsigned long long q, bool valid) {
    const unsigned active = __ballot_sync(0xffffffffu, valid);
    if (!valid) return;
    const unsigned peers = __match_any_sync(active, bucket);
    unsigned long long sum = 0;
    for (unsigned m = peers; m; m &= m - 1) sum += __shfl_sync(peers, q, __ffs(m) - 1);
    if ((threadIdx.x & 31) == __ffs(peers) - 1) {
        atomicAdd(&hist[bucket], sum);
        atomicAdd(&hcount[bucket], __popc(peers));
    }
}

struct SampleShared {
    unsigned long long hist[kSampleBuckets];
    int hcount[kSampleBuckets];
    uint32_t cand_key[kSampleCap];
    int cand_id[kSampleCap];
    unsigned long long cand_w[kSampleCap];
    float red_f[32], red_g[32];
    int red_i[32];
    unsigned long long warp_tot[32];
    unsigned long long s_draw;
    uint32_t s_prefix;
    int s_bits, s_ncand, s_chosen, s_last;
};

// Scan of the bucket masses from the highest bucket (highest scores) down. With `first`,
// the draw is derived from the row total. Leaves in S.s_chosen the bucket where the running
// mass first reaches the draw and in S.s_draw the part of the draw left inside it.
__device__ void sample_locate(SampleShared& S, int nb, bool first, uint64_t seed, int k) {
    constexpr int PER = kSampleBuckets / kSampleThreads;  // buckets per thread
    // thread t owns descending positions [t*PER, t*PER + PER); position p <-> bucket nb-1-p
    unsigned long long mine = 0;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        const int bk = nb - 1 - (static_cast<int>(threadIdx.x) * PER + e);
        if (bk >= 0) mine += S.hist[bk];
    }
    const unsigned long long incl = block_scan_incl(mine, S.warp_tot);
    if (first) {
        if (threadIdx.x == kSampleThreads - 1) S.s_draw = sample_draw(seed, k, incl);
        __syncthreads();
    }
    if (threadIdx.x == 0) { S.s_chosen = -1; S.s_last = 0x7fffffff; }
    __syncthreads();
    const unsigned long long draw = S.s_draw;
    unsigned long long run = incl - mine;  // mass of all higher buckets
    int last_here = 0x7fffffff;
    __syncthreads();  // every thread has read the draw before it is rewritten
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        const int bk = nb - 1 - (static_cast<int>(threadIdx.x) * PER + e);
        if (bk < 0 || S.hcount[bk] == 0) continue;
        last_here = bk;
        if (run < draw && run + S.hist[bk] >= draw) {
            S.s_chosen = bk;
            S.s_draw = draw - run;
        }
        run += S.hist[bk];
    }
    if (last_here != 0x7fffffff) atomicMin(&S.s_last, last_here);
    __syncthreads();
    if (threadIdx.x == 0 && S.s_chosen < 0) {
        S.s_chosen = S.s_last;  // only when every weight rounded to zero below the draw
        S.s_draw = ~0ull;
    }
    __syncthreads();
}

// Gathers the scores selected by `in_set` (at most kSampleCap of them), sorts them (score
// descending, id ascending) and returns the id where their running mass reaches S.s_draw
// (the last one when none does; `none` when the set is empty).
// `each(f)` calls f(id, score) for this thread's share of the row.
template <class Each, class Pred>
__device__ int sample_pick(SampleShared& S, Each each, float s0, double T, Pred in_set, int none) {
    if (threadIdx.x == 0) S.s_ncand = 0;
    __syncthreads();
    each([&](int j, float v) {
        if (in_set(v)) {
            const int slot = atomicAdd(&S.s_ncand, 1);
            if (slot < kSampleCap) {
                S.cand_key[slot] = float_key(v);
                S.cand_id[slot] = j;
                S.cand_w[slot] = sample_weight_q(v, s0, T);
            }
        }
    });
    __syncthreads();
    const int n = min(S.s_ncand, kSampleCap);
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    // bitonic sort of the candidates (padded to a power of two): key descending, id ascending
    for (int i = n + threadIdx.x; i < np2; i += blockDim.x) {
        S.cand_key[i] = 0;
        S.cand_id[i] = 0x7fffffff;
        S.cand_w[i] = 0ull;
    }
    __syncthreads();
    for (int size = 2; size <= np2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < np2; i += blockDim.x) {
                const int jx = i ^ stride;
                if (jx > i) {
                    const bool desc = (i & size) == 0;
                    const bool i_before = S.cand_key[i] > S.cand_key[jx] ||
                                          (S.cand_key[i] == S.cand_key[jx] && S.cand_id[i] < S.cand_id[jx]);
                    if (desc != i_before) {
                        const uint32_t tk = S.cand_key[i]; S.cand_key[i] = S.cand_key[jx]; S.cand_key[jx] = tk;
                        const int ti = S.cand_id[i]; S.cand_id[i] = S.cand_id[jx]; S.cand_id[jx] = ti;
                        const unsigned long long tw = S.cand_w[i]; S.cand_w[i] = S.cand_w[jx]; S.cand_w[jx] = tw;
                    }
                }
            }
            __syncthreads();
        }
    }
    // first sorted candidate whose running sum reaches the remaining draw
    const unsigned long long rem = S.s_draw;
    constexpr int CPT = kSampleCap / kSampleThreads;  // candidates per thread
    unsigned long long mine = 0;
#pragma unroll
    for (int e = 0; e < CPT; ++e) {
        const int i = threadIdx.x * CPT + e;
        if (i < n) mine += S.cand_w[i];
    }
    const unsigned long long incl = block_scan_incl(mine, S.warp_tot);
    if (threadIdx.x == 0) S.s_chosen = 0x7fffffff;
    __syncthreads();
    unsigned long long run = incl - mine;
#pragma unroll
    for (int e = 0; e < CPT; ++e) {
        const int i = threadIdx.x * CPT + e;
        if (i < n) {
            run += S.cand_w[i];
            if (run >= rem) { atomicMin(&S.s_chosen, i); break; }
        }
    }
    __syncthreads();
    const int i = S.s_chosen == 0x7fffffff ? n - 1 : S.s_chosen;
    return n > 0 ? S.cand_id[i] : none;
}

// One block per sequence row of logits [B][ld] (vocab V <= 65535). Greedy when
// temperature == 0 (first index of the maximum). Otherwise the inverse CDF of
// sample_token with top_p = 1: scores sorted descending (ties: lower id first), weights
// w = exp(double(s - s0) / T), draw = u * sum(w) with the reference's 24-bit uniform u,
// first position whose running sum reaches the draw. Weights are summed in exact 2^-48
// fixed point (the sampled token equals the reference's except when the draw falls within
// ~1e-10 of a CDF boundary). The sorted order is found without a full sort:
//  1. one pass histograms the weights over 2048 buckets of equal score width between the
//     row minimum and maximum (an order-preserving map: a higher score never lands in a
//     lower bucket, and equal scores share one), so a row of 16384 spreads ~8 per bucket;
//  2. a block scan over the buckets, highest first, locates the bucket holding the crossing;
//  3. that bucket's scores are sorted in shared memory and a block scan finds the crossing.
// When the crossing bucket holds more than kSampleCap scores (a row of near-identical
// scores beside a distant maximum), the buckets are rebuilt from the order-preserving
// integer key of each score instead, 11 bits at a time, until the selected prefix holds at
// most kSampleCap scores (or all 32 bits are fixed).
// Rows with active[b] == 0 are skipped. The draw index of row b is draw_index[b] (or 0) +
// draw_offset + *counter (when given); the token goes to out[b * out_stride + *counter]
// (counter 0 when null), so a replayed graph can advance both through device memory.
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(
    const float* __restrict__ logits, long long ld, int V, float temperature,
    const uint64_t* __restrict__ seeds, const int* __restrict__ draw_index, int draw_offset,
    const int* __restrict__ counter, const int* __restrict__ active, uint16_t* __restrict__ out,
    long long out_stride) {
    MM_PDL_ENTRY();
    __shared__ SampleShared S;
    const int step = counter ? *counter : 0;
    out += step;
    draw_offset += step;
    const int b = blockIdx.x;
    if (active && !active[b]) return;
    const float* row = logits + b * ld;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    // Rows up to kSampleCache * kSampleThreads scores stay in registers across the passes.
    const bool cached = V <= kSampleCache * kSampleThreads;
    float vals[kSampleCache];
    if (cached) {
#pragma unroll
        for (int k = 0; k < kSampleCache; ++k) {
            const int j = threadIdx.x + k * kSampleThreads;
            vals[k] = j < V ? row[j] : 0.f;
        }
    }
    auto each = [&](auto&& f) {
        if (cached) {
#pragma unroll
            for (int k = 0; k < kSampleCache; ++k) {
                const int j = threadIdx.x + k * kSampleThreads;
                if (j < V) f(j, vals[k]);
            }
        } else {
            for (int j = threadIdx.x; j < V; j += kSampleThreads) f(j, row[j]);
        }
    };

    // maximum with its first index, and minimum
    float mx = -INFINITY, mn = INFINITY;
    int mi = 0x7fffffff;
    each([&](int j, float v) {
        if (v > mx) { mx = v; mi = j; }
        mn = fminf(mn, v);
    });
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, mx, o);
        const int oi = __shfl_xor_sync(0xffffffffu, mi, o);
        if (ov > mx || (ov == mx && oi < mi)) { mx = ov; mi = oi; }
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    }
    if (lane == 0) { S.red_f[warp] = mx; S.red_i[warp] = mi; S.red_g[warp] = mn; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float bm = S.red_f[0], bn = S.red_g[0];
        int bi = S.red_i[0];
        for (int w = 1; w < nw; ++w) {
            if (S.red_f[w] > bm || (S.red_f[w] == bm && S.red_i[w] < bi)) { bm = S.red_f[w]; bi = S.red_i[w]; }
            bn = fminf(bn, S.red_g[w]);
        }
        S.red_f[0] = bm;
        S.red_i[0] = bi;
        S.red_g[0] = bn;
    }
    __syncthreads();
    const float s0 = S.red_f[0], smin = S.red_g[0];
    const int best = S.red_i[0];
    if (temperature == 0.f) {
        if (threadIdx.x == 0) out[b * out_stride] = static_cast<uint16_t>(best);
        return;
    }
    const double T = static_cast<double>(temperature);
    const uint64_t seed = seeds[b];
    const int k = (draw_index ? draw_index[b] : 0) + draw_offset;

    // 1-3: buckets of equal score width, bucket kSampleBuckets-1 holding the maximum
    const float range = __fsub_rn(s0, smin);
    float scale = range > 0.f ? __fdiv_rn(static_cast<float>(kSampleBuckets), range) : 0.f;
    if (!(scale <= 3.0e38f)) scale = 0.f;
    if (scale > 0.f) {
        auto bucket_of = [&](float v) {
            const float p = fminf(__fmul_rn(__fsub_rn(s0, v), scale), static_cast<float>(kSampleBuckets - 1));
            return kSampleBuckets - 1 - static_cast<int>(p);
        };
        for (int i = threadIdx.x; i < kSampleBuckets; i += blockDim.x) { S.hist[i] = 0ull; S.hcount[i] = 0; }
        __syncthreads();
        each([&](int, float v) {
            const int bk = bucket_of(v);
            atomicAdd(&S.hist[bk], sample_weight_q(v, s0, T));
            atomicAdd(&S.hcount[bk], 1);
        });
        __syncthreads();
        sample_locate(S, kSampleBuckets, true, seed, k);
        const int chosen = S.s_chosen;
        if (S.hcount[chosen] <= kSampleCap) {
            const int tok = sample_pick(S, each, s0, T, [&](float v) { return bucket_of(v) == chosen; }, best);
            if (threadIdx.x == 0) out[b * out_stride] = static_cast<uint16_t>(tok);
            return;
        }
        __syncthreads();
    }

    // fallback: buckets of the order-preserving key, refined 11 bits at a time
    if (threadIdx.x == 0) { S.s_prefix = 0; S.s_bits = 0; }
    __syncthreads();
    bool first = true;
    while (true) {
        const int bits = S.s_bits;
        const uint32_t prefix = S.s_prefix;
        const int width = min(11, 32 - bits);
        const int nb = 1 << width;
        for (int i = threadIdx.x; i < kSampleBuckets; i += blockDim.x) { S.hist[i] = 0ull; S.hcount[i] = 0; }
        __syncthreads();
        for (int j0 = 0; j0 < V; j0 += blockDim.x) {
            const int j = j0 + threadIdx.x;
            bool valid = j < V;
            const float v = valid ? row[j] : 0.f;
            const uint32_t key = float_key(v);
            if (bits > 0) valid = valid && (key >> (32 - bits)) == prefix;
            const int bk = static_cast<int>((key >> (32 - bits - width)) & (nb - 1));
            const unsigned long long q = valid ? sample_weight_q(v, s0, T) : 0ull;
            warp_bucket_add(S.hist, S.hcount, bk, q, valid);
        }
        __syncthreads();
        sample_locate(S, nb, first, seed, k);
        first = false;
        if (threadIdx.x == 0) {
            const int chosen = S.s_chosen;
            S.s_prefix = (prefix << width) | static_cast<uint32_t>(chosen);
            S.s_bits = bits + width;
            S.s_ncand = S.hcount[chosen];
        }
        __syncthreads();
        if (S.s_ncand <= kSampleCap || S.s_bits >= 32) break;
    }
    const int bits = S.s_bits;
    const uint32_t prefix = S.s_prefix;
    const int ncand = S.s_ncand;
    __syncthreads();
    if (ncand > kSampleCap) {
        // More than kSampleCap scores share one exact value (every key bit fixed): equal
        // weights w, ordered by id, so the crossing is position m = ceil(rem / w) - 1 among
        // them, found by an id-ordered block scan over the row.
        const uint32_t u = (prefix & 0x80000000u) ? (prefix & 0x7fffffffu) : ~prefix;
        const unsigned long long w = sample_weight_q(__uint_as_float(u), s0, T);
        const unsigned long long rem = S.s_draw;
        long long m = ncand - 1;
        if (w > 0 && rem <= static_cast<unsigned long long>(ncand) * w) m = static_cast<long long>((rem + w - 1) / w) - 1;
        m = max(0LL, min(m, static_cast<long long>(ncand - 1)));
        long long seen = 0;
        for (int j0 = 0; j0 < V; j0 += blockDim.x) {
            const int j = j0 + threadIdx.x;
            const int hit = (j < V && float_key(row[j]) == prefix) ? 1 : 0;
            const unsigned long long incl = block_scan_incl(static_cast<unsigned long long>(hit), S.warp_tot);
            const long long before = seen + static_cast<long long>(incl) - hit;
            if (hit && before == m) out[b * out_stride] = static_cast<uint16_t>(j);
            // the block's count for this chunk is the last thread's inclusive sum
            if (threadIdx.x == kSampleThreads - 1) S.s_last = static_cast<int>(incl);
            __syncthreads();
            seen += S.s_last;
            __syncthreads();
            if (seen > m) break;
        }
        return;
    }
    const int tok = sample_pick(S, each, s0, T, [&](float v) {
        const uint32_t key = float_key(v);
        return (bits >= 32 ? key : (key >> (32 - bits))) == prefix;
    }, best);
    if (threadIdx.x == 0) out[b * out_stride] = static_cast<uint16_t>(tok);
}

} // namespace mm

namespace mm {
// max |x| over n floats, as float bits into *out (atomicMax on non-negative floats).
__global__ void absmax_kernel(const float* __restrict__ x, int n, unsigned int* __restrict__ out) {
    MM_PDL_ENTRY();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    float v = i < n ? fabsf(x[i]) : 0.f;
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0 && v > 0.f) atomicMax(out, __float_as_uint(v));
}
} // namespace mm
