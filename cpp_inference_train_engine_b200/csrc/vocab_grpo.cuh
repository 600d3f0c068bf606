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
// epilogue, part[j * T + t] for j < ntiles: lse[t] = M + log(sum_j s_j exp(m_j - M)),
// lp[t] = target logit - lse[t]. A block of 256 threads takes 64 rows; the four 64-thread
// groups each merge a quarter of every row's partials (groups of 8 loaded together with
// streaming loads: the partials are read once, 32 consecutive rows per warp load), with the
// running maximum raised group by group and the sum rescaled, 8 terms added in float and the
// groups in double (the reference sums in double, ops.cpp:195-201); the quarters are then
// merged in shared memory in a fixed order. A partial that drained no column carries
// (-inf, 0) and adds nothing.
constexpr int kLseRows = 64;
__global__ void __launch_bounds__(256) lse_combine_kernel(const float2* __restrict__ part, int ntiles, int T,
                                                          const float* __restrict__ tgt_logit, float* __restrict__ lp,
                                                          float* __restrict__ lse, int* err) {
    MM_PDL_ENTRY();
    __shared__ float sm[4][kLseRows];
    __shared__ double sz[4][kLseRows];
    const int q = threadIdx.x / kLseRows, r = threadIdx.x % kLseRows;
    const int t = blockIdx.x * kLseRows + r;
    const int per = (ntiles + 3) / 4;
    const int j0 = q * per, j1 = min(ntiles, j0 + per);
    float mx = -INFINITY;
    double z = 0.0;
    if (t < T) {
        const float2* p = part + t;
        constexpr int U = 8;
        for (int j = j0; j < j1; j += U) {
            float2 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u)
                v[u] = j + u < j1 ? __ldcs(p + static_cast<long long>(j + u) * T) : make_float2(-INFINITY, 0.f);
            float cm = v[0].x;
#pragma unroll
            for (int u = 1; u < U; ++u) cm = fmaxf(cm, v[u].x);
            if (cm > mx) {
                z *= static_cast<double>(__expf(mx - cm));  // 0 while nothing was added (mx = -inf)
                mx = cm;
            }
            float s = 0.f;
#pragma unroll
            for (int u = 0; u < U; ++u) s += v[u].x == -INFINITY ? 0.f : v[u].y * __expf(v[u].x - mx);
            z += static_cast<double>(s);
        }
    }
    sm[q][r] = mx;
    sz[q][r] = z;
    __syncthreads();
    if (q != 0 || t >= T) return;
    float M = sm[0][r];
    for (int g = 1; g < 4; ++g) M = fmaxf(M, sm[g][r]);
    double Z = 0.0;
    for (int g = 0; g < 4; ++g)
        if (sm[g][r] != -INFINITY) Z += sz[g][r] * static_cast<double>(__expf(sm[g][r] - M));
    const double l = log(Z) + static_cast<double>(M);
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
    double rejected_ranks;       // ranks that rejected a token, summed across ranks
    unsigned int max_coef_bits;  // max |coef| of the current chunk, as float bits
    int rejected;                // tokens this rank rejected
};

// Per token t of a chunk (rows t in [0, T), sequence = t / S): when mask[t] != 0,
// coef[t] = float(float(nll_coefficient) / (n_total * supervised[seq])), and the block's loss/kl
// sums (objective/denominator, in double) go to part[block] for grpo_sums_kernel. Masked
// tokens get coef 0.
__global__ void grpo_coef_kernel(const float* __restrict__ lp, const float* __restrict__ old_lp,
                                 const float* __restrict__ ref_lp, const float* __restrict__ mask,
                                 const float* __restrict__ adv, const int* __restrict__ supervised,
                                 int T, int S, double n_total, float clip, float klc,
                                 float* __restrict__ coef, GrpoSums* __restrict__ sums,
                                 double2* __restrict__ part) {
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
                // grpo_objective hands back the coefficient as a float (trainer.cpp:368-369),
                // which the loop divides by the double denominator and rounds again (:842-843)
                cf = static_cast<float>(static_cast<double>(static_cast<float>(c)) / den);
                if (!isfinite(obj) || !(fabs(c) <= 3.4028234663852886e38)) atomicAdd(&sums->rejected, 1);
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
        part[blockIdx.x] = make_double2(a, b);
    }
}

// DPO on a preference pair (trainer.cpp:107-121, 345-350, 765-783): rows 2p (chosen) and
// 2p + 1 (rejected) of a chunk, S positions each. One block per pair: the masked sums of the
// policy and reference log-probs in double (fixed-order block reduction), then
// dpo_objective -- margin = (chosen - rejected) - (ref_chosen - ref_rejected), z = beta * margin,
// loss = max(-z, 0) + log1p(exp(-|z|)), scale = beta * sigmoid(float(-z)) -- and the per-token
// coefficients mask * (+-scale / pairs) (float, as the reference's coefficient loop).
// part[p] = (loss / pairs, margin) for an ordered sum; the pair's margin also to margins[p].
__global__ void dpo_coef_kernel(const float* __restrict__ lp, const float* __restrict__ ref_lp,
                                const float* __restrict__ mask, int S, float beta, float pairs,
                                double pairs_d, float* __restrict__ coef, double2* __restrict__ part,
                                double* __restrict__ margins) {
    MM_PDL_ENTRY();
    __shared__ double red[4][32];
    const int p = blockIdx.x;
    const long long base = 2LL * p * S;
    double a[4] = {0.0, 0.0, 0.0, 0.0};  // chosen, rejected, ref chosen, ref rejected
    for (int t = threadIdx.x; t < 2 * S; t += blockDim.x) {
        if (mask[base + t] == 0.f) continue;
        const int r = t < S ? 0 : 1;
        a[r] += static_cast<double>(lp[base + t]);
        a[2 + r] += static_cast<double>(ref_lp[base + t]);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        a[i] = warp_sum(a[i]);
        if (lane == 0) red[i][warp] = a[i];
    }
    __syncthreads();
    double sum[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        sum[i] = 0.0;
        for (int w = 0; w < nw; ++w) sum[i] += red[i][w];
    }
    const double margin = (sum[0] - sum[1]) - (sum[2] - sum[3]);
    const double z = static_cast<double>(beta) * margin;
    const double loss = fmax(-z, 0.0) + log1p(exp(-fabs(z)));
    const float scale = beta * sigmoid_ref(static_cast<float>(-z));
    const float cc = scale / pairs, cr = -scale / pairs;
    for (int t = threadIdx.x; t < 2 * S; t += blockDim.x) coef[base + t] = mask[base + t] * (t < S ? cc : cr);
    if (threadIdx.x == 0) {
        part[p] = make_double2(loss / pairs_d, margin);
        if (margins) margins[p] = margin;
    }
}

// Adds grpo_coef_kernel's per-block (loss, kl) partials into the sums in block order, so
// the reported objective does not depend on the order in which blocks finish.
__global__ void grpo_sums_kernel(const double2* __restrict__ part, int nblocks, GrpoSums* __restrict__ sums) {
    MM_PDL_ENTRY();
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    double a = 0.0, b = 0.0;
    for (int i = 0; i < nblocks; ++i) {
        a += part[i].x;
        b += part[i].y;
    }
    sums->loss += a;
    sums->kl += b;
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

// One block of kSampleThreads per row. Shared memory per row: an equal-width bucket
// histogram (later reused for the candidates) and per-bucket exponential bases.
constexpr int kSampleThreads = 256;
constexpr int kSampleBuckets = 512;
constexpr int kSampleRadixBits = 9;  // key bits fixed per fallback round (512 buckets)
constexpr int kSampleCap = 384;      // candidates ranked exactly in shared memory
constexpr int kSampleBatch = 2;      // row loads in flight per thread (more unrolling overflows the i-cache)

struct SampleShared {
    union {
        // bucket mass in 2^-48 fixed point as three 16-bit limbs summed with 32-bit shared
        // atomics (no sum overflows: weights <= 2^48, at most 65535 of them)
        struct {
            unsigned lo[kSampleBuckets], mid[kSampleBuckets], hi[kSampleBuckets];
            unsigned count[kSampleBuckets];
        } h;
        struct {
            unsigned long long w[kSampleCap];
            uint32_t key[kSampleCap];
            int id[kSampleCap];
        } c;
    };
    double xb[kSampleBuckets];     // centre x_b of bucket b in units of s - s0
    double ebase[kSampleBuckets];  // exp(x_b) * 2^48
    float red_f[kSampleThreads / 32], red_g[kSampleThreads / 32];
    int red_i[kSampleThreads / 32];
    uint32_t red_k[kSampleThreads / 32];
    unsigned long long draw;
    int chosen, ncand;
};

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

__device__ __forceinline__ void sample_hist_add(SampleShared& S, int bk, unsigned long long w) {
    atomicAdd(&S.h.lo[bk], static_cast<unsigned>(w & 0xffffu));
    atomicAdd(&S.h.mid[bk], static_cast<unsigned>((w >> 16) & 0xffffu));
    atomicAdd(&S.h.hi[bk], static_cast<unsigned>(w >> 32));
    atomicAdd(&S.h.count[bk], 1u);
}
// The first round's form: masses only. Its candidate count comes from the gather that ranks
// the crossing bucket (sample_pick), which reports an overflow instead.
__device__ __forceinline__ void sample_hist_add_mass(SampleShared& S, int bk, unsigned long long w) {
    atomicAdd(&S.h.lo[bk], static_cast<unsigned>(w & 0xffffu));
    atomicAdd(&S.h.mid[bk], static_cast<unsigned>((w >> 16) & 0xffffu));
    atomicAdd(&S.h.hi[bk], static_cast<unsigned>(w >> 32));
}
__device__ __forceinline__ unsigned long long sample_hist_mass(const SampleShared& S, int bk) {
    return (static_cast<unsigned long long>(S.h.hi[bk]) << 32) + (static_cast<unsigned long long>(S.h.mid[bk]) << 16) +
           S.h.lo[bk];
}
__device__ __forceinline__ void sample_hist_clear(SampleShared& S) {
    for (int i = threadIdx.x; i < kSampleBuckets; i += kSampleThreads)
        S.h.lo[i] = S.h.mid[i] = S.h.hi[i] = S.h.count[i] = 0u;
}

// Weights of one row. At temperature 1 with equal-width buckets at most 0.1 wide (score
// range <= 51.2), w = exp(x_b) * exp(x - x_b) with exp(x_b) from a per-bucket table and
// exp(d), |d| <= 0.0501, from its Taylor series to degree 8 (truncation below 6e-18
// relative): a weight agrees with the directly computed double exponential to within a
// few units of the last place before the rounding to 2^-48. Otherwise sample_weight_q.
struct SampleRowWeight {
    float s0, scale;
    double T;
    bool poly;
    const double* xb;
    const double* ebase;
    __device__ __forceinline__ int bucket(float v) const {
        const float p = fminf(__fmul_rn(__fsub_rn(s0, v), scale), static_cast<float>(kSampleBuckets - 1));
        return kSampleBuckets - 1 - static_cast<int>(p);
    }
    __device__ __forceinline__ unsigned long long operator()(float v, int b) const {
        if (!poly) return sample_weight_q(v, s0, T);
        const double d = static_cast<double>(__fsub_rn(v, s0)) - xb[b];
        double p = 1.0 / 40320.0;
        p = fma(p, d, 1.0 / 5040.0);
        p = fma(p, d, 1.0 / 720.0);
        p = fma(p, d, 1.0 / 120.0);
        p = fma(p, d, 1.0 / 24.0);
        p = fma(p, d, 1.0 / 6.0);
        p = fma(p, d, 0.5);
        p = fma(p, d, 1.0);
        p = fma(p, d, 1.0);
        return __double2ull_rn(ebase[b] * p);
    }
};

// Warp 0 scans the histogram in descending bucket order (lane L owns positions
// [16L, 16L + 16), position p <-> bucket nb - 1 - p). With `first` the draw comes from the
// row total, otherwise S.draw is the part left inside the previously fixed prefix. Leaves in
// S.chosen the bucket where the running mass first reaches the draw and in S.draw the part
// of it inside that bucket; when every weight rounded to zero below the draw, the lowest
// non-empty bucket with S.draw = ~0 (`counted`: emptiness from the counts, else from the
// masses; the first round's draw is below the row total, so it always finds a crossing).
// Called by warp 0 only.
__device__ __forceinline__ void sample_locate(SampleShared& S, int nb, bool first, uint64_t seed, int k,
                                              bool counted) {
    constexpr int PER = kSampleBuckets / 32;
    const int lane = threadIdx.x & 31;
    unsigned long long mine = 0;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        const int bk = nb - 1 - (lane * PER + e);
        if (bk >= 0) mine += sample_hist_mass(S, bk);
    }
    unsigned long long incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    const unsigned long long draw = first ? sample_draw(seed, k, __shfl_sync(0xffffffffu, incl, 31)) : S.draw;
    unsigned long long run = incl - mine, rem = 0;
    int found = -1, last_here = 0x7fffffff;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
        const int bk = nb - 1 - (lane * PER + e);
        if (bk < 0) continue;
        const unsigned long long m = sample_hist_mass(S, bk);
        // without counts an empty bucket is one of zero mass, which can never hold the crossing
        if (counted ? S.h.count[bk] == 0 : m == 0) continue;
        last_here = bk;
        if (found < 0 && run < draw && run + m >= draw) {
            found = bk;
            rem = draw - run;
        }
        run += m;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, found >= 0);
    if (hit) {
        if (lane == __ffs(hit) - 1) {
            S.chosen = found;
            S.draw = rem;
        }
        return;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) last_here = min(last_here, __shfl_xor_sync(0xffffffffu, last_here, o));
    if (lane == 0) {
        S.chosen = last_here;
        S.draw = ~0ull;
    }
}

// Among the scores selected by `in_set` (at most kSampleCap, gathered into shared memory)
// ordered by score descending then id ascending, the id where the running mass first
// reaches S.draw (the last one when none does; `none` when the set is empty). Ranks by
// counting: the mass before candidate i is the sum over the candidates ordered before it.
// kSamplePickOverflow when the set holds more than kSampleCap scores. Called by the whole block.
constexpr int kSamplePickOverflow = -2;
template <class Each, class Pred>
__device__ int sample_pick(SampleShared& S, Each each, const SampleRowWeight& wt, Pred in_set, int none) {
    const unsigned long long rem = S.draw;
    __syncthreads();  // every thread has read the draw and the chosen bucket
    if (threadIdx.x == 0) { S.ncand = 0; S.chosen = -1; }
    __syncthreads();
    each([&](int j, float v) {
        if (in_set(v)) {
            const int slot = atomicAdd(&S.ncand, 1);
            if (slot < kSampleCap) {
                S.c.key[slot] = float_key(v);
                S.c.id[slot] = j;
                S.c.w[slot] = wt(v, wt.poly ? wt.bucket(v) : 0);
            }
        }
    });
    __syncthreads();
    if (S.ncand > kSampleCap) return kSamplePickOverflow;
    const int n = S.ncand;
    if (n == 0) return none;
    uint32_t last_key = 0xffffffffu;
    int last_id = -1;
    for (int i = threadIdx.x; i < n; i += kSampleThreads) {
        const uint32_t ki = S.c.key[i];
        const int ii = S.c.id[i];
        unsigned long long before = 0;
        for (int j = 0; j < n; ++j) {
            const uint32_t kj = S.c.key[j];
            if (kj > ki || (kj == ki && S.c.id[j] < ii)) before += S.c.w[j];
        }
        if (before < rem && before + S.c.w[i] >= rem) S.chosen = ii;
        if (ki < last_key || (ki == last_key && ii > last_id)) { last_key = ki; last_id = ii; }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint32_t ok = __shfl_xor_sync(0xffffffffu, last_key, o);
        const int oi = __shfl_xor_sync(0xffffffffu, last_id, o);
        if (ok < last_key || (ok == last_key && oi > last_id)) { last_key = ok; last_id = oi; }
    }
    if (lane == 0) { S.red_k[warp] = last_key; S.red_i[warp] = last_id; }
    __syncthreads();
    if (S.chosen >= 0) return S.chosen;
    uint32_t bk = S.red_k[0];
    int bi = S.red_i[0];
    for (int w = 1; w < kSampleThreads / 32; ++w)
        if (S.red_k[w] < bk || (S.red_k[w] == bk && S.red_i[w] > bi)) { bk = S.red_k[w]; bi = S.red_i[w]; }
    return bi;
}

// One block per sequence row of logits [B][ld] (vocab V <= 65535). Greedy when
// temperature == 0 (first index of the maximum). Otherwise the inverse CDF of
// sample_token with top_p = 1 (inference.cpp:345-426): scores sorted descending (ties:
// lower id first), weights w = exp(double(s - s0) / T), draw = u * sum(w) with the
// reference's 24-bit uniform u, first position whose running sum reaches the draw. Weights
// are summed in exact 2^-48 fixed point (the sampled token equals the reference's except
// when the draw falls within ~1e-10 of a CDF boundary). The sorted order is found without
// a full sort:
//  1. one pass histograms the weights over 512 buckets of equal score width between the
//     row minimum and maximum (an order-preserving map: a higher score never lands in a
//     lower bucket, and equal scores share one), so a row of 16384 spreads ~32 per bucket;
//  2. a warp scan over the buckets, highest first, locates the bucket holding the crossing;
//  3. that bucket's scores are ranked in shared memory and the crossing read off.
// When the crossing bucket holds more than kSampleCap scores (a row of near-identical
// scores beside a distant maximum), the buckets are rebuilt from the order-preserving
// integer key of each score instead, 9 bits at a time, until the selected prefix holds at
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
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int b = blockIdx.x;
    const int step = counter ? *counter : 0;
    out += step;
    draw_offset += step;
    if (active && !active[b]) return;
    const float* row = logits + b * ld;
    const bool vec = (V & 3) == 0 && (ld & 3) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
    auto each = [&](auto&& f) {
        if (vec) {
            // kSampleBatch 16-byte loads in flight per thread before any is used
            const float4* r4 = reinterpret_cast<const float4*>(row);
            const int n4 = V >> 2;
            for (int base = 0; base < n4; base += kSampleThreads * kSampleBatch) {
                float4 x[kSampleBatch];
#pragma unroll
                for (int u = 0; u < kSampleBatch; ++u) {
                    const int j4 = base + u * kSampleThreads + tid;
                    x[u] = j4 < n4 ? r4[j4] : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < kSampleBatch; ++u) {
                    const int j4 = base + u * kSampleThreads + tid;
                    if (j4 < n4) {
                        f(4 * j4, x[u].x);
                        f(4 * j4 + 1, x[u].y);
                        f(4 * j4 + 2, x[u].z);
                        f(4 * j4 + 3, x[u].w);
                    }
                }
            }
        } else {
            for (int j = tid; j < V; j += kSampleThreads) f(j, row[j]);
        }
    };

    // maximum with its first index, and minimum
    float mx = -INFINITY, mn = INFINITY;
    int mi = 0x7fffffff;
    each([&](int j, float v) {
        if (v > mx || (v == mx && j < mi)) { mx = v; mi = j; }
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
    float s0 = S.red_f[0], smin = S.red_g[0];
    int best = S.red_i[0];
    for (int w = 1; w < kSampleThreads / 32; ++w) {
        if (S.red_f[w] > s0 || (S.red_f[w] == s0 && S.red_i[w] < best)) { s0 = S.red_f[w]; best = S.red_i[w]; }
        smin = fminf(smin, S.red_g[w]);
    }
    if (temperature == 0.f) {
        if (tid == 0) out[b * out_stride] = static_cast<uint16_t>(best);
        return;
    }
    const double T = static_cast<double>(temperature);
    const uint64_t seed = seeds[b];
    const int k = (draw_index ? draw_index[b] : 0) + draw_offset;

    // 1-3: buckets of equal score width, bucket kSampleBuckets-1 holding the maximum
    const float range = __fsub_rn(s0, smin);
    float scale = range > 0.f ? __fdiv_rn(static_cast<float>(kSampleBuckets), range) : 0.f;
    if (!(scale <= 3.0e38f)) scale = 0.f;
    // bucket half-width 0.5 / scale <= 0.05
    const SampleRowWeight wt{s0, scale, T, T == 1.0 && scale >= 10.f, S.xb, S.ebase};
    if (scale > 0.f) {
        sample_hist_clear(S);
        if (wt.poly) {
            const double inv = 1.0 / static_cast<double>(scale);
            for (int i = tid; i < kSampleBuckets; i += kSampleThreads) {
                const double x = -(static_cast<double>(kSampleBuckets - i) - 0.5) * inv;
                S.xb[i] = x;
                S.ebase[i] = exp(x) * 281474976710656.0;
            }
        }
        __syncthreads();
        each([&](int, float v) {
            const int bk = wt.bucket(v);
            sample_hist_add_mass(S, bk, wt(v, bk));
        });
        __syncthreads();
        if (warp == 0) sample_locate(S, kSampleBuckets, true, seed, k, false);
        __syncthreads();
        const int chosen = S.chosen;
        const int tok = sample_pick(S, each, wt, [&](float v) { return wt.bucket(v) == chosen; }, best);
        if (tok != kSamplePickOverflow) {
            if (tid == 0) out[b * out_stride] = static_cast<uint16_t>(tok);
            return;
        }
        // more than kSampleCap scores in the crossing bucket: every thread has passed the
        // gather's barrier, so the histogram (which the candidates share) may be rebuilt
    }

    // fallback: buckets of the order-preserving key, refined kSampleRadixBits at a time
    uint32_t prefix = 0;
    int bits = 0;
    unsigned ncand = 0;
    bool first = true;
    while (true) {
        const int width = min(kSampleRadixBits, 32 - bits);
        const int nb = 1 << width;
        sample_hist_clear(S);
        __syncthreads();
        each([&](int, float v) {
            const uint32_t key = float_key(v);
            if (bits > 0 && (key >> (32 - bits)) != prefix) return;
            const int bk = static_cast<int>((key >> (32 - bits - width)) & (nb - 1));
            sample_hist_add(S, bk, wt(v, wt.poly ? wt.bucket(v) : 0));
        });
        __syncthreads();
        if (warp == 0) sample_locate(S, nb, first, seed, k, true);
        __syncthreads();
        first = false;
        const int chosen = S.chosen;
        prefix = (prefix << width) | static_cast<uint32_t>(chosen);
        bits += width;
        ncand = S.h.count[chosen];
        __syncthreads();  // every thread has read the count before the next clear
        if (ncand <= static_cast<unsigned>(kSampleCap) || bits >= 32) break;
    }
    if (ncand > static_cast<unsigned>(kSampleCap)) {
        // More than kSampleCap scores share one exact value (every key bit fixed): equal
        // weights w, ordered by id, so the crossing is position m = ceil(rem / w) - 1 among
        // them, found by an id-ordered scan of warp 0 over the row.
        if (warp != 0) return;
        const uint32_t u = (prefix & 0x80000000u) ? (prefix & 0x7fffffffu) : ~prefix;
        const float fv = __uint_as_float(u);
        const unsigned long long w = wt(fv, wt.poly ? wt.bucket(fv) : 0);
        const unsigned long long rem = S.draw;
        long long m = static_cast<long long>(ncand) - 1;
        if (w > 0 && rem <= static_cast<unsigned long long>(ncand) * w) m = static_cast<long long>((rem + w - 1) / w) - 1;
        m = max(0LL, min(m, static_cast<long long>(ncand) - 1));
        long long seen = 0;
        for (int j0 = 0; j0 < V; j0 += 32) {
            const int j = j0 + lane;
            const bool hit = j < V && float_key(row[j]) == prefix;
            const unsigned mask = __ballot_sync(0xffffffffu, hit);
            const long long before = seen + __popc(mask & ((1u << lane) - 1u));
            if (hit && before == m) out[b * out_stride] = static_cast<uint16_t>(j);
            seen += __popc(mask);
            if (seen > m) break;
        }
        return;
    }
    const int tok = sample_pick(S, each, wt, [&](float v) {
        const uint32_t key = float_key(v);
        return (bits >= 32 ? key : (key >> (32 - bits))) == prefix;
    }, best);
    if (tid == 0) out[b * out_stride] = static_cast<uint16_t>(tok);
}
} // namespace mm

namespace mm {
// max |x| over n floats (NaN ignored), as float bits into *out: grid-stride 16-byte loads,
// a block maximum, one atomicMax per block (the bits of non-negative floats order like them).
__global__ void absmax_kernel(const float* __restrict__ x, long long n, unsigned int* __restrict__ out) {
    MM_PDL_ENTRY();
    __shared__ float red[32];
    float m = 0.f;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const long long i0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        const long long n4 = n >> 2;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        for (long long i = i0; i < n4; i += stride) {
            const float4 v = x4[i];
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        for (long long i = (n4 << 2) + i0; i < n; i += stride) m = fmaxf(m, fabsf(x[i]));
    } else {
        for (long long i = i0; i < n; i += stride) m = fmaxf(m, fabsf(x[i]));
    }
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
        if (m > 0.f) atomicMax(out, __float_as_uint(m));
    }
}
} // namespace mm
