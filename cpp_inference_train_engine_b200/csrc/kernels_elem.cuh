// Row-wise and elementwise kernels of the MLA block: embedding gather/scatter, RMSNorm
// forward/backward, adjacent-pair RoPE, SwiGLU forward/backward and the small layout
// moves around the latent projections. One warp per token row; rows are short
// (<= a few thousand elements), so a warp-stride loop with shuffle reductions keeps
// every load coalesced and needs no shared memory.
#pragma once
#include "common.cuh"

namespace mm {

__device__ __forceinline__ int warp_row() { return (blockIdx.x * blockDim.x + threadIdx.x) >> 5; }

// x[t, :] = E[token[t], :] (fp32 master table), ops-equivalent of model.cpp:94-98.
__global__ void embed_kernel(const uint16_t* __restrict__ tokens, const float* __restrict__ E,
                             float* __restrict__ x, int T, int d, int V, int* err) {
    MM_PDL_ENTRY();
    const int t = warp_row(), lane = threadIdx.x & 31;
    if (t >= T) return;
    const int tok = tokens[t];
    if (tok >= V) {
        if (lane == 0) raise_error(err, kErrBadIndex);
        return;
    }
    const float* src = E + static_cast<long long>(tok) * d;
    float* dst = x + static_cast<long long>(t) * d;
    for (int j = lane; j < d; j += 32) dst[j] = src[j];
}

// RMSNorm (ops.cpp:33-45): y = x * rsqrt(mean(x^2) + eps) * w. Writes any of: fp32 y,
// fp16 y, and the row's inverse rms for the backward pass.
__global__ void rmsnorm_kernel(const float* __restrict__ x, long long ldx, const float* __restrict__ w,
                               int T, int n, float eps, float* __restrict__ y32, long long ld32,
                               __half* __restrict__ y16, long long ld16, float* __restrict__ inv_out,
                               int split16 = 0) {
    MM_PDL_ENTRY();
    const int t = warp_row(), lane = threadIdx.x & 31;
    if (t >= T) return;
    const float* xr = x + t * ldx;
    float ss = 0.f;
    for (int j = lane; j < n; j += 32) ss += xr[j] * xr[j];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
    if (inv_out && lane == 0) inv_out[t] = inv;
    for (int j = lane; j < n; j += 32) {
        const float v = xr[j] * inv * w[j];
        if (y32) y32[t * ld32 + j] = v;
        if (y16) {
            const __half hi = __float2half_rn(v);
            y16[t * ld16 + j] = hi;
            if (split16) y16[t * ld16 + n + j] = __float2half_rn(v - __half2float(hi));
            if (split16 == 2) y16[t * ld16 + 2 * n + j] = hi;
        }
    }
}

// RMSNorm backward (ops.cpp:46-64). dx = dy*w*inv - x*(dot*inv^3/n), optionally plus
// `add` (the residual branch), written as fp32 and/or fp16. dw += grad_scale * sum_t
// dy*x*inv, reduced per block in shared memory, then one atomicAdd per column.
__global__ void rmsnorm_backward_kernel(const float* __restrict__ x, long long ldx,
                                        const float* __restrict__ w, const float* __restrict__ dy,
                                        long long lddy, const float* __restrict__ add, long long ldadd,
                                        int T, int n, float eps, float* __restrict__ dx32,
                                        long long lddx, __half* __restrict__ dx16, long long lddx16,
                                        float* __restrict__ dw, const float* __restrict__ grad_scale) {
    MM_PDL_ENTRY();
    extern __shared__ float dw_acc[];  // [n]
    for (int j = threadIdx.x; j < n; j += blockDim.x) dw_acc[j] = 0.f;
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
        const float* xr = x + t * ldx;
        const float* gr = dy + t * lddy;
        float sq = 0.f, dot = 0.f;
        for (int j = lane; j < n; j += 32) {
            sq += xr[j] * xr[j];
            dot += gr[j] * w[j] * xr[j];
        }
        sq = warp_sum(sq);
        dot = warp_sum(dot);
        const float inv = 1.0f / sqrtf(sq / static_cast<float>(n) + eps);
        const float corr = dot * inv * inv * inv / static_cast<float>(n);
        for (int j = lane; j < n; j += 32) {
            float v = gr[j] * w[j] * inv - xr[j] * corr;
            if (add) v += add[t * ldadd + j];
            if (dx32) dx32[t * lddx + j] = v;
            if (dx16) dx16[t * lddx16 + j] = __float2half_rn(v);
            atomicAdd(&dw_acc[j], gr[j] * xr[j] * inv);
        }
    }
    __syncthreads();
    const float s = grad_scale ? *grad_scale : 1.0f;
    for (int j = threadIdx.x; j < n; j += blockDim.x) atomicAdd(&dw[j], dw_acc[j] * s);
}

// Adjacent-pair RoPE (ops.cpp:88-108) on columns [begin, begin+rope) of each of `heads`
// groups of `width` columns. cos/sin tables [max_seq][rope/2] are built on the host with
// the reference's own float arithmetic. Position = pos_base[row / seq] + row % seq (or
// row % seq when pos_base is null). `inverse` negates the angle (the backward pass).
// Reads fp32 `in`, writes fp32 `out32` and/or fp16 `out16` for the whole row width, so it
// doubles as the fp32->fp16 conversion of q.
__global__ void rope_rows_kernel(const float* __restrict__ in, long long ldin, int T, int seq,
                                 const int* __restrict__ pos_base, int heads, int width, int begin,
                                 int rope, const float* __restrict__ cos_t,
                                 const float* __restrict__ sin_t, int inverse,
                                 float* __restrict__ out32, long long ld32,
                                 __half* __restrict__ out16, long long ld16) {
    MM_PDL_ENTRY();
    const int t = warp_row(), lane = threadIdx.x & 31;
    if (t >= T) return;
    const int p = (pos_base ? pos_base[t / seq] : 0) + t % seq;
    const int half_r = rope / 2;
    const float* xr = in + t * ldin;
    const int total = heads * width;
    for (int j = lane; j < total; j += 32) {
        const int c = j % width;
        float v = xr[j];
        if (c >= begin && c < begin + rope) {
            const int pair = (c - begin) >> 1;
            const float cs = cos_t[p * half_r + pair];
            const float sn = inverse ? -sin_t[p * half_r + pair] : sin_t[p * half_r + pair];
            if (((c - begin) & 1) == 0) {
                const float b = xr[j + 1];
                v = v * cs - b * sn;
            } else {
                const float a = xr[j - 1];
                v = a * sn + v * cs;
            }
        }
        if (out32) out32[t * ld32 + j] = v;
        if (out16) out16[t * ld16 + j] = __float2half_rn(v);
    }
}

// Latent split after w_dkv (model.cpp:110-121): from kv_pack [T][kv_rank + rope] the
// rope key is rotated into k_rope32 [T][rope]; the raw latent stays in place for the
// RMSNorm that follows.
__global__ void rope_key_kernel(const float* __restrict__ kvp, long long ldkvp, int kv_rank,
                                int rope, int T, int seq, const int* __restrict__ pos_base,
                                const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                float* __restrict__ k_rope, __half* __restrict__ cache_rope,
                                long long cache_ld) {
    MM_PDL_ENTRY();
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    const int half_r = rope / 2;
    if (idx >= T * half_r) return;
    const int t = idx / half_r, pair = idx % half_r;
    const int p = (pos_base ? pos_base[t / seq] : 0) + t % seq;
    const float a = kvp[t * ldkvp + kv_rank + 2 * pair], b = kvp[t * ldkvp + kv_rank + 2 * pair + 1];
    const float cs = cos_t[p * half_r + pair], sn = sin_t[p * half_r + pair];
    const float x0 = a * cs - b * sn, x1 = a * sn + b * cs;
    if (k_rope) {
        k_rope[t * rope + 2 * pair] = x0;
        k_rope[t * rope + 2 * pair + 1] = x1;
    }
    if (cache_rope) {
        cache_rope[t * cache_ld + 2 * pair] = __float2half_rn(x0);
        cache_rope[t * cache_ld + 2 * pair + 1] = __float2half_rn(x1);
    }
}

// k = [k_nope_h | k_rope] per head (model.cpp:124-131), fp16 [T][H*qk].
__global__ void assemble_k_kernel(const float* __restrict__ k_nope, long long ldn,
                                  const float* __restrict__ k_rope, int T, int H, int nope, int rope,
                                  __half* __restrict__ k, long long ldk) {
    MM_PDL_ENTRY();
    const int qk = nope + rope;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(T) * H * qk) return;
    const int t = static_cast<int>(idx / (H * qk));
    const int c = static_cast<int>(idx % (H * qk));
    const int h = c / qk, j = c % qk;
    const float v = j < nope ? k_nope[t * ldn + h * nope + j] : k_rope[t * rope + (j - nope)];
    k[t * ldk + c] = __float2half_rn(v);
}


// gated = gate * sigmoid(gate) * up (ops.cpp:71-77).
__global__ void swiglu_kernel(const __half* __restrict__ gate, const __half* __restrict__ up,
                              long long ld, int T, int n, __half* __restrict__ out, long long ldo) {
    MM_PDL_ENTRY();
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(T) * n) return;
    const int t = static_cast<int>(idx / n), j = static_cast<int>(idx % n);
    const float g = __half2float(gate[t * ld + j]), u = __half2float(up[t * ld + j]);
    out[t * ldo + j] = __float2half_rn(g * sigmoid_ref(g) * u);
}

// SwiGLU backward (ops.cpp:78-87) to fp16 dgate/dup.
__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__half v) { return __half2float(v); }

// dy in fp32 or fp16 (the scaled backward carries it in fp16)
template <class DY>
__global__ void swiglu_backward_kernel(const __half* __restrict__ gate, const __half* __restrict__ up,
                                       long long ld, const DY* __restrict__ dy, long long lddy,
                                       int T, int n, __half* __restrict__ dg, __half* __restrict__ du,
                                       long long ldo) {
    MM_PDL_ENTRY();
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(T) * n) return;
    const int t = static_cast<int>(idx / n), j = static_cast<int>(idx % n);
    const float x = __half2float(gate[t * ld + j]), u = __half2float(up[t * ld + j]);
    const float g = to_float(dy[t * lddy + j]);
    const float s = sigmoid_ref(x);
    dg[t * ldo + j] = __float2half_rn(g * u * (s + x * s * (1.f - s)));
    du[t * ldo + j] = __float2half_rn(g * x * s);
}

// fp32 -> fp16 copy of a [T][n] block (optionally scaled).
__global__ void to_half_kernel(const float* __restrict__ in, long long ldin, int T, int n,
                               __half* __restrict__ out, long long ldo) {
    MM_PDL_ENTRY();
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(T) * n) return;
    const int t = static_cast<int>(idx / n), j = static_cast<int>(idx % n);
    out[t * ldo + j] = __float2half_rn(in[t * ldin + j]);
}

// Vocabulary-head operand: h3 = [hi(h) | lo(h) | hi(h)] in fp16, [T][3d], so that one
// GEMM against E3 = [hi(64E) | hi(64E) | lo(64E)] accumulates hi*hi + lo*hi + hi*lo:
// a float32-accurate h * E^T on the fp16 tensor pipe.
__global__ void split3_rows_kernel(const float* __restrict__ h, long long ldh, int T, int d,
                                   __half* __restrict__ h3, long long ld3) {
    MM_PDL_ENTRY();
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(T) * d) return;
    const int t = static_cast<int>(idx / d), j = static_cast<int>(idx % d);
    const float v = h[t * ldh + j];
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(v - __half2float(hi));
    h3[t * ld3 + j] = hi;
    h3[t * ld3 + d + j] = lo;
    h3[t * ld3 + 2 * d + j] = hi;
}

// Embedding gradient from the input gather (model.cpp:238-240): dE[tok] += s * dy[t], made
// independent of the order in which tokens sharing an id arrive: each row's sum is taken
// exactly in 64-bit fixed point (integer additions commute), then converted once. The unit
// is 2^-k with k from the chunk's max |dy| (m < 2^e) and token count (T < 2^et),
// k = 62 - e - et, so |q| < 2^(62 - et) and no sum of T terms reaches 2^62.
__device__ __forceinline__ int embed_fixed_shift(unsigned int max_bits, int T) {
    const float m = __uint_as_float(max_bits);
    if (!(m > 0.f) || !isfinite(m)) return 0;
    int e = 0, et = 0;
    frexpf(m, &e);
    frexpf(static_cast<float>(T), &et);
    return 62 - e - et;
}
// dy rows in fixed point into acc[V][d]; a non-finite dy sets *nonfinite instead.
__global__ void embed_grad_fixed_kernel(const uint16_t* __restrict__ tokens, const float* __restrict__ dy, int T,
                                        int d, unsigned long long* __restrict__ acc,
                                        const unsigned int* __restrict__ max_bits, int* __restrict__ nonfinite) {
    MM_PDL_ENTRY();
    const int t = warp_row(), lane = threadIdx.x & 31;
    if (t >= T) return;
    const int k = embed_fixed_shift(*max_bits, T);
    const long long row = static_cast<long long>(tokens[t]) * d;
    for (int j = lane; j < d; j += 32) {
        const float v = dy[static_cast<long long>(t) * d + j];
        if (!isfinite(v)) {
            *nonfinite = 1;
            continue;
        }
        const long long q = __double2ll_rn(ldexp(static_cast<double>(v), k));
        if (q) atomicAdd(&acc[row + j], static_cast<unsigned long long>(q));
    }
}
// dE += s * acc * 2^-k over every entry, clearing acc for the next chunk; a non-finite input
// is passed on as a NaN in dE[0] (the optimizer's finiteness check reports it).
__global__ void embed_grad_convert_kernel(unsigned long long* __restrict__ acc, long long n, int T,
                                          const unsigned int* __restrict__ max_bits,
                                          const int* __restrict__ nonfinite, const float* __restrict__ grad_scale,
                                          float* __restrict__ dE) {
    MM_PDL_ENTRY();
    const int k = embed_fixed_shift(*max_bits, T);
    const float s = grad_scale ? *grad_scale : 1.0f;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long q = static_cast<long long>(acc[i]);
        if (q) {
            dE[i] += static_cast<float>(ldexp(static_cast<double>(q), -k)) * s;
            acc[i] = 0ull;
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0 && *nonfinite) dE[0] = __int_as_float(0x7fc00000);
}

// Key gradient split (model.cpp:204-215): dk_nope (fp16, per head) and the rope-key
// gradient summed over heads (fp32), before its inverse rotation.
__global__ void split_dk_kernel(const float* __restrict__ dk, int T, int H, int nope, int rope,
                                __half* __restrict__ dkn, long long lddkn, float* __restrict__ drope) {
    MM_PDL_ENTRY();
    const int t = warp_row(), lane = threadIdx.x & 31;
    if (t >= T) return;
    const int qk = nope + rope;
    const float* row = dk + static_cast<long long>(t) * H * qk;
    for (int c = lane; c < H * nope; c += 32) {
        const int h = c / nope, j = c % nope;
        dkn[t * lddkn + c] = __float2half_rn(row[h * qk + j]);
    }
    for (int j = lane; j < rope; j += 32) {
        float s = 0.f;
        for (int h = 0; h < H; ++h) s += row[h * qk + nope + j];
        drope[t * rope + j] = s;
    }
}

// kv_pack gradient = [d(raw latent) | d(rope key)] in fp16 (model.cpp:221-227).
__global__ void pack_dkv_kernel(const float* __restrict__ dlat, const float* __restrict__ drope,
                                int T, int kv_rank, int rope, __half* __restrict__ out, long long ldo) {
    MM_PDL_ENTRY();
    const int w = kv_rank + rope;
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<long long>(T) * w) return;
    const int t = static_cast<int>(idx / w), j = static_cast<int>(idx % w);
    const float v = j < kv_rank ? dlat[t * kv_rank + j] : drope[t * rope + (j - kv_rank)];
    out[t * ldo + j] = __float2half_rn(v);
}

} // namespace mm
