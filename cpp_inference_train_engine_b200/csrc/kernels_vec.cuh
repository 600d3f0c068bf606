// Bandwidth-shaped versions of the row-wise and elementwise kernels: 16-byte loads and
// stores, 32-bit index arithmetic, rows held in registers between their reduction and
// their output. Each kernel computes exactly what its scalar counterpart in
// kernels_elem.cuh computes (same float expressions per element); the host picks the
// vector form when every row pitch and base address allows 16-byte (8-byte for 4-half
// stores) accesses, and the scalar form otherwise (the tiny test model's odd widths).
#pragma once
#include "kernels_elem.cuh"

namespace mm {

__device__ __forceinline__ float4 ld_f4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st_f4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ uint2 pack_h4(float a, float b, float c, float d) {
    const __half2 x = __floats2half2_rn(a, b), y = __floats2half2_rn(c, d);
    return make_uint2(*reinterpret_cast<const unsigned*>(&x), *reinterpret_cast<const unsigned*>(&y));
}
__device__ __forceinline__ uint4 pack_h8(const float* f) {
    uint4 u;
    const __half2 a = __floats2half2_rn(f[0], f[1]), b = __floats2half2_rn(f[2], f[3]);
    const __half2 c = __floats2half2_rn(f[4], f[5]), d = __floats2half2_rn(f[6], f[7]);
    u.x = *reinterpret_cast<const unsigned*>(&a);
    u.y = *reinterpret_cast<const unsigned*>(&b);
    u.z = *reinterpret_cast<const unsigned*>(&c);
    u.w = *reinterpret_cast<const unsigned*>(&d);
    return u;
}
__device__ __forceinline__ void unpack_h8(uint4 u, float* f) {
    const unsigned w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        f[2 * i] = p.x;
        f[2 * i + 1] = p.y;
    }
}

// RMSNorm, one warp per row, n <= 128 * MAXV and n % 4 == 0.
template <int MAXV>
__global__ void rmsnorm_v4_kernel(const float* __restrict__ x, long long ldx, const float* __restrict__ w, int T,
                                  int n, float eps, float* __restrict__ y32, long long ld32, __half* __restrict__ y16,
                                  long long ld16, float* __restrict__ inv_out, int split16 = 0) {
    MM_PDL_ENTRY();
    const int t = warp_row(), lane = threadIdx.x & 31;
    if (t >= T) return;
    const float* xr = x + t * ldx;
    float4 v[MAXV];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < MAXV; ++k) {
        const int j = (k * 32 + lane) * 4;
        if (j < n) {
            v[k] = ld_f4(xr + j);
            ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
        }
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
    if (inv_out && lane == 0) inv_out[t] = inv;
#pragma unroll
    for (int k = 0; k < MAXV; ++k) {
        const int j = (k * 32 + lane) * 4;
        if (j < n) {
            const float4 wv = ld_f4(w + j);
            const float4 o = make_float4(v[k].x * inv * wv.x, v[k].y * inv * wv.y, v[k].z * inv * wv.z,
                                         v[k].w * inv * wv.w);
            if (y32) st_f4(y32 + t * ld32 + j, o);
            if (y16) {
                const uint2 hi = pack_h4(o.x, o.y, o.z, o.w);
                *reinterpret_cast<uint2*>(y16 + t * ld16 + j) = hi;
                if (split16) {  // [hi | lo (| hi)]: lo = fp16(y - hi) at column n + j
                    const __half2 a = *reinterpret_cast<const __half2*>(&hi.x), b = *reinterpret_cast<const __half2*>(&hi.y);
                    *reinterpret_cast<uint2*>(y16 + t * ld16 + n + j) =
                        pack_h4(o.x - __low2float(a), o.y - __high2float(a), o.z - __low2float(b), o.w - __high2float(b));
                    if (split16 == 2) *reinterpret_cast<uint2*>(y16 + t * ld16 + 2 * n + j) = hi;
                }
            }
        }
    }
}

// RMSNorm backward, one warp per row over a fixed row assignment; dw partial sums per
// block go to dw_part[blockIdx.x][n] in a fixed order (colsum_kernel adds them up), so the
// norm-weight gradient is reproducible run to run. Block = 256 threads, dynamic shared
// memory 8 * n floats.
template <int MAXV>
__global__ void __launch_bounds__(256) rmsnorm_backward_v4_kernel(
    const float* __restrict__ x, long long ldx, const float* __restrict__ w, const float* __restrict__ dy,
    long long lddy, const float* __restrict__ add, long long ldadd, int T, int n, float eps,
    float* __restrict__ dx32, long long lddx, __half* __restrict__ dx16, long long lddx16,
    float* __restrict__ dw_part) {
    MM_PDL_ENTRY();
    extern __shared__ float4 acc_sh[];  // [warps][n / 4]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    const int nq = n >> 2;
    float4 wv[MAXV], acc[MAXV];
#pragma unroll
    for (int k = 0; k < MAXV; ++k) {
        const int j = (k * 32 + lane) * 4;
        acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < n) wv[k] = ld_f4(w + j);
    }
    for (int t = blockIdx.x * warps + warp; t < T; t += gridDim.x * warps) {
        const float* xr = x + t * ldx;
        const float* gr = dy + t * lddy;
        float4 xv[MAXV], gv[MAXV], av[MAXV];
        float sq = 0.f, dot = 0.f;
        // the added gradient is loaded with x and dy, so its latency hides behind theirs
#pragma unroll
        for (int k = 0; k < MAXV; ++k) {
            const int j = (k * 32 + lane) * 4;
            av[k] = (add && j < n) ? ld_f4(add + t * ldadd + j) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < MAXV; ++k) {
            const int j = (k * 32 + lane) * 4;
            if (j < n) {
                xv[k] = ld_f4(xr + j);
                gv[k] = ld_f4(gr + j);
                sq += xv[k].x * xv[k].x + xv[k].y * xv[k].y + xv[k].z * xv[k].z + xv[k].w * xv[k].w;
                dot += gv[k].x * wv[k].x * xv[k].x + gv[k].y * wv[k].y * xv[k].y + gv[k].z * wv[k].z * xv[k].z +
                       gv[k].w * wv[k].w * xv[k].w;
            }
        }
        sq = warp_sum(sq);
        dot = warp_sum(dot);
        const float inv = 1.0f / sqrtf(sq / static_cast<float>(n) + eps);
        const float corr = dot * inv * inv * inv / static_cast<float>(n);
#pragma unroll
        for (int k = 0; k < MAXV; ++k) {
            const int j = (k * 32 + lane) * 4;
            if (j < n) {
                float4 o = make_float4(gv[k].x * wv[k].x * inv - xv[k].x * corr, gv[k].y * wv[k].y * inv - xv[k].y * corr,
                                       gv[k].z * wv[k].z * inv - xv[k].z * corr, gv[k].w * wv[k].w * inv - xv[k].w * corr);
                if (add) {
                    o.x += av[k].x;
                    o.y += av[k].y;
                    o.z += av[k].z;
                    o.w += av[k].w;
                }
                if (dx32) st_f4(dx32 + t * lddx + j, o);
                if (dx16) *reinterpret_cast<uint2*>(dx16 + t * lddx16 + j) = pack_h4(o.x, o.y, o.z, o.w);
                acc[k].x += gv[k].x * xv[k].x * inv;
                acc[k].y += gv[k].y * xv[k].y * inv;
                acc[k].z += gv[k].z * xv[k].z * inv;
                acc[k].w += gv[k].w * xv[k].w * inv;
            }
        }
    }
#pragma unroll
    for (int k = 0; k < MAXV; ++k) {
        const int j = (k * 32 + lane) * 4;
        if (j < n) acc_sh[warp * nq + (j >> 2)] = acc[k];
    }
    __syncthreads();
    for (int q = threadIdx.x; q < nq; q += blockDim.x) {
        float4 s = acc_sh[q];
        for (int v = 1; v < warps; ++v) {
            const float4 o = acc_sh[v * nq + q];
            s.x += o.x;
            s.y += o.y;
            s.z += o.z;
            s.w += o.w;
        }
        st_f4(dw_part + static_cast<long long>(blockIdx.x) * n + 4 * q, s);
    }
}

// dw[j] += scale * sum_r part[r][j] in a fixed order: block (32, kColsumGroups) covers 32
// columns, row group y sums rows y, y + kColsumGroups, ... and the group sums are added in
// order (many short row walks in flight instead of a few long ones).
constexpr int kColsumGroups = 32;
__global__ void colsum_kernel(const float* __restrict__ part, int rows, int n, const float* __restrict__ scale,
                              float* __restrict__ dw) {
    MM_PDL_ENTRY();
    __shared__ float grp[kColsumGroups][33];
    const int j = blockIdx.x * 32 + threadIdx.x;
    float s = 0.f;
    if (j < n)
        for (int r = threadIdx.y; r < rows; r += kColsumGroups) s += part[static_cast<long long>(r) * n + j];
    grp[threadIdx.y][threadIdx.x] = s;
    __syncthreads();
    if (threadIdx.y == 0 && j < n) {
        float t = grp[0][threadIdx.x];
        for (int y = 1; y < kColsumGroups; ++y) t += grp[y][threadIdx.x];
        dw[j] += t * (scale ? *scale : 1.0f);
    }
}

// SwiGLU forward, 8 columns per thread.
__global__ void swiglu_v8_kernel(const __half* __restrict__ gate, const __half* __restrict__ up, long long ld, int T,
                                 int n, __half* __restrict__ out, long long ldo) {
    MM_PDL_ENTRY();
    const int nv = n >> 3;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * nv) return;
    const int t = i / nv, c = (i - t * nv) << 3;
    float g[8], u[8], o[8];
    unpack_h8(*reinterpret_cast<const uint4*>(gate + t * ld + c), g);
    unpack_h8(*reinterpret_cast<const uint4*>(up + t * ld + c), u);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = g[k] * sigmoid_ref(g[k]) * u[k];
    *reinterpret_cast<uint4*>(out + t * ldo + c) = pack_h8(o);
}

// SwiGLU backward, 8 columns per thread.
__global__ void swiglu_backward_v8_kernel(const __half* __restrict__ gate, const __half* __restrict__ up,
                                          long long ld, const float* __restrict__ dy, long long lddy, int T, int n,
                                          __half* __restrict__ dg, __half* __restrict__ du, long long ldo) {
    MM_PDL_ENTRY();
    const int nv = n >> 3;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * nv) return;
    const int t = i / nv, c = (i - t * nv) << 3;
    float x[8], u[8], g[8], a[8], b[8];
    unpack_h8(*reinterpret_cast<const uint4*>(gate + t * ld + c), x);
    unpack_h8(*reinterpret_cast<const uint4*>(up + t * ld + c), u);
    const float4 g0 = ld_f4(dy + t * lddy + c), g1 = ld_f4(dy + t * lddy + c + 4);
    g[0] = g0.x; g[1] = g0.y; g[2] = g0.z; g[3] = g0.w;
    g[4] = g1.x; g[5] = g1.y; g[6] = g1.z; g[7] = g1.w;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float s = sigmoid_ref(x[k]);
        a[k] = g[k] * u[k] * (s + x[k] * s * (1.f - s));
        b[k] = g[k] * x[k] * s;
    }
    *reinterpret_cast<uint4*>(dg + t * ldo + c) = pack_h8(a);
    *reinterpret_cast<uint4*>(du + t * ldo + c) = pack_h8(b);
}

// swiglu_backward_v8_kernel with dy in fp16.
__global__ void swiglu_backward_h8_kernel(const __half* __restrict__ gate, const __half* __restrict__ up,
                                          long long ld, const __half* __restrict__ dy, long long lddy, int T, int n,
                                          __half* __restrict__ dg, __half* __restrict__ du, long long ldo) {
    MM_PDL_ENTRY();
    const int nv = n >> 3;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * nv) return;
    const int t = i / nv, c = (i - t * nv) << 3;
    float x[8], u[8], g[8], a[8], b[8];
    unpack_h8(*reinterpret_cast<const uint4*>(gate + t * ld + c), x);
    unpack_h8(*reinterpret_cast<const uint4*>(up + t * ld + c), u);
    unpack_h8(*reinterpret_cast<const uint4*>(dy + t * lddy + c), g);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float s = sigmoid_ref(x[k]);
        a[k] = g[k] * u[k] * (s + x[k] * s * (1.f - s));
        b[k] = g[k] * x[k] * s;
    }
    *reinterpret_cast<uint4*>(dg + t * ldo + c) = pack_h8(a);
    *reinterpret_cast<uint4*>(du + t * ldo + c) = pack_h8(b);
}

// fp32 -> fp16, 4 columns per thread.
__global__ void to_half_v4_kernel(const float* __restrict__ in, long long ldin, int T, int n, __half* __restrict__ out,
                                  long long ldo) {
    MM_PDL_ENTRY();
    const int nv = n >> 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * nv) return;
    const int t = i / nv, c = (i - t * nv) << 2;
    const float4 v = ld_f4(in + t * ldin + c);
    *reinterpret_cast<uint2*>(out + t * ldo + c) = pack_h4(v.x, v.y, v.z, v.w);
}

// k = [k_nope_h | k_rope] per head, 8 output columns per thread (nope % 8 == 0, rope % 8 == 0).
__global__ void assemble_k_v8_kernel(const float* __restrict__ k_nope, long long ldn, const float* __restrict__ k_rope,
                                     int T, int H, int nope, int rope, __half* __restrict__ k, long long ldk) {
    MM_PDL_ENTRY();
    const int qk = nope + rope, nv = (H * qk) >> 3;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * nv) return;
    const int t = i / nv, c = (i - t * nv) << 3;
    const int h = c / qk, j = c - h * qk;
    const float* src = j < nope ? k_nope + t * ldn + h * nope + j : k_rope + t * rope + (j - nope);
    const float4 a = ld_f4(src), b = ld_f4(src + 4);
    const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    *reinterpret_cast<uint4*>(k + t * ldk + c) = pack_h8(f);
}

// Adjacent-pair RoPE over rows of `heads` groups of `width` columns, 4 columns per thread
// (width, begin and rope even; the row widths multiples of 4).
__global__ void rope_rows_v4_kernel(const float* __restrict__ in, long long ldin, int T, int seq,
                                    const int* __restrict__ pos_base, int heads, int width, int begin, int rope,
                                    const float* __restrict__ cos_t, const float* __restrict__ sin_t, int inverse,
                                    float* __restrict__ out32, long long ld32, __half* __restrict__ out16,
                                    long long ld16) {
    MM_PDL_ENTRY();
    const int nv = (heads * width) >> 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * nv) return;
    const int t = i / nv, c = (i - t * nv) << 2;
    const int p = (pos_base ? pos_base[t / seq] : 0) + t % seq;
    const int half_r = rope / 2;
    float4 v = ld_f4(in + t * ldin + c);
    float* f = reinterpret_cast<float*>(&v);
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
        const int cc = (c + e) % width;
        if (cc >= begin && cc < begin + rope) {
            const int pair = (cc - begin) >> 1;
            const float cs = cos_t[p * half_r + pair];
            const float sn = inverse ? -sin_t[p * half_r + pair] : sin_t[p * half_r + pair];
            const float a = f[e], b = f[e + 1];
            f[e] = a * cs - b * sn;
            f[e + 1] = a * sn + b * cs;
        }
    }
    if (out32) st_f4(out32 + t * ld32 + c, v);
    if (out16) *reinterpret_cast<uint2*>(out16 + t * ld16 + c) = pack_h4(v.x, v.y, v.z, v.w);
}

// D[t, h] = sum_c dout[t, h, c] * out[t, h, c] in column order, 8 columns per load.
__global__ void attn_rowdot_v8_kernel(const __half* __restrict__ dout, const __half* __restrict__ out, int T, int H,
                                      int DV, float* __restrict__ Dd) {
    MM_PDL_ENTRY();
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= T * H) return;
    const long long o = static_cast<long long>(idx) * DV;  // rows are H * DV wide
    float s = 0.f;
    for (int c = 0; c < DV; c += 8) {
        float a[8], b[8];
        unpack_h8(*reinterpret_cast<const uint4*>(dout + o + c), a);
        unpack_h8(*reinterpret_cast<const uint4*>(out + o + c), b);
#pragma unroll
        for (int k = 0; k < 8; ++k) s += a[k] * b[k];
    }
    Dd[idx] = s;
}

// g[t, j] = scale * coef[t] * (exp(l - lse) - [j == target]) in fp16, 4 columns per thread.
__global__ void vocab_grad_v4_kernel(const float* __restrict__ logits, long long ld, int V,
                                     const uint16_t* __restrict__ target, const float* __restrict__ lse,
                                     const float* __restrict__ coef, const float* __restrict__ scale, int T,
                                     __half* __restrict__ g, long long ldg) {
    MM_PDL_ENTRY();
    const int nv = V >> 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * nv) return;
    const int t = i / nv, c = (i - t * nv) << 2;
    const float cf = coef[t] * *scale;
    uint2* dst = reinterpret_cast<uint2*>(g + t * ldg + c);
    if (cf == 0.f) {
        *dst = make_uint2(0u, 0u);
        return;
    }
    const float L = lse[t];
    const int tg = target[t];
    const float4 l = ld_f4(logits + t * ld + c);
    const float p0 = __expf(l.x - L), p1 = __expf(l.y - L), p2 = __expf(l.z - L), p3 = __expf(l.w - L);
    *dst = pack_h4(cf * (p0 - (c == tg ? 1.f : 0.f)), cf * (p1 - (c + 1 == tg ? 1.f : 0.f)),
                   cf * (p2 - (c + 2 == tg ? 1.f : 0.f)), cf * (p3 - (c + 3 == tg ? 1.f : 0.f)));
}

// Split-K reduction, 4 columns per thread (N % 4 == 0, 16-byte aligned rows).
__global__ void splitk_reduce_v4_kernel(const float* __restrict__ part, int splits, long long split_stride, int M,
                                        int N, float* __restrict__ out, long long ldc, float alpha,
                                        const float* __restrict__ alpha_ptr) {
    MM_PDL_ENTRY();
    const int nv = N >> 2;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= M * nv) return;
    const int r = i / nv, c = (i - r * nv) << 2;
    const long long e = static_cast<long long>(r) * N + c;
    float4 s = ld_f4(part + e);
    for (int z = 1; z < splits; ++z) {
        const float4 v = ld_f4(part + z * split_stride + e);
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
    }
    const float a = alpha * (alpha_ptr ? *alpha_ptr : 1.0f);
    float4 o = ld_f4(out + r * ldc + c);
    o.x += a * s.x;
    o.y += a * s.y;
    o.z += a * s.z;
    o.w += a * s.w;
    st_f4(out + r * ldc + c, o);
}

} // namespace mm
