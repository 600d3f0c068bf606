// Causal attention forward/backward on the tensor pipe for the teacher-forced passes
// (ops::attention / ops::attention_backward, ops.cpp:109-172), FlashAttention-2 style:
// 64x64 tiles staged in shared memory, warp-level mma.sync m16n8k16 (fp16 in, fp32
// accumulate) with ldmatrix fragment loads, online softmax in registers. The [T, T]
// probability matrix is never materialised; the forward keeps the per-row log-sum-exp
// (base 2) and the backward recomputes probabilities from it.
//
// Backward is two kernels with no atomics (deterministic): dK/dV per key tile iterating
// over the query tiles at or below the diagonal, and dQ per query tile iterating over the
// key tiles at or above it.
#pragma once
#include "common.cuh"

namespace mm {

namespace fa {

constexpr int kTile = 64;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
// D = A * B + D, m16n8k16, fp16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Copies rows [row0, row0 + 64) of a head's [*, D] slice (row pitch ld elements) into a
// padded shared tile; rows at or beyond `rows` are zero.
template <int D, int LD>
__device__ __forceinline__ void load_tile(__half (*dst)[LD], const __half* __restrict__ src, long long ld,
                                          int rows) {
    constexpr int VPR = D / 8;  // 16-byte vectors per row
    for (int e = threadIdx.x; e < kTile * VPR; e += blockDim.x) {
        const int r = e / VPR, c = (e % VPR) * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < rows) v = *reinterpret_cast<const uint4*>(src + r * ld + c);
        *reinterpret_cast<uint4*>(&dst[r][c]) = v;
    }
}

// load_tile through cp.async (no register round trip); the caller commits and waits.
template <int D, int LD>
__device__ __forceinline__ void load_tile_async(__half (*dst)[LD], const __half* __restrict__ src, long long ld,
                                                int rows) {
    constexpr int VPR = D / 8;
    for (int e = threadIdx.x; e < kTile * VPR; e += blockDim.x) {
        const int r = e / VPR, c = (e % VPR) * 8;
        const bool ok = r < rows;
        cp_async16(&dst[r][c], src + (ok ? r : 0) * ld + c, ok);
    }
}

// A fragments (16 rows x D) of rows [r0, r0+16) of a shared tile.
template <int D, int LD>
__device__ __forceinline__ void load_a_frags(uint32_t (&a)[D / 16][4], __half (*tile)[LD], int r0, int lane) {
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) ldsm_x4(a[kk], &tile[r0 + (lane & 15)][kk * 16 + (lane >> 4) * 8]);
}

// acc[NT n-tiles of 8] += A(16 x D) * rows[0..8 NT)^T of `tile` (B operand: tile rows are n,
// cols k). NT = kTile / 8 covers a whole tile; pass tile + r0 for rows [r0, r0 + 8 NT).
template <int D, int LD, int NT = kTile / 8>
__device__ __forceinline__ void mma_abt(float (&acc)[NT][4], const uint32_t (&a)[D / 16][4], __half (*tile)[LD],
                                        int lane) {
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
#pragma unroll
        for (int n2 = 0; n2 < NT / 2; ++n2) {
            uint32_t b[4];
            ldsm_x4(b, &tile[n2 * 16 + (lane & 7) + ((lane >> 4) << 3)][kk * 16 + ((lane >> 3) & 1) * 8]);
            mma16816(acc[2 * n2], a[kk], b[0], b[1]);
            mma16816(acc[2 * n2 + 1], a[kk], b[2], b[3]);
        }
}

// acc[D/8 n-tiles] += P(16 x 8 NT, given as accumulator fragments) * tile(8 NT x D) (B
// operand stored with k as rows: transposed ldmatrix). Pass tile + r0 for rows [r0, r0 + 8 NT).
template <int D, int LD, int NT = kTile / 8>
__device__ __forceinline__ void mma_pb(float (&acc)[D / 8][4], const float (&p)[NT][4], __half (*tile)[LD],
                                       int lane) {
#pragma unroll
    for (int k2 = 0; k2 < NT / 2; ++k2) {
        uint32_t a[4];
        a[0] = pack_half2(p[2 * k2][0], p[2 * k2][1]);
        a[1] = pack_half2(p[2 * k2][2], p[2 * k2][3]);
        a[2] = pack_half2(p[2 * k2 + 1][0], p[2 * k2 + 1][1]);
        a[3] = pack_half2(p[2 * k2 + 1][2], p[2 * k2 + 1][3]);
#pragma unroll
        for (int n2 = 0; n2 < D / 16; ++n2) {
            uint32_t b[4];
            ldsm_x4_t(b, &tile[k2 * 16 + (lane & 7) + ((lane >> 3) & 1) * 8][n2 * 16 + (lane >> 4) * 8]);
            mma16816(acc[2 * n2], a, b[0], b[1]);
            mma16816(acc[2 * n2 + 1], a, b[2], b[3]);
        }
    }
}

}  // namespace fa

// Forward. q, k, v, out: fp16 [B*S][H*D]; lse2 fp32 [B*S][H] = log2-sum-exp of the scaled
// scores (base 2). grid (H, B, ceil(S/64)), block 128 (4 warps x 16 query rows); K/V tiles
// stream through a two-deep cp.async ring. Dynamic shared memory: flash_fwd_smem<D>() bytes
// (87 KB at D = 128).
template <int D> constexpr int flash_fwd_smem() { return 5 * fa::kTile * (D + 8) * 2; }
template <int D>
__global__ void __launch_bounds__(128) flash_fwd_mma_kernel(const __half* __restrict__ q, const __half* __restrict__ k,
                                                            const __half* __restrict__ v, int S, int H, float scale,
                                                            __half* __restrict__ out, float* __restrict__ lse2) {
    MM_PDL_ENTRY();
    using namespace fa;
    constexpr int LD = D + 8;
    extern __shared__ __align__(16) unsigned char fa_smem[];
    auto tiles = reinterpret_cast<__half (*)[kTile][LD]>(fa_smem);
    __half (*Qs)[LD] = tiles[0];
    __half (*Ks)[kTile][LD] = tiles + 1;  // K/V tile kt in buffer kt & 1
    __half (*Vs)[kTile][LD] = tiles + 3;
    // grid (H, B, query tiles): every head and sequence of the longest rows (most key
    // tiles) is scheduled before any shorter one
    const int qt = gridDim.z - 1 - blockIdx.z;
    const int h = blockIdx.x, b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const long long ld = static_cast<long long>(H) * D;
    const long long base = static_cast<long long>(b) * S;
    const float c = scale * kLog2e;
    load_tile_async<D, LD>(Qs, q + (base + qt * kTile) * ld + h * D, ld, S - qt * kTile);
    load_tile_async<D, LD>(Ks[0], k + base * ld + h * D, ld, S);
    load_tile_async<D, LD>(Vs[0], v + base * ld + h * D, ld, S);
    cp_async_commit();
    uint32_t qa[D / 16][4];
    float o[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const int row0 = qt * kTile + warp * 16 + g, row1 = row0 + 8;
    for (int kt = 0; kt <= qt; ++kt) {
        if (kt < qt) {  // prefetch tile kt + 1 while tile kt is used
            load_tile_async<D, LD>(Ks[(kt + 1) & 1], k + (base + (kt + 1) * kTile) * ld + h * D, ld, S - (kt + 1) * kTile);
            load_tile_async<D, LD>(Vs[(kt + 1) & 1], v + (base + (kt + 1) * kTile) * ld + h * D, ld, S - (kt + 1) * kTile);
        }
        cp_async_commit();
        cp_async_wait<1>();  // all but the newest group: tile kt (and Q) have landed
        __syncthreads();
        if (kt == 0) load_a_frags<D, LD>(qa, Qs, warp * 16, lane);
        __half (*Kt)[LD] = Ks[kt & 1];
        __half (*Vt)[LD] = Vs[kt & 1];
        float s[kTile / 8][4];
#pragma unroll
        for (int i = 0; i < kTile / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
        mma_abt<D, LD>(s, qa, Kt, lane);
        float mx0 = m0, mx1 = m1;
#pragma unroll
        for (int nt = 0; nt < kTile / 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = kt * kTile + nt * 8 + 2 * t + (e & 1);
                const int row = e < 2 ? row0 : row1;
                float x = s[nt][e] * c;
                if (key > row || key >= S) x = -INFINITY;
                s[nt][e] = x;
                if (e < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
            }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float b0 = mx0 == -INFINITY ? 0.f : mx0, b1 = mx1 == -INFINITY ? 0.f : mx1;
        const float corr0 = exp2f(m0 - b0), corr1 = exp2f(m1 - b1);
        m0 = mx0;
        m1 = mx1;
        l0 *= corr0;
        l1 *= corr1;
#pragma unroll
        for (int i = 0; i < D / 8; ++i) {
            o[i][0] *= corr0; o[i][1] *= corr0;
            o[i][2] *= corr1; o[i][3] *= corr1;
        }
#pragma unroll
        for (int nt = 0; nt < kTile / 8; ++nt) {
            s[nt][0] = exp2f(s[nt][0] - b0); s[nt][1] = exp2f(s[nt][1] - b0);
            s[nt][2] = exp2f(s[nt][2] - b1); s[nt][3] = exp2f(s[nt][3] - b1);
            l0 += s[nt][0] + s[nt][1];
            l1 += s[nt][2] + s[nt][3];
        }
        mma_pb<D, LD>(o, s, Vt, lane);
        __syncthreads();  // buffer kt & 1 is refilled by the prefetch issued next iteration
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float inv0 = 1.f / l0, inv1 = 1.f / l1;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
        const int col = h * D + i * 8 + 2 * t;
        if (row0 < S) *reinterpret_cast<__half2*>(out + (base + row0) * ld + col) = __floats2half2_rn(o[i][0] * inv0, o[i][1] * inv0);
        if (row1 < S) *reinterpret_cast<__half2*>(out + (base + row1) * ld + col) = __floats2half2_rn(o[i][2] * inv1, o[i][3] * inv1);
    }
    if (t == 0) {
        if (row0 < S) lse2[(base + row0) * H + h] = m0 + log2f(l0);
        if (row1 < S) lse2[(base + row1) * H + h] = m1 + log2f(l1);
    }
}

// D[t, h] = sum_c dO[t, h, c] * O[t, h, c] over fp16 rows (the softmax-backward row term).
__global__ void attn_rowdot_kernel(const __half* __restrict__ dout, const __half* __restrict__ out, int T, int H,
                                   int DV, float* __restrict__ Dd) {
    MM_PDL_ENTRY();
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= T * H) return;
    const long long o = static_cast<long long>(idx / H) * H * DV + (idx % H) * DV;
    float s = 0.f;
    for (int c = 0; c < DV; ++c) s += __half2float(dout[o + c]) * __half2float(out[o + c]);
    Dd[idx] = s;
}

// dQ for one query tile (4 warps x 16 query rows). dout fp16 [B*S][H*D]. dq16 fp16 [B*S][ld],
// including the softmax scale, with the inverse RoPE of columns [rope_begin, rope_begin +
// rope) of every head applied at the row's position (the backward of the query rotation;
// rope_rows_kernel's arithmetic with the angle negated). grid (H, B, ceil(S/64)), longest rows first; K/V tiles stream
// through a two-deep cp.async ring. Dynamic shared memory: flash_dq_smem<D>() bytes.
template <int D> constexpr int flash_dq_smem() { return 6 * fa::kTile * (D + 8) * 2; }
template <int D>
__global__ void __launch_bounds__(128, D >= 128 ? 1 : 4) flash_bwd_dq_mma_kernel(
    const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
    const __half* __restrict__ dout, const float* __restrict__ lse2, const float* __restrict__ Dd, int S, int H,
    float scale, __half* __restrict__ dq16, long long ld_dq, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, int rope_begin, int rope) {
    MM_PDL_ENTRY();
    using namespace fa;
    constexpr int LD = D + 8;
    extern __shared__ __align__(16) unsigned char fa_smem[];
    auto tiles = reinterpret_cast<__half (*)[kTile][LD]>(fa_smem);  // Q, dO, K[2], V[2]
    __half (*Qs)[LD] = tiles[0];
    __half (*Gs)[LD] = tiles[1];
    const int qt = gridDim.z - 1 - blockIdx.z, h = blockIdx.x, b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const long long ld = static_cast<long long>(H) * D;
    const long long base = static_cast<long long>(b) * S;
    const float c = scale * kLog2e;
    load_tile_async<D, LD>(Qs, q + (base + qt * kTile) * ld + h * D, ld, S - qt * kTile);
    load_tile_async<D, LD>(Gs, dout + (base + qt * kTile) * ld + h * D, ld, S - qt * kTile);
    load_tile_async<D, LD>(tiles[2], k + base * ld + h * D, ld, S);
    load_tile_async<D, LD>(tiles[4], v + base * ld + h * D, ld, S);
    cp_async_commit();
    const int row0 = qt * kTile + warp * 16 + g, row1 = row0 + 8;
    const float L0 = row0 < S ? lse2[(base + row0) * H + h] : 0.f, L1 = row1 < S ? lse2[(base + row1) * H + h] : 0.f;
    const float D0 = row0 < S ? Dd[(base + row0) * H + h] : 0.f, D1 = row1 < S ? Dd[(base + row1) * H + h] : 0.f;
    uint32_t qa[D / 16][4], ga[D / 16][4];
    float acc[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    for (int kt = 0; kt <= qt; ++kt) {
        if (kt < qt) {
            load_tile_async<D, LD>(tiles[2 + ((kt + 1) & 1)], k + (base + (kt + 1) * kTile) * ld + h * D, ld,
                                   S - (kt + 1) * kTile);
            load_tile_async<D, LD>(tiles[4 + ((kt + 1) & 1)], v + (base + (kt + 1) * kTile) * ld + h * D, ld,
                                   S - (kt + 1) * kTile);
        }
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        if (kt == 0) {
            load_a_frags<D, LD>(qa, Qs, warp * 16, lane);
            load_a_frags<D, LD>(ga, Gs, warp * 16, lane);
        }
        __half (*Ks)[LD] = tiles[2 + (kt & 1)];
        __half (*Vs)[LD] = tiles[4 + (kt & 1)];
        // the 64 keys of the tile in two halves of 32 (half the live fragments)
#pragma unroll
        for (int hk = 0; hk < 2; ++hk) {
            constexpr int NT = kTile / 16;
            float s[NT][4], dp[NT][4];
#pragma unroll
            for (int i = 0; i < NT; ++i) {
                s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
                dp[i][0] = dp[i][1] = dp[i][2] = dp[i][3] = 0.f;
            }
            mma_abt<D, LD, NT>(s, qa, Ks + hk * 32, lane);
            mma_abt<D, LD, NT>(dp, ga, Vs + hk * 32, lane);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int key = kt * kTile + hk * 32 + nt * 8 + 2 * t + (e & 1);
                    const int row = e < 2 ? row0 : row1;
                    const float p =
                        (key > row || key >= S || row >= S) ? 0.f : exp2f(s[nt][e] * c - (e < 2 ? L0 : L1));
                    s[nt][e] = p * (dp[nt][e] - (e < 2 ? D0 : D1)) * scale;
                }
            mma_pb<D, LD, NT>(acc, s, Ks + hk * 32, lane);
        }
        __syncthreads();
    }
    const int half_r = rope / 2;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
        const int cc = i * 8 + 2 * t;  // column pair (cc, cc + 1) within the head
        const bool rot = cc >= rope_begin && cc < rope_begin + rope;
        const int pair = (cc - rope_begin) >> 1;
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            const int row = hr ? row1 : row0;
            if (row >= S) continue;
            float a = acc[i][2 * hr], bb = acc[i][2 * hr + 1];
            if (rot) {
                const float cs = cos_t[row * half_r + pair], sn = -sin_t[row * half_r + pair];
                const float x0 = a * cs - bb * sn, x1 = a * sn + bb * cs;
                a = x0;
                bb = x1;
            }
            *reinterpret_cast<__half2*>(dq16 + (base + row) * ld_dq + h * D + cc) = __floats2half2_rn(a, bb);
        }
    }
}

// dK, dV for one key tile (4 warps x 16 keys). dk (fp32) includes the softmax scale; dV
// goes out in fp16 (dv16, row pitch ld_dv), the operand form its products use. grid (H, B,
// ceil(S/64)), key tile = blockIdx.z (the first key tiles meet the most query tiles and
// are scheduled first); Q/dO tiles and their lse/D rows stream through a two-deep cp.async
// ring. Dynamic shared memory: flash_dkdv_smem<D>() bytes.
template <int D> constexpr int flash_dkdv_smem() { return 6 * fa::kTile * (D + 8) * 2 + 4 * fa::kTile * 4; }
template <int D>
__global__ void __launch_bounds__(128, D >= 128 ? 1 : 3) flash_bwd_dkdv_mma_kernel(
    const __half* __restrict__ q, const __half* __restrict__ k, const __half* __restrict__ v,
    const __half* __restrict__ dout, const float* __restrict__ lse2, const float* __restrict__ Dd, int S, int H,
    float scale, float* __restrict__ dk, __half* __restrict__ dv16, long long ld_dv) {
    MM_PDL_ENTRY();
    using namespace fa;
    constexpr int LD = D + 8;
    extern __shared__ __align__(16) unsigned char fa_smem[];
    auto tiles = reinterpret_cast<__half (*)[kTile][LD]>(fa_smem);  // K, V, Q[2], dO[2]
    float (*Ls)[kTile] = reinterpret_cast<float (*)[kTile]>(fa_smem + 6 * kTile * LD * 2);
    float (*Ds)[kTile] = Ls + 2;
    const int kt = blockIdx.z, h = blockIdx.x, b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const long long ld = static_cast<long long>(H) * D;
    const long long base = static_cast<long long>(b) * S;
    const float c = scale * kLog2e;
    const int ntiles = (S + kTile - 1) / kTile;
    // query tile qt (its Q, dO, lse and D rows) into ring slot qt & 1
    auto issue = [&](int qt) {
        const int sl = qt & 1;
        load_tile_async<D, LD>(tiles[2 + sl], q + (base + qt * kTile) * ld + h * D, ld, S - qt * kTile);
        load_tile_async<D, LD>(tiles[4 + sl], dout + (base + qt * kTile) * ld + h * D, ld, S - qt * kTile);
        for (int e = threadIdx.x; e < kTile; e += blockDim.x) {
            const int r = qt * kTile + e;
            const bool ok = r < S;
            cp_async4(&Ls[sl][e], lse2 + (base + (ok ? r : 0)) * H + h, ok);
            cp_async4(&Ds[sl][e], Dd + (base + (ok ? r : 0)) * H + h, ok);
        }
    };
    load_tile_async<D, LD>(tiles[0], k + (base + kt * kTile) * ld + h * D, ld, S - kt * kTile);
    load_tile_async<D, LD>(tiles[1], v + (base + kt * kTile) * ld + h * D, ld, S - kt * kTile);
    issue(kt);
    cp_async_commit();
    uint32_t ka[D / 16][4], va[D / 16][4];
    const int key0 = kt * kTile + warp * 16 + g, key1 = key0 + 8;
    float accK[D / 8][4], accV[D / 8][4];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
        accK[i][0] = accK[i][1] = accK[i][2] = accK[i][3] = 0.f;
        accV[i][0] = accV[i][1] = accV[i][2] = accV[i][3] = 0.f;
    }
    for (int qt = kt; qt < ntiles; ++qt) {
        if (qt + 1 < ntiles) issue(qt + 1);
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        if (qt == kt) {
            load_a_frags<D, LD>(ka, tiles[0], warp * 16, lane);
            load_a_frags<D, LD>(va, tiles[1], warp * 16, lane);
        }
        const int sl = qt & 1;
        __half (*Qs)[LD] = tiles[2 + sl];
        __half (*Gs)[LD] = tiles[4 + sl];
        // the 64 queries of the tile in two halves of 32 (half the live fragments)
#pragma unroll
        for (int hq = 0; hq < 2; ++hq) {
            constexpr int NT = kTile / 16;
            float st[NT][4], dpt[NT][4];
#pragma unroll
            for (int i = 0; i < NT; ++i) {
                st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;
                dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.f;
            }
            mma_abt<D, LD, NT>(st, ka, Qs + hq * 32, lane);   // S^T: keys x queries
            mma_abt<D, LD, NT>(dpt, va, Gs + hq * 32, lane);  // dP^T
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int qi = hq * 32 + nt * 8 + 2 * t + (e & 1);
                    const int query = qt * kTile + qi;
                    const int key = e < 2 ? key0 : key1;
                    const float p = (key > query || query >= S || key >= S) ? 0.f : exp2f(st[nt][e] * c - Ls[sl][qi]);
                    st[nt][e] = p;
                    dpt[nt][e] = p * (dpt[nt][e] - Ds[sl][qi]) * scale;
                }
            mma_pb<D, LD, NT>(accV, st, Gs + hq * 32, lane);   // dV += P^T dO
            mma_pb<D, LD, NT>(accK, dpt, Qs + hq * 32, lane);  // dK += dS^T Q * scale
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
        const int col = h * D + i * 8 + 2 * t;
        if (key0 < S) {
            *reinterpret_cast<float2*>(dk + (base + key0) * ld + col) = make_float2(accK[i][0], accK[i][1]);
            *reinterpret_cast<__half2*>(dv16 + (base + key0) * ld_dv + col) = __floats2half2_rn(accV[i][0], accV[i][1]);
        }
        if (key1 < S) {
            *reinterpret_cast<float2*>(dk + (base + key1) * ld + col) = make_float2(accK[i][2], accK[i][3]);
            *reinterpret_cast<__half2*>(dv16 + (base + key1) * ld_dv + col) = __floats2half2_rn(accV[i][2], accV[i][3]);
        }
    }
}

} // namespace mm
