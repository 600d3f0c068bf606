// tcgen05 + TMA GEMM for sm_100a: D[M,N] = alpha * A[M,K] * B[K,N] (+ residual | += D),
// fp16 or bf16 operands, fp32 accumulation in tensor memory.
//
// Each operand is either K-major (rows of the tile contiguous along K) or MN-major
// (contiguous along M or N), both loaded by TMA with 128-byte swizzling:
//   A K-major : global [M][K], box {64 K, 128 M}      -> 128 rows x 128 B
//   A MN-major: global [K][M], 2 boxes {64 M, 64 K}    -> two 8 KB chunks (LBO 8192 B)
//   B K-major : global [N][K], box {64 K, BN N}
//   B MN-major: global [K][N], BN/64 boxes {64 N, 64 K}
// so x*W (W stored [in][out]) is "B MN-major", dY*W^T is "B K-major" and X^T*dY is
// "A and B MN-major": no transposed copies of weights or activations are ever made.
//
// One output tile (128 x BN) per CTA, 6 warps: warp 0 issues TMA (one elected thread),
// warp 1 issues tcgen05.mma (one thread) and commits each stage back to the producer,
// warps 2-5 drain tensor memory (lane quarter = warp % 4) and store. Every mbarrier
// wait is bounded; a timeout sets the device error word and the CTA unwinds, freeing its
// tensor memory.
#pragma once
#include "common.cuh"

namespace mm {

enum GemmOut : int { kOutF32 = 0, kOutF32Acc = 1, kOutF16 = 2, kOutBF16 = 3 };

struct GemmArgs {
    int M, N, K;
    int a_mn, b_mn, bf16;
    void* out;
    long long ldc;
    int out_kind;
    const float* residual; // optional, fp32 [M][ldr], added in the kOutF32 epilogue
    long long ldr;
    float alpha;
    const float* alpha_ptr; // optional device scalar multiplied into alpha
    int* err;
    int k_tiles_per_split;   // split-K: CTA z covers k-tiles [z*per, (z+1)*per); 0 = all
    long long split_stride;  // split-K: output of CTA z starts at out + z * split_stride
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;

template <int BN, int STAGES> struct GemmCfg {
    static constexpr int A_BYTES = kGemmBM * 128;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
};

__device__ __forceinline__ void gemm_store16(const GemmArgs& g, float alpha, int row, int col0,
                                             const float (&v)[16]) {
    const bool full = col0 + 16 <= g.N;
    if (g.out_kind == kOutF32 || g.out_kind == kOutF32Acc) {
        float* o = static_cast<float*>(g.out) + static_cast<long long>(row) * g.ldc + col0;
        const float* r = g.residual ? g.residual + static_cast<long long>(row) * g.ldr + col0 : nullptr;
        const bool vec = full && (g.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(o) & 15) == 0) &&
                         (!r || ((g.ldr % 4 == 0) && ((reinterpret_cast<uintptr_t>(r) & 15) == 0)));
        if (vec) {
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
                float4 x = make_float4(alpha * v[i], alpha * v[i + 1], alpha * v[i + 2],
                                       alpha * v[i + 3]);
                if (g.out_kind == kOutF32Acc) {
                    float4 y = *reinterpret_cast<const float4*>(o + i);
                    x.x += y.x; x.y += y.y; x.z += y.z; x.w += y.w;
                } else if (r) {
                    float4 y = *reinterpret_cast<const float4*>(r + i);
                    x.x += y.x; x.y += y.y; x.z += y.z; x.w += y.w;
                }
                *reinterpret_cast<float4*>(o + i) = x;
            }
        } else {
            for (int i = 0; i < 16 && col0 + i < g.N; ++i) {
                float x = alpha * v[i];
                if (g.out_kind == kOutF32Acc) x += o[i];
                else if (r) x += r[i];
                o[i] = x;
            }
        }
    } else {
        // 16-bit outputs.
        uint16_t* o = static_cast<uint16_t*>(g.out) + static_cast<long long>(row) * g.ldc + col0;
        uint16_t h[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            float x = alpha * v[i];
            h[i] = g.out_kind == kOutF16 ? __half_as_ushort(__float2half_rn(x))
                                         : __bfloat16_as_ushort(__float2bfloat16_rn(x));
        }
        const bool vec = full && (g.ldc % 8 == 0) && ((reinterpret_cast<uintptr_t>(o) & 15) == 0);
        if (vec) {
            *reinterpret_cast<uint4*>(o) = *reinterpret_cast<const uint4*>(h);
            *reinterpret_cast<uint4*>(o + 8) = *reinterpret_cast<const uint4*>(h + 8);
        } else {
            for (int i = 0; i < 16 && col0 + i < g.N; ++i) o[i] = h[i];
        }
    }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Persistent: CTA c processes tiles c, c + gridDim.x, ... of the (m, n, split) tile list,
// n fastest (consecutive CTAs share the A row tile in L2). The shared-memory ring of
// STAGES (A, B) stages runs across tile boundaries; two TMEM accumulators of BN columns
// alternate, so the epilogue of tile j overlaps the MMAs of tile j + 1.
template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   GemmArgs g) {
    using C = GemmCfg<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;  // [2] MMA -> epilogue
    uint64_t* acc_empty = acc_full + 2;   // [2] epilogue -> MMA (4 warp arrivals)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_k = (g.K + kGemmBK - 1) / kGemmBK;
    const int per = g.k_tiles_per_split > 0 ? g.k_tiles_per_split : num_k;
    const int splits = (num_k + per - 1) / per;
    const int tiles_n = (g.N + BN - 1) / BN, tiles_m = (g.M + kGemmBM - 1) / kGemmBM;
    const int tiles = tiles_n * tiles_m * splits;

    if (warp == 0) {
        if (lane == 0) {
            for (int s = 0; s < STAGES; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            mbar_init(&acc_full[0], 1);
            mbar_init(&acc_full[1], 1);
            mbar_init(&acc_empty[0], 4);
            mbar_init(&acc_empty[1], 4);
            fence_mbar_init();
            prefetch_tmap(&tmA);
            prefetch_tmap(&tmB);
        }
        __syncwarp();
        tmem_alloc(tmem_slot, 2 * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        int it = 0;  // ring position across tiles
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
            const int z = tile / (tiles_n * tiles_m), mn = tile % (tiles_n * tiles_m);
            const int m0 = (mn / tiles_n) * kGemmBM, n0 = (mn % tiles_n) * BN;
            const int kb = z * per, ke = min(num_k, kb + per);
            for (int kt = kb; kt < ke; ++kt, ++it) {
                const int s = it % STAGES;
                const uint32_t ph = (it / STAGES) & 1;
                if (!mbar_wait_bounded(&empty[s], ph ^ 1, g.err)) { ok = false; break; }
                uint8_t* sa = smem + s * C::STAGE_BYTES;
                uint8_t* sb = sa + C::A_BYTES;
                mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
                const int k0 = kt * kGemmBK;
                if (!g.a_mn) {
                    tma_load_2d(sa, &tmA, &full[s], k0, m0);
                } else {
                    tma_load_2d(sa, &tmA, &full[s], m0, k0);
                    tma_load_2d(sa + 8192, &tmA, &full[s], m0 + 64, k0);
                }
                if (!g.b_mn) {
                    tma_load_2d(sb, &tmB, &full[s], k0, n0);
                } else {
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j)
                        tma_load_2d(sb + j * 8192, &tmB, &full[s], n0 + 64 * j, k0);
                }
            }
        }
    } else if (warp == 1 && lane == 0) {
        int it = 0, j = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++j) {
            const int z = tile / (tiles_n * tiles_m), mn = tile % (tiles_n * tiles_m);
            const int n0 = (mn % tiles_n) * BN;
            const int kb = z * per, ke = min(num_k, kb + per);
            const int n_mma = min(BN, ((g.N - n0) + 15) / 16 * 16);
            const uint32_t idesc = umma_idesc_f16(g.bf16 != 0, g.a_mn != 0, g.b_mn != 0, kGemmBM, n_mma);
            const int buf = j & 1;
            if (!mbar_wait_bounded(&acc_empty[buf], ((j >> 1) & 1) ^ 1, g.err)) break;
            tc_fence_after();
            const uint32_t dst = tmem + static_cast<uint32_t>(buf * BN);
            for (int kt = kb; kt < ke; ++kt, ++it) {
                const int s = it % STAGES;
                const uint32_t ph = (it / STAGES) & 1;
                if (!mbar_wait_bounded(&full[s], ph, g.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
                const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
                for (int k = 0; k < kGemmBK / 16; ++k) {
                    const uint64_t ad = g.a_mn ? umma_desc_sw128(sa + k * 2048, 8192, 1024)
                                               : umma_desc_sw128(sa + k * 32, 16, 1024);
                    const uint64_t bd = g.b_mn ? umma_desc_sw128(sb + k * 2048, 8192, 1024)
                                               : umma_desc_sw128(sb + k * 32, 16, 1024);
                    tc_mma_f16(dst, ad, bd, idesc, (kt != kb || k != 0) ? 1u : 0u);
                }
                tc_commit(&empty[s]);
            }
            tc_commit(&acc_full[buf]);
        }
    } else if (warp >= 2) {
        const int q = warp & 3;
        const float alpha = g.alpha * (g.alpha_ptr ? *g.alpha_ptr : 1.0f);
        int j = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++j) {
            const int z = tile / (tiles_n * tiles_m), mn = tile % (tiles_n * tiles_m);
            const int m0 = (mn / tiles_n) * kGemmBM, n0 = (mn % tiles_n) * BN;
            const int n_mma = min(BN, ((g.N - n0) + 15) / 16 * 16);
            const int buf = j & 1;
            if (!mbar_wait_bounded(&acc_full[buf], (j >> 1) & 1, g.err)) break;
            tc_fence_after();
            GemmArgs gz = g;
            if (g.k_tiles_per_split > 0)
                gz.out = static_cast<char*>(g.out) +
                         z * g.split_stride * (g.out_kind >= kOutF16 ? 2 : 4);
            const int row = m0 + q * 32 + lane;
            const uint32_t src = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN);
            // Drain the whole accumulator into registers in 16-column pieces, store each.
            for (int c = 0; c < n_mma; c += 16) {
                float v[16];
                tmem_ld16(src + static_cast<uint32_t>(c), v);
                if (c + 16 >= n_mma) {
                    // last read of this buffer: hand it back to the MMA warp before storing
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty[buf]);
                }
                if (row < g.M && n0 + c < g.N) gemm_store16(gz, alpha, row, n0 + c, v);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * BN);
    }
}

} // namespace mm
