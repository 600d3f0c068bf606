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
// Persistent: CTA c processes tiles c, c + gridDim.x, ... of the (m, n, k-split) tile
// list, n fastest (consecutive CTAs share the A row tile in L2). 6 warps: warp 0 issues
// TMA into a ring of STAGES (A, B) stages that runs across tile boundaries; warp 1 issues
// tcgen05.mma (one thread) into one of two TMEM accumulators of BN columns, so the
// epilogue of tile j overlaps the MMAs of tile j + 1; warps 2-5 drain tensor memory
// (lane quarter = warp % 4) 128 bytes per row at a time into a 128-byte-swizzled shared
// staging tile and hand it to a TMA bulk tensor store (fp32 += uses the TMA reduce-add),
// which also clips the ragged edges. Every mbarrier wait is bounded; a timeout sets the
// device error word and the CTA unwinds, freeing its tensor memory.
#pragma once
#include "common.cuh"

namespace mm {

enum GemmOut : int { kOutF32 = 0, kOutF32Acc = 1, kOutF16 = 2, kOutBF16 = 3 };

struct GemmArgs {
    int M, N, K;
    int a_mn, b_mn, bf16;
    int out_kind;
    const float* residual; // optional, fp32 [M][ldr], added in the kOutF32 epilogue
    long long ldr;
    float alpha;
    const float* alpha_ptr; // optional device scalar multiplied into alpha
    int* err;
    int k_tiles_per_split;  // split-K: tiles of split z cover k-tiles [z*per, (z+1)*per); 0 = all
    int split_rows;         // split-K: rows of the output map per split (M rounded up to 128)
    // Row log-sum-exp partials (the vocabulary head, fp32 output, no split): per output
    // tile, epilogue half (0/1) and row, (max, sum exp(x - max)) over the columns that half
    // drains into lse_part[(n_tile * 2 + half) * M + row] (max -inf, sum 0 when it drains
    // none), and the value in column targets[row] into tgt_logit[row] (written by the one
    // warp holding that column). no_store skips the output itself.
    float2* lse_part;
    const uint16_t* targets;
    float* tgt_logit;
    int no_store;
    // SwiGLU output (B MN-major, fp16 out): B holds [gate | up] with the up half starting
    // glu_n columns after the gate half; a BN-wide tile multiplies gate columns
    // [n0, n0 + BN/2) and the matching up columns into one accumulator and stores
    // gate * sigmoid(gate) * up for output columns [n0, n0 + BN/2). 0 = off.
    int glu_n;
    // Adjacent-pair RoPE on an fp16 output: within every rope_period columns, pairs in
    // [rope_begin, rope_begin + rope_len) are rotated to position row % rope_seq with the
    // tables rope_cos/rope_sin [positions][rope_len / 2]. Null = off.
    const float* rope_cos;
    const float* rope_sin;
    int rope_seq, rope_period, rope_begin, rope_len;
    // With glu_n: also store the fp16 pre-activations, gate columns through the map tmD and
    // up columns through tmE (the training forward keeps them for the backward).
    int glu_pre;
    // SwiGLU backward in the epilogue of dH (fp16 out, dglu_n = N = d_ff): with gate and up
    // read from dglu_gu (row pitch dglu_ld, up at column offset dglu_n), stores d gate
    // through tmC and d up through tmD. 0 = off.
    const __half* dglu_gu;
    long long dglu_ld;
    int dglu_n;
    // B K-row wrap (MN-major B only): A's k-block at k reads B rows k % b_k_wrap, so
    // A = [hi | lo] over K = 2 b_k_wrap against the same weights gives the two-term product;
    // with b_k3, B holds [W_hi; W_lo] (2 b_k_wrap rows) and k in [2 w, 3 w) reads rows k - w,
    // so A = [hi | lo | hi] gives hi.W_hi + lo.W_hi + hi.W_lo. 0 = off.
    int b_k_wrap;
    int b_k3;
    // Weighted-NLL gradient of recomputed logits (the vocabulary backward, fp16 output): the
    // product's value v (after alpha) of row r, column c becomes
    // vg_coef[r] * vg_scale[0] * (exp(v - vg_lse[r]) - (c == targets[r])). Null = off.
    const float* vg_lse;
    const float* vg_coef;
    const float* vg_scale;
};

__device__ __forceinline__ int gemm_b_row(const GemmArgs& g, int k0) {
    if (!g.b_k_wrap) return k0;
    if (g.b_k3 && k0 >= 2 * g.b_k_wrap) return k0 - g.b_k_wrap;
    return k0 % g.b_k_wrap;
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// 64 fp16 values (32 packed words) of one staged 128-byte row, 128-byte swizzled.
__device__ __forceinline__ void stage_row_words(uint8_t* rowp, int lane, const uint32_t (&w)[32]) {
#pragma unroll
    for (int cc = 0; cc < 8; ++cc)
        *reinterpret_cast<uint4*>(rowp + ((cc ^ (lane & 7)) << 4)) =
            make_uint4(w[4 * cc], w[4 * cc + 1], w[4 * cc + 2], w[4 * cc + 3]);
}

// One 32-row x 64-column fp16 tile from a warp's staging buffer to global through `map`,
// after the previous store from that buffer has finished reading it.
__device__ __forceinline__ void stage_and_store(uint8_t* stage, int lane, const uint32_t (&w)[32],
                                                const CUtensorMap* map, int x, int y) {
    if (lane == 0) bulk_wait_read0();
    __syncwarp();
    stage_row_words(stage + lane * 128, lane, w);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(map, stage, x, y);
        bulk_commit();
    }
}

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
// Epilogue warps: two per TMEM lane quadrant for the 256-wide tile (one CTA per SM; they
// take alternate column chunks, so a short-K product's epilogue keeps up with its MMAs),
// one per quadrant for the narrower tiles (two CTAs per SM). Each owns one 32-row x
// 128-byte staging tile.
template <int BN> constexpr int epi_warps() { return BN == 256 ? 8 : 4; }

template <int BN, int STAGES> struct GemmCfg {
    static constexpr int A_BYTES = kGemmBM * 128;
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int EPI_WARPS = epi_warps<BN>();
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int EPI_BYTES = EPI_WARPS * 4096;
    static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 256;
};

// Drains one finished accumulator tile (tensor memory columns from `src`, which already
// points at this warp's lane quadrant q) into global memory: the warp takes column chunks
// half, half + nhalf, ... of CH columns. Right after its last read of the accumulator the
// warp arrives on the mbarrier at shared::cluster address `release_bar` (the MMA issuer's
// "accumulator free" barrier, possibly in the peer CTA).
__device__ __forceinline__ void gemm_release_acc(uint32_t release_bar, int lane) {
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(release_bar);
}
// Epilogue families, one kernel instantiation each, so the common products carry none of
// the SwiGLU paths' registers: kEpiPlain (store / accumulate / residual / log-sum-exp
// partials / RoPE), kEpiGlu (SwiGLU, optionally with the pre-activations), kEpiDglu (SwiGLU
// backward of dH).
enum GemmEpi : int { kEpiPlain = 0, kEpiGlu = 1, kEpiDglu = 2 };

template <int BN, int EPI_WARPS, int EPI>
__device__ __forceinline__ void gemm_drain_tile(const GemmArgs g, const CUtensorMap& tmC, const CUtensorMap& tmD,
                                                const CUtensorMap& tmE, uint8_t* stage_base, uint32_t src, int m0,
                                                int n0, int map_row0, int q, int half, int lane, float alpha,
                                                uint32_t release_bar) {
    constexpr int nhalf = EPI_WARPS / 4;  // warps per quadrant
    const bool half_out = g.out_kind >= kOutF16;
    const int CH = half_out ? 64 : 32;  // columns per 128-byte staged row
    const int TW = EPI == kEpiGlu ? BN / 2 : BN;
    const int n_mma = min(BN, ((g.N - n0) + 15) / 16 * 16);
    const int row0 = m0 + q * 32;
    const int row = row0 + lane;
    if constexpr (EPI == kEpiGlu) {
        // accumulator columns [0, TW) gate, [TW, 2 TW) up; 64 fp16 outputs per staged row
        if (half * 64 >= TW) {  // no chunk for this warp: release the accumulator
            gemm_release_acc(release_bar, lane);
        }
        for (int c = half * 64; c < TW; c += 64 * nhalf) {
            if (g.glu_pre) {
                // the fp16 pre-activations first: gate columns, then up columns, each
                // read from tensor memory into the warp's staging tile
#pragma unroll 1
                for (int part = 0; part < 2; ++part) {
                    if (lane == 0) bulk_wait_read0();
                    __syncwarp();
                    uint8_t* rowp = stage_base + lane * 128;
#pragma unroll
                    for (int sub = 0; sub < 2; ++sub) {
                        float t[32];
                        tmem_ld32_nowait(src + static_cast<uint32_t>(part * TW + c + 32 * sub), t);
                        tmem_wait_ld();
#pragma unroll
                        for (int ch = 0; ch < 4; ++ch) {
                            const float* f = t + 8 * ch;
                            const int cc = sub * 4 + ch;
                            *reinterpret_cast<uint4*>(rowp + ((cc ^ (lane & 7)) << 4)) =
                                make_uint4(pack_half2(f[0] * alpha, f[1] * alpha), pack_half2(f[2] * alpha, f[3] * alpha),
                                           pack_half2(f[4] * alpha, f[5] * alpha), pack_half2(f[6] * alpha, f[7] * alpha));
                        }
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(part ? &tmE : &tmD, stage_base, n0 + c, map_row0);
                        bulk_commit();
                    }
                }
            }
            uint8_t* stage = stage_base;
            if (lane == 0) bulk_wait_read0();  // the store that last read `stage` is done
            __syncwarp();
            uint8_t* rowp = stage + lane * 128;
#pragma unroll
            for (int sub = 0; sub < 2; ++sub) {
                float gv[32], uv[32];
                tmem_ld32_nowait(src + static_cast<uint32_t>(c + 32 * sub), gv);
                tmem_ld32_nowait(src + static_cast<uint32_t>(TW + c + 32 * sub), uv);
                tmem_wait_ld();
                if (sub == 1 && c + 64 * nhalf >= TW) {
                    gemm_release_acc(release_bar, lane);
                }
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int i = ch * 8 + 2 * e;
                        // g * sigmoid(g) = g / (1 + e^-g), branch-free on the SFU
                        // (the result is rounded to fp16)
                        const float ga = gv[i] * alpha, gb = gv[i + 1] * alpha;
                        const float a = __fdividef(ga, 1.f + __expf(-ga)) * (uv[i] * alpha);
                        const float b = __fdividef(gb, 1.f + __expf(-gb)) * (uv[i + 1] * alpha);
                        w[e] = pack_half2(a, b);
                    }
                    const int cc = sub * 4 + ch;
                    *reinterpret_cast<uint4*>(rowp + ((cc ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(&tmC, stage, n0 + c, map_row0);
                bulk_commit();
            }
        }
        return;
    }
    // online (max, sum of exp) over this tile's columns of the row, and its target
    float run_m = -INFINITY, run_s = 0.f, run_t = 0.f;
    const int tg = (g.lse_part && row < g.M) ? static_cast<int>(g.targets[row]) : -1;
    if (half * CH >= n_mma) {  // no chunk for this warp: release the accumulator
        gemm_release_acc(release_bar, lane);
    }
    for (int c = half * CH; c < n_mma; c += CH * nhalf) {
        if constexpr (EPI == kEpiDglu) {
            // SwiGLU backward of dH columns [col0, col0 + 64) of this row, 32 at a time from
            // tensor memory; x = gate, u = up from the forward: d gate = dh u s (1 + x (1 - s)),
            // d up = dh x s, s = sigmoid(x). d gate goes straight into the staging tile, d up
            // waits packed until that tile is stored.
            const int col0 = n0 + c;
            const __half* gr = g.dglu_gu + static_cast<long long>(row < g.M ? row : 0) * g.dglu_ld;
            uint32_t du[32];
            if (lane == 0) bulk_wait_read0();
            __syncwarp();
            uint8_t* rowp = stage_base + lane * 128;
            if (row < g.M && col0 < g.N) {
                // this row's 64 gate and 64 up values (128 B each, at most two lines apiece),
                // requested before anything waits on them; addresses inside the row only
                prefetch_l1(gr + col0);
                prefetch_l1(gr + g.dglu_n + col0);
                if (col0 + 32 < g.N) {
                    prefetch_l1(gr + col0 + 32);
                    prefetch_l1(gr + g.dglu_n + col0 + 32);
                }
            }
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                float t[32];
                tmem_ld32_nowait(src + static_cast<uint32_t>(c + 32 * hf), t);
                tmem_wait_ld();
                if (hf == 1 && c + CH * nhalf >= n_mma) gemm_release_acc(release_bar, lane);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    // 8 columns at a time (L1 hits after the prefetch above); the barrier keeps
                    // the next group's loads behind this group's math (registers)
                    asm volatile("" ::: "memory");
                    const int col = col0 + 32 * hf + 8 * j;
                    const bool in = row < g.M && col < g.N;  // N % 8 == 0
                    const uint4 xq = in ? *reinterpret_cast<const uint4*>(gr + col) : make_uint4(0, 0, 0, 0);
                    const uint4 uq = in ? *reinterpret_cast<const uint4*>(gr + g.dglu_n + col) : make_uint4(0, 0, 0, 0);
                    const uint32_t xw[4] = {xq.x, xq.y, xq.z, xq.w};
                    const uint32_t uw[4] = {uq.x, uq.y, uq.z, uq.w};
                    uint32_t da[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float x0 = __half2float(__ushort_as_half(static_cast<unsigned short>(xw[e] & 0xFFFFu)));
                        const float x1 = __half2float(__ushort_as_half(static_cast<unsigned short>(xw[e] >> 16)));
                        const float u0 = __half2float(__ushort_as_half(static_cast<unsigned short>(uw[e] & 0xFFFFu)));
                        const float u1 = __half2float(__ushort_as_half(static_cast<unsigned short>(uw[e] >> 16)));
                        const float d0 = t[8 * j + 2 * e] * alpha, d1 = t[8 * j + 2 * e + 1] * alpha;
                        // sigmoid on the SFU (the results are rounded to fp16)
                        const float s0 = __fdividef(1.f, 1.f + __expf(-x0));
                        const float s1 = __fdividef(1.f, 1.f + __expf(-x1));
                        da[e] = pack_half2(d0 * u0 * (s0 + x0 * s0 * (1.f - s0)), d1 * u1 * (s1 + x1 * s1 * (1.f - s1)));
                        du[16 * hf + 4 * j + e] = pack_half2(d0 * x0 * s0, d1 * x1 * s1);
                    }
                    const int cc = 4 * hf + j;
                    *reinterpret_cast<uint4*>(rowp + ((cc ^ (lane & 7)) << 4)) = make_uint4(da[0], da[1], da[2], da[3]);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(&tmC, stage_base, col0, map_row0);
                bulk_commit();
            }
            stage_and_store(stage_base, lane, du, &tmD, col0, map_row0);
            continue;
        }
        float v[64];
        tmem_ld32_nowait(src + static_cast<uint32_t>(c), v);
        if (half_out) tmem_ld32_nowait(src + static_cast<uint32_t>(c + 32), v + 32);
        tmem_wait_ld();
        if (c + CH * nhalf >= n_mma) {
            // last read of this accumulator: hand it back to the MMA warp first
            gemm_release_acc(release_bar, lane);
        }
        const int col0 = n0 + c;
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] *= alpha;
        if (g.residual && row < g.M) {
            const float* r = g.residual + static_cast<long long>(row) * g.ldr + col0;
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (col0 + i < g.N) v[i] += r[i];
        }
        if (g.vg_lse && row < g.M) {
            // coef * (softmax - onehot) of this row's recomputed logits (vocab_grad's arithmetic)
            const float L = g.vg_lse[row], cf = g.vg_coef[row] * *g.vg_scale;
            const int rel = static_cast<int>(g.targets[row]) - col0;
#pragma unroll
            for (int i = 0; i < 64; ++i) v[i] = cf * (__expf(v[i] - L) - (i == rel ? 1.f : 0.f));
        }
        if (g.lse_part) {  // fp32 output: 32 columns per chunk
            float cm = -INFINITY;
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (col0 + i < g.N) cm = fmaxf(cm, v[i]);
            const float nm = fmaxf(run_m, cm);  // finite: every chunk holds a column < N
            float add = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (col0 + i < g.N) add += __expf(v[i] - nm);
            run_s = (run_m == -INFINITY ? 0.f : run_s * __expf(run_m - nm)) + add;
            run_m = nm;
            const int rel = tg - col0;
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (rel == i) run_t = v[i];
            if (g.no_store) continue;
        }
        // the store issued last (from this staging tile) has finished reading it
        uint8_t* stage = stage_base;
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
        uint8_t* rowp = stage + lane * 128;
        if (half_out && g.rope_cos && row < g.M) {
            const int p = row % g.rope_seq, hr = g.rope_len >> 1;
#pragma unroll
            for (int i = 0; i < 64; i += 2) {
                const int cc = (col0 + i) % g.rope_period - g.rope_begin;
                if (cc >= 0 && cc < g.rope_len) {
                    const float cs = g.rope_cos[p * hr + (cc >> 1)], sn = g.rope_sin[p * hr + (cc >> 1)];
                    const float a = v[i], bb = v[i + 1];
                    v[i] = a * cs - bb * sn;
                    v[i + 1] = a * sn + bb * cs;
                }
            }
        }
        if (half_out) {
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float a = v[ch * 8 + 2 * e], b = v[ch * 8 + 2 * e + 1];
                    if (g.out_kind == kOutF16) {
                        const __half2 h = __floats2half2_rn(a, b);
                        w[e] = *reinterpret_cast<const uint32_t*>(&h);
                    } else {
                        const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
                        w[e] = *reinterpret_cast<const uint32_t*>(&h);
                    }
                }
                *reinterpret_cast<uint4*>(rowp + ((ch ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        } else {
#pragma unroll
            for (int ch = 0; ch < 8; ++ch)
                *reinterpret_cast<float4*>(rowp + ((ch ^ (lane & 7)) << 4)) =
                    make_float4(v[4 * ch], v[4 * ch + 1], v[4 * ch + 2], v[4 * ch + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            if (g.out_kind == kOutF32Acc) tma_reduce_add_2d(&tmC, stage, col0, map_row0);
            else tma_store_2d(&tmC, stage, col0, map_row0);
            bulk_commit();
        }
    }
    if (g.lse_part && row < g.M) {
        // one partial per tile and quadrant warp: [n_tile * 2 + half][row]
        g.lse_part[static_cast<long long>((n0 / BN) * 2 + half) * g.M + row] = make_float2(run_m, run_s);
        if (nhalf == 1)  // one warp per quadrant: the second slot holds nothing
            g.lse_part[static_cast<long long>((n0 / BN) * 2 + 1) * g.M + row] = make_float2(-INFINITY, 0.f);
        const int rel = tg - n0;  // the warp whose chunks hold the target column writes it
        if (rel >= 0 && rel < n_mma && ((rel / CH) % nhalf) == half) g.tgt_logit[row] = run_t;
    }
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(320, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                   const __grid_constant__ CUtensorMap tmE, GemmArgs g) {
    using C = GemmCfg<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* epi = smem + STAGES * C::STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(epi + C::EPI_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;  // [2] MMA -> epilogue
    uint64_t* acc_empty = acc_full + 2;   // [2] epilogue -> MMA (4 warp arrivals)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_k = (g.K + kGemmBK - 1) / kGemmBK;
    const int per = g.k_tiles_per_split > 0 ? g.k_tiles_per_split : num_k;
    const int splits = (num_k + per - 1) / per;
    const int TW = EPI == kEpiGlu ? BN / 2 : BN;  // output columns per tile
    const int tiles_n = (g.N + TW - 1) / TW, tiles_m = (g.M + kGemmBM - 1) / kGemmBM;
    const int tiles = tiles_n * tiles_m * splits;

    if (warp == 0) {
        if (lane == 0) {
            for (int s = 0; s < STAGES; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            mbar_init(&acc_full[0], 1);
            mbar_init(&acc_full[1], 1);
            mbar_init(&acc_empty[0], C::EPI_WARPS);
            mbar_init(&acc_empty[1], C::EPI_WARPS);
            fence_mbar_init();
            prefetch_tmap(&tmA);
            prefetch_tmap(&tmB);
            prefetch_tmap(&tmC);
        }
        __syncwarp();
        tmem_alloc(tmem_slot, 2 * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // barriers, tensor memory and descriptor prefetch overlap the predecessor's tail
    MM_PDL_ENTRY();

    if (warp == 0 && lane == 0) {
        int it = 0;  // ring position across tiles
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
            const int z = tile / (tiles_n * tiles_m), mn = tile % (tiles_n * tiles_m);
            const int m0 = (mn / tiles_n) * kGemmBM, n0 = (mn % tiles_n) * TW;
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
                    const int kB = gemm_b_row(g, k0);
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j) {
                        const int col = EPI != kEpiGlu ? n0 + 64 * j
                                                 : (j < BN / 128 ? n0 + 64 * j : g.glu_n + n0 + 64 * (j - BN / 128));
                        tma_load_2d(sb + j * 8192, &tmB, &full[s], col, kB);
                    }
                }
            }
        }
    } else if (warp == 1 && lane == 0) {
        int it = 0, j = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++j) {
            const int z = tile / (tiles_n * tiles_m), mn = tile % (tiles_n * tiles_m);
            const int n0 = (mn % tiles_n) * TW;
            const int kb = z * per, ke = min(num_k, kb + per);
            const int n_mma = EPI == kEpiGlu ? BN : min(BN, ((g.N - n0) + 15) / 16 * 16);
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
        const int q = warp & 3;            // TMEM lane quadrant of this warp
        const int half = (warp - 2) >> 2;  // which of the quadrant's warps (0 or 1)
        uint8_t* stage_base = epi + (warp - 2) * 4096;
        const float alpha = g.alpha * (g.alpha_ptr ? *g.alpha_ptr : 1.0f);
        int j = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++j) {
            const int z = tile / (tiles_n * tiles_m), mn = tile % (tiles_n * tiles_m);
            const int m0 = (mn / tiles_n) * kGemmBM, n0 = (mn % tiles_n) * TW;
            const int buf = j & 1;
            if (!mbar_wait_bounded(&acc_full[buf], (j >> 1) & 1, g.err)) break;
            tc_fence_after();
            const int map_row0 = m0 + q * 32 + (g.k_tiles_per_split > 0 ? z * g.split_rows : 0);
            const uint32_t src = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN);
            gemm_drain_tile<BN, C::EPI_WARPS, EPI>(g, tmC, tmD, tmE, stage_base, src, m0, n0, map_row0, q, half, lane,
                                              alpha, smem_u32(&acc_empty[buf]));
        }
        if (lane == 0) bulk_wait0();
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * BN);
    }
}

// ------------------------------------------------------------------ CTA-pair variant
// The same product on pairs of CTAs (clusters of 2, tcgen05 cta_group::2) for the large
// 256-wide-tile products: a pair computes a 256-row x 256-column accumulator (TW output
// columns). CTA r of the pair loads rows [m0 + 128 r, +128) of A and 128 of the tile's B
// columns (columns [n0 + 128 r, +128); with SwiGLU the gate columns in CTA 0 and the up
// columns in CTA 1) into its own shared memory; the leader (rank 0) issues one M = 256,
// N = 256 MMA per 16-deep K step over both CTAs' operands, and each CTA's tensor memory holds
// its own 128 rows x 256 columns, which its epilogue warps drain exactly as in the
// single-CTA kernel. Per SM a 64-deep K step moves 32 KB for 128 x 256 outputs (48 KB with
// one CTA), so a 6-stage ring fits and hides 1.5x the load latency at the same MMA rate.
// Barriers: full[s] (leader: its producer expects both CTAs' bytes, both CTAs' loads count
// on it), empty[s] and acc_full[b] (every CTA: the leader's commits are multicast to both),
// acc_empty[b] (leader: all 16 epilogue warps of the pair arrive). Every wait is bounded;
// both CTAs always reach the final cluster barrier and free their tensor memory together.
constexpr int kPairStages = 6;
struct PairCfg {
    static constexpr int A_BYTES = kGemmBM * 128;  // 128 rows x 64 K
    static constexpr int B_BYTES = 128 * 128;      // 128 columns x 64 K
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int EPI_WARPS = 8;
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
    static constexpr int EPI_BYTES = EPI_WARPS * 4096;
    static constexpr int SMEM = kPairStages * STAGE_BYTES + EPI_BYTES + 1024 + 256;
};

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                        const __grid_constant__ CUtensorMap tmE, GemmArgs g) {
    using C = PairCfg;
    constexpr int BN = 256;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* epi = smem + kPairStages * C::STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(epi + C::EPI_BYTES);
    uint64_t* empty = full + kPairStages;
    uint64_t* acc_full = empty + kPairStages;  // [2] leader's MMAs -> both epilogues
    uint64_t* acc_empty = acc_full + 2;        // [2] both epilogues -> leader (16 warp arrivals)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
    const int num_k = (g.K + kGemmBK - 1) / kGemmBK;
    const int TW = EPI == kEpiGlu ? BN / 2 : BN;  // output columns per tile
    const int tiles_n = (g.N + TW - 1) / TW, tiles_m = (g.M + 2 * kGemmBM - 1) / (2 * kGemmBM);
    const int tiles = tiles_n * tiles_m;

    if (warp == 0) {
        if (lane == 0) {
            for (int s = 0; s < kPairStages; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            mbar_init(&acc_full[0], 1);
            mbar_init(&acc_full[1], 1);
            mbar_init(&acc_empty[0], 2 * C::EPI_WARPS);
            mbar_init(&acc_empty[1], 2 * C::EPI_WARPS);
            fence_mbar_init();
            prefetch_tmap(&tmA);
            prefetch_tmap(&tmB);
            prefetch_tmap(&tmC);
        }
        __syncwarp();
        tmem_alloc_pair(tmem_slot, 2 * BN);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers exist before any load or arrive crosses the pair
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    MM_PDL_ENTRY();

    if (warp == 0 && lane == 0) {
        int it = 0;  // ring position across tiles
        bool ok = true;
        for (int tile = pair; tile < tiles && ok; tile += npairs) {
            const int m0 = (tile / tiles_n) * (2 * kGemmBM) + kGemmBM * static_cast<int>(rank);
            const int n0 = (tile % tiles_n) * TW;
            const int nb = EPI == kEpiGlu ? (rank == 0 ? n0 : g.glu_n + n0) : n0 + 128 * static_cast<int>(rank);
            for (int kt = 0; kt < num_k; ++kt, ++it) {
                const int s = it % kPairStages;
                const uint32_t ph = (it / kPairStages) & 1;
                if (!mbar_wait_bounded(&empty[s], ph ^ 1, g.err)) { ok = false; break; }
                uint8_t* sa = smem + s * C::STAGE_BYTES;
                uint8_t* sb = sa + C::A_BYTES;
                if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * C::STAGE_BYTES);
                const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
                const int k0 = kt * kGemmBK;
                if (!g.a_mn) {
                    tma_load_2d_pair(sa, &tmA, fb, k0, m0);
                } else {
                    tma_load_2d_pair(sa, &tmA, fb, m0, k0);
                    tma_load_2d_pair(sa + 8192, &tmA, fb, m0 + 64, k0);
                }
                if (!g.b_mn) {
                    tma_load_2d_pair(sb, &tmB, fb, k0, nb);
                } else {
                    const int kB = gemm_b_row(g, k0);
                    tma_load_2d_pair(sb, &tmB, fb, nb, kB);
                    tma_load_2d_pair(sb + 8192, &tmB, fb, nb + 64, kB);
                }
            }
        }
    } else if (warp == 1 && lane == 0 && rank == 0) {
        int it = 0, j = 0;
        bool ok = true;
        const uint32_t idesc = umma_idesc_f16(g.bf16 != 0, g.a_mn != 0, g.b_mn != 0, 2 * kGemmBM, BN);
        for (int tile = pair; tile < tiles && ok; tile += npairs, ++j) {
            const int buf = j & 1;
            if (!mbar_wait_bounded_cluster(&acc_empty[buf], ((j >> 1) & 1) ^ 1, g.err)) break;
            tc_fence_after();
            const uint32_t dst = tmem + static_cast<uint32_t>(buf * BN);
            for (int kt = 0; kt < num_k; ++kt, ++it) {
                const int s = it % kPairStages;
                const uint32_t ph = (it / kPairStages) & 1;
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
                    tc_mma_f16_pair(dst, ad, bd, idesc, (kt != 0 || k != 0) ? 1u : 0u);
                }
                tc_commit_pair(&empty[s], 0x3);
            }
            tc_commit_pair(&acc_full[buf], 0x3);
        }
    } else if (warp >= 2) {
        const int q = warp & 3;            // TMEM lane quadrant of this warp
        const int half = (warp - 2) >> 2;  // which of the quadrant's warps (0 or 1)
        uint8_t* stage_base = epi + (warp - 2) * 4096;
        const float alpha = g.alpha * (g.alpha_ptr ? *g.alpha_ptr : 1.0f);
        int j = 0;
        for (int tile = pair; tile < tiles; tile += npairs, ++j) {
            const int m0 = (tile / tiles_n) * (2 * kGemmBM) + kGemmBM * static_cast<int>(rank);
            const int n0 = (tile % tiles_n) * TW;
            const int buf = j & 1;
            if (!mbar_wait_bounded(&acc_full[buf], (j >> 1) & 1, g.err)) break;
            tc_fence_after();
            const uint32_t src = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN);
            gemm_drain_tile<BN, C::EPI_WARPS, EPI>(g, tmC, tmD, tmE, stage_base, src, m0, n0, m0 + q * 32, q, half, lane,
                                              alpha, mapa_shared(smem_u32(&acc_empty[buf]), 0));
        }
        if (lane == 0) bulk_wait0();
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // neither CTA leaves while the other may still signal its barriers
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 2 * BN);
    }
}

} // namespace mm
