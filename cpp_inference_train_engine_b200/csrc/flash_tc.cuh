// Causal attention forward on the 5th-generation tensor cores for 64- and 128-wide heads (the
// 35.8M model: qk = 48 nope + 16 rope = dv = 64; the scaled model: 96 + 32 = dv = 128), the
// teacher-forced passes of ops::attention (ops.cpp:109-140). Output and per-row base-2 log-sum-exp are those of
// flash_fwd_mma_kernel, so either backward consumes them.
//
// One CTA per (head, sequence, 128-query tile), 10 warps:
//   warp 8   TMA: Q once, then K tiles into a 2-deep ring and V tiles into one buffer;
//   warp 9   one thread issues tcgen05.mma: S = Q K^T (128 x 128, fp32 in TMEM columns
//            [0, 128)), then O_j = P_j V_j (128 x 64, TMEM columns [128, 192));
//   warps 0-7 softmax, two warps per TMEM lane quadrant (lane = query row): warp w reads
//            key columns [64 (w / 4), +64) of its rows. Pass 1 takes the row maximum (the
//            two halves exchange theirs through shared memory), pass 2 writes
//            P = exp2(S - max) as fp16 into its 64-key half of a 128-byte-swizzled shared
//            tile (the A operand of P V), then the warp folds value columns
//            [32 (w / 4), +32) of O_j into registers with the online-softmax correction.
// Only the diagonal key tile is masked (keys after the query or past the sequence end).
// Every mbarrier wait is bounded; a timeout sets the device error word and the CTA unwinds
// and frees its tensor memory. 96 KB of shared memory and 256 TMEM columns: two CTAs per SM.
#pragma once
#include "common.cuh"

namespace mm {

namespace fatc {
constexpr int kRows = 128;                 // queries per CTA and keys per tile
constexpr int kSub = kRows * 64 * 2;       // one 128 x 64 fp16 box, 128-byte rows
constexpr int kSoftmaxWarps = 8;
constexpr int kThreads = 32 * (kSoftmaxWarps + 2);
// A 128-row tile of width D: D / 64 boxes of 64 columns, one after the other.
template <int D> constexpr int tile_bytes() { return (D / 64) * kSub; }
// Q, K[2], V, P (two 64-key halves), then barriers and the row exchange of the two softmax
// halves: maxima [parity][half][row] and sums [half][row]. 96 KB at D = 64, 160 KB at 128.
template <int D> constexpr int smem_bytes() { return 4 * tile_bytes<D>() + 2 * kSub + 1024 + 256 + 6 * kRows * 4; }
constexpr uint32_t kTmemCols = 256;
constexpr int kColS = 0, kColO = 128;      // S: 128 key columns; O: D value columns
}  // namespace fatc

// q, k, v, out: fp16 [T][H * D] (row pitch H * D), D = 64 or 128 (qk = dv), T = sequences * S,
// viewed through the tensor maps tmQ/tmK/tmV (box {64, 128}, 128-byte swizzle: a tile is D / 64
// boxes); lse2 fp32 [T][H]. Persistent: a 1-D grid of at most the resident CTAs (two per SM
// at D = 64, one at 128: 160 KB of shared memory) walks the work items (query tile, sequence,
// head), longest query tiles first, round robin; barrier phases run on across items (the
// producer loads the next item's Q as soon as the MMA warp has issued the current item's last
// S product), so the setup (barriers, tensor memory) is paid once per CTA. At D = 128 the
// softmax warps fold 64 value columns each.
template <int D>
__global__ void __launch_bounds__(fatc::kThreads, D == 64 ? 2 : 1)
    flash_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, int S, int H, int nseq, float scale,
                        __half* __restrict__ out, float* __restrict__ lse2, int* err) {
    using namespace fatc;
    static_assert(D == 64 || D == 128, "64- or 128-wide heads");
    constexpr int kD = D;
    constexpr int kTileBytes = tile_bytes<D>();
    constexpr int kBoxes = D / 64;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = smem + kTileBytes;      // [2]
    uint8_t* sV = smem + 3 * kTileBytes;
    uint8_t* sP = smem + 4 * kTileBytes;  // keys [0, 64) then [64, 128)
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 4 * kTileBytes + 2 * kSub);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;   // [2]
    uint64_t* k_empty = bars + 3;  // [2]
    uint64_t* v_full = bars + 5;
    uint64_t* v_empty = bars + 6;
    uint64_t* s_full = bars + 7;
    uint64_t* s_empty = bars + 8;  // softmax warps
    uint64_t* p_full = bars + 9;   // softmax warps
    uint64_t* p_empty = bars + 10;
    uint64_t* o_full = bars + 11;
    uint64_t* o_empty = bars + 12; // softmax warps
    uint64_t* xbar = bars + 13;    // [4] the two softmax warps of a lane quadrant
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
    uint64_t* q_empty = bars + 18;  // the MMA warp: the item's S products have read Q
    float* xchg = reinterpret_cast<float*>(smem + 4 * kTileBytes + 2 * kSub + 256);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // persistent: work item i = (query tile, sequence, head), longest query tiles first
    const int qtiles = (S + kRows - 1) / kRows, hs = H * nseq, items = hs * qtiles;
    auto item_of = [&](int i, int& h, int& b, int& qt) {
        qt = qtiles - 1 - i / hs;
        const int r = i - (qtiles - 1 - qt) * hs;
        b = r / H;
        h = r - b * H;
    };

    if (warp == 8) {
        if (lane == 0) {
            mbar_init(q_full, 1);
            mbar_init(q_empty, 1);
            mbar_init(&k_full[0], 1);
            mbar_init(&k_full[1], 1);
            mbar_init(&k_empty[0], 1);
            mbar_init(&k_empty[1], 1);
            mbar_init(v_full, 1);
            mbar_init(v_empty, 1);
            mbar_init(s_full, 1);
            mbar_init(s_empty, kSoftmaxWarps);
            mbar_init(p_full, kSoftmaxWarps);
            mbar_init(p_empty, 1);
            mbar_init(o_full, 1);
            mbar_init(o_empty, kSoftmaxWarps);
            for (int i = 0; i < 4; ++i) mbar_init(&xbar[i], 2);
            fence_mbar_init();
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
        }
        __syncwarp();
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    MM_PDL_ENTRY();

    if (warp == 8) {
        if (lane == 0) {
            bool ok = true;
            int kc = 0;  // key tiles loaded so far (ring position)
            for (int it = blockIdx.x, n = 0; it < items && ok; it += gridDim.x, ++n) {
                int h, b, qt;
                item_of(it, h, b, qt);
                const int row_base = b * S;
                // the previous item's S products have read Q
                if (!mbar_wait_bounded(q_empty, (n & 1) ^ 1, err)) { ok = false; break; }
                mbar_arrive_expect_tx(q_full, kTileBytes);
#pragma unroll
                for (int x = 0; x < kBoxes; ++x) tma_load_2d(sQ + x * kSub, &tmQ, q_full, h * kD + 64 * x, row_base + qt * kRows);
                for (int j = 0; j <= qt; ++j, ++kc) {
                    const int s = kc & 1, u = kc >> 1;
                    if (!mbar_wait_bounded(&k_empty[s], (u & 1) ^ 1, err)) { ok = false; break; }
                    mbar_arrive_expect_tx(&k_full[s], kTileBytes);
#pragma unroll
                    for (int x = 0; x < kBoxes; ++x)
                        tma_load_2d(sK + s * kTileBytes + x * kSub, &tmK, &k_full[s], h * kD + 64 * x, row_base + j * kRows);
                    if (!mbar_wait_bounded(v_empty, (kc & 1) ^ 1, err)) { ok = false; break; }
                    mbar_arrive_expect_tx(v_full, kTileBytes);
#pragma unroll
                    for (int x = 0; x < kBoxes; ++x) tma_load_2d(sV + x * kSub, &tmV, v_full, h * kD + 64 * x, row_base + j * kRows);
                }
            }
        }
    } else if (warp == 9) {
        if (lane == 0) {
            const uint32_t id_s = umma_idesc_f16(false, false, false, kRows, kRows);  // Q K^T, both K-major
            const uint32_t id_o = umma_idesc_f16(false, false, true, kRows, kD);      // P V, V MN-major
            const uint32_t aq = smem_u32(sQ), ap = smem_u32(sP), bv = smem_u32(sV);
            bool ok = true;
            int kc = 0;
            for (int it = blockIdx.x, n = 0; it < items && ok; it += gridDim.x, ++n) {
                int h, b, qt;
                item_of(it, h, b, qt);
                if (!mbar_wait_bounded(q_full, n & 1, err)) { ok = false; break; }
                for (int j = 0; j <= qt; ++j, ++kc) {
                    const int s = kc & 1, u = kc >> 1;
                    if (!mbar_wait_bounded(&k_full[s], u & 1, err)) { ok = false; break; }
                    if (!mbar_wait_bounded(s_empty, (kc & 1) ^ 1, err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t bk = smem_u32(sK + s * kTileBytes);
#pragma unroll
                    for (int k = 0; k < kD / 16; ++k)  // k-steps 4x..4x+3 in box x
                        tc_mma_f16(tmem + kColS, umma_desc_sw128(aq + (k >> 2) * kSub + (k & 3) * 32, 16, 1024),
                                   umma_desc_sw128(bk + (k >> 2) * kSub + (k & 3) * 32, 16, 1024), id_s, k ? 1u : 0u);
                    tc_commit(s_full);
                    tc_commit(&k_empty[s]);
                    if (j == qt) tc_commit(q_empty);  // the item's last read of Q
                    if (!mbar_wait_bounded(p_full, kc & 1, err)) { ok = false; break; }
                    if (!mbar_wait_bounded(v_full, kc & 1, err)) { ok = false; break; }
                    if (!mbar_wait_bounded(o_empty, (kc & 1) ^ 1, err)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int k = 0; k < kRows / 16; ++k)
                        // V MN-major: 16 keys = 2048 B down a box; the next 64 value columns one box on
                        tc_mma_f16(tmem + kColO, umma_desc_sw128(ap + (k >> 2) * kSub + (k & 3) * 32, 16, 1024),
                                   umma_desc_sw128(bv + k * 2048, D == 64 ? 8192 : kSub, 1024), id_o, k ? 1u : 0u);
                    tc_commit(o_full);
                    tc_commit(v_empty);
                    tc_commit(p_empty);
                }
            }
        }
    } else {
        // softmax: thread = query row r of the tile (TMEM lane r), key/value half hh
        const int q = warp & 3, hh = warp >> 2;
        const int r = q * 32 + lane;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
        const float cs = scale * 1.4426950408889634f;
        uint8_t* prow = sP + hh * kSub + r * 128;
        constexpr int kHalf = kD / 2;  // value columns this warp folds
        bool ok = true;
        int kc = 0;  // key tiles consumed so far (barrier phases)
        int xc = 0;  // uses of this quadrant's exchange barrier so far
        for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
            int h, b, qt;
            item_of(it, h, b, qt);
            const int nk = qt + 1;  // key tiles at or below the diagonal
            const int row_base = b * S;
            const int qpos = qt * kRows + r;
            float acc[kHalf];
#pragma unroll
            for (int i = 0; i < kHalf; ++i) acc[i] = 0.f;
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < nk; ++j, ++kc) {
                if (!mbar_wait_bounded(s_full, kc & 1, err)) { ok = false; break; }
                tc_fence_after();
                const bool diag = j == qt;
                // diagonal tile: columns after the query or past the sequence end are masked
                const int lim = diag ? min(qpos, S - 1) - j * kRows - hh * 64 : 63;
                float mx = -INFINITY;
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    float v[32];
                    tmem_ld32_nowait(lane_base + kColS + hh * 64 + c * 32, v);
                    tmem_wait_ld();
                    if (diag) {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (c * 32 + i <= lim) mx = fmaxf(mx, v[i]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) mx = fmaxf(mx, v[i]);
                    }
                }
                float* xm = xchg + (kc & 1) * 2 * kRows;
                xm[hh * kRows + r] = mx;
                __syncwarp();
                if (lane == 0) mbar_arrive(&xbar[q]);
                if (!mbar_wait_bounded(&xbar[q], xc & 1, err)) { ok = false; break; }
                ++xc;
                mx = fmaxf(mx, xm[(hh ^ 1) * kRows + r]) * cs;  // cs > 0: max commutes with the scale
                const float m_new = fmaxf(m_run, mx);
                const float base = m_new == -INFINITY ? 0.f : m_new;
                const float corr = fast_exp2(m_run - base);
                if (!mbar_wait_bounded(p_empty, (kc & 1) ^ 1, err)) { ok = false; break; }
                float ls = 0.f;
#pragma unroll 1
                for (int c = 0; c < 2; ++c) {
                    float v[32];
                    tmem_ld32_nowait(lane_base + kColS + hh * 64 + c * 32, v);
                    tmem_wait_ld();
                    uint32_t w[16];
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        float p0 = fast_exp2(fmaf(v[i], cs, -base));
                        float p1 = fast_exp2(fmaf(v[i + 1], cs, -base));
                        if (diag) {
                            if (c * 32 + i > lim) p0 = 0.f;
                            if (c * 32 + i + 1 > lim) p1 = 0.f;
                        }
                        ls += p0 + p1;
                        const __half2 hp = __floats2half2_rn(p0, p1);
                        w[i >> 1] = *reinterpret_cast<const uint32_t*>(&hp);
                    }
                    // keys [32c, 32c + 32) of this half: four 16-byte chunks, 128-byte swizzle
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const int cc = c * 4 + q4;
                        *reinterpret_cast<uint4*>(prow + ((cc ^ (r & 7)) << 4)) =
                            make_uint4(w[4 * q4], w[4 * q4 + 1], w[4 * q4 + 2], w[4 * q4 + 3]);
                    }
                }
                tc_fence_before();
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(s_empty);
                    mbar_arrive(p_full);
                }
                if (!mbar_wait_bounded(o_full, kc & 1, err)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int oc = 0; oc < kHalf; oc += 32) {
                    float o[32];
                    tmem_ld32_nowait(lane_base + kColO + hh * kHalf + oc, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) acc[oc + i] = acc[oc + i] * corr + o[i];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(o_empty);
                l_run = l_run * corr + ls;
                m_run = m_new;
            }
            if (!ok) break;
            // the row sum is the two halves' sums (same maxima, same corrections)
            float* xl = xchg + 2 * 2 * kRows;
            xl[hh * kRows + r] = l_run;
            __syncwarp();
            if (lane == 0) mbar_arrive(&xbar[q]);
            if (!mbar_wait_bounded(&xbar[q], xc & 1, err)) { ok = false; break; }
            ++xc;
            if (qpos < S) {
                const float l = l_run + xl[(hh ^ 1) * kRows + r];
                const float inv = 1.f / l;
                __half* dst = out + (static_cast<long long>(row_base) + qpos) * (static_cast<long long>(H) * kD) + h * kD +
                              hh * kHalf;
#pragma unroll
                for (int i = 0; i < kHalf; i += 8) {
                    const __half2 h0 = __floats2half2_rn(acc[i] * inv, acc[i + 1] * inv);
                    const __half2 h1 = __floats2half2_rn(acc[i + 2] * inv, acc[i + 3] * inv);
                    const __half2 h2 = __floats2half2_rn(acc[i + 4] * inv, acc[i + 5] * inv);
                    const __half2 h3 = __floats2half2_rn(acc[i + 6] * inv, acc[i + 7] * inv);
                    *reinterpret_cast<uint4*>(dst + i) =
                        make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                                   *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
                }
                if (hh == 0) lse2[(static_cast<long long>(row_base) + qpos) * H + h] = m_run + log2f(l);
            }
            // the partner half reads xl before its next exchange, which this warp waits for
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}


namespace fadq {
constexpr int kRows = 128;                  // queries per CTA
constexpr int kKeys = 64;                   // keys per tile
constexpr int kD = 64;
constexpr int kQBytes = kRows * kD * 2;     // 16 KB
constexpr int kKBytes = kKeys * kD * 2;     // 8 KB
constexpr int kSoftmaxWarps = 8;
constexpr int kThreads = 32 * (kSoftmaxWarps + 2);
// Q, dO, K[2], V[2], dS [128 queries][64 keys], then barriers
constexpr int kSmem = 2 * kQBytes + 4 * kKBytes + kQBytes + 1024 + 256;
constexpr uint32_t kTmemCols = 128;
constexpr int kColS = 0, kColDP = 64, kColDQ = 0;  // dQ_j reuses S's columns once S is consumed
}  // namespace fadq

// dQ of causal attention on the tensor cores (the backward of ops::attention, ops.cpp:143-172):
// one CTA per (head, sequence, 128-query tile), 64-key tiles at or below the diagonal.
// warp 8 TMA (Q and dO once, K and V tiles into a 2-deep ring), warp 9 tcgen05.mma
// (S = Q K^T and dP = dO V^T into TMEM, then dQ_j = dS K_j), warps 0-7 one thread per query
// row and 32-key half: P = exp2(S c - lse2) from the forward's base-2 log-sum-exp,
// dS = P (dP - D) scale in fp16 into the A operand of dQ_j, dQ accumulated in registers.
// The epilogue applies the inverse query RoPE and writes fp16 dq16, as
// flash_bwd_dq_mma_kernel does. 82 KB of shared memory, 128 TMEM columns: two CTAs per SM.
__global__ void __launch_bounds__(fadq::kThreads, 2)
    flash_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                           const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                           const float* __restrict__ lse2, const float* __restrict__ Dd, int S, int H, float scale,
                           __half* __restrict__ dq16, long long ld_dq, const float* __restrict__ cos_t,
                           const float* __restrict__ sin_t, int rope_begin, int rope, int* err) {
    using namespace fadq;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* sQ = smem;
    uint8_t* sG = smem + kQBytes;              // dO
    uint8_t* sK = smem + 2 * kQBytes;          // [2]
    uint8_t* sV = sK + 2 * kKBytes;            // [2]
    uint8_t* sDS = sV + 2 * kKBytes;           // [128][64] fp16
    uint64_t* bars = reinterpret_cast<uint64_t*>(sDS + kQBytes);
    uint64_t* q_full = bars + 0;
    uint64_t* kv_full = bars + 1;   // [2]
    uint64_t* kv_empty = bars + 3;  // [2]
    uint64_t* s_full = bars + 5;
    uint64_t* ds_full = bars + 6;   // softmax warps
    uint64_t* dq_full = bars + 7;
    uint64_t* dq_empty = bars + 8;  // softmax warps
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.x, b = blockIdx.y;
    const int qt = gridDim.z - 1 - blockIdx.z;
    const int nk = min(2 * qt + 2, (S + kKeys - 1) / kKeys);  // key tiles at or below the diagonal
    const int row_base = b * S;

    if (warp == 8) {
        if (lane == 0) {
            mbar_init(q_full, 1);
            mbar_init(&kv_full[0], 1);
            mbar_init(&kv_full[1], 1);
            mbar_init(&kv_empty[0], 1);
            mbar_init(&kv_empty[1], 1);
            mbar_init(s_full, 1);
            mbar_init(ds_full, kSoftmaxWarps);
            mbar_init(dq_full, 1);
            mbar_init(dq_empty, kSoftmaxWarps);
            fence_mbar_init();
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmDO);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
        }
        __syncwarp();
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    MM_PDL_ENTRY();

    if (warp == 8) {
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, 2 * kQBytes);
            tma_load_2d(sQ, &tmQ, q_full, h * kD, row_base + qt * kRows);
            tma_load_2d(sG, &tmDO, q_full, h * kD, row_base + qt * kRows);
            for (int j = 0; j < nk; ++j) {
                const int s = j & 1, u = j >> 1;
                if (!mbar_wait_bounded(&kv_empty[s], (u & 1) ^ 1, err)) break;
                mbar_arrive_expect_tx(&kv_full[s], 2 * kKBytes);
                tma_load_2d(sK + s * kKBytes, &tmK, &kv_full[s], h * kD, row_base + j * kKeys);
                tma_load_2d(sV + s * kKBytes, &tmV, &kv_full[s], h * kD, row_base + j * kKeys);
            }
        }
    } else if (warp == 9) {
        if (lane == 0) {
            const uint32_t id_s = umma_idesc_f16(false, false, false, kRows, kKeys);  // Q K^T, dO V^T
            const uint32_t id_q = umma_idesc_f16(false, false, true, kRows, kD);     // dS K, K MN-major
            const uint32_t aq = smem_u32(sQ), ag = smem_u32(sG), ads = smem_u32(sDS);
            bool ok = mbar_wait_bounded(q_full, 0, err);
            for (int j = 0; j < nk && ok; ++j) {
                const int s = j & 1, u = j >> 1;
                if (!mbar_wait_bounded(&kv_full[s], u & 1, err)) { ok = false; break; }
                if (j > 0 && !mbar_wait_bounded(dq_empty, (j - 1) & 1, err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t bk = smem_u32(sK + s * kKBytes), bv = smem_u32(sV + s * kKBytes);
#pragma unroll
                for (int k = 0; k < kD / 16; ++k) {
                    tc_mma_f16(tmem + kColS, umma_desc_sw128(aq + k * 32, 16, 1024),
                               umma_desc_sw128(bk + k * 32, 16, 1024), id_s, k ? 1u : 0u);
                    tc_mma_f16(tmem + kColDP, umma_desc_sw128(ag + k * 32, 16, 1024),
                               umma_desc_sw128(bv + k * 32, 16, 1024), id_s, k ? 1u : 0u);
                }
                tc_commit(s_full);
                if (!mbar_wait_bounded(ds_full, j & 1, err)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < kKeys / 16; ++k)
                    tc_mma_f16(tmem + kColDQ, umma_desc_sw128(ads + k * 32, 16, 1024),
                               umma_desc_sw128(bk + k * 2048, 8192, 1024), id_q, k ? 1u : 0u);
                tc_commit(dq_full);
                tc_commit(&kv_empty[s]);
            }
        }
    } else {
        // thread = query row r (TMEM lane r), key half hh of each 64-key tile, dQ columns [32 hh, +32)
        const int q = warp & 3, hh = warp >> 2;
        const int r = q * 32 + lane;
        const int qpos = qt * kRows + r;
        const bool row_ok = qpos < S;
        const float L = row_ok ? lse2[(static_cast<long long>(row_base) + qpos) * H + h] : 0.f;
        const float D = row_ok ? Dd[(static_cast<long long>(row_base) + qpos) * H + h] : 0.f;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
        const float cs = scale * 1.4426950408889634f;
        uint8_t* drow = sDS + r * 128;
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.f;
        bool ok = true;
        for (int j = 0; j < nk && ok; ++j) {
            if (!mbar_wait_bounded(s_full, j & 1, err)) { ok = false; break; }
            tc_fence_after();
            const int key0 = j * kKeys + hh * 32;
            // last key of this half the row may attend (causal, inside the sequence)
            const int lim = row_ok ? min(qpos, S - 1) - key0 : -1;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                float sv[16], dp[16];
                tmem_ld16(lane_base + kColS + hh * 32 + c * 16, sv);
                tmem_ld16(lane_base + kColDP + hh * 32 + c * 16, dp);
                uint32_t w[8];
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    const float p0 = c * 16 + i <= lim ? fast_exp2(fmaf(sv[i], cs, -L)) : 0.f;
                    const float p1 = c * 16 + i + 1 <= lim ? fast_exp2(fmaf(sv[i + 1], cs, -L)) : 0.f;
                    const __half2 hv = __floats2half2_rn(p0 * (dp[i] - D) * scale, p1 * (dp[i + 1] - D) * scale);
                    w[i >> 1] = *reinterpret_cast<const uint32_t*>(&hv);
                }
                // keys [32 hh + 16 c, +16): two 16-byte chunks of the 128-byte row, swizzled
#pragma unroll
                for (int q2 = 0; q2 < 2; ++q2) {
                    const int cc = hh * 4 + c * 2 + q2;
                    *reinterpret_cast<uint4*>(drow + ((cc ^ (r & 7)) << 4)) =
                        make_uint4(w[4 * q2], w[4 * q2 + 1], w[4 * q2 + 2], w[4 * q2 + 3]);
                }
            }
            tc_fence_before();
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(ds_full);
            if (!mbar_wait_bounded(dq_full, j & 1, err)) { ok = false; break; }
            tc_fence_after();
            {
                float o[32];
                tmem_ld32_nowait(lane_base + kColDQ + hh * 32, o);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) acc[i] += o[i];
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(dq_empty);
        }
        if (ok && row_ok) {
            // inverse RoPE of the query rotation on columns [rope_begin, rope_begin + rope)
            const int half_r = rope / 2;
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
                const int cc = hh * 32 + i;
                if (cc >= rope_begin && cc < rope_begin + rope) {
                    const int pair = (cc - rope_begin) >> 1;
                    const float cn = cos_t[qpos * half_r + pair], sn = -sin_t[qpos * half_r + pair];
                    const float a = acc[i], bb = acc[i + 1];
                    acc[i] = a * cn - bb * sn;
                    acc[i + 1] = a * sn + bb * cn;
                }
            }
            __half* dst = dq16 + (static_cast<long long>(row_base) + qpos) * ld_dq + h * kD + hh * 32;
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
                const __half2 h0 = __floats2half2_rn(acc[i], acc[i + 1]);
                const __half2 h1 = __floats2half2_rn(acc[i + 2], acc[i + 3]);
                const __half2 h2 = __floats2half2_rn(acc[i + 4], acc[i + 5]);
                const __half2 h3 = __floats2half2_rn(acc[i + 6], acc[i + 7]);
                *reinterpret_cast<uint4*>(dst + i) =
                    make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                               *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 8) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace mm
