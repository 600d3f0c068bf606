// One rollout decode step of the 35.8M MLA model as ONE persistent cooperative kernel
// (CpuDecoder::decode, inference.cpp:69-174, absorbed form, for every row at once): token
// embedding, the 10 layers, the final norm and the fp32-accurate split of the vocabulary
// head's input. The vocabulary product and the sampler stay separate launches.
//
// Why: at a few hundred rows a decode step is ~100 dependent launches of a few microseconds
// of work each, so launch and pipeline fill/drain latency, not HBM or the tensor pipe, set
// the step time. Here one CTA per SM lives through the whole step and the kernel-boundary
// round trips become grid barriers (a global arrival counter, release/acquire, every wait
// bounded). Per layer, eight phases:
//   1 [W_dq | W_dkv] on tcgen05 with the latent epilogue: q-latent RMSNorm -> fp16 cq, and
//     kv-latent RMSNorm + rope-key rotation written straight into the latent cache row
//     (a thread owns a row, so the norms need no cross-thread reduction)
//   2 absorbed W_uq (query per head against the latent cache) on tcgen05 -> fp32 q
//   3 latent attention, one warp per (row, context split) (decode_attention_item); the last
//     split of a row to finish merges the row's partials (per-row arrival counter)
//   4 W_uv.W_o on tcgen05, K split -> fp32 partials
//   5 residual + partials (fixed order) -> x, RMSNorm -> fp16 h2
//   6 [W_gate | W_up] on tcgen05 with the SwiGLU epilogue -> fp16
//   7 W_down on tcgen05, K split -> fp32 partials
//   8 residual + partials -> x, RMSNorm -> next layer's fp16 input (after the last layer:
//     the final norm, split into the [hi | lo | hi] fp16 rows of the vocabulary head, and
//     every row's position advanced)
// GEMM phases: warp 0 issues TMA loads (128-byte swizzle, K-major activations, MN-major
// weights read in place) into a 4-stage mbarrier ring that runs across units and phases,
// warp 1 issues tcgen05.mma (one thread) into one of two tensor-memory accumulators, warps
// 4-7 drain tensor memory (lane quadrant = warp % 4, one row per thread) with plain global
// stores. All sums are in a fixed order: a step is bit-reproducible.
#pragma once
#include "attention.cuh"
#include "common.cuh"
#include "gemm_tc.cuh"
#include "kernels_vec.cuh"

namespace mm {
namespace mk {
constexpr int D = 512, QR = 192, KVR = 128, ROPE = 16, KVW = 144, H = 8, DFF = 1360;
constexpr int HKV = H * KVR;   // 1024: latent context of all heads
constexpr int QW = H * KVW;    // 1152: absorbed query of all heads
constexpr int QKV = QR + KVW;  // 336: [W_dq | W_dkv]
constexpr int kMaxLayers = 16;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kStages = 4;
constexpr int kABytes = 128 * 128;  // 128 rows x 64 k, fp16
constexpr int kBChunk = 64 * 128;   // 64 k x 64 n, fp16
constexpr int kBChunks = 3;
constexpr int kStageBytes = kABytes + kBChunks * kBChunk;
constexpr int kRingBytes = kStages * kStageBytes;
// the attention phase reuses the ring's shared memory: each warp a 2-deep cache-tile ring
// (deeper rings, up to 4 tiles in flight per item, measured no faster: the phase is bound by
// its chain of dependent reads and the split merge, not by the tile loads)
constexpr int kAttnStages = 2;
constexpr int kAttnBytes = kWarps * dec::warp_smem<kAttnStages>();
constexpr int kDataBytes = kRingBytes > kAttnBytes ? kRingBytes : kAttnBytes;
constexpr int kSmem = kDataBytes + 1024 + 256;
constexpr int kTmemCols = 512;
constexpr int kAccStride = 256;  // tensor-memory columns between the two accumulators
constexpr int kMaxKs = 6;
static_assert(dec::H == H && dec::KV == KVR && dec::R == ROPE, "latent attention shape");
}  // namespace mk

// Everything one fused decode step reads and writes. The tensor maps: K-major activation
// maps (box 64 x 128 rows) and MN-major weight maps (box 64 x 64) per layer.
struct MkParams {
    CUtensorMap a_h16, a_ctx16, a_h2, a_gated;
    // wf: the query weights W_dq . diag(g_q) . Wq folded for the latent phase [D][QW]
    CUtensorMap wa[mk::kMaxLayers], wf[mk::kMaxLayers], wo[mk::kMaxLayers], wgu[mk::kMaxLayers],
        wdown[mk::kMaxLayers];
    const float* attn_norm[mk::kMaxLayers];
    const float* ffn_norm[mk::kMaxLayers];
    const float* q_norm[mk::kMaxLayers];
    const float* kv_norm[mk::kMaxLayers];
    const float* final_norm;
    const float* E;  // fp32 token table [V][D]
    const uint16_t* tok;
    int V, B, L, Sc;
    int ns;                  // attention context splits per row
    int ks_o, per_o;         // K splits of W_o and k-blocks per split
    int ks_d, per_d;         // the same for W_down
    float eps, scale;
    float* x;                // [B][D] residual stream
    __half* h16;             // [B][D] normed layer input
    float* qs;               // [B] the q latent's RMSNorm scale 1 / rms (the query's row factor)
    float* qf;               // [B][QW] absorbed query before its row factor
    __half* ctx16;           // [B][HKV]
    __half* h2;              // [B][D]
    __half* gated;           // [B][DFF]
    __half* h3;              // [B][ld3] vocabulary-head input [hi | lo | hi]
    long long ld3;
    float* part;             // [kMaxKs][B][D] split-K partials
    float* attn_part;        // [B][ns][H][KV + 2]
    int* attn_cnt;           // [B] arrivals per row, zero between uses
    __half* cache;           // [L][B][Sc][KVW]
    int* pos;                // [B] this step's position per row
    const float* cos_t;
    const float* sin_t;
    unsigned* bar;           // grid barrier arrivals, zero at launch
    int* err;
    // optional: CTA 0 records the global timer (ns) at the start and after every barrier,
    // so consecutive differences are the phases' wall times
    unsigned long long* trace;
    // each layer's five decode matrices as contiguous byte ranges, for L2 prefetch
    const void* wbase[mk::kMaxLayers][5];
    long long wbytes[mk::kMaxLayers][5];
};

__device__ __forceinline__ void mk_trace(const MkParams& p, int& k) {
    if (p.trace && blockIdx.x == 0 && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        p.trace[k] = t;
    }
    ++k;
}

enum MkEpi : int { kMkLatent = 0, kMkF32 = 1, kMkGlu = 2, kMkPartial = 3 };

__device__ __forceinline__ unsigned mk_ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid-wide barrier. Every thread first orders its own generic global writes before later
// async-proxy (TMA) reads of them anywhere; after the CTA barrier, thread 0 arrives on the
// counter with release semantics and spins with acquire loads (bounded: a CTA that never
// arrives turns into kErrWaitTimeout and an abort, not a hang). Returns false when this CTA
// must stop.
__device__ __forceinline__ bool mk_sync(const MkParams& p, unsigned& epoch, int* s_abort) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncthreads();
    epoch += gridDim.x;
    if (threadIdx.x == 0) {
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar) : "memory");
        for (uint32_t i = 0;; ++i) {
            if (mk_ld_acquire(p.bar) >= epoch) break;
            if (i > (1u << 24) || *s_abort) {
                raise_error(p.err, kErrWaitTimeout);
                *s_abort = 1;
                break;
            }
            if (i > 512) __nanosleep(64);
        }
    }
    __syncthreads();
    return *s_abort == 0;
}

// L2 prefetch of this CTA's share of `bytes` contiguous bytes at `base` (16-byte aligned
// base and size), by one thread: the next phases' weights arrive in L2 while the current
// phase runs, so their tensor-core phases read weights at L2 latency.
__device__ __forceinline__ void mk_prefetch_l2(const void* base, long long bytes) {
    const long long per = ((bytes + gridDim.x - 1) / gridDim.x + 15) / 16 * 16;
    const long long off = static_cast<long long>(blockIdx.x) * per;
    long long n = bytes - off < per ? bytes - off : per;
    const char* src = static_cast<const char*>(base) + off;
    while (n > 0) {
        const int chunk = static_cast<int>(n < 65536 ? n : 65536);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(chunk) : "memory");
        src += chunk;
        n -= chunk;
    }
}

// One GEMM unit's place: rows [m0, m0 + 128), MMA width n_mma from B columns bcol(j) of the
// chunks, k-blocks [kb0, kb1), split z.
struct MkUnit {
    int m0, nt, z, kb0, kb1;
};

template <int EPI>
__device__ __forceinline__ int mk_b_col(int nt, int j) {
    // latent units: q 0,64,128 and kv 192,256,320 of Wa; then 192-column tiles of Wf
    if constexpr (EPI == kMkLatent) return nt < 2 ? nt * mk::QR + 64 * j : (nt - 2) * mk::QR + 64 * j;
    if constexpr (EPI == kMkGlu) return j == 0 ? 64 * nt : mk::DFF + 64 * nt;  // gate, up
    return 128 * nt + 64 * j;
}
template <int EPI> __host__ __device__ constexpr int mk_chunks() { return EPI == kMkLatent ? 3 : 2; }
template <int EPI> __device__ __forceinline__ int mk_n_mma(int nt) {
    if constexpr (EPI == kMkLatent) return nt == 1 ? mk::KVW : mk::QR;
    return 128;
}

// The shared pieces of one CTA's tensor-core pipeline.
struct MkPipe {
    uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    uint64_t* acc_full;
    uint64_t* acc_empty;
    uint32_t tmem;
    int* s_abort;
};

// A GEMM phase over units u = blockIdx.x, blockIdx.x + gridDim.x, ... of
// (split z, m-tile, n-tile). prod_it / mma_it (ring positions) and acc_j (accumulator
// uses) persist across phases in the threads that own them.
__device__ __forceinline__ void mk_stamp(const MkParams& p, int slot) {
    if (p.trace && blockIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        p.trace[slot] = t;
    }
}

// Trace slots of the GEMM phases' inner stamps (CTA 0's first unit): per GEMM phase g,
// [kMkStampBase + 3 g] producer start, + 1 accumulator ready (epilogue), + 2 epilogue done.
constexpr int kMkStampBase = 128;
// Trace slots of the attention phases: per layer l, [kMkAttnStamp + 4 l] CTA 0 warp 0's first
// item starts, + 1 its queries are in registers, + 2 its cache tiles are done, + 3 merged.
constexpr int kMkAttnStamp = 256;

template <int EPI>
__device__ __forceinline__ void mk_gemm_phase(const MkParams& p, const MkPipe& pp, const CUtensorMap* ta,
                                              const CUtensorMap* tb, int n_tiles, int nk, int ks, int per, int l,
                                              int& prod_it, int& mma_it, int& acc_j, int gidx) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int MT = (p.B + 127) / 128;
    const int units = MT * n_tiles * ks;
    auto unit_of = [&](int u) {
        MkUnit t;
        t.z = u / (MT * n_tiles);
        const int r = u - t.z * MT * n_tiles;
        t.m0 = (r / n_tiles) * 128;
        t.nt = r % n_tiles;
        t.kb0 = t.z * per;
        t.kb1 = min(nk, t.kb0 + per);
        return t;
    };
    constexpr int CH = mk_chunks<EPI>();
    if (warp == 0) {
        if (lane == 0) {
            // the activations this phase loads were written by generic stores before the barrier
            asm volatile("fence.proxy.async.global;" ::: "memory");
            mk_stamp(p, kMkStampBase + 3 * gidx);
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                const MkUnit t = unit_of(u);
                for (int kb = t.kb0; kb < t.kb1; ++kb, ++prod_it) {
                    const int s = prod_it % mk::kStages;
                    const uint32_t ph = (prod_it / mk::kStages) & 1;
                    if (!mbar_wait_bounded(&pp.empty[s], ph ^ 1, p.err)) { ok = false; break; }
                    uint8_t* sa = pp.ring + s * mk::kStageBytes;
                    uint8_t* sb = sa + mk::kABytes;
                    mbar_arrive_expect_tx(&pp.full[s], mk::kABytes + CH * mk::kBChunk);
                    tma_load_2d(sa, ta, &pp.full[s], kb * 64, t.m0);
#pragma unroll
                    for (int j = 0; j < CH; ++j)
                        tma_load_2d(sb + j * mk::kBChunk, (EPI == kMkLatent && t.nt >= 2) ? &p.wf[l] : tb, &pp.full[s],
                                    mk_b_col<EPI>(t.nt, j), kb * 64);
                }
            }
            if (!ok) *pp.s_abort = 1;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++acc_j) {
                const MkUnit t = unit_of(u);
                const int buf = acc_j & 1;
                if (!mbar_wait_bounded(&pp.acc_empty[buf], ((acc_j >> 1) & 1) ^ 1, p.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t dst = pp.tmem + static_cast<uint32_t>(buf * mk::kAccStride);
                const uint32_t idesc = umma_idesc_f16(false, false, true, 128, mk_n_mma<EPI>(t.nt));
                for (int kb = t.kb0; kb < t.kb1; ++kb, ++mma_it) {
                    const int s = mma_it % mk::kStages;
                    const uint32_t ph = (mma_it / mk::kStages) & 1;
                    if (!mbar_wait_bounded(&pp.full[s], ph, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(pp.ring + s * mk::kStageBytes);
                    const uint32_t sb = sa + mk::kABytes;
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        tc_mma_f16(dst, umma_desc_sw128(sa + k * 32, 16, 1024), umma_desc_sw128(sb + k * 2048, 8192, 1024),
                                   idesc, (kb != t.kb0 || k != 0) ? 1u : 0u);
                    tc_commit(&pp.empty[s]);
                }
                if (!ok) break;
                tc_commit(&pp.acc_full[buf]);
            }
            if (!ok) *pp.s_abort = 1;
        }
    } else if (warp >= 4) {
        const int q = warp & 3;
        for (int u = blockIdx.x; u < units; u += gridDim.x, ++acc_j) {
            const MkUnit t = unit_of(u);
            const int buf = acc_j & 1;
            const int r = t.m0 + q * 32 + lane;
            const bool live = r < p.B;
            // what the kv unit's epilogue reads besides the accumulator, fetched while the MMAs
            // run: its norm weights (into L1), the row's position and its rope table entries
            int ps = 0;
            bool in = false;
            float cs[mk::ROPE / 2], sn[mk::ROPE / 2];
            if constexpr (EPI == kMkLatent) {
                if (t.nt == 1) {
                    if (q * 32 + lane < mk::KVR / 32) prefetch_l1(p.kv_norm[l] + 32 * (q * 32 + lane));
                    ps = live ? __ldcg(p.pos + r) : 0;
                    in = live && ps >= 0 && ps < p.Sc;
#pragma unroll
                    for (int h = 0; h < mk::ROPE / 2; ++h) {
                        cs[h] = in ? p.cos_t[ps * (mk::ROPE / 2) + h] : 0.f;
                        sn[h] = in ? p.sin_t[ps * (mk::ROPE / 2) + h] : 0.f;
                    }
                }
            }
            if (!mbar_wait_bounded(&pp.acc_full[buf], (acc_j >> 1) & 1, p.err)) {
                *pp.s_abort = 1;
                break;
            }
            tc_fence_after();
            if (u == static_cast<int>(blockIdx.x) && warp == 4 && lane == 0) mk_stamp(p, kMkStampBase + 3 * gidx + 1);
            const uint32_t src = pp.tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * mk::kAccStride);
            float v[32];
            if constexpr (EPI == kMkLatent) {
              if (t.nt >= 2) {
                // query columns [192 (nt - 2), +192) of h . Wf in fp32; their row factor is qs
                float* o = p.qf + static_cast<long long>(r) * mk::QW + mk::QR * (t.nt - 2);
#pragma unroll 1
                for (int c = 0; c < mk::QR; c += 32) {
                    tmem_ld32_nowait(src + c, v);
                    tmem_wait_ld();
                    if (live) {
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            *reinterpret_cast<float4*>(o + c + 4 * e) =
                                make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
                    }
                    __syncwarp();
                }
              } else {
                // whole-row norms by one thread: tensor-memory reads in batches of 96 columns
                // (three 32-column loads per wait)
                float b3[96];
                const int nn = t.nt == 0 ? mk::QR : mk::KVR;  // columns under the norm
                float ss = 0.f;
                for (int c = 0; c < nn; c += 96) {
                    tmem_ld32_nowait(src + c, b3);
                    tmem_ld32_nowait(src + c + 32, b3 + 32);
                    if (c + 64 < nn) tmem_ld32_nowait(src + c + 64, b3 + 64);
                    tmem_wait_ld();
                    const int m = min(96, nn - c);
#pragma unroll
                    for (int i = 0; i < 96; ++i)
                        if (i < m) ss += b3[i] * b3[i];
                }
                const float inv = 1.0f / sqrtf(ss / static_cast<float>(nn) + p.eps);
                if (t.nt == 0) {
                    // the query's row factor (g_q is folded into Wf)
                    if (live) p.qs[r] = inv;
                } else {
                    const float* w = p.kv_norm[l];
                    if (live && !in) raise_error(p.err, kErrBadIndex);
                    __half* o = p.cache + ((static_cast<long long>(l) * p.B + r) * p.Sc + (in ? ps : 0)) * mk::KVW;
                    for (int c = 0; c < mk::KVW; c += 96) {  // columns [0, 96), [96, 192): latent 128 | rope 16
                        tmem_ld32_nowait(src + c, b3);
                        tmem_ld32_nowait(src + c + 32, b3 + 32);
                        if (c == 0) tmem_ld32_nowait(src + c + 64, b3 + 64);
                        tmem_wait_ld();
                        if (in) {
                            const int lat = min(96, mk::KVR - c);  // latent columns in this batch
#pragma unroll
                            for (int e = 0; e < 12; ++e) {
                                if (8 * e >= lat) break;
                                const float4 w0 = *reinterpret_cast<const float4*>(w + c + 8 * e);
                                const float4 w1 = *reinterpret_cast<const float4*>(w + c + 8 * e + 4);
                                const float* f = b3 + 8 * e;
                                *reinterpret_cast<uint4*>(o + c + 8 * e) = make_uint4(
                                    pack_half2(f[0] * inv * w0.x, f[1] * inv * w0.y), pack_half2(f[2] * inv * w0.z, f[3] * inv * w0.w),
                                    pack_half2(f[4] * inv * w1.x, f[5] * inv * w1.y), pack_half2(f[6] * inv * w1.z, f[7] * inv * w1.w));
                            }
                            if (c + 96 > mk::KVR) {  // the rope key: adjacent pairs rotated to this row's position
                                const float* f = b3 + (mk::KVR - c);
                                uint32_t wd[8];
#pragma unroll
                                for (int h = 0; h < mk::ROPE / 2; ++h) {
                                    const float a = f[2 * h], b = f[2 * h + 1];
                                    wd[h] = pack_half2(a * cs[h] - b * sn[h], a * sn[h] + b * cs[h]);
                                }
                                *reinterpret_cast<uint4*>(o + mk::KVR) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
                                *reinterpret_cast<uint4*>(o + mk::KVR + 8) = make_uint4(wd[4], wd[5], wd[6], wd[7]);
                            }
                        }
                        __syncwarp();
                    }
                }
              }
            } else if constexpr (EPI == kMkGlu) {
                __half* o = p.gated + static_cast<long long>(r) * mk::DFF + 64 * t.nt;
#pragma unroll 1
                for (int c = 0; c < 64; c += 32) {
                    float u[32];
                    tmem_ld32_nowait(src + c, v);
                    tmem_ld32_nowait(src + 64 + c, u);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        if (!live || 64 * t.nt + c + 8 * e + 8 > mk::DFF) continue;
                        uint32_t wd[4];
#pragma unroll
                        for (int h = 0; h < 4; ++h) {
                            const int i = 8 * e + 2 * h;
                            // g * sigmoid(g) * u, rounded to fp16 (the product epilogue's arithmetic)
                            const float a = __fdividef(v[i], 1.f + __expf(-v[i])) * u[i];
                            const float b = __fdividef(v[i + 1], 1.f + __expf(-v[i + 1])) * u[i + 1];
                            wd[h] = pack_half2(a, b);
                        }
                        *reinterpret_cast<uint4*>(o + c + 8 * e) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
                    }
                    __syncwarp();
                }
            } else {
                float* o = EPI == kMkF32 ? p.qf + static_cast<long long>(r) * mk::QW + 128 * t.nt
                                         : p.part + (static_cast<long long>(t.z) * p.B + r) * mk::D + 128 * t.nt;
#pragma unroll 1
                for (int c = 0; c < 128; c += 32) {
                    tmem_ld32_nowait(src + c, v);
                    tmem_wait_ld();
                    if (live) {
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            *reinterpret_cast<float4*>(o + c + 4 * e) =
                                make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
                    }
                    __syncwarp();
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&pp.acc_empty[buf]);
            if (u == static_cast<int>(blockIdx.x) && warp == 4 && lane == 0) mk_stamp(p, kMkStampBase + 3 * gidx + 2);
        }
    }
}

// Rows of the residual stream, one warp per row (16 values per lane): x = base + the split
// partials in order, stored back when partials were added; then RMSNorm with weights w into
// fp16 out (or, for the final norm, the vocabulary head's [hi | lo | hi] fp16 rows and the
// row's position advanced).
__device__ __forceinline__ void mk_rows_phase(const MkParams& p, int mode, int ks, const float* w, __half* out) {
    // mode 0: x = E[tok] (embedding), 1: x += partials -> out, 2: x += partials -> final split
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float4 wv[4];  // the norm weights, loaded before the rows' data
#pragma unroll
    for (int k = 0; k < 4; ++k) wv[k] = *reinterpret_cast<const float4*>(w + 4 * (k * 32 + lane));
    for (int r = blockIdx.x * mk::kWarps + warp; r < p.B; r += gridDim.x * mk::kWarps) {
        float4 v[4];
        float* xr = p.x + static_cast<long long>(r) * mk::D;
        if (mode == 0) {
            const int tok = __ldcg(p.tok + r);
            const bool ok = tok < p.V;
            if (!ok && lane == 0) raise_error(p.err, kErrBadIndex);
            const float* er = p.E + static_cast<long long>(ok ? tok : 0) * mk::D;
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = *reinterpret_cast<const float4*>(er + 4 * (k * 32 + lane));
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = __ldcg(reinterpret_cast<const float4*>(xr + 4 * (k * 32 + lane)));
            for (int s = 0; s < ks; ++s) {
                const float* pr = p.part + (static_cast<long long>(s) * p.B + r) * mk::D;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float4 a = __ldcg(reinterpret_cast<const float4*>(pr + 4 * (k * 32 + lane)));
                    v[k].x += a.x;
                    v[k].y += a.y;
                    v[k].z += a.z;
                    v[k].w += a.w;
                }
            }
        }
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            *reinterpret_cast<float4*>(xr + 4 * (k * 32 + lane)) = v[k];
            ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
        }
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(mk::D) + p.eps);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int j = 4 * (k * 32 + lane);
            const float o0 = v[k].x * inv * wv[k].x, o1 = v[k].y * inv * wv[k].y, o2 = v[k].z * inv * wv[k].z,
                        o3 = v[k].w * inv * wv[k].w;
            if (mode != 2) {
                *reinterpret_cast<uint2*>(out + static_cast<long long>(r) * mk::D + j) = pack_h4(o0, o1, o2, o3);
            } else {
                __half* h3 = p.h3 + static_cast<long long>(r) * p.ld3;
                const float f[4] = {o0, o1, o2, o3};
                __half hi[4], lo[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    hi[e] = __float2half_rn(f[e]);
                    lo[e] = __float2half_rn(f[e] - __half2float(hi[e]));
                }
                const uint2 H = make_uint2(pack_half2(__half2float(hi[0]), __half2float(hi[1])),
                                           pack_half2(__half2float(hi[2]), __half2float(hi[3])));
                const uint2 Lo = make_uint2(pack_half2(__half2float(lo[0]), __half2float(lo[1])),
                                            pack_half2(__half2float(lo[2]), __half2float(lo[3])));
                *reinterpret_cast<uint2*>(h3 + j) = H;
                *reinterpret_cast<uint2*>(h3 + mk::D + j) = Lo;
                *reinterpret_cast<uint2*>(h3 + 2 * mk::D + j) = H;
            }
        }
        if (mode == 2 && lane == 0) p.pos[r] = __ldcg(p.pos + r) + 1;
    }
}

// Latent attention of layer l: one warp per (row, split) item; with several splits the
// last split of a row to finish merges the row (the others' partials are visible to it:
// each writer fences before its arrival, the merger after).
__device__ __forceinline__ void mk_attention_phase(const MkParams& p, int l, uint8_t* smem) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const __half* cache_l = p.cache + static_cast<long long>(l) * p.B * p.Sc * mk::KVW;
    const int items = p.B * p.ns;
    for (int it = blockIdx.x * mk::kWarps + warp; it < items; it += gridDim.x * mk::kWarps) {
        const int b = it / p.ns, sp = it - b * p.ns;
        // trace: CTA 0's warp 0 stamps its first item (start, queries ready, tiles done, merged)
        unsigned long long* st = (p.trace && blockIdx.x == 0 && warp == 0 && it == 0) ? p.trace + kMkAttnStamp + 4 * l
                                                                                        : nullptr;
        if (st && lane == 0) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(st[0]));
        decode_attention_item<mk::kAttnStages>(p.qf, cache_l, static_cast<long long>(p.Sc) * mk::KVW, p.pos, b, sp,
                                               p.ns, p.scale, p.ctx16, p.attn_part, p.cos_t, p.sin_t,
                                               smem + warp * dec::warp_smem<mk::kAttnStages>(), p.qs,
                                               st ? st + 1 : nullptr);
        if (p.ns > 1) {
            __threadfence();
            __syncwarp();
            int old = 0;
            if (lane == 0) old = atomicAdd(p.attn_cnt + b, 1);
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old == p.ns - 1) {
                __threadfence();
                decode_attention_merge_row(p.attn_part, p.ns, b, p.ctx16);
                if (lane == 0) atomicExch(p.attn_cnt + b, 0);
            }
        }
        if (st && lane == 0) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(st[3]));
        __syncwarp();
    }
    // the warps' generic shared-memory use ends before the next phase's TMA writes there
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mk_prefetch_layer(const MkParams& p, int l) {
    if (l < p.L && threadIdx.x == 32)
        for (int k = 0; k < 5; ++k) mk_prefetch_l2(p.wbase[l][k], p.wbytes[l][k]);
}

__global__ void __launch_bounds__(mk::kThreads, 1) decode_mk_kernel(const __grid_constant__ MkParams p) {
    extern __shared__ uint8_t mk_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(mk_smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + mk::kDataBytes);
    MkPipe pp;
    pp.ring = smem;
    pp.full = bars;
    pp.empty = bars + mk::kStages;
    pp.acc_full = bars + 2 * mk::kStages;
    pp.acc_empty = pp.acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pp.acc_empty + 2);
    int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);
    pp.s_abort = s_abort;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        for (int s = 0; s < mk::kStages; ++s) {
            mbar_init(&pp.full[s], 1);
            mbar_init(&pp.empty[s], 1);
        }
        mbar_init(&pp.acc_full[0], 1);
        mbar_init(&pp.acc_full[1], 1);
        mbar_init(&pp.acc_empty[0], 4);
        mbar_init(&pp.acc_empty[1], 4);
        fence_mbar_init();
        *s_abort = 0;
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, mk::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pp.tmem = *tmem_slot;

    int prod_it = 0, mma_it = 0, acc_j = 0;
    unsigned epoch = 0;
    int tk = 0;
    mk_trace(p, tk);
    if (threadIdx.x == 0) {
        prefetch_tmap(&p.a_h16);
        prefetch_tmap(&p.a_ctx16);
        prefetch_tmap(&p.a_h2);
        prefetch_tmap(&p.a_gated);
        for (int l = 0; l < p.L; ++l) {
            prefetch_tmap(&p.wa[l]);
            prefetch_tmap(&p.wf[l]);
            prefetch_tmap(&p.wo[l]);
            prefetch_tmap(&p.wgu[l]);
            prefetch_tmap(&p.wdown[l]);
        }
    }
    mk_prefetch_layer(p, 0);
    mk_prefetch_layer(p, 1);
    [&] {
        mk_rows_phase(p, 0, 0, p.attn_norm[0], p.h16);
        if (!mk_sync(p, epoch, s_abort)) return;
            mk_trace(p, tk);
        for (int l = 0; l < p.L; ++l) {
            if (l > 0) mk_prefetch_layer(p, l + 1);
            // the latent phase also computes the queries (h . Wf; 6 tiles of 192 columns)
            mk_gemm_phase<kMkLatent>(p, pp, &p.a_h16, &p.wa[l], 2 + mk::QW / mk::QR, mk::D / 64, 1, mk::D / 64, l,
                                     prod_it, mma_it, acc_j, 4 * l);
            if (!mk_sync(p, epoch, s_abort)) return;
            mk_trace(p, tk);
            mk_attention_phase(p, l, smem);
            if (!mk_sync(p, epoch, s_abort)) return;
            mk_trace(p, tk);
            mk_gemm_phase<kMkPartial>(p, pp, &p.a_ctx16, &p.wo[l], mk::D / 128, mk::HKV / 64, p.ks_o, p.per_o, l,
                                      prod_it, mma_it, acc_j, 4 * l + 1);
            if (!mk_sync(p, epoch, s_abort)) return;
            mk_trace(p, tk);
            mk_rows_phase(p, 1, p.ks_o, p.ffn_norm[l], p.h2);
            if (!mk_sync(p, epoch, s_abort)) return;
            mk_trace(p, tk);
            mk_gemm_phase<kMkGlu>(p, pp, &p.a_h2, &p.wgu[l], (mk::DFF + 63) / 64, mk::D / 64, 1, mk::D / 64, l, prod_it,
                                  mma_it, acc_j, 4 * l + 2);
            if (!mk_sync(p, epoch, s_abort)) return;
            mk_trace(p, tk);
            mk_gemm_phase<kMkPartial>(p, pp, &p.a_gated, &p.wdown[l], mk::D / 128, (mk::DFF + 63) / 64, p.ks_d, p.per_d,
                                      l, prod_it, mma_it, acc_j, 4 * l + 3);
            if (!mk_sync(p, epoch, s_abort)) return;
            mk_trace(p, tk);
            const bool last = l + 1 == p.L;
            mk_rows_phase(p, last ? 2 : 1, p.ks_d, last ? p.final_norm : p.attn_norm[l + 1], p.h16);
            if (last) break;
            if (!mk_sync(p, epoch, s_abort)) return;
            mk_trace(p, tk);
        }
    }();
    __syncthreads();
    mk_trace(p, tk);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(pp.tmem, mk::kTmemCols);
    }
}

}  // namespace mm
