/*
 * mm_cuda_kernels.h -- kernel-level entry points of the sm_100a backend on DEVICE pointers,
 * for the parity tests and the benchmark's timing. They have no counterpart in the
 * reference's Execution interface (the reference's GPU path is MPSGraph programs,
 * src/backends/mps_backend.mm:1597-1738); they expose single kernels of the same path.
 * Each entry first waits for all work already submitted to the device, so inputs written on
 * any stream are complete before they are read.
 */
#ifndef MM_CUDA_KERNELS_H
#define MM_CUDA_KERNELS_H

#include <stdint.h>

#include "mm_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Tensor-core GEMM: out[M][N] = alpha * A * B (+ residual), fp16 (or bf16) operands,
 * fp32 accumulation. A is [M][K] rows (a_mn = 0) or [K][M] rows (a_mn = 1); B is [N][K]
 * rows (b_mn = 0) or [K][N] rows (b_mn = 1); pitches in elements, multiples of 8.
 * out_kind: 0 fp32 store, 1 fp32 accumulate (+=), 2 fp16 store, 3 bf16 store.
 * residual (fp32 [M][ldr], may be NULL) is added for out_kind 0. */
int mm_cuda_gemm_f16(mm_cuda_ctx* ctx, int M, int N, int K, const void* a, int64_t lda, int a_mn,
                     const void* b, int64_t ldb, int b_mn, void* out, int64_t ldc, int out_kind,
                     float alpha, const float* residual, int64_t ldr, int bf16);

/* Absorbed latent-cache decode attention (CpuDecoder::decode, src/infer/inference.cpp:116-153)
 * for the 8-head [128 latent | 16 rope] cache of the 35.8M model, on device pointers:
 *   q      fp32 [batch][8][144]  absorbed query then rotated rope query, per head
 *   cache  fp16 rows of 144, row b starts at b * cache_seq_stride elements
 *   pos    int32 [batch]: positions 0..pos[b] (inclusive) are attended
 *   out    fp16 [batch][8 * 128] latent context per head
 * splits in [1, 16] divides each row's context over that many CTAs; the partials live in
 * scratch owned by the context. Runs on the context's stream and returns when done. */
int mm_cuda_decode_attention(mm_cuda_ctx* ctx, const float* q, const void* cache,
                             int64_t cache_seq_stride, const int32_t* pos, int batch, int splits,
                             float scale, void* out);

/* The same decode attention without any allocation, for callers that may not allocate
 * device memory: a serving process that hands all device memory to its own pool at
 * start-up and forbids allocations afterwards, or a plugin host that lends device buffers
 * for inputs and outputs only. No counterpart in the reference (its decode runs inside a
 * CpuDecoder or an MPSGraph program).
 *
 * Arguments mean what they mean for mm_cuda_decode_attention; `stream` is the caller's
 * cudaStream_t (NULL = the legacy default stream) and the call returns when that stream
 * has finished the work. No context, cudaMalloc, cudaFree or allocating library routine is
 * involved: the split partials live in one static device array of 256 (row, split) slots
 * (1,064,960 bytes) that every GPU loading this library holds until the process exits.
 *   - The first call with splits > 1 on a device resolves that array's device address
 *     (cudaGetSymbolAddress, with the device current) and caches it for the process. Under
 *     lazy module loading that first call is also when the driver loads this library's
 *     device code and the array, which allocates: make it at start-up, before any stream
 *     capture, like any other set-up. After cudaDeviceReset the cached address is stale:
 *     a process that resets a device must be restarted before calling this again.
 *   - Launch failures are read from the launches themselves; an error an earlier call left
 *     pending is neither reported nor cleared here.
 *   - Returns MM_INVALID_ARGUMENT when splits > 1 and batch * splits > 256 (the array's
 *     capacity), for splits outside [1, 16], a null pointer or a row stride below 144;
 *     MM_GPU_ERROR when a CUDA call fails.
 *   - Every call shares the array and it keeps the last call's partials (each call writes
 *     every slot it reads, so nothing needs clearing). Calls that overlap on the GPU
 *     (different streams, or threads racing on one device) race on the array. */
int mm_decode_attention_noalloc(const float* q, const void* cache, int64_t cache_seq_stride,
                                const int32_t* pos, int batch, int splits, float scale, void* out,
                                void* stream);

/* Device time (CUDA events on the context's stream, resolved at this call) accumulated
 * since the last reset, 16 entries each of ms, calls and algorithmic work:
 *   0-7  phases: prefill, decode, sample, logprob, backward, adamw, allreduce, prep;
 *   8-15 kernel classes: gemm (flops), decode attention (bytes), flash forward (flops),
 *        flash backward (flops), sampler (bytes), log-softmax (bytes), adamw (bytes), other.
 * enable: 1 start/reset, 0 stop/reset, -1 read only. Any pointer may be NULL. */
int mm_cuda_profile(mm_cuda_ctx* ctx, int enable, double* ms, int64_t* calls, double* work);

/* While profiling: one text line per GEMM launch shape ("M.. N.. K.. a.. b.. bn.. out..
 * calls= ms= tflops="), NUL-terminated into buf. Returns the full length, or -(1 + code). */
int64_t mm_cuda_profile_gemm_shapes(mm_cuda_ctx* ctx, char* buf, int64_t cap);

/* Phase trace of the fused rollout decode step (no reference counterpart; the reference
 * logs per-update counters only, execution.hpp:25-27): while enabled (enable = 1; 0 turns it
 * off, -1 leaves it) every fused step records the device global timer (ns) at its start,
 * after each of its grid barriers and at its end. out_ns (cap entries) receives the last
 * step's record; *count the entries copied. Tracing adds one timer read per barrier. */
int mm_cuda_decode_trace(mm_cuda_ctx* ctx, int enable, uint64_t* out_ns, int cap, int* count);

/* The context's CUDA stream (cudaStream_t), for events recorded by a caller. */
int mm_cuda_stream(mm_cuda_ctx* ctx, void** stream);

/* Self-test of the bounded-wait failure path (no reference counterpart; the reference's
 * backends report device failures as gpu_error and mark the execution unusable,
 * mps_backend.mm:1050-1065). Launches one kernel that waits on an mbarrier no thread
 * arrives at for at most `polls` polls (1 <= polls <= 2^22), after which it records a wait
 * timeout in the context's device error word and returns: no trap, no fault. The call
 * returns MM_GPU_ERROR ("device wait timed out") and the context is unusable afterwards,
 * exactly as after a GEMM whose pipeline stalled. */
int mm_cuda_selftest_wait_timeout(mm_cuda_ctx* ctx, uint32_t polls);

/* Measurement entry (no reference counterpart): the product of mm_cuda_gemm_f16 (fp32
 * store, accumulate, fp16 or bf16 output, no residual) launched `reps` times back to back
 * inside one CUDA graph, so that consecutive launches overlap as in the engine's own
 * passes; *ms_per_launch receives the device time of one replay divided by reps.
 * out_kind 4 and 5 time the vocabulary head's two epilogues instead: 4 the forward's
 * row log-sum-exp partials and target logits with no store (fp32 product; `out` unused but
 * non-NULL), 5 the backward's weighted-NLL gradient of the recomputed logits into fp16 `out`
 * (row log-sum-exp 0, coefficient 1, targets row % N: the arithmetic, not a gradient). */
int mm_cuda_bench_gemm(mm_cuda_ctx* ctx, int reps, int M, int N, int K, const void* a, int64_t lda,
                       int a_mn, const void* b, int64_t ldb, int b_mn, void* out, int64_t ldc,
                       int out_kind, float* ms_per_launch);

#ifdef __cplusplus
}
#endif
#endif /* MM_CUDA_KERNELS_H */
