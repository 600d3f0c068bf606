"""Microbenchmark of the tcgen05 GEMM at one shape through the kernel-level entry point
(mm_cuda_gemm_f16 in include/mm_cuda_kernels.h).

Device time per launch: by default `--iters` launches are captured in one CUDA graph and
replayed back to back (mm_cuda_bench_gemm), as the engine's passes issue them, so neither
host launch cost nor a synchronisation per call is counted. `--eager` instead times each
call of mm_cuda_gemm_f16 with the library's CUDA-event profile (events around every
launch; each call also waits for completion, so short products read long).
The default shape is the vocabulary head of one 32,640-token teacher-forced chunk:
[T, 3d] x [V, 3d]^T with K = 3 * 512 (the fp32-accurate three-term split), fp32 output.

    python -m cpp_inference_train_engine_b200.gemm_bench --shape 32640,16384,1536
"""
import argparse
import json


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--shape", default="32640,16384,1536", help="M,N,K")
    ap.add_argument("--a-mn", type=int, default=0, help="A stored [K][M] (1) or [M][K] (0)")
    ap.add_argument("--b-mn", type=int, default=0, help="B stored [K][N] (1) or [N][K] (0)")
    ap.add_argument("--out", default="f32", choices=["f32", "f16", "acc", "lse", "vgrad"],
                    help="lse: the vocabulary head's log-sum-exp epilogue, no store; vgrad: its "
                         "backward's gradient epilogue, fp16 out (graph mode only)")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--eager", action="store_true", help="time each eager call instead")
    args = ap.parse_args(argv)

    import torch

    import cpp_inference_train_engine_b200 as E

    M, N, K = (int(v) for v in args.shape.split(","))
    kind = {"f32": 0, "acc": 1, "f16": 2, "lse": 4, "vgrad": 5}[args.out]
    ex = E.CudaExecution(E.TINY)
    g = torch.Generator(device="cuda").manual_seed(M + 3 * N + 7 * K)
    pad = (K + 7) // 8 * 8
    A = (torch.randn(K, (M + 7) // 8 * 8, device="cuda", generator=g) if args.a_mn
         else torch.randn(M, pad, device="cuda", generator=g)).half()
    B = (torch.randn(K, (N + 7) // 8 * 8, device="cuda", generator=g) if args.b_mn
         else torch.randn(N, pad, device="cuda", generator=g)).half()
    C = torch.zeros(M, N, device="cuda", dtype=torch.half if kind in (2, 5) else torch.float32)
    torch.cuda.synchronize()

    def run():
        ex.gemm(M, N, K, A.data_ptr(), A.shape[1], args.a_mn, B.data_ptr(), B.shape[1],
                args.b_mn, C.data_ptr(), N, kind)

    if not args.eager:
        ms = ex.bench_gemm(args.iters, M, N, K, A.data_ptr(), A.shape[1], args.a_mn, B.data_ptr(),
                           B.shape[1], args.b_mn, C.data_ptr(), N, kind)
        print(json.dumps({"shape": [M, N, K], "a_mn": args.a_mn, "b_mn": args.b_mn, "out": args.out,
                          "graph_launches": args.iters, "ms_per_launch": ms,
                          "tflops": 2.0 * M * N * K / (ms / 1e3) / 1e12}))
        ex.close()
        return
    for _ in range(args.warmup):
        run()
    ex.profile(1)
    for _ in range(args.iters):
        run()
    prof = ex.profile(0)
    ms, launches, flops = prof["k_gemm"]
    line = {"shape": [M, N, K], "a_mn": args.a_mn, "b_mn": args.b_mn, "out": args.out,
            "launches": launches, "ms_per_launch": ms / max(launches, 1),
            "tflops": flops / (ms / 1e3) / 1e12 if ms else None}
    print(json.dumps(line))
    ex.close()


if __name__ == "__main__":
    main()
