"""Rollout decode throughput and the latent decode-attention kernel alone.

Decode mode (default) runs the batched rollout of the 35.8M model without its log-prob
pass: B random prompts of --prompt ids, prefill, then --new tokens per row (greedy or
temperature sampling), and reports the decode phase (all steps after the first token,
which comes from the prefill logits) as tokens/s and against the HBM roofline of
2·P weight bytes (fp16) plus B·ctx·2880 cache bytes (latent 128 + rope 16 in fp16 over 10
layers) per step, ctx averaged over the steps. Decode-only after long prompts is
``--batch 1,16,64 --prompt 1024 --new 128``; the full GRPO step's rollout decode is
``--batch 2048 --prompt 128 --new 256``.

Attention mode times one launch of the split latent attention (mm_cuda_decode_attention)
over a synthetic fp16 cache of --ctx positions per row:

    python -m cpp_inference_train_engine_b200.decode_bench --attention --batch 2048 --ctx 256

Sample mode times the exact sampler (mm_cuda_sample) on synthetic Gaussian logits of
standard deviation --logit-sd over the 16384-word vocabulary, per launch:

    python -m cpp_inference_train_engine_b200.decode_bench --sample --batch 2048 --temperature 1.0
"""
import argparse
import json


def _peak_hbm():
    import os
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def attention(args):
    import torch

    import cpp_inference_train_engine_b200 as E
    H, KV, W = 8, 128, 144
    ex = E.CudaExecution(E.MLA36M)
    g = torch.Generator(device="cuda").manual_seed(1)
    for B in args.batch:
        Sc = args.ctx
        q = torch.randn(B, H, W, device="cuda", generator=g)
        cache = (torch.randn(B, Sc, W, device="cuda", generator=g) * 0.5).half()
        pos = torch.full((B,), args.ctx - 1, device="cuda", dtype=torch.int32)
        out = torch.empty(B, H * KV, device="cuda", dtype=torch.half)
        splits = args.splits or (1 if B >= 1184 else max(1, min((1184 + B - 1) // B, (args.ctx + 63) // 64, 16)))
        torch.cuda.synchronize()
        # device time of the kernel launches alone, from the library's per-launch events (each
        # call first waits for all earlier device work, which a pair of events around the
        # call would count)
        for _ in range(args.warmup):
            ex.decode_attention(q.data_ptr(), cache.data_ptr(), Sc * W, pos.data_ptr(), B, splits, 0.125,
                                out.data_ptr())
        ex.profile(1)
        for _ in range(args.iters):
            ex.decode_attention(q.data_ptr(), cache.data_ptr(), Sc * W, pos.data_ptr(), B, splits, 0.125,
                                out.data_ptr())
        tot, calls, _ = ex.profile(0)["k_decode_attention"]
        ms = tot / max(calls, 1)
        byts = B * args.ctx * W * 2 + B * H * W * 4 + B * H * KV * 2
        peak, src = _peak_hbm()
        print(json.dumps({"kernel": "decode_attention", "batch": B, "ctx": args.ctx, "splits": splits,
                          "us": ms * 1e3, "gbs": byts / (ms / 1e3) / 1e9,
                          "hbm_frac": byts / (ms / 1e3) / 1e9 / peak, "peak_source": src}))
    ex.close()


def sample(args):
    import numpy as np

    import cpp_inference_train_engine_b200 as E
    ex = E.CudaExecution(E.MLA36M)
    rng = np.random.default_rng(0)
    V = E.MLA36M.vocab_size
    for B in args.batch:
        logits = (rng.normal(size=(B, V)) * args.logit_sd).astype(np.float32)
        seeds = rng.integers(0, 2 ** 63, B).astype(np.uint64)
        draws = rng.integers(0, 300, B).astype(np.int32)
        for temp in args.temperature:
            for _ in range(args.warmup):
                ex.sample(logits, temp, seeds, draws)
            ex.profile(1)
            for _ in range(args.iters):
                ex.sample(logits, temp, seeds, draws)
            ms, n, _ = ex.profile(0)["k_sample"]
            peak, src = _peak_hbm()
            us = ms / max(n, 1) * 1e3
            print(json.dumps({"kernel": "sample", "batch": B, "vocab": V, "temperature": temp,
                              "logit_sd": args.logit_sd, "us": us,
                              "hbm_frac": 4.0 * B * V / (us / 1e6) / 1e9 / peak, "peak_source": src}))
    ex.close()


def decode(args):
    import numpy as np

    import cpp_inference_train_engine_b200 as E
    from cpp_inference_train_engine_b200.config import MLA1B, MLA36M, ModelConfig
    from cpp_inference_train_engine_b200.rng import Rng

    # MLA1B's attention shapes (16 heads, kv rank 512, rope 32) on 2 layers of width 256: a
    # small device footprint for single-kernel captures of its decode attention
    MLA1B_ATTN = ModelConfig(vocab_size=2048, max_sequence_length=2048, n_layers=2, d_model=256, n_heads=16,
                             head_dim_nope=96, head_dim_rope=32, head_dim_value=128, q_lora_rank=192,
                             kv_lora_rank=512, d_ff=512)

    cfg = {"mla36m": MLA36M, "mla1b": MLA1B, "mla1b-attn": MLA1B_ATTN}[args.model]
    P = E.parameter_count(cfg)
    kv_bytes = 2.0 * (cfg.kv_lora_rank + cfg.head_dim_rope) * cfg.n_layers  # per row and position
    ex = E.make_execution(cfg, E.init_params(cfg, 0))
    peak, src = _peak_hbm()
    for B in args.batch:
        r = Rng(2)
        prompts = np.array([[r.bounded(cfg.vocab_size) for _ in range(args.prompt)] for _ in range(B)],
                           np.uint16)
        r1 = Rng(1)
        seeds = np.array([r1.next() for _ in range(B)], np.uint64)
        S = args.prompt + args.new
        for temp in args.temperature:
            if args.trace:
                ex.decode_trace(1)
            for it in range(args.warmup + 1):
                if it == args.warmup:
                    ex.profile(1)
                ex.rollout(prompts, args.new, S, seeds, temp, with_batches=False)
            if args.gemm_shapes:
                for row in ex.gemm_shapes()[:20]:
                    print(json.dumps({"gemm_shape": row["shape"], "ms": row["ms"], "calls": row["calls"],
                                      "tflops": row["tflops"]}))
            prof = ex.profile(0)
            if args.gemm_shapes:
                print(json.dumps({"mode": "phases", "batch": B,
                                  "ms": {k: round(v[0], 3) for k, v in prof.items() if v[0]}}))
            if args.trace:
                raw = ex.decode_trace_raw()
                ph = ex.decode_trace(0)
                # the fused step's four products per layer (the latent phase also makes the
                # queries) and its seven phases per layer
                kinds = ["wa", "wo", "wgu", "wdown"]
                inner = {k: [0.0, 0.0] for k in kinds}
                for g in range(4 * cfg.n_layers):
                    a, b, c = raw[128 + 3 * g: 131 + 3 * g]
                    if a > 0 and b > a and c > b:
                        inner[kinds[g % 4]][0] += (b - a) / 1e3
                        inner[kinds[g % 4]][1] += (c - b) / 1e3
                # the attention phases: CTA 0 warp 0's first item per layer
                att = [0.0, 0.0, 0.0]
                for l in range(cfg.n_layers):
                    st = raw[256 + 4 * l: 260 + 4 * l]
                    if len(st) == 4 and all(x > 0 for x in st) and st[0] <= st[1] <= st[2] <= st[3]:
                        for k in range(3):
                            att[k] += (st[k + 1] - st[k]) / 1e3
                print(json.dumps({"mode": "decode_trace_attention", "batch": B,
                                  "us_over_layers": {"to_queries_ready": round(att[0], 2),
                                                     "cache_tiles": round(att[1], 2),
                                                     "partial_and_merge": round(att[2], 2)}}))
                print(json.dumps({"mode": "decode_trace_inner", "batch": B,
                                  "load_mma_us": {k: round(v[0], 2) for k, v in inner.items()},
                                  "epilogue_us": {k: round(v[1], 2) for k, v in inner.items()}}))
                names = ["embed"] + [f"{n}{l}" for l in range(cfg.n_layers) for n in
                                     ("wa", "attn", "wo", "norm2", "wgu", "wdown", "norm1")]
                per = {}
                for n, us in zip(names, ph):
                    key = n.rstrip("0123456789")
                    per[key] = per.get(key, 0.0) + us
                print(json.dumps({"mode": "decode_trace", "batch": B, "phases": len(ph), "total_us": sum(ph),
                                  "by_kind_us": {k: round(v, 2) for k, v in per.items()},
                                  "layer0_us": [round(x, 2) for x in ph[1:8]]}))
            ms = prof["decode"][0] + prof["sample"][0]
            steps = args.new - 1
            ctx = args.prompt + (args.new - 1) / 2.0  # mean positions attended per step
            byts = steps * (2.0 * P + B * ctx * kv_bytes)
            print(json.dumps({"mode": "decode", "batch": B, "prompt": args.prompt, "new": args.new,
                              "temperature": temp, "decode_ms": ms, "ms_per_step": ms / steps,
                              "tok_s": B * steps / (ms / 1e3),
                              "hbm_roofline_frac": byts / (ms / 1e3) / 1e9 / peak, "peak_source": src,
                              "prefill_ms": prof["prefill"][0],
                              # event-timed launches only (eager steps; graph replays are not)
                              "attention": {"ms": prof["k_decode_attention"][0],
                                            "launches": prof["k_decode_attention"][1],
                                            "gbs": prof["k_decode_attention"][2] / max(prof["k_decode_attention"][0], 1e-9) / 1e6}}))
    ex.close()


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--attention", action="store_true")
    ap.add_argument("--sample", action="store_true")
    ap.add_argument("--logit-sd", type=float, default=1.0)
    ap.add_argument("--batch", type=lambda s: [int(x) for x in s.split(",")], default=[1, 16, 64])
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--new", type=int, default=128)
    ap.add_argument("--temperature", type=lambda s: [float(x) for x in s.split(",")], default=[0.0, 1.0])
    ap.add_argument("--ctx", type=int, default=256)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--model", default="mla36m", choices=["mla36m", "mla1b", "mla1b-attn"])
    ap.add_argument("--gemm-shapes", action="store_true", help="per-shape GEMM device time of the timed run")
    ap.add_argument("--trace", action="store_true",
                    help="print the fused decode step's per-phase times (device global timer)")
    args = ap.parse_args(argv)
    if args.attention:
        attention(args)
    elif args.sample:
        sample(args)
    else:
        decode(args)


if __name__ == "__main__":
    main()
