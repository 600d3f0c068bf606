#!/usr/bin/env python3
"""Benchmark: one full online GRPO step of the 35.8M-parameter MLA model:
256 prompts x group 8 = 2048 rollouts, prompt 128 tokens, 256 new tokens at temperature 1
(sequence 384), Bernoulli(0.3) rewards, clip 0.2, KL 0.04, AdamW lr 1e-5 on fp32 master
weights with fp16 tensor-core compute. Random-init weights (seed 0) and synthetic prompt ids;
the frozen reference model equals the initial policy.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = rollout (prefill + 256 batched decode steps with on-device sampling + the
old-policy log-prob pass) and the GRPO update (reference-model log-probs, policy forward +
fused objective + backward, gradient all-reduce, AdamW). Rollouts are sharded over ranks
(whole groups per rank, no collective on the rollout path); gradients are all-reduced.

Printed once by rank 0: a JSON line with value = generated rollout tokens per second of
device step time (whole job), e2e = the same through the public API with host buffers,
ms_per_step, roofline of the dominant kernel class, the reference CPU baseline, clocks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GRPO rollout tok/s + step time, 35.8M MLA, 1/2/4/8 B200; % HBM roofline"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--prompts", type=int, default=256, help="prompts per step (whole job)")
    ap.add_argument("--group", type=int, default=8)
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--new-tokens", type=int, default=256)
    ap.add_argument("--cpu-rollouts", type=int, default=2,
                    help="rollouts in the bounded CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gemm-shapes", action="store_true",
                    help="print per-shape GEMM device time to stderr")
    return ap.parse_args()


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[3 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return {"hbm_gbs": j["hbm_gbs"], "tflops": j["bf16_tflops_sustained"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "source": "fallback"}


# ---------------------------------------------------------------------------- CPU baseline
def cpu_baseline(args, steps=1):
    """The reference engine's own CPU path (oracle/_ref, OpenBLAS on all host cores) on a
    bounded sample of the same workload: `cpu_rollouts` rollouts of the same prompt shape
    and length, then their GRPO update. Returns tokens/s per step."""
    from cpp_inference_train_engine_b200.config import MLA36M, AdamWConfig
    from cpp_inference_train_engine_b200.rng import grpo_workload
    from oracle import ref
    if not ref.available():
        return None, "oracle/_ref not built"
    n = args.cpu_rollouts
    prompts, seeds, rewards = grpo_workload(1, n, args.prompt_len, MLA36M.vocab_size, 0.3)
    rewards[0], rewards[-1] = 1.0, 0.0
    seq = args.prompt_len + args.new_tokens
    pol = ref.Session(MLA36M, 0, optimizer=AdamWConfig().as_list())
    refm = ref.Session(MLA36M, 0)
    rates = []
    for _ in range(steps):
        t0 = time.perf_counter()
        rolls = [pol.rollout(prompts[i], args.new_tokens, seq, MLA36M.eos_id, MLA36M.pad_id,
                             int(seeds[i])) for i in range(n)]
        stack = lambda k: np.stack([r[k] for r in rolls])
        ref.grpo_update(pol, refm, n, stack("input"), stack("target"), stack("mask"),
                        stack("old_lp"), rewards, 0.2, 0.04, 1e-5)
        dt = time.perf_counter() - t0
        rates.append(sum(len(r["tokens"]) for r in rolls) / dt)
    sample = (f"{n} rollouts (prompt {args.prompt_len}, {args.new_tokens} new tokens, S={seq}) "
              f"+ their GRPO update (group {n}), reference CPU build, OpenBLAS")
    return {"value": statistics.median(rates), "unit": "tok/s", "cores": os.cpu_count(),
            "kind": "reference", "sample": sample}, None


def run_reference(args, rank, world):
    if rank != 0:
        return
    for _ in range(max(args.warmup, 0)):
        pass  # the bounded sample has no warm-up state to build; W is honoured by step count
    res, err = cpu_baseline(args, steps=args.steps)
    if res is None:
        print(json.dumps({"impl": "reference", "unavailable": err}))
        return
    line = {"metric": METRIC, "value": res["value"], "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "impl": "reference",
            "higher_is_better": True, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args, world),
            "cpu_baseline": res,
            "e2e": {"value": res["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def workload_config(args, world):
    n = args.prompts * args.group
    return {"workload": "grpo_step_mla36m", "rollouts": n, "prompts": args.prompts,
            "group": args.group, "prompt_len": args.prompt_len, "new_tokens": args.new_tokens,
            "sequence": args.prompt_len + args.new_tokens, "temperature": 1.0,
            "reward": "bernoulli(0.3)", "clip": 0.2, "kl": 0.04, "lr": 1e-5,
            "parallelism": f"dp{world}", "l2": "inputs larger than L2 (cache 2.3 GB, logits)"}


# ---------------------------------------------------------------------------- ours
def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    if args.impl == "reference":
        run_reference(args, rank, world)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return

    import torch

    import cpp_inference_train_engine_b200 as E
    from cpp_inference_train_engine_b200 import distributed as D
    from cpp_inference_train_engine_b200.config import MLA36M, AdamWConfig
    from cpp_inference_train_engine_b200.rng import grpo_workload

    cfg = MLA36M
    n_total = args.prompts * args.group
    try:
        sl = D.rollout_shard(n_total, args.group, rank, world)
    except ValueError as e:
        raise SystemExit(str(e))
    seq = args.prompt_len + args.new_tokens
    prompts, seeds, rewards = grpo_workload(args.prompts, args.group, args.prompt_len,
                                            cfg.vocab_size, 0.3)
    prompts, seeds, rewards = prompts[sl].copy(), seeds[sl].copy(), rewards[sl].copy()

    W = E.init_params(cfg, 0)
    pol = E.make_execution(cfg, W, optimizer=AdamWConfig(), device=local)
    refm = E.make_execution(cfg, W, device=local)
    if world > 1:
        D.init_comm(pol, rank, world)
    stream = torch.cuda.ExternalStream(pol.stream, device=local)

    def one_step(step_idx):
        # The rollout seeds advance per update like the trainer's Rng(seed) stream.
        with np.errstate(over="ignore"):  # arithmetic mod 2^64 is intended
            s = (seeds + np.uint64(step_idx) * np.uint64(0x9E3779B97F4A7C15)).astype(np.uint64)
        r = pol.rollout(prompts, args.new_tokens, seq, s, 1.0)
        out = pol.grpo_step(refm, r["input"], r["target"], r["mask"], r["old_lp"], rewards,
                            args.group, n_total=n_total, clip=0.2, klc=0.04, learning_rate=1e-5)
        return r, out

    def barrier():
        torch.cuda.synchronize(local)
        if dist:
            dist.barrier()

    for i in range(args.warmup):
        one_step(i)
    barrier()
    pol.profile(1)
    refm.profile(1)
    launches0 = pol.kernel_launches + refm.kernel_launches
    toks = 0
    h2d = d2h = 0
    results = []
    with ClockSampler(local) as clocks:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        barrier()
        # A profiler started with --profile-from-start off sees only the timed steps.
        torch.cuda.profiler.start()
        start.record(stream)
        for i in range(args.steps):
            r, out = one_step(args.warmup + i)
            results.append(out)
            toks += int(r["lengths"].sum())
            # host<->device traffic of the public calls: prompts + seeds in, tokens, lengths,
            # batches and old log-probs out; batches, old log-probs and rewards back in.
            h2d += prompts.nbytes + seeds.nbytes + r["input"].nbytes * 2 + r["mask"].nbytes * 2 + \
                rewards.nbytes
            d2h += r["tokens"].nbytes + r["lengths"].nbytes + r["old_lp"].nbytes
        end.record(stream)
        barrier()
        torch.cuda.profiler.stop()
    e2e_ms = start.elapsed_time(end)
    if args.gemm_shapes and rank == 0:
        for name, ctx in (("policy", pol), ("reference", refm)):
            for row in ctx.gemm_shapes()[:25]:
                print(json.dumps({"gemm_shape": row["shape"], "ctx": name,
                                  "ms_per_step": round(row["ms"] / args.steps, 3),
                                  "calls_per_step": row["calls"] // args.steps,
                                  "tflops": row["tflops"]}), file=sys.stderr)
    prof_p = pol.profile(0)
    prof_r = refm.profile(0)
    launches = pol.kernel_launches + refm.kernel_launches - launches0
    dev_ms = sum(prof_p[k][0] for k in ("prefill", "decode", "sample", "logprob", "backward",
                                        "adamw", "allreduce")) + prof_r["logprob"][0]
    if dist:
        t = torch.tensor([e2e_ms, dev_ms, float(toks)], device=f"cuda:{local}", dtype=torch.float64)
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = t.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        e2e_ms, dev_ms, toks = float(mx[0]), float(mx[1]), int(sm[2])
    if rank == 0:
        pk = peaks()
        kern = {}
        for k in ("k_gemm", "k_decode_attention", "k_flash_fwd", "k_flash_bwd", "k_sample",
                  "k_logsoftmax", "k_adamw"):
            ms = prof_p[k][0] + prof_r[k][0]
            n = prof_p[k][1] + prof_r[k][1]
            work = prof_p[k][2] + prof_r[k][2]
            kern[k] = {"ms": ms, "launches": n, "work": work}
        top = max(kern, key=lambda k: kern[k]["ms"])
        tensor = top in ("k_gemm", "k_flash_fwd", "k_flash_bwd")
        sec = kern[top]["ms"] / 1e3
        achieved = (kern[top]["work"] / sec / 1e12) if tensor else (kern[top]["work"] / sec / 1e9)
        peak = pk["tflops"] if tensor else pk["hbm_gbs"]
        roofline = {"kernel": top, "bound": "tensor" if tensor else "hbm",
                    "achieved": achieved, "peak": peak, "unit": "TFLOP/s" if tensor else "GB/s",
                    "frac": achieved / peak, "peak_source": pk["source"] + " (sustained)",
                    "launches": kern[top]["launches"],
                    "avg_launch_us": 1e3 * kern[top]["ms"] / max(kern[top]["launches"], 1),
                    "traffic": None}
        phases = {k: round(prof_p[k][0] / args.steps, 3) for k in
                  ("prefill", "decode", "sample", "logprob", "backward", "adamw", "allreduce")}
        phases["reference_logprob"] = round(prof_r["logprob"][0] / args.steps, 3)
        decode_ms = (prof_p["decode"][0] + prof_p["sample"][0] + prof_p["prefill"][0]) / args.steps
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu, _ = cpu_baseline(args, steps=1)
        line = {
            "metric": METRIC, "value": toks / (dev_ms / 1e3), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp16 tensor-core compute, fp32 master/accumulate", "data": "synthetic",
            "config": workload_config(args, world),
            "e2e": {"value": toks / (e2e_ms / 1e3), "unit": "tok/s",
                    "ms_per_step": e2e_ms / args.steps,
                    "h2d_bytes_per_step": h2d // args.steps, "d2h_bytes_per_step": d2h // args.steps},
            "rollout_tokens_per_step": toks // args.steps,
            "rollout_decode_tok_s": toks / (decode_ms * args.steps / 1e3) if decode_ms else None,
            "phases_ms_per_step": phases,
            "kernels": {k: {"ms_per_step": round(v["ms"] / args.steps, 3),
                            "launches_per_step": v["launches"] // args.steps} for k, v in kern.items()},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "grpo": {"loss": results[-1]["loss"], "kl": results[-1]["kl"],
                     "grad_norm": results[-1]["grad_norm"], "skipped": results[-1]["skipped"]},
        }
        print(json.dumps(line))
    pol.close()
    refm.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
