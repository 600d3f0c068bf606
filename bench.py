#!/usr/bin/env python3
"""Benchmark: one full online GRPO step of the 35.8M-parameter MLA model: 256 prompts x
group 8 = 2048 rollouts, prompt 128 tokens, 256 new tokens at temperature 1 (sequence 384),
Bernoulli(0.3) rewards, clip 0.2, KL 0.04, AdamW lr 1e-5 on fp32 master weights with fp16
tensor-core compute. Random-init weights (seed 0) and synthetic prompt ids; the frozen
reference model equals the initial policy.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --workload mla1b [--gpus N] ...

--workload mla1b runs the scaled model instead (24 blocks, width 2048, 16 heads, query rank
768, kv rank 512, SwiGLU 5632, tied 32,768-token vocabulary, 1.14 B parameters): 128 prompts
x group 16 = 2048 rollouts, prompt 512, 1536 new tokens (context 2048), N(0, 1) rewards. It
has no CPU baseline (the reference's CPU path would take days per step) and no fixed-input
check by default.

One step = rollout (prefill + 256 batched decode steps with on-device sampling + the
old-policy log-prob pass) and the GRPO update (reference-model log-probs, policy forward +
fused objective + backward, gradient all-reduce, AdamW). Rollouts are sharded over ranks
(whole groups per rank, no collective on the rollout path); gradients are all-reduced.

Printed once by rank 0: a JSON line with value = generated rollout tokens per second of
device step time (whole job), e2e = the same through the public API with host buffers,
ms_per_step, the roofline of the dominant kernel class (algorithmic FLOPs) and of the decode
phase (algorithmic HBM bytes), a fixed-input GRPO update whose loss / grad norm must not
depend on the rank count, the reference CPU baseline, clocks.

--impl reference times the reference engine's own CPU path (oracle/_ref, OpenBLAS on every
host core) on a bounded sample of the same workload; only rank 0 works, and it touches no GPU.
"""
import os
import sys


def _host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


if "reference" in sys.argv[1:] or "--impl=reference" in sys.argv[1:]:
    # Before numpy (and the OpenBLAS it bundles, which the reference build calls) loads: a
    # launcher that set OMP_NUM_THREADS=1 for its workers must not leave the CPU baseline on
    # one thread.
    os.environ["OPENBLAS_NUM_THREADS"] = str(_host_threads())
    os.environ["OMP_NUM_THREADS"] = str(_host_threads())

import argparse  # noqa: E402
import json  # noqa: E402
import statistics  # noqa: E402
import subprocess  # noqa: E402
import threading  # noqa: E402
import time  # noqa: E402

import numpy as np  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GRPO rollout tok/s + step time, 35.8M MLA, 1/2/4/8 B200; % HBM roofline"
METRIC_MLA1B = "GRPO rollout tok/s + step time, scaled 1.14B MLA (context 2048), 1/2/4/8 B200; % HBM roofline"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="mla36m", choices=["mla36m", "mla1b"])
    ap.add_argument("--prompts", type=int, default=None, help="prompts per step (whole job)")
    ap.add_argument("--group", type=int, default=None)
    ap.add_argument("--prompt-len", type=int, default=None)
    ap.add_argument("--new-tokens", type=int, default=None)
    ap.add_argument("--cpu-rollouts", type=int, default=8,
                    help="rollouts (one group) in the bounded CPU-baseline sample of the GPU arm")
    ap.add_argument("--reference-budget", type=float, default=240.0,
                    help="seconds the --impl reference run may take (sizes its per-step sample)")
    ap.add_argument("--no-fixed-check", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gemm-shapes", action="store_true",
                    help="print per-shape GEMM device time to stderr")
    args = ap.parse_args()
    dflt = WORKLOADS[args.workload]
    for k in ("prompts", "group", "prompt_len", "new_tokens"):
        if getattr(args, k) is None:
            setattr(args, k, dflt[k])
    return args


# prompts, group, prompt length, new tokens, reward (Bernoulli p; None = N(0, 1)), learning rate
WORKLOADS = {
    "mla36m": {"prompts": 256, "group": 8, "prompt_len": 128, "new_tokens": 256, "p_reward": 0.3, "lr": 1e-5},
    "mla1b": {"prompts": 128, "group": 16, "prompt_len": 512, "new_tokens": 1536, "p_reward": None, "lr": 1e-5},
}


def model_config(args):
    from cpp_inference_train_engine_b200.config import MLA1B, MLA36M
    return MLA36M if args.workload == "mla36m" else MLA1B


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
def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class CpuSample:
    """The reference engine's own CPU path (oracle/_ref, OpenBLAS) on a bounded sample of the
    workload: `n` rollouts of one prompt (one group) with the workload's prompt length and new
    tokens, then their GRPO update. Each run() returns generated tokens per second."""

    def __init__(self, args, n):
        from cpp_inference_train_engine_b200.config import MLA36M, AdamWConfig
        from cpp_inference_train_engine_b200.rng import grpo_workload
        from oracle import ref
        self.ref, self.cfg, self.args, self.n = ref, MLA36M, args, n
        prompts, seeds, rewards = grpo_workload(1, n, args.prompt_len, MLA36M.vocab_size, 0.3)
        rewards[0], rewards[-1] = 1.0, 0.0
        self.prompts, self.seeds, self.rewards = prompts, seeds, rewards
        self.seq = args.prompt_len + args.new_tokens
        self.pol = ref.Session(MLA36M, 0, optimizer=AdamWConfig().as_list())
        self.refm = ref.Session(MLA36M, 0)

    def run(self):
        a, c, r = self.args, self.cfg, self.ref
        t0 = time.perf_counter()
        rolls = [self.pol.rollout(self.prompts[i], a.new_tokens, self.seq, c.eos_id, c.pad_id, int(self.seeds[i]))
                 for i in range(self.n)]
        stack = lambda k: np.stack([x[k] for x in rolls])  # noqa: E731
        r.grpo_update(self.pol, self.refm, self.n, stack("input"), stack("target"), stack("mask"),
                      stack("old_lp"), self.rewards, 0.2, 0.04, 1e-5)
        dt = time.perf_counter() - t0
        return sum(len(x["tokens"]) for x in rolls) / dt, dt

    def describe(self):
        threads = os.environ.get("OPENBLAS_NUM_THREADS", str(_host_threads()))
        return (f"one group of {self.n} rollouts (prompt {self.args.prompt_len}, {self.args.new_tokens} new "
                f"tokens, S={self.seq}) + their GRPO update, reference CPU build, OpenBLAS 0.3.30 "
                f"(numpy-bundled) on {threads} threads; host: {cpu_model()}")


def cpu_baseline(args):
    """The GPU arm's reported CPU baseline (rank 0, one GPU): one timed group of rollouts."""
    from oracle import ref
    if not ref.available():
        return None
    smp = CpuSample(args, args.cpu_rollouts)
    rate, _ = smp.run()
    return {"value": rate, "unit": "tok/s", "cores": int(os.environ.get("OPENBLAS_NUM_THREADS", _host_threads())),
            "host_threads": _host_threads(), "cpu_model": cpu_model(), "kind": "reference",
            "sample": smp.describe()}


def run_reference(args, rank, world):
    """--impl reference: rank 0 alone times the reference CPU path; the sample per step is one
    group of 8, 4 or 2 rollouts, the largest whose W + K steps fit the time budget."""
    if rank != 0:
        return
    if args.workload != "mla36m":
        print(json.dumps({"impl": "reference", "unavailable": "the reference's CPU path takes days per step "
                          "of the 1.14 B model (2048 rollouts x 2048 positions); no CPU sample is run"}))
        return
    from oracle import ref
    if not ref.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref (the reference CPU build) is not built"}))
        return
    probe = CpuSample(args, 2)
    _, dt = probe.run()  # untimed: first-touch of the weights, thread pool start-up
    per_rollout = dt / 2
    steps = max(args.warmup, 0) + args.steps
    n = 2
    for g in (8, 4):
        if steps * g * per_rollout <= args.reference_budget:
            n = g
            break
    smp = probe if n == 2 else CpuSample(args, n)
    for _ in range(max(args.warmup, 0)):
        smp.run()
    rates = [smp.run()[0] for _ in range(args.steps)]
    value = statistics.median(rates)
    res = {"value": value, "unit": "tok/s", "cores": int(os.environ["OPENBLAS_NUM_THREADS"]),
           "host_threads": _host_threads(), "cpu_model": cpu_model(), "kind": "reference",
           "sample": smp.describe()}
    line = {"metric": METRIC if args.workload == "mla36m" else METRIC_MLA1B, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "impl": "reference",
            "higher_is_better": True, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args, world),
            "cpu_baseline": res,
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def workload_config(args, world):
    n = args.prompts * args.group
    w = WORKLOADS[args.workload]
    cfg = model_config(args)
    seq = args.prompt_len + args.new_tokens
    cache_gb = n * seq * (cfg.kv_lora_rank + cfg.head_dim_rope) * 2 * cfg.n_layers / 1e9
    return {"workload": "grpo_step_" + args.workload, "rollouts": n, "prompts": args.prompts,
            "group": args.group, "prompt_len": args.prompt_len, "new_tokens": args.new_tokens,
            "sequence": seq, "temperature": 1.0,
            "reward": "normal(0,1)" if w["p_reward"] is None else f"bernoulli({w['p_reward']})",
            "clip": 0.2, "kl": 0.04, "lr": w["lr"],
            "parallelism": f"dp{world}", "l2": f"inputs larger than L2 (cache {cache_gb:.1f} GB, logits)"}


# ---------------------------------------------------------------------------- ours
def fixed_batch(args, cfg, n_total, prompts_all):
    """A teacher-forced GRPO batch for the whole job, the same on every rank count: each
    rollout is its prompt followed by new_tokens fixed ids (np.random seed 6), laid out as
    completion_batch does (trainer.cpp:386-408)."""
    seq = args.prompt_len + args.new_tokens
    comp = np.random.default_rng(6).integers(0, cfg.vocab_size - 8, (n_total, args.new_tokens)).astype(np.uint16)
    ids = np.concatenate([prompts_all, comp], axis=1)
    inp = np.full((n_total, seq), cfg.pad_id, np.uint16)
    tgt = np.full((n_total, seq), cfg.pad_id, np.uint16)
    mask = np.zeros((n_total, seq), np.float32)
    inp[:, :seq - 1] = ids[:, :-1]
    tgt[:, :seq - 1] = ids[:, 1:]
    mask[:, args.prompt_len - 1:seq - 1] = 1
    return inp, tgt, mask


def gemm_algorithmic_flops(cfg, rollouts, seq, prompt_len):
    """Algorithmic tensor-core work of one step's event-timed products on one rank: every
    teacher-forced token passes the model's matrices (2 x their entries: 2 x 27,374,720
    flops for the 35.8M model) and the vocabulary
    head (2 x d x V) five times (old-policy, frozen-reference and policy forwards, the backward
    at twice a forward), and every prompt token passes the matrices once in the prefill. The
    fp32-accurate head's three fp16 terms count once: their extra work is an implementation
    cost, not algorithmic work. Attention is its own kernel class."""
    mats = 0
    for _, (r, c), role in cfg.parameter_shapes()[2:]:
        if role != "norm_scale":
            mats += r * c
    model = 2.0 * mats
    vocab = 2.0 * cfg.d_model * cfg.vocab_size
    return rollouts * seq * 5 * (model + vocab) + rollouts * prompt_len * model


def decode_algorithmic_bytes(cfg, n_params, rollouts, prompt_len, new_tokens):
    """HBM bytes one rank's rollout decode must move: per decode step the fp16 weights once
    (2 x P) and every row's latent cache, (kv rank + rope) fp16 values per cached position and
    layer; decode step k (1 <= k < new_tokens) attends prompt_len + k positions."""
    kv = 2 * (cfg.kv_lora_rank + cfg.head_dim_rope) * cfg.n_layers
    return sum(2.0 * n_params + rollouts * (prompt_len + k) * kv for k in range(1, new_tokens))


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)  # CPU only: no process group, no GPU
        return

    import datetime

    import torch

    import cpp_inference_train_engine_b200 as E
    from cpp_inference_train_engine_b200 import distributed as D
    from cpp_inference_train_engine_b200.config import MLA36M, AdamWConfig
    from cpp_inference_train_engine_b200.rng import grpo_workload

    dist = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        # harness only (barriers, max over ranks of the timings); the engine's own NCCL
        # communicator is bootstrapped by distributed.init_comm without torch
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))

    cfg = model_config(args)
    wl = WORKLOADS[args.workload]
    n_total = args.prompts * args.group
    try:
        sl = D.rollout_shard(n_total, args.group, rank, world)
    except ValueError as e:
        raise SystemExit(str(e))
    seq = args.prompt_len + args.new_tokens
    prompts_all, seeds, rewards_all = grpo_workload(args.prompts, args.group, args.prompt_len,
                                                    cfg.vocab_size, wl["p_reward"])
    prompts, seeds, rewards = prompts_all[sl].copy(), seeds[sl].copy(), rewards_all[sl].copy()

    W = E.init_params(cfg, 0)
    pol = E.make_execution(cfg, W, optimizer=AdamWConfig(), device=local)
    refm = E.make_execution(cfg, W, device=local)
    if world > 1:
        D.init_comm(pol, rank, world)
    stream = torch.cuda.ExternalStream(pol.stream, device=local)

    def barrier():
        torch.cuda.synchronize(local)
        if dist:
            dist.barrier()

    fixed = None
    if not args.no_fixed_check and args.workload == "mla36m":
        # One GRPO update on a fixed teacher-forced batch of the whole job: its loss and
        # pre-clip gradient norm are global sums, so they must not depend on the rank count.
        inp, tgt, mask = fixed_batch(args, cfg, n_total, prompts_all)
        inp, tgt, mask = inp[sl].copy(), tgt[sl].copy(), mask[sl].copy()
        R = inp.shape[0]
        lp = pol.log_probabilities(inp, tgt, R, seq).reshape(R, seq)
        phase = np.arange(n_total * seq, dtype=np.float64).reshape(n_total, seq)[sl]
        old = (lp + 0.3 * np.sin(phase) * mask).astype(np.float32)
        out = pol.grpo_step(refm, inp, tgt, mask, old, rewards, args.group, n_total=n_total,
                            clip=0.2, klc=0.04, learning_rate=wl["lr"])
        fixed = {"loss": out["loss"], "kl": out["kl"], "grad_norm": out["grad_norm"],
                 "batch": f"{n_total} x {seq} teacher-forced, fixed ids (seed 6), old = lp + 0.3 sin"}
        pol.upload(W)  # back to the initial weights, zero moments, step 0
        barrier()

    def one_step(step_idx):
        # The rollout seeds advance per update like the trainer's Rng(seed) stream.
        with np.errstate(over="ignore"):  # arithmetic mod 2^64 is intended
            s = (seeds + np.uint64(step_idx) * np.uint64(0x9E3779B97F4A7C15)).astype(np.uint64)
        r = pol.rollout(prompts, args.new_tokens, seq, s, 1.0)
        out = pol.grpo_step(refm, r["input"], r["target"], r["mask"], r["old_lp"], rewards,
                            args.group, n_total=n_total, clip=0.2, klc=0.04, learning_rate=wl["lr"])
        return r, out

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
    decode_ms = (prof_p["decode"][0] + prof_p["sample"][0]) / args.steps
    if dist:
        t = torch.tensor([e2e_ms, dev_ms, float(toks), decode_ms], device=f"cuda:{local}", dtype=torch.float64)
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = t.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        e2e_ms, dev_ms, toks, decode_ms = float(mx[0]), float(mx[1]), int(sm[2]), float(mx[3])
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
        R = prompts.shape[0]
        if top == "k_gemm":
            work = gemm_algorithmic_flops(cfg, R, seq, args.prompt_len) * args.steps
            how = ("algorithmic flops: rollouts x S x 5 x (2 x matrix entries + 2 d V) + prompt tokens x "
                   "2 x matrix entries, over the class's event-timed launches")
        else:
            work = kern[top]["work"]
            how = "work as counted per launch"
        tensor = top in ("k_gemm", "k_flash_fwd", "k_flash_bwd")
        sec = kern[top]["ms"] / 1e3
        achieved = (work / sec / 1e12) if tensor else (work / sec / 1e9)
        peak = pk["tflops"] if tensor else pk["hbm_gbs"]
        roofline = {"kernel": top, "bound": "tensor" if tensor else "hbm",
                    "achieved": achieved, "peak": peak, "unit": "TFLOP/s" if tensor else "GB/s",
                    "frac": achieved / peak, "peak_source": pk["source"] + " (sustained bf16)",
                    "work": how, "launches": kern[top]["launches"],
                    "avg_launch_us": 1e3 * kern[top]["ms"] / max(kern[top]["launches"], 1),
                    # DRAM bytes of one vocabulary-head launch (the class's largest shape),
                    # single-launch ncu capture at M = 8,192 scaled to this chunk's M
                    "traffic": vocab_head_traffic(seq, R) if args.workload == "mla36m" else None,
                    "traffic_kernel": "gemm_tc_pair_kernel, vocabulary head M x 16384 x 1536, log-sum-exp epilogue, no store"}
        dec_bytes = decode_algorithmic_bytes(cfg, pol.n_params, R, args.prompt_len, args.new_tokens)
        dec_gbs = dec_bytes / (decode_ms / 1e3) / 1e9 if decode_ms else None
        roofline_decode = {"phase": "rollout decode + sampling (per rank, slowest rank's time)",
                           "bound": "hbm", "achieved": dec_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                           "frac": dec_gbs / pk["hbm_gbs"] if dec_gbs else None,
                           "bytes_per_step": dec_bytes, "ms_per_step": decode_ms,
                           "work": "sum over decode steps of 2 P (fp16 weights) + rows x ctx x 2 (kv + rope) L B"}
        phases = {k: round(prof_p[k][0] / args.steps, 3) for k in
                  ("prefill", "decode", "sample", "logprob", "backward", "adamw", "allreduce")}
        phases["reference_logprob"] = round(prof_r["logprob"][0] / args.steps, 3)
        cpu = None
        if world == 1 and not args.no_cpu_baseline and args.workload == "mla36m":
            cpu = cpu_baseline(args)
        line = {
            "metric": METRIC if args.workload == "mla36m" else METRIC_MLA1B, "value": toks / (dev_ms / 1e3), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp16 tensor-core compute, fp32 master/accumulate", "data": "synthetic",
            "config": workload_config(args, world),
            "e2e": {"value": toks / (e2e_ms / 1e3), "unit": "tok/s",
                    "ms_per_step": e2e_ms / args.steps,
                    "h2d_bytes_per_step": h2d // args.steps, "d2h_bytes_per_step": d2h // args.steps},
            "rollout_tokens_per_step": toks // args.steps,
            "phases_ms_per_step": phases,
            "kernels": {k: {"ms_per_step": round(v["ms"] / args.steps, 3),
                            "launches_per_step": v["launches"] // args.steps} for k, v in kern.items()},
            "roofline": roofline,
            "roofline_decode": roofline_decode,
            "fixed_update": fixed,
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


def vocab_head_traffic(seq, rollouts):
    """DRAM bytes of one vocabulary-head launch at this workload's chunk size: the committed
    single-launch capture of the CTA-pair kernel with the log-sum-exp epilogue and no logits
    store (76.8 MB read + 8.4 MB written at M = 8,192; operands read 1.02x), scaled by M, as
    its partials and the re-reads of B grow with the number of M-tiles."""
    chunk = min(rollouts, max(1, 196608 // seq)) * seq
    return 85.2e6 * chunk / 8192.0


if __name__ == "__main__":
    main()
