"""Teacher-forced phases of the GRPO step on one chunk of rollouts, timed alone.

Runs, on synthetic rollouts of the 35.8M model (random ids, prompt positions masked),
the rollout's old-log-prob pass (``log_probabilities`` of the policy) and the GRPO update
(``grpo_step``: frozen-reference and policy passes, loss, backward, AdamW), and reports
their device times with CUDA events on the library stream. The last iteration is bracketed
by cudaProfilerStart/Stop, so a profiler started with ``--profile-from-start off`` sees
exactly one old-log-prob pass and one update.

    python -m cpp_inference_train_engine_b200.phase_bench --rollouts 80 --seq 384
"""
import argparse
import json


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--rollouts", type=int, default=80, help="whole groups of --group")
    ap.add_argument("--group", type=int, default=8)
    ap.add_argument("--seq", type=int, default=384)
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    args = ap.parse_args(argv)

    import numpy as np
    import torch

    import cpp_inference_train_engine_b200 as E
    from cpp_inference_train_engine_b200.config import MLA36M, AdamWConfig

    cfg = MLA36M
    n, S = args.rollouts, args.seq
    rng = np.random.default_rng(4)
    inp = rng.integers(0, cfg.vocab_size, (n, S)).astype(np.uint16)
    tgt = rng.integers(0, cfg.vocab_size, (n, S)).astype(np.uint16)
    mask = np.zeros((n, S), np.float32)
    mask[:, args.prompt - 1:] = 1
    rewards = (rng.uniform(size=n) < 0.3).astype(np.float32)
    rewards[::args.group] = 1.0  # no constant group: never skipped
    rewards[1::args.group] = 0.0
    W = E.init_params(cfg, 0)
    pol = E.make_execution(cfg, W, optimizer=AdamWConfig())
    refm = E.make_execution(cfg, E.init_params(cfg, 1))
    stream = torch.cuda.ExternalStream(pol.stream)
    ev = lambda: torch.cuda.Event(enable_timing=True)
    times = {"old_lp": [], "grpo_step": []}
    for it in range(args.warmup + args.iters):
        last = it == args.warmup + args.iters - 1
        torch.cuda.synchronize()
        if last:
            torch.cuda.profiler.start()
        e0, e1, e2 = ev(), ev(), ev()
        e0.record(stream)
        old = pol.log_probabilities(inp, tgt, n, S).reshape(n, S)
        e1.record(stream)
        pol.grpo_step(refm, inp, tgt, mask, old, rewards, args.group, learning_rate=1e-5)
        e2.record(stream)
        torch.cuda.synchronize()
        if last:
            torch.cuda.profiler.stop()
        if it >= args.warmup:
            times["old_lp"].append(e0.elapsed_time(e1))
            times["grpo_step"].append(e1.elapsed_time(e2))
    tokens = n * S
    out = {k: {"ms": float(np.median(v)), "tokens_per_s": tokens / (float(np.median(v)) / 1e3)}
           for k, v in times.items()}
    print(json.dumps({"rollouts": n, "seq": S, "tokens": tokens, **out}))
    pol.close()
    refm.close()


if __name__ == "__main__":
    main()
