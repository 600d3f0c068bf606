"""The reference engine's own GRPO trainer, run as its users run it: its training CLI
(apps/train_main.cpp -> train_model, src/train/trainer.cpp:409, GRPO branch :784-891), both
unmodified, built by oracle/Makefile as oracle/_ref/mini_mla_train (CPU) and
oracle/_ref/mini_mla_train_cuda, whose make_execution also takes backend "cuda" (the one-branch
factory of cpp_inference_train_engine_b200/reference_adapter/make_execution_cuda.cpp) and so
reaches this backend. Everything around the hot path is the reference's: the byte tokenizer
file, chat prompts, text rewards ("contains"), rollouts.jsonl, metrics.jsonl, validation, and
the checkpoint directories written by save_checkpoint after synchronize_to_host.

* CPU (no GPU): the CLI on the reference's own CPU backend over the files this test writes
  (the plumbing the GPU tests reuse).
* GPU: a cuda run of 4 updates with checkpoints every 2, then a resume from the step-2
  checkpoint. The reference trainer itself compares the replayed step-4 state with the
  checkpoint already on disk (trainer.cpp:556-574: weights, Adam moments, step count, RNG and
  trainer state, exact) and fails on any difference, so the run finishing IS the byte-exact
  replay check (the reference's own gate, tests/test_tools.py:560-567).
* GPU: the first update on "cpu" and on "cuda" from the same seed: the same prompts and
  rollout seeds; when both backends sample the same completions (the tiny model's logits
  agree to ~1e-5, so a T = 1 draw differs only when it lands that close to a CDF boundary),
  rewards are equal and loss, KL and gradient norm agree within 1e-3 relative.
"""
import json
import os
import subprocess

import numpy as np
import pytest

from tests.gpu_util import ROOT, require_gpu

SPECIALS = ["<|pad|>", "<|bos|>", "<|eos|>", "<|user|>", "<|assistant|>", "<|system|>", "<|tool|>", "<|sep|>"]


def write_run_files(root, backend, steps=4, checkpoint_every=2, seed=7, output="run"):
    """The byte tokenizer (264 ids: 256 bytes, then the 8 specials the chat template expects,
    include/mini_mla/tokenizer.hpp), the tiny model config, prompt/answer records of our own,
    and the TrainOptions object train_model reads."""
    os.makedirs(root, exist_ok=True)
    tok = {"format": "mini-mla-tokenizer", "version": 1, "pretokenizer": "bytes-v1", "vocab_size": 264,
           "merges": [], "specials": {n: 256 + i for i, n in enumerate(SPECIALS)}}
    model = {"model_type": "mla_dense_decoder", "version": 1, "vocab_size": 264, "max_sequence_length": 64,
             "n_layers": 2, "d_model": 32, "n_heads": 2, "head_dim_nope": 12, "head_dim_rope": 4,
             "head_dim_value": 16, "q_lora_rank": 16, "kv_lora_rank": 8, "d_ff": 64, "norm_epsilon": 1e-5,
             "rope_theta": 10000, "norm": "rmsnorm", "activation": "swiglu", "mla_latent_norms": True,
             "tie_word_embeddings": True, "bias": False}
    letters = "etaoinsr"
    train = [{"prompt": f"Type the letter {c} somewhere.", "answer": c} for c in letters]
    val = [{"prompt": "Which letter comes after d?", "answer": "e"}]
    paths = {k: os.path.join(root, k) for k in ("tokenizer.json", "model.json", "train.jsonl", "val.jsonl")}
    with open(paths["tokenizer.json"], "w") as f:
        json.dump(tok, f)
    with open(paths["model.json"], "w") as f:
        json.dump(model, f)
    with open(paths["train.jsonl"], "w") as f:
        f.write("".join(json.dumps(r) + "\n" for r in train))
    with open(paths["val.jsonl"], "w") as f:
        f.write("".join(json.dumps(r) + "\n" for r in val))
    return {"model_config": paths["model.json"], "tokenizer": paths["tokenizer.json"],
            "output": os.path.join(root, output), "train": [paths["train.jsonl"]],
            "validation": [paths["val.jsonl"]], "mode": "grpo", "backend": backend, "precision": "fp32",
            "reward": "contains", "sequence_length": 48, "microbatch": 1, "grad_accum": 1, "steps": steps,
            "warmup_steps": 1, "seed": seed, "learning_rate": 2e-3, "log_every": 1,
            "checkpoint_every": checkpoint_every, "validate_every": 2, "validation_batches": 1,
            "group_size": 8, "completion_tokens": 12, "gradient_epochs": 2, "kl_coefficient": 0.05}


def read_jsonl(path):
    with open(path) as f:
        return [json.loads(line) for line in f if line.strip()]


CLI = {"cpu": os.path.join(ROOT, "oracle", "_ref", "mini_mla_train"),
       "cuda": os.path.join(ROOT, "oracle", "_ref", "mini_mla_train_cuda")}


def cli_args(o):
    """The TrainOptions of write_run_files as the CLI's flags (apps/train_main.cpp:82-140)."""
    flag = {"model_config": "config", "sequence_length": "sequence-length", "grad_accum": "grad-accum",
            "warmup_steps": "warmup-steps", "learning_rate": "learning-rate", "log_every": "log-every",
            "checkpoint_every": "checkpoint-every", "validate_every": "validate-every",
            "validation_batches": "validation-batches", "group_size": "group-size",
            "completion_tokens": "completion-tokens", "gradient_epochs": "gradient-epochs",
            "kl_coefficient": "kl-coefficient"}
    args = []
    for k, v in o.items():
        args += ["--" + flag.get(k, k), ",".join(v) if isinstance(v, list) else str(v)]
    return args


def run_cli(build, args, timeout=900):
    r = subprocess.run([CLI[build]] + args, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    return r


def test_reference_trainer_runs_on_its_cpu_backend(tmp_path):
    if not os.path.exists(CLI["cpu"]):
        pytest.skip("oracle/_ref not built")
    o = write_run_files(str(tmp_path), "cpu", steps=2, checkpoint_every=2)
    run_cli("cpu", cli_args(o))
    metrics = read_jsonl(os.path.join(o["output"], "metrics.jsonl"))
    assert [m["step"] for m in metrics if "train_loss" in m][-1] == 2
    assert os.path.exists(os.path.join(o["output"], "checkpoint-00000002", "weights.bin"))
    assert len(read_jsonl(os.path.join(o["output"], "rollouts.jsonl"))) >= 16


@pytest.mark.gpu
def test_reference_trainer_on_cuda_replays_a_resumed_run_exactly(tmp_path):
    require_gpu()
    if not os.path.exists(CLI["cuda"]):
        pytest.skip("oracle/_ref cuda build missing")
    o = write_run_files(str(tmp_path), "cuda", steps=4, checkpoint_every=2)
    run_cli("cuda", cli_args(o))
    out = o["output"]
    metrics = [m for m in read_jsonl(os.path.join(out, "metrics.jsonl")) if "train_loss" in m]
    assert metrics[-1]["step"] == 4
    assert all(np.isfinite(m["train_loss"]) and np.isfinite(m["grad_norm"]) for m in metrics)
    state = json.load(open(os.path.join(out, "checkpoint-00000004", "trainer_state.json")))
    assert state["device"].startswith("NVIDIA B200") and state["options"]["backend"] == "cuda"
    weights = open(os.path.join(out, "checkpoint-00000004", "weights.bin"), "rb").read()
    moments = open(os.path.join(out, "checkpoint-00000004", "optimizer.bin"), "rb").read()
    # resume at step 2: the trainer replays updates 3 and 4 and, reaching the step-4 checkpoint
    # that exists, throws unless its state equals the replayed one exactly
    run_cli("cuda", ["--resume", os.path.join(out, "checkpoint-00000002")])
    assert open(os.path.join(out, "checkpoint-00000004", "weights.bin"), "rb").read() == weights
    assert open(os.path.join(out, "checkpoint-00000004", "optimizer.bin"), "rb").read() == moments


@pytest.mark.gpu
def test_reference_trainer_first_update_cpu_vs_cuda(tmp_path):
    require_gpu()
    if not os.path.exists(CLI["cuda"]):
        pytest.skip("oracle/_ref cuda build missing")
    runs = {}
    for backend in ("cpu", "cuda"):
        o = write_run_files(str(tmp_path / backend), backend, steps=1, checkpoint_every=1)
        run_cli("cuda", cli_args(o))  # the cuda build runs backend "cpu" unchanged
        runs[backend] = (read_jsonl(os.path.join(o["output"], "rollouts.jsonl")),
                         [m for m in read_jsonl(os.path.join(o["output"], "metrics.jsonl")) if "train_loss" in m])
    (rc, mc), (rg, mg) = runs["cpu"], runs["cuda"]
    # prompts and rollout seeds come from the trainer's own Rng: identical on both backends
    assert [(r["prompt"], r["seed"]) for r in rc] == [(r["prompt"], r["seed"]) for r in rg]
    same = sum(a["completion"] == b["completion"] for a, b in zip(rc, rg))
    assert same >= 0.8 * len(rc), (same, len(rc))
    if same == len(rc):  # identical samples: the update itself is compared
        assert [r["reward"] for r in rc] == [r["reward"] for r in rg]
        a, b = mc[-1], mg[-1]
        for k in ("train_loss", "kl", "grad_norm"):
            assert abs(a[k] - b[k]) <= 1e-3 * max(abs(a[k]), 1e-12), (k, a[k], b[k])
