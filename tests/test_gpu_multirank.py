"""Data-parallel GRPO step on 2 GPUs (one process per GPU, NCCL gradient all-reduce inside
mm_cuda_grpo_step) against the same step on one GPU over the whole batch: loss, KL and
pre-clip gradient norm within 1e-4 relative, updated weights within one AdamW move, and the
per-row log-probs bit-identical. Skipped on a box with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest

from tests.gpu_util import require_gpu

pytestmark = pytest.mark.gpu

WORLD = 2
N, G, S, PROMPT = 16, 4, 64, 16
LR = 1e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch():
    from cpp_inference_train_engine_b200.config import TINY
    rng = np.random.default_rng(5)
    inp = rng.integers(0, TINY.vocab_size, (N, S)).astype(np.uint16)
    tgt = rng.integers(0, TINY.vocab_size, (N, S)).astype(np.uint16)
    mask = np.zeros((N, S), np.float32)
    mask[:, PROMPT - 1:] = 1
    mask[5, 40:] = 0
    rewards = (rng.uniform(size=N) < 0.5).astype(np.float32)
    rewards[G:2 * G] = 1.0  # one constant group
    return inp, tgt, mask, rewards


def _step(device, rows, n_total, comm=None):
    """One GRPO step of the tiny model over `rows`; returns lp, result and updated weights."""
    import cpp_inference_train_engine_b200 as E
    from cpp_inference_train_engine_b200.config import TINY, AdamWConfig
    inp, tgt, mask, rewards = (a[rows] for a in _batch())
    W = E.init_params(TINY, 0)
    pol = E.make_execution(TINY, W, optimizer=AdamWConfig(), device=device)
    refm = E.make_execution(TINY, E.init_params(TINY, 1), device=device)
    if comm:
        comm(pol)
    n = inp.shape[0]
    lp = pol.log_probabilities(inp, tgt, n, S).reshape(n, S)
    old = (lp + 0.05 * np.sin(np.arange(N * S).reshape(N, S)[rows])).astype(np.float32)
    res = pol.grpo_step(refm, inp, tgt, mask, old, rewards, G, n_total=n_total, learning_rate=LR)
    w = pol.synchronize_to_host(params=True)["params"]
    pol.close()
    refm.close()
    return lp, res, w


def _worker(rank, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from cpp_inference_train_engine_b200 import distributed as D
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        sl = D.rollout_shard(N, G, rank, WORLD)
        lp, res, w = _step(rank, np.arange(N)[sl], N, comm=lambda e: D.init_comm(e, rank, WORLD))
        out[rank] = dict(lp=lp, res=res, w=w)
    finally:
        dist.destroy_process_group()


def test_two_gpus_match_one():
    require_gpu()
    import torch
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, port, out)) for r in range(WORLD)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        res = [dict(out[r]) for r in range(WORLD)]
    lp, one, w = _step(0, np.arange(N), N)
    np.testing.assert_array_equal(np.concatenate([r["lp"] for r in res]), lp)
    for r in res:
        assert r["res"]["skipped"] == one["skipped"] is False
        for k in ("loss", "kl", "grad_norm"):
            assert abs(r["res"][k] - one[k]) <= 1e-4 * abs(one[k]), (k, r["res"][k], one[k])
        # the ranks hold identical replicas, within one AdamW move of the single-GPU weights
        np.testing.assert_array_equal(r["w"], res[0]["w"])
        assert np.abs(r["w"] - w).max() <= 2.05 * LR
