"""Data-parallel GRPO on CPU ranks (gloo, world size 2), no GPU: the rollout sharding, the
NCCL unique-id bootstrap over the engine's TCP rendezvous, and the algebra of the sharded update that
the engine runs on device — each rank's coefficients divided by the global rollout count,
gradients and loss/KL summed over ranks, the skip flag OR-ed — against one process over the
whole batch (oracle restatement of trainer.cpp:784-891 on the tiny model)."""
import os
import socket

import numpy as np
import pytest

from cpp_inference_train_engine_b200 import distributed as D
from cpp_inference_train_engine_b200.config import TINY

WORLD = 2
N, G, S, PROMPT = 16, 4, 24, 8


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(3)
    inp = rng.integers(0, TINY.vocab_size, (N, S)).astype(np.uint16)
    tgt = rng.integers(0, TINY.vocab_size, (N, S)).astype(np.uint16)
    mask = np.zeros((N, S), np.float32)
    mask[:, PROMPT - 1:] = 1
    mask[3, 20:] = 0  # ragged response
    rewards = rng.uniform(size=N).astype(np.float32)
    rewards[:G] = 0.5  # a constant group: zero advantages
    return inp, tgt, mask, rewards


def _grpo(rows, n_total):
    """Loss, KL and flat gradient of the GRPO objective over `rows` of the batch."""
    from oracle import mla_oracle as O
    inp, tgt, mask, rewards = _inputs()
    pol = O.Params(TINY, O.init_params(TINY, 0))
    refp = O.Params(TINY, O.init_params(TINY, 1))
    inp, tgt, mask, rewards = inp[rows], tgt[rows], mask[rows], rewards[rows]
    n = inp.shape[0]
    lp = O.log_probabilities(TINY, pol, inp, tgt, n, S).reshape(n, S)
    ref = O.log_probabilities(TINY, refp, inp, tgt, n, S).reshape(n, S)
    phase = np.arange(N * S).reshape(N, S)[rows]  # global positions: same perturbation per shard
    old = (lp + 0.05 * np.sin(phase)).astype(np.float32)
    adv = np.concatenate([O.group_advantages(rewards[g:g + G]) for g in range(0, n, G)])
    loss, kl, coef = O.grpo_coefficients(lp, old, ref, mask, adv, 0.2, 0.04, n_total=n_total)
    _, grads = O.accumulate(TINY, pol, inp, tgt, coef, n, S)
    flat = np.concatenate([g.reshape(-1) for g in grads]).astype(np.float64)
    return loss, kl, flat, int(np.any(adv != 0))


def _worker(rank, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        sl = D.rollout_shard(N, G, rank, WORLD)
        from cpp_inference_train_engine_b200.engine import CudaExecution
        uid = D.exchange_unique_id(rank, WORLD, CudaExecution.nccl_unique_id, "127.0.0.1", port + 1,
                                   timeout=60)
        ids = [None] * WORLD
        dist.all_gather_object(ids, uid)
        loss, kl, flat, any_nz = _grpo(np.arange(N)[sl], N)
        g = torch.from_numpy(flat)
        dist.all_reduce(g)  # the engine's gradient all-reduce (SUM)
        s = torch.tensor([loss, kl], dtype=torch.float64)
        dist.all_reduce(s)  # loss / KL sums
        a = torch.tensor([any_nz], dtype=torch.int32)
        dist.all_reduce(a, op=dist.ReduceOp.MAX)  # skip rule: any non-zero advantage anywhere
        out[rank] = dict(sl=(sl.start, sl.stop), same_id=all(i == ids[0] for i in ids),
                         local_any=any_nz, any=int(a.item()), loss=float(s[0]), kl=float(s[1]),
                         grad=g.numpy().copy())
    finally:
        dist.destroy_process_group()


def test_rollout_shard_rules():
    assert D.rollout_shard(2048, 8, 3, 8) == slice(768, 1024)
    assert D.rollout_shard(16, 4, 1, 2) == slice(8, 16)
    for args in ((16, 4, 0, 3), (16, 4, 2, 2), (12, 8, 0, 1), (16, 8, 0, 4)):
        with pytest.raises(ValueError):
            D.rollout_shard(*args)


def test_two_gloo_ranks_match_one_process():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, port, out)) for r in range(WORLD)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(180)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        res = [dict(out[r]) for r in range(WORLD)]
    assert [r["sl"] for r in res] == [(0, 8), (8, 16)]
    assert all(r["same_id"] for r in res)
    # rank 0 holds the constant group next to a varying one; the flag is global either way
    assert all(r["any"] == 1 for r in res)
    loss, kl, flat, any_nz = _grpo(np.arange(N), N)
    assert any_nz == 1
    for r in res:
        assert abs(r["loss"] - loss) <= 1e-9 * max(1.0, abs(loss))
        assert abs(r["kl"] - kl) <= 1e-9 * max(1.0, abs(kl))
        np.testing.assert_allclose(r["grad"], flat, rtol=0, atol=1e-6 * np.abs(flat).max())


def _failing_worker(rank, port, out):
    """Rank 1 exits before the bootstrap; rank 0 then serves the NCCL id to nobody."""
    if rank == 1:
        os._exit(0)  # a rank that dies between steps, with no collective in flight
    import time
    t0 = time.time()
    try:
        D.exchange_unique_id(rank, WORLD, lambda: bytes(128), "127.0.0.1", port, timeout=10)
        out[rank] = ("completed", time.time() - t0)
    except Exception as e:  # the peer is gone: the bootstrap must fail, not hang
        out[rank] = ("error " + type(e).__name__, time.time() - t0)


def test_rendezvous_without_rank0_fails_in_time():
    import time
    t0 = time.time()
    with pytest.raises(RuntimeError):
        D.exchange_unique_id(1, 2, lambda: bytes(128), "127.0.0.1", _free_port(), timeout=2)
    assert time.time() - t0 < 30


def test_rank_failure_is_reported_not_hung():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_failing_worker, args=(r, port, out)) for r in range(WORLD)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        alive = [p.is_alive() for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        assert not any(alive), "a rank hung after its peer left"
        status, seconds = out[0]
    assert status.startswith("error"), status
    assert seconds < 60
