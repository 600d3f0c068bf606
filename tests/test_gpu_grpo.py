"""GRPO objective kernel, rollouts and the full update (config 1 of the benchmark plan:
tiny model, 2 prompts x group 4, prompt 16, 32 new tokens, S=48) against the reference."""
import numpy as np
import pytest

import cpp_inference_train_engine_b200 as E
from cpp_inference_train_engine_b200.config import TINY, AdamWConfig
from oracle import mla_oracle as O
from oracle import ref
from tests.gpu_util import require_gpu

pytestmark = pytest.mark.gpu


def test_grpo_coefficients_match_restatement():
    require_gpu()
    ex = E.CudaExecution(TINY)
    rng = np.random.default_rng(3)
    n, S, G = 8, 20, 4
    lp = rng.normal(-3, 1, (n, S)).astype(np.float32)
    old = (lp + rng.normal(0, 0.3, (n, S))).astype(np.float32)
    rf = (lp + rng.normal(0, 0.3, (n, S))).astype(np.float32)
    mask = (rng.random((n, S)) < 0.6).astype(np.float32)
    mask[:, 0] = 1
    rewards = (rng.random(n) < 0.5).astype(np.float32)
    out = ex.grpo_coefficients(lp, old, rf, mask, rewards, G, n, 0.2, 0.04)
    adv = np.concatenate([O.group_advantages(rewards[g * G:(g + 1) * G]) for g in range(n // G)])
    assert np.array_equal(out["advantages"], adv)
    loss, kl, coef = O.grpo_coefficients(lp, old, rf, mask, adv, 0.2, 0.04)
    assert abs(out["loss"] - loss) <= 1e-9 * max(1, abs(loss))
    assert abs(out["kl"] - kl) <= 1e-9 * max(1, abs(kl))
    assert np.array_equal(out["coefficients"], coef)
    bad = old.copy()
    bad[0, 0] = lp[0, 0] + 100
    with pytest.raises(E.EngineError) as e:
        ex.grpo_coefficients(lp, bad, rf, mask, rewards, G, n, 0.2, 0.04)
    assert e.value.name == "numerical_error"


def tiny_rollouts(pol):
    prng, srng = O.Rng(2), O.Rng(1)
    prompts = np.array([[prng.bounded(256) for _ in range(16)] for _ in range(2)], np.uint16)
    prompts = np.repeat(prompts, 4, axis=0)
    seeds = np.array([srng.next() for _ in range(8)], np.uint64)
    return prompts, seeds, pol.rollout(prompts, 32, 48, seeds, 1.0)


def test_tiny_rollout_semantics_and_old_logprobs():
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    W = E.init_params(TINY, 0)
    pol = E.make_execution(TINY, W, optimizer=AdamWConfig())
    prompts, seeds, r = tiny_rollouts(pol)
    s = ref.Session(TINY, 0)
    for i in range(8):
        L = int(r["lengths"][i])
        toks = r["tokens"][i, :L]
        assert 1 <= L <= 32
        assert (toks[:-1] != TINY.eos_id).all()
        if L < 32:
            assert toks[-1] == TINY.eos_id
        inp, tgt, mask = ref.completion_batch(prompts[i], toks, 48, TINY.pad_id)
        assert np.array_equal(inp, r["input"][i]) and np.array_equal(tgt, r["target"][i])
        assert np.array_equal(mask, r["mask"][i])
        want = s.log_probs(inp, tgt, mask, 1, 48)
        assert np.abs((r["old_lp"][i] - want)[mask > 0]).max() < 2e-3


def test_tiny_grpo_step_matches_reference():
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    W = E.init_params(TINY, 0)
    W1 = E.init_params(TINY, 1)  # a frozen reference that differs, so the KL term is real
    opt = AdamWConfig()
    pol = E.make_execution(TINY, W, optimizer=opt)
    refm = E.make_execution(TINY, W1)
    prompts, seeds, r = tiny_rollouts(pol)
    # old log-probs off the current policy, identical on both sides: ratios != 1
    old = (r["old_lp"] + np.random.default_rng(5).normal(0, 0.05, r["old_lp"].shape)).astype(np.float32)
    rr = O.Rng(3)
    rewards = np.array([1.0 if rr.uniform() < 0.5 else 0.0 for _ in range(8)], np.float32)
    rewards[0], rewards[1] = 0.0, 1.0  # a measurable signal in both groups
    rewards[4], rewards[5] = 1.0, 0.0
    out = pol.grpo_step(refm, r["input"], r["target"], r["mask"], old, rewards, 4,
                        clip=0.2, klc=0.04, learning_rate=1e-4)
    ps = ref.Session(TINY, 0, optimizer=opt.as_list())
    rs = ref.Session(TINY, 1)
    want = ref.grpo_update(ps, rs, 4, r["input"], r["target"], r["mask"], old, rewards,
                           0.2, 0.04, 1e-4)
    assert not out["skipped"] and not want["skipped"]
    assert abs(out["loss"] - want["loss"]) <= 1e-3 * abs(want["loss"])
    assert abs(out["grad_norm"] - want["grad_norm"]) <= 1e-3 * want["grad_norm"]
    assert abs(out["kl"] - want["kl"]) <= 1e-3 * abs(want["kl"])
    after = pol.synchronize_to_host()
    assert after["steps"] == 1
    assert np.abs(after["params"] - ps.params()).max() <= 2.05e-4


def test_constant_rewards_skip_the_update():
    require_gpu()
    W = E.init_params(TINY, 0)
    pol = E.make_execution(TINY, W, optimizer=AdamWConfig())
    refm = E.make_execution(TINY, W)
    prompts, seeds, r = tiny_rollouts(pol)
    out = pol.grpo_step(refm, r["input"], r["target"], r["mask"], r["old_lp"],
                        np.ones(8, np.float32), 4)
    assert out["skipped"]
    after = pol.synchronize_to_host()
    assert after["steps"] == 0 and np.array_equal(after["params"], W)
