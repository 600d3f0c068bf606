"""Pins the CPU checker (oracle/) to the reference: the numpy restatement against the
reference's own golden vectors and against the reference CPU build, plus the reference
unit tests' known answers for the GRPO helpers (tests/test_training.cpp:135-172,
tests/test_ops.cpp:37-47 in the reference)."""
import json
import math

import numpy as np
import pytest

from cpp_inference_train_engine_b200.config import ModelConfig, TINY
from oracle import mla_oracle as O
from oracle import ref

needs_ref = pytest.mark.skipif(not ref.available(), reason="oracle/_ref not built")


def golden_setup(golden):
    cfg = ModelConfig.from_json(json.loads(str(golden["config"])))
    names = list(golden["param_names"])
    P = O.Params(cfg, [golden["t:" + n + ".weight"].astype(np.float32) for n in names])
    return cfg, names, P


def test_restatement_matches_golden_logits_loss_grads(golden):
    cfg, names, P = golden_setup(golden)
    x, t, m = golden["input"], golden["targets"], golden["mask"]
    f = O.Forward(cfg, P, x, 1, len(x))
    assert np.abs(f.logits - golden["t:logits"]).max() < 2e-5
    coef = m / m.sum()
    loss, grads = O.accumulate(cfg, P, x, t, coef, 1, len(x))
    assert abs(loss - float(golden["loss"])) < 1e-5
    for n, g in zip(names, grads):
        want = golden["t:" + n + ".gradient"]
        assert np.abs(g - want).max() < 1e-4 * max(1.0, np.abs(want).max()), n


def test_restatement_adamw_matches_golden_update(golden):
    cfg, names, P = golden_setup(golden)
    params = [a.copy() for a in P.t]
    grads = [golden["t:" + n + ".gradient"].astype(np.float32) for n in names]
    m = [np.zeros_like(a) for a in params]
    v = [np.zeros_like(a) for a in params]
    norm, steps = O.adamw_step(cfg, params, grads, m, v, 0, float(golden["learning_rate"]),
                               list(golden["optimizer"]))
    assert steps == 1 and norm > 1.0
    for n, p in zip(names, params):
        assert np.abs(p - golden["t:" + n + ".updated"]).max() < 2e-6, n


@needs_ref
def test_reference_build_reproduces_golden(golden):
    cfg, names, P = golden_setup(golden)
    s = ref.Session(cfg, 0, optimizer=list(golden["optimizer"]))
    s.set_params(np.concatenate([a.ravel() for a in P.t]))
    x, t, m = golden["input"], golden["targets"], golden["mask"]
    assert np.abs(s.forward(x, 1, len(x)) - golden["t:logits"]).max() < 1e-5
    s.zero_grad()
    loss = s.accumulate(x, t, m, m / m.sum(), 1, len(x))
    assert abs(loss - float(golden["loss"])) < 1e-6
    G = np.concatenate([golden["t:" + n + ".gradient"].ravel() for n in names])
    assert np.abs(s.grads() - G).max() < 1e-5
    s.update(float(golden["learning_rate"]))
    U = np.concatenate([golden["t:" + n + ".updated"].ravel() for n in names])
    assert np.abs(s.params() - U).max() < 2e-6


@needs_ref
def test_rng_matches_reference():
    a, b = O.Rng(12345), ref.Rng(12345)
    for _ in range(50):
        assert a.next() == b.next()
    for _ in range(50):
        assert a.uniform() == b.uniform()
    for bound in (1, 7, 256, 16384, 3 ** 30):
        assert a.bounded(bound) == b.bounded(bound)
    for _ in range(20):
        assert abs(a.normal() - b.normal()) < 1e-6
    # The counter form used on the device equals the sequential stream.
    seq = O.Rng(99)
    for k in range(10):
        assert O.counter_uniform(99, k) == seq.uniform()


@needs_ref
def test_init_params_matches_reference_model_create():
    s = ref.Session(TINY, 7)
    want = s.params()
    got = np.concatenate([a.ravel() for a in O.init_params(TINY, 7)])
    assert np.abs(got - want).max() < 1e-6


@needs_ref
def test_forward_backward_matches_reference_random_model():
    cfg = TINY
    s = ref.Session(cfg, 3, optimizer=[0.9, 0.95, 1e-8, 0.1, 1.0])
    P = O.Params(cfg, O.split_params(cfg, s.params()))
    rng = np.random.default_rng(0)
    B, S = 2, 12
    x = rng.integers(0, cfg.vocab_size, (B, S)).astype(np.uint16)
    t = rng.integers(0, cfg.vocab_size, (B, S)).astype(np.uint16)
    m = (rng.random((B, S)) < 0.7).astype(np.float32)
    coef = (m * rng.normal(size=(B, S)) * 0.1).astype(np.float32)
    assert np.abs(O.log_probabilities(cfg, P, x, t, B, S) -
                  s.log_probs(x, t, m, B, S)).max() < 2e-5
    s.zero_grad()
    loss_ref = s.accumulate(x, t, m, coef, B, S)
    loss, grads = O.accumulate(cfg, P, x, t, coef, B, S)
    assert abs(loss - loss_ref) < 1e-5 * max(1, abs(loss_ref))
    G = s.grads()
    assert np.abs(np.concatenate([g.ravel() for g in grads]) - G).max() < 1e-5


@needs_ref
def test_decoder_matches_reference_decoder():
    cfg = TINY
    s = ref.Session(cfg, 5)
    P = O.Params(cfg, O.split_params(cfg, s.params()))
    d = O.Decoder(cfg, P)
    ids = [1, 2, 3, 4, 5]
    assert np.abs(d.prefill(ids) - s.prefill(ids)).max() < 2e-5
    for tok in [7, 200, 9, 263, 0, 15]:
        assert np.abs(d.decode(tok) - s.decode(tok)).max() < 2e-5


@needs_ref
def test_sampler_matches_reference():
    rng = np.random.default_rng(1)
    for trial in range(40):
        n = int(rng.integers(2, 300))
        lg = (rng.normal(size=n) * rng.uniform(0.1, 4)).astype(np.float32)
        if trial % 5 == 0:
            lg[rng.integers(0, n, 5)] = lg.max()  # ties
        seed = int(rng.integers(0, 2 ** 63))
        for temp in (0.0, 1.0, 0.7):
            tok, st = ref.sample_token(lg, seed, temperature=temp)
            u = O.Rng(seed).uniform() if temp > 0 else 0.0
            assert O.sample_token(lg, u, temp) == tok
            assert st == (seed if temp == 0 else (seed + 0x9E3779B97F4A7C15) % 2 ** 64)


def test_grpo_known_answers():
    # tests/test_training.cpp:135-161 of the reference.
    for adv in (-1.0, 1.0):
        for lp in (-2.1, -1.95, -1.5, -2.5):
            o = O.grpo_objective(lp, -2, -2.2, adv, 0.2, 0.02)
            e = 0.0005
            num = (O.grpo_objective(lp + e, -2, -2.2, adv, 0.2, 0.02)[0] -
                   O.grpo_objective(lp - e, -2, -2.2, adv, 0.2, 0.02)[0]) / (2 * e)
            assert abs(num + o[2]) < 3e-4
    assert O.grpo_objective(-1, -2, -1, 1, 0.2, 0)[2] == 0
    assert O.grpo_objective(0, -100, 0, 1, 0.2, 0) is None
    a = O.group_advantages([0, 1, 1, 0])
    assert abs(a[0] + 1) < 1e-5 and abs(a[1] - 1) < 1e-5
    assert all(x == 0 for x in O.group_advantages([1, 1, 1]))
    # tests/test_training.cpp:162-172.
    i, t, m = O.completion_batch([1, 2, 3], [4, 5], 6, 0)
    assert list(m) == [0, 0, 1, 1, 0, 0] and list(t) == [2, 3, 4, 5, 0, 0]
    with pytest.raises(ValueError):
        O.completion_batch([1, 2, 3], [4, 5], 3, 0)
    assert abs(O.cosine_learning_rate(0, 100, 10, 0.001, 0.1) - 0.0001) < 1e-9
    assert abs(O.cosine_learning_rate(9, 100, 10, 0.001, 0.1) - 0.001) < 1e-9
    assert abs(O.cosine_learning_rate(100, 100, 10, 0.001, 0.1) - 0.0001) < 1e-9
    # tests/test_ops.cpp:37-47: stable cross-entropy and the prompt mask.
    lg = np.array([[1000, 999, 998], [-999, -1000, -1001]], np.float32)
    loss, _, g = O.weighted_nll(lg, np.array([0, 1]), np.array([0, 1], np.float32), True)
    assert abs(loss - 1.407605964) < 1e-6
    assert (g[0] == 0).all() and abs(g[1].sum()) < 1e-7


@needs_ref
def test_grpo_helpers_match_reference():
    rng = np.random.default_rng(2)
    for _ in range(200):
        lp, old, rf = rng.normal(-3, 1, 3)
        adv = rng.normal()
        want = ref.grpo_objective(lp, old, rf, adv, 0.2, 0.04)
        got = O.grpo_objective(lp, old, rf, adv, 0.2, 0.04)
        assert got[0] == pytest.approx(want[0], abs=1e-12)
        assert np.float32(got[2]) == want[2]
    for g in range(20):
        r = (rng.random(8) < 0.4).astype(np.float32) if g % 2 else rng.normal(size=8)
        assert np.array_equal(O.group_advantages(r), ref.group_advantages(r))
    for done in range(0, 120, 7):
        assert O.cosine_learning_rate(done, 100, 10, 1e-3, 0.1) == ref.cosine_lr(done, 100, 10, 1e-3, 0.1)


@needs_ref
def test_tiny_grpo_update_matches_reference():
    """Config 1 shapes (2 prompts x group 4, prompt 16, 32 new tokens, S=48) through the
    restated rollout + update on both checkers."""
    cfg = TINY
    opt = [0.9, 0.95, 1e-8, 0.1, 1.0]
    pol = ref.Session(cfg, 0, optimizer=opt)
    refm = ref.Session(cfg, 0)
    P = O.Params(cfg, O.split_params(cfg, pol.params()))
    prng, srng = O.Rng(2), O.Rng(1)
    S, G, n_prompts = 48, 4, 2
    rolls = []
    for _ in range(n_prompts):
        prompt = [prng.bounded(256) for _ in range(16)]
        for _ in range(G):
            r = pol.rollout(prompt, 32, S, cfg.eos_id, cfg.pad_id, srng.next())
            rolls.append(r)
    inp = np.stack([r["input"] for r in rolls])
    tgt = np.stack([r["target"] for r in rolls])
    mask = np.stack([r["mask"] for r in rolls])
    old = np.stack([r["old_lp"] for r in rolls])
    lp = O.log_probabilities(cfg, P, inp, tgt, len(rolls), S).reshape(len(rolls), S)
    assert np.abs((lp - old)[mask > 0]).max() < 2e-5
    rewards = np.array([1.0 if O.Rng(3 + i).uniform() < 0.5 else 0.0 for i in range(8)],
                       np.float32)
    rewards[:2] = [0, 1]
    # the reference's own current and frozen log-probs, as its update body computes them
    n = len(rolls)
    cur = pol.log_probs(inp, tgt, mask, n, S).reshape(n, S)
    frozen = refm.log_probs(inp, tgt, mask, n, S).reshape(n, S)
    out = ref.grpo_update(pol, refm, G, inp, tgt, mask, old, rewards, 0.2, 0.04, 1e-4)
    adv = np.concatenate([O.group_advantages(rewards[g * G:(g + 1) * G]) for g in range(2)])
    assert np.array_equal(adv, out["advantages"])
    loss, kl, coef = O.grpo_coefficients(lp, old, lp, mask, adv, 0.2, 0.04)
    assert abs(loss - out["loss"]) < 1e-5 and abs(kl - out["kl"]) < 1e-6
    # on the reference's own log-probs the restated coefficients are the reference's, bit for
    # bit (float objective coefficient / double denominator, trainer.cpp:842-843)
    loss, kl, coef = O.grpo_coefficients(cur, old, frozen, mask, adv, 0.2, 0.04)
    assert np.array_equal(coef, out["coefficients"])
    assert loss == pytest.approx(out["loss"], rel=1e-12, abs=1e-15)
    assert kl == pytest.approx(out["kl"], rel=1e-12, abs=1e-15)


@needs_ref
def test_dpo_objective_matches_reference():
    rng = np.random.default_rng(4)
    for k in range(300):
        c, r, rc, rr = rng.normal(-40, 15, 4)
        beta = [0.1, 0.5, 2.0][k % 3]
        if k % 10 == 0:  # large margins exercise the stable softplus branches
            c += 400 * (1 if k % 20 else -1)
        want = ref.dpo_objective(c, r, rc, rr, beta)
        got = O.dpo_objective(c, r, rc, rr, beta)
        assert got[0] == pytest.approx(want[0], rel=1e-12, abs=1e-300)
        assert got[1] == want[1]
        assert np.float32(got[2]) == np.float32(want[2]) and np.float32(got[3]) == np.float32(want[3])


@needs_ref
def test_tiny_dpo_update_matches_reference():
    """Preference pairs through the reference's DPO update body (restated over its public API)
    against the numpy restatement's objective and coefficients on the same log-probs."""
    cfg = TINY
    opt = [0.9, 0.95, 1e-8, 0.1, 1.0]
    pol = ref.Session(cfg, 0, optimizer=opt)
    refm = ref.Session(cfg, 1)
    rng = np.random.default_rng(8)
    n, S = 3, 32
    inp = rng.integers(0, 256, (2 * n, S)).astype(np.uint16)
    tgt = rng.integers(0, 256, (2 * n, S)).astype(np.uint16)
    mask = np.zeros((2 * n, S), np.float32)
    for row in range(2 * n):
        mask[row, 10:10 + 4 + 3 * row] = 1
    ones = np.ones((2 * n, S), np.float32)
    lp = pol.log_probs(inp, tgt, ones, 2 * n, S).reshape(2 * n, S)
    rl = refm.log_probs(inp, tgt, ones, 2 * n, S).reshape(2 * n, S)
    loss, margins, _ = O.dpo_coefficients(lp, rl, mask, 0.1)
    out = ref.dpo_update(pol, refm, inp, tgt, mask, 0.1, 1e-3)
    assert abs(out["loss"] - loss) < 1e-12 * max(1.0, abs(loss))
    np.testing.assert_allclose(out["margins"], margins, rtol=0, atol=1e-9)
    assert pol.steps == 1
