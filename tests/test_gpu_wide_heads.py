"""The attention shapes of the scaled MLA model (MLA1B: 16 heads, query/key and value heads
128 wide = nope 96 + rope 32, kv rank 512, so a 544-wide latent cache row) on a reduced
width and depth, against the reference's CPU build on identical seeded weights and tokens:
the 128-wide flash forward/backward (3 query tiles), the 16-head tensor-core latent decode
attention at kv rank 512 (one pass, and split over the context with the partials merged), and
one GRPO update. Tolerances as everywhere: log-probs 2e-3 absolute, loss,
KL and gradient norm 1e-3 relative, greedy tokens equal wherever the reference's top-2
margin exceeds 1e-3."""
import numpy as np
import pytest

import cpp_inference_train_engine_b200 as E
from cpp_inference_train_engine_b200.config import AdamWConfig, ModelConfig
from oracle import mla_oracle as O
from oracle import ref
from tests.gpu_util import rel, require_gpu

pytestmark = pytest.mark.gpu

WIDE = ModelConfig(vocab_size=2048, max_sequence_length=1024, n_layers=2, d_model=256, n_heads=16,
                   head_dim_nope=96, head_dim_rope=32, head_dim_value=128, q_lora_rank=192,
                   kv_lora_rank=512, d_ff=512)


@pytest.fixture(scope="module")
def wide():
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    W = E.init_params(WIDE, 0)
    s = ref.Session(WIDE, 0, optimizer=AdamWConfig().as_list())
    ex = E.make_execution(WIDE, W, optimizer=AdamWConfig())
    return W, s, ex


def test_wide_log_probs_match_reference(wide):
    W, s, ex = wide
    rng = O.Rng(4)
    B, S = 2, 150
    ids = np.array([[rng.bounded(WIDE.vocab_size) for _ in range(S + 1)] for _ in range(B)], np.uint16)
    x, t = np.ascontiguousarray(ids[:, :-1]), np.ascontiguousarray(ids[:, 1:])
    want = s.log_probs(x, t, np.ones((B, S), np.float32), B, S)
    got = ex.log_probabilities(x, t, B, S)
    assert np.abs(got - want).max() < 2e-3


def test_wide_gradient_matches_reference(wide):
    W, s, ex = wide
    rng = np.random.default_rng(9)
    B, S = 2, 150
    x = rng.integers(0, WIDE.vocab_size, (B, S)).astype(np.uint16)
    t = rng.integers(0, WIDE.vocab_size, (B, S)).astype(np.uint16)
    coef = (rng.normal(size=(B, S)) * 1e-3).astype(np.float32)
    s.zero_grad()
    loss_ref = s.accumulate(x, t, np.ones((B, S), np.float32), coef, B, S)
    ex.zero_grad()
    loss = ex.accumulate(x, t, coef, B, S)
    assert abs(loss - loss_ref) <= 1e-3 * abs(loss_ref)
    g = ex.synchronize_to_host(params=False, grads=True)["grads"]
    G = s.grads()
    assert abs(np.linalg.norm(g) / np.linalg.norm(G) - 1) < 1e-3
    assert rel(g, G) < 2e-2


@pytest.mark.parametrize("B,P,steps", [(3, 70, 10), (2, 600, 4)])
def test_wide_decode_matches_reference_decoder(B, P, steps):
    """3 rows of 70: one work item per row. 2 rows of 600: the context is split (5 splits of
    4 tiles) and the partials merged."""
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    W = E.init_params(WIDE, 3)
    ex = E.make_execution(WIDE, W)
    rng = np.random.default_rng(1)
    prompts = rng.integers(0, 256, (B, P)).astype(np.uint16)
    sessions = [ref.Session(WIDE, 3) for _ in range(B)]
    want = np.stack([s.prefill(prompts[b]) for b, s in enumerate(sessions)])
    got = ex.prefill_batch(prompts)
    assert np.abs(got - want).max() < 2e-2
    agree = total = 0
    for k in range(steps):
        tok = want.argmax(axis=1).astype(np.uint16)
        top2 = np.sort(want, axis=1)[:, -2:]
        margin = top2[:, 1] - top2[:, 0]
        mine = got.argmax(axis=1)
        for b in range(B):
            if margin[b] > 1e-3:
                total += 1
                agree += int(mine[b] == tok[b])
        want = np.stack([s.decode(tok[b]) for b, s in enumerate(sessions)])
        got = ex.decode_batch(tok)
        assert np.abs(got - want).max() < 2e-2, k
    assert agree == total and total > 0


def test_wide_grpo_update_matches_reference():
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    G, n, P, new, S = 4, 8, 24, 40, 64
    prng, srng, rr = O.Rng(2), O.Rng(1), O.Rng(3)
    prompts = np.array([[prng.bounded(WIDE.vocab_size) for _ in range(P)] for _ in range(n // G)], np.uint16)
    prompts = np.repeat(prompts, G, axis=0)
    seeds = np.array([srng.next() for _ in range(n)], np.uint64)
    opt = AdamWConfig()
    pol = E.make_execution(WIDE, E.init_params(WIDE, 0), optimizer=opt)
    refm = E.make_execution(WIDE, E.init_params(WIDE, 1))
    r = pol.rollout(prompts, new, S, seeds, 1.0)
    for i in range(n):
        L = int(r["lengths"][i])
        inp, tgt, mask = ref.completion_batch(prompts[i], r["tokens"][i, :L], S, WIDE.pad_id)
        assert np.array_equal(inp, r["input"][i]) and np.array_equal(tgt, r["target"][i])
        assert np.array_equal(mask, r["mask"][i])
    # old log-probs off the policy's by up to a few tenths, kept clear of the clip edges
    lp = pol.log_probabilities(r["input"], r["target"], n, S).reshape(n, S)
    old = (lp + np.random.default_rng(5).normal(0, 0.3, lp.shape) * r["mask"]).astype(np.float32)
    for edge in (np.log(1.2), np.log(0.8)):
        d = lp.astype(np.float64) - old - edge
        near = (r["mask"] > 0) & (np.abs(d) < 5e-3)
        old = np.where(near, old + np.where(d >= 0, -1e-2, 1e-2), old).astype(np.float32)
    rewards = np.array([rr.normal() for _ in range(n)], np.float32)
    out = pol.grpo_step(refm, r["input"], r["target"], r["mask"], old, rewards, G, clip=0.2, klc=0.04,
                        learning_rate=1e-4)
    ps = ref.Session(WIDE, 0, optimizer=opt.as_list())
    rs = ref.Session(WIDE, 1)
    want = ref.grpo_update(ps, rs, G, r["input"], r["target"], r["mask"], old, rewards, 0.2, 0.04, 1e-4)
    assert not out["skipped"] and not want["skipped"]
    for k in ("loss", "kl", "grad_norm"):
        assert abs(out[k] - want[k]) <= 1e-3 * abs(want[k]), (k, out, want)
    after = pol.synchronize_to_host()["params"]
    assert np.abs(after - ps.params()).max() <= 2.05e-4
