"""Device-state checkpoint/resume and run-to-run determinism of the GRPO step on the GPU.

The reference checkpoints a GPU run by `synchronize_to_host` into its host Model/Optimizer
and `save_checkpoint`, and resumes by `load_checkpoint` and a fresh execution over those
host tensors (trainer.cpp:536-577); its replay test demands byte-identical weights and
moments (tests/test_tools.py:560-567). Here the host side of that round trip is the
download (params, moments, step count) and upload of the C ABI, and:
  * the same GRPO step (rollout + update) from the same state, twice, gives bit-identical
    weights, moments and step count and identical loss / KL / gradient norm;
  * two steps in one execution equal one step, a download, a fresh execution with that state
    uploaded, and the second step there — bit for bit.
Every reduction on the update path has a fixed order (split-K partials, norm-weight
partials, AdamW norm, GRPO loss/KL partials) or is exact (the embedding-gather gradient in
64-bit fixed point), which is what makes this hold."""
import numpy as np
import pytest

import cpp_inference_train_engine_b200 as E
from cpp_inference_train_engine_b200.config import MLA36M, TINY, AdamWConfig
from tests.gpu_util import require_gpu

pytestmark = pytest.mark.gpu

CASES = {
    # cfg, rollouts, group, prompt length, new tokens
    "tiny": (TINY, 16, 4, 8, 24),
    "36m": (MLA36M, 16, 8, 32, 48),
}


def _inputs(cfg, n, prompt, k):
    rng = np.random.default_rng(1000 + k)
    hi = min(cfg.vocab_size - 8, 256) if cfg is TINY else cfg.vocab_size - 8
    prompts = rng.integers(0, hi, (n, prompt)).astype(np.uint16)
    seeds = rng.integers(0, 2 ** 63, n).astype(np.uint64)
    rewards = rng.uniform(size=n).astype(np.float32)  # never a constant group
    return prompts, seeds, rewards


def _run(case, steps, state=None):
    cfg, n, G, prompt, new = CASES[case]
    W0 = E.init_params(cfg, 0)
    if state is None:
        pol = E.make_execution(cfg, W0, optimizer=AdamWConfig())
    else:
        pol = E.make_execution(cfg, state["params"], optimizer=AdamWConfig(), moments=(state["m"], state["v"]),
                               steps=state["steps"])
    ref = E.make_execution(cfg, W0)  # the frozen reference: the initial weights
    outs = []
    for k in steps:
        prompts, seeds, rewards = _inputs(cfg, n, prompt, k)
        r = pol.rollout(prompts, new, prompt + new, seeds, 1.0)
        outs.append(pol.grpo_step(ref, r["input"], r["target"], r["mask"], r["old_lp"], rewards, G,
                                  clip=0.2, klc=0.04, learning_rate=1e-4))
        outs[-1]["tokens"] = r["tokens"].copy()
    st = pol.synchronize_to_host(params=True, moments=True)
    pol.close()
    ref.close()
    return outs, st


def _same_state(a, b):
    assert a["steps"] == b["steps"]
    for key in ("params", "m", "v"):
        np.testing.assert_array_equal(a[key].view(np.uint32), b[key].view(np.uint32), err_msg=key)


@pytest.mark.parametrize("case", sorted(CASES))
def test_grpo_step_is_deterministic(case):
    require_gpu()
    o1, s1 = _run(case, [0])
    o2, s2 = _run(case, [0])
    assert not o1[0]["skipped"]
    np.testing.assert_array_equal(o1[0]["tokens"], o2[0]["tokens"])
    for key in ("loss", "kl", "grad_norm"):
        assert o1[0][key] == o2[0][key], key
    _same_state(s1, s2)
    assert s1["steps"] == 1


@pytest.mark.parametrize("case", sorted(CASES))
def test_resume_from_downloaded_state_replays_bit_exact(case):
    require_gpu()
    straight, s_straight = _run(case, [0, 1])
    first, s_first = _run(case, [0])
    resumed, s_resumed = _run(case, [1], state=s_first)
    assert s_first["steps"] == 1 and s_resumed["steps"] == 2
    np.testing.assert_array_equal(straight[1]["tokens"], resumed[0]["tokens"])
    for key in ("loss", "kl", "grad_norm"):
        assert straight[1][key] == resumed[0][key], key
    _same_state(s_straight, s_resumed)
