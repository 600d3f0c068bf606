"""DPO on the GPU (mm_cuda_dpo_step) against the reference's own DPO update body
(trainer.cpp:765-783 with preference_objective :107-121 and dpo_objective :345-350, run by
oracle/_ref on its CPU path) on the same preference pairs: rows 2p (chosen) and 2p + 1
(rejected), masks on the completion tokens, policy and frozen reference from different seeds so
the margins are not zero. Tolerances as the GRPO gates: loss and pre-clip gradient norm 1e-3
relative; per-pair margins (sums of ~20-60 token log-probs of two models) 2e-2 absolute; after
the AdamW step every weight within 2.05 lr of the reference's (the first step moves each by
about lr times the sign of its gradient). A second update from the same state is
bit-identical (the update path is deterministic)."""
import numpy as np
import pytest

import cpp_inference_train_engine_b200 as E
from cpp_inference_train_engine_b200.config import MLA36M, TINY, AdamWConfig
from oracle import ref
from tests.gpu_util import require_gpu

pytestmark = pytest.mark.gpu

CASES = {"tiny": (TINY, 4, 48), "36m": (MLA36M, 3, 96)}
BETA, LR = 0.1, 1e-3


def _pairs(cfg, n, S, seed):
    rng = np.random.default_rng(seed)
    hi = min(256, cfg.vocab_size - 8)
    inp = rng.integers(0, hi, (2 * n, S)).astype(np.uint16)
    tgt = rng.integers(0, hi, (2 * n, S)).astype(np.uint16)
    mask = np.zeros((2 * n, S), np.float32)
    for row in range(2 * n):
        start = int(rng.integers(4, S // 3))
        mask[row, start:start + int(rng.integers(S // 4, S // 2))] = 1
    return inp, tgt, mask


@pytest.mark.parametrize("case", sorted(CASES))
def test_dpo_step_matches_reference_update(case):
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    cfg, n, S = CASES[case]
    inp, tgt, mask = _pairs(cfg, n, S, 31)
    opt = AdamWConfig()
    rp = ref.Session(cfg, 0, optimizer=opt.as_list())
    rr = ref.Session(cfg, 1)
    want = ref.dpo_update(rp, rr, inp, tgt, mask, BETA, LR)
    W_after = rp.params()
    pol = E.make_execution(cfg, E.init_params(cfg, 0), optimizer=opt)
    refm = E.make_execution(cfg, E.init_params(cfg, 1))
    got = pol.dpo_step(refm, inp, tgt, mask, beta=BETA, learning_rate=LR)
    assert abs(got["loss"] - want["loss"]) <= 1e-3 * abs(want["loss"])
    assert abs(got["grad_norm"] - want["grad_norm"]) <= 1e-3 * want["grad_norm"]
    np.testing.assert_allclose(got["margins"], want["margins"], rtol=0, atol=2e-2)
    assert abs(got["margin"] - want["margins"].mean()) < 2e-2
    assert np.abs(want["margins"]).max() > 0.1  # a non-trivial objective
    st = pol.synchronize_to_host(params=True)
    assert st["steps"] == 1
    assert np.abs(st["params"] - W_after).max() <= 2.05 * LR


def test_dpo_step_is_deterministic():
    require_gpu()
    cfg, n, S = CASES["36m"]
    inp, tgt, mask = _pairs(cfg, n, S, 32)
    outs = []
    for _ in range(2):
        pol = E.make_execution(cfg, E.init_params(cfg, 0), optimizer=AdamWConfig())
        refm = E.make_execution(cfg, E.init_params(cfg, 1))
        o = pol.dpo_step(refm, inp, tgt, mask, beta=BETA, learning_rate=LR)
        outs.append((o, pol.synchronize_to_host(params=True, moments=True)))
        pol.close()
        refm.close()
    (a, sa), (b, sb) = outs
    assert a["loss"] == b["loss"] and a["grad_norm"] == b["grad_norm"]
    for key in ("params", "m", "v"):
        np.testing.assert_array_equal(sa[key].view(np.uint32), sb[key].view(np.uint32))
