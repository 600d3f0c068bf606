"""The sm_100a backend behind the reference's own C++ interface. The reference-side adapter
(cpp_inference_train_engine_b200/reference_adapter/cuda_execution.cpp: `class Execution`,
include/mini_mla/execution.hpp:28-61, over include/mm_cuda.h) is compiled with the
reference's unmodified CPU sources (`make -C oracle cuda`), and the reference's
Execution-API drivers -- forward, log_probabilities, rollout() (trainer.cpp:187-213) and
the GRPO update body (trainer.cpp:814-883), as restated in oracle/ref_harness.cpp -- run
once on make_execution("cpu") and once on the adapter, from the same Model::create weights.
Tolerances as the model tests: logits 2e-2 and log-probs 2e-3 absolute, loss / KL /
pre-clip gradient norm 1e-3 relative; greedy rollout tokens identical; after one AdamW step
every weight within 2.05 lr of the CPU run's (the first step moves each by about lr times
the sign of its gradient)."""
import numpy as np
import pytest

from cpp_inference_train_engine_b200.config import TINY, AdamWConfig
from oracle import mla_oracle as O
from oracle import ref
from tests.gpu_util import require_gpu

pytestmark = pytest.mark.gpu

G, N, PROMPT, S, NEW = 4, 8, 16, 48, 32


@pytest.fixture(scope="module")
def sessions():
    require_gpu()
    if not (ref.available("cpu") and ref.available("cuda")):
        pytest.skip("oracle/_ref not built with the adapter (make -C oracle cuda)")
    opt = AdamWConfig().as_list()
    mk = lambda backend, seed, o: ref.Session(TINY, seed, optimizer=o, backend=backend)
    return {b: (mk(b, 0, opt), mk(b, 1, None)) for b in ("cpu", "cuda")}


def test_forward_and_log_probs_through_the_adapter(sessions):
    rng = np.random.default_rng(5)
    x = rng.integers(0, 256, (2, 40)).astype(np.uint16)
    t = rng.integers(0, 256, (2, 40)).astype(np.uint16)
    m = np.ones((2, 40), np.float32)
    cpu, gpu = sessions["cpu"][0], sessions["cuda"][0]
    assert np.abs(gpu.forward(x, 2, 40) - cpu.forward(x, 2, 40)).max() < 2e-2
    assert np.abs(gpu.log_probs(x, t, m, 2, 40) - cpu.log_probs(x, t, m, 2, 40)).max() < 2e-3


def test_host_weight_edit_reaches_the_device(sessions):
    rng = np.random.default_rng(6)
    x = rng.integers(0, 256, (1, 24)).astype(np.uint16)
    t = rng.integers(0, 256, (1, 24)).astype(np.uint16)
    m = np.ones((1, 24), np.float32)
    cpu, gpu = sessions["cpu"][1], sessions["cuda"][1]
    W = cpu.params()
    W2 = (W * 1.5).astype(np.float32)  # Model::mark_weights_changed on both hosts
    cpu.set_params(W2)
    gpu.set_params(W2)
    try:
        assert np.abs(gpu.log_probs(x, t, m, 1, 24) - cpu.log_probs(x, t, m, 1, 24)).max() < 2e-3
    finally:
        cpu.set_params(W)
        gpu.set_params(W)


def test_grpo_round_through_the_adapter(sessions):
    eos, pad = TINY.vocab_size - 6, TINY.vocab_size - 8
    r = O.Rng(2)
    prompts = [np.array([r.bounded(256) for _ in range(PROMPT)], np.uint16) for _ in range(N)]
    rr = O.Rng(1)
    seeds = [rr.next() for _ in range(N)]
    rewards = np.array([0.1, 0.9, 0.3, 0.7, 1.0, 0.0, 0.5, 0.25], np.float32)
    res = {}
    for b in ("cpu", "cuda"):
        pol, refm = sessions[b]
        rolls = [pol.rollout(prompts[i], NEW, S, eos, pad, seeds[i], temperature=0.0) for i in range(N)]
        stack = lambda k: np.stack([x[k] for x in rolls])
        upd = ref.grpo_update(pol, refm, G, stack("input"), stack("target"), stack("mask"),
                              stack("old_lp"), rewards, 0.2, 0.04, 1e-3)
        res[b] = dict(rolls=rolls, upd=upd, params=pol.params(), steps=pol.steps)
    c, g = res["cpu"], res["cuda"]
    for a, b in zip(c["rolls"], g["rolls"]):
        np.testing.assert_array_equal(a["tokens"], b["tokens"])
        assert np.abs(a["old_lp"] - b["old_lp"]).max() < 2e-3
    assert not c["upd"]["skipped"] and not g["upd"]["skipped"]
    for key in ("loss", "kl", "grad_norm"):
        assert abs(g["upd"][key] - c["upd"][key]) <= 1e-3 * max(abs(c["upd"][key]), 1e-12), key
    assert c["steps"] == g["steps"] == 1
    assert np.abs(g["params"] - c["params"]).max() <= 2.05 * 1e-3
