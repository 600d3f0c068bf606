"""Teacher-forced forward, weighted-NLL backward and AdamW on the GPU against the
reference: its golden vectors (tiny config) and its CPU build (35.8M config).
Tolerances: log-probs 2e-3 absolute; loss and gradient norm 1e-3 relative."""
import numpy as np
import pytest

import cpp_inference_train_engine_b200 as E
from cpp_inference_train_engine_b200.config import MLA36M, AdamWConfig
from oracle import mla_oracle as O
from oracle import ref
from tests.gpu_util import golden_model, rel, require_gpu

pytestmark = pytest.mark.gpu


def lp_from_logits(logits, targets):
    _, lp, _ = O.weighted_nll(logits, np.asarray(targets, np.int64), np.zeros(len(targets)))
    return lp


@pytest.fixture(scope="module")
def golden_exec(golden):
    require_gpu()
    cfg, names, W = golden_model(golden)
    opt = AdamWConfig(*[float(x) for x in golden["optimizer"]])
    return cfg, names, W, E.make_execution(cfg, W, optimizer=opt)


def test_golden_forward_logprobs(golden, golden_exec):
    cfg, names, W, ex = golden_exec
    x, t = golden["input"], golden["targets"]
    logits = ex.forward(x, 1, len(x))
    want = golden["t:logits"]
    assert np.abs(logits - want).max() < 2e-2
    assert np.abs(lp_from_logits(logits, t) - lp_from_logits(want, t)).max() < 2e-3
    lp = ex.log_probabilities(x, t, 1, len(x))
    assert np.abs(lp - lp_from_logits(want, t)).max() < 2e-3


def test_golden_loss_gradients_and_adamw(golden, golden_exec):
    cfg, names, W, ex = golden_exec
    x, t, m = golden["input"], golden["targets"], golden["mask"]
    ex.upload(W)
    ex.zero_grad()
    loss = ex.accumulate(x, t, m / m.sum(), 1, len(x))
    assert abs(loss - float(golden["loss"])) <= 1e-3 * abs(float(golden["loss"]))
    st = ex.synchronize_to_host(params=False, grads=True)
    G = np.concatenate([golden["t:" + n + ".gradient"].ravel() for n in names])
    assert abs(np.linalg.norm(st["grads"]) / np.linalg.norm(G) - 1) < 1e-3
    assert rel(st["grads"], G) < 2e-2
    # AdamW on the device's own gradients must equal the reference update of them.
    norm = ex.update(float(golden["learning_rate"]))
    assert abs(norm / np.linalg.norm(G.astype(np.float64)) - 1) < 1e-3
    after = ex.synchronize_to_host(params=True, moments=True)
    params = O.split_params(cfg, W.copy())
    grads = O.split_params(cfg, st["grads"])
    mm = [np.zeros_like(a) for a in params]
    vv = [np.zeros_like(a) for a in params]
    O.adamw_step(cfg, params, grads, mm, vv, 0, float(golden["learning_rate"]),
                 list(golden["optimizer"]))
    want = np.concatenate([p.ravel() for p in params])
    diff = np.abs(after["params"] - want)
    ulp = np.spacing(np.abs(want).astype(np.float32))
    assert (diff <= ulp).all(), float((diff / ulp).max())
    assert after["steps"] == 1
    # and close to the reference's golden update. AdamW's first step moves every weight by
    # about lr * sign(g), so only gradients well above the fp16 noise have a defined sign.
    U = np.concatenate([golden["t:" + n + ".updated"].ravel() for n in names])
    lr = float(golden["learning_rate"])
    assert np.abs(after["params"] - U).max() <= 2.05 * lr
    firm = np.abs(G) > 1e-2 * np.abs(G).max()
    assert np.abs(after["params"] - U)[firm].max() < 0.05 * lr


@pytest.fixture(scope="module")
def big():
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    W = E.init_params(MLA36M, 0)
    s = ref.Session(MLA36M, 0, optimizer=AdamWConfig().as_list())
    ex = E.make_execution(MLA36M, W, optimizer=AdamWConfig())
    return W, s, ex


def test_36m_log_probs_match_reference(big):
    W, s, ex = big
    rng = O.Rng(4)
    B, S = 2, 96
    ids = np.array([[rng.bounded(16384) for _ in range(S + 1)] for _ in range(B)], np.uint16)
    x, t = ids[:, :-1], ids[:, 1:]
    want = s.log_probs(x, t, np.ones((B, S), np.float32), B, S)
    got = ex.log_probabilities(x, t, B, S)
    assert np.abs(got - want).max() < 2e-3


def test_36m_gradient_norm_matches_reference(big):
    W, s, ex = big
    rng = np.random.default_rng(9)
    B, S = 2, 64
    x = rng.integers(0, 16384, (B, S)).astype(np.uint16)
    t = rng.integers(0, 16384, (B, S)).astype(np.uint16)
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
