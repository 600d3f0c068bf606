"""Continuous batching (cpp_inference_train_engine_b200.serving.Server over mm_cuda_serve_*)
against the reference's one-request generation (generate_tokens, inference.cpp:469-579, as
CpuDecoder prefill/decode + sample_token at top_p 1): seven requests of different prompt
lengths and token budgets arrive in two waves over three slots, so requests are queued,
admitted into freed slots and decoded beside others at different positions. Greedy tokens
must equal the reference's one-request generation step for step wherever the reference's
top-2 logit margin exceeds 1e-3 (the parity gate for greedy tokens); the comparison stops
at the first narrower margin. Sampled (T = 1) generation is reproducible run to run."""
import numpy as np
import pytest

import cpp_inference_train_engine_b200 as E
from cpp_inference_train_engine_b200.config import MLA36M, TINY
from cpp_inference_train_engine_b200.serving import Server
from oracle import ref
from tests.gpu_util import require_gpu

pytestmark = pytest.mark.gpu

CASES = {"tiny": (TINY, 3), "36m": (MLA36M, 3)}


def _requests(cfg, seed):
    rng = np.random.default_rng(seed)
    hi = min(256, cfg.vocab_size - 8)
    out = []
    for i in range(7):
        n = int(rng.integers(3, 21))
        out.append((rng.integers(0, hi, n).astype(np.uint16), int(rng.integers(2, 18)), int(rng.integers(1, 2 ** 62))))
    return out


def _reference_greedy(cfg, W_seed, prompt, max_new, eos):
    """generate_tokens at temperature 0: tokens and the top-2 margin behind each."""
    s = ref.Session(cfg, W_seed)
    logits = s.prefill(prompt)
    toks, margins = [], []
    for i in range(max_new):
        top2 = np.sort(logits)[-2:]
        margins.append(float(top2[1] - top2[0]))
        t = int(np.argmax(logits))
        toks.append(t)
        if t == eos or i + 1 == max_new:
            break
        logits = s.decode(t)
    s.close()
    return toks, margins


def _serve(cfg, reqs, slots, temperature):
    ex = E.make_execution(cfg, E.init_params(cfg, 3))
    srv = Server(ex, slots, temperature=temperature)
    ids = [srv.submit(p, m, seed=sd) for p, m, sd in reqs[:4]]
    for _ in range(3):
        srv.step()
    ids += [srv.submit(p, m, seed=sd) for p, m, sd in reqs[4:]]
    done = srv.run()
    ex.close()
    return [done[i] for i in ids]


@pytest.mark.parametrize("case", sorted(CASES))
def test_greedy_serving_matches_reference_generation(case):
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    cfg, slots = CASES[case]
    reqs = _requests(cfg, 40)
    eos = cfg.vocab_size - 6
    got = _serve(cfg, reqs, slots, 0.0)
    compared = 0
    for (prompt, max_new, _), r in zip(reqs, got):
        want, margins = _reference_greedy(cfg, 3, prompt, max_new, eos)
        for i, (a, m) in enumerate(zip(want, margins)):
            if m <= 1e-3:
                break
            assert r.tokens[i] == a, (list(prompt), i, r.tokens, want)
            compared += 1
        else:
            assert r.tokens == want
            assert r.finish_reason == ("stop" if want[-1] == eos else "length")
        assert 1 <= len(r.tokens) <= max_new
    assert compared >= 20


def test_sampled_serving_is_reproducible():
    require_gpu()
    reqs = _requests(TINY, 41)
    a = _serve(TINY, reqs, 3, 1.0)
    b = _serve(TINY, reqs, 3, 1.0)
    assert [r.tokens for r in a] == [r.tokens for r in b]
    assert all(0 <= t < TINY.vocab_size for r in a for t in r.tokens)
