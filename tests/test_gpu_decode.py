"""Batched latent-cache decode and the on-device sampler against the reference's
CpuDecoder and sample_token."""
import dataclasses

import numpy as np
import pytest

import cpp_inference_train_engine_b200 as E
from cpp_inference_train_engine_b200.config import MLA36M, TINY
from oracle import mla_oracle as O
from oracle import ref
from tests.gpu_util import require_gpu

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=["tiny", "36m"])
def setup(request):
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    cfg = TINY if request.param == "tiny" else MLA36M
    W = E.init_params(cfg, 3)
    return cfg, W, E.make_execution(cfg, W)


def test_prefill_and_decode_match_reference_decoder(setup):
    cfg, W, ex = setup
    rng = np.random.default_rng(1)
    B, P, steps = 3, 17, 12
    prompts = rng.integers(0, min(256, cfg.vocab_size), (B, P)).astype(np.uint16)
    sessions = [ref.Session(cfg, 3) for _ in range(B)]
    want = np.stack([s.prefill(prompts[b]) for b, s in enumerate(sessions)])
    got = ex.prefill_batch(prompts)
    tol = 5e-3 if cfg is TINY else 2e-2
    assert np.abs(got - want).max() < tol
    agree = total = 0
    for k in range(steps):
        # teacher-force the reference's greedy choice so one divergence cannot compound
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
        assert np.abs(got - want).max() < tol, k
    assert agree == total


@pytest.mark.parametrize("B,P,steps", [(2, 300, 6), (300, 24, 3)])
def test_36m_decode_split_and_wide_batches(B, P, steps):
    """Long contexts over few rows take the split-context path; >= 296 rows the one-CTA-per
    row path. Rows 0, B/2 and B-1 are checked against the reference decoder."""
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    W = E.init_params(MLA36M, 3)
    ex = E.make_execution(MLA36M, W)
    rng = np.random.default_rng(B)
    prompts = rng.integers(0, 16384, (B, P)).astype(np.uint16)
    rows = sorted({0, B // 2, B - 1})
    sessions = {r: ref.Session(MLA36M, 3) for r in rows}
    got = ex.prefill_batch(prompts)
    want = {r: s.prefill(prompts[r]) for r, s in sessions.items()}
    for k in range(steps):
        for r in rows:
            assert np.abs(got[r] - want[r]).max() < 2e-2, (k, r)
        tok = got.argmax(axis=1).astype(np.uint16)
        for r in rows:
            tok[r] = np.uint16(want[r].argmax())
        want = {r: s.decode(tok[r]) for r, s in sessions.items()}
        got = ex.decode_batch(tok)


def test_sampler_matches_reference_sample_token():
    require_gpu()
    # 261: a vocabulary that is not a multiple of 4 takes the scalar row loads
    execs = {264: E.CudaExecution(TINY), 16384: E.CudaExecution(MLA36M),
             261: E.CudaExecution(dataclasses.replace(TINY, vocab_size=261))}
    rng = np.random.default_rng(7)
    for V in (264, 261, 16384):
        ex = execs[V]
        B = 64
        logits = (rng.normal(size=(B, V)) * rng.uniform(0.2, 3, size=(B, 1))).astype(np.float32)
        logits[::7, :50] = logits[::7, :50].max()  # ties
        seeds = rng.integers(0, 2 ** 63, B).astype(np.uint64)
        draws = rng.integers(0, 300, B).astype(np.int32)
        for temp in (1.0, 0.7, 0.0):
            got = ex.sample(logits, temp, seeds, draws)
            for b in range(B):
                st = (int(seeds[b]) + int(draws[b]) * 0x9E3779B97F4A7C15) % 2 ** 64
                tok, _ = ref.sample_token(logits[b], st, temperature=temp)
                assert got[b] == tok, (V, temp, b)


def test_sampler_crowded_and_tied_rows():
    """Rows whose crossing lands among crowded or exactly tied scores: a distant maximum
    beside a tight cluster (more than 1024 scores per equal-width bucket), whole rows of one
    value, and 3000 exact ties inside a spread row."""
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    ex = E.CudaExecution(MLA36M)
    V, B = 16384, 48
    rng = np.random.default_rng(11)
    logits = np.empty((B, V), np.float32)
    for b in range(B):
        kind = b % 4
        if kind == 0:  # distant maximum, cluster of width 1e-3
            row = rng.uniform(0, 1e-3, V)
            row[rng.integers(V)] = 3.0
        elif kind == 1:  # one value everywhere
            row = np.full(V, 0.25)
        elif kind == 2:  # 3000 exact ties at a mid-range value
            row = rng.normal(size=V) * 0.5
            row[rng.choice(V, 3000, replace=False)] = 0.0
        else:  # ties at the maximum
            row = rng.normal(size=V)
            row[rng.choice(V, 2000, replace=False)] = row.max()
        logits[b] = row
    seeds = rng.integers(0, 2 ** 63, B).astype(np.uint64)
    draws = rng.integers(0, 300, B).astype(np.int32)
    for temp in (1.0, 0.3):
        got = ex.sample(logits, temp, seeds, draws)
        for b in range(B):
            st = (int(seeds[b]) + int(draws[b]) * 0x9E3779B97F4A7C15) % 2 ** 64
            tok, _ = ref.sample_token(logits[b], st, temperature=temp)
            assert got[b] == tok, (temp, b)
    ex.close()
