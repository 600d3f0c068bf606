"""Parity of the headline GRPO path at the benchmark's own shapes, against the reference's CPU
path (oracle/_ref) on identical seeded weights and tokens.

* GRPO update at rollout shapes (35.8M model, prompt 128 + 256 new tokens, S = 384, 2 groups of
  8) with the teacher-forced passes split into 4 chunks (MM_CHUNK_TOKENS, a fresh process):
  per-chunk power-of-two backward scale, the fixed-point embedding gradient summed across
  chunks, the frozen reference's forward on its own stream beside the policy's backward, and
  host inputs in pinned memory so every host-to-device copy is truly asynchronous. Old
  log-probs are moved off the policy's so both clip branches fire; the frozen reference is a
  different init (seed 1). Loss, KL and pre-clip gradient norm within 1e-3 relative of
  the reference's update body (trainer.cpp:814-883); rollout lengths, eos stops and masks
  exact (completion_batch, trainer.cpp:386-408).
* DPO over 3 chunks of preference pairs, pinned inputs, against the reference's DPO update.
* Teacher-forced log-probs and the GRPO update at 64 x 512 (prompt mask 128), policy seed 0,
  frozen reference seed 1, rewards N(0, 1) in groups of 8: log-probs within 2e-3 absolute,
  loss / KL / gradient norm within 1e-3 relative.
* Decode after 1,024-token prompts, 128 teacher-forced greedy steps, at 64 rows and at 2,048
  rows (the size at which the step's vocabulary head runs on CTA pairs):
  the greedy token equals the reference decoder's wherever its top-2 margin exceeds 1e-3.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

import cpp_inference_train_engine_b200 as E
from cpp_inference_train_engine_b200.config import MLA36M, AdamWConfig
from oracle import mla_oracle as O
from oracle import ref
from tests.gpu_util import ROOT, require_gpu

pytestmark = pytest.mark.gpu

PROMPT, NEW, SEQ, G, N_ROLL = 128, 256, 384, 8, 16


def _pin(a):
    """A copy of `a` in page-locked host memory: a numpy view of a pinned torch buffer (the
    view's base keeps the buffer alive), so the engine's host-to-device copies run
    asynchronously to the host."""
    import torch
    a = np.ascontiguousarray(a)
    t = torch.empty(a.size * a.itemsize, dtype=torch.uint8, pin_memory=True)
    out = t.numpy().view(a.dtype).reshape(a.shape)
    out[...] = a
    return out


def _run_case(name, env):
    code = ("import json, sys; sys.path.insert(0, %r); from tests import test_gpu_headline_parity as m; "
            "print('RESULT ' + json.dumps(m.%s()))") % (ROOT, name)
    e = dict(os.environ, **env)
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=e, capture_output=True, text=True,
                       timeout=1500)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = [x for x in r.stdout.splitlines() if x.startswith("RESULT ")][-1]
    return json.loads(line[len("RESULT "):])


# ------------------------------------------------------------------ GRPO over several chunks
def case_grpo_chunks():
    """Runs in a fresh process (MM_CHUNK_TOKENS is read once per process)."""
    prng, srng, rr = O.Rng(2), O.Rng(1), O.Rng(3)
    prompts = np.array([[prng.bounded(MLA36M.vocab_size) for _ in range(PROMPT)] for _ in range(N_ROLL // G)],
                       np.uint16)
    prompts = np.repeat(prompts, G, axis=0)
    seeds = np.array([srng.next() for _ in range(N_ROLL)], np.uint64)
    opt = AdamWConfig()
    pol = E.make_execution(MLA36M, E.init_params(MLA36M, 0), optimizer=opt)
    refm = E.make_execution(MLA36M, E.init_params(MLA36M, 1))
    r = pol.rollout(prompts, NEW, SEQ, seeds, 1.0)
    # rollout integers against the reference's completion_batch
    exact = True
    for i in range(N_ROLL):
        L = int(r["lengths"][i])
        toks = r["tokens"][i, :L]
        exact &= bool(1 <= L <= NEW and (toks[:-1] != MLA36M.eos_id).all())
        exact &= bool(L == NEW or toks[-1] == MLA36M.eos_id)
        inp, tgt, mask = ref.completion_batch(prompts[i], toks, SEQ, MLA36M.pad_id)
        exact &= bool(np.array_equal(inp, r["input"][i]) and np.array_equal(tgt, r["target"][i])
                      and np.array_equal(mask, r["mask"][i]))
    noise = np.random.default_rng(5).normal(0, 0.3, r["old_lp"].shape).astype(np.float32)
    old = (r["old_lp"] + noise * r["mask"]).astype(np.float32)
    # A token whose ratio sits on a clip edge (within the engines' log-prob difference, max
    # ~2e-3) is clipped in one engine and not in the other, which adds or removes that token's
    # whole gradient: no tolerance covers that step. Such tokens move 1e-2 off the edge, judged
    # on the policy's own teacher-forced log-probs (the update's lp).
    lp = pol.log_probabilities(r["input"], r["target"], N_ROLL, SEQ).reshape(N_ROLL, SEQ)
    for edge in (np.log(1.2), np.log(0.8)):
        d = lp.astype(np.float64) - old - edge
        near = (r["mask"] > 0) & (np.abs(d) < 5e-3)
        old = np.where(near, old + np.where(d >= 0, -1e-2, 1e-2), old).astype(np.float32)
    rewards = np.array([1.0 if rr.uniform() < 0.3 else 0.0 for _ in range(N_ROLL)], np.float32)
    rewards[0], rewards[1], rewards[G], rewards[G + 1] = 1.0, 0.0, 0.0, 1.0
    # both clip branches (advantage sign x ratio outside [1 - eps, 1 + eps]) on the policy's lp
    adv = np.concatenate([O.group_advantages(rewards[g * G:(g + 1) * G]) for g in range(N_ROLL // G)])
    ratio = np.exp(r["old_lp"].astype(np.float64) - old)
    on = r["mask"] > 0
    clipped_pos = int((on & (adv[:, None] > 0) & (ratio > 1.2)).sum())
    clipped_neg = int((on & (adv[:, None] < 0) & (ratio < 0.8)).sum())
    args = [_pin(a) for a in (r["input"], r["target"], r["mask"], old, rewards)]
    out = pol.grpo_step(refm, *args, G, clip=0.2, klc=0.04, learning_rate=1e-5)
    after = pol.synchronize_to_host()["params"]
    ps = ref.Session(MLA36M, 0, optimizer=opt.as_list())
    rs = ref.Session(MLA36M, 1)
    want = ref.grpo_update(ps, rs, G, r["input"], r["target"], r["mask"], old, rewards, 0.2, 0.04, 1e-5)
    return dict(exact=exact, got=out, want={k: want[k] for k in ("loss", "kl", "grad_norm", "skipped")},
                adv_equal=bool(np.array_equal(adv, want["advantages"])),
                max_param_diff=float(np.abs(after - ps.params()).max()),
                clipped_pos=clipped_pos, clipped_neg=clipped_neg,
                chunk_tokens=int(os.environ.get("MM_CHUNK_TOKENS", "0")))


def test_grpo_update_over_chunks_matches_reference():
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    # 5 rollouts per chunk: chunks of 5, 5, 5 and 1 rollouts
    res = _run_case("case_grpo_chunks", {"MM_CHUNK_TOKENS": str(5 * SEQ)})
    got, want = res["got"], res["want"]
    assert res["exact"] and res["adv_equal"]
    assert res["clipped_pos"] > 0 and res["clipped_neg"] > 0
    assert not got["skipped"] and not want["skipped"]
    assert abs(got["loss"] - want["loss"]) <= 1e-3 * abs(want["loss"]), (got, want)
    assert abs(got["kl"] - want["kl"]) <= 1e-3 * abs(want["kl"]), (got, want)
    assert abs(got["grad_norm"] - want["grad_norm"]) <= 1e-3 * want["grad_norm"], (got, want)
    # the first AdamW step moves each weight by about lr times the sign of its gradient
    assert res["max_param_diff"] <= 2.05e-5


# ------------------------------------------------------------------ DPO over several chunks
def case_dpo_chunks():
    rng = np.random.default_rng(31)
    n, S = 6, 96
    inp = rng.integers(0, 256, (2 * n, S)).astype(np.uint16)
    tgt = rng.integers(0, 256, (2 * n, S)).astype(np.uint16)
    mask = np.zeros((2 * n, S), np.float32)
    for row in range(2 * n):
        start = int(rng.integers(4, S // 3))
        mask[row, start:start + int(rng.integers(S // 4, S // 2))] = 1
    opt = AdamWConfig()
    pol = E.make_execution(MLA36M, E.init_params(MLA36M, 0), optimizer=opt)
    refm = E.make_execution(MLA36M, E.init_params(MLA36M, 1))
    got = pol.dpo_step(refm, _pin(inp), _pin(tgt), _pin(mask), beta=0.1, learning_rate=1e-3)
    rp = ref.Session(MLA36M, 0, optimizer=opt.as_list())
    rr = ref.Session(MLA36M, 1)
    want = ref.dpo_update(rp, rr, inp, tgt, mask, 0.1, 1e-3)
    return dict(loss=[got["loss"], want["loss"]], grad_norm=[got["grad_norm"], want["grad_norm"]],
                margins=[np.asarray(got["margins"]).tolist(), np.asarray(want["margins"]).tolist()])


def test_dpo_update_over_chunks_matches_reference():
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    res = _run_case("case_dpo_chunks", {"MM_CHUNK_TOKENS": str(2 * 2 * 96)})  # 2 pairs per chunk
    (gl, wl), (gn, wn) = res["loss"], res["grad_norm"]
    assert abs(gl - wl) <= 1e-3 * abs(wl)
    assert abs(gn - wn) <= 1e-3 * wn
    np.testing.assert_allclose(res["margins"][0], res["margins"][1], rtol=0, atol=2e-2)


# ------------------------------------------------------------------ 64 x 512 teacher-forced
def test_teacher_forced_64x512_and_grpo_update_match_reference():
    require_gpu()
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    B, S, P0 = 64, 512, 128
    r4 = O.Rng(4)
    ids = np.array([[r4.bounded(MLA36M.vocab_size) for _ in range(S + 1)] for _ in range(B)], np.uint16)
    inp, tgt = np.ascontiguousarray(ids[:, :S]), np.ascontiguousarray(ids[:, 1:])
    mask = np.zeros((B, S), np.float32)
    mask[:, P0:] = 1
    r5 = O.Rng(5)
    rewards = np.array([r5.normal() for _ in range(B)], np.float32)
    opt = AdamWConfig()
    pol = E.make_execution(MLA36M, E.init_params(MLA36M, 0), optimizer=opt)
    refm = E.make_execution(MLA36M, E.init_params(MLA36M, 1))
    lp = pol.log_probabilities(inp, tgt, B, S).reshape(B, S)
    rlp = refm.log_probabilities(inp, tgt, B, S).reshape(B, S)
    ps = ref.Session(MLA36M, 0, optimizer=opt.as_list())
    rs = ref.Session(MLA36M, 1)
    want_lp = ps.log_probs(inp, tgt, mask, B, S).reshape(B, S)
    want_rlp = rs.log_probs(inp, tgt, mask, B, S).reshape(B, S)
    on = mask > 0
    assert np.abs(lp - want_lp)[on].max() < 2e-3
    assert np.abs(rlp - want_rlp)[on].max() < 2e-3
    # old log-probs := the frozen reference's (identical arrays on both sides), so the ratio
    # exp(lp - old) leaves [1 - eps, 1 + eps] on some tokens
    old = rlp.astype(np.float32)
    out = pol.grpo_step(refm, inp, tgt, mask, old, rewards, 8, clip=0.2, klc=0.04, learning_rate=1e-5)
    want = ref.grpo_update(ps, rs, 8, inp, tgt, mask, old, rewards, 0.2, 0.04, 1e-5)
    assert not out["skipped"] and not want["skipped"]
    assert abs(out["loss"] - want["loss"]) <= 1e-3 * abs(want["loss"]), (out, want)
    assert abs(out["kl"] - want["kl"]) <= 1e-3 * abs(want["kl"]), (out, want)
    assert abs(out["grad_norm"] - want["grad_norm"]) <= 1e-3 * want["grad_norm"], (out, want)


# ------------------------------------------------------------------ decode after 1,024-token prompts
_DECODE_ROWS_CHECKED = 6
_DECODE_STEPS = 128


@pytest.fixture(scope="module")
def cpu_greedy_1024():
    """The reference decoder (CpuDecoder through make_execution("cpu")) on the first rows'
    prompts: greedy tokens, top-2 margins, 128 steps after a 1,024-token prefill."""
    if not ref.available():
        pytest.skip("oracle/_ref not built")
    r2 = O.Rng(2)
    prompts = np.array([[r2.bounded(MLA36M.vocab_size) for _ in range(1024)] for _ in range(64)], np.uint16)
    s = ref.Session(MLA36M, 0)
    toks = np.zeros((_DECODE_ROWS_CHECKED, _DECODE_STEPS + 1), np.int64)
    margins = np.zeros((_DECODE_ROWS_CHECKED, _DECODE_STEPS + 1))
    for i in range(_DECODE_ROWS_CHECKED):
        lg = s.prefill(prompts[i])
        for k in range(_DECODE_STEPS + 1):
            top = np.sort(lg)[-2:]
            toks[i, k] = int(np.argmax(lg))
            margins[i, k] = float(top[1] - top[0])
            if k < _DECODE_STEPS:
                lg = s.decode(toks[i, k])
    return prompts, toks, margins


@pytest.mark.parametrize("rows", [64, 2048])
def test_decode_after_1024_prompt_matches_reference_greedy(cpu_greedy_1024, rows):
    require_gpu()
    prompts, want, margins = cpu_greedy_1024
    ex = E.make_execution(MLA36M, E.init_params(MLA36M, 0))
    batch = prompts[np.arange(rows) % prompts.shape[0]]
    lg = ex.prefill_batch(batch)
    agree = checked = 0
    for k in range(_DECODE_STEPS + 1):
        got = np.argmax(lg, axis=1)
        for i in range(_DECODE_ROWS_CHECKED):
            if margins[i, k] > 1e-3:
                checked += 1
                agree += int(got[i] == want[i, k])
        if k == _DECODE_STEPS:
            break
        feed = got.astype(np.uint16)
        for i in range(rows):  # teacher-force the reference's tokens on every row of a checked prompt
            if i % prompts.shape[0] < _DECODE_ROWS_CHECKED:
                feed[i] = want[i % prompts.shape[0], k]
        lg = ex.decode_batch(feed)
    assert checked > 0.5 * _DECODE_ROWS_CHECKED * (_DECODE_STEPS + 1)
    assert agree == checked, (agree, checked)
