"""The fused decode step (decode_mk_kernel: one cooperative launch for all layers) against
the per-layer chain of launches (MM_DECODE_MK=0) on the same weights, prompts and tokens.

Both paths feed the tensor cores the same fp16 operands; they differ only in the order of
fp32 additions (the fused step sums K-split partials of W_o and W_down into the residual in
a fixed order, and each latent RMSNorm's squares per row in one thread). So after a prefill
and teacher-forced decode steps the logits agree to 2e-3 absolute, greedy tokens agree
wherever the top-2 margin exceeds 1e-3, and the fused step repeats bit for bit. Rows: 1 and
100 (one partial 128-row tile), 256 (two tiles, context split over several warps), 1,300 (no
context split). Each path runs in a fresh process (the switch is read once per process).
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from tests.gpu_util import ROOT, require_gpu

pytestmark = pytest.mark.gpu


def case_decode(rows, prompt, steps):
    """Prefill `rows` random prompts, then `steps` teacher-forced decode steps whose tokens are
    a fixed random stream; returns every step's logits of a few rows and the greedy tokens of
    all rows, twice over (the second pass repeats the first from a fresh prefill)."""
    import cpp_inference_train_engine_b200 as E
    from cpp_inference_train_engine_b200.config import MLA36M
    rng = np.random.default_rng(rows)
    prompts = rng.integers(0, MLA36M.vocab_size, (rows, prompt)).astype(np.uint16)
    feed = rng.integers(0, MLA36M.vocab_size, (steps, rows)).astype(np.uint16)
    ex = E.make_execution(MLA36M, E.init_params(MLA36M, 0))
    watch = sorted({0, rows // 2, rows - 1})
    out = []
    for _ in range(2):
        lg = ex.prefill_batch(prompts)
        logits, greedy, margin = [lg[watch]], [np.argmax(lg, 1)], []
        for k in range(steps):
            lg = ex.decode_batch(feed[k])
            logits.append(lg[watch])
            greedy.append(np.argmax(lg, 1))
            top = np.sort(lg, axis=1)[:, -2:]
            margin.append(top[:, 1] - top[:, 0])
        out.append((np.stack(logits), np.stack(greedy), np.stack(margin)))
    (l0, g0, m0), (l1, g1, _) = out
    return {"logits": l0.tolist(), "greedy": g0.tolist(), "margin": m0.tolist(),
            "repeat_equal": bool(np.array_equal(l0, l1) and np.array_equal(g0, g1))}


def _run(rows, prompt, steps, fused):
    code = ("import json, sys; sys.path.insert(0, %r); from tests import test_gpu_decode_fused as m; "
            "print('RESULT ' + json.dumps(m.case_decode(%d, %d, %d)))") % (ROOT, rows, prompt, steps)
    # every row count through the fused step when it is on (it is the default only up to 512)
    env = dict(os.environ, MM_DECODE_MK="1" if fused else "0", MM_DECODE_MK_MAX_ROWS="100000")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = [x for x in r.stdout.splitlines() if x.startswith("RESULT ")][-1]
    return json.loads(line[len("RESULT "):])


@pytest.mark.parametrize("rows,prompt,steps", [(1, 40, 6), (100, 70, 6), (256, 130, 5), (1300, 20, 4)])
def test_fused_decode_matches_layer_by_layer(rows, prompt, steps):
    require_gpu()
    fused = _run(rows, prompt, steps, True)
    plain = _run(rows, prompt, steps, False)
    lf, lp = np.array(fused["logits"]), np.array(plain["logits"])
    assert np.abs(lf - lp).max() < 2e-3, np.abs(lf - lp).max()
    gf, gp = np.array(fused["greedy"])[1:], np.array(plain["greedy"])[1:]
    safe = np.array(plain["margin"]) > 1e-3
    assert safe.mean() > 0.5
    assert np.array_equal(gf[safe], gp[safe])
    assert fused["repeat_equal"]
