"""The GRPO update's vocabulary head on the selected rows only (mask != 0, listed on the device)
and its backward with recomputed logits, against the same update on every row
(MM_VOCAB_ROWS=all) and with stored logits (MM_VOCAB_RECOMPUTE=0), each in a fresh process
(the switches are read once). The mask is irregular (random, about half the tokens, a row with
one token and a full row) and the batch spans several chunks (MM_CHUNK_TOKENS), so the selection
differs per chunk. The rows left out have coefficient 0. With stored logits the update is the
same arithmetic: loss and KL identical, the gradient norm too. Against every row, each kept
row's log-probability is its own product row and log-sum-exp, but at these small chunks the two
row counts can get different GEMM tile widths (the log-sum-exp partials then group columns
differently), and the backward's vocabulary products split their K (= rows) differently: 1e-5
relative, a hundred times inside the 1e-3 gate against the reference."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from tests.gpu_util import ROOT, require_gpu

pytestmark = pytest.mark.gpu

_RUN = """
import json, sys
import numpy as np
sys.path.insert(0, {root!r})
import cpp_inference_train_engine_b200 as E
from cpp_inference_train_engine_b200.config import MLA36M, AdamWConfig
B, S, G = 16, 96, 4
rng = np.random.default_rng(11)
inp = rng.integers(0, MLA36M.vocab_size - 8, (B, S)).astype(np.uint16)
tgt = rng.integers(0, MLA36M.vocab_size - 8, (B, S)).astype(np.uint16)
mask = (rng.random((B, S)) < 0.5).astype(np.float32)
mask[3] = 0.0   # a row with one token selected (a batch row needs one, src/train/data.cpp:49)
mask[3, 7] = 1.0
mask[5] = 1.0   # a row with everything selected
pol = E.make_execution(MLA36M, E.init_params(MLA36M, 0), optimizer=AdamWConfig())
ref = E.make_execution(MLA36M, E.init_params(MLA36M, 1))
lp = pol.log_probabilities(inp, tgt, B, S).reshape(B, S)
old = (lp + 0.2 * np.sin(np.arange(B * S).reshape(B, S)) * mask).astype(np.float32)
rewards = rng.normal(size=B).astype(np.float32)
out = pol.grpo_step(ref, inp, tgt, mask, old, rewards, G, clip=0.2, klc=0.04, learning_rate=1e-5)
print("RESULT " + json.dumps({{k: out[k] for k in ("loss", "kl", "grad_norm", "skipped")}}))
"""


def _run(env):
    e = dict(os.environ, MM_CHUNK_TOKENS=str(5 * 96), **env)  # chunks of 5, 5, 5 and 1 rows
    r = subprocess.run([sys.executable, "-c", _RUN.format(root=ROOT)], cwd=ROOT, env=e, capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    line = [x for x in r.stdout.splitlines() if x.startswith("RESULT ")][-1]
    return json.loads(line[len("RESULT "):])


def test_selected_rows_and_recomputed_logits_match_the_full_update():
    require_gpu()
    base = _run({})
    full = _run({"MM_VOCAB_ROWS": "all"})
    stored = _run({"MM_VOCAB_RECOMPUTE": "0"})
    assert not base["skipped"]
    assert stored["loss"] == base["loss"] and stored["kl"] == base["kl"], (base, stored)
    assert stored["grad_norm"] == base["grad_norm"], (base, stored)
    for k in ("loss", "kl", "grad_norm"):
        assert abs(full[k] - base[k]) <= 1e-5 * abs(base[k]), (k, base, full)
