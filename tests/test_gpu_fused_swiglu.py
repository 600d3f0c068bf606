"""SwiGLU inside the products' epilogues on the training path: the policy pass with tape runs
SwiGLU in the [W_gate | W_up] product's epilogue and also stores the fp16 pre-activations,
and the backward computes [d gate | d up] in the epilogue of dH = dY W_down^T (the
reference's swiglu forward/backward, ops.cpp). Checked against the same engine with both as
separate elementwise kernels around plain products (MM_FUSED_SWIGLU=0, a separate process):
the fused forward takes SwiGLU from the fp32 accumulator instead of fp16-rounded gate/up,
and the fused backward takes dH from the fp32 accumulator instead of an fp16 copy, so the
two agree to fp16 rounding: weighted-NLL loss to 1e-4 relative, gradient to 1e-2 relative
(largest-magnitude normalised), and the log-probabilities of the pass without tape (which
both builds run identically) bit for bit. The tape pass's SwiGLU now matches the pass
without tape, so a GRPO step's old-policy and current log-probabilities agree exactly: the
loss of the step equals the loss rebuilt from its own old log-probabilities."""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from tests.gpu_util import ROOT, rel, require_gpu

pytestmark = pytest.mark.gpu

# query tiles of 128, 128 and 8 rows; M = 4,224 rows: 33 row tiles, enough for the 256-wide
# tiles the full-size chunks use (the last tile of d_ff = 1,360 is 80 columns wide)
B, S = 16, 264

_RUN = textwrap.dedent("""
    import sys
    import numpy as np
    import cpp_inference_train_engine_b200 as E
    from cpp_inference_train_engine_b200.config import MLA36M
    B, S = int(sys.argv[2]), int(sys.argv[3])
    rng = np.random.default_rng(33)
    x = rng.integers(0, 16384, (B, S)).astype(np.uint16)
    t = rng.integers(0, 16384, (B, S)).astype(np.uint16)
    coef = (rng.normal(size=(B, S)) * 1e-3).astype(np.float32)
    ex = E.make_execution(MLA36M, E.init_params(MLA36M, 9), optimizer=E.AdamWConfig())
    lp = ex.log_probabilities(x, t, B, S)
    ex.zero_grad()
    loss = ex.accumulate(x, t, coef, B, S)
    g = ex.synchronize_to_host(params=False, grads=True)["grads"]
    np.savez(sys.argv[1], lp=lp, g=g, loss=np.float64(loss))
""")


def _run(path, fused):
    env = dict(os.environ, PYTHONPATH=ROOT, MM_FUSED_SWIGLU="1" if fused else "0")
    out = subprocess.run([sys.executable, "-c", _RUN, path, str(B), str(S)], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    return np.load(path)


def test_fused_swiglu_matches_separate_kernels(tmp_path):
    require_gpu()
    a = _run(str(tmp_path / "fused.npz"), True)
    b = _run(str(tmp_path / "plain.npz"), False)
    np.testing.assert_array_equal(a["lp"], b["lp"])
    assert abs(float(a["loss"]) - float(b["loss"])) <= 1e-4 * abs(float(b["loss"]))
    assert rel(a["g"], b["g"]) < 1e-2, rel(a["g"], b["g"])


def test_tape_pass_log_probs_equal_pass_without_tape():
    """A GRPO step whose old log-probs come from log_probabilities and whose frozen reference
    has the policy's weights: the policy's tape pass reproduces both bit for bit, so every
    ratio is exactly 1 and the KL term exactly 0, and the loss is the one the restatement
    gives for lp = old = ref. (The KL term is summed in double: any difference between the
    passes, even one float ulp, leaves it nonzero.)"""
    require_gpu()
    import cpp_inference_train_engine_b200 as E
    from cpp_inference_train_engine_b200.config import MLA36M, AdamWConfig
    from oracle import mla_oracle as O
    n, G, S2 = 16, 8, 200
    rng = np.random.default_rng(5)
    x = rng.integers(0, 16384, (n, S2)).astype(np.uint16)
    t = rng.integers(0, 16384, (n, S2)).astype(np.uint16)
    mask = np.zeros((n, S2), np.float32)
    mask[:, 63:] = 1
    rewards = rng.uniform(size=n).astype(np.float32)
    W = E.init_params(MLA36M, 3)
    pol = E.make_execution(MLA36M, W, optimizer=AdamWConfig())
    ref = E.make_execution(MLA36M, W)
    old = pol.log_probabilities(x, t, n, S2)
    r = pol.grpo_step(ref, x, t, mask, old, rewards, G, clip=0.2, klc=0.04, learning_rate=1e-5)
    pol.close()
    ref.close()
    assert r["kl"] == 0.0, r["kl"]
    adv = np.concatenate([O.group_advantages(rewards[g:g + G]) for g in range(0, n, G)])
    o2 = np.asarray(old, np.float32).reshape(n, S2)
    want, kl, _ = O.grpo_coefficients(o2, o2, o2, mask, adv, 0.2, 0.04)
    assert kl == 0.0
    # advantages in float on both sides, sums in double in different orders
    assert abs(r["loss"] - want) <= 1e-6 * max(1.0, abs(want)), (r["loss"], want)
