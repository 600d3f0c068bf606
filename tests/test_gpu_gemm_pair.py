"""The CTA-pair GEMM (clusters of 2, tcgen05 cta_group::2, 256 x 256 tiles) that the large
256-wide products run on: plain products over every operand layout against a PyTorch fp32
product of the same fp16 operands (ragged M and N included), and the 35.8M model's
teacher-forced log-probabilities and weighted-NLL gradient, whose vocabulary head
(log-sum-exp epilogue), SwiGLU forward (with pre-activation stores) and SwiGLU backward
products run on it at 8,448 tokens, against the same engine with every product on the
single-CTA kernel (MM_GEMM_PAIR=0, a separate process)."""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from tests.gpu_util import ROOT, rel, require_gpu

pytestmark = pytest.mark.gpu

# (M, N, K): chunk-sized (M >= 8192) with at least one full wave of pair tiles, so the pair
# kernel is chosen; ragged M (8320 = 32.5 x 256), N (1360, 2056) and K (200)
PAIR_SHAPES = [(8192, 4096, 512), (8320, 1360, 512), (8192, 8192, 1536), (8200, 2056, 200)]


@pytest.fixture(scope="module")
def ex():
    require_gpu()
    import cpp_inference_train_engine_b200 as E
    return E.CudaExecution(E.TINY)


def pad8(n):
    return (n + 7) // 8 * 8


@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("shape", PAIR_SHAPES)
def test_pair_gemm_layouts(ex, shape, a_mn, b_mn):
    import torch
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M + 5 * N + 3 * K + a_mn * 17 + b_mn * 19)
    A = torch.randn(M, K, device="cuda", generator=g).half()
    B = torch.randn(K, N, device="cuda", generator=g).half()
    if a_mn:
        As = torch.zeros(K, pad8(M), device="cuda", dtype=torch.half)
        As[:, :M] = A.t()
    else:
        As = torch.zeros(M, pad8(K), device="cuda", dtype=torch.half)
        As[:, :K] = A
    if b_mn:
        Bs = torch.zeros(K, pad8(N), device="cuda", dtype=torch.half)
        Bs[:, :N] = B
    else:
        Bs = torch.zeros(N, pad8(K), device="cuda", dtype=torch.half)
        Bs[:, :K] = B.t()
    out = torch.full((M, N), float("nan"), device="cuda")
    torch.cuda.synchronize()
    ex.gemm(M, N, K, As.data_ptr(), As.shape[1], a_mn, Bs.data_ptr(), Bs.shape[1], b_mn,
            out.data_ptr(), N, 0)
    want = A.float() @ B.float()
    err = (out - want).abs().max().item()
    assert err <= 1e-3 * max(1.0, want.abs().max().item()), err


_RUN = textwrap.dedent("""
    import sys
    import numpy as np
    import cpp_inference_train_engine_b200 as E
    from cpp_inference_train_engine_b200.config import MLA36M
    B, S = 32, 264
    rng = np.random.default_rng(41)
    x = rng.integers(0, 16384, (B, S)).astype(np.uint16)
    t = rng.integers(0, 16384, (B, S)).astype(np.uint16)
    coef = (rng.normal(size=(B, S)) * 1e-3).astype(np.float32)
    ex = E.make_execution(MLA36M, E.init_params(MLA36M, 4), optimizer=E.AdamWConfig())
    lp = ex.log_probabilities(x, t, B, S)
    ex.zero_grad()
    loss = ex.accumulate(x, t, coef, B, S)
    g = ex.synchronize_to_host(params=False, grads=True)["grads"]
    np.savez(sys.argv[1], lp=lp, g=g, loss=np.float64(loss))
""")


def _run(path, pair):
    env = dict(os.environ, PYTHONPATH=ROOT, MM_GEMM_PAIR="1" if pair else "0")
    out = subprocess.run([sys.executable, "-c", _RUN, path], cwd=ROOT, env=env, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stdout + out.stderr
    return np.load(path)


def test_pair_products_match_single_cta_in_the_model(tmp_path):
    require_gpu()
    a = _run(str(tmp_path / "pair.npz"), True)
    b = _run(str(tmp_path / "single.npz"), False)
    d = np.abs(a["lp"].astype(np.float64) - b["lp"])
    assert d.max() < 1e-4, d.max()
    assert abs(float(a["loss"]) - float(b["loss"])) <= 1e-5 * abs(float(b["loss"]))
    assert rel(a["g"], b["g"]) < 1e-3, rel(a["g"], b["g"])
