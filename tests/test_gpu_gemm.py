"""tcgen05 GEMM parity against a plain PyTorch fp32 product of the same fp16 operands,
over every operand layout the passes use, ragged tiles and every epilogue."""
import pytest

from tests.gpu_util import require_gpu

pytestmark = pytest.mark.gpu

SHAPES = [(128, 128, 64), (200, 144, 96), (24, 12, 32), (300, 512, 1360), (1000, 264, 96),
          (64, 2720, 512), (2048, 336, 512), (130, 16384, 96)]


@pytest.fixture(scope="module")
def ex():
    require_gpu()
    import cpp_inference_train_engine_b200 as E
    return E.CudaExecution(E.TINY)


def pad8(n):
    return (n + 7) // 8 * 8


@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("shape", SHAPES)
def test_gemm_layouts(ex, shape, a_mn, b_mn):
    import torch
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K + a_mn * 11 + b_mn * 13)
    A = torch.randn(M, K, device="cuda", generator=g).half()
    B = torch.randn(K, N, device="cuda", generator=g).half()
    # stored operands with padded pitches
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


@pytest.mark.parametrize("kind", ["acc", "f16", "bf16", "residual", "alpha"])
def test_gemm_epilogues(ex, kind):
    import torch
    M, N, K = 260, 200, 192
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(M, K, device="cuda", generator=g).half()
    B = torch.randn(K, N, device="cuda", generator=g).half()
    Bs = torch.zeros(K, pad8(N), device="cuda", dtype=torch.half)
    Bs[:, :N] = B
    want = A.float() @ B.float()
    R = torch.randn(M, N, device="cuda", generator=g)
    if kind == "acc":
        out = R.clone()
        ex.gemm(M, N, K, A.data_ptr(), K, 0, Bs.data_ptr(), Bs.shape[1], 1, out.data_ptr(), N, 1)
        want = want + R
    elif kind in ("f16", "bf16"):
        dt = torch.half if kind == "f16" else torch.bfloat16
        out = torch.zeros(M, N, device="cuda", dtype=dt)
        ex.gemm(M, N, K, A.data_ptr(), K, 0, Bs.data_ptr(), Bs.shape[1], 1, out.data_ptr(), N,
                2 if kind == "f16" else 3)
        out = out.float()
    elif kind == "residual":
        out = torch.zeros(M, N, device="cuda")
        ex.gemm(M, N, K, A.data_ptr(), K, 0, Bs.data_ptr(), Bs.shape[1], 1, out.data_ptr(), N, 0,
                residual_ptr=R.data_ptr(), ldr=N)
        want = want + R
    else:
        out = torch.zeros(M, N, device="cuda")
        ex.gemm(M, N, K, A.data_ptr(), K, 0, Bs.data_ptr(), Bs.shape[1], 1, out.data_ptr(), N, 0,
                alpha=0.125)
        want = want * 0.125
    tol = 1e-2 if kind in ("f16", "bf16") else 1e-3
    assert (out - want).abs().max().item() <= tol * max(1.0, want.abs().max().item())


@pytest.mark.parametrize("shape", [(4096, 4096, 256), (2048, 16384, 1536), (4000, 1360, 512)])
def test_gemm_persistent_multiple_tiles_per_cta(ex, shape):
    """More output tiles than resident CTAs: each CTA walks several tiles and alternates
    its two tensor-memory accumulators."""
    import torch
    M, N, K = shape
    A = torch.randn(M, K, device="cuda").half()
    Bt = torch.randn(N, K, device="cuda").half()
    out = torch.zeros(M, N, device="cuda")
    ex.gemm(M, N, K, A.data_ptr(), K, 0, Bt.data_ptr(), K, 0, out.data_ptr(), N, 0)
    want = A.float() @ Bt.float().t()
    assert (out - want).abs().max().item() <= 1e-3 * want.abs().max().item()


@pytest.mark.parametrize("shape", [(512, 192, 32768), (128, 384, 24576), (1360, 512, 8192)])
def test_gemm_split_k_accumulate(ex, shape):
    """Weight-gradient pattern: out += alpha * X^T dY with X, dY stored [tokens][features]
    (both operands MN-major) and K = tokens: split over K, reduced in order."""
    import torch
    M, N, K = shape
    X = (torch.randn(K, M, device="cuda") * 0.1).half()
    dY = (torch.randn(K, N, device="cuda") * 0.1).half()
    R = torch.randn(M, N, device="cuda")
    out = R.clone()
    ex.gemm(M, N, K, X.data_ptr(), M, 1, dY.data_ptr(), N, 1, out.data_ptr(), N, 1, alpha=0.5)
    want = R + 0.5 * (X.float().t() @ dY.float())
    assert (out - want).abs().max().item() <= 1e-3 * max(1.0, want.abs().max().item())


def test_gemm_bf16_operands(ex):
    import torch
    M, N, K = 256, 256, 256
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = torch.randn(N, K, device="cuda").bfloat16()
    out = torch.zeros(M, N, device="cuda")
    ex.gemm(M, N, K, A.data_ptr(), K, 0, B.data_ptr(), K, 0, out.data_ptr(), N, 0, bf16=True)
    want = A.float() @ B.float().t()
    assert (out - want).abs().max().item() <= 1e-3 * want.abs().max().item()
