"""Kernel-level entry points (include/mm_cuda_kernels.h) against plain PyTorch fp32
references of the same operation."""
import numpy as np
import pytest

import cpp_inference_train_engine_b200 as E
from cpp_inference_train_engine_b200.config import MLA36M
from tests.gpu_util import require_gpu

pytestmark = pytest.mark.gpu

H, KV, R = 8, 128, 16
W = KV + R


def decode_attention_torch(q, cache, pos, scale):
    """Absorbed decode attention (inference.cpp:116-153) in fp32: per head scores over the
    latent|rope cache rows 0..pos, softmax, context = P . latent."""
    import torch
    out = []
    for b in range(q.shape[0]):
        n = int(pos[b]) + 1
        c = cache[b, :n].float()                       # [n, W]
        s = (q[b].float() @ c.t()) * scale             # [H, n]
        p = torch.softmax(s, dim=1)
        out.append(p @ c[:, :KV])                      # [H, KV]
    return torch.stack(out).reshape(q.shape[0], H * KV)


def make_case(B, ctx, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    Sc = ctx + 5
    cache = (torch.randn(B, Sc, W, device="cuda", generator=g) * 0.5).half()
    q = torch.randn(B, H, W, device="cuda", generator=g) * 0.5
    pos = torch.randint(max(ctx - 40, 0), ctx, (B,), device="cuda", generator=g).int()
    return q, cache, pos, Sc


@pytest.mark.parametrize("B,ctx,splits", [(1, 1100, 16), (16, 700, 4), (64, 300, 2), (300, 200, 1),
                                          (3, 20, 1), (5, 17, 3)])
def test_decode_attention_entry_matches_torch(B, ctx, splits):
    require_gpu()
    import torch
    ex = E.CudaExecution(MLA36M)
    q, cache, pos, Sc = make_case(B, ctx, B * 31 + splits)
    out = torch.zeros(B, H * KV, device="cuda", dtype=torch.half)
    scale = 1.0 / 8.0
    torch.cuda.synchronize()
    ex.decode_attention(q.data_ptr(), cache.data_ptr(), Sc * W, pos.data_ptr(), B, splits, scale,
                        out.data_ptr())
    want = decode_attention_torch(q, cache, pos, scale)
    err = (out.float() - want).abs().max().item()
    assert err < 2e-2 * max(1.0, want.abs().max().item()), err


def test_decode_attention_entry_rejects_bad_splits():
    require_gpu()
    ex = E.CudaExecution(MLA36M)
    with pytest.raises(E.EngineError) as e:
        ex.decode_attention(1, 1, W, 1, 1, 17, 0.125, 1)
    assert e.value.name == "invalid_argument"
