"""The allocation-free decode attention (mm_decode_attention_noalloc) against the existing
entry point (mm_cuda_decode_attention), through the C ABI.

Some callers cannot allocate device memory while they run -- a server that gave all of it to
its own pool at start-up, a plugin host that only lends input and output buffers -- so this
entry point keeps its split partials in a static device array instead. Two calls in a row
must match the allocating entry point within this suite's decode-attention tolerance, a
call after the first must leave the device's free memory unchanged, and a split plan larger
than the static array must be refused.
"""
import ctypes

import pytest

from tests.gpu_util import require_gpu

pytestmark = pytest.mark.gpu

H, KV, R = 8, 128, 16
W = KV + R
SLOTS = 256  # (row, split) partial slots of the static array


def noalloc_fn():
    import cpp_inference_train_engine_b200 as E
    f = E.lib().mm_decode_attention_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int,
                  ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
    return f


def case(B, ctx, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    Sc = ctx + 3
    cache = (torch.randn(B, Sc, W, device="cuda", generator=g) * 0.5).half()
    q = torch.randn(B, H, W, device="cuda", generator=g) * 0.5
    pos = torch.randint(max(ctx - 30, 0), ctx, (B,), device="cuda", generator=g).int()
    return q, cache, pos, Sc


def test_noalloc_matches_allocating_entry_point_twice():
    require_gpu()
    import torch

    import cpp_inference_train_engine_b200 as E
    from cpp_inference_train_engine_b200.config import MLA36M
    f = noalloc_fn()
    ex = E.CudaExecution(MLA36M)
    stream = torch.cuda.current_stream().cuda_stream
    scale = 0.125
    for call, (B, ctx, splits) in enumerate([(16, 900, 16), (40, 500, 6)]):
        q, cache, pos, Sc = case(B, ctx, 100 + call)
        want = torch.zeros(B, H * KV, device="cuda", dtype=torch.half)
        got = torch.full((B, H * KV), float("nan"), device="cuda", dtype=torch.half)
        torch.cuda.synchronize()
        ex.decode_attention(q.data_ptr(), cache.data_ptr(), Sc * W, pos.data_ptr(), B, splits, scale,
                            want.data_ptr())
        rc = f(q.data_ptr(), cache.data_ptr(), Sc * W, pos.data_ptr(), B, splits, scale,
               got.data_ptr(), stream)
        assert rc == 0, rc
        err = (got.float() - want.float()).abs().max().item()
        assert err < 2e-2 * max(1.0, want.float().abs().max().item()), (call, err)


def test_noalloc_call_allocates_nothing():
    require_gpu()
    import torch
    f = noalloc_fn()
    q, cache, pos, Sc = case(32, 700, 11)
    out = torch.zeros(32, H * KV, device="cuda", dtype=torch.half)
    stream = torch.cuda.current_stream().cuda_stream
    # the first call is the set-up (module load, symbol address); later calls allocate nothing
    assert f(q.data_ptr(), cache.data_ptr(), Sc * W, pos.data_ptr(), 32, 8, 0.125, out.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert f(q.data_ptr(), cache.data_ptr(), Sc * W, pos.data_ptr(), 32, 8, 0.125, out.data_ptr(),
                 stream) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)


def test_noalloc_rejects_plans_beyond_its_static_scratch():
    require_gpu()
    import torch
    f = noalloc_fn()
    q, cache, pos, Sc = case(20, 64, 7)
    out = torch.zeros(20, H * KV, device="cuda", dtype=torch.half)
    stream = torch.cuda.current_stream().cuda_stream
    # 20 rows x 16 splits = 320 slots > 256: refused, output untouched
    rc = f(q.data_ptr(), cache.data_ptr(), Sc * W, pos.data_ptr(), 20, 16, 0.125, out.data_ptr(),
           stream)
    assert rc == 1
    assert out.abs().max().item() == 0
    # one split needs no scratch at all, so any batch is accepted
    rc = f(q.data_ptr(), cache.data_ptr(), Sc * W, pos.data_ptr(), 20, 1, 0.125, out.data_ptr(),
           stream)
    assert rc == 0
