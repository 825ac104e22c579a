"""The backward entry point that allocates no device memory.

Callers that cannot allocate device memory themselves (their device memory
belongs to a host framework's pool or another runtime, or their path may not
call cudaMalloc) use ``sdk_topk_attn_bwd_noalloc``; it keeps its fp32
accumulators in a fixed array owned by the library.  These tests call it
through the C ABI and check it against the allocating entry point
(``sdk_topk_attn_bwd`` + ``sdk_finalize_grad``) on two calls in a row, so the
second call also shows that the shared array is cleared between calls.

This file is collected last on purpose: a run that stops at its first
failure has then already run every other test.
"""

import ctypes

import pytest
import torch

from sparsedict_b200 import _native, _ops

pytestmark = pytest.mark.gpu

SDK_DTYPE = {torch.float32: _native.DTYPE_F32, torch.bfloat16: _native.DTYPE_BF16, torch.float16: _native.DTYPE_F16}
TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def _noalloc_backward(lib, q, k, v, dout, idx, lse, scale):
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    slices, n, d = q.shape
    m, dv_dim = k.shape[1], v.shape[2]
    rc = lib.sdk_topk_attn_bwd_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), dout.data_ptr(), idx.data_ptr(), lse.data_ptr(),
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), slices, n, m, d, dv_dim, idx.shape[-1], scale,
        SDK_DTYPE[q.dtype], torch.cuda.current_stream().cuda_stream)
    assert rc == _native.SDK_OK, lib.sdk_status_string(rc)
    return dq, dk, dv


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_backward_matches_allocating_backward_on_two_calls(dtype):
    lib = _native.load()
    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev).manual_seed(23)
    slices, n, m, d, k, scale = 4, 300, 700, 64, 32, 0.125
    q, kk, v, dout = (torch.randn(slices, x, d, device=dev, generator=gen).to(dtype) for x in (n, m, m, n))
    _, idx, lse, _ = _ops.topk_attn_fwd(q, kk, v, k, scale)
    dq_ref, dk_acc, dv_acc = _ops.topk_attn_bwd(q, kk, v, dout, idx, lse, scale)
    dk_ref, dv_ref = _ops.finalize_grad(dk_acc, dtype), _ops.finalize_grad(dv_acc, dtype)
    for _ in range(2):
        dq, dk, dv = _noalloc_backward(lib, q, kk, v, dout, idx, lse, scale)
        torch.cuda.synchronize(dev)
        assert torch.equal(dq, dq_ref)  # dq is written once per row, no atomics
        for got, ref in ((dk, dk_ref), (dv, dv_ref)):
            assert torch.allclose(got.float(), ref.float(), rtol=TOL[dtype], atol=TOL[dtype]), (
                (got.float() - ref.float()).abs().max().item())


def test_noalloc_backward_refuses_requests_beyond_its_scratch():
    lib = _native.load()
    dev = torch.device("cuda:0")
    t = torch.zeros(16, device=dev)
    idx = torch.zeros(16, dtype=torch.int32, device=dev)
    cap = _native.NOALLOC_SCRATCH_FLOATS
    m = cap // 64  # slices * m * (d + dv) = 2 * cap
    rc = lib.sdk_topk_attn_bwd_noalloc(*(t.data_ptr(),) * 4, idx.data_ptr(), t.data_ptr(), *(t.data_ptr(),) * 3,
                                       1, 1, m, 64, 64, 1, 0.125, _native.DTYPE_F32,
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == _native.SDK_ERR_TOO_LARGE
    assert b"scratch" in lib.sdk_status_string(rc)
