"""The tensor-core forward's bounded waits, made to run out on purpose.

Every mbarrier wait of the streaming kernel gives up after a bound (2 s by
default).  With the bound set to 200 ns for one call, the first wait on a
copy from memory runs out: the kernel must return (no hang), raise device
status bit 2, write NaN outputs and LSE and index -1 for the rows it gave up
on, leave every other row exactly as a normal call computes it, and leave
the context usable for the next call.  Nothing faults: the waits that let
in-flight copies land before a CTA exits keep their 2 s bound.
"""

import pytest
import torch

from sparsedict_b200 import _native, _ops

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _inputs():
    g = torch.Generator().manual_seed(31)
    bh, n, m, d = 4, 1024, 8192, 64
    return [torch.randn(bh, x, d, generator=g).to(torch.bfloat16).to(DEV) for x in (n, m, m)]


def test_short_wait_limit_gives_up_cleanly_and_context_stays_usable():
    q, k, v = _inputs()
    assert _native.device_status(clear=True) == 0
    out0, idx0, lse0, _ = _ops.topk_attn_fwd(q, k, v, 32, 0.125)
    assert _native.device_status(clear=True) == 0
    try:
        _native.set_wait_limit(200)
        out1, idx1, lse1, _ = _ops.topk_attn_fwd(q, k, v, 32, 0.125)
        torch.cuda.synchronize()
    finally:
        _native.set_wait_limit(0)
    assert _native.device_status(clear=True) & 2
    out1 = out1.reshape(-1, 64)
    gave_up = (idx1 == -1).all(dim=1)
    assert int(gave_up.sum()) > 0
    assert torch.isnan(lse1[gave_up]).all()
    assert torch.isnan(out1[gave_up].float()).all()
    done = ~gave_up
    assert torch.equal(idx1[done], idx0[done])
    assert torch.equal(lse1[done], lse0[done])
    assert torch.equal(out1[done], out0.reshape(-1, 64)[done])
    # the same context, default bound again: a normal call
    out2, idx2, lse2, _ = _ops.topk_attn_fwd(q, k, v, 32, 0.125)
    assert _native.device_status(clear=True) == 0
    assert torch.equal(idx2, idx0) and torch.equal(lse2, lse0) and torch.equal(out2, out0)


def test_wait_limit_bounds_are_checked():
    with pytest.raises(_native.NativeError):
        _native.set_wait_limit(61 * 10**9)
    _native.set_wait_limit(0)
