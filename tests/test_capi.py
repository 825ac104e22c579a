"""The C-ABI library loads on a CPU-only machine and exports every declared
entry point; argument checks answer without touching a GPU."""

import ctypes
import re
from pathlib import Path

import pytest

from sparsedict_b200 import _native

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        names.update(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\**\s+\**(sdk_[a-z0-9_]+)\(", text, re.M))
    return sorted(names)


def test_header_declares_the_entry_points():
    names = declared_symbols()
    for required in ("sdk_topk_attn_fwd", "sdk_topk_attn_bwd", "sdk_topk_select", "sdk_topk_aggregate",
                     "sdk_affinity", "sdk_status_string", "sdk_device_status"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert sorted(_native.SIGNATURES) == declared_symbols()


def test_status_strings_and_version():
    lib = _native.load()
    assert lib.sdk_version() >= 1
    assert lib.sdk_status_string(0) == b"ok"
    assert b"invalid" in lib.sdk_status_string(1)
    assert lib.sdk_status_string(99) == b"unknown status"


def test_invalid_arguments_are_rejected_before_any_device_work():
    lib = _native.load()
    # null tensors
    rc = lib.sdk_topk_attn_fwd(None, None, None, None, None, None, None, None, None,
                               1, 4, 8, 16, 16, 2, 0.25, 0, 0, None)
    assert rc == _native.SDK_ERR_INVALID_ARGUMENT
    # k > m and bad dtype with non-null pointers (never dereferenced)
    fake = 0x1000
    rc = lib.sdk_topk_attn_fwd(fake, fake, fake, fake, fake, fake, None, None, None,
                               1, 4, 8, 16, 16, 9, 0.25, 0, 0, None)
    assert rc == _native.SDK_ERR_INVALID_ARGUMENT
    rc = lib.sdk_topk_attn_fwd(fake, fake, fake, fake, fake, fake, None, None, None,
                               1, 4, 8, 16, 16, 2, 0.25, 0, 7, None)
    assert rc == _native.SDK_ERR_INVALID_ARGUMENT
    rc = lib.sdk_topk_select(fake, fake, fake, 4, 8, 4, 2, 0, None)  # row stride < m
    assert rc == _native.SDK_ERR_INVALID_ARGUMENT
    rc = lib.sdk_topk_aggregate(fake, fake, fake, fake, 4, 2, 8, 16, 2, 2, 16, 0, 48, 0, None)
    assert rc == _native.SDK_ERR_INVALID_ARGUMENT
    # per-row budgets: the row_k array is required; the common checks still apply
    rc = lib.sdk_topk_attn_fwd_adaptive(fake, fake, fake, fake, fake, fake, None, None, None,
                                        1, 4, 8, 16, 16, 2, 0.25, 0, None, 0, None)
    assert rc == _native.SDK_ERR_INVALID_ARGUMENT
    rc = lib.sdk_topk_attn_fwd_adaptive(fake, fake, fake, fake, fake, fake, None, None, None,
                                        1, 4, 8, 16, 16, 9, 0.25, 0, fake, 0, None)
    assert rc == _native.SDK_ERR_INVALID_ARGUMENT
    rc = lib.sdk_topk_attn_fwd_adaptive(None, fake, fake, fake, fake, fake, None, None, None,
                                        1, 4, 8, 16, 16, 2, 0.25, 0, fake, 0, None)
    assert rc == _native.SDK_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("dtype", [0, 1, 2, 3])
def test_max_topk_covers_the_benchmark_configurations(dtype):
    lib = _native.load()
    assert lib.sdk_max_topk(dtype, 64) >= 64
    assert lib.sdk_max_topk(dtype, 128) >= 128
    assert lib.sdk_max_topk(9, 64) == 0


def test_forward_workspace_size_follows_the_tensor_core_shapes():
    # Nonzero exactly when the call takes the tensor-core path: bf16/fp16,
    # d = dv = 64, 1 <= k <= 64, m <= 65536, no score grid; uniform or grouped
    # slices alike.
    lib = _native.load()
    size = lib.sdk_topk_attn_fwd_workspace_size
    per_row = 192 * 2 + 20  # candidate keys of the four selection threads, four counts and a check word
    for code in (_native.DTYPE_BF16, _native.DTYPE_F16):
        assert size(1000, 16384, 64, 64, 64, 0, 0, code) == 1000 * per_row
        assert size(3, 100, 64, 64, 1, 0, 0, code) == 3 * per_row
        assert size(1000, 65536, 64, 64, 64, 0, 0, code) == 1000 * per_row
        assert size(1000, 65537, 64, 64, 64, 0, 0, code) == 0
        assert size(1000, 16384, 64, 64, 65, 0, 0, code) == 0
        assert size(1000, 16384, 32, 32, 8, 0, 0, code) == 0
        assert size(0, 16384, 64, 64, 8, 0, 0, code) == 0
        assert size(1000, 16384, 64, 64, 8, 64, 0, code) == 0
        assert size(1000, 16384, 64, 64, 8, 0, 1, code) == 1000 * per_row
    for code in (_native.DTYPE_F32, _native.DTYPE_F64):
        assert size(1000, 16384, 64, 64, 64, 0, 0, code) == 0


def test_forward_workspace_pointer_and_size_must_agree():
    lib = _native.load()
    fake = 0x1000
    rc = lib.sdk_topk_attn_fwd_ws(fake, fake, fake, fake, fake, fake, None, None, None,
                                  1, 4, 8, 16, 16, 2, 0.25, 0, 0, None, 64, None)
    assert rc == _native.SDK_ERR_INVALID_ARGUMENT
