"""ctypes binding of ``libsparsedict_b200.so`` (the C ABI in ``include/sparsedict_b200.h``).

There is no fallback: if the library is missing or cannot be loaded, every
call raises ``RuntimeError`` naming the build command.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libsparsedict_b200.so"

DTYPE_F32, DTYPE_F64, DTYPE_BF16, DTYPE_F16 = 0, 1, 2, 3
SDK_OK, SDK_ERR_INVALID_ARGUMENT, SDK_ERR_UNSUPPORTED, SDK_ERR_CUDA, SDK_ERR_NO_DEVICE, SDK_ERR_TOO_LARGE = range(6)
NOALLOC_SCRATCH_FLOATS = 4 * 1024 * 1024

TORCH_TO_SDK = {
    torch.float32: DTYPE_F32,
    torch.float64: DTYPE_F64,
    torch.bfloat16: DTYPE_BF16,
    torch.float16: DTYPE_F16,
}

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f64 = ctypes.c_double

# name -> argtypes; every entry returns int unless listed in _RESTYPES.
SIGNATURES = {
    "sdk_version": [],
    "sdk_status_string": [ctypes.c_int],
    "sdk_last_cuda_error": [],
    "sdk_max_topk": [_i32, _i32],
    "sdk_device_status": [ctypes.POINTER(ctypes.c_uint), _i32, _p],
    "sdk_set_wait_limit": [ctypes.c_uint64],
    "sdk_topk_attn_fwd": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i32, _i32, _i32, _f64, _i32, _i32, _p],
    "sdk_topk_attn_fwd_adaptive": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i32, _i32, _i32, _f64, _i32,
                                   _p, _i32, _p],
    "sdk_topk_attn_fwd_workspace_size": [_i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32],
    "sdk_topk_attn_fwd_ws": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i32, _i32, _i32, _f64, _i32, _i32,
                             _p, ctypes.c_size_t, _p],
    "sdk_topk_attn_bwd": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i32, _i32, _i32, _f64, _i32,
                          _i32, _i32, _p],
    "sdk_topk_attn_fwd_biased": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i32, _i32, _i32, _f64, _i32,
                                 _p, _i64, _i32, _i32, _p],
    "sdk_topk_attn_bwd_biased": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i32, _i32, _i32, _f64,
                                 _i32, _i32, _p, _p, _i64, _i32, _i32, _p],
    "sdk_finalize_grad": [_p, _p, _i64, _f64, _i32, _p],
    "sdk_topk_attn_bwd_workspace_size": [_i64, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32],
    "sdk_topk_attn_bwd_direct": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i32, _i32, _i32,
                                 _f64, _i32, _i32, _p, ctypes.c_size_t, _p],
    "sdk_topk_attn_bwd_noalloc": [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i32, _i32, _i32, _f64, _i32, _p],
    "sdk_affinity": [_p, _p, _p, _i64, _i64, _i32, _i64, _i64, _i32, _p],
    "sdk_topk_select": [_p, _p, _p, _i64, _i64, _i64, _i32, _i32, _p],
    "sdk_topk_aggregate": [_p, _p, _p, _p, _i64, _i32, _i64, _i32, _i64, _i64, _i64, _i32, _i32, _i32, _p],
    "sdk_route_top1": [_p, _i64, _i32, _p, _p, _p, _p],
    "sdk_sparse_topk_attn_fwd": [_p, _p, _p, _p, _p, _p, _i64, _i64, _i32, _i64, _i32, _i32, _i32, _p],
    "sdk_sparse_topk_attn_bwd": [_p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i32, _i64, _i32, _i32, _i32, _p],
    "sdk_fill_scatter": [_p, _p, _p, _i64, _i32, _i64, _f64, _i32, _p],
}
_RESTYPES = {"sdk_status_string": ctypes.c_char_p, "sdk_last_cuda_error": ctypes.c_char_p,
             "sdk_topk_attn_fwd_workspace_size": ctypes.c_size_t, "sdk_topk_attn_bwd_workspace_size": ctypes.c_size_t}

_lock = threading.Lock()
_lib = None
_load_error: str | None = None


def load() -> ctypes.CDLL:
    """Load (once) and return the native library, or raise RuntimeError."""
    global _lib, _load_error
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            _load_error = f"{LIB_PATH.name} is not built"
        else:
            try:
                lib = ctypes.CDLL(str(LIB_PATH))
                for name, args in SIGNATURES.items():
                    fn = getattr(lib, name)
                    fn.argtypes = args
                    fn.restype = _RESTYPES.get(name, ctypes.c_int)
                _lib = lib
                return lib
            except OSError as exc:  # pragma: no cover - depends on the machine
                _load_error = str(exc)
        raise RuntimeError(
            f"sparsedict_b200 native library unavailable ({_load_error}); "
            "build it with `python -m sparsedict_b200.build`"
        )


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class NativeError(RuntimeError):
    """A native call returned a non-OK status."""

    def __init__(self, fn: str, status: int, detail: str = ""):
        self.status = status
        lib = load()
        text = lib.sdk_status_string(status).decode()
        msg = f"{fn} failed: {text}"
        if detail:
            msg += f" ({detail})"
        super().__init__(msg)


def call(name: str, *args) -> None:
    lib = load()
    status = getattr(lib, name)(*args)
    if status != SDK_OK:
        detail = lib.sdk_last_cuda_error().decode() if status == SDK_ERR_CUDA else ""
        raise NativeError(name, status, detail)


def max_topk(dtype: torch.dtype, d: int) -> int:
    return int(load().sdk_max_topk(TORCH_TO_SDK[dtype], int(d)))


def device_status(clear: bool = True, device: torch.device | None = None) -> int:
    """Read (and by default clear) the device status word of ``device``."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    bits = ctypes.c_uint(0)
    with torch.cuda.device(device):
        call("sdk_device_status", ctypes.byref(bits), int(clear), stream_of(device))
    return int(bits.value)


def set_wait_limit(ns: int) -> None:
    """Bound (ns) of each pipeline wait of the tensor-core forward; 0 restores 2 s."""
    call("sdk_set_wait_limit", int(ns))
