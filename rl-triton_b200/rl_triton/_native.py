"""ctypes binding of librlscan.so (C ABI declared in include/rlscan.h).

The library is the only compute path: there is no CPU or PyTorch fallback.
If the shared object is missing or fails to load, importing this module
raises, so a broken build can never silently run some other code.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("RLSCAN_LIB", os.path.join(_HERE, "_lib", "librlscan.so"))

RLS_OK = 0
RLS_F32 = 0
RLS_BF16 = 1
RLS_ETOOLARGE = 6
RLS_ENOTDEVICE = 7
NOALLOC_MAX_ELEMENTS = 1 << 27

BOOT_NONE = 0
BOOT_ROW = 1
BOOT_LASTCOL = 2
BOOT_FULL_ADD = 3
BOOT_FULL_SEL = 4

ALG_GAE = 0
ALG_LAMBDA = 1
ALG_DISCOUNTED = 2
ALG_ELIGIBILITY = 3
ALG_PREFIX = 4
ALG_SCAN_BWD = 5
ALG_SCAN_FWD = 6


class Segment(ctypes.Structure):
    """Mirror of rls_segment_t."""

    _fields_ = [("t0", ctypes.c_int64), ("total_len", ctypes.c_int64), ("halo", ctypes.c_void_p)]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"librlscan.so not found at {LIB_PATH}; build it with "
            "`python rl-triton_b200/build.py` (nvcc, sm_100a)"
        )
    return ctypes.CDLL(LIB_PATH)


lib = _load()

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_F = ctypes.c_float
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_SEG = ctypes.POINTER(Segment)

_SIGS = {
    "rls_workspace_bytes": (_SZ, [_I64]),
    "rls_workspace_error": (_I, [_P, _P]),
    "rls_status_string": (ctypes.c_char_p, [_I]),
    "rls_build_info": (ctypes.c_char_p, []),
    "rls_gae": (_I, [_P, _P, _P, _P, _P, _I, _P, _I64, _I64, _F, _F, _I, _SEG, _P, _SZ, _P]),
    "rls_vtrace": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _I64, _I64, _F, _F, _F, _I, _P, _SZ, _P]),
    "rls_retrace": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _F, _F, _F, _F, _P, _SZ, _P]),
    "rls_lambda_returns": (_I, [_P, _P, _P, _P, _P, _I, _P, _I64, _I64, _F, _F, _I, _SEG, _P, _SZ, _P]),
    "rls_discounted_returns": (_I, [_P, _P, _P, _P, _I, _P, _I64, _I64, _F, _I, _SEG, _P, _SZ, _P]),
    "rls_eligibility_traces": (_I, [_P, _P, _P, _P, _I64, _I64, _F, _F, _I, _SEG, _P, _SZ, _P]),
    "rls_prefix_sum": (_I, [_P, _P, _P, _I, _P, _I64, _I64, _I, _SEG, _P, _SZ, _P]),
    "rls_affine_scan": (_I, [_P, _P, _P, _I, _P, _I64, _I64, _SEG, _P, _SZ, _P]),
    "rls_segment_reduce": (_I, [_I, _P, _P, _I, _P, _P, _P, _I64, _I64, _F, _I, _SEG, _P]),
    "rls_segment_fixup": (_I, [_I, _P, _P, _I, _P, _P, _I64, _I64, _F, _I, _SEG, _P]),
    "rls_gae_noalloc": (_I, [_P, _P, _P, _P, _P, _I, _P, _I64, _I64, _F, _F, _I, _SEG, _P]),
    "rls_gae_noalloc_error": (_I, [_P]),
}
for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args

EXPORTED = tuple(_SIGS)


def check(status: int, what: str, device: torch.device | None = None) -> None:
    """Raise RuntimeError for a non-OK status.  With
    RL_TRITON_CORRECTNESS_WARNINGS=1 also wait for the call and raise if one
    of its bounded device waits ran out (see raise_if_device_error)."""
    if status != RLS_OK:
        msg = lib.rls_status_string(status).decode()
        raise RuntimeError(f"{what}: librlscan status {status} ({msg})")
    if device is not None and os.environ.get("RL_TRITON_CORRECTNESS_WARNINGS", "0") == "1":
        raise_if_device_error(device)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return RLS_F32
    if t.dtype == torch.bfloat16:
        return RLS_BF16
    raise AssertionError(f"unsupported dtype {t.dtype}")


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ---------------------------------------------------------------------------
# Per-(device, stream) workspace: tile status words for the decoupled
# look-back.  Zero-filled once at allocation; the kernels keep it consistent
# across calls on the same stream (an epoch counter lives in its header).
# ---------------------------------------------------------------------------
_ws_lock = threading.Lock()
_ws_cache: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device, stream: int, num_elements: int) -> tuple[int, int]:
    need = int(lib.rls_workspace_bytes(max(int(num_elements), 1)))
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, stream)
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < need:
            size = max(need, 1 << 16)
            if buf is not None:
                size = max(size, 2 * buf.numel())
            buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
            _ws_cache[key] = buf
    return buf.data_ptr(), buf.numel()


def workspace_error(device: torch.device | None = None) -> int:
    """Bounded-wait error latch of the current stream's workspace (syncs)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    idx = device.index if device.index is not None else torch.cuda.current_device()
    s = stream_handle(device)
    buf = _ws_cache.get((idx, s))
    if buf is None:
        return 0
    return int(lib.rls_workspace_error(ctypes.c_void_p(buf.data_ptr()), ctypes.c_void_p(s)))


def raise_if_device_error(device: torch.device | None = None) -> None:
    """Raise RuntimeError if a bounded device wait ran out on the current
    stream's workspace since the last read (synchronises the stream).  The
    estimators call it after every launch when RL_TRITON_CORRECTNESS_WARNINGS=1;
    otherwise callers may call it when they choose."""
    err = workspace_error(device)
    if err:
        raise RuntimeError(
            f"librlscan: a bounded device wait ran out (error bits {err:#x}); the results of the calls on this "
            "stream since the last check are not valid")


def build_info() -> str:
    return lib.rls_build_info().decode()
