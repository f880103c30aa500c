"""ctypes binding of librlscan.so (C ABI declared in include/rlscan.h).

The library is the only compute path: there is no CPU or PyTorch fallback.
If the shared object is missing or fails to load, importing this module
raises, so a broken build can never silently run some other code.
"""
from __future__ import annotations

import ctypes
import os

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
SEG_EXCLUSIVE = 2
LOSS_MSE = 0
LOSS_HUBER = 1


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

TORCH_LIB_PATH = os.path.join(os.path.dirname(LIB_PATH), "librlscan_torch.so")
if not os.path.exists(TORCH_LIB_PATH):
    raise ImportError(f"librlscan_torch.so not found at {TORCH_LIB_PATH}; build it with "
                      "`python rl-triton_b200/build.py`")
torch.ops.load_library(TORCH_LIB_PATH)
ops = torch.ops.rl_triton  # the estimators as PyTorch operators (csrc/torch_ops.cpp)


# Fake (meta) kernels: output shapes and dtypes without running anything, so
# torch.compile can trace through the operators.
def _f32_like(t):
    return torch.empty(t.shape, dtype=torch.float32, device=t.device)


@torch.library.register_fake("rl_triton::gae")
def _(rewards, values, terminateds, truncateds, bootstrap, boot_kind, gamma, lambda_, t0=-1, total=-1, halo=None):
    return _f32_like(rewards)


@torch.library.register_fake("rl_triton::gae_normalized")
def _(rewards, values, terminateds, truncateds, bootstrap, boot_kind, gamma, lambda_, eps):
    return _f32_like(rewards), _f32_like(rewards)


@torch.library.register_fake("rl_triton::gae_value_loss")
def _(rewards, values, terminateds, truncateds, bootstrap, boot_kind, new_values, gamma, lambda_, loss_kind, delta):
    return (_f32_like(rewards), _f32_like(rewards), torch.empty((), dtype=torch.float32, device=rewards.device),
            _f32_like(rewards))


@torch.library.register_fake("rl_triton::gae_obs_skip")
def _(rewards, values, mask, gamma, lambda_):
    return _f32_like(rewards), _f32_like(rewards)


@torch.library.register_fake("rl_triton::vtrace")
def _(lpt, lpb, values, rewards, terminateds, truncateds, bootstrap, boot_kind, gamma, rho_bar, c_bar):
    return _f32_like(rewards), _f32_like(rewards)


@torch.library.register_fake("rl_triton::retrace")
def _(pi, mu, q, nq, actions, rewards, terminateds, truncateds, gamma, lambda_, c_bar, rho_bar):
    return _f32_like(rewards), _f32_like(rewards)


@torch.library.register_fake("rl_triton::lambda_returns")
def _(rewards, next_values, terminateds, truncateds, bootstrap, boot_kind, gamma, lambda_, t0=-1, total=-1,
      halo=None):
    return _f32_like(rewards)


@torch.library.register_fake("rl_triton::discounted_returns")
def _(rewards, terminateds, truncateds, bootstrap, boot_kind, gamma, t0=-1, total=-1, halo=None):
    return _f32_like(rewards)


@torch.library.register_fake("rl_triton::eligibility_traces")
def _(gradients, dones, seed_values, gamma, lambda_, t0=-1, total=-1, halo=None):
    return _f32_like(gradients)


@torch.library.register_fake("rl_triton::prefix_sum")
def _(inputs, dones, seed_values, ends_at, t0=-1, total=-1, halo=None):
    return _f32_like(inputs)


@torch.library.register_fake("rl_triton::affine_scan")
def _(u, v, carry, direction, t0=-1, total=-1, halo=None):
    return _f32_like(u)

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
    "rls_segment_summary": (_I, [_I, _P, _P, _P, _I, _P, _P, _I64, _I64, _F, _F, _I, _SEG, _P]),
    "rls_segment_compose": (_I, [_P, _I, _I, _I, _I64, _P, _P]),
    "rls_gae_normalized": (_I, [_P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _I64, _I64, _F, _F, _F, _I, _P, _SZ, _P]),
    "rls_gae_value_loss": (_I, [_P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _P, _I64, _I64, _F, _F, _I, _F, _I, _P, _SZ,
                                _P]),
    "rls_gae_obs_skip": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _F, _F, _I, _P]),
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
    if (device is not None and os.environ.get("RL_TRITON_CORRECTNESS_WARNINGS", "0") == "1"
            and not torch.cuda.is_current_stream_capturing()):  # a capture cannot synchronise
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
# Per-(device, stream) workspace: tile records for the decoupled look-back.
# Owned by the operator library (one cache for every caller); zero-filled once
# at allocation, kept consistent across calls on the same stream by the
# kernels (an epoch counter lives in its header).
# ---------------------------------------------------------------------------
def workspace(device: torch.device, stream: int, num_elements: int) -> tuple[int, int]:
    """(pointer, bytes) of the current stream's workspace on `device`, large
    enough for num_elements; for callers of the C ABI on that stream."""
    like = torch.empty(0, device=device)
    assert stream == stream_handle(like.device), "workspace() serves the device's current stream"
    buf = ops.workspace(like, max(int(num_elements), 1))
    return buf.data_ptr(), buf.numel()


def workspace_error(device: torch.device | None = None) -> int:
    """Bounded-wait error latch of the current stream's workspace (syncs the
    stream, clears the latch)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    return int(ops.workspace_error(torch.empty(0, device=device)))


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
