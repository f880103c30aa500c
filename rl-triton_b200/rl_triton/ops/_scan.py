"""
Internal scan dispatch shared by all estimators (drop-in for
src/rl_triton/ops/_scan.py of the reference).

Both directions of the first-order affine recurrence run on the same
single-pass CUDA scan (librlscan.so):

Backward (right-to-left): A[t] = u[t] + v[t] * A[t+1],  A[T] = bootstrap
Forward  (left-to-right): e[t] = u[t] + v[t] * e[t-1],  e[-1] = seed

Unlike the reference there is no flat/chunked split: the kernel tiles the
time axis across CTAs with a decoupled look-back, so every length runs on the
same fused path.  `_FLAT_MAX_SEQ_LEN` is kept only because callers and tests
import it; it marks where the reference switches to its unfused chunked path
and where this package reproduces that path's input conventions.
"""
from __future__ import annotations

import os
import warnings

import torch

from rl_triton import _native as nat

# Set RL_TRITON_PERF_WARNINGS=1 to be warned about implicit copies
# (read once at import, like the reference: src/rl_triton/ops/_scan.py:27).
_PERF_WARNINGS = os.environ.get("RL_TRITON_PERF_WARNINGS", "0") == "1"


# Set RL_TRITON_CORRECTNESS_WARNINGS=1 to enable the expensive input checks
# (read per call: src/rl_triton/ops/_scan.py:30-31).
# Under torch.compile the data-dependent checks are skipped (they would
# synchronise and break the graph).
def _CORRECTNESS_WARNINGS() -> bool:
    if torch.compiler.is_compiling():
        return False
    return os.environ.get("RL_TRITON_CORRECTNESS_WARNINGS", "0") == "1"


def _perf_warn(msg: str) -> None:
    if _PERF_WARNINGS:
        warnings.warn(msg, stacklevel=3)


def _correctness_warn(msg: str) -> None:
    if _CORRECTNESS_WARNINGS():
        warnings.warn(msg, stacklevel=3)


_FLAT_MAX_SEQ_LEN = 131072

_FLOAT_DTYPES = (torch.float32, torch.bfloat16)


def _float_ok(t: torch.Tensor) -> bool:
    return t.dtype in _FLOAT_DTYPES


def _placed(ref: torch.Tensor, *others: torch.Tensor | None) -> None:
    """Always-on placement check: every tensor a kernel reads or writes is a
    CUDA tensor on `ref`'s device (the library checks the pointers again and
    refuses host memory before it launches anything)."""
    assert ref.is_cuda, "inputs must be on CUDA"
    dev = ref.device
    for t in others:
        if t is not None:
            assert t.is_cuda and t.device == dev, \
                f"all tensors of one call must be on {dev}; got a tensor on {t.device}"


def _warn_copies(named: dict) -> None:
    """RL_TRITON_PERF_WARNINGS=1: warn about the copies the operator will make
    (non-contiguous or not 16-byte aligned inputs)."""
    if not _PERF_WARNINGS:
        return
    for name, t in named.items():
        if t is None:
            continue
        if not t.is_contiguous():
            _perf_warn(f"{name} is not contiguous; a copy will be made. Call .contiguous() before the hot loop to avoid this overhead.")
        elif t.data_ptr() % 16 != 0:
            _perf_warn(f"{name} is not 16-byte aligned; a copy will be made.")


def _done(ref: torch.Tensor) -> None:
    """RL_TRITON_CORRECTNESS_WARNINGS=1: wait for the call and raise if one of
    its bounded device waits ran out."""
    if _CORRECTNESS_WARNINGS() and not torch.cuda.is_current_stream_capturing():
        nat.raise_if_device_error(ref.device)


def _seg(segment):
    """(t0, total, halo) of a time-split call, or the whole-rows defaults."""
    return segment if segment is not None else (-1, -1, None)


def _run_scan(
    u: torch.Tensor,
    v: torch.Tensor,
    bootstrap: torch.Tensor | None = None,
) -> torch.Tensor:
    """
    Backward linear scan: A[t] = u[t] + v[t] * A[t+1], A[T] = bootstrap.

    Same contract as src/rl_triton/ops/_scan.py:69-144.  Any seq_len runs on
    the single-pass tiled kernel (the reference splits at 131072 into a
    serial-chunk kernel).

    Args:
        u:         Additive term [num_envs, seq_len], float32, CUDA.
        v:         Multiplicative decay [num_envs, seq_len], float32, CUDA.
        bootstrap: Per-environment boundary value A[T], shape [num_envs], float32.

    Returns:
        out: A[t] values, shape [num_envs, seq_len], float32.
    """
    if not u.is_contiguous():
        _perf_warn("u is not contiguous; a copy will be made. Call .contiguous() before the hot loop to avoid this overhead.")
    if not v.is_contiguous():
        _perf_warn("v is not contiguous; a copy will be made. Call .contiguous() before the hot loop to avoid this overhead.")

    assert u.is_cuda and v.is_cuda, "u and v must be on CUDA"  # always on: a host pointer never reaches a kernel
    if _CORRECTNESS_WARNINGS():
        assert u.shape == v.shape,      "u and v must have the same shape"
        assert u.dtype == torch.float32, f"u: expected float32, got {u.dtype}"
        assert v.dtype == torch.float32, f"v: expected float32, got {v.dtype}"
        if bootstrap is not None:
            assert bootstrap.shape == (u.shape[0],), \
                f"bootstrap must have shape [{u.shape[0]}], got {bootstrap.shape}"
            assert bootstrap.is_cuda, "bootstrap must be on CUDA"
    return _affine(u, v, bootstrap, direction=0)


def _run_scan_forward(
    u: torch.Tensor,
    v: torch.Tensor,
    seed: torch.Tensor | None = None,
) -> torch.Tensor:
    """
    Forward linear scan: e[t] = u[t] + v[t] * e[t-1], e[-1] = seed.

    Same contract as src/rl_triton/ops/_scan.py:147-213, without the
    reference's seq_len <= 131072 limit (its forward scan has no chunked
    kernel; this one is tiled over time like the backward scan).
    """
    if not u.is_contiguous():
        _perf_warn("u is not contiguous; a copy will be made. Call .contiguous() before the hot loop to avoid this overhead.")
    if not v.is_contiguous():
        _perf_warn("v is not contiguous; a copy will be made. Call .contiguous() before the hot loop to avoid this overhead.")

    assert u.is_cuda and v.is_cuda, "u and v must be on CUDA"  # always on: a host pointer never reaches a kernel
    if _CORRECTNESS_WARNINGS():
        assert u.shape == v.shape,      "u and v must have the same shape"
        assert u.dtype == torch.float32, f"u: expected float32, got {u.dtype}"
        assert v.dtype == torch.float32, f"v: expected float32, got {v.dtype}"
        if seed is not None:
            assert seed.shape == (u.shape[0],), \
                f"seed must have shape [{u.shape[0]}], got {seed.shape}"
            assert seed.is_cuda, "seed must be on CUDA"
    return _affine(u, v, seed, direction=1)


def _affine(u, v, carry, direction, segment=None):
    _placed(u, v, carry)
    _warn_copies({"u": u, "v": v})
    t0, total, halo = _seg(segment)
    out = nat.ops.affine_scan(u, v, carry, direction, t0, total, halo)
    _done(u)
    return out
