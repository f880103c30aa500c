"""compute_episodic_prefix_sum -- drop-in for src/rl_triton/ops/prefix_sum.py."""
from __future__ import annotations

import torch

from rl_triton import _native as nat
from rl_triton.ops._scan import (
    _CORRECTNESS_WARNINGS,
    _launch_ctx,
    _ready,
    _scalar_f32,
    _unify,
)


def compute_episodic_prefix_sum(
    inputs: torch.Tensor,
    dones: torch.Tensor,
    seed_values: torch.Tensor | None = None,
    boundary: str = "ends_at",
    *,
    _segment=None,
) -> torch.Tensor:
    """
    Cumulative sum that resets at episode / segment boundaries
    (src/rl_triton/ops/prefix_sum.py:23-111).

    - "ends_at" (default): C[t] = x[t] + (1 - done[t-1]) * C[t-1],  done[-1] := 0
    - "starts_at":         C[t] = x[t] + (1 - done[t]) * C[t-1]
    - C[-1] = seed (or 0).

    Deliberate difference: the reference asserts seq_len <= 131072 (it has no
    chunked forward kernel); the tiled single-pass scan here accepts any
    length, e.g. one 2^28-step sequence.

    Returns:
        prefix_sums: C[t], [num_envs, seq_len], float32.
    """
    num_envs, seq_len = inputs.shape

    assert inputs.is_cuda and dones.is_cuda, "inputs and dones must be on CUDA"  # always on
    if _CORRECTNESS_WARNINGS():
        assert inputs.dtype in (torch.float32, torch.bfloat16), f"inputs: expected float32, got {inputs.dtype}"
        assert dones.dtype in (torch.float32, torch.bfloat16),  f"dones: expected float32, got {dones.dtype}"
        assert inputs.shape == dones.shape,   "inputs and dones must have the same shape"
        if seed_values is not None:
            assert seed_values.shape == (num_envs,), \
                f"seed_values must have shape [{num_envs}], got {seed_values.shape}"
            assert seed_values.is_cuda, "seed_values must be on CUDA"
        assert boundary in ("ends_at", "starts_at"), \
            f"boundary must be 'ends_at' or 'starts_at', got {boundary!r}"

    # The reference compiles any other string as "starts_at"
    # (BOUNDARY_ENDS_AT=(boundary == "ends_at"), ops/prefix_sum.py:110).
    ends_at = 1 if boundary == "ends_at" else 0
    (inputs, dones), dt = _unify([inputs, dones])
    inputs = _ready(inputs, "inputs")
    dones = _ready(dones, "dones")
    seed = _scalar_f32(seed_values)
    out = torch.empty(inputs.shape, dtype=torch.float32, device=inputs.device)
    dev, s = _launch_ctx(inputs, dones, seed, out)
    ws, wsb = nat.workspace(dev, s, num_envs * seq_len)
    st = nat.lib.rls_prefix_sum(
        inputs.data_ptr(), dones.data_ptr(), nat.ptr(seed), ends_at, out.data_ptr(),
        num_envs, seq_len, dt, _segment, ws, wsb, s,
    )
    nat.check(st, "rls_prefix_sum", dev)
    return out
