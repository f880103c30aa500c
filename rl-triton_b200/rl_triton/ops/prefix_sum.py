"""compute_episodic_prefix_sum -- drop-in for src/rl_triton/ops/prefix_sum.py."""
from __future__ import annotations

import torch

from rl_triton import _native as nat
from rl_triton.ops._scan import _CORRECTNESS_WARNINGS, _done, _placed, _seg, _warn_copies


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
    _placed(inputs, dones, seed_values)
    _warn_copies({"inputs": inputs, "dones": dones})
    t0, total, halo = _seg(_segment)
    out = nat.ops.prefix_sum(inputs, dones, seed_values, bool(ends_at), t0, total, halo)
    _done(inputs)
    return out
