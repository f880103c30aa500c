"""compute_lambda_returns / compute_discounted_returns / compute_eligibility_traces --
drop-in for src/rl_triton/ops/returns.py (reference v0.1.3)."""
from __future__ import annotations

import torch

from rl_triton import _native as nat
from rl_triton.ops._scan import _CORRECTNESS_WARNINGS, _done, _float_ok, _placed, _seg, _warn_copies


def _boot_kind(has_truncations: bool, bootstrap_values) -> int:
    """Reference semantics (ops/returns.py:122-152, :235-263): with truncations
    the bootstrap enters u at truncated steps and seeds the carry from its last
    column; without, only the last column seeds the carry."""
    if bootstrap_values is None:
        return nat.BOOT_NONE
    return nat.BOOT_FULL_ADD if has_truncations else nat.BOOT_LASTCOL


def _check_common(names_tensors, rewards, truncateds, bootstrap_values):
    for name, t in names_tensors:
        assert t.is_cuda,                f"{name} must be on CUDA"
        assert _float_ok(t),             f"{name}: expected float32 (or bfloat16), got {t.dtype}"
        assert t.shape == rewards.shape, f"{name} shape {t.shape} != rewards shape {rewards.shape}"
    if truncateds is not None:
        assert truncateds.is_cuda,                "truncateds must be on CUDA"
        assert _float_ok(truncateds),             "truncateds: expected float32"
        assert truncateds.shape == rewards.shape, \
            f"truncateds shape {truncateds.shape} != rewards shape {rewards.shape}"
    if bootstrap_values is not None:
        assert bootstrap_values.is_cuda,                "bootstrap_values must be on CUDA"
        assert _float_ok(bootstrap_values),             "bootstrap_values: expected float32"
        assert bootstrap_values.shape == rewards.shape, \
            f"bootstrap_values shape {bootstrap_values.shape} != rewards shape {rewards.shape}"


def compute_lambda_returns(
    rewards: torch.Tensor,
    next_values: torch.Tensor,
    terminateds: torch.Tensor,
    truncateds: torch.Tensor | None = None,
    gamma: float = 0.99,
    lambda_: float = 0.95,
    bootstrap_values: torch.Tensor | None = None,
    *,
    _segment=None,
) -> torch.Tensor:
    """
    Compute TD(λ) targets (λ-returns) via a backward affine scan.

    Recurrence (src/rl_triton/ops/returns.py:42-74):

    - G[t] = r[t] + γ*(1-done[t]) * [(1-λ)*V(s_{t+1}) + λ*G[t+1]] + γ*truncated[t]*bootstrap[t]
    - done[t] = terminated[t] | truncated[t];  G[T] = bootstrap[:, -1] (or 0)

    The caller must zero next_values at truncated steps.

    Returns:
        lambda_returns: G[t], [num_envs, seq_len], float32.
    """
    num_envs, seq_len = rewards.shape
    has_truncations = truncateds is not None
    _check_common([("rewards", rewards), ("next_values", next_values), ("terminateds", terminateds)],
                  rewards, truncateds, bootstrap_values)
    if _CORRECTNESS_WARNINGS():
        if has_truncations:
            assert not (terminateds.bool() & truncateds.bool()).any(), \
                "terminated and truncated are mutually exclusive: a step cannot be both"

    kind = _boot_kind(has_truncations, bootstrap_values)
    _placed(rewards, next_values, terminateds, truncateds, bootstrap_values)
    _warn_copies({"rewards": rewards, "next_values": next_values, "terminateds": terminateds,
                  "truncateds": truncateds, "bootstrap_values": bootstrap_values})
    t0, total, halo = _seg(_segment)
    out = nat.ops.lambda_returns(rewards, next_values, terminateds, truncateds, bootstrap_values, kind, float(gamma),
                                 float(lambda_), t0, total, halo)
    _done(rewards)
    return out


def compute_discounted_returns(
    rewards: torch.Tensor,
    terminateds: torch.Tensor,
    truncateds: torch.Tensor | None = None,
    gamma: float = 0.99,
    bootstrap_values: torch.Tensor | None = None,
    *,
    _segment=None,
) -> torch.Tensor:
    """
    Compute discounted returns (reward-to-go) via a backward affine scan.

    Recurrence (src/rl_triton/ops/returns.py:162-176):

    - G[t] = r[t] + γ*(1-done[t])*G[t+1] + γ*truncated[t]*bootstrap[t]
    - done[t] = terminated[t] | truncated[t];  G[T] = bootstrap[:, -1] (or 0)

    Returns:
        returns: G[t], [num_envs, seq_len], float32.
    """
    num_envs, seq_len = rewards.shape
    has_truncations = truncateds is not None
    _check_common([("rewards", rewards), ("terminateds", terminateds)], rewards, truncateds, bootstrap_values)
    if _CORRECTNESS_WARNINGS():
        if has_truncations:
            assert not (terminateds.bool() & truncateds.bool()).any(), \
                "terminated and truncated are mutually exclusive: a step cannot be both"

    kind = _boot_kind(has_truncations, bootstrap_values)
    _placed(rewards, terminateds, truncateds, bootstrap_values)
    _warn_copies({"rewards": rewards, "terminateds": terminateds, "truncateds": truncateds,
                  "bootstrap_values": bootstrap_values})
    t0, total, halo = _seg(_segment)
    out = nat.ops.discounted_returns(rewards, terminateds, truncateds, bootstrap_values, kind, float(gamma), t0,
                                     total, halo)
    _done(rewards)
    return out


def compute_eligibility_traces(
    gradients: torch.Tensor,
    dones: torch.Tensor,
    gamma: float,
    lambda_: float,
    seed_values: torch.Tensor | None = None,
    *,
    _segment=None,
) -> torch.Tensor:
    """
    Compute accumulating eligibility traces via a forward affine scan.

    Recurrence (src/rl_triton/ops/returns.py:273-290):

    - z[t] = g[t] + γ·λ·(1 - done[t-1]) * z[t-1],  z[-1] = seed,  done[-1] := 0

    `dones` uses the package-wide convention (done[t]=1: the episode ends at
    t); the carry into t is cut by done[t-1].  No seq_len limit (the reference
    asserts seq_len <= 131072; the tiled forward scan here has none).

    Returns:
        traces: z[t], [num_envs, seq_len], float32.
    """
    num_envs, seq_len = gradients.shape
    assert gradients.is_cuda and dones.is_cuda, "gradients and dones must be on CUDA"
    assert _float_ok(gradients), f"gradients: expected float32 (or bfloat16), got {gradients.dtype}"
    assert _float_ok(dones),     f"dones: expected float32 (or bfloat16), got {dones.dtype}"
    assert gradients.shape == dones.shape,   "gradients and dones must have the same shape"
    if seed_values is not None:
        assert seed_values.shape == (num_envs,), \
            f"seed_values must have shape [{num_envs}], got {seed_values.shape}"
        assert seed_values.is_cuda, "seed_values must be on CUDA"

    _placed(gradients, dones, seed_values)
    _warn_copies({"gradients": gradients, "dones": dones})
    t0, total, halo = _seg(_segment)
    out = nat.ops.eligibility_traces(gradients, dones, seed_values, float(gamma), float(lambda_), t0, total, halo)
    _done(gradients)
    return out
