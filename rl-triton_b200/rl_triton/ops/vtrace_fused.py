"""compute_vtrace_fused -- drop-in for src/rl_triton/ops/vtrace_fused.py.

The reference keeps a separate fused entry point for seq_len <= 131072 with
always-on argument checks; compute_vtrace (ops/vtrace.py) routes there.  Both
run the same single-pass CUDA kernel here.
"""
from __future__ import annotations

import torch

from rl_triton import _native as nat
from rl_triton.ops._scan import _CORRECTNESS_WARNINGS, _FLAT_MAX_SEQ_LEN, _done, _float_ok, _placed, _warn_copies


def _vtrace_launch(log_pi_target, log_pi_behavior, values, rewards, terminateds, truncateds,
                   gamma, rho_bar, c_bar, bootstrap_values, last_value, flat):
    """Shared launcher: picks the bootstrap kind of the reference path taken."""
    num_envs, seq_len = rewards.shape
    has_truncations = truncateds is not None
    boot = None
    if last_value is not None:
        kind = nat.BOOT_ROW
    elif bootstrap_values is not None:
        boot = bootstrap_values
        if flat and not has_truncations:
            kind = nat.BOOT_LASTCOL  # ops/vtrace_fused.py:203-206: scalar bootstrap[:, -1]
        else:
            kind = nat.BOOT_FULL_ADD  # ops/vtrace_fused.py:161-171, ops/vtrace.py:163-177
    else:
        kind = nat.BOOT_NONE

    _placed(rewards, log_pi_target, log_pi_behavior, values, terminateds, truncateds, boot, last_value)
    _warn_copies({"log_pi_target": log_pi_target, "log_pi_behavior": log_pi_behavior, "values": values,
                  "rewards": rewards, "terminateds": terminateds, "truncateds": truncateds,
                  "bootstrap_values": boot})
    targets, advantages = nat.ops.vtrace(log_pi_target, log_pi_behavior, values, rewards, terminateds, truncateds,
                                         last_value if kind == nat.BOOT_ROW else boot, kind, float(gamma),
                                         float(rho_bar), float(c_bar))
    _done(rewards)
    return targets, advantages


def compute_vtrace_fused(
    log_pi_target: torch.Tensor,
    log_pi_behavior: torch.Tensor,
    values: torch.Tensor,
    rewards: torch.Tensor,
    terminateds: torch.Tensor,
    truncateds: torch.Tensor | None = None,
    gamma: float = 0.99,
    rho_bar: float = 1.0,
    c_bar: float = 1.0,
    bootstrap_values: torch.Tensor | None = None,
    last_value: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """
    Fused V-Trace targets and advantages (src/rl_triton/ops/vtrace_fused.py:23-220).

    Same arguments, checks and results as the reference; valid for
    seq_len <= 131072 (use compute_vtrace for any length).

    Returns:
        vtrace_targets:    [num_envs, seq_len], float32.
        vtrace_advantages: [num_envs, seq_len], float32.
    """
    num_envs, seq_len = rewards.shape
    has_truncations = truncateds is not None

    # Always-on structural checks (ops/vtrace_fused.py:97-125).
    for name, t in [
        ("log_pi_target",   log_pi_target),
        ("log_pi_behavior", log_pi_behavior),
        ("values",          values),
        ("rewards",         rewards),
        ("terminateds",     terminateds),
    ]:
        assert t.is_cuda,                f"{name} must be on CUDA"
        assert _float_ok(t),             f"{name}: expected float32 (or bfloat16), got {t.dtype}"
        assert t.shape == rewards.shape, f"{name} shape {t.shape} != rewards shape {rewards.shape}"
    if has_truncations:
        assert truncateds.is_cuda,                "truncateds must be on CUDA"
        assert _float_ok(truncateds),             "truncateds: expected float32"
        assert truncateds.shape == rewards.shape, \
            f"truncateds shape {truncateds.shape} != rewards shape {rewards.shape}"
    if last_value is not None:
        assert bootstrap_values is None, \
            "pass either last_value (shape [num_envs], convenience for the " \
            "window boundary) or bootstrap_values (shape [num_envs, seq_len], " \
            "full per-step control), not both."
        assert last_value.shape == (num_envs,), \
            f"last_value must have shape [{num_envs}], got {last_value.shape}"
        assert last_value.is_cuda,                "last_value must be on CUDA"
        assert last_value.dtype == torch.float32, "last_value: expected float32"
    if bootstrap_values is not None:
        assert bootstrap_values.is_cuda,                "bootstrap_values must be on CUDA"
        assert _float_ok(bootstrap_values),             "bootstrap_values: expected float32"
        assert bootstrap_values.shape == rewards.shape, \
            f"bootstrap_values shape {bootstrap_values.shape} != rewards shape {rewards.shape}"

    if _CORRECTNESS_WARNINGS():
        if has_truncations:
            assert not (terminateds.bool() & truncateds.bool()).any(), \
                "terminated and truncated are mutually exclusive: a step cannot be both"
        if has_truncations and bootstrap_values is not None:
            interior = torch.ones_like(truncateds, dtype=torch.bool)
            interior[:, -1] = False
            stray = (bootstrap_values != 0) & (truncateds == 0) & interior
            assert not stray.any(), (
                "bootstrap_values must be zero at non-truncated interior steps. "
                "Nonzero entries there double-count via the additive v_next trick "
                "and corrupt delta. Populate bootstrap_values only at truncated "
                "steps and at the final column (window boundary)."
            )

    assert seq_len <= _FLAT_MAX_SEQ_LEN, (
        f"seq_len={seq_len} exceeds the flat kernel limit {_FLAT_MAX_SEQ_LEN}. "
        "Use compute_vtrace for longer sequences (it auto-dispatches to chunked)."
    )
    return _vtrace_launch(log_pi_target, log_pi_behavior, values, rewards, terminateds, truncateds,
                          gamma, rho_bar, c_bar, bootstrap_values, last_value, flat=True)
