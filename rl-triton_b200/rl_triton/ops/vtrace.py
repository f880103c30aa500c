"""compute_vtrace -- drop-in for src/rl_triton/ops/vtrace.py (reference v0.1.3)."""
from __future__ import annotations

import torch

from rl_triton.ops._scan import _CORRECTNESS_WARNINGS, _FLAT_MAX_SEQ_LEN, _float_ok
from rl_triton.ops.vtrace_fused import _vtrace_launch, compute_vtrace_fused


def compute_vtrace(
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
    Compute V-Trace targets and advantages (IMPALA, Espeholt et al. 2018).

    Recurrence (src/rl_triton/ops/vtrace.py:20-90):

    - Δ[t] = δ[t] + β[t] * Δ[t+1],   Δ[T] = 0
    - δ[t] = ρ[t] * (r[t] + γ * V(s_{t+1}) * (1 - terminated[t]) - V(s_t))
    - β[t] = γ * c[t] * (1 - done[t])
    - ρ[t] = min(ρ_bar, π/μ),  c[t] = min(c_bar, π/μ),  π/μ = exp(log_pi_target - log_pi_behavior)

    Outputs: vs[t] = Δ[t] + V(s_t) and A[t] = ρ[t] * (r[t] + γ * vs[t+1] * (1-terminated[t]) - V(s_t)).

    One fused kernel for every seq_len: the advantage's vs[t+1] is the scan
    carry entering step t, so there is no store/reload of the targets.

    Returns:
        vtrace_targets, vtrace_advantages: [num_envs, seq_len], float32.
    """
    num_envs, seq_len = rewards.shape
    has_truncations = truncateds is not None
    # Always on, whichever path serves the call: a host tensor never reaches a kernel.
    for name, t in [("log_pi_target", log_pi_target), ("log_pi_behavior", log_pi_behavior), ("values", values),
                    ("rewards", rewards), ("terminateds", terminateds), ("truncateds", truncateds),
                    ("bootstrap_values", bootstrap_values), ("last_value", last_value)]:
        if t is not None:
            assert t.is_cuda, f"{name} must be on CUDA"

    if _CORRECTNESS_WARNINGS():
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
            assert not (terminateds.bool() & truncateds.bool()).any(), \
                "terminated and truncated are mutually exclusive: a step cannot be both"
        if last_value is not None:
            assert bootstrap_values is None, \
                "pass either last_value (shape [num_envs], convenience for the " \
                "window boundary) or bootstrap_values (shape [num_envs, seq_len], " \
                "full per-step control), not both."
            assert last_value.shape == (num_envs,), \
                f"last_value must have shape [{num_envs}], got {last_value.shape}"
        if bootstrap_values is not None:
            assert bootstrap_values.is_cuda,                "bootstrap_values must be on CUDA"
            assert _float_ok(bootstrap_values),             "bootstrap_values: expected float32"
            assert bootstrap_values.shape == rewards.shape, \
                f"bootstrap_values shape {bootstrap_values.shape} != rewards shape {rewards.shape}"
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

    if seq_len <= _FLAT_MAX_SEQ_LEN:
        return compute_vtrace_fused(
            log_pi_target, log_pi_behavior,
            values, rewards, terminateds,
            truncateds=truncateds if has_truncations else None,
            gamma=gamma, rho_bar=rho_bar, c_bar=c_bar,
            bootstrap_values=bootstrap_values,
            last_value=last_value,
        )

    # seq_len > 131072: the reference's chunked path prefers last_value when
    # both are given (ops/vtrace.py:172-177) and forms next values additively.
    if last_value is not None:
        bootstrap_values = None
    return _vtrace_launch(log_pi_target, log_pi_behavior, values, rewards, terminateds, truncateds,
                          gamma, rho_bar, c_bar, bootstrap_values, last_value, flat=False)
