"""compute_retrace -- drop-in for src/rl_triton/ops/retrace.py (reference v0.1.3)."""
from __future__ import annotations

import torch

from rl_triton.ops._scan import _CORRECTNESS_WARNINGS
from rl_triton.ops.retrace_fused import _retrace_launch

# Kept for import compatibility: the reference reroutes seq_len above this to
# an unfused PyTorch + scan path (src/rl_triton/ops/retrace.py:49).  Here the
# fused kernel serves every length; the results are the same recurrence.
_TRITON_SEQ_LEN_CEILING = 2048


def compute_retrace(
    action_probs_target: torch.Tensor,
    action_probs_behavior: torch.Tensor,
    q_values: torch.Tensor,
    next_q_values_all: torch.Tensor,
    actions: torch.Tensor,
    rewards: torch.Tensor,
    terminateds: torch.Tensor,
    truncateds: torch.Tensor,
    gamma: float,
    lambda_: float = 1.0,
    c_bar: float = 1.0,
    rho_bar: float = 1.0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """
    Compute Retrace(λ) Q-value targets and advantages (Munos et al. 2016).

    Recurrence (src/rl_triton/ops/retrace.py:66-114):

    - Δ[t] = δ[t] + decay[t] * Δ[t+1],   Δ[T] = 0
    - δ[t]     = r[t] + γ · E_π[Q(s_{t+1},·)] · (1-terminated[t]) - Q(s_t,a_t)
    - decay[t] = γ · c[t+1] · (1-done[t]),  c[t] = λ · min(c_bar, π(a_t|s_t)/μ(a_t|s_t)),  c[T] = 0
    - Q_ret[t] = Q(s_t,a_t) + Δ[t]
    - A[t] = min(rho_bar, π/μ)[t] · (r[t] + γ · Q_ret[t+1] · (1-terminated[t]) - Q(s_t,a_t)),  Q_ret[T] = 0

    Actions outside [0, num_actions) contribute π(a_t|s_t) = 0 (the fused
    reference kernel's one-hot gather behaves the same way).

    Returns:
        retrace_targets, advantages: [num_envs, seq_len], float32.
    """
    # Cheap structural checks -- always-on (src/rl_triton/ops/retrace.py:116-141).
    for name, t in [
        ("action_probs_behavior", action_probs_behavior),
        ("q_values",              q_values),
        ("rewards",               rewards),
        ("terminateds",           terminateds),
        ("truncateds",            truncateds),
    ]:
        assert t.is_cuda,                 f"{name} must be on CUDA"
        assert t.dtype == torch.float32,  f"{name}: expected float32, got {t.dtype}"
        assert t.shape == rewards.shape,  f"{name} shape {t.shape} != rewards shape {rewards.shape}"

    assert action_probs_target.is_cuda,                "action_probs_target must be on CUDA"
    assert action_probs_target.dtype == torch.float32, "action_probs_target: expected float32"
    assert action_probs_target.shape[:2] == rewards.shape, (
        f"action_probs_target shape {action_probs_target.shape} incompatible with rewards {rewards.shape}"
    )
    assert next_q_values_all.is_cuda,                "next_q_values_all must be on CUDA"
    assert next_q_values_all.dtype == torch.float32, "next_q_values_all: expected float32"
    assert next_q_values_all.shape == action_probs_target.shape, (
        f"next_q_values_all {next_q_values_all.shape} != action_probs_target {action_probs_target.shape}"
    )
    assert actions.is_cuda,              "actions must be on CUDA"
    assert actions.dtype == torch.int64, f"actions: expected int64, got {actions.dtype}"
    assert actions.shape == rewards.shape, \
        f"actions shape {actions.shape} != rewards shape {rewards.shape}"

    if _CORRECTNESS_WARNINGS():
        assert not (terminateds.bool() & truncateds.bool()).any(), \
            "terminated and truncated are mutually exclusive: a step cannot be both"

    return _retrace_launch(action_probs_target, action_probs_behavior, q_values, next_q_values_all,
                           actions, rewards, truncateds, terminateds, gamma, lambda_, c_bar, rho_bar)
