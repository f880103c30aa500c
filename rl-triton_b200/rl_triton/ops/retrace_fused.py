"""compute_retrace_fused -- drop-in for src/rl_triton/ops/retrace_fused.py.

The reference uses its fused Triton kernel only up to seq_len 2048 (register
spills above that).  Here one kernel serves every length: the [N, T, A]
tensors are staged per warp into shared memory with bulk copies, so register
use does not grow with seq_len or with the number of actions.
"""
from __future__ import annotations

import torch

from rl_triton import _native as nat
from rl_triton.ops._scan import _done, _placed, _warn_copies


def _retrace_launch(action_probs_target, action_probs_behavior, q_values, next_q_values_all, actions,
                    rewards, truncateds, terminateds, gamma, lambda_, c_bar, rho_bar):
    _placed(rewards, action_probs_target, action_probs_behavior, q_values, next_q_values_all, actions, terminateds,
            truncateds)
    _warn_copies({"action_probs_target": action_probs_target, "action_probs_behavior": action_probs_behavior,
                  "q_values": q_values, "next_q_values_all": next_q_values_all, "actions": actions,
                  "rewards": rewards, "terminateds": terminateds, "truncateds": truncateds})
    targets, advantages = nat.ops.retrace(action_probs_target, action_probs_behavior, q_values, next_q_values_all,
                                          actions, rewards, terminateds, truncateds, float(gamma), float(lambda_),
                                          float(c_bar), float(rho_bar))
    _done(rewards)
    return targets, advantages


def compute_retrace_fused(
    action_probs_target: torch.Tensor,
    action_probs_behavior: torch.Tensor,
    q_values: torch.Tensor,
    next_q_values_all: torch.Tensor,
    actions: torch.Tensor,
    rewards: torch.Tensor,
    truncateds: torch.Tensor,
    terminated: torch.Tensor,
    gamma: float,
    lambda_: float = 1.0,
    c_bar: float = 1.0,
    rho_bar: float = 1.0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """
    Fused Retrace(λ) (src/rl_triton/ops/retrace_fused.py:26-118; note the
    reference's argument order: truncateds before terminated).

    Returns:
        retrace_targets: Q_ret[t], [num_envs, seq_len], float32.
        advantages:      A[t],     [num_envs, seq_len], float32.
    """
    seq_len = rewards.shape[1]
    assert seq_len <= 131072, (
        f"seq_len={seq_len} exceeds flat kernel limit 131072."
    )
    return _retrace_launch(action_probs_target, action_probs_behavior, q_values, next_q_values_all,
                           actions, rewards, truncateds, terminated, gamma, lambda_, c_bar, rho_bar)
