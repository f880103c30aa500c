"""compute_retrace_fused -- drop-in for src/rl_triton/ops/retrace_fused.py.

The reference uses its fused Triton kernel only up to seq_len 2048 (register
spills above that).  Here one kernel serves every length: the [N, T, A]
tensors are staged per warp into shared memory with bulk copies, so register
use does not grow with seq_len or with the number of actions.
"""
from __future__ import annotations

import torch

from rl_triton import _native as nat
from rl_triton.ops._scan import _launch_ctx, _ready


def _retrace_launch(action_probs_target, action_probs_behavior, q_values, next_q_values_all, actions,
                    rewards, truncateds, terminateds, gamma, lambda_, c_bar, rho_bar):
    num_envs, seq_len = rewards.shape
    num_actions = action_probs_target.shape[2]
    f = lambda t, n: _ready(t if t.dtype == torch.float32 else t.float(), n)  # noqa: E731
    pi = f(action_probs_target, "action_probs_target")
    mu = f(action_probs_behavior, "action_probs_behavior")
    q = f(q_values, "q_values")
    nq = f(next_q_values_all, "next_q_values_all")
    act = _ready(actions, "actions")
    r = f(rewards, "rewards")
    term = f(terminateds, "terminateds")
    trunc = f(truncateds, "truncateds")
    targets = torch.empty(rewards.shape, dtype=torch.float32, device=rewards.device)
    advantages = torch.empty_like(targets)
    dev, s = _launch_ctx(rewards, pi, mu, q, nq, act, term, trunc, targets, advantages)
    ws, wsb = nat.workspace(dev, s, num_envs * seq_len)
    st = nat.lib.rls_retrace(
        pi.data_ptr(), mu.data_ptr(), q.data_ptr(), nq.data_ptr(), act.data_ptr(), r.data_ptr(),
        term.data_ptr(), trunc.data_ptr(), targets.data_ptr(), advantages.data_ptr(),
        num_envs, seq_len, num_actions, float(gamma), float(lambda_), float(c_bar), float(rho_bar),
        ws, wsb, s,
    )
    nat.check(st, "rls_retrace", dev)
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
