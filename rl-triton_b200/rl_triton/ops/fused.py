"""Fused epilogues of the estimators for a PPO update (no counterpart in the
reference, whose ROADMAP.md lists "fused GAE + advantage normalisation" for
v0.2).  Same argument conventions and checks as compute_gae."""
from __future__ import annotations

import torch

from rl_triton import _native as nat
from rl_triton.ops._scan import _done, _placed, _warn_copies
from rl_triton.ops.gae import _gae_args


def compute_gae_normalized(
    rewards: torch.Tensor,
    values: torch.Tensor,
    terminateds: torch.Tensor,
    truncateds: torch.Tensor | None = None,
    gamma: float = 0.99,
    lambda_: float = 0.95,
    bootstrap_values: torch.Tensor | None = None,
    last_value: torch.Tensor | None = None,
    eps: float = 1e-8,
    return_returns: bool = False,
):
    """
    GAE advantages normalised over the whole batch, in one kernel when the
    batch fits on chip:

        A = compute_gae(...)                      (same arguments and rules)
        normalized = (A - A.mean()) / (A.std() + eps)   (unbiased std)

    With return_returns=True also returns the value targets A + V (V =
    `values`), computed in the same pass.

    Returns:
        normalized advantages [num_envs, seq_len] float32, or
        (normalized advantages, returns) when return_returns is True.
    """
    kind, boot = _gae_args(rewards, values, terminateds, truncateds, bootstrap_values, last_value)
    _placed(rewards, values, terminateds, truncateds, boot, last_value)
    _warn_copies({"rewards": rewards, "values": values, "terminateds": terminateds, "truncateds": truncateds,
                  "bootstrap_values": boot})
    norm, rets = nat.ops.gae_normalized(rewards, values, terminateds, truncateds,
                                        last_value if kind == nat.BOOT_ROW else boot, kind, float(gamma),
                                        float(lambda_), float(eps))
    _done(rewards)
    return (norm, rets) if return_returns else norm


class _GaeValueLoss(torch.autograd.Function):
    """Forward: the fused kernel (advantages, returns, loss and d loss / d V').
    Backward: the stored gradient scaled by the loss's incoming gradient."""

    @staticmethod
    def forward(ctx, new_values, rewards, values, terminateds, truncateds, boot, kind, gamma, lambda_, loss_kind,
                delta):
        adv, rets, loss, grad = nat.ops.gae_value_loss(rewards, values, terminateds, truncateds, boot, kind,
                                                       new_values.detach(), gamma, lambda_, loss_kind, delta)
        ctx.save_for_backward(grad)
        ctx.nv_dtype = new_values.dtype
        ctx.mark_non_differentiable(adv, rets)
        return adv, rets, loss

    @staticmethod
    def backward(ctx, g_adv, g_rets, g_loss):
        (grad,) = ctx.saved_tensors
        return ((grad * g_loss).to(ctx.nv_dtype),) + (None,) * 10


def compute_gae_value_loss(
    rewards: torch.Tensor,
    values: torch.Tensor,
    terminateds: torch.Tensor,
    new_values: torch.Tensor,
    truncateds: torch.Tensor | None = None,
    gamma: float = 0.99,
    lambda_: float = 0.95,
    bootstrap_values: torch.Tensor | None = None,
    last_value: torch.Tensor | None = None,
    loss: str = "mse",
    delta: float = 1.0,
):
    """
    GAE and the PPO value loss in one pass over the rollout:

        A = compute_gae(rewards, values, terminateds, ...)   (same rules)
        returns = A + values
        value_loss = mse_loss(new_values, returns)            (loss="mse")
                   = huber_loss(new_values, returns, delta)   (loss="huber")

    `new_values` are the value head's predictions for the same steps; the loss
    is differentiable with respect to them (the gradient is computed in the
    same pass and stored for backward).  Returns (advantages, returns,
    value_loss); advantages and returns carry no gradient.
    """
    assert loss in ("mse", "huber"), f"loss must be 'mse' or 'huber', got {loss!r}"
    assert new_values.shape == rewards.shape, \
        f"new_values shape {new_values.shape} != rewards shape {rewards.shape}"
    kind, boot = _gae_args(rewards, values, terminateds, truncateds, bootstrap_values, last_value)
    _placed(rewards, values, terminateds, truncateds, boot, last_value, new_values)
    bt = last_value if kind == nat.BOOT_ROW else boot
    adv, rets, vloss = _GaeValueLoss.apply(new_values, rewards, values, terminateds, truncateds, bt, kind, float(gamma),
                                           float(lambda_), nat.LOSS_MSE if loss == "mse" else nat.LOSS_HUBER,
                                           float(delta))
    _done(rewards)
    return adv, rets, vloss


def compute_gae_obs_skip(
    rewards: torch.Tensor,
    values: torch.Tensor,
    response_mask: torch.Tensor,
    gamma: float = 1.0,
    lambda_: float = 1.0,
    return_returns: bool = True,
):
    """
    GAE for multi-turn / tool-use LLM rollouts with observation tokens
    (ROADMAP.md of the reference, v0.2 "observation-skip masking"):
    tokens with response_mask 0 pass the recurrence through unchanged, and a
    generated token's TD error uses the value of the next generated token.

        NV[t] = values at the next t' > t with mask 1 (0 if none)
        A[t]  = mask[t] ? r[t] + gamma*NV[t] - V[t] + gamma*lambda*A[t+1] : A[t+1]
        A[T]  = 0,  returns = A + V

    response_mask may be bool, integer or floating ({0, 1}).  Returns
    (advantages, returns) [num_envs, seq_len] float32, or the advantages only.
    """
    assert rewards.shape == values.shape == response_mask.shape, \
        f"rewards {rewards.shape}, values {values.shape} and response_mask {response_mask.shape} must match"
    _placed(rewards, values, response_mask)
    mask = response_mask if response_mask.dtype in (torch.float32, torch.bfloat16) else response_mask.float()
    num_envs, seq_len = rewards.shape
    if num_envs < _OBS_SKIP_MIN_ROWS and seq_len >= _OBS_SKIP_LONG_ROW:
        adv, rets = _obs_skip_long_rows(rewards, values, mask, float(gamma), float(lambda_))
    else:
        adv, rets = nat.ops.gae_obs_skip(rewards, values, mask, float(gamma), float(lambda_))
    _done(rewards)
    return (adv, rets) if return_returns else adv


# The fused kernel gives each row one warp: a handful of very long rows (a few
# sequences of 10^5+ tokens) would leave the GPU idle.  They take the two scans
# as generic affine scans instead, which split rows across the whole GPU.
_OBS_SKIP_MIN_ROWS = 8 * 148
_OBS_SKIP_LONG_ROW = 4096


def _obs_skip_long_rows(rewards, values, mask, gamma, lambda_):
    from rl_triton.ops._scan import _affine

    r, v, m = rewards.float(), values.float(), mask.float()
    # NV[t] = m[t+1] V[t+1] + (1 - m[t+1]) NV[t+1], NV[T-1] = 0
    m_next = torch.nn.functional.pad(m[:, 1:], (0, 1))
    v_next = torch.nn.functional.pad(v[:, 1:], (0, 1))
    nv = _affine((m_next * v_next).contiguous(), (1.0 - m_next).contiguous(), None, 0)
    # A[t] = m[t] (r + gamma NV - V) + (m[t] gamma lambda + 1 - m[t]) A[t+1], A[T] = 0
    u = m * (r + gamma * nv - v)
    b = m * (gamma * lambda_) + (1.0 - m)
    adv = _affine(u.contiguous(), b.contiguous(), None, 0)
    return adv, adv + v
