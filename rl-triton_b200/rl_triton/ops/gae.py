"""compute_gae -- drop-in for src/rl_triton/ops/gae.py (reference v0.1.3)."""
from __future__ import annotations

import torch

from rl_triton import _native as nat
from rl_triton.ops._scan import _CORRECTNESS_WARNINGS, _FLAT_MAX_SEQ_LEN, _done, _float_ok, _placed, _seg, _warn_copies


def compute_gae(
    rewards: torch.Tensor,
    values: torch.Tensor,
    terminateds: torch.Tensor,
    truncateds: torch.Tensor | None = None,
    gamma: float = 0.99,
    lambda_: float = 0.95,
    bootstrap_values: torch.Tensor | None = None,
    last_value: torch.Tensor | None = None,
    *,
    _segment=None,
) -> torch.Tensor:
    """
    Compute Generalized Advantage Estimation via a backward affine scan.

    Recurrence (src/rl_triton/ops/gae.py:44-103):

    - A[t] = δ[t] + β[t] * A[t+1],  A[T] = 0
    - δ[t] = r[t] + γ·(1-terminated[t]) * v_next[t] - V(s_t)
    - β[t] = γ·λ·(1-done[t]),   done[t] = terminated[t] | truncated[t]

    v_next[t] is values[t+1] inside an episode; bootstrap_values[t] at a
    truncated step and at the window end t=T-1 (or last_value / 0 there).  The
    additive boundary carry A[T] is always 0.

    Inputs are float32 (as in the reference) or bfloat16 (all [N, T] streams
    bf16); arithmetic and the output are float32.  Any seq_len runs on the
    fused single-pass kernel.  For seq_len > 131072 the reference's chunked
    path forms v_next additively (values[t+1]*(1-truncated) + bootstrap);
    that form is reproduced there, the select form below it.

    Returns:
        advantages: A[t], shape [num_envs, seq_len], float32.
    """
    kind, boot = _gae_args(rewards, values, terminateds, truncateds, bootstrap_values, last_value)
    _placed(rewards, values, terminateds, truncateds, boot, last_value)
    _warn_copies({"rewards": rewards, "values": values, "terminateds": terminateds, "truncateds": truncateds,
                  "bootstrap_values": boot})
    t0, total, halo = _seg(_segment)
    out = nat.ops.gae(rewards, values, terminateds, truncateds, last_value if kind == nat.BOOT_ROW else boot, kind,
                      float(gamma), float(lambda_), t0, total, halo)
    _done(rewards)
    return out


def _gae_args(rewards, values, terminateds, truncateds, bootstrap_values, last_value):
    """The reference's argument checks (src/rl_triton/ops/gae.py:106-145) and
    its bootstrap dispatch (:153-215); returns (boot_kind, bootstrap tensor)."""
    num_envs, seq_len = rewards.shape
    has_truncations = truncateds is not None

    # Cheap structural checks -- always-on (src/rl_triton/ops/gae.py:106-129).
    for name, t in [("rewards", rewards), ("values", values), ("terminateds", terminateds)]:
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
        assert not has_truncations, \
            "last_value cannot be combined with truncateds; use bootstrap_values instead."
    if bootstrap_values is not None:
        assert bootstrap_values.is_cuda,                "bootstrap_values must be on CUDA"
        assert _float_ok(bootstrap_values),             "bootstrap_values: expected float32"
        assert bootstrap_values.shape == rewards.shape, \
            f"bootstrap_values shape {bootstrap_values.shape} != rewards shape {rewards.shape}"

    # Expensive tensor scans -- correctness-warning path only (ops/gae.py:132-145).
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

    # Bootstrap kind reproducing the reference's dispatch (ops/gae.py:153-215).
    flat = seq_len <= _FLAT_MAX_SEQ_LEN
    boot = None
    if last_value is not None:
        kind = nat.BOOT_ROW
    elif bootstrap_values is not None:
        if flat:
            kind = nat.BOOT_FULL_SEL if has_truncations else nat.BOOT_LASTCOL
        else:
            kind = nat.BOOT_FULL_ADD
        boot = bootstrap_values
    else:
        kind = nat.BOOT_NONE
    return kind, boot
