"""rl_triton (B200 build) -- drop-in for the seven return-estimation scans of
simonsays1980/rl-triton v0.1.3, computed by hand-written sm_100a CUDA kernels
(librlscan.so) instead of Triton.  Same function names, signatures, module
paths and error behaviour as the reference's src/rl_triton/__init__.py, plus
fused PPO epilogues (compute_gae_normalized, compute_gae_value_loss) and the
observation-skip masking mode (compute_gae_obs_skip) the reference does not
have."""

__version__ = "0.1.3"

from rl_triton.ops.gae import compute_gae
from rl_triton.ops.retrace import compute_retrace
from rl_triton.ops.prefix_sum import compute_episodic_prefix_sum
from rl_triton.ops.returns import compute_discounted_returns, compute_eligibility_traces, compute_lambda_returns
from rl_triton.ops.vtrace import compute_vtrace
from rl_triton.ops.fused import (  # additions: fused PPO epilogues and masking modes
    compute_gae_normalized,
    compute_gae_obs_skip,
    compute_gae_value_loss,
)

__all__ = [
    "compute_discounted_returns",
    "compute_eligibility_traces",
    "compute_episodic_prefix_sum",
    "compute_gae",
    "compute_gae_normalized",
    "compute_gae_obs_skip",
    "compute_gae_value_loss",
    "compute_lambda_returns",
    "compute_retrace",
    "compute_vtrace",
]
