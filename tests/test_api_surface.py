"""The drop-in surface (CPU): the public names, the internal module paths the
reference's tests import, and the signatures (names, order, defaults) of the
reference's functions (src/rl_triton/__init__.py:3-17, src/rl_triton/ops/*.py).
When the unmodified reference is installed under baseline/_ref its signatures
are compared directly; the hard-coded table below holds either way."""
import importlib
import inspect
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

EXPECTED = {
    "compute_gae": "(rewards, values, terminateds, truncateds=None, gamma=0.99, lambda_=0.95, "
                   "bootstrap_values=None, last_value=None)",
    "compute_vtrace": "(log_pi_target, log_pi_behavior, values, rewards, terminateds, truncateds=None, gamma=0.99, "
                      "rho_bar=1.0, c_bar=1.0, bootstrap_values=None, last_value=None)",
    "compute_retrace": "(action_probs_target, action_probs_behavior, q_values, next_q_values_all, actions, rewards, "
                       "terminateds, truncateds, gamma, lambda_=1.0, c_bar=1.0, rho_bar=1.0)",
    "compute_lambda_returns": "(rewards, next_values, terminateds, truncateds=None, gamma=0.99, lambda_=0.95, "
                              "bootstrap_values=None)",
    "compute_discounted_returns": "(rewards, terminateds, truncateds=None, gamma=0.99, bootstrap_values=None)",
    "compute_eligibility_traces": "(gradients, dones, gamma, lambda_, seed_values=None)",
    "compute_episodic_prefix_sum": "(inputs, dones, seed_values=None, boundary='ends_at')",
}


def _public_sig(fn):
    """Signature without keyword-only extensions and annotations."""
    ps = [p.replace(annotation=inspect.Parameter.empty) for p in inspect.signature(fn).parameters.values()
          if p.kind != inspect.Parameter.KEYWORD_ONLY]
    return str(inspect.Signature(ps))


@pytest.mark.parametrize("name", sorted(EXPECTED))
def test_public_signatures(name):
    import rl_triton
    assert _public_sig(getattr(rl_triton, name)) == EXPECTED[name]


def test_internal_module_paths_the_reference_tests_import():
    from rl_triton.ops._scan import _FLAT_MAX_SEQ_LEN, _run_scan, _run_scan_forward  # noqa: F401
    from rl_triton.ops.gae import compute_gae  # noqa: F401
    from rl_triton.ops.prefix_sum import compute_episodic_prefix_sum  # noqa: F401
    from rl_triton.ops.retrace import compute_retrace  # noqa: F401
    from rl_triton.ops.retrace_fused import compute_retrace_fused  # noqa: F401
    from rl_triton.ops.returns import (compute_discounted_returns, compute_eligibility_traces,  # noqa: F401
                                       compute_lambda_returns)
    from rl_triton.ops.vtrace import compute_vtrace  # noqa: F401
    from rl_triton.ops.vtrace_fused import compute_vtrace_fused  # noqa: F401
    assert _FLAT_MAX_SEQ_LEN == 131072
    import rl_triton
    assert rl_triton.__version__ == "0.1.3"


def test_signatures_match_the_installed_reference():
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "rl_triton")):
        pytest.skip("reference not installed under baseline/_ref")
    code = ("import inspect, json, rl_triton as r; print(json.dumps({n: [[p.name, repr(p.default)] for p in "
            f"inspect.signature(getattr(r, n)).parameters.values()] for n in {sorted(EXPECTED)!r}}}))")
    env = dict(os.environ, PYTHONPATH=ref, PYTHONDONTWRITEBYTECODE="1")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, cwd="/", timeout=300)
    if out.returncode != 0:
        pytest.skip(f"reference import failed here: {out.stderr.strip().splitlines()[-1][:200]}")
    import json
    theirs = json.loads(out.stdout.strip().splitlines()[-1])
    import rl_triton
    for name, params in theirs.items():
        ps = inspect.signature(getattr(rl_triton, name)).parameters.values()
        mine = [[p.name, repr(p.default)] for p in ps if p.kind != inspect.Parameter.KEYWORD_ONLY]
        assert mine == params, name
