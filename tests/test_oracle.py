"""Pins the CPU oracle (oracle/rlscan_oracle.c) to the reference.

Every golden case -- the reference tests' hand-derived known answers and the
outputs of the reference's own sequential PyTorch loops on seeded inputs
(tests/golden/make_golden.py) -- must be reproduced by the fp32 oracle to
1e-5 and by the fp64 oracle to the case tolerance.  Runs on CPU only.
"""
import numpy as np
import pytest

from _cases import load_cases, oracle_replay

CASES = load_cases()


@pytest.mark.parametrize("case,tens,exp", CASES, ids=[c[0]["name"] for c in CASES])
def test_oracle_f32_matches_golden(case, tens, exp):
    got = oracle_replay(case, tens, "f32")
    for k, want in exp.items():
        np.testing.assert_allclose(got[k], want, atol=1e-5, rtol=1e-5, err_msg=f"{case['name']}:{k}")


@pytest.mark.parametrize("case,tens,exp", CASES, ids=[c[0]["name"] for c in CASES])
def test_oracle_f64_matches_golden(case, tens, exp):
    got = oracle_replay(case, tens, "f64")
    for k, want in exp.items():
        np.testing.assert_allclose(got[k], want, atol=case["atol"], rtol=case["rtol"],
                                   err_msg=f"{case['name']}:{k}")


def test_golden_covers_every_function():
    apis = {c[0]["api"] for c in CASES}
    assert apis == {"compute_gae", "compute_vtrace", "compute_retrace", "compute_lambda_returns",
                    "compute_discounted_returns", "compute_eligibility_traces",
                    "compute_episodic_prefix_sum", "_run_scan"}
    kinds = {(c[0]["api"], c[0]["kind"]) for c in CASES}
    for api in apis - {"_run_scan"}:
        assert (api, "kat") in kinds and (api, "ref") in kinds, api


def test_obs_skip_oracle_known_answer():
    """Observation-skip GAE worked by hand: gamma 0.9, lambda 0.8, mask [1, 0, 1, 1].
    t=3: 4 - 0.3 = 3.7;  t=2: 3 + 0.9*0.3 - 0.2 + 0.72*3.7 = 5.734;  t=1 (observation):
    carried 5.734;  t=0: 1 + 0.9*0.2 - 0.5 + 0.72*5.734 = 4.80848."""
    import numpy as np
    from oracle import oracle as orc
    r = np.array([[1, 2, 3, 4]], np.float32)
    v = np.array([[0.5, 0.1, 0.2, 0.3]], np.float32)
    m = np.array([[1, 0, 1, 1]], np.float32)
    adv, ret = orc.gae_obs_skip(r, v, m, 0.9, 0.8, precision="f64")
    np.testing.assert_allclose(adv, [[4.80848, 5.734, 5.734, 3.7]], rtol=1e-6)
    np.testing.assert_allclose(ret, adv + v, rtol=1e-6)
    # all-ones mask: plain GAE with no terminations
    g = np.random.default_rng(0)
    r, v = g.standard_normal((3, 50)).astype(np.float32), g.standard_normal((3, 50)).astype(np.float32)
    a, _ = orc.gae_obs_skip(r, v, np.ones_like(r), 0.97, 0.9)
    np.testing.assert_allclose(a, orc.gae(r, v, np.zeros_like(r), gamma=0.97, lam=0.9), rtol=1e-5, atol=1e-5)
