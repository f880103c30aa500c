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
