"""Generate the golden parity fixtures (tests/golden/golden.npz + cases.json).

Run in a container that has the reference source (simonsays1980/rl-triton
v0.1.3) checked out read-only; the committed fixtures are what the tests use,
so the reference is not needed at test time or on the GPU box:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference /path/to/rl-triton

Two kinds of cases:
  * "kat": the hand-derived known-answer vectors written in the reference's
    tests (cited file:line), transcribed as numbers;
  * "ref": seeded random inputs whose expected outputs are computed HERE by
    calling the reference's own sequential PyTorch oracles (reference_gae,
    _ref_gae_sequential, reference_vtrace, ...) on CPU tensors.

Each case records the public rl_triton call (api + tensor kwargs + scalar
kwargs) so the GPU tests can replay it through the drop-in API, and the CPU
tests can replay it through the C oracle.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


class Builder:
    def __init__(self):
        self.arrays: dict[str, np.ndarray] = {}
        self.cases: list[dict] = []

    def add(self, name, api, tensors, scalars, expected, source, kind, atol=1e-5, rtol=1e-5):
        rec = {"name": name, "api": api, "kind": kind, "source": source, "atol": atol, "rtol": rtol,
               "tensors": {}, "scalars": scalars, "expected": {}}
        for k, t in tensors.items():
            if t is None:
                continue
            key = f"{name}/in/{k}"
            self.arrays[key] = t.detach().cpu().numpy()
            rec["tensors"][k] = key
        for k, t in expected.items():
            key = f"{name}/out/{k}"
            self.arrays[key] = t.detach().cpu().to(torch.float32).numpy()
            rec["expected"][k] = key
        self.cases.append(rec)


def T(x):
    return torch.tensor(x, dtype=torch.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("RL_TRITON_REFERENCE"),
                    help="checkout of simonsays1980/rl-triton v0.1.3 (or set RL_TRITON_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or RL_TRITON_REFERENCE) is required")
    sys.dont_write_bytecode = True
    sys.path.insert(0, os.path.join(args.reference, "tests"))
    sys.path.insert(0, os.path.join(args.reference, "src"))
    import test_gae as tg  # noqa: E402  (the reference's own test modules)
    import test_prefix_sum as tp  # noqa: E402
    import test_retrace as tr  # noqa: E402
    import test_returns as tre  # noqa: E402
    import test_scan_chunked as tsc  # noqa: E402
    import test_vtrace as tv  # noqa: E402

    b = Builder()
    g = torch.Generator().manual_seed(2024)

    def randn(*s):
        return torch.randn(*s, generator=g)

    def rand(*s):
        return torch.rand(*s, generator=g)

    def flags(n, t, p):
        return (rand(n, t) < p).float()

    # ------------------------------------------------------------------ GAE
    z3 = torch.zeros(1, 3)
    b.add("gae_kat_single_env", "compute_gae", dict(rewards=T([[1, 2, 3]]), values=z3, terminateds=z3),
          dict(gamma=1.0, lambda_=1.0), dict(out=T([[6, 5, 3]])), "tests/test_gae.py:126-139", "kat")
    b.add("gae_kat_delta", "compute_gae", dict(rewards=T([[1, 2, 3]]), values=torch.ones(1, 3), terminateds=z3),
          dict(gamma=1.0, lambda_=1.0), dict(out=T([[5, 4, 2]])), "tests/test_gae.py:142-158", "kat")
    b.add("gae_kat_gamma", "compute_gae", dict(rewards=T([[1, 2]]), values=torch.zeros(1, 2),
          terminateds=torch.zeros(1, 2)), dict(gamma=0.9, lambda_=1.0), dict(out=T([[2.8, 2.0]])),
          "tests/test_gae.py:161-174", "kat")
    b.add("gae_kat_lambda0", "compute_gae", dict(rewards=T([[1, 2, 3]]), values=z3, terminateds=z3),
          dict(gamma=1.0, lambda_=0.0), dict(out=T([[1, 2, 3]])), "tests/test_gae.py:177-186", "kat")
    b.add("gae_kat_truncated_last_value", "compute_gae",
          dict(rewards=T([[1, 2, 3]]), values=z3, terminateds=z3, last_value=T([2.0])),
          dict(gamma=1.0, lambda_=1.0), dict(out=T([[8, 7, 5]])), "tests/test_gae.py:189-208", "kat")
    b.add("gae_kat_episode_boundary", "compute_gae",
          dict(rewards=T([[1, 2, 3]]), values=z3, terminateds=T([[0, 1, 0]])),
          dict(gamma=1.0, lambda_=1.0), dict(out=T([[3, 2, 3]])), "tests/test_gae.py:235-249", "kat")
    b.add("gae_kat_batch", "compute_gae", dict(rewards=T([[1, 2], [3, 4]]), values=torch.zeros(2, 2),
          terminateds=torch.zeros(2, 2)), dict(gamma=1.0, lambda_=1.0), dict(out=T([[3, 2], [7, 4]])),
          "tests/test_gae.py:252-264", "kat")

    for (n, t) in [(1, 1), (1, 7), (8, 37), (4, 128), (3, 333)]:
        r, v, term = randn(n, t), randn(n, t), flags(n, t, 0.05)
        exp = tg.reference_gae(r, v, term, gamma=0.99, lambda_=0.95)
        b.add(f"gae_ref_{n}x{t}", "compute_gae", dict(rewards=r, values=v, terminateds=term),
              dict(gamma=0.99, lambda_=0.95), dict(out=exp), "tests/test_gae.py:34-60 reference_gae", "ref",
              atol=1e-4, rtol=1e-4)
    r, v, term = randn(6, 50), randn(6, 50), flags(6, 50, 0.05)
    lv = rand(6)
    exp = tg.reference_gae(r, v, term, gamma=0.99, lambda_=0.95, bootstrap_values=lv)
    b.add("gae_ref_last_value", "compute_gae", dict(rewards=r, values=v, terminateds=term, last_value=lv),
          dict(gamma=0.99, lambda_=0.95), dict(out=exp), "tests/test_gae.py:34-60 reference_gae", "ref",
          atol=1e-4, rtol=1e-4)
    bv = torch.zeros(6, 50)
    bv[:, -1] = lv
    b.add("gae_ref_bootstrap_lastcol", "compute_gae",
          dict(rewards=r, values=v, terminateds=term, bootstrap_values=bv), dict(gamma=0.99, lambda_=0.95),
          dict(out=exp), "tests/test_gae.py:540-556 (last_value == bootstrap_values[:, -1])", "ref",
          atol=1e-4, rtol=1e-4)
    for name, with_boot in [("gae_ref_trunc_boot", True), ("gae_ref_trunc_noboot", False)]:
        n, t = 5, 40
        r, v, term = randn(n, t), randn(n, t), flags(n, t, 0.05)
        trunc = flags(n, t, 0.05) * (1 - term)
        bv = torch.zeros(n, t)
        if with_boot:
            bv[trunc.bool()] = randn(int(trunc.sum().item()))
            bv[:, -1] = randn(n)
        exp = tg._ref_gae_sequential(r, v, term, trunc, bv, gamma=0.99, lambda_=0.95)
        tens = dict(rewards=r, values=v, terminateds=term, truncateds=trunc)
        if with_boot:
            tens["bootstrap_values"] = bv
        b.add(name, "compute_gae", tens, dict(gamma=0.99, lambda_=0.95), dict(out=exp),
              "tests/test_gae.py:418-450 _ref_gae_sequential", "ref")

    # -------------------------------------------------------------- V-trace
    lp0 = torch.zeros(1, 2)
    b.add("vtrace_kat_single_env", "compute_vtrace",
          dict(log_pi_target=lp0, log_pi_behavior=lp0, values=lp0, rewards=torch.ones(1, 2), terminateds=lp0),
          dict(gamma=1.0, rho_bar=100.0, c_bar=100.0), dict(targets=T([[2, 1]]), advantages=T([[2, 1]])),
          "tests/test_vtrace.py:179-199", "kat")
    b.add("vtrace_kat_truncated_last_value", "compute_vtrace",
          dict(log_pi_target=lp0, log_pi_behavior=lp0, values=lp0, rewards=torch.ones(1, 2), terminateds=lp0,
               last_value=T([0.5])),
          dict(gamma=1.0, rho_bar=100.0, c_bar=100.0), dict(targets=T([[2.5, 1.5]]), advantages=T([[2.5, 1.5]])),
          "tests/test_vtrace.py:202-226", "kat")
    b.add("vtrace_kat_done", "compute_vtrace",
          dict(log_pi_target=lp0, log_pi_behavior=lp0, values=lp0, rewards=torch.ones(1, 2),
               terminateds=T([[1, 0]])),
          dict(gamma=1.0, rho_bar=100.0, c_bar=100.0), dict(targets=T([[1, 1]])),
          "tests/test_vtrace.py:229-251", "kat")
    b.add("vtrace_kat_clipping", "compute_vtrace",
          dict(log_pi_target=lp0, log_pi_behavior=torch.full((1, 2), float(np.log(np.float32(2.0)))),
               values=lp0, rewards=torch.ones(1, 2), terminateds=lp0),
          dict(gamma=1.0, rho_bar=1.0, c_bar=1.0), dict(targets=T([[0.75, 0.5]])),
          "tests/test_vtrace.py:254-272", "kat")

    def vt_inputs(n, t):
        return (-rand(n, t), -rand(n, t), randn(n, t), randn(n, t), flags(n, t, 0.05))

    for (n, t, rho, c) in [(1, 1, 1.0, 1.0), (1, 7, 1.0, 1.0), (8, 37, 1.0, 1.0), (4, 129, 1.5, 0.8)]:
        lpt, lpb, v, r, term = vt_inputs(n, t)
        vs, adv = tv.reference_vtrace(lpt, lpb, v, r, term, gamma=0.99, rho_bar=rho, c_bar=c)
        b.add(f"vtrace_ref_{n}x{t}", "compute_vtrace",
              dict(log_pi_target=lpt, log_pi_behavior=lpb, values=v, rewards=r, terminateds=term),
              dict(gamma=0.99, rho_bar=rho, c_bar=c), dict(targets=vs, advantages=adv),
              "tests/test_vtrace.py:56-101 reference_vtrace", "ref", atol=1e-4, rtol=1e-4)
    lpt, lpb, v, r, term = vt_inputs(6, 20)
    lv = randn(6)
    vs, adv = tv.reference_vtrace(lpt, lpb, v, r, term, gamma=0.99, bootstrap_values=lv)
    b.add("vtrace_ref_last_value", "compute_vtrace",
          dict(log_pi_target=lpt, log_pi_behavior=lpb, values=v, rewards=r, terminateds=term, last_value=lv),
          dict(gamma=0.99), dict(targets=vs, advantages=adv), "tests/test_vtrace.py:56-101 reference_vtrace",
          "ref", atol=1e-4, rtol=1e-4)
    for name, with_boot in [("vtrace_ref_trunc_boot", True), ("vtrace_ref_trunc_noboot", False)]:
        n, t = 5, 40
        lpt, lpb, v, r, term = vt_inputs(n, t)
        trunc = flags(n, t, 0.05) * (1 - term)
        bv = torch.zeros(n, t)
        if with_boot:
            bv[trunc.bool()] = randn(int(trunc.sum().item()))
            bv[:, -1] = randn(n)
        vs, adv = tv._ref_vtrace_sequential(lpt, lpb, v, r, term, trunc, bv, gamma=0.99)
        tens = dict(log_pi_target=lpt, log_pi_behavior=lpb, values=v, rewards=r, terminateds=term,
                    truncateds=trunc)
        if with_boot:
            tens["bootstrap_values"] = bv
        b.add(name, "compute_vtrace", tens, dict(gamma=0.99), dict(targets=vs, advantages=adv),
              "tests/test_vtrace.py:424-480 _ref_vtrace_sequential", "ref")

    # -------------------------------------------------------------- Retrace
    one12 = torch.ones(1, 2, 1)
    a0 = torch.zeros(1, 2, dtype=torch.int64)

    def rt_kat(name, pt, pb, q, qn, act, r, term, trunc, exp_t=None, exp_a=None, src=""):
        exp = {}
        if exp_t is not None:
            exp["targets"] = T(exp_t)
        if exp_a is not None:
            exp["advantages"] = T(exp_a)
        b.add(name, "compute_retrace",
              dict(action_probs_target=pt, action_probs_behavior=pb, q_values=q, next_q_values_all=qn,
                   actions=act, rewards=r, terminateds=term, truncateds=trunc),
              dict(gamma=1.0), exp, src, "kat")

    z2 = torch.zeros(1, 2)
    rt_kat("retrace_kat_single_env", one12, torch.ones(1, 2), z2, T([[[2.0], [3.0]]]), a0, torch.ones(1, 2), z2,
           z2, exp_t=[[7, 4]], src="tests/test_retrace.py:147-160")
    rt_kat("retrace_kat_done", one12, torch.ones(1, 2), z2, T([[[2.0], [3.0]]]), a0, torch.ones(1, 2),
           T([[1, 0]]), z2, exp_t=[[1, 4]], src="tests/test_retrace.py:163-178")
    rt_kat("retrace_kat_clipping", one12, torch.full((1, 2), 0.5), z2, torch.full((1, 2, 1), 0.5), a0,
           torch.ones(1, 2), z2, z2, exp_t=[[3, 1.5]], src="tests/test_retrace.py:181-197")
    rt_kat("retrace_kat_terminal_no_bootstrap", torch.ones(1, 1, 1), torch.ones(1, 1), torch.zeros(1, 1),
           torch.full((1, 1, 1), 5.0), torch.zeros(1, 1, dtype=torch.int64), torch.ones(1, 1), torch.ones(1, 1),
           torch.zeros(1, 1), exp_t=[[1]], src="tests/test_retrace.py:205-218")
    rt_kat("retrace_kat_truncated_keeps_bootstrap", torch.ones(1, 1, 1), torch.ones(1, 1), torch.zeros(1, 1),
           torch.full((1, 1, 1), 5.0), torch.zeros(1, 1, dtype=torch.int64), torch.ones(1, 1),
           torch.zeros(1, 1), torch.ones(1, 1), exp_t=[[6]], src="tests/test_retrace.py:221-234")
    rt_kat("retrace_kat_truncated_c_boundary", one12, torch.ones(1, 2), z2, torch.full((1, 2, 1), 5.0), a0,
           torch.ones(1, 2), z2, T([[0, 1]]), exp_t=[[12, 6]], src="tests/test_retrace.py:237-252")
    rt_kat("retrace_kat_advantages_single_env", one12, torch.ones(1, 2), z2, T([[[2.0], [3.0]]]), a0,
           torch.ones(1, 2), z2, z2, exp_a=[[5, 1]], src="tests/test_retrace.py:259-273")
    rt_kat("retrace_kat_advantages_terminal", one12, torch.ones(1, 2), z2, T([[[2.0], [3.0]]]), a0,
           torch.ones(1, 2), T([[1, 0]]), z2, exp_a=[[1, 1]], src="tests/test_retrace.py:276-290")

    for (n, t, A, lam, cb, rb, ptrunc) in [(1, 1, 4, 1.0, 1.0, 1.0, 0.0), (8, 37, 4, 0.95, 1.0, 1.0, 0.0),
                                           (4, 20, 3, 1.0, 1.0, 1.0, 0.05), (3, 17, 6, 0.9, 0.9, 1.2, 0.05),
                                           (2, 130, 4, 0.95, 1.0, 1.0, 0.02)]:
        pt = torch.softmax(randn(n, t, A), dim=-1)
        pb = rand(n, t) * 0.8 + 0.1
        q, qn = randn(n, t), randn(n, t, A)
        act = torch.randint(0, A, (n, t), generator=g)
        r, term = randn(n, t), flags(n, t, 0.05)
        trunc = flags(n, t, ptrunc) * (1 - term)
        qr, adv = tr.reference_retrace(pt, pb, q, qn, act, r, term, trunc, gamma=0.99, lambda_=lam, c_bar=cb,
                                       rho_bar=rb)
        b.add(f"retrace_ref_{n}x{t}x{A}", "compute_retrace",
              dict(action_probs_target=pt, action_probs_behavior=pb, q_values=q, next_q_values_all=qn,
                   actions=act, rewards=r, terminateds=term, truncateds=trunc),
              dict(gamma=0.99, lambda_=lam, c_bar=cb, rho_bar=rb), dict(targets=qr, advantages=adv),
              "tests/test_retrace.py:19-60 reference_retrace", "ref", atol=1e-4, rtol=1e-4)

    # ----------------------------------------------------------- lambda / disc
    def lam_kat(name, r, nv, d, lam, exp, src, boot=None):
        tens = dict(rewards=T(r), next_values=T(nv), terminateds=T(d))
        if boot is not None:
            tens["bootstrap_values"] = T(boot)
        b.add(name, "compute_lambda_returns", tens, dict(gamma=1.0, lambda_=lam), dict(out=T(exp)), src, "kat")

    lam_kat("lambda_kat_lambda0", [[1, 2]], [[3, 4]], [[0, 0]], 0.0, [[4, 6]], "tests/test_returns.py:183-191")
    lam_kat("lambda_kat_lambda1", [[1, 2]], [[99, 99]], [[0, 0]], 1.0, [[3, 2]], "tests/test_returns.py:194-202")
    lam_kat("lambda_kat_intermediate", [[1, 2]], [[3, 4]], [[0, 0]], 0.5, [[4.5, 4]],
            "tests/test_returns.py:205-216")
    lam_kat("lambda_kat_done", [[1, 2]], [[3, 4]], [[1, 0]], 0.5, [[1, 4]], "tests/test_returns.py:219-229")
    lam_kat("lambda_kat_bootstrap", [[1, 2]], [[99, 99]], [[0, 0]], 1.0, [[8, 7]],
            "tests/test_returns.py:232-243", boot=[[0, 5]])
    for (n, t, lam) in [(1, 1, 0.0), (1, 7, 1.0), (8, 37, 0.95), (4, 129, 0.5)]:
        r, nv, d = randn(n, t), randn(n, t), flags(n, t, 0.05)
        exp = tre.reference_lambda_returns(r, nv, d, gamma=0.99, lambda_=lam)
        b.add(f"lambda_ref_{n}x{t}", "compute_lambda_returns", dict(rewards=r, next_values=nv, terminateds=d),
              dict(gamma=0.99, lambda_=lam), dict(out=exp), "tests/test_returns.py:19-39 reference_lambda_returns",
              "ref", atol=1e-4, rtol=1e-4)
    r, nv, d = randn(6, 30), randn(6, 30), flags(6, 30, 0.05)
    bv = randn(6, 30)
    exp = tre.reference_lambda_returns(r, nv, d, gamma=0.99, lambda_=0.95, bootstrap_values=bv)
    b.add("lambda_ref_bootstrap", "compute_lambda_returns",
          dict(rewards=r, next_values=nv, terminateds=d, bootstrap_values=bv), dict(gamma=0.99, lambda_=0.95),
          dict(out=exp), "tests/test_returns.py:19-39 reference_lambda_returns", "ref", atol=1e-4, rtol=1e-4)
    n, t = 5, 40
    r, nv, term = randn(n, t), randn(n, t), flags(n, t, 0.05)
    trunc = flags(n, t, 0.05) * (1 - term)
    nv = nv * (1 - trunc)
    bv = torch.zeros(n, t)
    bv[trunc.bool()] = randn(int(trunc.sum().item()))
    bv[:, -1] = randn(n)
    exp = tre._ref_lambda_sequential(r, nv, term, trunc, bv, gamma=0.99, lambda_=0.95)
    b.add("lambda_ref_trunc_boot", "compute_lambda_returns",
          dict(rewards=r, next_values=nv, terminateds=term, truncateds=trunc, bootstrap_values=bv),
          dict(gamma=0.99, lambda_=0.95), dict(out=exp), "tests/test_returns.py:449-483 _ref_lambda_sequential",
          "ref")

    b.add("discounted_kat", "compute_discounted_returns", dict(rewards=T([[1, 2]]), terminateds=T([[0, 0]])),
          dict(gamma=0.9), dict(out=T([[2.8, 2.0]])), "tests/test_returns.py:419-425", "kat")
    b.add("discounted_kat_done", "compute_discounted_returns", dict(rewards=T([[1, 2]]), terminateds=T([[1, 0]])),
          dict(gamma=0.9), dict(out=T([[1.0, 2.0]])), "tests/test_returns.py:428-435", "kat")
    for (n, t) in [(1, 1), (1, 7), (8, 37), (4, 129)]:
        r, d = randn(n, t), flags(n, t, 0.05)
        exp = tre.reference_discounted_returns(r, d, gamma=0.99)
        b.add(f"discounted_ref_{n}x{t}", "compute_discounted_returns", dict(rewards=r, terminateds=d),
              dict(gamma=0.99), dict(out=exp), "tests/test_returns.py:42-57 reference_discounted_returns", "ref",
              atol=1e-4, rtol=1e-4)
    r, d, bv = randn(6, 30), flags(6, 30, 0.05), randn(6, 30)
    exp = tre.reference_discounted_returns(r, d, gamma=0.99, bootstrap_values=bv)
    b.add("discounted_ref_bootstrap", "compute_discounted_returns", dict(rewards=r, terminateds=d, bootstrap_values=bv),
          dict(gamma=0.99), dict(out=exp), "tests/test_returns.py:42-57 reference_discounted_returns", "ref",
          atol=1e-4, rtol=1e-4)
    r, term = randn(n, t), flags(n, t, 0.05)
    trunc = flags(n, t, 0.05) * (1 - term)
    bv = torch.zeros(n, t)
    bv[trunc.bool()] = randn(int(trunc.sum().item()))
    bv[:, -1] = randn(n)
    exp = tre._ref_discounted_sequential(r, term, trunc, bv, gamma=0.99)
    b.add("discounted_ref_trunc_boot", "compute_discounted_returns",
          dict(rewards=r, terminateds=term, truncateds=trunc, bootstrap_values=bv), dict(gamma=0.99),
          dict(out=exp), "tests/test_returns.py:486-511 _ref_discounted_sequential", "ref")

    # ------------------------------------------------- eligibility / prefix
    def el_kat(name, gr, d, lam, exp, src, seed=None):
        tens = dict(gradients=T(gr), dones=T(d))
        if seed is not None:
            tens["seed_values"] = T(seed)
        b.add(name, "compute_eligibility_traces", tens, dict(gamma=1.0, lambda_=lam), dict(out=T(exp)), src, "kat")

    el_kat("elig_kat_basic", [[1, 2, 3]], [[0, 0, 0]], 1.0, [[1, 3, 6]], "tests/test_returns.py:297-303")
    el_kat("elig_kat_decay", [[1, 2]], [[0, 0]], 0.5, [[1, 2.5]], "tests/test_returns.py:306-312")
    el_kat("elig_kat_done", [[1, 2, 3]], [[0, 1, 0]], 0.9, [[1, 2.9, 3]], "tests/test_returns.py:315-330")
    el_kat("elig_kat_seed", [[1, 2]], [[0, 0]], 1.0, [[3, 5]], "tests/test_returns.py:333-341", seed=[2.0])
    for (n, t, lam, with_seed) in [(1, 1, 0.0, False), (1, 7, 1.0, True), (8, 37, 0.9, False),
                                   (4, 129, 0.9, True)]:
        gr, d = randn(n, t), flags(n, t, 0.05)
        sd = randn(n) if with_seed else None
        exp = tre.reference_eligibility_traces(gr, d, gamma=0.99, lambda_=lam, seed_values=sd)
        tens = dict(gradients=gr, dones=d)
        if sd is not None:
            tens["seed_values"] = sd
        b.add(f"elig_ref_{n}x{t}", "compute_eligibility_traces", tens, dict(gamma=0.99, lambda_=lam),
              dict(out=exp), "tests/test_returns.py:362-385 reference_eligibility_traces", "ref",
              atol=1e-4, rtol=1e-4)

    def ps_kat(name, x, d, boundary, exp, src, seed=None):
        tens = dict(inputs=T(x), dones=T(d))
        if seed is not None:
            tens["seed_values"] = T(seed)
        b.add(name, "compute_episodic_prefix_sum", tens, dict(boundary=boundary), dict(out=T(exp)), src, "kat")

    for bd in ("ends_at", "starts_at"):
        ps_kat(f"prefix_kat_no_reset_{bd}", [[1, 2, 3]], [[0, 0, 0]], bd, [[1, 3, 6]],
               "tests/test_prefix_sum.py:64-76")
        ps_kat(f"prefix_kat_seed_{bd}", [[1, 2]], [[0, 0]], bd, [[11, 13]], "tests/test_prefix_sum.py:170-184",
               seed=[10.0])
    ps_kat("prefix_kat_reset_at_start_starts_at", [[5, 2, 3]], [[1, 0, 0]], "starts_at", [[5, 7, 10]],
           "tests/test_prefix_sum.py:79-92")
    ps_kat("prefix_kat_reset_at_start_ends_at", [[5, 2, 3]], [[1, 0, 0]], "ends_at", [[5, 2, 5]],
           "tests/test_prefix_sum.py:95-108")
    ps_kat("prefix_kat_mid_reset_starts_at", [[1, 2, 3, 4]], [[0, 0, 1, 0]], "starts_at", [[1, 3, 3, 7]],
           "tests/test_prefix_sum.py:111-124")
    ps_kat("prefix_kat_mid_reset_ends_at", [[1, 2, 3, 4]], [[0, 0, 1, 0]], "ends_at", [[1, 3, 6, 4]],
           "tests/test_prefix_sum.py:127-140")
    ps_kat("prefix_kat_seed_cancelled_starts_at", [[1, 2]], [[1, 0]], "starts_at", [[1, 3]],
           "tests/test_prefix_sum.py:187-199", seed=[10.0])
    for (n, t, bd, with_seed) in [(1, 1, "ends_at", False), (1, 7, "starts_at", True), (8, 37, "ends_at", True),
                                  (4, 129, "starts_at", False), (3, 300, "ends_at", False)]:
        x, d = randn(n, t), flags(n, t, 0.05)
        sd = randn(n) if with_seed else None
        exp = tp.reference_episodic_prefix_sum(x, d, seed_values=sd, boundary=bd)
        tens = dict(inputs=x, dones=d)
        if sd is not None:
            tens["seed_values"] = sd
        b.add(f"prefix_ref_{n}x{t}_{bd}", "compute_episodic_prefix_sum", tens, dict(boundary=bd), dict(out=exp),
              "tests/test_prefix_sum.py:18-58 reference_episodic_prefix_sum", "ref", atol=1e-4, rtol=1e-4)

    # ------------------------------------------------------- generic scan
    for (n, t, with_boot) in [(1, 1, False), (4, 40, True), (3, 257, False)]:
        u, v = randn(n, t), rand(n, t) * 0.99
        bt = randn(n) if with_boot else None
        exp = tsc._reference_scan(u, v, bt)
        tens = dict(u=u, v=v)
        if bt is not None:
            tens["bootstrap"] = bt
        b.add(f"scan_ref_{n}x{t}", "_run_scan", tens, {}, dict(out=exp),
              "tests/test_scan_chunked.py:15-29 _reference_scan", "ref", atol=1e-4, rtol=1e-4)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **b.arrays)
    with open(os.path.join(HERE, "cases.json"), "w") as f:
        json.dump({"reference": "simonsays1980/rl-triton v0.1.3", "generator": "tests/golden/make_golden.py",
                   "cases": b.cases}, f, indent=1)
    print(f"{len(b.cases)} cases, {len(b.arrays)} arrays")


if __name__ == "__main__":
    main()
