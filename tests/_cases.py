"""Golden cases (tests/golden/) and their replay through the C oracle or the
drop-in API.  Test helper only."""
from __future__ import annotations

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")


def load_cases():
    with open(os.path.join(GOLDEN, "cases.json")) as f:
        meta = json.load(f)
    arrays = np.load(os.path.join(GOLDEN, "golden.npz"))
    out = []
    for c in meta["cases"]:
        tens = {k: arrays[v] for k, v in c["tensors"].items()}
        exp = {k: arrays[v] for k, v in c["expected"].items()}
        out.append((c, tens, exp))
    return out


def oracle_replay(case, t, precision="f32"):
    """Run a case through oracle/oracle.py with the reference's dispatch
    (flat path: every golden case has seq_len <= 131072)."""
    from oracle import oracle as orc

    api, s = case["api"], case["scalars"]
    if api == "compute_gae":
        trunc, bv, lv = t.get("truncateds"), t.get("bootstrap_values"), t.get("last_value")
        if lv is not None:
            kind, boot = orc.BOOT_ROW, lv
        elif bv is not None:
            kind, boot = (orc.BOOT_FULL_SEL if trunc is not None else orc.BOOT_LASTCOL), bv
        else:
            kind, boot = orc.BOOT_NONE, None
        return {"out": orc.gae(t["rewards"], t["values"], t["terminateds"], trunc, boot, kind,
                               s.get("gamma", 0.99), s.get("lambda_", 0.95), precision)}
    if api == "compute_vtrace":
        trunc, bv, lv = t.get("truncateds"), t.get("bootstrap_values"), t.get("last_value")
        if lv is not None:
            kind, boot = orc.BOOT_ROW, lv
        elif bv is not None:
            kind, boot = (orc.BOOT_FULL_ADD if trunc is not None else orc.BOOT_LASTCOL), bv
        else:
            kind, boot = orc.BOOT_NONE, None
        vs, adv = orc.vtrace(t["log_pi_target"], t["log_pi_behavior"], t["values"], t["rewards"], t["terminateds"],
                             trunc, boot, kind, s.get("gamma", 0.99), s.get("rho_bar", 1.0), s.get("c_bar", 1.0),
                             precision)
        return {"targets": vs, "advantages": adv}
    if api == "compute_retrace":
        qr, adv = orc.retrace(t["action_probs_target"], t["action_probs_behavior"], t["q_values"],
                              t["next_q_values_all"], t["actions"], t["rewards"], t["terminateds"], t["truncateds"],
                              s["gamma"], s.get("lambda_", 1.0), s.get("c_bar", 1.0), s.get("rho_bar", 1.0),
                              precision)
        return {"targets": qr, "advantages": adv}
    if api == "compute_lambda_returns":
        trunc, bv = t.get("truncateds"), t.get("bootstrap_values")
        kind = orc.BOOT_NONE if bv is None else (orc.BOOT_FULL_ADD if trunc is not None else orc.BOOT_LASTCOL)
        return {"out": orc.lambda_returns(t["rewards"], t["next_values"], t["terminateds"], trunc, bv, kind,
                                          s.get("gamma", 0.99), s.get("lambda_", 0.95), precision)}
    if api == "compute_discounted_returns":
        trunc, bv = t.get("truncateds"), t.get("bootstrap_values")
        kind = orc.BOOT_NONE if bv is None else (orc.BOOT_FULL_ADD if trunc is not None else orc.BOOT_LASTCOL)
        return {"out": orc.discounted_returns(t["rewards"], t["terminateds"], trunc, bv, kind,
                                              s.get("gamma", 0.99), precision)}
    if api == "compute_eligibility_traces":
        return {"out": orc.eligibility_traces(t["gradients"], t["dones"], s["gamma"], s["lambda_"],
                                              t.get("seed_values"), precision)}
    if api == "compute_episodic_prefix_sum":
        return {"out": orc.prefix_sum(t["inputs"], t["dones"], t.get("seed_values"),
                                      s.get("boundary", "ends_at") == "ends_at", precision)}
    if api == "_run_scan":
        return {"out": orc.affine_scan(t["u"], t["v"], t.get("bootstrap"), 0, precision)}
    raise KeyError(api)


def api_replay(case, t, device="cuda"):
    """Run a case through the public rl_triton API on `device`."""
    import torch

    import rl_triton
    from rl_triton.ops._scan import _run_scan

    fn = _run_scan if case["api"] == "_run_scan" else getattr(rl_triton, case["api"])
    kw = {k: torch.from_numpy(np.ascontiguousarray(v)).to(device) for k, v in t.items()}
    kw.update(case["scalars"])
    res = fn(**kw)
    if isinstance(res, tuple):
        res = {"targets": res[0], "advantages": res[1]}
    else:
        res = {"out": res}
    return {k: v.detach().cpu().numpy() for k, v in res.items()}
