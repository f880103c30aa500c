"""Parity at the full sizes and input distributions of the benchmark
configurations, on the library's own kernel choice (no RLS_PATH override).

Inputs come from bench.make_inputs (seeded torch.Generator on the device, the
distributions the benchmark times), so these are the shapes, dtypes and
done-rates the bench numbers rest on:

  cfg2  4096 x 128 fp32, terminateds Bernoulli(0.01), all seven estimators
  cfg3  4096 x 128 fp32, terminateds and truncateds Bernoulli(0.005) each,
        disjoint, bootstrap values at truncations and at column T-1
  cfg4  131072 x 1024 bf16 inputs, Bernoulli(0.002): GAE and V-trace
  cfg5a 64 x 131072 fp32: V-trace
  cfg5b 1 x 2^28 fp32, Bernoulli(1e-4): episodic prefix sum and GAE

Every output is compared with the whole fp32 C oracle run on the same values
(bf16 inputs: on the bf16-rounded values) at rtol = atol = 1e-5 through
oracle.compare, which accepts a larger error only where the fp32 oracle
itself deviates from the fp64 oracle by more than 1e-5 (long running sums);
the errors are printed either way.
"""
import numpy as np
import pytest
import torch

import bench
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-5


def _inputs(name, **over):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    cfg = dict(bench.CONFIGS[name], **over)
    x = bench.make_inputs(cfg, torch.device("cuda"), seed=4242)
    return cfg, x, {k: (v.float() if v.dtype == torch.bfloat16 else v).cpu().numpy() for k, v in x.items()}


def _check(got, oracle, what):
    res = orc.compare(got.cpu().numpy() if torch.is_tensor(got) else got, oracle, RTOL, ATOL)
    print(f"{what}: {res}")
    assert res["ok"], f"{what}: {res}"


def _no_device_error():
    from rl_triton import _native as nat
    torch.cuda.synchronize()
    assert nat.workspace_error() == 0


@pytest.fixture(autouse=True)
def _auto_path(monkeypatch):
    monkeypatch.delenv("RLS_PATH", raising=False)
    yield
    _no_device_error()


@pytest.mark.parametrize("name", ["cfg2", "cfg3"])
def test_config_4096x128(name):
    import rl_triton
    cfg, x, h = _inputs(name)
    tr = cfg["trunc"]
    assert not np.any((h["term"] == 1) & (h.get("trunc", np.zeros(1)) == 1)), "inputs must be disjoint"
    calls = bench.make_calls(cfg, x)
    trunc, boot = (h["trunc"], h["boot"]) if tr else (None, None)
    for f, call in calls.items():
        out = call()
        if f == "gae":
            _check(out, lambda p: orc.gae(h["r"], h["v"], h["term"], trunc, boot,
                                          orc.BOOT_FULL_SEL if tr else orc.BOOT_NONE, 0.99, 0.95, p), f"{name} gae")
        elif f == "vtrace":
            for k, o in enumerate(out):
                _check(o, lambda p: orc.vtrace(h["lpt"], h["lpb"], h["v"], h["r"], h["term"], trunc, boot,
                                               orc.BOOT_FULL_ADD if tr else orc.BOOT_NONE, 0.99, 1.0, 1.0, p)[k],
                       f"{name} vtrace[{k}]")
        elif f == "retrace":
            tr32 = h["trunc"] if tr else np.zeros_like(h["r"])
            for k, o in enumerate(out):
                _check(o, lambda p: orc.retrace(h["pi"], h["mu"], h["q"], h["nq"], h["act"], h["r"], h["term"],
                                                tr32, 0.99, 0.95, 1.0, 1.0, p)[k], f"{name} retrace[{k}]")
        elif f == "lambda":
            _check(out, lambda p: orc.lambda_returns(h["r"], h["nv"], h["term"], trunc, boot,
                                                     orc.BOOT_FULL_ADD if tr else orc.BOOT_NONE, 0.99, 0.95, p),
                   f"{name} lambda")
        elif f == "discounted":
            _check(out, lambda p: orc.discounted_returns(h["r"], h["term"], trunc, boot,
                                                         orc.BOOT_FULL_ADD if tr else orc.BOOT_NONE, 0.99, p),
                   f"{name} discounted")
        elif f == "eligibility":
            _check(out, lambda p: orc.eligibility_traces(h["r"], h["term"], 0.99, 0.95, precision=p),
                   f"{name} eligibility")
        elif f == "prefix":
            _check(out, lambda p: orc.prefix_sum(h["r"], h["term"], precision=p), f"{name} prefix")


def test_config4_bf16_full_size():
    """131072 x 1024 bf16 (each input 256 MiB) on the lean row kernel."""
    import rl_triton
    cfg, x, h = _inputs("cfg4")
    assert x["r"].dtype == torch.bfloat16 and x["r"].shape == (131072, 1024)
    got = rl_triton.compute_gae(x["r"], x["v"], x["term"], gamma=0.99, lambda_=0.95)
    _check(got, lambda p: orc.gae(h["r"], h["v"], h["term"], gamma=0.99, lam=0.95, precision=p), "cfg4 gae")
    del got
    vs, adv = rl_triton.compute_vtrace(x["lpt"], x["lpb"], x["v"], x["r"], x["term"], gamma=0.99)
    for k, o in enumerate((vs, adv)):
        _check(o, lambda p: orc.vtrace(h["lpt"], h["lpb"], h["v"], h["r"], h["term"], gamma=0.99, precision=p)[k],
               f"cfg4 vtrace[{k}]")


def test_config5a_vtrace_long_rows():
    import rl_triton
    cfg, x, h = _inputs("cfg5a")
    vs, adv = rl_triton.compute_vtrace(x["lpt"], x["lpb"], x["v"], x["r"], x["term"], gamma=0.99)
    for k, o in enumerate((vs, adv)):
        _check(o, lambda p: orc.vtrace(h["lpt"], h["lpb"], h["v"], h["r"], h["term"], gamma=0.99, precision=p)[k],
               f"cfg5a vtrace[{k}]")


def test_config5b_single_sequence_2pow28():
    """One sequence of 2^28 steps at a 1e-4 done rate: the virtual-row path
    with segments of tens of thousands of steps."""
    import rl_triton
    cfg, x, h = _inputs("cfg5b")
    got = rl_triton.compute_episodic_prefix_sum(x["r"], x["term"])
    _check(got, lambda p: orc.prefix_sum(h["r"], h["term"], precision=p), "cfg5b prefix")
    del got
    got = rl_triton.compute_gae(x["r"], x["v"], x["term"], gamma=0.99, lambda_=0.95)
    _check(got, lambda p: orc.gae(h["r"], h["v"], h["term"], gamma=0.99, lam=0.95, precision=p), "cfg5b gae")


def test_many_unaligned_rows_default_path():
    """4096 rows of 131 steps (rows not 16-byte aligned: the first row kernel
    with per-element accesses on the default path), all seven estimators."""
    cfg, x, h = _inputs("unaligned")
    calls = bench.make_calls(cfg, x)
    for f, call in calls.items():
        out = call()
        outs = out if isinstance(out, tuple) else (out,)
        for k, o in enumerate(outs):
            _check(o, lambda p: bench.oracle_output(f, h, cfg, p)[k], f"unaligned {f}[{k}]")
