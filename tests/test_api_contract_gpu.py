"""The reference test suite's categories, restated against the CPU oracle:
its shape sweeps per function, non-contiguous inputs, closed-form identities
(lambda = 0 and lambda = 1 limits, on-policy V-trace, decay-free and all-reset
prefix sums, zero-decay scans) and the 131072-step dispatch threshold.  The
parameter lists follow the reference's tests (file:line in each docstring);
the inputs come from this file's own seeded generators."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-5


def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def close(got, want, rtol=RTOL, atol=ATOL, msg=""):
    got = got.cpu().numpy() if torch.is_tensor(got) else got
    np.testing.assert_allclose(np.asarray(got, np.float64), np.asarray(want, np.float64), rtol=rtol, atol=atol,
                               err_msg=msg)


def gen(n, t, seed, p=0.1):
    g = np.random.default_rng(seed)
    return dict(r=g.standard_normal((n, t)).astype(np.float32), v=g.standard_normal((n, t)).astype(np.float32),
                d=(g.random((n, t)) < p).astype(np.float32),
                lpt=(-g.random((n, t))).astype(np.float32), lpb=(-g.random((n, t))).astype(np.float32),
                lv=g.standard_normal(n).astype(np.float32))


def D(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


SHAPES = [(1, 1), (1, 7), (4, 128), (32, 333), (128, 1024), (256, 2048)]


@pytest.mark.parametrize("n,t", SHAPES)
def test_gae_shapes(n, t):
    """tests/test_gae.py:280-292."""
    _cuda()
    import rl_triton
    x = gen(n, t, 40 + t)
    close(rl_triton.compute_gae(D(x["r"]), D(x["v"]), D(x["d"])), orc.gae(x["r"], x["v"], x["d"]))


@pytest.mark.parametrize("n,t", SHAPES)
def test_vtrace_shapes(n, t):
    """tests/test_vtrace.py:278-290 (log-probs -U(0,1))."""
    _cuda()
    import rl_triton
    x = gen(n, t, 42 + t)
    vs, adv = rl_triton.compute_vtrace(D(x["lpt"]), D(x["lpb"]), D(x["v"]), D(x["r"]), D(x["d"]), gamma=0.99)
    wvs, wadv = orc.vtrace(x["lpt"], x["lpb"], x["v"], x["r"], x["d"], gamma=0.99)
    close(vs, wvs)
    close(adv, wadv)


@pytest.mark.parametrize("n,t,a", [(1, 1, 2), (1, 7, 4), (4, 128, 8), (32, 333, 4), (128, 1024, 6)])
def test_retrace_shapes(n, t, a):
    """tests/test_retrace.py:307-320."""
    _cuda()
    import rl_triton
    g = np.random.default_rng(n + t + a)
    logits = g.standard_normal((n, t, a)).astype(np.float32)
    pi = np.exp(logits) / np.exp(logits).sum(-1, keepdims=True)
    pi = pi.astype(np.float32)
    mu = (0.1 + 0.8 * g.random((n, t))).astype(np.float32)
    q = g.standard_normal((n, t)).astype(np.float32)
    nq = g.standard_normal((n, t, a)).astype(np.float32)
    act = g.integers(0, a, (n, t)).astype(np.int64)
    r = g.standard_normal((n, t)).astype(np.float32)
    term = (g.random((n, t)) < 0.1).astype(np.float32)
    trunc = ((g.random((n, t)) < 0.05) * (1 - term)).astype(np.float32)
    tg, adv = rl_triton.compute_retrace(D(pi), D(mu), D(q), D(nq), D(act), D(r), D(term), D(trunc), gamma=0.99,
                                        lambda_=0.9)
    wt, wa = orc.retrace(pi, mu, q, nq, act, r, term, trunc, 0.99, 0.9)
    close(tg, wt)
    close(adv, wa)


@pytest.mark.parametrize("n,t,lam", [(1, 1, 0.0), (1, 7, 1.0), (4, 128, 0.5), (32, 333, 0.95), (128, 1024, 0.9)])
def test_lambda_returns_and_traces_shapes(n, t, lam):
    """tests/test_returns.py:258-270 and :388-400."""
    _cuda()
    import rl_triton
    x = gen(n, t, 7 + t)
    close(rl_triton.compute_lambda_returns(D(x["r"]), D(x["v"]), D(x["d"]), gamma=0.99, lambda_=lam),
          orc.lambda_returns(x["r"], x["v"], x["d"], gamma=0.99, lam=lam))
    close(rl_triton.compute_eligibility_traces(D(x["r"]), D(x["d"]), 0.99, lam),
          orc.eligibility_traces(x["r"], x["d"], 0.99, lam))


@pytest.mark.parametrize("n,t", [(1, 1), (1, 7), (4, 128), (32, 512), (128, 1024)])
def test_discounted_shapes(n, t):
    """tests/test_returns.py:437-446."""
    _cuda()
    import rl_triton
    x = gen(n, t, 10)
    close(rl_triton.compute_discounted_returns(D(x["r"]), D(x["d"]), gamma=0.99),
          orc.discounted_returns(x["r"], x["d"], gamma=0.99))


@pytest.mark.parametrize("boundary", ["ends_at", "starts_at"])
@pytest.mark.parametrize("n,t", SHAPES)
def test_prefix_shapes(n, t, boundary):
    """tests/test_prefix_sum.py:250-268."""
    _cuda()
    import rl_triton
    x = gen(n, t, 3 + t)
    close(rl_triton.compute_episodic_prefix_sum(D(x["r"]), D(x["d"]), boundary=boundary),
          orc.prefix_sum(x["r"], x["d"], None, boundary == "ends_at"))


@pytest.mark.parametrize("n,t", [(1, 1), (1, 7), (4, 1024), (4, 1025), (8, 2048), (32, 3000)])
def test_scan_shapes(n, t):
    """tests/test_scan_chunked.py:44-58: chunk-edge lengths of the reference's chunked kernel."""
    _cuda()
    from rl_triton.ops._scan import _run_scan
    g = np.random.default_rng(t)
    u = g.standard_normal((n, t)).astype(np.float32)
    v = (0.9 + 0.1 * g.random((n, t))).astype(np.float32)
    b = g.standard_normal(n).astype(np.float32)
    close(_run_scan(D(u), D(v)), orc.affine_scan(u, v, None, 0))
    close(_run_scan(D(u), D(v), D(b)), orc.affine_scan(u, v, b, 0))


# ---------------------------------------------------------------- non-contiguous inputs
def _strided(a):
    """A non-contiguous CUDA view holding `a` (every other element of a wider buffer)."""
    wide = torch.zeros(*a.shape, 2, device="cuda")
    wide[..., 0] = torch.from_numpy(a).cuda()
    view = wide[..., 0]
    assert not view.is_contiguous()
    return view


def test_non_contiguous_inputs_every_function():
    """tests/test_gae.py, test_vtrace.py, test_retrace.py:364-380, test_prefix_sum.py non-contiguous cases."""
    _cuda()
    import rl_triton
    x = gen(16, 256, 7, p=0.05)
    close(rl_triton.compute_gae(_strided(x["r"]), _strided(x["v"]), _strided(x["d"])), orc.gae(x["r"], x["v"], x["d"]))
    vs, adv = rl_triton.compute_vtrace(_strided(x["lpt"]), _strided(x["lpb"]), _strided(x["v"]), _strided(x["r"]),
                                       _strided(x["d"]))
    wvs, wadv = orc.vtrace(x["lpt"], x["lpb"], x["v"], x["r"], x["d"])
    close(vs, wvs)
    close(adv, wadv)
    close(rl_triton.compute_lambda_returns(_strided(x["r"]), _strided(x["v"]), _strided(x["d"])),
          orc.lambda_returns(x["r"], x["v"], x["d"]))
    close(rl_triton.compute_discounted_returns(_strided(x["r"]), _strided(x["d"])),
          orc.discounted_returns(x["r"], x["d"]))
    close(rl_triton.compute_eligibility_traces(_strided(x["r"]), _strided(x["d"]), 0.99, 0.9),
          orc.eligibility_traces(x["r"], x["d"], 0.99, 0.9))
    for bd in ("ends_at", "starts_at"):
        close(rl_triton.compute_episodic_prefix_sum(_strided(x["r"]), _strided(x["d"]), boundary=bd),
              orc.prefix_sum(x["r"], x["d"], None, bd == "ends_at"))
    g = np.random.default_rng(1)
    a = 4
    logits = g.standard_normal((16, 256, a)).astype(np.float32)
    pi = (np.exp(logits) / np.exp(logits).sum(-1, keepdims=True)).astype(np.float32)
    nq = g.standard_normal((16, 256, a)).astype(np.float32)
    act = g.integers(0, a, (16, 256)).astype(np.int64)
    mu = (0.1 + 0.8 * g.random((16, 256))).astype(np.float32)
    z = np.zeros((16, 256), np.float32)
    tg, ad = rl_triton.compute_retrace(_strided(pi), _strided(mu), _strided(x["v"]), _strided(nq), D(act)[:, :],
                                       _strided(x["r"]), _strided(z), _strided(z), gamma=0.99, lambda_=1.0,
                                       c_bar=1e6, rho_bar=1e6)
    wt, wa = orc.retrace(pi, mu, x["v"], nq, act, x["r"], z, z, 0.99, 1.0, 1e6, 1e6)
    close(tg, wt, rtol=1e-4, atol=1e-4)
    close(ad, wa, rtol=1e-4, atol=1e-4)


# ---------------------------------------------------------------- identities
def test_gae_lambda0_is_td_error():
    """tests/test_gae.py: lambda = 0 gives the one-step TD error."""
    _cuda()
    import rl_triton
    x = gen(8, 50, 2)
    lv = x["lv"]
    vnext = np.concatenate([x["v"][:, 1:], lv[:, None]], axis=1)
    want = x["r"] + 0.97 * vnext * (1 - x["d"]) - x["v"]
    got = rl_triton.compute_gae(D(x["r"]), D(x["v"]), D(x["d"]), gamma=0.97, lambda_=0.0, last_value=D(lv))
    close(got, want, rtol=1e-5, atol=1e-5)


def test_lambda1_lambda_returns_equal_discounted_returns():
    """tests/test_returns.py: lambda-returns with lambda = 1 are discounted returns."""
    _cuda()
    import rl_triton
    x = gen(8, 300, 3, p=0.02)
    a = rl_triton.compute_lambda_returns(D(x["r"]), D(x["v"]), D(x["d"]), gamma=0.98, lambda_=1.0)
    b = rl_triton.compute_discounted_returns(D(x["r"]), D(x["d"]), gamma=0.98)
    torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)


def test_eligibility_lambda0_is_the_gradient():
    _cuda()
    import rl_triton
    x = gen(4, 64, 4)
    close(rl_triton.compute_eligibility_traces(D(x["r"]), D(x["d"]), 0.99, 0.0), x["r"])


def test_vtrace_on_policy_is_discounted_return():
    """tests/test_vtrace.py on-policy identity: with pi == mu and unclipped
    ratios, v-trace targets are the discounted returns bootstrapped with the
    last value."""
    _cuda()
    import rl_triton
    x = gen(8, 100, 5, p=0.03)
    lp = x["lpt"]
    vs, _ = rl_triton.compute_vtrace(D(lp), D(lp), D(x["v"]), D(x["r"]), D(x["d"]), gamma=0.95,
                                     last_value=D(x["lv"]))
    ret = np.zeros_like(x["r"], dtype=np.float64)
    c = x["lv"].astype(np.float64)
    for k in reversed(range(x["r"].shape[1])):
        c = x["r"][:, k] + 0.95 * (1 - x["d"][:, k]) * c
        ret[:, k] = c
    close(vs, ret, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("boundary", ["ends_at", "starts_at"])
def test_prefix_no_dones_and_all_dones(boundary):
    """tests/test_prefix_sum.py no-dones / all-dones cases."""
    _cuda()
    import rl_triton
    x = gen(4, 333, 6)
    none = np.zeros_like(x["d"])
    close(rl_triton.compute_episodic_prefix_sum(D(x["r"]), D(none), boundary=boundary),
          np.cumsum(x["r"].astype(np.float64), axis=1), rtol=1e-4, atol=1e-4)
    allx = np.ones_like(x["d"])
    got = rl_triton.compute_episodic_prefix_sum(D(x["r"]), D(allx), boundary=boundary)
    close(got, x["r"])


def test_scan_zero_decay_is_the_input():
    """tests/test_scan_chunked.py: zero decay leaves u unchanged."""
    _cuda()
    from rl_triton.ops._scan import _run_scan, _run_scan_forward
    u = np.random.default_rng(0).standard_normal((3, 5000)).astype(np.float32)
    z = np.zeros_like(u)
    close(_run_scan(D(u), D(z)), u)
    close(_run_scan_forward(D(u), D(z)), u)


# ---------------------------------------------------------------- dispatch threshold
@pytest.mark.parametrize("t", [131072, 131073])
def test_dispatch_threshold(t):
    """tests/test_scan_chunked.py:96-133: at and just above _FLAT_MAX_SEQ_LEN the
    results agree with the oracle, including the reference's above-threshold
    bootstrap convention (additive per-step bootstrap values)."""
    _cuda()
    import rl_triton
    from rl_triton.ops._scan import _FLAT_MAX_SEQ_LEN, _run_scan
    assert _FLAT_MAX_SEQ_LEN == 131072
    g = np.random.default_rng(t)
    u = g.standard_normal((2, t)).astype(np.float32)
    v = (0.9 + 0.1 * g.random((2, t))).astype(np.float32)
    close(_run_scan(D(u), D(v)), orc.affine_scan(u, v, None, 0), rtol=1e-4, atol=1e-4)
    x = gen(2, t, t, p=0.001)
    boot = np.zeros_like(x["r"])
    boot[:, -1] = x["lv"]
    kind = orc.BOOT_LASTCOL if t <= 131072 else orc.BOOT_FULL_ADD
    vs, adv = rl_triton.compute_vtrace(D(x["lpt"]), D(x["lpb"]), D(x["v"]), D(x["r"]), D(x["d"]),
                                       bootstrap_values=D(boot))
    wvs, wadv = orc.vtrace(x["lpt"], x["lpb"], x["v"], x["r"], x["d"], None, boot, kind)
    close(vs, wvs)
    close(adv, wadv)
