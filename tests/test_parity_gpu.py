"""CUDA path (librlscan.so via the rl_triton drop-in API) against the CPU
oracle and the golden fixtures.

Tolerance: rtol = atol = 1e-5 against the fp32 sequential oracle (the bar
stated for this port); bf16 inputs are compared with the oracle run on the
same bf16-rounded values (1e-5) and with the fp32-input oracle at rtol 1e-2.
"""
import numpy as np
import pytest
import torch

from _cases import api_replay, load_cases
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-5
CASES = load_cases()


def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    return torch.device("cuda")


def close(got, want, rtol=RTOL, atol=ATOL, msg=""):
    np.testing.assert_allclose(np.asarray(got, dtype=np.float64), np.asarray(want, dtype=np.float64),
                               rtol=rtol, atol=atol, err_msg=msg)


def T(a, dev="cuda", dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=dev, dtype=dtype)


@pytest.fixture(autouse=True, params=["auto", "rows2", "vrows", "flat4", "flat3", "flat2", "tile", "rows", "flat"])
def kernel_path(request, monkeypatch):
    """Run every case on each kernel family: the library's own choice ("auto"),
    the TMA-staged tile kernel, the row-parallel register kernel (one warp per
    row) and the flat register kernel with decoupled look-back."""
    if request.param == "auto":
        monkeypatch.delenv("RLS_PATH", raising=False)
    else:
        monkeypatch.setenv("RLS_PATH", request.param)
    return request.param


@pytest.fixture(autouse=True)
def _no_device_errors(kernel_path):
    _cuda()
    yield
    from rl_triton import _native as nat
    torch.cuda.synchronize()
    assert nat.workspace_error() == 0, "a bounded device wait ran out"


# ---------------------------------------------------------------- golden
@pytest.mark.parametrize("case,tens,exp", CASES, ids=[c[0]["name"] for c in CASES])
def test_golden_replay(case, tens, exp):
    got = api_replay(case, tens)
    for k, want in exp.items():
        close(got[k], want, msg=f"{case['name']}:{k}")


# ---------------------------------------------------------------- random
SHAPES = [(1, 1), (1, 2), (3, 7), (5, 31), (2, 127), (4, 128), (3, 129), (7, 333), (64, 512), (4096, 128),
          (1, 4095), (1, 4097), (2, 20000), (3, 70001), (1, 262147)]


def rng_inputs(n, t, seed, p_done=0.05):
    g = np.random.default_rng(seed)
    term = (g.random((n, t)) < p_done).astype(np.float32)
    trunc = ((g.random((n, t)) < p_done) & (term == 0)).astype(np.float32)
    boot = np.where(trunc == 1, g.standard_normal((n, t)), 0).astype(np.float32)
    boot[:, -1] = g.standard_normal(n)
    return dict(
        r=g.standard_normal((n, t)).astype(np.float32),
        v=g.standard_normal((n, t)).astype(np.float32),
        term=term, trunc=trunc, boot=boot,
        lv=g.standard_normal(n).astype(np.float32),
        lpt=(0.5 * g.standard_normal((n, t))).astype(np.float32),
        lpb=(0.5 * g.standard_normal((n, t))).astype(np.float32),
        seed=g.standard_normal(n).astype(np.float32),
    )


@pytest.mark.parametrize("n,t", SHAPES)
@pytest.mark.parametrize("mode", ["plain", "last_value", "trunc_boot", "trunc_noboot", "boot_lastcol"])
def test_gae_random(n, t, mode):
    import rl_triton
    x = rng_inputs(n, t, seed=n * 1000 + t)
    kw = dict(gamma=0.99, lambda_=0.95)
    trunc = boot = None
    kind = orc.BOOT_NONE
    if mode == "last_value":
        kw["last_value"] = T(x["lv"])
        kind, boot = orc.BOOT_ROW, x["lv"]
    elif mode == "trunc_boot":
        trunc = x["trunc"]
        kw["truncateds"], kw["bootstrap_values"] = T(trunc), T(x["boot"])
        kind, boot = orc.BOOT_FULL_SEL, x["boot"]
    elif mode == "trunc_noboot":
        trunc = x["trunc"]
        kw["truncateds"] = T(trunc)
    elif mode == "boot_lastcol":
        kw["bootstrap_values"] = T(x["boot"])
        # Above 131072 steps the reference's chunked path adds bootstrap_values
        # at every step (src/rl_triton/ops/gae.py:200-205); below, only the last column.
        kind, boot = (orc.BOOT_LASTCOL if t <= 131072 else orc.BOOT_FULL_ADD), x["boot"]
    got = rl_triton.compute_gae(T(x["r"]), T(x["v"]), T(x["term"]), **kw).cpu().numpy()
    want = orc.gae(x["r"], x["v"], x["term"], trunc, boot, kind, 0.99, 0.95)
    close(got, want)


@pytest.mark.parametrize("n,t", SHAPES)
@pytest.mark.parametrize("mode", ["plain", "last_value", "trunc_boot", "clip"])
def test_vtrace_random(n, t, mode):
    import rl_triton
    x = rng_inputs(n, t, seed=7 + n * 1000 + t)
    kw = dict(gamma=0.99)
    trunc = boot = None
    kind = orc.BOOT_NONE
    rho, c = 1.0, 1.0
    if mode == "last_value":
        kw["last_value"] = T(x["lv"])
        kind, boot = orc.BOOT_ROW, x["lv"]
    elif mode == "trunc_boot":
        trunc = x["trunc"]
        kw["truncateds"], kw["bootstrap_values"] = T(trunc), T(x["boot"])
        kind, boot = orc.BOOT_FULL_ADD, x["boot"]
    elif mode == "clip":
        rho, c = 1.3, 0.7
    kw.update(rho_bar=rho, c_bar=c)
    vs, adv = rl_triton.compute_vtrace(T(x["lpt"]), T(x["lpb"]), T(x["v"]), T(x["r"]), T(x["term"]), **kw)
    wvs, wadv = orc.vtrace(x["lpt"], x["lpb"], x["v"], x["r"], x["term"], trunc, boot, kind, 0.99, rho, c)
    close(vs.cpu().numpy(), wvs, msg="targets")
    close(adv.cpu().numpy(), wadv, msg="advantages")


@pytest.mark.parametrize("n,t", [(1, 300001), (64, 20000)])
@pytest.mark.parametrize("regime", ["no_resets", "trunc_boot"])
def test_vtrace_long_walks(n, t, regime, kernel_path):
    """Few long rows with no episode resets and c = c_bar everywhere (target
    log-probs above the behaviour ones): on the virtual-row path the carry
    fix-up walks until gamma^k underflows, the longest walk it can take."""
    import rl_triton
    if kernel_path not in ("auto", "vrows", "flat3"):
        pytest.skip("long-row families only")
    g = np.random.default_rng(n + t)
    lpb = (-g.random((n, t))).astype(np.float32)
    lpt = (lpb + 0.1 + 0.2 * g.random((n, t))).astype(np.float32)
    v = g.standard_normal((n, t)).astype(np.float32)
    r = g.standard_normal((n, t)).astype(np.float32)
    term = np.zeros((n, t), np.float32)
    kw = dict(gamma=0.99, rho_bar=1.0, c_bar=1.0)
    trunc = boot = None
    kind = orc.BOOT_NONE
    if regime == "trunc_boot":
        trunc = (g.random((n, t)) < 1e-4).astype(np.float32)
        boot = np.where(trunc == 1, g.standard_normal((n, t)), 0).astype(np.float32)
        kw["truncateds"], kw["bootstrap_values"] = T(trunc), T(boot)
        kind = orc.BOOT_FULL_ADD
    vs, adv = rl_triton.compute_vtrace(T(lpt), T(lpb), T(v), T(r), T(term), **kw)

    def oracle(k):
        return lambda pr: orc.vtrace(lpt, lpb, v, r, term, trunc, boot, kind, 0.99, 1.0, 1.0, precision=pr)[k]

    # Targets reach ~10 here and the advantages subtract them back to O(1):
    # the shared element-wise rule (fp32 oracle, fp64 oracle, or no less
    # accurate than the fp32 loop) decides.
    _no_less_accurate(vs.cpu().numpy(), oracle(0), f"targets {n}x{t} {regime}")
    _no_less_accurate(adv.cpu().numpy(), oracle(1), f"advantages {n}x{t} {regime}")


@pytest.mark.parametrize("n,t,A", [(1, 1, 4), (3, 7, 4), (5, 129, 4), (64, 512, 4), (4096, 128, 4), (2, 3000, 4),
                                   (1, 70001, 4), (4, 33, 1), (3, 50, 3), (2, 77, 7), (2, 40, 18), (1, 300, 80)])
def test_retrace_random(n, t, A):
    import rl_triton
    g = np.random.default_rng(n * 31 + t * 7 + A)
    logits = g.standard_normal((n, t, A)).astype(np.float32)
    pi = np.exp(logits - logits.max(-1, keepdims=True))
    pi = (pi / pi.sum(-1, keepdims=True)).astype(np.float32)
    act = g.integers(0, A, (n, t)).astype(np.int64)
    mu = (g.random((n, t)) * 0.8 + 0.1).astype(np.float32)
    q = g.standard_normal((n, t)).astype(np.float32)
    nq = g.standard_normal((n, t, A)).astype(np.float32)
    r = g.standard_normal((n, t)).astype(np.float32)
    term = (g.random((n, t)) < 0.05).astype(np.float32)
    trunc = ((g.random((n, t)) < 0.05) & (term == 0)).astype(np.float32)
    qr, adv = rl_triton.compute_retrace(T(pi), T(mu), T(q), T(nq), T(act, dtype=torch.int64), T(r), T(term),
                                        T(trunc), gamma=0.99, lambda_=0.95, c_bar=1.0, rho_bar=1.0)
    wq, wa = orc.retrace(pi, mu, q, nq, act, r, term, trunc, 0.99, 0.95, 1.0, 1.0)
    close(qr.cpu().numpy(), wq, msg="targets")
    close(adv.cpu().numpy(), wa, msg="advantages")


@pytest.mark.parametrize("n,t", SHAPES)
@pytest.mark.parametrize("mode", ["plain", "boot", "trunc_boot"])
def test_returns_random(n, t, mode):
    import rl_triton
    x = rng_inputs(n, t, seed=11 + n * 1000 + t)
    trunc = boot = None
    kind = orc.BOOT_NONE
    kw = {}
    nv = x["v"].copy()
    if mode == "boot":
        kw["bootstrap_values"] = T(x["boot"])
        kind, boot = orc.BOOT_LASTCOL, x["boot"]
    elif mode == "trunc_boot":
        trunc = x["trunc"]
        nv = nv * (1 - trunc)
        kw["truncateds"], kw["bootstrap_values"] = T(trunc), T(x["boot"])
        kind, boot = orc.BOOT_FULL_ADD, x["boot"]
    got = rl_triton.compute_lambda_returns(T(x["r"]), T(nv), T(x["term"]), gamma=0.99, lambda_=0.9, **kw)
    close(got.cpu().numpy(), orc.lambda_returns(x["r"], nv, x["term"], trunc, boot, kind, 0.99, 0.9), msg="lambda")
    got = rl_triton.compute_discounted_returns(T(x["r"]), T(x["term"]), gamma=0.97, **kw)
    close(got.cpu().numpy(), orc.discounted_returns(x["r"], x["term"], trunc, boot, kind, 0.97), msg="disc")


@pytest.mark.parametrize("n,t", SHAPES)
@pytest.mark.parametrize("seeded", [False, True])
def test_forward_random(n, t, seeded):
    import rl_triton
    x = rng_inputs(n, t, seed=13 + n * 1000 + t)
    sd = x["seed"] if seeded else None
    kws = dict(seed_values=T(sd)) if seeded else {}
    got = rl_triton.compute_eligibility_traces(T(x["r"]), T(x["term"]), 0.99, 0.9, **kws)
    close(got.cpu().numpy(), orc.eligibility_traces(x["r"], x["term"], 0.99, 0.9, sd), msg="elig")
    for bd in ("ends_at", "starts_at"):
        got = rl_triton.compute_episodic_prefix_sum(T(x["r"]), T(x["term"]), boundary=bd, **kws)
        want = orc.prefix_sum(x["r"], x["term"], sd, bd == "ends_at")
        close(got.cpu().numpy(), want, msg=bd)


@pytest.mark.parametrize("n,t", [(1, 1), (3, 7), (4, 129), (64, 512), (2, 20000), (1, 262147)])
def test_generic_scans(n, t):
    from rl_triton.ops._scan import _run_scan, _run_scan_forward
    g = np.random.default_rng(n + t)
    u = g.standard_normal((n, t)).astype(np.float32)
    v = (g.random((n, t)) * 0.99).astype(np.float32)
    c = g.standard_normal(n).astype(np.float32)
    close(_run_scan(T(u), T(v), T(c)).cpu().numpy(), orc.affine_scan(u, v, c, 0))
    close(_run_scan(T(u), T(v)).cpu().numpy(), orc.affine_scan(u, v, None, 0))
    close(_run_scan_forward(T(u), T(v), T(c)).cpu().numpy(), orc.affine_scan(u, v, c, 1))


# ---------------------------------------------------------------- bf16
@pytest.mark.parametrize("n,t", [(3, 129), (64, 512), (4096, 128), (1, 100003)])
def test_bf16_inputs(n, t):
    import rl_triton
    x = rng_inputs(n, t, seed=17 + t)
    bf = {k: torch.from_numpy(x[k]).to(torch.bfloat16) for k in ("r", "v", "term", "lpt", "lpb")}
    rd = {k: bf[k].float().numpy() for k in bf}  # the values the kernel actually sees
    dev = {k: bf[k].cuda() for k in bf}
    got = rl_triton.compute_gae(dev["r"], dev["v"], dev["term"], gamma=0.99, lambda_=0.95)
    assert got.dtype == torch.float32
    close(got.cpu().numpy(), orc.gae(rd["r"], rd["v"], rd["term"], gamma=0.99, lam=0.95), msg="gae bf16")
    close(got.cpu().numpy(), orc.gae(x["r"], x["v"], x["term"], gamma=0.99, lam=0.95), rtol=1e-2, atol=1e-1,
          msg="gae bf16 vs fp32 inputs")
    vs, adv = rl_triton.compute_vtrace(dev["lpt"], dev["lpb"], dev["v"], dev["r"], dev["term"], gamma=0.99)
    wvs, wadv = orc.vtrace(rd["lpt"], rd["lpb"], rd["v"], rd["r"], rd["term"], gamma=0.99)
    close(vs.cpu().numpy(), wvs, msg="vtrace bf16 targets")
    close(adv.cpu().numpy(), wadv, msg="vtrace bf16 advantages")
    for fn, ofn in [(lambda: rl_triton.compute_discounted_returns(dev["r"], dev["term"], gamma=0.99),
                     lambda: orc.discounted_returns(rd["r"], rd["term"], gamma=0.99)),
                    (lambda: rl_triton.compute_episodic_prefix_sum(dev["r"], dev["term"]),
                     lambda: orc.prefix_sum(rd["r"], rd["term"]))]:
        close(fn().cpu().numpy(), ofn())


# ---------------------------------------------------------------- contract
def test_determinism_bit_identical():
    import rl_triton
    x = rng_inputs(1, 1 << 20, seed=5, p_done=1e-4)
    a = T(x["r"]), T(x["term"])
    outs = [rl_triton.compute_episodic_prefix_sum(*a).cpu().numpy() for _ in range(3)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
    outs = [rl_triton.compute_gae(T(x["r"]), T(x["v"]), T(x["term"])).cpu().numpy() for _ in range(3)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])


def test_mutual_exclusion_message():
    import rl_triton
    r = torch.rand(4, 16, device="cuda")
    with pytest.raises(AssertionError, match="not both"):
        rl_triton.compute_gae(r, r, torch.zeros_like(r), bootstrap_values=torch.zeros_like(r),
                              last_value=torch.rand(4, device="cuda"))
    with pytest.raises(AssertionError, match="not both"):
        rl_triton.compute_vtrace(r, r, r, r, torch.zeros_like(r), bootstrap_values=torch.zeros_like(r),
                                 last_value=torch.rand(4, device="cuda"))


def test_last_value_equals_bootstrap_column():
    import rl_triton
    x = rng_inputs(8, 64, seed=3)
    lv = T(x["lv"])
    bv = torch.zeros(8, 64, device="cuda")
    bv[:, -1] = lv
    a = rl_triton.compute_gae(T(x["r"]), T(x["v"]), T(x["term"]), last_value=lv)
    b = rl_triton.compute_gae(T(x["r"]), T(x["v"]), T(x["term"]), bootstrap_values=bv)
    torch.testing.assert_close(a, b, atol=1e-6, rtol=1e-6)


def test_non_contiguous_and_misaligned_inputs():
    import rl_triton
    x = rng_inputs(16, 65, seed=9)
    big = torch.randn(16, 130, device="cuda")
    r = big[:, ::2]  # non-contiguous view
    assert not r.is_contiguous()
    want = rl_triton.compute_gae(r.contiguous(), T(x["v"]), T(x["term"]))
    torch.testing.assert_close(rl_triton.compute_gae(r, T(x["v"]), T(x["term"])), want)
    flat = torch.randn(16 * 65 + 1, device="cuda")
    mis = flat[1:].view(16, 65)  # contiguous, 4-byte offset
    assert mis.data_ptr() % 16 != 0
    want = rl_triton.compute_gae(mis.clone(), T(x["v"]), T(x["term"]))
    torch.testing.assert_close(rl_triton.compute_gae(mis, T(x["v"]), T(x["term"])), want)


def test_empty_inputs():
    import rl_triton
    e = torch.zeros(0, 5, device="cuda")
    assert rl_triton.compute_gae(e, e, e).shape == (0, 5)
    e = torch.zeros(3, 0, device="cuda")
    assert rl_triton.compute_episodic_prefix_sum(e, e).shape == (3, 0)


def test_prefix_sum_accepts_long_sequences():
    """Deliberate difference from the reference (which asserts T <= 131072)."""
    import rl_triton
    x = rng_inputs(2, 131073, seed=21, p_done=1e-3)
    got = rl_triton.compute_episodic_prefix_sum(T(x["r"]), T(x["term"]))
    close(got.cpu().numpy(), orc.prefix_sum(x["r"], x["term"]), rtol=1e-5, atol=1e-4)


def test_lambda1_gae_is_monte_carlo():
    """lambda = 1 GAE telescopes to G_t - V(s_t) (tests/test_gae.py:340-411)."""
    import rl_triton
    g = np.random.default_rng(123)
    n, t, gamma = 16, 37, 0.97
    r = g.standard_normal((n, t)).astype(np.float32)
    v = g.standard_normal((n, t)).astype(np.float32)
    lv = g.standard_normal(n).astype(np.float32)
    ret = np.zeros((n, t))
    c = lv.astype(np.float64)
    for k in reversed(range(t)):
        c = r[:, k] + gamma * c
        ret[:, k] = c
    got = rl_triton.compute_gae(T(r), T(v), T(np.zeros((n, t), np.float32)), gamma=gamma, lambda_=1.0,
                                last_value=T(lv))
    close(got.cpu().numpy(), ret - v, rtol=1e-4, atol=1e-4)


def test_kernel_families_share_one_workspace():
    """Every look-back kernel family leaves the per-stream workspace ready for the
    next launch of any family (each launch runs under a fresh epoch)."""
    import os
    import rl_triton
    from rl_triton import _native as nat
    old = os.environ.get("RLS_PATH")
    try:
        for path in ["vrows", "flat3", "flat2", "tile", "vrows", "flat", "flat2", "flat3", "vrows", "tile", "flat2"]:
            os.environ["RLS_PATH"] = path
            for n, t in [(64, 512), (1, 4095), (3, 5000)]:
                x = rng_inputs(n, t, seed=n + t)
                got = rl_triton.compute_gae(T(x["r"]), T(x["v"]), T(x["term"])).cpu().numpy()
                close(got, orc.gae(x["r"], x["v"], x["term"]), msg=f"{path} {n}x{t}")
                torch.cuda.synchronize()
                assert nat.workspace_error() == 0, f"{path} {n}x{t}"
    finally:
        if old is None:
            os.environ.pop("RLS_PATH", None)
        else:
            os.environ["RLS_PATH"] = old


def _no_less_accurate(got, oracle, msg):
    """oracle.compare's element-wise criterion (the one every parity check in
    this repository uses): within rtol / atol of the fp32 sequential oracle, or
    of the fp64 oracle, or -- where cutting a running sum over 10^4-10^5-step
    episodes reassociates it -- no further from fp64 than twice the fp32
    oracle's worst error, plus atol."""
    res = orc.compare(got, oracle, RTOL, ATOL)
    assert res["ok"], f"{msg}: {res}"


def test_virtual_row_fixup_paths(kernel_path):
    """Virtual rows on long rows: the flag-free fix-up (prefix sums over binary
    dones, episodes longer than a segment, so some segments hold no reset at
    all), the product-walk fix-up (fractional dones, decaying traces, GAE), both
    scan directions and a row count that does not divide the segments."""
    if kernel_path != "vrows":
        pytest.skip("runs once, with RLS_PATH=vrows")
    import rl_triton
    g = np.random.default_rng(77)
    for n, t in [(1, 1 << 20), (3, 300032)]:
        x = rng_inputs(n, t, seed=n, p_done=2e-5)
        for bd in ["ends_at", "starts_at"]:
            got = rl_triton.compute_episodic_prefix_sum(T(x["r"]), T(x["term"]), boundary=bd).cpu().numpy()
            _no_less_accurate(got, lambda pr: orc.prefix_sum(x["r"], x["term"], None, bd == "ends_at", precision=pr),
                              f"prefix {bd} {n}x{t}")
        frac = np.where(g.random((n, t)) < 1e-4, 0.5, x["term"]).astype(np.float32)
        got = rl_triton.compute_episodic_prefix_sum(T(x["r"]), T(frac)).cpu().numpy()
        _no_less_accurate(got, lambda pr: orc.prefix_sum(x["r"], frac, precision=pr), f"prefix fractional {n}x{t}")
        got = rl_triton.compute_eligibility_traces(T(x["r"]), T(x["term"]), 0.99, 0.95).cpu().numpy()
        close(got, orc.eligibility_traces(x["r"], x["term"], 0.99, 0.95), msg=f"traces {n}x{t}")
        got = rl_triton.compute_gae(T(x["r"]), T(x["v"]), T(x["term"]), gamma=0.99, lambda_=0.95).cpu().numpy()
        close(got, orc.gae(x["r"], x["v"], x["term"]), msg=f"gae {n}x{t}")


def test_chained_calls_read_the_previous_output():
    """A call whose input is the previous call's output (and calls whose outputs
    reuse freed memory) on one stream, eagerly and replayed from a CUDA graph:
    the row kernels overlap consecutive launches, so a kernel that reads the
    previous launch's output must wait for it."""
    import rl_triton
    x = rng_inputs(4096, 128, seed=31, p_done=0.01)
    r, term, v = T(x["r"]), T(x["term"]), T(x["v"])
    d = (term > 0).float()

    def chain():
        a = rl_triton.compute_episodic_prefix_sum(r, d)
        b = rl_triton.compute_discounted_returns(a, term, gamma=0.97)
        c = rl_triton.compute_gae(b, a, term, gamma=0.99, lambda_=0.95)
        e = rl_triton.compute_eligibility_traces(c, d, 0.99, 0.9)
        return a, b, c, e

    def oracle_chain(pr):
        a = orc.prefix_sum(x["r"], x["term"], precision=pr)
        b = orc.discounted_returns(a, x["term"], gamma=0.97, precision=pr)
        c = orc.gae(b, a, x["term"], gamma=0.99, lam=0.95, precision=pr)
        return a, b, c, orc.eligibility_traces(c, x["term"], 0.99, 0.9, precision=pr)

    # Chained returns reach magnitudes ~10^3, where fp32 reassociation alone
    # moves results by more than 1e-5: oracle.compare's fp64 criterion applies.
    def check(outs, how):
        for k, name in enumerate("abce"):
            res = orc.compare(outs[k].cpu().numpy(), lambda pr: oracle_chain(pr)[k], RTOL, ATOL)
            assert res["ok"], f"{how} {name}: {res}"

    check(chain(), "eager")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chain()  # workspace for this stream
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        outs = chain()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    check(outs, "graph")
