"""CPU oracle -- TEST INFRASTRUCTURE ONLY.

numpy front end of oracle/rlscan_oracle.c (the C restatement of the
reference's sequential estimators).  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm import this module; the rl_triton
package never does.

Every function takes numpy float32 arrays (int64 for Retrace actions) and
returns float32 or float64 arrays (`precision="f32"` reproduces the
reference's fp32 sequential loops, `"f64"` is the higher-precision yardstick).
Rows are split over a thread pool; each ctypes call releases the GIL.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")


def build() -> str:
    """Compile the oracle with its Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def _load():
    if not os.path.exists(LIB_PATH):
        build()
    return ctypes.CDLL(LIB_PATH)


_lib = _load()
_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_D = ctypes.c_double
_I = ctypes.c_int

_ARGS = {
    "orc_gae": [_P, _P, _P, _P, _P, _I, _P, _I64, _I64, _D, _D],
    "orc_vtrace": [_P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _I64, _I64, _D, _D, _D],
    "orc_retrace": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _D, _D, _D, _D],
    "orc_lambda": [_P, _P, _P, _P, _P, _I, _P, _I64, _I64, _D, _D],
    "orc_discounted": [_P, _P, _P, _P, _I, _P, _I64, _I64, _D],
    "orc_eligibility": [_P, _P, _P, _P, _I64, _I64, _D, _D],
    "orc_prefix": [_P, _P, _P, _I, _P, _I64, _I64],
    "orc_scan": [_P, _P, _P, _I, _P, _I64, _I64],
    "orc_gae_obs_skip": [_P, _P, _P, _P, _P, _I64, _I64, _D, _D],
}
for _n, _a in _ARGS.items():
    for _s in ("_f32", "_f64"):
        f = getattr(_lib, _n + _s)
        f.argtypes = _a
        f.restype = None

BOOT_NONE, BOOT_ROW, BOOT_LASTCOL, BOOT_FULL_ADD, BOOT_FULL_SEL = range(5)

_THREADS = int(os.environ.get("RLS_ORACLE_THREADS", os.cpu_count() or 1))


def threads() -> int:
    return _THREADS


def _f32(a):
    if a is None:
        return None
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a, off=0):
    if a is None:
        return None
    return a.ctypes.data + off * a.itemsize


def _rows(N: int, fn, nthreads: int | None = None) -> None:
    """Run fn(row_start, row_count) over row blocks on a thread pool."""
    nt = max(1, min(nthreads or _THREADS, N))
    if nt == 1:
        fn(0, N)
        return
    bounds = np.linspace(0, N, nt + 1).astype(np.int64)
    with ThreadPoolExecutor(nt) as ex:
        list(ex.map(lambda k: fn(int(bounds[k]), int(bounds[k + 1] - bounds[k])), range(nt)))


def _out(shape, precision):
    return np.empty(shape, dtype=np.float32 if precision == "f32" else np.float64)


def gae(r, v, term, trunc=None, boot=None, kind=BOOT_NONE, gamma=0.99, lam=0.95, precision="f32", nthreads=None):
    r, v, term, trunc, boot = map(_f32, (r, v, term, trunc, boot))
    N, T = r.shape
    out = _out((N, T), precision)
    fn = getattr(_lib, "orc_gae_" + precision)
    row_boot = kind == BOOT_ROW

    def go(n0, cnt):
        o = n0 * T
        fn(_p(r, o), _p(v, o), _p(term, o), _p(trunc, o), _p(boot, n0 if row_boot else o), kind,
           _p(out, o), cnt, T, gamma, lam)

    _rows(N, go, nthreads)
    return out


def vtrace(lpt, lpb, v, r, term, trunc=None, boot=None, kind=BOOT_NONE, gamma=0.99, rho_bar=1.0, c_bar=1.0,
           precision="f32", nthreads=None):
    lpt, lpb, v, r, term, trunc, boot = map(_f32, (lpt, lpb, v, r, term, trunc, boot))
    N, T = r.shape
    vs, adv = _out((N, T), precision), _out((N, T), precision)
    fn = getattr(_lib, "orc_vtrace_" + precision)
    row_boot = kind == BOOT_ROW

    def go(n0, cnt):
        o = n0 * T
        fn(_p(lpt, o), _p(lpb, o), _p(v, o), _p(r, o), _p(term, o), _p(trunc, o),
           _p(boot, n0 if row_boot else o), kind, _p(vs, o), _p(adv, o), cnt, T, gamma, rho_bar, c_bar)

    _rows(N, go, nthreads)
    return vs, adv


def retrace(pi, mu, q, nq, act, r, term, trunc, gamma=0.99, lam=1.0, c_bar=1.0, rho_bar=1.0, precision="f32",
            nthreads=None):
    pi, mu, q, nq, r, term, trunc = map(_f32, (pi, mu, q, nq, r, term, trunc))
    act = np.ascontiguousarray(act, dtype=np.int64)
    N, T = r.shape
    A = pi.shape[2]
    qret, adv = _out((N, T), precision), _out((N, T), precision)
    fn = getattr(_lib, "orc_retrace_" + precision)

    def go(n0, cnt):
        o = n0 * T
        fn(_p(pi, o * A), _p(mu, o), _p(q, o), _p(nq, o * A), _p(act, o), _p(r, o), _p(term, o), _p(trunc, o),
           _p(qret, o), _p(adv, o), cnt, T, A, gamma, lam, c_bar, rho_bar)

    _rows(N, go, nthreads)
    return qret, adv


def lambda_returns(r, nv, term, trunc=None, boot=None, kind=BOOT_NONE, gamma=0.99, lam=0.95, precision="f32",
                   nthreads=None):
    r, nv, term, trunc, boot = map(_f32, (r, nv, term, trunc, boot))
    N, T = r.shape
    out = _out((N, T), precision)
    fn = getattr(_lib, "orc_lambda_" + precision)

    def go(n0, cnt):
        o = n0 * T
        fn(_p(r, o), _p(nv, o), _p(term, o), _p(trunc, o), _p(boot, o), kind, _p(out, o), cnt, T, gamma, lam)

    _rows(N, go, nthreads)
    return out


def discounted_returns(r, term, trunc=None, boot=None, kind=BOOT_NONE, gamma=0.99, precision="f32",
                       nthreads=None):
    r, term, trunc, boot = map(_f32, (r, term, trunc, boot))
    N, T = r.shape
    out = _out((N, T), precision)
    fn = getattr(_lib, "orc_discounted_" + precision)

    def go(n0, cnt):
        o = n0 * T
        fn(_p(r, o), _p(term, o), _p(trunc, o), _p(boot, o), kind, _p(out, o), cnt, T, gamma)

    _rows(N, go, nthreads)
    return out


def eligibility_traces(g, dones, gamma, lam, seed=None, precision="f32", nthreads=None):
    g, dones, seed = map(_f32, (g, dones, seed))
    N, T = g.shape
    out = _out((N, T), precision)
    fn = getattr(_lib, "orc_eligibility_" + precision)

    def go(n0, cnt):
        o = n0 * T
        fn(_p(g, o), _p(dones, o), _p(seed, n0), _p(out, o), cnt, T, gamma, lam)

    _rows(N, go, nthreads)
    return out


def prefix_sum(x, dones, seed=None, ends_at=True, precision="f32", nthreads=None):
    x, dones, seed = map(_f32, (x, dones, seed))
    N, T = x.shape
    out = _out((N, T), precision)
    fn = getattr(_lib, "orc_prefix_" + precision)

    def go(n0, cnt):
        o = n0 * T
        fn(_p(x, o), _p(dones, o), _p(seed, n0), 1 if ends_at else 0, _p(out, o), cnt, T)

    _rows(N, go, nthreads)
    return out


def affine_scan(u, v, carry=None, direction=0, precision="f32", nthreads=None):
    u, v, carry = map(_f32, (u, v, carry))
    N, T = u.shape
    out = _out((N, T), precision)
    fn = getattr(_lib, "orc_scan_" + precision)

    def go(n0, cnt):
        o = n0 * T
        fn(_p(u, o), _p(v, o), _p(carry, n0), direction, _p(out, o), cnt, T)

    _rows(N, go, nthreads)
    return out


def gae_obs_skip(r, v, mask, gamma=1.0, lam=1.0, precision="f32", nthreads=None):
    """Observation-skip GAE (the boundary mode of the reference's ROADMAP.md
    v0.2; no code counterpart there): returns (advantages, returns)."""
    r, v, mask = map(_f32, (r, v, mask))
    N, T = r.shape
    adv, ret = _out((N, T), precision), _out((N, T), precision)
    fn = getattr(_lib, "orc_gae_obs_skip_" + precision)

    def go(n0, cnt):
        o = n0 * T
        fn(_p(r, o), _p(v, o), _p(mask, o), _p(adv, o), _p(ret, o), cnt, T, gamma, lam)

    _rows(N, go, nthreads)
    return adv, ret


def compare(got, oracle, rtol=1e-5, atol=1e-5):
    """Parity verdict of a result against the oracle, element by element.

    `oracle(precision)` returns the oracle's output ("f32" or "f64").  An
    element passes when it is within rtol / atol of the fp32 sequential oracle
    (the reference's own fp32 loop order), or within rtol / atol of the fp64
    oracle (the exact answer), or when its distance to the fp64 oracle is at
    most twice the fp32 oracle's worst distance to it, plus atol: no less
    accurate than the sequential fp32 reference is on the same data (long
    running sums, values that end near zero after large intermediates).  Where
    the fp32 oracle is exact to within atol the last rule is the tolerance.  Returns a dict:
    ok, max_abs_err (vs fp32 oracle), criterion, and, when the fp64 leg ran,
    err_vs_f64, oracle_f32_err_vs_f64 and how many elements needed each rule."""
    got = np.asarray(got, dtype=np.float64)
    w32 = np.asarray(oracle("f32"), dtype=np.float64)
    diff = np.abs(got - w32)
    res = {"max_abs_err": float(diff.max()) if diff.size else 0.0, "rtol": rtol, "atol": atol}
    pass32 = diff <= atol + rtol * np.abs(w32)
    if not diff.size or bool(np.all(pass32)):
        res.update(ok=True, criterion="fp32 oracle within rtol/atol")
        return res
    w64 = np.asarray(oracle("f64"), dtype=np.float64)
    d64 = np.abs(got - w64)
    ref_dev = np.abs(w32 - w64)
    pass64 = d64 <= atol + rtol * np.abs(w64)
    ref_max = float(ref_dev.max())
    pass_ref = d64 <= 2 * ref_max + atol
    ok = pass32 | pass64 | pass_ref
    res.update(ok=bool(np.all(ok)), err_vs_f64=float(d64.max()), oracle_f32_err_vs_f64=ref_max,
               elements_outside_fp32_tol=int((~pass32).sum()),
               of_which_within_fp64_tol=int((~pass32 & pass64).sum()),
               of_which_within_2x_fp32_oracle_worst_error=int((~pass32 & ~pass64 & pass_ref).sum()),
               criterion="per element: fp32 oracle within rtol/atol, or fp64 oracle within rtol/atol, or "
                         "distance to fp64 <= 2x the fp32 oracle's worst distance to fp64 + atol")
    return res
