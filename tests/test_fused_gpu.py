"""compute_gae_normalized: GAE with batch-normalised advantages and the value
targets A + V, against the fp32 C oracle's GAE normalised in fp64
((A - mean) / (std + eps), unbiased std, as torch.std), on the single-pass
on-chip path (rows of a multiple of 4 steps that fit in one wave) and the
three-pass path (everything else), for every bootstrap mode and bf16 inputs."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu
RTOL = ATOL = 1e-5


def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def _inputs(n, t, seed, p=0.02):
    g = np.random.default_rng(seed)
    term = (g.random((n, t)) < p).astype(np.float32)
    trunc = ((g.random((n, t)) < p) & (term == 0)).astype(np.float32)
    boot = np.where(trunc == 1, g.standard_normal((n, t)), 0).astype(np.float32)
    boot[:, -1] = g.standard_normal(n)
    return dict(r=g.standard_normal((n, t)).astype(np.float32), v=g.standard_normal((n, t)).astype(np.float32),
                term=term, trunc=trunc, boot=boot, lv=g.standard_normal(n).astype(np.float32))


def _want(adv, v, eps):
    a = adv.astype(np.float64)
    m, s = a.mean(), a.std(ddof=1) if a.size > 1 else 0.0
    return (a - m) / (s + eps), a + v


def D(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("n,t", [(4096, 128), (64, 512), (3, 333), (1, 1), (2, 7), (4096, 1024), (9000, 1024),
                                 (1, 70001)])
@pytest.mark.parametrize("mode", ["plain", "last_value", "trunc_boot"])
def test_gae_normalized_matches_oracle(n, t, mode):
    _cuda()
    import rl_triton
    x = _inputs(n, t, n + t)
    kw = dict(gamma=0.99, lambda_=0.95)
    trunc = boot = None
    kind = orc.BOOT_NONE
    if mode == "last_value":
        kw["last_value"] = D(x["lv"])
        kind, boot = orc.BOOT_ROW, x["lv"]
    elif mode == "trunc_boot":
        trunc = x["trunc"]
        kw["truncateds"], kw["bootstrap_values"] = D(trunc), D(x["boot"])
        kind, boot = (orc.BOOT_FULL_SEL if t <= 131072 else orc.BOOT_FULL_ADD), x["boot"]
    norm, rets = rl_triton.compute_gae_normalized(D(x["r"]), D(x["v"]), D(x["term"]), return_returns=True, **kw)
    adv = orc.gae(x["r"], x["v"], x["term"], trunc, boot, kind, 0.99, 0.95)
    wn, wr = _want(adv, x["v"], 1e-8)
    np.testing.assert_allclose(norm.cpu().numpy(), wn, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(rets.cpu().numpy(), wr, rtol=RTOL, atol=ATOL)


def test_gae_normalized_equals_unfused_torch():
    _cuda()
    import rl_triton
    x = _inputs(4096, 128, 5)
    r, v, term = D(x["r"]), D(x["v"]), D(x["term"])
    adv = rl_triton.compute_gae(r, v, term)
    want = (adv - adv.mean()) / (adv.std() + 1e-8)
    got = rl_triton.compute_gae_normalized(r, v, term)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)


def test_gae_normalized_bf16_and_deterministic():
    _cuda()
    import rl_triton
    x = _inputs(2048, 256, 9)
    bf = {k: torch.from_numpy(x[k]).to(torch.bfloat16).cuda() for k in ("r", "v", "term")}
    rd = {k: bf[k].float().cpu().numpy() for k in bf}
    outs = [rl_triton.compute_gae_normalized(bf["r"], bf["v"], bf["term"]) for _ in range(3)]
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    wn, _ = _want(orc.gae(rd["r"], rd["v"], rd["term"]), rd["v"], 1e-8)
    np.testing.assert_allclose(outs[0].cpu().numpy(), wn, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("n,t", [(4096, 128), (64, 512), (3, 333), (1, 70001)])
@pytest.mark.parametrize("loss", ["mse", "huber"])
def test_gae_value_loss_matches_torch(n, t, loss):
    """Advantages and returns against the oracle; the loss and its gradient
    against torch.nn.functional.mse_loss / huber_loss on the oracle's returns."""
    _cuda()
    import rl_triton
    x = _inputs(n, t, 3 * n + t)
    g = np.random.default_rng(1)
    nv_np = (x["v"] + 0.5 * g.standard_normal((n, t))).astype(np.float32)
    nv = D(nv_np).requires_grad_(True)
    adv, rets, vl = rl_triton.compute_gae_value_loss(D(x["r"]), D(x["v"]), D(x["term"]), nv, loss=loss, delta=0.7)
    vl.backward()
    a = orc.gae(x["r"], x["v"], x["term"])
    np.testing.assert_allclose(adv.detach().cpu().numpy(), a, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(rets.detach().cpu().numpy(), a + x["v"], rtol=RTOL, atol=ATOL)
    ref_nv = D(nv_np).requires_grad_(True)
    target = D((a + x["v"]).astype(np.float32))
    fn = torch.nn.functional.mse_loss if loss == "mse" else (
        lambda i, tt: torch.nn.functional.huber_loss(i, tt, delta=0.7))
    ref = fn(ref_nv.double(), target.double())
    ref.backward()
    np.testing.assert_allclose(float(vl), float(ref), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(nv.grad.cpu().numpy(), ref_nv.grad.cpu().numpy(), rtol=1e-4, atol=1e-9)


def _compacted(r, v, m, gamma, lam):
    """Observation-skip GAE by its defining property: drop the mask-0 tokens,
    run plain GAE on what is left, and give each observation token the
    advantage of the next generated token (0 after the last one)."""
    n, t = r.shape
    out = np.zeros((n, t), np.float64)
    for k in range(n):
        idx = np.nonzero(m[k])[0]
        if idx.size:
            a = orc.gae(r[k:k + 1, idx], v[k:k + 1, idx], np.zeros((1, idx.size), np.float32), gamma=gamma,
                        lam=lam, precision="f64")[0]
        nxt = 0.0
        j = idx.size - 1
        for c in range(t - 1, -1, -1):
            if m[k, c]:
                nxt = a[j]
                j -= 1
            out[k, c] = nxt
    return out


@pytest.mark.parametrize("n,t", [(1, 1), (3, 7), (64, 333), (256, 1024), (5, 4097)])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_gae_obs_skip(n, t, dtype):
    _cuda()
    import rl_triton
    g = np.random.default_rng(n * 7 + t)
    r = g.standard_normal((n, t)).astype(np.float32)
    v = g.standard_normal((n, t)).astype(np.float32)
    # spans of observation tokens between generated spans
    m = (np.cumsum(g.random((n, t)) < 0.05, axis=1) % 2 == 0).astype(np.float32)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    rd, vd = torch.from_numpy(r).to(tdt), torch.from_numpy(v).to(tdt)
    rq, vq = rd.float().numpy(), vd.float().numpy()
    adv, rets = rl_triton.compute_gae_obs_skip(rd.cuda(), vd.cuda(), torch.from_numpy(m > 0).cuda(), gamma=0.99,
                                               lambda_=0.95)
    wa, wr = orc.gae_obs_skip(rq, vq, m, 0.99, 0.95)
    np.testing.assert_allclose(adv.cpu().numpy(), wa, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(rets.cpu().numpy(), wr, rtol=RTOL, atol=ATOL)
    if n * t <= 64 * 333:
        np.testing.assert_allclose(adv.cpu().numpy(), _compacted(rq, vq, m, 0.99, 0.95), rtol=1e-4, atol=1e-4)


def test_fused_outputs_feed_the_next_calls():
    """Each fused call's outputs read by the next call on the same stream (the
    launches overlap under programmatic dependent launch, so a reader of the
    previous launch's output must wait for it): normalised advantages -> their
    discounted sums; returns -> observation-skip GAE; its advantages -> value
    loss targets."""
    _cuda()
    import rl_triton
    x = _inputs(1024, 256, 77)
    r, v, term = D(x["r"]), D(x["v"]), D(x["term"])
    mask = D((x["term"] == 0).astype(np.float32))
    for _ in range(2):
        norm, rets = rl_triton.compute_gae_normalized(r, v, term, return_returns=True)
        disc = rl_triton.compute_discounted_returns(norm, term, gamma=0.9)
        a2, _ = rl_triton.compute_gae_obs_skip(rets, v, mask, gamma=0.99, lambda_=0.95)
        _, _, vl = rl_triton.compute_gae_value_loss(a2, v, term, rets)
    wn, wr = _want(orc.gae(x["r"], x["v"], x["term"]), x["v"], 1e-8)
    wn32, wr32 = wn.astype(np.float32), wr.astype(np.float32)
    res = orc.compare(disc.cpu().numpy(), lambda p: orc.discounted_returns(wn32, x["term"], gamma=0.9, precision=p))
    assert res["ok"], res
    wa2, _ = orc.gae_obs_skip(wr32, x["v"], (x["term"] == 0).astype(np.float32), 0.99, 0.95)
    np.testing.assert_allclose(a2.cpu().numpy(), wa2, rtol=1e-4, atol=1e-4)
    adv3 = orc.gae(a2.cpu().numpy(), x["v"], x["term"])
    want_loss = np.mean((rets.cpu().numpy().astype(np.float64) - (adv3 + x["v"])) ** 2)
    np.testing.assert_allclose(float(vl), want_loss, rtol=1e-4)


def test_gae_obs_skip_few_long_rows():
    """A few very long rows take the two generic affine scans (split across the
    whole GPU) instead of one warp per row."""
    _cuda()
    import rl_triton
    g = np.random.default_rng(3)
    n, t = 2, 300000
    r = g.standard_normal((n, t)).astype(np.float32)
    v = g.standard_normal((n, t)).astype(np.float32)
    m = (np.cumsum(g.random((n, t)) < 1e-3, axis=1) % 2 == 0).astype(np.float32)
    adv, rets = rl_triton.compute_gae_obs_skip(D(r), D(v), D(m), gamma=0.999, lambda_=0.95)
    res = orc.compare(adv.cpu().numpy(), lambda p: orc.gae_obs_skip(r, v, m, 0.999, 0.95, precision=p)[0], RTOL, ATOL)
    assert res["ok"], res
    res = orc.compare(rets.cpu().numpy(), lambda p: orc.gae_obs_skip(r, v, m, 0.999, 0.95, precision=p)[1], RTOL, ATOL)
    assert res["ok"], res
