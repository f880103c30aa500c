"""The estimators as PyTorch operators (torch.ops.rl_triton.*): registered
schemas with fake kernels, so a step that calls them compiles into one graph
(torch.compile fullgraph=True) and records into a CUDA graph, with results
equal to eager calls."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    return torch.device("cuda")


def _inputs(n=512, t=128, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = torch.randn(n, t, device="cuda", generator=g)
    v = torch.randn(n, t, device="cuda", generator=g)
    term = (torch.rand(n, t, device="cuda", generator=g) < 0.01).float()
    lpt = 0.5 * torch.randn(n, t, device="cuda", generator=g)
    lpb = 0.5 * torch.randn(n, t, device="cuda", generator=g)
    return r, v, term, lpt, lpb


def _step(r, v, term, lpt, lpb):
    import rl_triton
    adv = rl_triton.compute_gae(r, v, term, gamma=0.99, lambda_=0.95)
    vs, vadv = rl_triton.compute_vtrace(lpt, lpb, v, r, term, gamma=0.99)
    ret = rl_triton.compute_discounted_returns(r, term, gamma=0.99)
    norm = (adv - adv.mean()) / (adv.std() + 1e-8)
    return norm, vs, vadv, ret


def test_compile_fullgraph_matches_eager(monkeypatch):
    _dev()
    monkeypatch.setenv("RL_TRITON_CORRECTNESS_WARNINGS", "0")
    x = _inputs()
    torch._dynamo.reset()
    compiled = torch.compile(_step, fullgraph=True)
    got = compiled(*x)
    want = _step(*x)
    for a, b in zip(got, want):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)
    h = [t.cpu().numpy() for t in x]
    np.testing.assert_allclose(got[1].cpu().numpy(), orc.vtrace(h[3], h[4], h[1], h[0], h[2], gamma=0.99)[0],
                               rtol=1e-5, atol=1e-5)


def test_operator_schemas_and_fake_kernels():
    """torch.library.opcheck: schema, fake kernel and dispatch consistency."""
    _dev()
    r, v, term, lpt, lpb = _inputs(64, 40)
    ops = torch.ops.rl_triton
    checks = [
        (ops.gae, (r, v, term, None, None, 0, 0.99, 0.95)),
        (ops.vtrace, (lpt, lpb, v, r, term, None, None, 0, 0.99, 1.0, 1.0)),
        (ops.discounted_returns, (r, term, None, None, 0, 0.99)),
        (ops.lambda_returns, (r, v, term, None, None, 0, 0.99, 0.95)),
        (ops.eligibility_traces, (r, term, None, 0.99, 0.9)),
        (ops.prefix_sum, (r, term, None, True)),
        (ops.affine_scan, (r, 0.9 * torch.rand_like(r), None, 0)),
    ]
    for op, args in checks:
        torch.library.opcheck(op, args, test_utils=("test_schema", "test_faketensor"))


def test_graph_capture_through_the_public_api():
    _dev()
    x = _inputs(seed=3)
    want = _step(*x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _step(*x)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        out = _step(*x)
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(out, want):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)
