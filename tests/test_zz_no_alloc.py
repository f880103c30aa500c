"""rls_gae_noalloc: GAE for callers that cannot allocate device memory.

Some callers of this library cannot call cudaMalloc at the moment they need
advantages: code running while a CUDA graph is captured into a memory pool it
does not own, a real-time training loop whose memory budget is frozen after
start-up, or a host runtime that only hands out buffers it allocated itself.
rls_gae_noalloc serves them: its look-back scratch is a fixed array inside the
library, so the caller passes only inputs and outputs.

These tests call the entry point through the C ABI (ctypes) and check it
against rls_gae with a caller-provided workspace and against the fp32 C
oracle, twice in a row (the second call reuses the array the first one left
behind), at the parity tolerance of the other GPU tests, on the library's own
kernel choice and on every kernel family that keeps records in the scratch.
After each pair of calls the scratch's error latch must read 0.  The file is
named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from rl_triton import _native as nat

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-5


def _inputs(n, t, seed):
    g = torch.Generator().manual_seed(seed)
    r = torch.randn(n, t, generator=g)
    v = torch.randn(n, t, generator=g)
    term = (torch.rand(n, t, generator=g) < 0.01).float()
    return [x.cuda() for x in (r, v, term)]


def _gae_with_workspace(r, v, term, out):
    n, t = r.shape
    dev = r.device
    stream = torch.cuda.current_stream(dev).cuda_stream
    ws, wsb = nat.workspace(dev, stream, n * t)
    st = nat.lib.rls_gae(r.data_ptr(), v.data_ptr(), term.data_ptr(), None, None, nat.BOOT_NONE, out.data_ptr(),
                         n, t, 0.99, 0.95, nat.RLS_F32, None, ws, wsb, stream)
    assert st == nat.RLS_OK, nat.lib.rls_status_string(st).decode()


def _gae_noalloc(r, v, term, out):
    n, t = r.shape
    stream = torch.cuda.current_stream(r.device).cuda_stream
    st = nat.lib.rls_gae_noalloc(r.data_ptr(), v.data_ptr(), term.data_ptr(), None, None, nat.BOOT_NONE,
                                 out.data_ptr(), n, t, 0.99, 0.95, nat.RLS_F32, None, stream)
    assert st == nat.RLS_OK, nat.lib.rls_status_string(st).decode()


# Short rows (many rows per tile) and long rows (many tiles per row, so the
# look-back carries values through the fixed scratch).
# The kernel families: the library's choice (auto), and forced families whose
# look-back records live in the scratch (tile, flat, flat2, flat3) or that use
# it for segment maps (vrows).
@pytest.mark.parametrize("path", ["auto", "tile", "flat", "flat2", "flat3", "vrows"])
@pytest.mark.parametrize("n,t", [(4096, 128), (3, 70001), (1, 1 << 20)])
def test_noalloc_matches_workspace_entry_point_twice(n, t, path, monkeypatch):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    if path == "auto":
        monkeypatch.delenv("RLS_PATH", raising=False)
    else:
        monkeypatch.setenv("RLS_PATH", path)
    for call in range(2):
        r, v, term = _inputs(n, t, seed=100 * call + n + t)
        want = torch.empty(n, t, device="cuda")
        got = torch.full((n, t), float("nan"), device="cuda")
        _gae_with_workspace(r, v, term, want)
        _gae_noalloc(r, v, term, got)
        torch.cuda.synchronize()
        g = got.cpu().numpy()
        np.testing.assert_allclose(g, want.cpu().numpy(), rtol=RTOL, atol=ATOL, err_msg=f"call {call}")
        rn, vn, tn = (x.cpu().numpy() for x in (r, v, term))
        np.testing.assert_allclose(g, orc.gae(rn, vn, tn, gamma=0.99, lam=0.95), rtol=RTOL, atol=ATOL,
                                   err_msg=f"call {call} vs oracle")
    stream = torch.cuda.current_stream().cuda_stream
    assert nat.lib.rls_gae_noalloc_error(ctypes.c_void_p(stream)) == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    # Checked before anything touches the device: no buffers needed.
    n = nat.NOALLOC_MAX_ELEMENTS // 1024 + 1
    st = nat.lib.rls_gae_noalloc(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), None, None,
                                 nat.BOOT_NONE, ctypes.c_void_p(16), n, 1024, 0.99, 0.95, nat.RLS_F32, None, None)
    assert st == nat.RLS_ETOOLARGE
    assert "RLS_NOALLOC_MAX_ELEMENTS" in nat.lib.rls_status_string(st).decode()
