"""rls_gae_noalloc: GAE for callers that cannot allocate device memory.

Some callers of this library cannot call cudaMalloc at the moment they need
advantages: code running while a CUDA graph is captured into a memory pool it
does not own, a real-time training loop whose memory budget is frozen after
start-up, or a host runtime that only hands out buffers it allocated itself.
rls_gae_noalloc serves them: its look-back scratch is a fixed array inside the
library, so the caller passes only inputs and outputs.

These tests call the entry point through the C ABI (ctypes) and check it
against rls_gae with a caller-provided workspace, twice in a row (the second
call reuses the array the first one left behind), at the parity tolerance of
the other GPU tests.  The file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

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
@pytest.mark.parametrize("n,t", [(4096, 128), (3, 70001), (1, 1 << 20)])
def test_noalloc_matches_workspace_entry_point_twice(n, t):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    for call in range(2):
        r, v, term = _inputs(n, t, seed=100 * call + n + t)
        want = torch.empty(n, t, device="cuda")
        got = torch.full((n, t), float("nan"), device="cuda")
        _gae_with_workspace(r, v, term, want)
        _gae_noalloc(r, v, term, got)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=RTOL, atol=ATOL,
                                   err_msg=f"call {call}")


def test_noalloc_rejects_sizes_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    # Checked before anything touches the device: no buffers needed.
    n = nat.NOALLOC_MAX_ELEMENTS // 1024 + 1
    st = nat.lib.rls_gae_noalloc(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), None, None,
                                 nat.BOOT_NONE, ctypes.c_void_p(16), n, 1024, 0.99, 0.95, nat.RLS_F32, None, None)
    assert st == nat.RLS_ETOOLARGE
    assert "RLS_NOALLOC_MAX_ELEMENTS" in nat.lib.rls_status_string(st).decode()
