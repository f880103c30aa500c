"""The C-ABI library loads and exports every entry point include/rlscan.h
declares; argument validation answers without touching a GPU.  CPU only."""
import ctypes
import os
import re
import subprocess

import pytest

from rl_triton import _native as nat

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rlscan.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(rls_[a-z_0-9]+)\s*\(", src)))


def test_header_declares_the_estimators():
    syms = declared_symbols()
    for s in ["rls_gae", "rls_vtrace", "rls_retrace", "rls_lambda_returns", "rls_discounted_returns",
              "rls_eligibility_traces", "rls_prefix_sum", "rls_affine_scan", "rls_segment_reduce",
              "rls_segment_fixup", "rls_workspace_bytes", "rls_status_string"]:
        assert s in syms


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", nat.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (rls_[a-z_0-9]+)$", out, flags=re.M))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    for s in declared_symbols():
        assert hasattr(nat.lib, s)
    assert set(nat.EXPORTED) <= set(declared_symbols())


def test_library_is_sm100a():
    info = nat.build_info()
    assert "sm_100a" in info


def test_workspace_bytes_grows_with_tiles():
    a = nat.lib.rls_workspace_bytes(512)
    b = nat.lib.rls_workspace_bytes(512 * 1000)
    assert b > a >= 64
    assert nat.lib.rls_workspace_bytes(0) == 64


@pytest.mark.parametrize("code,text", [(0, "ok"), (1, "invalid argument"), (2, "pointer not 16-byte aligned"),
                                       (3, "workspace missing or too small"), (5, "unsupported")])
def test_status_strings(code, text):
    assert text in nat.lib.rls_status_string(code).decode()


def test_null_arguments_are_rejected_without_a_gpu():
    P = None
    assert nat.lib.rls_gae(P, P, P, P, P, 0, P, 4, 8, 0.99, 0.95, 0, None, P, 0, P) == nat.RLS_OK + 1
    assert nat.lib.rls_prefix_sum(P, P, P, 1, P, 4, 8, 0, None, P, 0, P) == 1
    assert nat.lib.rls_affine_scan(P, P, P, 3, P, 4, 8, None, P, 0, P) == 1
    assert nat.lib.rls_retrace(*([P] * 10), 4, 8, 0, 0.99, 1.0, 1.0, 1.0, P, 0, P) == 1
    assert nat.lib.rls_segment_reduce(99, P, P, 0, P, P, P, 1, 1, 1.0, 0, None, P) == 1


def test_misaligned_pointer_rejected():
    buf = (ctypes.c_float * 64)()
    base = ctypes.addressof(buf)
    a = base + (16 - base % 16) % 16
    bad = a + 4
    st = nat.lib.rls_discounted_returns(bad, a, None, None, 0, a, 2, 8, 0.99, 0, None, a, 1 << 16, None)
    assert st == 2


def test_host_pointers_are_rejected_before_any_launch():
    """Aligned, non-null host memory: every entry point answers RLS_ENOTDEVICE
    before it enqueues anything (here there is not even a GPU to enqueue on)."""
    buf = (ctypes.c_float * 256)()
    base = ctypes.addressof(buf)
    a = base + (16 - base % 16) % 16
    assert nat.lib.rls_gae(a, a, a, None, None, 0, a, 2, 8, 0.99, 0.95, 0, None, a, 512, None) == nat.RLS_ENOTDEVICE
    assert nat.lib.rls_prefix_sum(a, a, None, 1, a, 2, 8, 0, None, a, 512, None) == nat.RLS_ENOTDEVICE
    assert nat.lib.rls_affine_scan(a, a, None, 0, a, 2, 8, None, a, 512, None) == nat.RLS_ENOTDEVICE
    assert nat.lib.rls_vtrace(a, a, a, a, a, None, None, 0, a, a, 2, 8, 0.99, 1.0, 1.0, 0, a, 512,
                              None) == nat.RLS_ENOTDEVICE
    assert nat.lib.rls_gae_noalloc(a, a, a, None, None, 0, a, 2, 8, 0.99, 0.95, 0, None, None) == nat.RLS_ENOTDEVICE
    assert "not device memory" in nat.lib.rls_status_string(nat.RLS_ENOTDEVICE).decode()
