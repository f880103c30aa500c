"""Time-split scans (rl_triton.dist): one sequence cut along time across ranks.

CPU: world_size 2 and 3 gloo ranks drive the real driver (length / halo
exchange, carry composition, fix-up placement) with the C oracle standing in
for the per-segment kernels, and every rank's columns are compared with the
oracle run on the whole sequence.  A rank that leaves before the exchange makes
the others fail with an error within the process-group timeout, not hang.

GPU: the same driver with the real kernels, ranks emulated as threads sharing
one GPU (their launches are ordered on one stream; nothing spins across ranks),
compared with the oracle on the whole sequence.
"""
import datetime
import os
import socket
import tempfile
import threading

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from rl_triton import dist as D

RTOL = ATOL = 1e-5
ALGS = ["gae", "gae_trunc", "lambda", "discounted", "eligibility", "prefix_ends", "prefix_starts"]


def _inputs(n, t, seed):
    g = np.random.default_rng(seed)
    term = (g.random((n, t)) < 0.01).astype(np.float32)
    trunc = ((g.random((n, t)) < 0.01) & (term == 0)).astype(np.float32)
    return dict(r=g.standard_normal((n, t)).astype(np.float32), v=g.standard_normal((n, t)).astype(np.float32),
                term=term, trunc=trunc, lv=g.standard_normal(n).astype(np.float32),
                seed=g.standard_normal(n).astype(np.float32))


def _whole(alg, x, precision="f32"):
    pr = dict(precision=precision)
    if alg == "gae":
        return orc.gae(x["r"], x["v"], x["term"], None, x["lv"], orc.BOOT_ROW, 0.99, 0.95, **pr)
    if alg == "gae_trunc":
        return orc.gae(x["r"], x["v"], x["term"], x["trunc"], None, orc.BOOT_NONE, 0.99, 0.95, **pr)
    if alg == "lambda":
        return orc.lambda_returns(x["r"], x["v"], x["term"], x["trunc"], None, orc.BOOT_NONE, 0.99, 0.9, **pr)
    if alg == "discounted":
        return orc.discounted_returns(x["r"], x["term"], x["trunc"], None, orc.BOOT_NONE, 0.97, **pr)
    if alg == "eligibility":
        return orc.eligibility_traces(x["r"], x["term"], 0.99, 0.9, x["seed"], **pr)
    return orc.prefix_sum(x["r"], x["term"], x["seed"], alg == "prefix_ends", **pr)


def _close(got, alg, x, rtol=RTOL, atol=ATOL):
    """oracle.compare against the oracle on the whole sequence (element-wise:
    within rtol / atol of the fp32 or the fp64 oracle, or -- where splitting the
    sequence reassociates a long fp32 running sum -- no further from fp64 than
    twice the fp32 oracle's worst error, plus atol)."""
    res = orc.compare(got, lambda p: _whole(alg, x, p), rtol, atol)
    assert res["ok"], f"{alg}: {res}"


def _segment_call(alg, x, rank, world, to, **kw):
    if "all_gather" in kw:  # ranks emulated in one process: say who we are
        kw.update(rank=rank, world=world)

    def cols(a):
        return to(D.split_columns(torch.from_numpy(a), rank, world).contiguous())

    if alg == "gae":
        return D.compute_gae(cols(x["r"]), cols(x["v"]), cols(x["term"]), None, 0.99, 0.95,
                             last_value=to(torch.from_numpy(x["lv"])), **kw)
    if alg == "gae_trunc":
        return D.compute_gae(cols(x["r"]), cols(x["v"]), cols(x["term"]), cols(x["trunc"]), 0.99, 0.95, **kw)
    if alg == "lambda":
        return D.compute_lambda_returns(cols(x["r"]), cols(x["v"]), cols(x["term"]), cols(x["trunc"]), 0.99, 0.9,
                                        **kw)
    if alg == "discounted":
        return D.compute_discounted_returns(cols(x["r"]), cols(x["term"]), cols(x["trunc"]), 0.97, **kw)
    if alg == "eligibility":
        return D.compute_eligibility_traces(cols(x["r"]), cols(x["term"]), 0.99, 0.9,
                                            to(torch.from_numpy(x["seed"])), **kw)
    return D.compute_episodic_prefix_sum(cols(x["r"]), cols(x["term"]), to(torch.from_numpy(x["seed"])),
                                         "ends_at" if alg == "prefix_ends" else "starts_at", **kw)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, outdir, mode):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from _segment_cpu import CpuKernels

    if mode == "leave" and rank == world - 1:
        os._exit(0)  # this rank leaves between steps, before the exchange
    try:
        if mode == "long":
            # Segment lengths that fp32 cannot hold exactly (2^24 + 1) still
            # give each rank its true t0 and the total length.
            n0, n1 = (1 << 24) + 1, 3
            x = _inputs(1, n0 + n1, 5)
            lo, hi = (0, n0) if rank == 0 else (n0, n0 + n1)
            seen = {}

            class Recording(CpuKernels):
                def scan(self, alg, xx, seg, halo, p):
                    seen.update(t0=seg.t0, total=seg.total)
                    return super().scan(alg, xx, seg, halo, p)

            got = D.compute_episodic_prefix_sum(torch.from_numpy(x["r"][:, lo:hi].copy()),
                                                torch.from_numpy(x["term"][:, lo:hi].copy()),
                                                kernels=Recording())
            assert seen == dict(t0=lo, total=n0 + n1), seen
            want = orc.prefix_sum(x["r"], x["term"])[:, lo:hi]
            res = orc.compare(got.numpy(), lambda pr: orc.prefix_sum(x["r"], x["term"], precision=pr)[:, lo:hi])
            assert res["ok"], res
            del want
            np.save(os.path.join(outdir, f"r{rank}.npy"), np.array([1]))
        elif mode == "leave":
            x = _inputs(2, 50, 0)
            _segment_call("prefix_ends", x, rank, world, lambda t: t, kernels=CpuKernels())
            np.save(os.path.join(outdir, f"r{rank}.npy"), np.array([0]))  # should not get here
        else:
            for alg in ALGS:
                x = _inputs(3, 1001, ALGS.index(alg))
                got = _segment_call(alg, x, rank, world, lambda t: t, kernels=CpuKernels())
                want = D.split_columns(torch.from_numpy(_whole(alg, x)), rank, world).numpy()
                np.testing.assert_allclose(got.numpy(), want, rtol=RTOL, atol=ATOL, err_msg=f"{alg} rank {rank}")
            np.save(os.path.join(outdir, f"r{rank}.npy"), np.array([1]))
    except Exception as e:  # noqa: BLE001
        with open(os.path.join(outdir, f"r{rank}.err"), "w") as f:
            f.write(repr(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _spawn(world, mode):
    import torch.multiprocessing as mp

    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, d, mode)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
            assert not p.is_alive(), "a rank hung"
        return {f: open(os.path.join(d, f), "rb").read() for f in os.listdir(d)}


@pytest.mark.parametrize("world", [2, 3])
def test_time_split_gloo_matches_whole_sequence(world):
    files = _spawn(world, "ok")
    errs = {k: v for k, v in files.items() if k.endswith(".err")}
    assert not errs, errs
    assert sorted(k for k in files if k.endswith(".npy")) == [f"r{r}.npy" for r in range(world)]


def test_time_split_lengths_beyond_fp32_exact_range():
    files = _spawn(2, "long")
    errs = {k: v for k, v in files.items() if k.endswith(".err")}
    assert not errs, errs
    assert sorted(k for k in files if k.endswith(".npy")) == ["r0.npy", "r1.npy"]


def test_time_split_rank_that_leaves_fails_the_others_without_hanging():
    files = _spawn(2, "leave")
    assert "r0.err" in files, files  # the remaining rank's collective ended with an error
    assert "r0.npy" not in files


def test_split_columns_covers_the_sequence():
    t = torch.arange(3 * 10).reshape(3, 10)
    parts = [D.split_columns(t, r, 4) for r in range(4)]
    assert torch.equal(torch.cat(parts, 1), t)


# ---------------------------------------------------------------- GPU
def _thread_gather(world):
    slots = [None] * world
    bar = threading.Barrier(world)

    def make(rank):
        def gather(t):
            slots[rank] = t.clone()
            bar.wait()
            out = list(slots)
            bar.wait()
            return out
        return gather

    return make


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("alg", ALGS)
def test_time_split_cuda_matches_whole_sequence(alg, world):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    x = _inputs(3, 70001, 11)
    make = _thread_gather(world)
    outs, errs = [None] * world, []

    def run(rank):
        try:
            outs[rank] = _segment_call(alg, x, rank, world, lambda t: t.cuda(),
                                       all_gather=make(rank)).cpu()
        except Exception as e:  # noqa: BLE001
            errs.append(repr(e))

    th = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=120)
    assert not errs, errs
    _close(torch.cat(outs, 1).numpy(), alg, x)


@pytest.mark.gpu
def test_time_split_cuda_long_prefix_and_gae():
    """One 2^22-step row split 4 ways: prefix sum and GAE against the oracle."""
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    g = np.random.default_rng(3)
    t = 1 << 22
    x = dict(r=g.standard_normal((1, t)).astype(np.float32), v=g.standard_normal((1, t)).astype(np.float32),
             term=(g.random((1, t)) < 1e-4).astype(np.float32), trunc=np.zeros((1, t), np.float32),
             lv=np.zeros(1, np.float32), seed=np.zeros(1, np.float32))
    for alg in ["prefix_ends", "gae"]:
        make = _thread_gather(4)
        outs = [None] * 4
        th = [threading.Thread(target=lambda r=r: outs.__setitem__(
            r, _segment_call(alg, x, r, 4, lambda a: a.cuda(), all_gather=make(r)).cpu()))
            for r in range(4)]
        for h in th:
            h.start()
        for h in th:
            h.join(timeout=120)
        _close(torch.cat(outs, 1).numpy(), alg, x)
