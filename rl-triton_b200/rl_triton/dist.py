"""Time-split scans: one long sequence cut along time across ranks.

No counterpart in the reference, which runs every scan on one device
(ROADMAP.md lists multi-GPU as future work).  Rank k of W holds columns
[t0_k, t0_k + S_k) of every row (its *segment*), with t0 given by the ranks'
order.  Each call:

1. scans its segment with the cut treated as carry 0 and every value from
   across the cut (the next segment's first V for backward GAE, the previous
   segment's last flag for the forward scans gated by done[t-1]) read as 0
   (one kernel launch);
2. summarises each row in five numbers (rls_segment_summary): the local state
   at the far edge, the decay product across the segment, and the weights with
   which the neighbour's value and state enter the entry element;
3. all-gathers the W summaries (20 bytes per row per rank: the only
   collective) and composes the correction entering its own segment
   (rls_segment_compose, one small kernel);
4. applies it with the bounded fix-up out[t] += P[t] * correction, which stops
   where the decay product P reaches 0 (rls_segment_fixup).

Without `t0` and `total` a first all-gather exchanges the segment lengths (and
reads them on the host); with them the call never synchronises the host, so it
can be captured in a CUDA graph.  The collective and the per-segment
primitives are injectable (`all_gather`, `kernels`): the default is
torch.distributed and librlscan; the tests drive the same code with gloo ranks
and a CPU stand-in for the kernels, and with threads sharing one GPU.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Sequence

import torch

from rl_triton import _native as nat

GAE, LAMBDA, DISCOUNTED, ELIGIBILITY, PREFIX = (nat.ALG_GAE, nat.ALG_LAMBDA, nat.ALG_DISCOUNTED,
                                                  nat.ALG_ELIGIBILITY, nat.ALG_PREFIX)
_BACKWARD = {GAE, LAMBDA, DISCOUNTED}


class Segment:
    """Where a rank's columns sit in the whole sequence."""

    def __init__(self, rank: int, world: int, t0: int, length: int, total: int):
        self.rank, self.world, self.t0, self.length, self.total = rank, world, t0, length, total

    def cstruct(self, halo: torch.Tensor | None):
        return ctypes.pointer(nat.Segment(self.t0, self.total, halo.data_ptr() if halo is not None else None))


class CudaKernels:
    """The per-segment primitives on librlscan (the product path)."""

    def scan(self, alg, x, seg: Segment, halo, p):
        import rl_triton

        c = (seg.t0, seg.total, halo)
        if alg == GAE:
            return rl_triton.compute_gae(x["rewards"], x["values"], x["terminateds"], x.get("truncateds"),
                                         p["gamma"], p["lambda_"], last_value=x.get("last_value"), _segment=c)
        if alg == LAMBDA:
            return rl_triton.compute_lambda_returns(x["rewards"], x["next_values"], x["terminateds"],
                                                    x.get("truncateds"), p["gamma"], p["lambda_"], _segment=c)
        if alg == DISCOUNTED:
            return rl_triton.compute_discounted_returns(x["rewards"], x["terminateds"], x.get("truncateds"),
                                                        p["gamma"], _segment=c)
        if alg == ELIGIBILITY:
            return rl_triton.compute_eligibility_traces(x["inputs"], x["dones"], p["gamma"], p["lambda_"],
                                                        x.get("seed_values"), _segment=c)
        return rl_triton.compute_episodic_prefix_sum(x["inputs"], x["dones"], x.get("seed_values"),
                                                     p["boundary"], _segment=c)

    @staticmethod
    def _flags(alg, x):
        if alg in _BACKWARD:
            f0, f1 = x["terminateds"], x.get("truncateds")
        else:
            f0, f1 = x["dones"], None
        dt = nat.dtype_code(f0)
        if f1 is not None and f1.dtype != f0.dtype:
            f1 = f1.to(f0.dtype)
        return f0.contiguous(), (f1.contiguous() if f1 is not None else None), dt

    def summary(self, alg, x, out, seg: Segment, p):
        f0, f1, dt = self._flags(alg, x)
        n, s = out.shape
        vals = None
        if alg == GAE:
            vals = x["values"]
            vals = (vals if vals.dtype == f0.dtype else vals.to(f0.dtype)).contiguous()
        sm = torch.empty(5, n, dtype=torch.float32, device=out.device)
        st = nat.lib.rls_segment_summary(alg, f0.data_ptr(), nat.ptr(f1), nat.ptr(vals), dt, out.data_ptr(),
                                         sm.data_ptr(), n, s, float(p.get("gamma", 0.0)), float(p["coef"]),
                                         int(p["flags"]), seg.cstruct(None), nat.stream_handle(out.device))
        nat.check(st, "rls_segment_summary")
        return sm

    def compose(self, maps: torch.Tensor, rank: int, world: int, backward: bool, n: int):
        maps = maps.contiguous()
        carry = torch.empty(n, dtype=torch.float32, device=maps.device)
        st = nat.lib.rls_segment_compose(maps.data_ptr(), rank, world, 1 if backward else 0, n, carry.data_ptr(),
                                         nat.stream_handle(maps.device))
        nat.check(st, "rls_segment_compose")
        return carry

    def fixup(self, alg, x, out, carry, seg: Segment, p):
        f0, f1, dt = self._flags(alg, x)
        n, s = out.shape
        st = nat.lib.rls_segment_fixup(alg, f0.data_ptr(), nat.ptr(f1), dt, out.data_ptr(), carry.data_ptr(), n, s,
                                       float(p["coef"]), int(p["flags"]) | nat.SEG_EXCLUSIVE, seg.cstruct(None),
                                       nat.stream_handle(out.device))
        nat.check(st, "rls_segment_fixup")


def torch_all_gather(group=None) -> Callable[[torch.Tensor], torch.Tensor]:
    """All-gather over torch.distributed into one [W, *shape] tensor."""
    import torch.distributed as dist

    def gather(t: torch.Tensor) -> torch.Tensor:
        t = t.contiguous()
        w = dist.get_world_size(group)
        out = torch.empty((w * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t, group=group)
        return out.view((w,) + tuple(t.shape))

    return gather


def _rank_world(group):
    import torch.distributed as dist

    return dist.get_rank(group), dist.get_world_size(group)


_zero_halos: dict = {}


def _zero_halo(n: int, device) -> torch.Tensor:
    """A cached [n] fp32 zero vector: the cut's neighbour values in step 1."""
    key = (str(device), n)
    z = _zero_halos.get(key)
    if z is None:
        z = _zero_halos[key] = torch.zeros(n, dtype=torch.float32, device=device)
    return z


def _stacked(parts) -> torch.Tensor:
    return parts if torch.is_tensor(parts) else torch.stack(list(parts))


def _run(alg, x: dict, p: dict, ref: torch.Tensor, group=None, all_gather=None, kernels=None, rank=None,
         world=None, t0=None, total=None) -> torch.Tensor:
    if all_gather is None:
        all_gather = torch_all_gather(group)
        rank, world = _rank_world(group)
    kernels = kernels or CudaKernels()
    n, s = ref.shape
    assert s >= 1, "every rank needs at least one step of the sequence"
    dev = ref.device
    backward = alg in _BACKWARD

    if t0 is None or total is None:  # learn the layout (reads the lengths on the host)
        lengths = [int(v) for v in _stacked(all_gather(torch.tensor([s], dtype=torch.int64, device=dev))).view(-1)]
        t0, total = sum(lengths[:rank]), sum(lengths)
    seg = Segment(rank, world, t0, s, total)
    at_end, at_start = t0 + s == total, t0 == 0
    halo = None
    if alg == GAE and not at_end:
        halo = _zero_halo(n, dev)
    elif (alg == ELIGIBILITY or (alg == PREFIX and p["boundary"] == "ends_at")) and not at_start:
        halo = _zero_halo(n, dev)

    out = kernels.scan(alg, x, seg, halo, p)                 # (1) local scan, cut as carry 0
    summary = kernels.summary(alg, x, out, seg, p)           # (2) [5, n]
    maps = _stacked(all_gather(summary))                     # (3) [W, 5, n]: the one collective
    carry = kernels.compose(maps, rank, world, backward, n)
    if not (at_end if backward else at_start):               # (4) bounded fix-up
        kernels.fixup(alg, x, out, carry, seg, p)
    return out


def compute_gae(rewards, values, terminateds, truncateds=None, gamma=0.99, lambda_=0.95, last_value=None, *,
                group=None, all_gather=None, kernels=None, rank=None, world=None, t0=None, total=None):
    """GAE over a sequence split along time; arguments are this rank's columns.
    `last_value` is read by the rank that holds the window end."""
    x = dict(rewards=rewards, values=values, terminateds=terminateds, truncateds=truncateds, last_value=last_value)
    p = dict(gamma=gamma, lambda_=lambda_, coef=gamma * lambda_, flags=0)
    return _run(GAE, x, p, rewards, group, all_gather, kernels, rank, world, t0, total)


def compute_lambda_returns(rewards, next_values, terminateds, truncateds=None, gamma=0.99, lambda_=0.95, *,
                           group=None, all_gather=None, kernels=None, rank=None, world=None, t0=None, total=None):
    x = dict(rewards=rewards, next_values=next_values, terminateds=terminateds, truncateds=truncateds)
    p = dict(gamma=gamma, lambda_=lambda_, coef=gamma * lambda_, flags=0)
    return _run(LAMBDA, x, p, rewards, group, all_gather, kernels, rank, world, t0, total)


def compute_discounted_returns(rewards, terminateds, truncateds=None, gamma=0.99, *, group=None, all_gather=None,
                               kernels=None, rank=None, world=None, t0=None, total=None):
    x = dict(rewards=rewards, terminateds=terminateds, truncateds=truncateds)
    p = dict(gamma=gamma, coef=gamma, flags=0)
    return _run(DISCOUNTED, x, p, rewards, group, all_gather, kernels, rank, world, t0, total)


def compute_eligibility_traces(gradients, dones, gamma, lambda_, seed_values=None, *, group=None, all_gather=None,
                               kernels=None, rank=None, world=None, t0=None, total=None):
    """Traces over a sequence split along time; `seed_values` is read by rank 0."""
    x = dict(inputs=gradients, dones=dones, seed_values=seed_values)
    p = dict(gamma=gamma, lambda_=lambda_, coef=gamma * lambda_, flags=0)
    return _run(ELIGIBILITY, x, p, gradients, group, all_gather, kernels, rank, world, t0, total)


def compute_episodic_prefix_sum(inputs, dones, seed_values=None, boundary="ends_at", *, group=None, all_gather=None,
                                kernels=None, rank=None, world=None, t0=None, total=None):
    """Episodic prefix sum over a sequence split along time; `seed_values` is read by rank 0."""
    x = dict(inputs=inputs, dones=dones, seed_values=seed_values)
    p = dict(boundary=boundary, coef=1.0, flags=1 if boundary == "ends_at" else 0)
    return _run(PREFIX, x, p, inputs, group, all_gather, kernels, rank, world, t0, total)


def split_columns(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Columns of rank `rank` when [N, T] is cut into `world` near-equal segments."""
    T = t.shape[1]
    lo, hi = rank * T // world, (rank + 1) * T // world
    return t[:, lo:hi]


__all__: Sequence[str] = ["compute_gae", "compute_lambda_returns", "compute_discounted_returns",
                          "compute_eligibility_traces", "compute_episodic_prefix_sum", "split_columns",
                          "CudaKernels", "Segment", "torch_all_gather"]
