"""Time-split scans: one long sequence cut along time across ranks.

No counterpart in the reference, which runs every scan on one device
(ROADMAP.md lists multi-GPU as future work).  Rank k of W holds columns
[t0_k, t0_k + S_k) of every row (its *segment*), with t0 given by the ranks'
order.  Each call:

1. exchanges the segment lengths (unless the caller passes `t0` and `total`,
   which spares a host synchronisation) and the one-column halos the recurrences
   read across a cut: backward GAE needs the next segment's first value
   V[t0+S]; the forward scans gated by done[t-1] need the previous segment's
   last flag;
2. scans its segment with the cut treated as carry 0 (one kernel launch);
3. summarises each row as the affine map (A, B): state at the far edge =
   A + B * carry entering at the near edge (rls_segment_reduce);
4. all-gathers the W maps (8 bytes per row per rank) and composes the true
   carry of its cut from the ranks beyond it;
5. applies it with the bounded fix-up out[t] += P[t] * carry, which stops
   where the decay product P reaches 0 (rls_segment_fixup).

Nothing else crosses ranks, so the collectives are two tiny all-gathers.  The
collective and the three per-segment primitives are injectable (`all_gather`,
`kernels`): the default is torch.distributed and librlscan; the tests drive the
same code with gloo ranks and a CPU stand-in for the kernels, and with threads
sharing one GPU.
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
        return f0.contiguous(), (f1.contiguous() if f1 is not None else None), dt

    def reduce(self, alg, x, out, seg: Segment, halo, p):
        f0, f1, dt = self._flags(alg, x)
        n, s = out.shape
        ab = torch.empty(2, n, dtype=torch.float32, device=out.device)
        st = nat.lib.rls_segment_reduce(alg, f0.data_ptr(), nat.ptr(f1), dt, out.data_ptr(), ab[0].data_ptr(),
                                        ab[1].data_ptr(), n, s, float(p["coef"]), int(p["flags"]),
                                        seg.cstruct(halo), nat.stream_handle(out.device))
        nat.check(st, "rls_segment_reduce")
        return ab

    def fixup(self, alg, x, out, carry, seg: Segment, halo, p):
        f0, f1, dt = self._flags(alg, x)
        n, s = out.shape
        st = nat.lib.rls_segment_fixup(alg, f0.data_ptr(), nat.ptr(f1), dt, out.data_ptr(), carry.data_ptr(), n, s,
                                       float(p["coef"]), int(p["flags"]), seg.cstruct(halo),
                                       nat.stream_handle(out.device))
        nat.check(st, "rls_segment_fixup")


def torch_all_gather(group=None) -> Callable[[torch.Tensor], list]:
    import torch.distributed as dist

    def gather(t: torch.Tensor) -> list:
        parts = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
        dist.all_gather(parts, t.contiguous(), group=group)
        return parts

    return gather


def _rank_world(group):
    import torch.distributed as dist

    return dist.get_rank(group), dist.get_world_size(group)


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

    # (1) segment lengths and halos in one gather: [length, edge column].
    if alg == GAE:
        edge = x["values"][:, 0].float()           # our first value: the previous rank's halo
    elif alg == ELIGIBILITY or (alg == PREFIX and p["boundary"] == "ends_at"):
        edge = x["dones"][:, -1].float()           # our last flag: the next rank's halo
    else:
        edge = torch.zeros(n, dtype=torch.float32, device=dev)
    # The length travels as two fp32 words (s // 2^20, s % 2^20), each exact
    # below 2^24, so any length up to 2^44 arrives unrounded.
    hi, lo = divmod(int(s), 1 << 20)
    meta = torch.cat([torch.tensor([float(hi), float(lo)], dtype=torch.float32, device=dev), edge])
    metas = all_gather(meta)
    if t0 is None or total is None:  # learn the layout (reads the lengths on the host)
        lengths = [int(m[0].item()) * (1 << 20) + int(m[1].item()) for m in metas]
        t0, total = sum(lengths[:rank]), sum(lengths)
    seg = Segment(rank, world, t0, s, total)
    halo = None
    if alg == GAE and rank + 1 < world:
        halo = metas[rank + 1][2:].contiguous()
    elif alg in (ELIGIBILITY, PREFIX) and rank > 0:
        halo = metas[rank - 1][2:].contiguous()

    # (2)-(3) local scan with a cut, then the segment's map.
    out = kernels.scan(alg, x, seg, halo, p)
    ab = kernels.reduce(alg, x, out, seg, halo, p)
    # (4) every rank's map; compose the carry entering this segment.
    maps = all_gather(ab)
    carry = torch.zeros(n, dtype=torch.float32, device=dev)
    order = range(world - 1, rank, -1) if backward else range(0, rank)
    for j in order:
        carry = maps[j][0] + maps[j][1] * carry
    # (5) bounded fix-up (a no-op on the segment holding the global edge).
    if (rank < world - 1) if backward else (rank > 0):
        kernels.fixup(alg, x, out, carry, seg, halo, p)
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
