"""CPU stand-in for the per-segment primitives of rl_triton.dist (local scan
with a cut, segment summary, carry composition, bounded fix-up), built on the
C oracle.
Test infrastructure only: it lets gloo ranks on CPU drive the real
time-split driver (halo exchange, carry composition, fix-up placement)."""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle as orc
from rl_triton import dist as D


def _np(t):
    return None if t is None else t.detach().float().cpu().numpy()


def _decays(alg, x, p, halo):
    """Decay b[t] of every element of the segment, without any cut."""
    if alg in (D.GAE, D.LAMBDA, D.DISCOUNTED):
        done = _np(x["terminateds"])
        if x.get("truncateds") is not None:
            done = np.minimum(done + _np(x["truncateds"]), 1.0)
        return np.float32(p["coef"]) * (1.0 - done)
    dn = _np(x["dones"])
    gate_prev = alg == D.ELIGIBILITY or p["boundary"] == "ends_at"
    if gate_prev:
        prev = np.concatenate([(_np(halo)[:, None] if halo is not None else np.zeros((dn.shape[0], 1), np.float32)),
                               dn[:, :-1]], axis=1)
        flag = prev
    else:
        flag = dn
    k = np.float32(p["coef"]) if alg == D.ELIGIBILITY else np.float32(1.0)
    return k * (1.0 - flag)


class CpuKernels:
    def scan(self, alg, x, seg, halo, p):
        n = x["dones" if alg in (D.ELIGIBILITY, D.PREFIX) else "rewards"].shape[0]
        end = seg.t0 + seg.length == seg.total
        start = seg.t0 == 0
        if alg == D.GAE:
            if end:
                lv = x.get("last_value")
                kind, boot = (orc.BOOT_ROW, _np(lv)) if lv is not None else (orc.BOOT_NONE, None)
            else:
                kind, boot = orc.BOOT_ROW, _np(halo)
            out = orc.gae(_np(x["rewards"]), _np(x["values"]), _np(x["terminateds"]), _np(x.get("truncateds")), boot,
                          kind, p["gamma"], p["lambda_"])
        elif alg == D.LAMBDA:
            out = orc.lambda_returns(_np(x["rewards"]), _np(x["next_values"]), _np(x["terminateds"]),
                                     _np(x.get("truncateds")), None, orc.BOOT_NONE, p["gamma"], p["lambda_"])
        elif alg == D.DISCOUNTED:
            out = orc.discounted_returns(_np(x["rewards"]), _np(x["terminateds"]), _np(x.get("truncateds")), None,
                                         orc.BOOT_NONE, p["gamma"])
        elif alg == D.ELIGIBILITY:
            seed = _np(x.get("seed_values")) if start else None
            out = orc.eligibility_traces(_np(x["inputs"]), _np(x["dones"]), p["gamma"], p["lambda_"], seed)
        else:
            seed = _np(x.get("seed_values")) if start else None
            out = orc.prefix_sum(_np(x["inputs"]), _np(x["dones"]), seed, p["boundary"] == "ends_at")
        assert out.shape[0] == n
        return torch.from_numpy(np.ascontiguousarray(out, dtype=np.float32))

    @staticmethod
    def _walk(alg, p):
        # columns from the edge where the carry enters inward
        return alg in (D.GAE, D.LAMBDA, D.DISCOUNTED)

    def _products(self, alg, x, p, halo, exclusive):
        b = _decays(alg, x, p, halo)
        if self._walk(alg, p):
            if exclusive:
                b = b.copy()
                b[:, -1] = 1.0  # the entry element's own decay is left out
            return np.flip(np.cumprod(np.flip(b, 1), axis=1, dtype=np.float32), 1)
        return np.cumprod(b, axis=1, dtype=np.float32)

    def summary(self, alg, x, out, seg, p):
        backward = self._walk(alg, p)
        global_edge = (seg.t0 + seg.length == seg.total) if backward else seg.t0 == 0
        P = self._products(alg, x, p, None, True)
        n = out.shape[0]
        sm = np.zeros((5, n), np.float32)
        sm[0] = out[:, 0 if backward else -1].numpy()
        sm[1] = 0.0 if global_edge else P[:, 0 if backward else -1]
        if backward:
            sm[3] = _decays(alg, x, p, None)[:, -1]
            if alg == D.GAE:
                term = _np(x["terminateds"])[:, -1]
                tr = _np(x["truncateds"])[:, -1] if x.get("truncateds") is not None else np.zeros(n, np.float32)
                sm[2] = np.where(tr == 0, np.float32(p["gamma"]) * (1 - term), 0).astype(np.float32)
                sm[4] = _np(x["values"])[:, 0]
        else:
            gate_prev = alg == D.ELIGIBILITY or p["boundary"] == "ends_at"
            sm[2] = (1 - _np(x["dones"])[:, -1]) if gate_prev else 1.0
        return torch.from_numpy(sm)

    def compose(self, maps, rank, world, backward, n):
        m = maps.numpy().astype(np.float32)
        if backward:
            if rank == world - 1:
                return torch.zeros(n)
            s0 = m[world - 1, 0]
            for k in range(world - 2, rank, -1):
                corr = m[k, 2] * m[k + 1, 4] + m[k, 3] * s0
                s0 = m[k, 0] + m[k, 1] * corr
            return torch.from_numpy((m[rank, 2] * m[rank + 1, 4] + m[rank, 3] * s0).astype(np.float32))
        c = np.zeros(n, np.float32)
        for k in range(rank):
            c = m[k, 2] * (m[k, 0] + m[k, 1] * c)
        return torch.from_numpy(c.astype(np.float32))

    def fixup(self, alg, x, out, carry, seg, p):
        P = self._products(alg, x, p, None, True)
        o = out.numpy()
        o += P * carry.numpy()[:, None]
