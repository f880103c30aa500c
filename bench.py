"""Benchmark of the B200 return-estimation scans (drop-in rl_triton).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config cfg2|...]

One step = one pass of the hot path over one batch: the seven estimators of
rl_triton (GAE, V-trace, Retrace, lambda-returns, discounted returns,
eligibility traces, episodic prefix sum) each called once on a batch of the
chosen configuration.  The default workload is configuration 2 of the
reference's headline metric: num_envs=4096, seq_len=128, fp32, synthetic
seeded inputs with the distributions the reference's benchmark uses.

Timing: W untimed steps, then K steps between a barrier + synchronize on both
sides, timed with CUDA events on the launching stream; the max over ranks is
reported.  Each step's launches are replayed from a CUDA graph captured per
input set; the input sets rotate so the working set exceeds the 126 MB L2
(inputs resident in HBM, no L2 reuse between consecutive steps).

Under torchrun (N > 1) every rank runs the same per-GPU workload on its own
environments (env-sharded, weak scaling, no collective in the data path).

After the timed region, and outside it:
  * per function, the device time per launch (graph replay) and the eager
    full-call time through the public API;
  * parity: every output of the first input set against the fp32 C oracle
    (oracle/, test infrastructure) at rtol = atol = 1e-5 -> "parity";
  * the reference's own Triton kernels (the unmodified package installed under
    baseline/_ref, run in a child process that never imports this repository's
    package) on the same inputs, rotation and timing -> "triton_reference",
    with the largest output difference against this arm;
  * end to end through the public API from pinned host buffers -> "e2e";
  * the CPU baseline (the C oracle on the host cores) -> "cpu_baseline".

`--impl reference` times the CPU restatement of the reference's sequential
estimators (oracle/, all host threads) on the same workload; rank 0 prints.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
REF_INSTALL = os.path.join(ROOT, "baseline", "_ref")  # the unmodified reference (pip --target), not in git
TRITON_WORKER = "--triton-worker" in sys.argv
if TRITON_WORKER:
    # The reference's own Triton kernels, imported from its install: this
    # process never puts this repository's package or library on its path.
    sys.path.insert(0, REF_INSTALL)
elif os.path.join(ROOT, "rl-triton_b200") not in sys.path:
    sys.path.insert(0, os.path.join(ROOT, "rl-triton_b200"))
sys.path.insert(1 if TRITON_WORKER else 0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

FUNCS = ["gae", "vtrace", "retrace", "lambda", "discounted", "eligibility", "prefix"]
# Steps captured per CUDA graph when the workload is small: consecutive steps
# in one graph overlap across step boundaries (programmatic dependent launch)
# instead of paying a graph launch per step.  Every step still runs all its
# calls on its own input set.
STEPS_PER_GRAPH = 8
# Algorithmic bytes per timestep (each input read once, each output written once).
A_RETRACE = 4


def bytes_per_step(fn: str, trunc: bool, bf16: bool) -> int:
    e = 2 if bf16 else 4
    if fn == "gae":
        return (3 + (2 if trunc else 0)) * e + 4
    if fn == "vtrace":
        return (5 + (2 if trunc else 0)) * e + 8
    if fn == "retrace":
        return 8 * A_RETRACE + 4 * 5 + 8 + 8  # pi, Qn (A each), mu, q, r, term, trunc, int64 action, 2 outs
    if fn == "lambda":
        return (3 + (2 if trunc else 0)) * e + 4
    if fn == "discounted":
        return (2 + (2 if trunc else 0)) * e + 4
    return 2 * e + 4  # eligibility, prefix


CONFIGS = {
    "cfg2": dict(N=4096, T=128, trunc=False, bf16=False, funcs=FUNCS, p_term=0.01,
                 desc="config 2: all seven estimators, num_envs=4096 seq_len=128 fp32"),
    "cfg3": dict(N=4096, T=128, trunc=True, bf16=False, funcs=["gae", "vtrace", "retrace", "lambda", "discounted"],
                 p_term=0.005, desc="config 3: 4096x128 fp32 with truncations + bootstrap values"),
    "cfg4": dict(N=131072, T=1024, trunc=False, bf16=True, funcs=["gae", "vtrace"], p_term=0.002,
                 desc="config 4: GAE + V-trace, num_envs=131072 seq_len=1024, bf16 inputs, fp32 out (per GPU)"),
    "cfg5a": dict(N=64, T=131072, trunc=False, bf16=False, funcs=["vtrace"], p_term=0.01,
                  desc="config 5a: V-trace num_envs=64 seq_len=131072 fp32"),
    "large": dict(N=131072, T=1024, trunc=False, bf16=False, funcs=FUNCS, p_term=0.01,
                  desc="all seven estimators, num_envs=131072 seq_len=1024 fp32 (the second shape of the "
                       "per-function roofline target; distributions of config 2)"),
    "unaligned": dict(N=4096, T=131, trunc=False, bf16=False, funcs=FUNCS, p_term=0.01,
                      desc="all seven estimators, num_envs=4096 seq_len=131 fp32 (rows not 16-byte aligned)"),
    "cfg5b": dict(N=1, T=1 << 28, trunc=False, bf16=False, funcs=["prefix", "gae"], p_term=1e-4, split=True,
                  desc="config 5b: prefix sum + GAE, num_envs=1 seq_len=2^28 fp32; under torchrun the sequence "
                       "is split along time across the ranks (carry exchange over NCCL)"),
}


# --------------------------------------------------------------------------
def make_inputs(cfg, device, seed, gen_device=None):
    """Seeded synthetic inputs with the distributions of the headline metric's configurations 2-5."""
    N, T = cfg["N"], cfg["T"]
    g = torch.Generator(device=device).manual_seed(seed)
    dt = torch.bfloat16 if cfg["bf16"] else torch.float32

    def randn(*s):
        return torch.randn(*s, generator=g, device=device)

    def bern(p):
        return (torch.rand(N, T, generator=g, device=device) < p).float()

    x = {}
    fs = cfg["funcs"]
    p = cfg["p_term"]
    x["r"] = randn(N, T).to(dt)
    x["term"] = bern(p).to(dt)
    if any(f in fs for f in ("gae", "vtrace", "lambda", "retrace")):
        x["v"] = randn(N, T).to(dt)
    if "vtrace" in fs:
        x["lpt"] = (0.5 * randn(N, T)).to(dt)
        x["lpb"] = (0.5 * randn(N, T)).to(dt)
    if cfg["trunc"]:
        tr = bern(p) * (1 - x["term"].float())
        x["trunc"] = tr.to(dt)
        boot = torch.where(tr.bool(), randn(N, T), torch.zeros((), device=device))
        boot[:, -1] = randn(N)
        x["boot"] = boot.to(dt)
        x["nv"] = (x["v"].float() * (1 - tr)).to(dt)
    else:
        x["nv"] = x.get("v", x["r"])
    if "retrace" in fs:
        A = A_RETRACE
        x["pi"] = torch.softmax(randn(N, T, A), dim=-1)
        x["act"] = torch.randint(0, A, (N, T), generator=g, device=device)
        pa = x["pi"].gather(-1, x["act"].unsqueeze(-1)).squeeze(-1)
        lt, lb = 0.5 * randn(N, T), 0.5 * randn(N, T)
        x["mu"] = pa * torch.exp(-(lt - lb))  # IS ratio pi_a/mu = exp(lt - lb)
        x["q"] = randn(N, T)
        x["nq"] = randn(N, T, A)
        if not cfg["trunc"]:
            # Retrace's API always takes truncateds; a workload without
            # truncations passes zeros (a constant, not per-step data).
            x["notrunc"] = torch.zeros(N, T, device=device)
    return x


def make_calls(cfg, x, split=False):
    """The public-API calls of one step (drop-in rl_triton; rl_triton.dist when
    the sequence is split along time across the ranks)."""
    import rl_triton

    if split:
        from rl_triton import dist as D

        rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
        lay = dict(t0=rank * cfg["T"], total=world * cfg["T"])  # equal segments: no length exchange
        return {k: v for k, v in {
            "prefix": lambda: D.compute_episodic_prefix_sum(x["r"], x["term"], **lay),
            "gae": lambda: D.compute_gae(x["r"], x["v"], x["term"], gamma=0.99, lambda_=0.95, **lay),
        }.items() if k in cfg["funcs"]}

    tr = cfg["trunc"]
    calls = {}
    calls["gae"] = lambda: rl_triton.compute_gae(
        x["r"], x["v"], x["term"], truncateds=x.get("trunc") if tr else None, gamma=0.99, lambda_=0.95,
        bootstrap_values=x.get("boot") if tr else None)
    calls["vtrace"] = lambda: rl_triton.compute_vtrace(
        x["lpt"], x["lpb"], x["v"], x["r"], x["term"], truncateds=x.get("trunc") if tr else None, gamma=0.99,
        rho_bar=1.0, c_bar=1.0, bootstrap_values=x.get("boot") if tr else None)
    calls["retrace"] = lambda: rl_triton.compute_retrace(
        x["pi"], x["mu"], x["q"], x["nq"], x["act"], x["r"], x["term"], x["trunc"] if tr else x["notrunc"], gamma=0.99,
        lambda_=0.95, c_bar=1.0, rho_bar=1.0)
    calls["lambda"] = lambda: rl_triton.compute_lambda_returns(
        x["r"], x["nv"], x["term"], truncateds=x.get("trunc") if tr else None, gamma=0.99, lambda_=0.95,
        bootstrap_values=x.get("boot") if tr else None)
    calls["discounted"] = lambda: rl_triton.compute_discounted_returns(
        x["r"], x["term"], truncateds=x.get("trunc") if tr else None, gamma=0.99,
        bootstrap_values=x.get("boot") if tr else None)
    calls["eligibility"] = lambda: rl_triton.compute_eligibility_traces(x["r"], x["term"], 0.99, 0.95)
    calls["prefix"] = lambda: rl_triton.compute_episodic_prefix_sum(x["r"], x["term"])
    return {k: calls[k] for k in cfg["funcs"]}


# --------------------------------------------------------------------------
class ClockSampler:
    """NVML sampling of SM clock and clock-event reasons during the timed region."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown", 0x1: "gpu_idle",
               0x2: "applications_clocks_setting", 0x100: "display_clock_setting"}

    def __init__(self, index: int):
        self.samples: list[tuple[float, int, int]] = []
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            try:
                props = torch.cuda.get_device_properties(index)
                bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:  # noqa: BLE001
                self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # noqa: BLE001
            self.err = str(e)
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.002)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self._t:
            self._stop.set()
            self._t.join()

    def summary(self, t0: float, t1: float) -> dict:
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable"}
        inside = [s for s in self.samples if t0 <= s[0] <= t1] or self.samples
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mask = 0
        for s in inside:
            mask |= s[2]
        reasons = sorted(v for k, v in self.REASONS.items() if mask & k and v != "gpu_idle")
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(inside)}


# --------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, device_id=torch.device("cuda", local) if backend == "nccl" else None)
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def read_traffic(fn: str, workload: str):
    """DRAM bytes per launch from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        parts = line.split()
        if len(parts) >= 3 and not line.startswith("#") and parts[0] == fn and parts[1] == workload:
            return float(parts[2])
    return None


def read_write_peaks(dev):
    """Context for fractions above 1.0: this GPU's read-only (sum over 4 GiB)
    and write-only (fill of 4 GiB) HBM bandwidth, best of 5, CUDA events.  The
    roofline denominator stays the driver-measured copy bandwidth."""
    x = torch.empty(1 << 30, dtype=torch.float32, device=dev)
    x.fill_(1.0)
    res = {}
    for name, fn in (("read_only_gbs", lambda: x.sum()), ("write_only_gbs", lambda: x.fill_(2.0))):
        fn()
        best = 1e9
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize(dev)
            best = min(best, e0.elapsed_time(e1))
        res[name] = round(x.numel() * 4 / (best * 1e-3) / 1e9, 1)
    del x
    torch.cuda.empty_cache()
    return res


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return 6650.0, "fallback"


# --------------------------------------------------------------------------
def cpu_oracle_step(cfg_name, cfg, x_np, nthreads):
    """One step of the CPU restatement (oracle/) over the same workload."""
    from oracle import oracle as orc

    tr = cfg["trunc"]
    out = []
    for f in cfg["funcs"]:
        if f == "gae":
            out.append(orc.gae(x_np["r"], x_np["v"], x_np["term"], x_np.get("trunc") if tr else None,
                               x_np.get("boot") if tr else None, orc.BOOT_FULL_SEL if tr else orc.BOOT_NONE,
                               nthreads=nthreads))
        elif f == "vtrace":
            out.append(orc.vtrace(x_np["lpt"], x_np["lpb"], x_np["v"], x_np["r"], x_np["term"],
                                  x_np.get("trunc") if tr else None, x_np.get("boot") if tr else None,
                                  orc.BOOT_FULL_ADD if tr else orc.BOOT_NONE, nthreads=nthreads))
        elif f == "retrace":
            out.append(orc.retrace(x_np["pi"], x_np["mu"], x_np["q"], x_np["nq"], x_np["act"], x_np["r"],
                                   x_np["term"], x_np["trunc"] if tr else x_np["notrunc"], 0.99, 0.95,
                                   nthreads=nthreads))
        elif f == "lambda":
            out.append(orc.lambda_returns(x_np["r"], x_np["nv"], x_np["term"], x_np.get("trunc") if tr else None,
                                          x_np.get("boot") if tr else None,
                                          orc.BOOT_FULL_ADD if tr else orc.BOOT_NONE, nthreads=nthreads))
        elif f == "discounted":
            out.append(orc.discounted_returns(x_np["r"], x_np["term"], x_np.get("trunc") if tr else None,
                                              x_np.get("boot") if tr else None,
                                              orc.BOOT_FULL_ADD if tr else orc.BOOT_NONE, nthreads=nthreads))
        elif f == "eligibility":
            out.append(orc.eligibility_traces(x_np["r"], x_np["term"], 0.99, 0.95, nthreads=nthreads))
        elif f == "prefix":
            out.append(orc.prefix_sum(x_np["r"], x_np["term"], nthreads=nthreads))
    return out


def to_numpy(x):
    return {k: (v.float() if v.dtype == torch.bfloat16 else v).cpu().numpy() for k, v in x.items()}


def cpu_sample(cfg, budget_s=15.0, max_steps=50):
    """Time the oracle on the host cores.  Returns (timesteps/s, cores, sample text)."""
    from oracle import oracle as orc

    n_rows = cfg["N"]
    # Bounded sample: whole rows of the workload, sized to ~budget_s of CPU work.
    sub = dict(cfg)
    if cfg["N"] * cfg["T"] > (1 << 22):
        sub["N"] = max(1, (1 << 22) // cfg["T"]) if cfg["T"] <= (1 << 22) else 1
        sub["T"] = min(cfg["T"], 1 << 22)
    x = to_numpy(make_inputs(sub, torch.device("cpu"), seed=123))
    nth = orc.threads()
    cpu_oracle_step(None, sub, x, nth)  # warm-up
    steps, t0 = 0, time.perf_counter()
    while True:
        cpu_oracle_step(None, sub, x, nth)
        steps += 1
        el = time.perf_counter() - t0
        if el > budget_s / 3 or steps >= max_steps:
            break
    per_step = el / steps
    ts = sub["N"] * sub["T"] / per_step
    sample = (f"{steps} step(s) of [{sub['N']}x{sub['T']}] ({', '.join(cfg['funcs'])}); "
              f"rows {'all' if sub['N'] == n_rows else 'prefix'} of the workload")
    return ts, nth, sample


# --------------------------------------------------------------------------
def input_sets(cfg):
    """Input sets rotated between launches so that every function's own working
    set (its bytes per launch x the sets) is at least 3x the 126 MB L2: a launch
    then finds (almost) none of its inputs in L2 from the launches before it.
    Capped at 64 sets and 12 GB of inputs."""
    per_set = sum(bytes_per_step(f, cfg["trunc"], cfg["bf16"]) for f in cfg["funcs"]) * cfg["N"] * cfg["T"]
    min_fn = min(bytes_per_step(f, cfg["trunc"], cfg["bf16"]) for f in cfg["funcs"]) * cfg["N"] * cfg["T"]
    n_sets = int(np.ceil(3 * 126e6 / min_fn))
    n_sets = max(1, min(n_sets, 64, int(12e9 // per_set)))
    return n_sets, per_set


def config_dict(cfg, world, split, n_sets, per_set, use_graph):
    """The `config` object of the JSON line; both arms print the same one."""
    return {"workload": cfg["desc"], "functions": cfg["funcs"], "num_envs_per_gpu": cfg["N"],
            "seq_len": cfg["T"],
            "parallelism": (f"time-split x{world}" if split else f"env-sharded x{world}") if world > 1
            else "single GPU",
            "l2": f"{n_sets} rotating input sets ({per_set * n_sets / 1e6:.0f} MB; every function's own inputs "
                  f"x {n_sets} >= 3x the 126 MB L2)" if n_sets > 1 else
                  f"1 input set ({per_set / 1e6:.0f} MB, > 3x the 126 MB L2)",
            "launch": (f"CUDA graphs of {STEPS_PER_GRAPH} consecutive steps (one input set each)"
                       if n_sets >= STEPS_PER_GRAPH and per_set < 1e9 else "CUDA graph per input set")
                      if use_graph else "eager"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    if args.config not in CONFIGS:
        print(json.dumps({"impl": "reference", "unavailable": f"{args.config}: no CPU arm for this harness"}))
        return
    cfg = CONFIGS[args.config]
    from oracle import oracle as orc

    split = world > 1 and cfg.get("split", False)
    n_sets, per_set = input_sets(dict(cfg, T=cfg["T"] // world) if split else cfg)
    sub = dict(cfg)
    if cfg["N"] * cfg["T"] > (1 << 22):
        sub["N"] = max(1, (1 << 22) // cfg["T"]) if cfg["T"] <= (1 << 22) else 1
        sub["T"] = min(cfg["T"], 1 << 22)
    x = to_numpy(make_inputs(sub, torch.device("cpu"), seed=123))
    nth = orc.threads()
    for _ in range(args.warmup):
        cpu_oracle_step(None, sub, x, nth)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_oracle_step(None, sub, x, nth)
    el = time.perf_counter() - t0
    ms = el / args.steps * 1e3
    value = sub["N"] * sub["T"] / (el / args.steps)
    sample = f"[{sub['N']}x{sub['T']}] of the {args.config} workload per step"
    line = {
        "impl": "reference", "metric": "timesteps/sec", "value": value, "unit": "timesteps/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong" if split else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded; distributions of the headline configurations)",
        "config": config_dict(dict(cfg, T=cfg["T"] // world) if split else cfg, world, split, n_sets, per_set,
                              not split),
        "cpu_baseline": {"value": value, "unit": "timesteps/s", "cores": nth, "kind": "port",
                         "sample": sample + "; CPU restatement of the reference's sequential estimators "
                                            "(oracle/rlscan_oracle.c), rows split over host threads"},
        "e2e": {"value": value, "unit": "timesteps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
def time_function(calls, fname, stream, use_graph, min_reps=8, max_reps=1000, budget_s=0.5, fixed_reps=0):
    """Device time per launch of one public call (CUDA graph of `reps` calls over
    the rotating input sets, CUDA events on the launching stream) and the eager
    full-call time (the same calls issued from Python, device-resident inputs).
    Up to 1000 launches per timing: outputs written back from L2 after the
    timed region (at most the 126 MB L2) are then a small share of the bytes."""
    n_sets = len(calls)
    with torch.cuda.stream(stream):
        t0 = time.perf_counter()
        calls[0][fname]()
        stream.synchronize()
        one = time.perf_counter() - t0
    reps = int(max(min_reps // 2, min(max_reps, budget_s / max(one, 1e-6))))
    reps = fixed_reps or max(3, reps)  # fixed: ranks must issue the same collectives
    out = {}
    g = None
    if use_graph:
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for k in range(reps):
                    calls[k % n_sets][fname]()
        except Exception as e:  # noqa: BLE001
            g = None
            out["graph_error"] = f"{type(e).__name__}: {str(e)[:200]}"
    # One warm replay, then three timed ones; the median is reported (a single
    # replay right after capture occasionally ran at half speed).
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(3)]
    with torch.cuda.stream(stream):
        if g is not None:
            g.replay()
            for e0, e1 in evs:
                e0.record(stream)
                g.replay()
                e1.record(stream)
    stream.synchronize()
    if g is not None:
        ts = sorted(e0.elapsed_time(e1) for e0, e1 in evs)
        out["us_per_launch"] = round(ts[1] * 1e3 / reps, 3)
        out["launch"] = "graph"
    del g
    with torch.cuda.stream(stream):
        for k in range(reps):
            calls[k % n_sets][fname]()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for k in range(reps):
            calls[k % n_sets][fname]()
        f1.record(stream)
    stream.synchronize()
    out["full_call_us"] = round(f0.elapsed_time(f1) * 1e3 / reps, 3)
    if "us_per_launch" not in out:
        out["us_per_launch"] = out["full_call_us"]
        out["launch"] = "eager"
    out["reps"] = reps
    return out


def time_fused(sets, stream, use_graph, world, hbm):
    """GAE + batch advantage normalisation + returns, fused (one call) and
    composed from compute_gae and PyTorch ops, on the rotating input sets."""
    import rl_triton

    def composed(x):
        a = rl_triton.compute_gae(x["r"], x["v"], x["term"], gamma=0.99, lambda_=0.95)
        ret = a + x["v"].float()
        return (a - a.mean()) / (a.std() + 1e-8), ret

    calls = [{"fused": (lambda x=x: rl_triton.compute_gae_normalized(x["r"], x["v"], x["term"], gamma=0.99,
                                                                      lambda_=0.95, return_returns=True)),
              "composed": (lambda x=x: composed(x))} for x in sets]
    x0 = sets[0]
    n, t = x0["r"].shape
    esz = x0["r"].element_size()
    alg = (3 * esz + 8) * n * t  # r, v, term in; normalised advantages and returns out
    out = {"workload": "advantages normalised over the batch + returns (A + V)",
           "algorithmic_bytes": alg}
    for name in ("fused", "composed"):
        r = time_function(calls, name, stream, use_graph, fixed_reps=8 if world > 1 else 0)
        out[name] = {"us_per_call": r["us_per_launch"], "full_call_us": r["full_call_us"],
                     "frac_of_peak": round(alg / (r["us_per_launch"] * 1e-6) / 1e9 / hbm, 4)}
    out["speedup"] = round(out["composed"]["us_per_call"] / out["fused"]["us_per_call"], 3)

    # GAE + returns + value loss and its gradient for the value head's outputs.
    nvs = [(x["v"].float() + 0.1).requires_grad_(True) for x in sets]

    def vl_fused(x, nv):
        _, _, loss = rl_triton.compute_gae_value_loss(x["r"], x["v"], x["term"], nv, gamma=0.99, lambda_=0.95)
        loss.backward()

    def vl_composed(x, nv):
        a = rl_triton.compute_gae(x["r"], x["v"], x["term"], gamma=0.99, lambda_=0.95)
        loss = torch.nn.functional.mse_loss(nv, a + x["v"].float())
        loss.backward()

    vcalls = [{"fused": (lambda x=x, nv=nv: vl_fused(x, nv)), "composed": (lambda x=x, nv=nv: vl_composed(x, nv))}
              for x, nv in zip(sets, nvs)]
    vl = {"workload": "advantages, returns, value loss (MSE) and its gradient (backward)"}
    for name in ("fused", "composed"):
        # Device time: forward and backward captured in a CUDA graph (the
        # gradient accumulates into new_values.grad in place); full call: eager,
        # which the autograd engine's host work dominates at this size.
        r = time_function(vcalls, name, stream, use_graph, fixed_reps=8 if world > 1 else 0)
        vl[name] = {"us_per_call": r["us_per_launch"], "launch": r.get("launch"), "full_call_us": r["full_call_us"]}
        if "graph_error" in r:
            vl[name]["graph_error"] = r["graph_error"]
    vl["speedup"] = round(vl["composed"]["us_per_call"] / vl["fused"]["us_per_call"], 3)
    vl["full_call_speedup"] = round(vl["composed"]["full_call_us"] / vl["fused"]["full_call_us"], 3)
    out["value_loss"] = vl
    return out


def sample_window(cfg):
    """Rows and columns of an output compared across the two GPU arms."""
    rows = min(cfg["N"], max(1, (1 << 22) // cfg["T"]))
    return rows, min(cfg["T"], 1 << 22)


def flat_outputs(fname, res):
    res = res if isinstance(res, tuple) else (res,)
    return {f"{fname}_{k}": r for k, r in enumerate(res)}


def triton_worker(args):
    """Runs in a child process with only the reference's install on sys.path:
    times the reference's stock rl_triton.compute_* (Triton JIT for this GPU)
    on the same inputs, rotation and timing method as the main arm."""
    import triton

    import rl_triton  # the unmodified reference, from baseline/_ref

    cfg = CONFIGS[args.config]
    dev = torch.device("cuda", args.device)
    torch.cuda.set_device(dev)
    n_sets, _ = input_sets(cfg)
    sets = []
    for k in range(n_sets):
        x = make_inputs(cfg, dev, seed=k)
        if cfg["bf16"]:  # the reference accepts fp32 only (src/rl_triton/ops/gae.py:109)
            x = {key: (v.float() if v.dtype == torch.bfloat16 else v) for key, v in x.items()}
        sets.append(x)
    calls = [make_calls(cfg, x) for x in sets]
    stream = torch.cuda.Stream(dev)
    res = {"module": os.path.relpath(rl_triton.__file__, ROOT), "version": getattr(rl_triton, "__version__", None),
           "triton": triton.__version__, "inputs": "fp32 copies of the bf16 inputs" if cfg["bf16"] else "same",
           "per_function": {}}
    outs = {}
    rows, cols = sample_window(cfg)
    for f in cfg["funcs"]:
        try:
            with torch.cuda.stream(stream):
                for c in calls:  # JIT compile + warm-up
                    c[f]()
            stream.synchronize()
            res["per_function"][f] = time_function(calls, f, stream, use_graph=not args.no_graph)
            with torch.cuda.stream(stream):
                o = calls[0][f]()
            stream.synchronize()
            for key, t in flat_outputs(f, o).items():
                outs[key] = t[:rows, :cols].float().cpu().numpy()
        except Exception as e:  # noqa: BLE001
            res["per_function"][f] = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
        torch.cuda.synchronize()
    if args.triton_out and outs:
        np.savez(args.triton_out, **outs)
    print("TRITON_REF_JSON " + json.dumps(res), flush=True)


def triton_reference(args, cfg, ours, ours_timing, local):
    """Launches triton_worker and compares its timings and outputs with this arm's."""
    import subprocess
    import tempfile

    if not os.path.isdir(os.path.join(REF_INSTALL, "rl_triton")):
        return {"reason": "reference not installed under baseline/_ref"}
    fd, path = tempfile.mkstemp(suffix=".npz")
    os.close(fd)
    cmd = [sys.executable, os.path.abspath(__file__), "--triton-worker", "--config", args.config,
           "--device", str(local), "--triton-out", path]
    if args.no_graph:
        cmd.append("--no-graph")
    env = dict(os.environ)
    env.pop("PYTHONPATH", None)
    env.pop("RLS_PATH", None)
    try:
        p = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env, cwd="/")
    except subprocess.TimeoutExpired:
        return {"reason": "reference worker timed out (900 s)"}
    line = [ln for ln in p.stdout.splitlines() if ln.startswith("TRITON_REF_JSON ")]
    if p.returncode != 0 or not line:
        tail = (p.stderr or p.stdout).strip().splitlines()[-3:]
        return {"reason": f"reference worker exit {p.returncode}: {' | '.join(tail)[:400]}"}
    res = json.loads(line[0][len("TRITON_REF_JSON "):])
    theirs = {}
    if os.path.exists(path):
        try:
            with np.load(path) as z:
                theirs = {k: z[k] for k in z.files}
        except Exception:  # noqa: BLE001
            theirs = {}
        os.unlink(path)
    for f, r in res["per_function"].items():
        if "error" in r:
            continue
        mine = ours_timing.get(f, {})
        r["ours_us"] = mine.get("us_per_launch")
        r["triton_us"] = r.get("us_per_launch")
        if r["ours_us"] and r["triton_us"]:
            r["speedup"] = round(r["triton_us"] / r["ours_us"], 3)
        if mine.get("full_call_us") and r.get("full_call_us"):
            r["full_call_speedup"] = round(r["full_call_us"] / mine["full_call_us"], 3)
        diffs = []
        for key, arr in ours.items():
            if key.startswith(f + "_") and key in theirs:
                diffs.append(float(np.max(np.abs(arr.astype(np.float64) - theirs[key]))) if arr.size else 0.0)
        if diffs:
            r["max_abs_diff_vs_ours"] = max(diffs)
    rows, cols = sample_window(cfg)
    res["compared_window"] = f"outputs [:{rows}, :{cols}] of input set 0"
    return res


# --------------------------------------------------------------------------
def oracle_output(fname, h, cfg, precision):
    """The fp32 / fp64 C oracle's outputs of one function on host inputs `h`."""
    from oracle import oracle as orc

    tr = cfg["trunc"]
    trunc, boot = (h["trunc"], h["boot"]) if tr else (None, None)
    if fname == "gae":
        return (orc.gae(h["r"], h["v"], h["term"], trunc, boot, orc.BOOT_FULL_SEL if tr else orc.BOOT_NONE,
                        0.99, 0.95, precision),)
    if fname == "vtrace":
        return orc.vtrace(h["lpt"], h["lpb"], h["v"], h["r"], h["term"], trunc, boot,
                          orc.BOOT_FULL_ADD if tr else orc.BOOT_NONE, 0.99, 1.0, 1.0, precision)
    if fname == "retrace":
        return orc.retrace(h["pi"], h["mu"], h["q"], h["nq"], h["act"], h["r"], h["term"],
                           h["trunc"] if tr else h["notrunc"], 0.99, 0.95, 1.0, 1.0, precision)
    if fname == "lambda":
        return (orc.lambda_returns(h["r"], h["nv"], h["term"], trunc, boot, orc.BOOT_FULL_ADD if tr else orc.BOOT_NONE,
                                   0.99, 0.95, precision),)
    if fname == "discounted":
        return (orc.discounted_returns(h["r"], h["term"], trunc, boot, orc.BOOT_FULL_ADD if tr else orc.BOOT_NONE,
                                       0.99, precision),)
    if fname == "eligibility":
        return (orc.eligibility_traces(h["r"], h["term"], 0.99, 0.95, precision=precision),)
    return (orc.prefix_sum(h["r"], h["term"], precision=precision),)


def check_parity(cfg, x, calls, split, world, rank):
    """After the timed region: every output of input set 0 (all ranks' segments
    gathered when the sequence is split along time) against the fp32 C oracle
    at rtol = atol = 1e-5 (oracle.compare)."""
    from oracle import oracle as orc

    outs = {}
    for f, c in calls.items():
        outs.update({k: v for k, v in flat_outputs(f, c()).items()})
    torch.cuda.synchronize()
    xs = {k: v for k, v in x.items() if _used(k, cfg) or k == "notrunc"}
    if split:
        import torch.distributed as dist

        def gather(t):
            t = t.contiguous().view(-1)
            full = torch.empty(world * t.numel(), dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(full, t)
            return full.view(1, -1)

        xs = {k: gather(v) for k, v in xs.items()}
        outs = {k: gather(v) for k, v in outs.items()}
        cfg = dict(cfg, T=cfg["T"] * world)
    if rank != 0:
        return None
    h = to_numpy(xs)
    per = {}
    for f in cfg["funcs"]:
        for k in range(2 if f in ("vtrace", "retrace") else 1):
            key = f"{f}_{k}"
            got = outs[key].cpu().numpy()
            res = orc.compare(got, lambda p: oracle_output(f, h, cfg, p)[k])
            per[key] = {kk: (round(v, 9) if isinstance(v, float) else v) for kk, v in res.items()
                        if kk not in ("rtol", "atol")}
    return {"ok": all(r["ok"] for r in per.values()), "max_abs_err": max(r["max_abs_err"] for r in per.values()),
            "rtol": 1e-5, "atol": 1e-5,
            "checked": f"every output of input set 0 ({cfg['N']}x{cfg['T']}) against the fp32 C oracle",
            "per_output": per}


# --------------------------------------------------------------------------
def run_e2e(cfg, x0, dev, split, world, ksteps):
    """The same step through the public API from pinned host buffers: every step
    copies its inputs host->device and its outputs device->host.  Copies in,
    the calls and copies out run on three streams with two buffer sets, so step
    k+1's inputs travel while step k computes and step k-1's results return."""
    keys = [k for k in x0 if _used(k, cfg)]
    host = {k: x0[k].to("cpu").pin_memory() for k in keys}
    const = {k: v for k, v in x0.items() if k == "notrunc"}  # device constant, not per-step data
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    bufs = [{k: torch.empty_like(x0[k]) for k in keys} for _ in range(2)]
    cs, ks, ds = (torch.cuda.Stream(dev) for _ in range(3))
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    pinned = [None, None]
    keep = [None, None]  # step k's outputs stay referenced until their copy-out has run

    def step(k):
        b = k % 2
        with torch.cuda.stream(cs):
            if k >= 2:
                cs.wait_event(ev_free[b])  # step k-2 finished reading this buffer set
            for key in keys:
                bufs[b][key].copy_(host[key], non_blocking=True)
            ev_in[b].record(cs)
        with torch.cuda.stream(ks):
            ks.wait_event(ev_in[b])
            if keep[b] is not None:
                # Step k-2's outputs return to the allocator only once the
                # kernel stream has waited for their copy-out: their memory is
                # reused in stream order, with no cross-stream record (which
                # makes the caching allocator fall back to fresh cudaMalloc
                # calls, and those synchronise the device).
                ks.wait_event(ev_out[b])
                keep[b] = None
            res = []
            for f, c in make_calls(cfg, {**bufs[b], **const}, split).items():
                res.extend(flat_outputs(f, c()).values())
            ev_free[b].record(ks)
        with torch.cuda.stream(ds):
            ds.wait_event(ev_free[b])
            if pinned[b] is None:
                pinned[b] = [torch.empty(r.shape, dtype=r.dtype, pin_memory=True) for r in res]
            for o, r in zip(pinned[b], res):
                o.copy_(r, non_blocking=True)
            ev_out[b].record(ds)
        keep[b] = res
        return res

    for k in range(4):  # warm-up, allocates the pinned result buffers
        step(k)
    torch.cuda.synchronize(dev)
    d2h = sum(o.numel() * o.element_size() for o in pinned[0])
    barrier(world)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(cs)
    ks.wait_stream(cs)
    ds.wait_stream(cs)
    for k in range(ksteps):
        step(k)
    a1.record(ds)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(a0.elapsed_time(a1) / ksteps, world)
    # The copies alone (same buffers and streams, no calls): the floor of the step.
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(cs):
        c0.record(cs)
        for k in range(ksteps):
            for key in keys:
                bufs[k % 2][key].copy_(host[key], non_blocking=True)
        c1.record(cs)
    res0 = make_calls(cfg, {**bufs[0], **const}, split)
    outs = [o for f, c in res0.items() for o in flat_outputs(f, c()).values()]
    torch.cuda.synchronize(dev)
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(ds):
        d0.record(ds)
        for k in range(ksteps):
            for o, r in zip(pinned[k % 2], outs):
                o.copy_(r, non_blocking=True)
        d1.record(ds)
    torch.cuda.synchronize(dev)
    h2d_ms, d2h_ms = c0.elapsed_time(c1) / ksteps, d0.elapsed_time(d1) / ksteps
    return {"value": world * cfg["N"] * cfg["T"] / (ms / 1e3), "unit": "timesteps/s", "ms_per_step": ms,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "copies_alone_ms": {"h2d": round(h2d_ms, 4), "d2h": round(d2h_ms, 4),
                                "h2d_gbs": round(h2d / h2d_ms / 1e6, 1), "d2h_gbs": round(d2h / d2h_ms / 1e6, 1)},
            "path": "rl_triton public API; pinned host buffers; per step H2D of every input, the calls, D2H of "
                    "every output; copies in / calls / copies out on three streams, two buffer sets"}


def measure_step(cfg, split, world, rank, local, steps, warmup, no_graph=False, sets_override=0):
    """Time `steps` steps of a workload (each step = one call of each of its
    functions on one input set, replayed from a CUDA graph per input set)
    between a barrier + synchronize on both sides; CUDA events on the launching
    stream, max over ranks.  Returns the timing and what the later legs reuse."""
    dev = torch.device("cuda", local)
    N, T = cfg["N"], cfg["T"]
    n_sets, per_set = input_sets(cfg)
    if sets_override:
        n_sets = sets_override
    sets = [make_inputs(cfg, dev, seed=1000 * rank + k) for k in range(n_sets)]
    calls = [make_calls(cfg, x, split) for x in sets]
    stream = torch.cuda.Stream(dev)

    # Warm up on the capture stream (allocates this stream's workspace).
    with torch.cuda.stream(stream):
        for c in calls:
            for f in c.values():
                f()
    stream.synchronize()

    # The time-split path passes t0 / total, so it never synchronises the host
    # and its collective is captured with the kernels.
    use_graph = not no_graph
    graphs = []      # one step (one input set) per graph
    multi = []       # STEPS_PER_GRAPH consecutive steps per graph (small workloads)
    per_graph = STEPS_PER_GRAPH if (n_sets >= STEPS_PER_GRAPH and per_set < 1e9) else 1
    if use_graph:
        for c in calls:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for f in c.values():
                    f()
            graphs.append(g)
        if per_graph > 1:
            for j in range(n_sets // per_graph):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for c in calls[j * per_graph:(j + 1) * per_graph]:
                        for f in c.values():
                            f()
                multi.append(g)

    def run_steps(k0, count):
        """Steps k0 .. k0+count-1 (step k uses input set k mod n_sets); graphs
        of several consecutive steps where they line up, single steps else."""
        k, end = k0, k0 + count
        while k < end:
            if use_graph and multi and k + per_graph <= end and \
                    (k % n_sets) % per_graph == 0 and (k % n_sets) // per_graph < len(multi):
                multi[(k % n_sets) // per_graph].replay()
                k += per_graph
            elif use_graph:
                graphs[k % n_sets].replay()
                k += 1
            else:
                for f in calls[k % n_sets].values():
                    f()
                k += 1

    sampler = ClockSampler(local)
    sampler.start()
    with torch.cuda.stream(stream):
        run_steps(0, warmup)
    stream.synchronize()
    barrier(world)
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tw0 = time.perf_counter()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        run_steps(0, steps)
        ev1.record(stream)
    stream.synchronize()
    tw1 = time.perf_counter()
    sampler.stop()
    clocks = sampler.summary(tw0, tw1)
    barrier(world)
    torch.cuda.synchronize(dev)
    ms_total = max_over_ranks(ev0.elapsed_time(ev1), world)
    ms = ms_total / steps
    graphs.clear()
    multi.clear()
    return {"value": world * N * T / (ms / 1e3), "ms": ms, "steps_per_graph": per_graph, "sets": sets, "calls": calls, "stream": stream,
            "use_graph": use_graph, "clocks": clocks, "n_sets": n_sets, "per_set": per_set}


def run_sharded(args, world, rank, local):
    """The two multi-GPU partitions in the same run as the headline line:
    config 4 sharded along num_envs (weak: every rank its own 131072 x 1024) and
    config 5b split along time (strong: one 2^28-step sequence cut into W
    segments, one all-gather per call)."""
    out = {}
    for name in ("cfg4", "cfg5b"):
        cfg = CONFIGS[name]
        split = cfg.get("split", False) and world > 1
        if split:
            cfg = dict(cfg, T=cfg["T"] // world)
        try:
            m = measure_step(cfg, split, world, rank, local, max(3, min(args.steps, 20)), 3, args.no_graph)
            out[name] = {"workload": CONFIGS[name]["desc"], "value": m["value"], "unit": "timesteps/s",
                         "ms_per_step": m["ms"], "scaling": "strong" if name == "cfg5b" else "weak",
                         "partition": ("time-split" if split else "single GPU") if name == "cfg5b"
                         else ("env-sharded" if world > 1 else "single GPU"),
                         "num_envs_per_gpu": cfg["N"], "seq_len_per_gpu": cfg["T"],
                         "launch": "CUDA graph per input set" if m["use_graph"] else "eager",
                         "clocks": m["clocks"]}
            del m
        except Exception as e:  # noqa: BLE001
            out[name] = {"error": f"{type(e).__name__}: {str(e)[:300]}"}
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return out


def run_b200(args, world, rank, local):
    cfg = CONFIGS[args.config]
    split = world > 1 and cfg.get("split", False)
    if split:  # strong scaling: each rank holds T / world columns of the one sequence
        cfg = dict(cfg, T=cfg["T"] // world)
    dev = torch.device("cuda", local)
    from rl_triton import _native as nat

    N, T = cfg["N"], cfg["T"]
    m = measure_step(cfg, split, world, rank, local, args.steps, args.warmup, args.no_graph, args.sets)
    value, ms, sets, calls, stream, use_graph = m["value"], m["ms"], m["sets"], m["calls"], m["stream"], m["use_graph"]
    clocks, n_sets, per_set = m["clocks"], m["n_sets"], m["per_set"]

    # Per-function device time per launch and eager full-call time.
    per_fn = {}
    hbm, peak_kind = peaks()
    # Two sweeps over the functions; the second is reported (the first warms
    # every function's graph and input sets -- the first function timed in a
    # fresh process otherwise varied by up to 2x from run to run).
    sweeps = {}
    for sweep in range(2):
        for fname in cfg["funcs"]:
            sweeps[fname] = time_function(calls, fname, stream, use_graph, fixed_reps=8 if world > 1 else 0)
    for fname in cfg["funcs"]:
        t = sweeps[fname]
        us = t["us_per_launch"]
        alg = bytes_per_step(fname, cfg["trunc"], cfg["bf16"]) * N * T
        per_fn[fname] = {"us_per_launch": us, "full_call_us": t["full_call_us"], "algorithmic_bytes": alg,
                         "achieved_gbs": round(alg / (us * 1e-6) / 1e9, 1),
                         "frac": round(alg / (us * 1e-6) / 1e9 / hbm, 4)}
    rw = read_write_peaks(dev) if rank == 0 else None
    dom = max(per_fn, key=lambda f: per_fn[f]["us_per_launch"])
    d = per_fn[dom]
    traffic = read_traffic(dom, args.config)

    # The fused epilogues against the same work composed from separate calls.
    fused = None
    if not args.no_fused and not split and not cfg["trunc"] and "gae" in cfg["funcs"]:
        fused = time_fused(sets, stream, use_graph, world, hbm)

    # Parity of the timed path's outputs.
    parity = None if args.no_parity else check_parity(cfg, sets[0], calls[0], split, world, rank)

    # The reference's own Triton kernels on this GPU (child process).
    tri = None
    if rank == 0 and world == 1 and not args.no_triton:
        rows, cols = sample_window(cfg)
        ours = {}
        with torch.cuda.stream(stream):
            for f, c in calls[0].items():
                for key, t in flat_outputs(f, c()).items():
                    ours[key] = t[:rows, :cols].float().cpu().numpy()
        tri = triton_reference(args, cfg, ours, per_fn, local)

    sharded = None
    if not args.no_sharded and args.config == "cfg2":
        sharded = run_sharded(args, world, rank, local)

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(cfg, sets[0], dev, split, world, max(3, min(args.steps, 20)))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        ts, cores, sample = cpu_sample(cfg)
        cpu = {"value": ts, "unit": "timesteps/s", "cores": cores, "kind": "port",
               "sample": sample + "; oracle/rlscan_oracle.c (CPU restatement of the reference's sequential "
                                  "estimators), rows split over host threads"}

    n_launch = launches_per_step(calls[0], stream)
    n_launch = n_launch * args.steps if n_launch is not None else len(cfg["funcs"]) * args.steps
    if rank == 0:
        line = {
            "metric": "timesteps/sec", "value": value, "unit": "timesteps/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if split else "weak", "vs_baseline": None,
            "dtype": "bf16->f32" if cfg["bf16"] else "f32",
            "data": "synthetic (seeded torch.Generator; distributions of the headline configurations)",
            "config": config_dict(cfg, world, split, n_sets, per_set, use_graph),
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": d["achieved_gbs"], "peak": hbm,
                         "unit": "GB/s", "frac": d["frac"], "traffic": traffic,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6650 GB/s",
                         "context": rw},
            "per_function": per_fn,
            "fused": fused,
            "parity": parity,
            "triton_reference": tri,
            "clocks": clocks,
            "e2e": e2e,
            "sharded": sharded,
            "cpu_baseline": cpu,
            "gpu_launches": n_launch,
            "lib": nat.build_info(),
        }
        print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# PPO-step harness: the estimators' share of a whole PPO update.
PPO = dict(N=4096, T=128, obs_dim=64, act_dim=4, hidden=256, epochs=4, minibatches=4, clip=0.2, lr=3e-4)


def _ppo_net(dev):
    torch.manual_seed(0)
    net = torch.nn.ModuleDict({
        "body": torch.nn.Sequential(torch.nn.Linear(PPO["obs_dim"], PPO["hidden"]), torch.nn.Tanh(),
                                    torch.nn.Linear(PPO["hidden"], PPO["hidden"]), torch.nn.Tanh()),
        "pi": torch.nn.Linear(PPO["hidden"], PPO["act_dim"]),
        "v": torch.nn.Linear(PPO["hidden"], 1),
    }).to(dev)
    log_std = torch.zeros(PPO["act_dim"], device=dev, requires_grad=True)
    return net, log_std


def _ppo_rollout(dev, seed):
    """bf16 rollout buffers of a continuous-action task (seeded synthetic data)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    n, t = PPO["N"], PPO["T"]
    return dict(obs=torch.randn(n, t, PPO["obs_dim"], generator=g, device=dev).to(torch.bfloat16),
                act=torch.randn(n, t, PPO["act_dim"], generator=g, device=dev).to(torch.bfloat16),
                old_logp=(-torch.rand(n, t, generator=g, device=dev) * 4).to(torch.bfloat16),
                rew=torch.randn(n, t, generator=g, device=dev).to(torch.bfloat16),
                done=(torch.rand(n, t, generator=g, device=dev) < 0.01).to(torch.bfloat16))


def ppo_update(net, log_std, opt, ro, estimator, ev=None):
    """One PPO update: values of the rollout, the estimator (GAE, advantage
    normalisation, returns), then epochs x minibatches of clipped-surrogate +
    value loss, backward and Adam.  `ev` = (start, end) events around the
    estimator."""
    import rl_triton

    n, t = PPO["N"], PPO["T"]
    flat_obs = ro["obs"].reshape(n * t, -1)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        values = net["v"](net["body"](flat_obs)).reshape(n, t)
    if ev:
        ev[0].record()
    if estimator == "fused":
        adv, ret = rl_triton.compute_gae_normalized(ro["rew"], values, ro["done"], gamma=0.99, lambda_=0.95,
                                                    return_returns=True)
    else:
        a = rl_triton.compute_gae(ro["rew"], values, ro["done"], gamma=0.99, lambda_=0.95)
        ret = a + values.float()
        adv = (a - a.mean()) / (a.std() + 1e-8)
    if ev:
        ev[1].record()
    adv, ret = adv.reshape(-1), ret.reshape(-1)
    act = ro["act"].reshape(n * t, -1).float()
    old_logp = ro["old_logp"].reshape(-1).float()
    mb = n * t // PPO["minibatches"]
    for _ in range(PPO["epochs"]):
        perm = torch.randperm(n * t, device=adv.device)
        for k in range(PPO["minibatches"]):
            idx = perm[k * mb:(k + 1) * mb]
            with torch.autocast("cuda", dtype=torch.bfloat16):
                h = net["body"](flat_obs[idx])
                mean, v = net["pi"](h).float(), net["v"](h).float().squeeze(-1)
            logp = (-0.5 * ((act[idx] - mean) / log_std.exp()) ** 2 - log_std).sum(-1)
            ratio = (logp - old_logp[idx]).exp()
            surr = torch.min(ratio * adv[idx], ratio.clamp(1 - PPO["clip"], 1 + PPO["clip"]) * adv[idx])
            loss = -surr.mean() + 0.5 * ((v - ret[idx]) ** 2).mean()
            opt.zero_grad(set_to_none=True)
            loss.backward()
            opt.step()


def run_ppo(args, local):
    """`--config ppo`: PPO updates on 4096 x 128 bf16 rollouts; the estimator
    is the fused normalising GAE (`fused`) or GAE + PyTorch normalisation
    (`unfused`).  Reports update throughput and the estimator's share."""
    dev = torch.device("cuda", local)
    ro = _ppo_rollout(dev, 0)
    arms = {}
    for est in ("fused", "unfused"):
        net, log_std = _ppo_net(dev)
        opt = torch.optim.Adam(list(net.parameters()) + [log_std], lr=PPO["lr"])
        for _ in range(args.warmup):
            ppo_update(net, log_std, opt, ro, est)
        arms[est] = (net, log_std, opt, [], [])
    torch.cuda.synchronize(dev)
    for k in range(args.steps):  # the arms alternate, in alternating order
        for est in (("fused", "unfused") if k % 2 == 0 else ("unfused", "fused")):
            net, log_std, opt, tot, est_ms = arms[est]
            e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            e[0].record()
            ppo_update(net, log_std, opt, ro, est, ev=(e[1], e[2]))
            e[3].record()
            torch.cuda.synchronize(dev)
            tot.append(e[0].elapsed_time(e[3]))
            est_ms.append(e[1].elapsed_time(e[2]))
    res = {}
    for est, (_, _, _, tot, est_ms) in arms.items():
        t_ms, e_ms = statistics.median(tot), statistics.median(est_ms)
        res[est] = {"ms_per_update": round(t_ms, 4), "estimator_ms": round(e_ms, 4),
                    "estimator_share": round(e_ms / t_ms, 4)}
    n, t = PPO["N"], PPO["T"]
    line = {"metric": "timesteps/sec", "value": n * t / (res["fused"]["ms_per_update"] / 1e3), "unit": "timesteps/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["fused"]["ms_per_update"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 rollout buffers, fp32 estimator arithmetic",
            "data": "synthetic (seeded torch.Generator)",
            "config": {"workload": "PPO update: 4096 x 128 bf16 rollout, MLP 64-256-256 policy/value, "
                                   f"{PPO['epochs']} epochs x {PPO['minibatches']} minibatches, Adam",
                       "timing": "CUDA events around each eager update (median) and around the estimator"},
            "ppo": res,
            "estimator_speedup_fused_vs_unfused": round(res["unfused"]["estimator_ms"] / res["fused"]["estimator_ms"], 3)}
    print(json.dumps(line), flush=True)


def run_ncu(args, local):
    cfg = CONFIGS[args.config]
    if args.envs:
        cfg = dict(cfg, N=args.envs)
    if args.len:
        cfg = dict(cfg, T=args.len)
    dev = torch.device("cuda", local)
    x = make_inputs(cfg, dev, seed=1)
    calls = make_calls(cfg, x)
    torch.cuda.synchronize(dev)
    for _ in range(args.warmup + args.steps):
        for f in calls.values():
            f()
    torch.cuda.synchronize(dev)


def launches_per_step(calls, stream):
    """Kernels of this library launched by one eager step, counted by the CUDA
    profiler in an untimed pass (library kernels live in namespace rls or are
    the epoch / segment helpers; PyTorch's own kernels and copies are not
    counted).  None when the profiler is unavailable."""
    try:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            with torch.cuda.stream(stream):
                for f in calls.values():
                    f()
            stream.synchronize()
        names = [e.name for e in prof.events() if e.device_type.name == "CUDA"]
        ours = [n for n in names if "at::" not in n and not n.startswith(("Memcpy", "Memset", "nccl", "ncclDevKernel"))
                and ("rls::" in n or "advance_epoch" in n or "vrows_" in n or "segment_walk" in n or "_kernel" in n)]
        return len(ours) or None
    except Exception:  # noqa: BLE001
        return None


def _used(key, cfg):
    fs = cfg["funcs"]
    need = {"r", "term"}
    if any(f in fs for f in ("gae", "vtrace", "lambda", "retrace")):
        need |= {"v"}
    if "vtrace" in fs:
        need |= {"lpt", "lpb"}
    if "lambda" in fs:
        need |= {"nv"}
    if cfg["trunc"]:
        need |= {"trunc", "boot", "nv"}
    if "retrace" in fs:
        need |= {"pi", "act", "mu", "q", "nq"}
    return key in need


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS) + ["ppo"])
    ap.add_argument("--sets", type=int, default=0, help="input sets to rotate (default: enough to exceed L2)")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--ncu", action="store_true",
                    help="profiling mode for ncu: W warm-up rounds then K rounds of one eager launch per "
                         "function, in --config order; no timing, no graphs, prints nothing")
    ap.add_argument("--only", default="", help="comma list of functions to run (default: all of the config)")
    ap.add_argument("--envs", type=int, default=0, help="--ncu mode: override num_envs (a smaller slice to profile)")
    ap.add_argument("--len", type=int, default=0, help="--ncu mode: override the sequence length T")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check of the timed outputs")
    ap.add_argument("--no-triton", action="store_true", help="skip timing the reference's Triton kernels")
    ap.add_argument("--no-fused", action="store_true", help="skip the fused-epilogue comparison")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the config 4 (env-sharded) and 5b (time-split) legs of the default run")
    ap.add_argument("--triton-worker", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--device", type=int, default=0, help=argparse.SUPPRESS)
    ap.add_argument("--triton-out", default="", help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.triton_worker:
        triton_worker(args)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        # CPU arm: no process group; under torchrun rank 0 alone runs and prints.
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    if args.only:
        for name in CONFIGS:
            CONFIGS[name] = dict(CONFIGS[name], funcs=[f for f in CONFIGS[name]["funcs"] if f in args.only.split(",")])
    world, rank, local = dist_setup()
    try:
        if args.ncu:
            run_ncu(args, local)
            return
        if args.config == "ppo":
            run_ppo(args, local)
            return
        run_b200(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
