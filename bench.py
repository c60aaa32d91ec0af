"""Benchmark of the selectssm selective-scan hot path on B200.

Metric: scan fwd+bwd tokens*channels/s and % of the HBM roofline
at 1/2/4/8 B200.  Headline workload at every N: config 5 of the benchmark
contract, the raw selective-scan op forward + backward (softplus(dt) preamble,
D skip and silu(z) gate fused) on batch=64, L=2048, d_inner=1536, N=16 with
bf16 I/O and fp32 state, the batch split over the N ranks (strong scaling: the
total problem is fixed).  Synthetic seeded inputs with config 2's distributions
(u, z ~ N(0,1); dt_raw ~ N(0,1) - 4; A = -U[1,16]; B, C ~ N(0,1);
D ~ N(1, 0.1); upstream grad ~ N(0,1)).  One step = one forward + one backward.
At N=1 the line also carries config 2 (batch=8, L=4096, float32) under
"config2".  Multi-GPU: one process per GPU (torchrun), no collective in the
forward, one NCCL all-reduce of dA / dD per backward, overlapped with the next
forward.  --parallel channels splits d_inner instead (config 4 with
--workload 4) and sums dB / dC over the ranks.

`--impl reference` times the reference algorithm on the host CPU instead: the
NumPy restatement of ssm_chunked_scan (forward) and of the ssm_scan custom-VJP
backward from oracle/, on a bounded sample of the same workload (JAX, the
reference's own runtime, is not installed on this image).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(batch=8, seqlen=4096, dim=1536, dstate=16)
METRIC = "scan fwd+bwd tokens*channels/s (and % HBM roofline)"
UNIT = "tokens*channels/s"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def alg_bytes(units, s, N, D):
    """Algorithmic HBM bytes: forward reads u, dt, z and writes y (4s per unit);
    backward reads u, dt, z, dy and writes du, ddt, dz (7s); B and C are read by
    both and dB, dC written (6 s N per (b,l), amortised over D channels)."""
    fwd = units * (4 * s + 2 * s * N / D)
    bwd = units * (7 * s + 4 * s * N / D)
    return fwd, bwd


def read_profile(name, key="traffic_bytes_per_launch"):
    """A per-launch figure recorded in a committed ncu summary (DRAM bytes by
    default, or warp_instructions_per_launch), else None."""
    p = os.path.join(ROOT, "profiles", name)
    try:
        with open(p) as f:
            for line in f:
                if line.startswith(key + ":"):
                    return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


def read_traffic(name):
    return read_profile(name)


SMS, SMSPS_PER_SM, MUFU_PER_SM_CLK = 148, 4, 16


def compute_floor(ms, units, mufu_per_unit, profile, mhz):
    """The kernel's compute-side floors at the sampled SM clock: special-function
    (MUFU) operations at 16 per SM per clock, and warp instructions (from the
    committed ncu count of the same launch) at one issue per scheduler per
    clock.  The fractions say how close the call runs to each."""
    hz = (mhz or 1965.0) * 1e6
    mufu_ms = units * mufu_per_unit / (SMS * MUFU_PER_SM_CLK * hz) * 1e3
    out = {"sm_mhz": mhz, "mufu_ops_per_unit": mufu_per_unit, "mufu_floor_ms": mufu_ms, "frac_of_mufu_floor": mufu_ms / ms}
    inst = read_profile(profile, "warp_instructions_per_launch")
    if inst:
        issue_ms = inst / (SMS * SMSPS_PER_SM * hz) * 1e3
        out.update({"warp_instructions": inst, "issue_floor_ms": issue_ms, "frac_of_issue_floor": issue_ms / ms})
    return out


class ClockSampler:
    """SM clock and throttle-reason samples taken in-process through NVML
    (read-only queries) every 5 ms while the timed region runs, so even a
    region of a few tens of milliseconds gets samples.  Falls back to an
    nvidia-smi poller (200 ms) when NVML cannot be loaded."""

    PERIOD_S = 0.005
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []  # (sm_mhz, max_mhz, set of active reason names)
        self.stop = threading.Event()
        self.thread = None
        self.proc = None
        self.nvml = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:  # the CUDA ordinal and NVML's index differ under CUDA_VISIBLE_DEVICES: match by PCI bus id
            import torch
            pr = torch.cuda.get_device_properties(self.index)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        bits = {"hw_slowdown": pynvml.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": pynvml.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": pynvml.nvmlClocksEventReasonSwPowerCap}
        mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        return pynvml, h, bits, mx

    def _poll_nvml(self):
        nv, h, bits, mx = self.nvml
        while not self.stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.rows.append((float(sm), float(mx), {n for n, bit in bits.items() if r & bit}))
            except Exception:
                pass
            self.stop.wait(self.PERIOD_S)

    def _read_smi(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 7 and parts[0].replace(".", "").isdigit():
                self.rows.append((float(parts[0]), float(parts[1]),
                                  {n for n, v in zip(self.NAMES, parts[3:7]) if v.lower() == "active"}))

    def __enter__(self):
        try:
            self.nvml = self._nvml_handle()
            self.thread = threading.Thread(target=self._poll_nvml, daemon=True)
        except Exception:
            self.nvml = None
            fields = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                      "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                      "clocks_event_reasons.sw_power_cap")
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={self.index}", f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                     "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.thread = threading.Thread(target=self._read_smi, daemon=True)
            except OSError:
                self.thread = None
        if self.thread:
            self.thread.start()
        return self

    def wait_first(self, timeout=3.0):
        t0 = time.time()
        while self.thread and not self.rows and time.time() - t0 < timeout:
            time.sleep(0.002)
        self.rows.clear()  # keep only samples taken during the timed region

    def __exit__(self, *a):
        self.stop.set()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=5)

    def summary(self):
        rows = list(self.rows)
        src = "nvml" if self.nvml else "nvidia-smi"
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0, "source": src}
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted(set().union(*(r[2] for r in rows))), "samples": len(rows), "source": src,
                "period_ms": self.PERIOD_S * 1e3 if self.nvml else 200}


# ----------------------------------------------------------------------------- inputs
def host_inputs(seed, B, L, D, N, bc_seed=None):
    """Seeded float32 host inputs of config 2 (one generator per tensor).
    bc_seed draws B and C from another seed (shared by channel shards)."""
    ss = np.random.SeedSequence(seed).spawn(8)
    g = [np.random.default_rng(s) for s in ss]
    if bc_seed is not None:
        sb = np.random.SeedSequence(bc_seed).spawn(8)
        g[4], g[5] = np.random.default_rng(sb[4]), np.random.default_rng(sb[5])
    f32 = np.float32
    return dict(
        u=g[0].standard_normal((B, L, D), dtype=f32),
        z=g[1].standard_normal((B, L, D), dtype=f32),
        delta=(g[2].standard_normal((B, L, D), dtype=f32) - f32(4.0)),
        A=(-g[3].uniform(1.0, 16.0, size=(D, N))).astype(f32),
        B=g[4].standard_normal((B, L, N), dtype=f32),
        C=g[5].standard_normal((B, L, N), dtype=f32),
        D=(1.0 + 0.1 * g[6].standard_normal(D)).astype(f32),
        dout=g[7].standard_normal((B, L, D), dtype=f32),
    )


# ----------------------------------------------------------------------------- CPU arm
def cpu_reference_step(inp, chunk_size=None):
    """One fwd+bwd of the fused op with the restated reference algorithm:
    ssm_chunked_scan forward (selectssm.py:37-109) and the ssm_scan custom-VJP
    backward (ssmrecscan.py:111-181, default min_recursion_length=2)."""
    from oracle import selectssm_oracle as O
    u, delta, z, dout = inp["u"], inp["delta"], inp["z"], inp["dout"]
    A, Bm, Cm, Dv = inp["A"], inp["B"], inp["C"], inp["D"]
    dt = O.softplus(delta)
    ys = O.ssm_chunked_scan(u, A, Bm, Cm, dt, chunk_size)
    pre = ys + u * Dv
    g = O.activation(z, "silu")
    out = pre * g
    dpre = dout * g
    dz = dout * pre * O.activation_grad(z, "silu")
    dx, dA, dB, dC, ddt = O.ssm_scan_backward(u, A, Bm, Cm, dt, dpre)
    du = dx + dpre * Dv
    dD = np.einsum("bld,bld->d", dpre, u)
    ddelta = ddt * O.sigmoid(delta)
    return out, du, ddelta, dz, dA, dB, dC, dD


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


_SAMPLE_INP = {}


def _one_thread():
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(1)
    except Exception:
        pass


def _run_shard(span):
    """Oracle fwd+bwd on channels [s, e) of the shared sample (B and C are
    shared by all channels; each channel's scan is independent)."""
    s, e = span
    inp = _SAMPLE_INP
    sub = {k: (v[..., s:e] if k in ("u", "delta", "z", "dout") else v[s:e] if k in ("A", "D") else v)
           for k, v in inp.items()}
    cpu_reference_step(sub)
    return e - s


class CpuSampler:
    """Times the NumPy restatement of the reference algorithm on all host
    cores: the channels of one fixed sample of the workload are split over one
    single-threaded process per core (the reference's JAX-on-CPU would also use
    every core).  The workers are forked after the sample is drawn, so they
    share it.  The sample is float32 (for a bf16 workload the oracle computes
    in float32 on the same distributions)."""

    def __init__(self, spec, seqlen, batch=1):
        import multiprocessing as mp
        global _SAMPLE_INP
        D, N = spec["dim"], CFG["dstate"]
        _SAMPLE_INP = host_inputs(0, batch, seqlen, D, N)
        self.procs = cpu_cores()
        k = self.procs
        self.spans = [(D * i // k, D * (i + 1) // k) for i in range(k)]
        self.units = batch * seqlen * D
        self.sample = (f"NumPy restatement of the reference algorithm (chunked scan fwd + custom-VJP bwd, float32) "
                       f"on batch={batch}, L={seqlen}, d_inner={D}, N={N} of the {spec['key']} workload, channels "
                       f"split over {k} single-threaded processes (one per host core), after one warm-up run")
        self.pool = mp.get_context("fork").Pool(k, initializer=_one_thread)
        self.pool.map(_run_shard, self.spans)  # warm-up (imports, page faults)

    def run(self):
        t0 = time.perf_counter()
        self.pool.map(_run_shard, self.spans)
        dt = time.perf_counter() - t0
        return self.units / dt, dt, self.sample

    def close(self):
        self.pool.close()
        self.pool.join()


def run_cpu_sample(spec, seqlen, batch=1):
    sampler = CpuSampler(spec, seqlen, batch)
    try:
        return sampler.run()
    finally:
        sampler.close()


# ----------------------------------------------------------------------------- other workloads
OTHER = {
    3: dict(workload="config 3: BidirectionalMamba scan pair, complement + tied gate + concat, bf16 I/O, "
                     "fp32 state", batch=2, seqlen=131072, dim=512, dtype="bf16", bidir=True),
    4: dict(workload="config 4: long-sequence raw op fwd+bwd (recursive-scan semantics), fp32",
            batch=1, seqlen=1 << 20, dim=1024, dtype="f32", bidir=False),
    5: dict(workload="config 5: raw op fwd+bwd, bf16 I/O, fp32 state", batch=64, seqlen=2048, dim=1536,
            dtype="bf16", bidir=False),
}


def run_other_config(args):
    """Device-resident fwd+bwd timing of configs 3-5 (seeded on the device with
    the configs' distributions), with the same event, warm-up and clock rules as
    the config-2 line.  Algorithmic bytes per unit: 11 s + 6 s N / D, where a
    unit is one (b, l, d) per direction; config 3's tied z is read once for
    both directions, so 9.5 s + 6 s N / D there."""
    import torch
    import selectssm_b200 as S
    from selectssm_b200 import _lib

    c = OTHER[args.config]
    Bsz, L, D, N = c["batch"], c["seqlen"], c["dim"], 16
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    dt = torch.bfloat16 if c["dtype"] == "bf16" else torch.float32
    g = torch.Generator(device=dev).manual_seed(args.config)

    def draw():
        n = lambda *s: torch.randn(*s, generator=g, device=dev)  # noqa: E731
        t = {"u": n(Bsz, L, D).to(dt), "delta": (n(Bsz, L, D) - 4.0).to(dt), "B": n(Bsz, L, N).to(dt),
             "C": n(Bsz, L, N).to(dt), "A": -(1.0 + 15.0 * torch.rand(D, N, generator=g, device=dev)),
             "D": 1.0 + 0.1 * n(D), "bias": 0.1 * n(D)}
        return {k: v.requires_grad_() for k, v in t.items()}

    dirs = 2 if c["bidir"] else 1
    fwd_in = draw()
    rev_in = draw() if c["bidir"] else None
    z = torch.randn(Bsz, L, D, generator=g, device=dev).to(dt).requires_grad_()
    dout = torch.randn(Bsz, L, dirs * D, generator=g, device=dev).to(dt)
    names = ("u", "delta", "A", "B", "C", "D", "bias")

    def step(marks=None):
        for t in (fwd_in, rev_in, {"z": z}):
            for v in (t or {}).values():
                v.grad = None
        if marks:
            marks[0].record()
        if c["bidir"]:
            out = S.selective_scan_bidir(*(fwd_in[k] for k in names), z, *(rev_in[k] for k in names), z,
                                         complement=True)
        else:
            f = fwd_in
            out = S.selective_scan(f["u"], f["delta"], f["A"], f["B"], f["C"], D=f["D"], z=z,
                                   delta_bias=f["bias"], delta_softplus=True)
        if marks:
            marks[1].record()
        out.backward(dout)
        if marks:
            marks[2].record()

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        clk.wait_first()
        n0 = lib.ssm_launch_count()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        n_launches = lib.ssm_launch_count() - n0
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    split = []  # per-call forward / backward times, calls queued back to back
    for _ in range(5):
        m = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        step(m)
        split.append(m)
    torch.cuda.synchronize()
    t_fwd = statistics.median(m[0].elapsed_time(m[1]) for m in split[1:])
    t_bwd = statistics.median(m[1].elapsed_time(m[2]) for m in split[1:])
    units = Bsz * L * D * dirs
    s = 2 if dt == torch.bfloat16 else 4
    per_unit = (9.5 if c["bidir"] else 11.0) * s + 6 * s * N / D
    hbm, src = peaks()
    achieved = units * per_unit / (ms * 1e-3) / 1e9
    line = {"metric": METRIC, "value": units / (ms * 1e-3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": c["dtype"], "data": "synthetic",
            "config": {"workload": c["workload"], "batch_per_gpu": Bsz, "seq_len": L, "d_inner": D, "d_state": N,
                       "directions": dirs, "parallelism": "single GPU",
                       "l2": "inputs larger than L2, no flush"},
            "roofline_step": {"bound": "hbm", "achieved": achieved, "peak": hbm, "peak_source": src, "unit": "GB/s",
                              "frac": achieved / hbm, "bytes_per_unit": per_unit},
            "ms_fwd_call": t_fwd, "ms_bwd_call": t_bwd,
            "e2e": None, "gpu_launches": n_launches, "clocks": clk.summary(),
            "library": lib.ssm_version().decode()}
    print(json.dumps(line))


# ----------------------------------------------------------------------------- GPU arm
# Workloads of the GPU arm.  The headline (every N) is config 5, the contract's
# scaling workload: the batch of 64 sequences is split over the N ranks, so the
# total problem is fixed (strong scaling).  At N=1 the line also carries config
# 2 (the raw op in float32) under "config2".  With --parallel channels the
# d_inner channels are split instead (config 4: 8 x 128 channels), B and C are
# replicated and dB / dC are summed over the ranks.
SPECS = {
    5: dict(key="config5", workload="config 5: raw selective-scan op fwd+bwd (softplus dt, D skip, silu gate "
                                    "fused), bf16 I/O, fp32 state", batch=64, seqlen=2048, dim=1536, dtype="bf16"),
    2: dict(key="config2", workload="config 2: raw selective-scan op fwd+bwd (softplus dt, D skip, silu gate "
                                    "fused), fp32", batch=8, seqlen=4096, dim=1536, dtype="f32"),
    4: dict(key="config4", workload="config 4: long-sequence raw op fwd+bwd (recursive-scan semantics), fp32",
            batch=1, seqlen=1 << 20, dim=1024, dtype="f32"),
}


def device_inputs(spec, batch, dim, seed, bc_seed, dev):
    """Seeded inputs on the device with config 2's distributions (u, z ~ N(0,1);
    dt_raw ~ N(0,1) - 4; A = -U[1,16]; B, C ~ N(0,1); D ~ N(1, 0.1); upstream
    grad ~ N(0,1)), in the workload's dtype.  B and C come from bc_seed (shared
    by channel shards)."""
    import torch
    dt = torch.bfloat16 if spec["dtype"] == "bf16" else torch.float32
    L, N = spec["seqlen"], CFG["dstate"]
    g = torch.Generator(device=dev).manual_seed(seed)
    gb = torch.Generator(device=dev).manual_seed(bc_seed)
    n = lambda gen, *s: torch.randn(*s, generator=gen, device=dev)  # noqa: E731
    t = {"u": n(g, batch, L, dim).to(dt), "delta": (n(g, batch, L, dim) - 4.0).to(dt), "z": n(g, batch, L, dim).to(dt),
         "A": -(1.0 + 15.0 * torch.rand(dim, N, generator=g, device=dev)),
         "B": n(gb, batch, L, N).to(dt), "C": n(gb, batch, L, N).to(dt),
         "D": 1.0 + 0.1 * n(g, dim), "dout": n(g, batch, L, dim).to(dt)}
    return t


GRAD_KEYS = ("u", "delta", "z", "A", "B", "C", "D")


def measure(spec, args, world, rank, dev, lib, chan=False, bc_sum_mode="multicast", e2e=True):
    """Times one workload on this rank: `steps` fwd+bwd steps device-resident
    (CUDA events, max over ranks), the per-call forward / backward split, and
    the same steps end to end from pinned host buffers.  Returns the fields of
    the JSON line."""
    import torch
    import torch.distributed as dist
    import selectssm_b200 as S
    from selectssm_b200.parallel import MulticastBCSum, allreduce_grads, replicated_bc

    N = CFG["dstate"]
    L = spec["seqlen"]
    if chan:
        Bsz, D = spec["batch"], spec["dim"] // world
    else:
        Bsz, D = spec["batch"] // world, spec["dim"]
    if args.batch:
        Bsz = args.batch
    t = device_inputs(spec, Bsz, D, 1234 + rank, 1234 if chan else 1234 + rank, dev)
    for k in GRAD_KEYS:
        t[k].requires_grad_(True)
    s = t["u"].element_size()
    pending = []
    bcs = None
    if chan and bc_sum_mode == "multicast":
        bcs = MulticastBCSum(Bsz, L, device=dev)
        if not bcs.available:
            bcs = None

    def finish_reduce():
        while pending:
            pending.pop().wait()

    def step(inputs):
        for k in GRAD_KEYS:
            inputs[k].grad = None
        Bm, Cm = inputs["B"], inputs["C"]
        if chan and bcs is None:  # dB / dC summed over the channel shards by NCCL after the backward
            Bm, Cm = replicated_bc(Bm, Cm)
        out = S.selective_scan(inputs["u"], inputs["delta"], inputs["A"], Bm, Cm, D=inputs["D"], z=inputs["z"],
                               delta_softplus=True, bc_sum=bcs)
        out.backward(inputs["dout"])
        if world > 1 and not chan:  # batch sharding: one all-reduce of the parameter gradients,
            finish_reduce()            # overlapped with the next step's forward
            pending.append(allreduce_grads([inputs["A"], inputs["D"]], async_op=True))
        return out

    for _ in range(max(3, args.warmup)):
        step(t)
    finish_reduce()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clk:
        clk.wait_first()
        n_launch0 = lib.ssm_launch_count()
        e0.record(stream)
        for _ in range(args.steps):
            step(t)
        finish_reduce()
        e1.record(stream)
        n_launches = lib.ssm_launch_count() - n_launch0
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        mt = torch.tensor([ms], device=dev)
        dist.all_reduce(mt, op=dist.ReduceOp.MAX)
        ms = float(mt.item())
        dist.barrier()
    units = Bsz * L * D  # per rank
    value = units * world / (ms * 1e-3)

    # per-call forward / backward times, calls queued back to back as in training
    marks = []
    torch.cuda.synchronize()
    for _ in range(8):
        a = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        for k in GRAD_KEYS:
            t[k].grad = None
        a[0].record(stream)
        out = S.selective_scan(t["u"], t["delta"], t["A"], t["B"], t["C"], D=t["D"], z=t["z"], delta_softplus=True,
                               bc_sum=bcs)
        a[1].record(stream)
        out.backward(t["dout"])
        a[2].record(stream)
        marks.append(a)
    torch.cuda.synchronize()
    t_fwd = statistics.median(a[0].elapsed_time(a[1]) for a in marks[1:])
    t_bwd = statistics.median(a[1].elapsed_time(a[2]) for a in marks[1:])
    hbm, src = peaks()
    fb, bb = alg_bytes(units, s, N, D)
    roof_bwd = {"kernel": "ssm_bwd call: ssm_bwd_kernel (decoupled-lookback segments) + finalize_kernel",
                "bound": "hbm", "achieved": bb / (t_bwd * 1e-3) / 1e9, "peak": hbm, "peak_source": src,
                "unit": "GB/s", "traffic": read_traffic(f"ssm_bwd_kernel_{spec['key']}.md"),
                "algorithmic_bytes": bb, "ms": t_bwd}
    roof_bwd["frac"] = roof_bwd["achieved"] / hbm
    # the library's rule for its one-lane-per-channel forward (single direction, whole tiles and chunks)
    lane = Bsz * D >= 65536 and L % 16 == 0 and D % 128 == 0
    fwd_kernel = "ssm_fwd_lane_kernel" if lane else "ssm_fwd_kernel"
    roof_fwd = {"kernel": f"ssm_fwd call: {fwd_kernel}" + (" (+ widen_bc_kernel for bf16 B/C)" if s == 2 else ""),
                "bound": "hbm",
                "achieved": fb / (t_fwd * 1e-3) / 1e9, "peak": hbm, "peak_source": src, "unit": "GB/s",
                "traffic": read_traffic(f"{fwd_kernel}_{spec['key']}.md"), "algorithmic_bytes": fb, "ms": t_fwd}
    roof_fwd["frac"] = roof_fwd["achieved"] / hbm
    # MUFU operations per unit: 16 state exponentials, softplus (ex2, lg2) and the silu gate (ex2, rcp) in the
    # forward; the backward adds softplus' derivative (rcp) and recomputes the same 16 exponentials.
    mhz = clk.summary().get("sm_mhz")
    roof_fwd["compute"] = compute_floor(t_fwd, units, 20, f"{fwd_kernel}_{spec['key']}.md", mhz)
    roof_bwd["compute"] = compute_floor(t_bwd, units, 21, f"ssm_bwd_kernel_{spec['key']}.md", mhz)
    step_roof = {"achieved": (fb + bb) / (ms * 1e-3) / 1e9, "peak": hbm, "peak_source": src, "unit": "GB/s",
                 "bytes_per_unit": (fb + bb) / units}
    step_roof["frac"] = step_roof["achieved"] / hbm
    res = {"value": value, "ms_per_step": ms, "units_per_rank": units, "batch_per_gpu": Bsz, "d_inner_per_gpu": D,
           "roofline": roof_bwd, "roofline_fwd": roof_fwd, "roofline_step": step_roof,
           "gpu_launches": n_launches, "clocks": clk.summary(), "dtype": spec["dtype"]}
    if e2e:
        res["e2e"] = measure_e2e(t, step, stream, world, args, units, dev, finish_reduce)
    return res


def measure_e2e(t, step, stream, world, args, units, dev, finish_reduce):
    """The same steps through the public API with host buffers: every step
    uploads its inputs from pinned host memory and downloads the output and
    all gradients to pinned host memory, inside the timed region.  Pipelined
    over steps on two copy streams (upload of step i+1 and download of step i-1
    overlap the compute of step i)."""
    import torch
    import torch.distributed as dist
    pin = {k: v.detach().cpu().pin_memory() for k, v in t.items()}
    h2d = sum(v.numel() * v.element_size() for v in pin.values())
    slots = [{k: torch.empty(v.shape, dtype=v.dtype, device=dev).requires_grad_(k in GRAD_KEYS)
              for k, v in pin.items()} for _ in range(2)]
    copy_in, copy_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    outs_host = [None, None]

    def upload(s):
        copy_in.wait_event(ev_done[s])  # the slot's previous step has finished reading it
        with torch.cuda.stream(copy_in), torch.no_grad():
            for k, v in pin.items():
                slots[s][k].copy_(v, non_blocking=True)
        ev_in[s].record(copy_in)

    def run(i):
        s = i % 2
        stream.wait_event(ev_in[s])
        out = step(slots[s])
        res = [out.detach()] + [slots[s][k].grad for k in GRAD_KEYS]
        ev_done[s].record(stream)
        if outs_host[s] is None:  # pinned result buffers, allocated before the timed region
            outs_host[s] = [torch.empty(r.shape, dtype=r.dtype, pin_memory=True) for r in res]
        copy_out.wait_event(ev_done[s])
        with torch.cuda.stream(copy_out):
            for hb, r in zip(outs_host[s], res):
                hb.copy_(r, non_blocking=True)
                r.record_stream(copy_out)

    def pipeline(n):
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload((i + 1) % 2)
            run(i)
        stream.wait_stream(copy_out)

    pipeline(2)
    finish_reduce()
    torch.cuda.synchronize()
    d2h = sum(r.numel() * r.element_size() for r in outs_host[0])
    ee0, ee1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ee0.record(stream)
    pipeline(args.e2e_steps)
    finish_reduce()
    ee1.record(stream)
    torch.cuda.synchronize()
    ems = ee0.elapsed_time(ee1) / args.e2e_steps
    # The copy floor: the same bytes moved host->device and device->host at
    # once on the same two streams, with no compute (PCIe, both directions).
    back = {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in pin.items()}
    cur = torch.cuda.current_stream()
    reps = 3
    torch.cuda.synchronize()
    ee0.record(cur)
    for _ in range(reps):
        for st in (copy_in, copy_out):
            st.wait_stream(cur)
        with torch.cuda.stream(copy_in), torch.no_grad():
            for k, v in pin.items():
                slots[0][k].copy_(v, non_blocking=True)
        with torch.cuda.stream(copy_out), torch.no_grad():
            for k, v in back.items():
                v.copy_(slots[1][k], non_blocking=True)
        cur.wait_stream(copy_in)
        cur.wait_stream(copy_out)
    ee1.record(cur)
    torch.cuda.synchronize()
    floor_ms = ee0.elapsed_time(ee1) / reps
    if world > 1:
        mt = torch.tensor([ems, floor_ms], device=dev)
        dist.all_reduce(mt, op=dist.ReduceOp.MAX)
        ems, floor_ms = (float(x) for x in mt.tolist())
    return {"value": units * world / (ems * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ems, "path": "selectssm_b200.selective_scan, pinned host "
            "buffers, copies inside the timed region",
            "copy_floor_ms": floor_ms, "frac_of_copy_floor": floor_ms / ems}


def config_of(spec, world, chan, res):
    par = ("single GPU" if world == 1 else
           f"d_inner-sharded x{world} ({res['d_inner_per_gpu']} channels per GPU), B/C replicated, dB/dC summed "
           "over the ranks" if chan else
           f"batch-sharded dp{world} ({res['batch_per_gpu']} sequences per GPU), one NCCL all-reduce of dA/dD "
           "per backward, overlapped with the next forward")
    return {"workload": spec["workload"], "global_batch": spec["batch"], "batch_per_gpu": res["batch_per_gpu"],
            "seq_len": spec["seqlen"], "d_inner": spec["dim"], "d_inner_per_gpu": res["d_inner_per_gpu"],
            "d_state": CFG["dstate"], "parallelism": par,
            "l2": "inputs larger than L2 (u, dt, z, dy of every step exceed 126 MB), no flush"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config2", action="store_true", help="skip the config-2 keys at N=1")
    ap.add_argument("--e2e-steps", type=int, default=30)
    ap.add_argument("--batch", type=int, default=None, help="override batch per GPU (small profiling cases)")
    ap.add_argument("--seqlen", type=int, default=None, help="override the sequence length (small profiling cases)")
    ap.add_argument("--workload", type=int, default=5, choices=[2, 4, 5],
                    help="5 (default): the scaling workload, batch of 64 split over the ranks; 2: config 2 alone; "
                         "4: config 4 (with --parallel channels)")
    ap.add_argument("--config", type=int, default=None, choices=[3, 4],
                    help="time config 3 or 4 device-resident on one GPU (no e2e or CPU legs)")
    ap.add_argument("--parallel", default="batch", choices=["batch", "channels"],
                    help="N>1 sharding: batch rows (default) or d_inner channels with B/C replicated")
    ap.add_argument("--bc-sum", default="multicast", choices=["multicast", "nccl"],
                    help="channel sharding: sum dB/dC inside the backward kernel over NVLink multicast "
                         "(default, when the GPUs support it) or with an NCCL all-reduce after it")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.config is not None:
        if world != 1 or args.impl != "ours":
            raise SystemExit("--config 3/4 time one GPU with the CUDA path only")
        return run_other_config(args)
    spec = SPECS[args.workload]
    if args.seqlen:
        spec = dict(spec, seqlen=args.seqlen)
    chan = args.parallel == "channels" and world > 1
    if args.impl == "reference":
        return reference_arm(spec, args, world, rank, chan)

    import torch
    import torch.distributed as dist
    from selectssm_b200 import _lib

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    lib = _lib.load()
    res = measure(spec, args, world, rank, dev, lib, chan=chan, bc_sum_mode=args.bc_sum)
    line = {"metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": res["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": res["dtype"], "data": "synthetic",
            "config": config_of(spec, world, chan, res),
            "roofline": res["roofline"], "roofline_fwd": res["roofline_fwd"], "roofline_step": res["roofline_step"],
            "e2e": res["e2e"], "gpu_launches": res["gpu_launches"], "clocks": res["clocks"],
            "library": lib.ssm_version().decode()}
    if world == 1 and args.workload != 2 and not args.no_config2:
        c2 = measure(SPECS[2], args, 1, 0, dev, lib, e2e=True)
        line["config2"] = {"value": c2["value"], "unit": UNIT, "ms_per_step": c2["ms_per_step"],
                           "dtype": "f32", "config": config_of(SPECS[2], 1, False, c2),
                           "roofline": c2["roofline"], "roofline_fwd": c2["roofline_fwd"],
                           "roofline_step": c2["roofline_step"], "e2e": c2["e2e"],
                           "gpu_launches": c2["gpu_launches"], "clocks": c2["clocks"]}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, secs, sample = run_cpu_sample(spec, seqlen=spec["seqlen"], batch=4)  # about 1 s on 16 cores
        line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cpu_cores(), "kind": "port",
                                "sample": sample, "seconds": secs}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


def reference_arm(spec, args, world, rank, chan):
    """The reference algorithm (NumPy restatement, oracle/) on the host cores,
    on rank 0 only; each step is a bounded sample of the workload."""
    if rank != 0:
        return
    steps = max(1, args.steps)
    vals = []
    # each step times the oracle on one full-width batch row of L=256, split
    # over all host cores (about 0.1 s), so the run stays within minutes
    sampler = CpuSampler(spec, 256)
    for _ in range(args.warmup):
        sampler.run()
    t0 = time.perf_counter()
    sample = ""
    for _ in range(steps):
        v, _, sample = sampler.run()
        vals.append(v)
    sampler.close()
    total = time.perf_counter() - t0
    v = statistics.median(vals)
    cfg = {"workload": spec["workload"], "global_batch": spec["batch"], "seq_len": spec["seqlen"],
           "d_inner": spec["dim"], "d_state": CFG["dstate"],
           "parallelism": "host CPU (rank 0 only)" if world > 1 else "host CPU"}
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * total / steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "impl": "reference",
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cpu_cores(), "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


if __name__ == "__main__":
    main()
