"""Benchmark of the selectssm selective-scan hot path on B200.

Metric: scan fwd+bwd tokens*channels/s and % of the HBM roofline.
Workload at N=1: config 2 of the benchmark contract -- the raw selective-scan op
forward + backward in float32, batch=8, L=4096, d_inner=1536, N=16, with the
softplus(dt) preamble, D skip and silu(z) gate fused in; synthetic seeded inputs
(u, z ~ N(0,1); dt_raw ~ N(0,1) - 4; A = -U[1,16]; B, C ~ N(0,1); D ~ N(1, 0.1);
upstream grad ~ N(0,1)).  One step = one forward + one backward over the batch.

Multi-GPU (torchrun, one process per GPU): weak scaling, each rank scans its own
batch of 8 sequences (batch sharding, no collective in the forward) and the
backward ends with one NCCL all-reduce of the small parameter gradients
(dA, dD) -- the only exchange the partition needs.

`--impl reference` times the reference algorithm on the host CPU instead: the
NumPy restatement of ssm_chunked_scan (forward) and of the ssm_scan custom-VJP
backward from oracle/, on a bounded prefix of the same workload (JAX, the
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


def read_traffic(name):
    """dram bytes per launch recorded in a committed ncu summary, else None."""
    p = os.path.join(ROOT, "profiles", name)
    try:
        with open(p) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


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
    cores: the channels of one fixed sample are split over one single-threaded
    process per core (the reference's JAX-on-CPU would also use every core).
    The workers are forked after the sample is drawn, so they share it."""

    def __init__(self, seqlen, batch=1):
        import multiprocessing as mp
        global _SAMPLE_INP
        D, N = CFG["dim"], CFG["dstate"]
        _SAMPLE_INP = host_inputs(0, batch, seqlen, D, N)
        self.procs = cpu_cores()
        k = self.procs
        self.spans = [(D * i // k, D * (i + 1) // k) for i in range(k)]
        self.units = batch * seqlen * D
        self.sample = (f"NumPy restatement of the reference algorithm (chunked scan fwd + custom-VJP bwd, float32) "
                       f"on batch={batch}, L={seqlen}, d_inner={D}, N={N} of the config-2 workload, channels split "
                       f"over {k} single-threaded processes (one per host core), after one warm-up run")
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


def run_cpu_sample(seqlen=4096, batch=1):
    sampler = CpuSampler(seqlen, batch)
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
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--batch", type=int, default=None, help="override batch per GPU (small profiling cases)")
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 4, 5],
                    help="2 (default) is the benchmark line; 3, 4 and 5 time the other contract workloads "
                         "device-resident on one GPU (no e2e or CPU legs)")
    ap.add_argument("--parallel", default="batch", choices=["batch", "channels"],
                    help="N>1 sharding: batch rows (default) or d_inner channels with B/C replicated")
    ap.add_argument("--bc-sum", default="multicast", choices=["multicast", "nccl"],
                    help="channel sharding: sum dB/dC inside the backward kernel over NVLink multicast "
                         "(default, when the GPUs support it) or with an NCCL all-reduce after it")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.config != 2:
        if world != 1 or args.impl != "ours":
            raise SystemExit("--config 3/4/5 time one GPU with the CUDA path only")
        return run_other_config(args)
    if args.batch:
        CFG["batch"] = args.batch
    Bsz, L, D, N = CFG["batch"], CFG["seqlen"], CFG["dim"], CFG["dstate"]
    config = {"workload": "config 2: raw selective-scan op fwd+bwd (softplus dt, D skip, silu gate fused)",
              "batch_per_gpu": Bsz, "global_batch": Bsz * world, "seq_len": L, "d_inner": D, "d_state": N,
              "parallelism": ("single GPU" if world == 1 else
                              f"batch-sharded dp{world}, NCCL all-reduce of dA/dD in bwd" if args.parallel == "batch"
                              else f"d_inner-sharded x{world} ({D} channels per GPU), B/C replicated, dB/dC"),
              "l2": "inputs larger than L2 (u, dt, z, dy = 805 MB per step), no flush"}

    if args.impl == "reference":
        if rank != 0:
            return
        steps = max(1, args.steps)
        vals = []
        # each step times the oracle on one full-width batch row of L=256, split
        # over all host cores (about 0.1 s), so 1000 steps stay within minutes
        sampler = CpuSampler(256)
        for _ in range(args.warmup):
            sampler.run()
        t0 = time.perf_counter()
        for _ in range(steps):
            v, _, sample = sampler.run()
            vals.append(v)
        sampler.close()
        total = time.perf_counter() - t0
        v = statistics.median(vals)
        line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": steps,
                "warmup": args.warmup, "ms_per_step": 1e3 * total / steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
                "impl": "reference",
                "cpu_baseline": {"value": v, "unit": UNIT, "cores": cpu_cores(), "kind": "port",
                                 "sample": sample},
                "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    import torch
    import torch.distributed as dist
    import selectssm_b200 as S
    from selectssm_b200 import _lib
    from selectssm_b200.parallel import MulticastBCSum, allreduce_grads, replicated_bc

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    lib = _lib.load()

    chan = world > 1 and args.parallel == "channels"
    h = host_inputs(1234 + rank, Bsz, L, D, N, bc_seed=1234 if chan else None)
    t = {k: torch.from_numpy(v).to(dev) for k, v in h.items()}
    for k in ("u", "delta", "z", "A", "B", "C", "D"):
        t[k].requires_grad_(True)

    pending = []
    bcs = None
    if chan and args.bc_sum == "multicast":
        bcs = MulticastBCSum(Bsz, L, device=dev)
        if not bcs.available:
            bcs = None
    if chan:
        config["parallelism"] += (" summed inside the backward kernel by NVLink multicast (multimem.red)" if bcs
                                  else " summed by an NCCL all-reduce after the backward")

    def step(inputs):
        for k in ("u", "delta", "z", "A", "B", "C", "D"):
            inputs[k].grad = None
        Bm, Cm = inputs["B"], inputs["C"]
        if chan and bcs is None:  # channel sharding: the B / C gradients are summed over ranks in the backward
            Bm, Cm = replicated_bc(Bm, Cm)
        out = S.selective_scan(inputs["u"], inputs["delta"], inputs["A"], Bm, Cm, D=inputs["D"],
                               z=inputs["z"], delta_softplus=True, bc_sum=bcs)
        out.backward(inputs["dout"])
        if world > 1 and not chan:  # batch sharding: one all-reduce of the parameter gradients,
            finish_reduce()            # overlapped with the next step's forward
            pending.append(allreduce_grads([inputs["A"], inputs["D"]], async_op=True))
        return out

    def finish_reduce():
        while pending:
            pending.pop().wait()

    for _ in range(max(3, args.warmup)):
        step(t)
    finish_reduce()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
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

    units = Bsz * L * D
    value = units * world / (ms * 1e-3)

    # --- per-call timing of the forward and backward (same stream).  The calls
    # are queued back to back, as in the training loop, so host-side overhead
    # overlaps the GPU work and the events time the kernels.
    p_fwd, p_bwd = [], []
    marks = []
    torch.cuda.synchronize()
    for _ in range(8):
        a0, a1, a2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        for k in ("u", "delta", "z", "A", "B", "C", "D"):
            t[k].grad = None
        a0.record(stream)
        out = S.selective_scan(t["u"], t["delta"], t["A"], t["B"], t["C"], D=t["D"], z=t["z"], delta_softplus=True)
        a1.record(stream)
        out.backward(t["dout"])
        a2.record(stream)
        marks.append((a0, a1, a2))
    torch.cuda.synchronize()
    for a0, a1, a2 in marks[1:]:
        p_fwd.append(a0.elapsed_time(a1))
        p_bwd.append(a1.elapsed_time(a2))
    t_fwd, t_bwd = statistics.median(p_fwd), statistics.median(p_bwd)
    hbm, src = peaks()
    fb, bb = alg_bytes(units, 4, N, D)
    roof_bwd = {"kernel": "ssm_bwd call: ssm_bwd_kernel<float,float> + segment pre-pass, fold, zero, finalize", "bound": "hbm",
                "achieved": bb / (t_bwd * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s", "peak_source": src,
                "traffic": read_traffic("ssm_bwd_kernel_config2.md"), "algorithmic_bytes": bb,
                "ms": t_bwd}
    roof_bwd["frac"] = roof_bwd["achieved"] / hbm
    roof_fwd = {"kernel": "ssm_fwd call: ssm_fwd_kernel<float,float,0,1> (+ segment pre-pass when segmented)", "bound": "hbm", "achieved": fb / (t_fwd * 1e-3) / 1e9,
                "peak": hbm, "unit": "GB/s", "traffic": read_traffic("ssm_fwd_kernel_config2.md"),
                "algorithmic_bytes": fb, "ms": t_fwd}
    roof_fwd["frac"] = roof_fwd["achieved"] / hbm
    step_roof = {"achieved": (fb + bb) / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s"}
    step_roof["frac"] = step_roof["achieved"] / hbm

    # --- end to end through the public API: pinned host inputs -> device, fwd+bwd,
    # outputs and gradients -> pinned host
    # Pipelined over steps on three streams: the upload of step i+1 (copy_in)
    # and the download of step i-1 (copy_out) overlap the compute of step i;
    # every step still moves all of its inputs and results across PCIe.
    pin = {k: torch.from_numpy(v).pin_memory() for k, v in h.items()}
    h2d = sum(v.numel() * v.element_size() for v in pin.values())
    grad_keys = ("u", "delta", "z", "A", "B", "C", "D")
    slots = [{k: torch.empty(v.shape, dtype=v.dtype, device=dev).requires_grad_(k in grad_keys)
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
        res = [out.detach()] + [slots[s][k].grad for k in grad_keys]
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
    if world > 1:
        mt = torch.tensor([ems], device=dev)
        dist.all_reduce(mt, op=dist.ReduceOp.MAX)
        ems = float(mt.item())

    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
            "roofline": roof_bwd, "roofline_fwd": roof_fwd, "roofline_step": step_roof,
            "e2e": {"value": units * world / (ems * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": ems},
            "gpu_launches": n_launches,
            "clocks": clk.summary(), "library": lib.ssm_version().decode()}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, secs, sample = run_cpu_sample(batch=2)  # about 1 s on 16 cores: ~16 core-seconds of work
        line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": cpu_cores(), "kind": "port",
                                "sample": sample, "seconds": secs}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
