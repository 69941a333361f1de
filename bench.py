#!/usr/bin/env python
"""Benchmark of the EACS gated cell on B200.

Workload (one "step"): the gated EACS cell inference forward -- event gate,
ZOH predict/update, commit -- over B=8 videos x L=4096 frames x H=768
channels x N=16 complex states, fp16 per-frame features, theta=0.12, with the
op-boundary tensors produced by a randomly initialised EACSLayer (seed 0,
same parameter construction order as the reference module) applied to
N(0,1) fp16 features; dt ~ U[0.25, 2] s with 10% of steps forced to 0.25 s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torch.distributed.run, one process per GPU, each on its own
videos (weak scaling, no collective on the data path).  Rank 0 prints one
JSON line.  `--impl reference` times the CPU restatement of the reference's
algorithm (oracle/) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "longvideo-main_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "EACS scan Gstate-updates/s and HBM GB/s (% of 8 TB/s) at 1/2/4/8 B200"
UNIT = "Gstate-updates/s"
B, L, H, N = 8, 4096, 768, 16
TAU = (0.1, 1.0)          # BranchSpec("short", 16, 0.1, 1.0), the default short branch
EPS_INIT = 0.12
ETA, VAR_EPS, DT_INIT, DT_MIN = 1e-6, 1e-5, 1.0, 1e-3
DT_MAX = max(1e3, 10.0 * TAU[1])
UPDATES = B * L * H * N
# Minimal (algorithmic) bytes of one call: read u (fp16), Bc, Cc (complex64),
# t (fp32); write y (fp32), gate, resid (fp32).
ALG_BYTES = B * L * H * 2 + 2 * B * L * N * 8 + B * L * 4 + B * L * H * 4 + 2 * B * L * 4
# Frames per chunk of the host-buffer (end-to-end) call: the copies of one
# chunk overlap the cell of the next.
E2E_CHUNK = 512
# Issue slots per state update of cell_chain<SPEC> at this workload (one
# 352-thread CTA per SM): ncu smsp__inst_executed.sum x 32 / updates
# = 927,565,016 x 32 / 402,653,184.
INSTR_PER_UPDATE = 73.7
CONFIG = {
    "workload": "gated EACS cell inference forward (event gate + ZOH predict/update + commit), "
                "B=8 L=4096 H=768 N=16",
    "B": B, "L": L, "H": H, "N": N, "u_dtype": "fp16", "state": "fp32 complex",
    "theta": EPS_INIT, "tau_s": list(TAU), "dt": "U[0.25,2] s, 10% forced 0.25 s",
    "l2": "256 MiB buffer written between timed steps (flushed)",
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="budget of the CPU baseline sample (rank 0, N=1)")
    ap.add_argument("--profile", action="store_true",
                    help="device-timed section only (no e2e, no CPU sample): for ncu captures")
    ap.add_argument("--eps", type=float, default=None,
                    help="gate threshold override for the cell workload (e.g. ~1.01 skips about "
                    "half the frames of the N(0,1) features and exercises the repair path)")
    ap.add_argument("--shape", default=None,
                    help="B,L,H,N override for --workload scan, ssm_train, train or longvideo (e.g. a small case for ncu)")
    ap.add_argument("--workload", choices=["cell", "scan", "ssm", "ssm_train", "train", "multiscale",
                                           "longvideo"],
                    default="cell", help="cell (default) is the headline; the others are the "
                    "materialised scan, the fused ungated SSM, the training step, the "
                    "three-branch multiscale cell and the long-video cell (B=64, H=2048, N=32)")
    ap.add_argument("--L", type=int, default=None, choices=[16384, 32768, 65536],
                    help="frames per video for --workload longvideo (default 16384)")
    return ap.parse_args()


# --------------------------------------------------------------------------
# inputs
# --------------------------------------------------------------------------
def layer_params():
    """EACSLayer(768, BranchSpec('short', 16, 0.1, 1.0), gate=EventGate(0.12))
    parameters as its constructor creates them under torch.manual_seed(0)
    (cst_ssm/modules/eacs.py:188-234, ops/spectral_init.py:28-47)."""
    torch.manual_seed(0)
    log_tau = torch.empty(H, N).uniform_(math.log(TAU[0]), math.log(TAU[1]))
    a_lnr = -log_tau
    a_imag = (math.pi * torch.arange(N, dtype=torch.float32)).unsqueeze(0).expand(H, N)
    norm = torch.nn.LayerNorm(H)
    proj_u = torch.nn.Linear(H, H)
    proj_B = torch.nn.Linear(H, 2 * N)
    proj_C = torch.nn.Linear(H, 2 * N)
    lam = torch.complex(-torch.exp(a_lnr), a_imag.contiguous())
    eps = float(0.01 + 0.89 * torch.sigmoid(torch.logit(torch.tensor((EPS_INIT - 0.01) / 0.89))))
    return dict(lam=lam, log_dt=torch.zeros(H), D=torch.zeros(H), mean=torch.zeros(H),
                var=torch.ones(H), norm=norm, proj_u=proj_u, proj_B=proj_B, proj_C=proj_C, eps=eps)


def make_inputs(rank: int, dev: torch.device):
    p = layer_params()
    g = torch.Generator().manual_seed(1000 + rank)
    x = torch.randn(B, L, H, generator=g).to(torch.float16)
    dt = 0.25 + 1.75 * torch.rand(B, L, generator=g)
    dt[torch.rand(B, L, generator=g) < 0.1] = 0.25
    t = torch.cumsum(dt, 1)
    mods = [p[k].to(dev) for k in ("norm", "proj_u", "proj_B", "proj_C")]
    with torch.no_grad():
        # fp32 projections rounded to fp16, as an fp16 autocast region emits them;
        # identical on CPU and GPU so both arms see the same kind of data.
        xn = mods[0](x.to(dev).float())
        u = mods[1](xn).half()                # fp16 per-frame features
        b = mods[2](xn).half().float()
        c = mods[3](xn).half().float()
    Bc = torch.complex(b[..., :N], b[..., N:]).contiguous()
    Cc = torch.complex(c[..., :N], c[..., N:]).contiguous()
    d = dict(lam=p["lam"].to(dev), log_dt=p["log_dt"].to(dev), u=u.contiguous(), Bc=Bc, Cc=Cc,
             t=t.to(dev), D=p["D"].to(dev), mean=p["mean"].to(dev), var=p["var"].to(dev))
    return d, p["eps"]


# --------------------------------------------------------------------------
# clocks (NVML, read-only)
# --------------------------------------------------------------------------
class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, dev_index: int):
        self.samples = []
        self.load = False
        self.ok = False
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(dev_index).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # pragma: no cover - no NVML
            self.err = repr(e)
        self.th = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                try:
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                except Exception:
                    rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                self.samples.append((self.load, mhz, rs))
            except Exception:
                pass
            time.sleep(0.01)

    def start(self):
        if self.ok:
            self.th.start()

    def stop(self):
        self._stop.set()
        if self.ok:
            self.th.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        under = [s for s in self.samples if s[0]] or self.samples
        reasons = set()
        for _, _, rs in under:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median([s[1] for s in under]) if under else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples_under_load": len([s for s in self.samples if s[0]])}


# --------------------------------------------------------------------------
# CPU side: oracle sample
# --------------------------------------------------------------------------
def oracle_sample_inputs(d):
    return {k: (v.float().cpu().numpy() if not v.is_complex() else v.cpu().numpy())
            for k, v in d.items()}


def oracle_rate(host, eps, L_s, threads):
    """Run the CPU oracle on the first L_s frames of all B videos."""
    from oracle import oracle
    oracle.set_threads(threads)
    sub = {k: (v[:, :L_s] if k in ("u", "Bc", "Cc", "t") else v) for k, v in host.items()}
    t0 = time.perf_counter()
    oracle.cell_fwd(sub["lam"], sub["log_dt"], sub["u"], sub["Bc"], sub["Cc"], sub["t"], sub["D"],
                    sub["mean"], sub["var"], eps, ETA, VAR_EPS, DT_INIT, DT_MIN, DT_MAX)
    dt = time.perf_counter() - t0
    return B * L_s * H * N / dt, dt


def pick_sample_len(host, eps, threads, seconds):
    rate, _ = oracle_rate(host, eps, 4, threads)
    return int(max(2, min(L, seconds * rate / (B * H * N))))


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# --------------------------------------------------------------------------
# multi-rank aggregation (weak scaling: every rank runs its own B videos)
# --------------------------------------------------------------------------
def max_over_ranks(ms: float, dev, world: int) -> float:
    """The slowest rank's time (device-measured ms); identity on one rank."""
    if world <= 1:
        return float(ms)
    import torch.distributed as dist
    t = torch.tensor([float(ms)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def job_rate(steps: int, seconds: float, world: int) -> float:
    """Whole-job state updates per second (in G) over all ranks."""
    return world * steps * UPDATES / seconds / 1e9


# --------------------------------------------------------------------------
# arms
# --------------------------------------------------------------------------
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    d, eps = make_inputs(0, torch.device("cpu")) if not torch.cuda.is_available() else \
        make_inputs(0, torch.device("cuda", 0))
    if args.eps is not None:
        eps = float(args.eps)
    host = oracle_sample_inputs(d)
    cores = cpu_cores()
    budget = 90.0 / max(1, args.steps + args.warmup)
    L_s = pick_sample_len(host, eps, cores, budget)
    for _ in range(args.warmup):
        oracle_rate(host, eps, L_s, cores)
    times = [oracle_rate(host, eps, L_s, cores)[1] for _ in range(args.steps)]
    total = sum(times)
    value = args.steps * B * L_s * H * N / total / 1e9
    sample = (f"first {L_s} of {L} frames of all {B} videos per step (full H={H}, N={N}); "
              f"CPU restatement of modules/eacs.py scan_range, {cores} OpenMP threads, {cpu_model()}")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": CONFIG,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch.distributed as dist
    from eacs_b200 import _lib
    from eacs_b200.ops.eacs_gated_scan import cell_forward_into, workspace_bytes

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                                device_id=dev)

    d, eps = make_inputs(rank, dev)
    if args.eps is not None:
        eps = float(args.eps)
    y = torch.empty(B, L, H, device=dev)
    gate = torch.empty(B, L, device=dev)
    resid = torch.empty(B, L, device=dev)
    ws = torch.empty(workspace_bytes(B, L, H, N), dtype=torch.uint8, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    args_op = (d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"], d["mean"], d["var"],
               eps, ETA, VAR_EPS, DT_INIT, DT_MIN, DT_MAX, None, "hard", 0.1)

    def op():
        cell_forward_into(*args_op, y, gate, resid, ws)

    def barrier():
        if world > 1:
            dist.barrier()

    sampler = ClockSampler(local)
    sampler.start()
    for _ in range(max(3, args.warmup)):
        op()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    update_rate = float(gate.mean())

    # ---- device-timed region: inputs resident in HBM ------------------------
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for a, b in kev:  # torch creates the CUDA event at its first record
        a.record()
        b.record()
    barrier()
    torch.cuda.synchronize()
    sampler.load = True
    launches0 = _lib.kernel_launches()
    for k in range(args.steps):
        flush.zero_()
        ev[k][0].record()
        _lib.set_kernel_events(*kev[k])
        op()
        _lib.set_kernel_events(None, None)
        ev[k][1].record()
    torch.cuda.synchronize()
    sampler.load = False
    launches = _lib.kernel_launches() - launches0
    barrier()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    kern_ms = [a.elapsed_time(b) for a, b in kev]
    total_ms = max_over_ranks(sum(step_ms), dev, world)
    total_s = total_ms / 1e3
    value = job_rate(args.steps, total_s, world)

    # ---- end to end through the public API, host buffers ------------------
    from eacs_b200.ops.eacs_gated_scan import eacs_cell_forward_host
    pin = {k: d[k].cpu().pin_memory() for k in ("u", "Bc", "Cc", "t")}
    out_host = [torch.empty(B, L, H).pin_memory(), torch.empty(B, L).pin_memory(),
                torch.empty(B, L).pin_memory()]
    h2d = sum(v.numel() * v.element_size() for v in pin.values())
    d2h = sum(v.numel() * v.element_size() for v in out_host)

    def e2e_step():
        # the host-buffer entry point: time chunks' copies overlap the cell
        eacs_cell_forward_host(d["lam"], d["log_dt"], pin["u"], pin["Bc"], pin["Cc"], pin["t"],
                               d["D"], d["mean"], d["var"], eps, ETA, VAR_EPS, DT_INIT, DT_MIN,
                               DT_MAX, chunk=E2E_CHUNK, out=out_host)

    e2e_steps = 0 if args.profile else max(3, min(args.steps, 30))
    for _ in range(3 if e2e_steps else 0):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    sampler.load = True
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    sampler.load = False
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), dev, world)
    e2e_value = job_rate(e2e_steps, e2e_ms / 1e3, world) if e2e_steps else None
    sampler.stop()
    assert _lib.device_status() == 0

    # ---- roofline of the dominant kernel ----------------------------------
    kmean_s = statistics.mean(kern_ms) / 1e3
    achieved = ALG_BYTES / kmean_s / 1e9
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(peaks_path):
        peak, peak_src = json.load(open(peaks_path))["hbm_gbs"], "measured"
    else:
        peak, peak_src = 6650.0, "fallback"
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "cell_chain_c1_traffic.json")
    if os.path.exists(tpath):
        traffic = json.load(open(tpath)).get("dram_bytes_per_launch")
    # The chain kernel is bound by instruction issue (FP32 + MUFU), not HBM:
    # its issue roofline from the ncu instruction count per state update.
    n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
    clk = sampler.summary().get("sm_mhz") or 1965.0
    issue_peak = n_sm * 4 * 32 * clk * 1e6  # 4 warp-instructions per SM clock, 32 lanes
    issue_achieved = UPDATES / kmean_s * INSTR_PER_UPDATE

    # ---- the reference's own CUDA kernel (K3), when built for sm_100a -----
    ref_cuda = None
    if rank == 0 and world == 1 and not args.profile:
        from bench_workloads import load_ref, timed
        ref = load_ref("ref_eacs_cell_cuda")
        if ref is not None:
            u32 = d["u"].float()  # its wrapper casts u to float32 (eacs_gated_scan.py:44-49)
            def ref_op():
                return ref.eacs_cell_fwd(d["lam"], d["log_dt"], u32, d["Bc"], d["Cc"], d["t"], d["D"],
                                         d["mean"], d["var"], eps, ETA, VAR_EPS, DT_INIT, DT_MIN, DT_MAX)
            r_ms, _ = timed(ref_op, 3, 1, flush)
            yr, gr, rr = ref_op()
            op()
            torch.cuda.synchronize()
            ref_cuda = {"kernel": "reference eacs_cell_fwd_kernel (K3), sm_100a build",
                        "value": UPDATES / (statistics.median(r_ms) / 1e3) / 1e9, "unit": UNIT,
                        "ms_per_step": statistics.median(r_ms),
                        "y_max_rel_diff": float((yr - y).abs().max() / yr.abs().max()),
                        "gates_equal": bool(torch.equal(gr, gate))}

    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) fp16 features through a seed-0 EACSLayer init)",
            "config": dict(CONFIG, update_rate=update_rate,
                           **({} if args.eps is None else {"eps_override": eps})),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_src,
                         "kernel": "cell_chain<SPEC> (speculative all-commit gated chain)",
                         "kernel_ms": 1e3 * kmean_s, "alg_bytes_per_launch": ALG_BYTES,
                         "kernel_gupdates_per_s": UPDATES / kmean_s / 1e9,
                         "issue": {"achieved_Tinstr_s": issue_achieved / 1e12,
                                   "peak_Tinstr_s": issue_peak / 1e12,
                                   "frac": issue_achieved / issue_peak,
                                   "instr_per_update": INSTR_PER_UPDATE,
                                   "peak_basis": f"{n_sm} SMs x 128 lanes x median SM clock"}},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "clocks": sampler.summary(),
        }
        if ref_cuda is not None:
            line["reference_cuda"] = ref_cuda
        if world == 1 and not args.profile:
            host = oracle_sample_inputs(d)
            cores = cpu_cores()
            L_s = pick_sample_len(host, eps, cores, args.cpu_seconds)
            rate, secs = oracle_rate(host, eps, L_s, cores)
            line["cpu_baseline"] = {
                "value": rate / 1e9, "unit": UNIT, "cores": cores, "kind": "port",
                "sample": f"first {L_s} of {L} frames of all {B} videos ({secs:.1f} s, {cpu_model()})"}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload != "cell":
        from bench_workloads import run_workload
        return run_workload(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
