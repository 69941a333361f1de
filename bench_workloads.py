"""Secondary bench.py workloads: the materialised scan, the fused ungated
SSM and the three-branch multiscale cell (one GPU), the training step (one
or more GPUs, gradients all-reduced) and the long-video gated cell (one or
more GPUs, videos split over the ranks).

Each prints one JSON line like bench.py's headline (state updates/s, the
dominant kernel's HBM roofline) and, where the reference's own CUDA kernels
were built into oracle/_ref (oracle/build_ref.py), times them on the same
tensors for comparison.  Inputs are seeded synthetic data with the reference
config shapes; L2 is flushed between timed steps.
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import json
import math
import os
import statistics
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
UNIT = "Gstate-updates/s"


def load_ref(name: str):
    """The reference's extension built for sm_100a, or None."""
    path = os.path.join(ROOT, "oracle", "_ref", name, name + ".so")
    if not os.path.exists(path):
        return None
    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_loader(name, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def peak_hbm():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return json.load(open(p))["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def timed(fn, steps, warmup, flush, kernel_events=False):
    """Per-step device times (ms) of fn, L2 flushed before each step; with
    kernel_events the library's events around its dominant kernel too."""
    from eacs_b200 import _lib
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in ev + kev:
        a.record()
        b.record()
    torch.cuda.synchronize()
    for k in range(steps):
        flush.zero_()
        ev[k][0].record()
        if kernel_events:
            _lib.set_kernel_events(*kev[k])
        fn()
        if kernel_events:
            _lib.set_kernel_events(None, None)
        ev[k][1].record()
    torch.cuda.synchronize()
    step = [a.elapsed_time(b) for a, b in ev]
    kern = [a.elapsed_time(b) for a, b in kev] if kernel_events else None
    return step, kern


def lam_init(g, H, N, tmin, tmax, imag_scale=1.0):
    log_tau = torch.empty(H, N).uniform_(math.log(tmin), math.log(tmax), generator=g)
    im = (math.pi * imag_scale * torch.arange(N, dtype=torch.float32)).expand(H, N)
    return torch.complex(-torch.exp(-log_tau), im.contiguous())


def times_exp(g, B, L, mean):
    dt = torch.empty(B, L).exponential_(1.0 / mean, generator=g).clamp(1 / 30, 2.0)
    return torch.cumsum(dt, 1)


def cell_inputs(g, B, L, H, N, tau, dev, u_dtype, mean_dt=0.25):
    s = 1.0 / math.sqrt(2 * N)
    d = dict(lam=lam_init(g, H, N, *tau), log_dt=torch.zeros(H),
             u=torch.randn(B, L, H, generator=g).to(u_dtype),
             Bc=torch.complex(torch.randn(B, L, N, generator=g) * s, torch.randn(B, L, N, generator=g) * s),
             Cc=torch.complex(torch.randn(B, L, N, generator=g) * s, torch.randn(B, L, N, generator=g) * s),
             t=times_exp(g, B, L, mean_dt), D=torch.randn(H, generator=g),
             mean=torch.zeros(H), var=torch.ones(H))
    return {k: v.to(dev) for k, v in d.items()}


def train_inputs(rank, dev, B=8, L=8192, H=768, N=16):
    """Gated-cell training inputs (tau band [0.5, 4] s, bf16 u, Exp(0.25 s)
    frame gaps) and the upstream gradient dL/dy ~ N(0,1) for one rank."""
    g = torch.Generator().manual_seed(9 + rank)
    d = cell_inputs(g, B, L, H, N, (0.5, 4.0), dev, torch.bfloat16)
    gy = torch.randn(B, L, H, generator=g).to(dev)
    return d, gy


MULTISCALE_SHAPE = (4, 16384, 1024, 16)
MULTISCALE_BANDS = [(0.5, 4.0), (4.0, 32.0), (32.0, 256.0)]


def multiscale_inputs(dev, B=None, L=None):
    """MultiScaleEACS inputs: the layer input x (bf16) and one op-boundary set
    per branch (tau bands [0.5,4], [4,32], [32,256] s, bf16 u); every branch
    sees the same timestamps (one video).  B, L below the full shape take
    the leading rows and frames of the same draw."""
    B0, L0, H, N = MULTISCALE_SHAPE
    g = torch.Generator().manual_seed(10)
    x = torch.randn(B0, L0, H, generator=g).to(torch.bfloat16)
    br = [cell_inputs(g, B0, L0, H, N, tb, "cpu", torch.bfloat16) for tb in MULTISCALE_BANDS]
    for d in br:
        d["t"] = br[0]["t"]
    B, L = B or B0, L or L0

    def cut(k, v):
        return v[:B, :L].contiguous() if k in ("u", "Bc", "Cc", "t") else v
    br = [{k: cut(k, v).to(dev) for k, v in d.items()} for d in br]
    return x[:B, :L].contiguous().to(dev), br


def line(metric, value, steps, warmup, ms, config, **extra):
    out = {"metric": metric, "value": value, "unit": UNIT, "n_gpus": 1, "steps": steps,
           "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config}
    out.update(extra)
    print(json.dumps(out), flush=True)


# ----------------------------------------------------------------------------
def wl_scan(args, dev, flush):
    """scan_fwd / scan_bwd on one multiscale branch (B=4 H=1024 N=16) at L=4096 (24 / 40 B per update);
    --shape B,L,H,N gives a small case for ncu."""
    from eacs_b200.ops.scan_cuda import EXT
    B, L, H, N = (4, 4096, 1024, 16) if getattr(args, "shape", None) is None else (int(v) for v in args.shape.split(","))
    g = torch.Generator().manual_seed(7)
    mag = (0.69 + 0.3 * torch.rand(B, L, H, N, generator=g))
    ph = 6.283185 * torch.rand(B, L, H, N, generator=g)
    a = torch.polar(mag, ph).to(dev)
    b = torch.complex(torch.randn(B, L, H, N, generator=g), torch.randn(B, L, H, N, generator=g)).to(dev)
    gh = torch.complex(torch.randn(B, L, H, N, generator=g), torch.randn(B, L, H, N, generator=g)).to(dev)
    upd = B * L * H * N
    peak, src = peak_hbm()
    h = EXT.scan_fwd(a, b)[0]
    fs, fk = timed(lambda: EXT.scan_fwd(a, b), args.steps, args.warmup, flush, True)
    bs, bk = timed(lambda: EXT.scan_bwd(a, h, gh), args.steps, args.warmup, flush, True)
    fk_s, bk_s = statistics.median(fk) / 1e3, statistics.median(bk) / 1e3
    extra = {}
    ref = load_ref("ref_eacs_scan_cuda")
    if ref is not None:
        rf, _ = timed(lambda: ref.scan_fwd(a, b), max(3, args.steps // 5), 2, flush)
        rb, _ = timed(lambda: ref.scan_bwd(a, h, gh), max(3, args.steps // 5), 2, flush)
        hr = ref.scan_fwd(a, b)[0]
        extra["reference_cuda"] = {
            "kernel": "reference scan_fwd_kernel / scan_bwd_kernel (sm_100a build)",
            "fwd_gupdates_per_s": upd / (statistics.median(rf) / 1e3) / 1e9,
            "bwd_gupdates_per_s": upd / (statistics.median(rb) / 1e3) / 1e9,
            "fwd_ms": statistics.median(rf), "bwd_ms": statistics.median(rb),
            "max_abs_diff_h": float((hr - h).abs().max())}
    line("EACS scan_fwd Gstate-updates/s (materialised a, b -> h)", upd / fk_s / 1e9, args.steps,
         args.warmup, statistics.median(fs),
         {"workload": "scan_fwd/scan_bwd complex64 (B,L,H,N)", "B": B, "L": L, "H": H, "N": N,
          "l2": "flushed between steps"},
         roofline={"bound": "hbm", "unit": "GB/s", "peak": peak, "peak_source": src,
                   "fwd": {"achieved": 24 * upd / fk_s / 1e9, "frac": 24 * upd / fk_s / 1e9 / peak,
                           "kernel_ms": fk_s * 1e3, "bytes_per_update": 24},
                   "bwd": {"achieved": 40 * upd / bk_s / 1e9, "frac": 40 * upd / bk_s / 1e9 / peak,
                           "kernel_ms": bk_s * 1e3, "bytes_per_update": 40}},
         bwd_gupdates_per_s=upd / bk_s / 1e9, **extra)


def wl_ssm(args, dev, flush):
    """Fused ungated continuous SSM forward, one multiscale branch (B=4 L=16384 H=1024 N=16, bf16 u)."""
    from eacs_b200.ops.continuous_ssm import ssm_forward
    B, L, H, N = 4, 16384, 1024, 16
    g = torch.Generator().manual_seed(8)
    d = cell_inputs(g, B, L, H, N, (0.5, 64.0), dev, torch.bfloat16)
    upd = B * L * H * N
    fn = lambda: ssm_forward(d["lam"], d["log_dt"], d["t"], d["Bc"], d["Cc"], d["u"], d["D"])
    st, kt = timed(fn, args.steps, args.warmup, flush, True)
    k_s = statistics.median(kt) / 1e3
    alg = B * L * H * 2 + 2 * B * L * N * 8 + B * L * 4 + B * L * H * 4
    peak, src = peak_hbm()
    line("EACS fused ungated SSM Gstate-updates/s", upd / (statistics.median(st) / 1e3) / 1e9,
         args.steps, args.warmup, statistics.median(st),
         {"workload": "ContinuousSSMLayer core fused (dt, ZOH, scan, readout)", "B": B, "L": L,
          "H": H, "N": N, "u_dtype": "bf16", "l2": "flushed between steps"},
         roofline={"bound": "hbm", "achieved": alg / k_s / 1e9, "peak": peak, "unit": "GB/s",
                   "frac": alg / k_s / 1e9 / peak, "peak_source": src, "kernel_ms": k_s * 1e3,
                   "alg_bytes_per_launch": alg})


class _RefScan(torch.autograd.Function):
    """The reference's _SelectiveScanCUDA (cst_ssm/ops/scan_cuda.py:36-49) over its
    own K1/K2 kernels built for sm_100a."""

    @staticmethod
    def forward(ctx, a, b, ext):
        h = ext.scan_fwd(a.contiguous(), b.contiguous())[0]
        ctx.save_for_backward(a, h)
        ctx.ext = ext
        return h

    @staticmethod
    def backward(ctx, gh):
        a, h = ctx.saved_tensors
        ga, gb = ctx.ext.scan_bwd(a, h, gh.contiguous())
        return ga, gb, None


def ref_ssm_core(lam, log_dt, t, Bc, Cc, u, D, ext):
    """ContinuousSSMLayer's core as the reference computes it under autograd
    (continuous_ssm.py:44-55 with discretization.py:10-82): materialised dt_eff,
    dA, dB, dB*u (B,L,H,N) complex64, the scan, the einsum readout."""
    dt = torch.zeros_like(t)
    dt[:, 1:] = (t[:, 1:] - t[:, :-1]).clamp_min(0)
    dt[:, 0] = dt[:, 1]
    dte = (dt.unsqueeze(-1) * torch.exp(log_dt)).clamp_min(1e-3).clamp_max(1e3)
    z = lam * dte.unsqueeze(-1).to(torch.complex64)
    dA = torch.exp(z)
    em1 = torch.complex(torch.expm1(z.real) * torch.cos(z.imag) - 2 * torch.sin(0.5 * z.imag) ** 2,
                        torch.exp(z.real) * torch.sin(z.imag))
    dB = em1 * torch.reciprocal(lam) * Bc.unsqueeze(2)
    dBu = dB * u.float().unsqueeze(-1)
    h = _RefScan.apply(dA, dBu, ext)
    return torch.einsum("bln,blhn->blh", Cc, h).real + D * u.float()


def wl_ssm_train(args, dev, flush):
    """Fused ungated SSM core, forward + backward (SSMCoreFunction), at
    the multiscale branch shape (B=4 L=16384 H=1024 N=16, bf16 u); beside it, at B=1 L=4096 (where
    its materialised (B,L,H,N) tensors fit), the reference's autograd path over
    its own scan kernels and ours on the same tensors."""
    from eacs_b200 import _lib
    from eacs_b200.ops.continuous_ssm import _backward, _forward, _prepare, ssm_forward

    def make(B, L, H, N, seed):
        g = torch.Generator().manual_seed(seed)
        d = cell_inputs(g, B, L, H, N, (0.5, 64.0), dev, torch.bfloat16)
        gy = torch.randn(B, L, H, generator=g).to(dev)
        leaves = {k: d[k].clone().requires_grad_(True) for k in ("lam", "log_dt", "Bc", "Cc", "u", "D")}
        return d, gy, leaves

    def ours(d, gy, lv):
        y = ssm_forward(lv["lam"], lv["log_dt"], d["t"], lv["Bc"], lv["Cc"], lv["u"], lv["D"])
        torch.autograd.backward([y], [gy])

    B, L, H, N = 4, 16384, 1024, 16
    if getattr(args, "shape", None):
        B, L, H, N = (int(v) for v in args.shape.split(","))
    d, gy, lv = make(B, L, H, N, 11)
    nsteps = max(3, args.steps // 10)
    st, _ = timed(lambda: ours(d, gy, lv), nsteps, 2, flush, False)
    upd = B * L * H * N
    n0 = _lib.kernel_launches()
    ours(d, gy, lv)
    torch.cuda.synchronize()
    launches = _lib.kernel_launches() - n0
    # the two chain kernels on their own (autograd runs the backward on its
    # own thread, where the library's per-thread timing events are not set)
    dev_, prep = _prepare(*(lv[k].detach() if k in lv else d[k]
                            for k in ("lam", "log_dt", "t", "Bc", "Cc", "u", "D")))
    _, ck = _forward(prep, dev_, 1e-3, 1e3, True)
    _, fk = timed(lambda: _forward(prep, dev_, 1e-3, 1e3, True), nsteps, 2, flush, True)
    _, kt = timed(lambda: _backward(prep, ck, gy, 1e-3, 1e3), nsteps, 2, flush, True)
    k_s = statistics.median(kt) / 1e3
    # backward chain kernel algorithmic bytes: inputs re-read (u bf16, gy fp32, Bc, Cc, t),
    # checkpoints read, du fp32 written, per-tile dB/dC partials written
    lanes = 4 if N <= 8 else 8 if N <= 16 else 16 if N <= 32 else 32
    ntiles = -(-H // (128 // lanes))  # backward CTAs per row: 128 threads, `lanes` per channel
    alg = (B * L * H * (2 + 4 + 4) + 2 * B * L * N * 8 + B * L * 4 + B * ((L + 7) // 8) * H * N * 8
           + B * ntiles * L * N * 16)
    peak, src = peak_hbm()
    extra = {}
    ext = None if args.profile else load_ref("ref_eacs_scan_cuda")
    if ext is not None:
        Bs, Ls = 1, 4096
        d2, gy2, lv2 = make(Bs, Ls, H, N, 12)

        def ref():
            y = ref_ssm_core(lv2["lam"], lv2["log_dt"], d2["t"], lv2["Bc"], lv2["Cc"], lv2["u"], lv2["D"], ext)
            torch.autograd.backward([y], [gy2])

        rt, _ = timed(ref, 3, 1, flush, False)
        ot, _ = timed(lambda: ours(d2, gy2, lv2), 5, 2, flush, False)
        u2 = Bs * Ls * H * N
        extra["reference_torch_autograd_gpu"] = {
            "workload": "reference autograd path (torch ops + its K1/K2 scan kernels)",
            "B": Bs, "L": Ls, "H": H, "N": N, "ms_per_step": statistics.median(rt),
            "Gstate_updates_per_s": u2 / (statistics.median(rt) / 1e3) / 1e9,
            "ours_same_shape_ms": statistics.median(ot),
            "ours_same_shape_Gstate_updates_per_s": u2 / (statistics.median(ot) / 1e3) / 1e9}
    line("EACS fused ungated SSM training fwd+bwd Gstate-updates/s",
         upd / (statistics.median(st) / 1e3) / 1e9, len(st), 2, statistics.median(st),
         {"workload": "ContinuousSSMLayer core fwd+bwd fused (checkpoint every 8 steps)", "B": B,
          "L": L, "H": H, "N": N, "u_dtype": "bf16", "l2": "flushed between steps"},
         roofline={"bound": "issue (FP32/MUFU); hbm fraction shown", "achieved": alg / k_s / 1e9,
                   "peak": peak, "unit": "GB/s", "frac": alg / k_s / 1e9 / peak, "peak_source": src,
                   "kernel": "ssm_bwd_chain", "kernel_ms": k_s * 1e3,
                   "kernel_Gstate_updates_per_s": upd / k_s / 1e9, "alg_bytes_per_launch": alg,
                   "forward_chain_kernel_ms": statistics.median(fk),
                   "forward_chain_Gstate_updates_per_s": upd / (statistics.median(fk) / 1e3) / 1e9},
         gpu_launches=launches, **extra)


def wl_train(args):
    """Gated-cell training: GatedEACSCellFunction forward + backward, B=8 L=8192 H=768 N=16, bf16 u
    (--shape B,L,H,N gives a small case for ncu).  Under torchrun every rank
    trains its own B videos (weak scaling), or with --global-batch its share
    of the 8 (strong scaling: one video per rank on 8 GPUs), and the cell's
    parameter gradients (lambda, log_dt, D, eps) are summed over the ranks
    with one NCCL all-reduce per step, as DDP does; time is device-measured,
    max over ranks."""
    import datetime
    import torch.distributed as dist
    from bench import max_over_ranks
    from eacs_b200.ops.eacs_cell_train import _train_bwd, _train_fwd, fused_gated_scan
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    B, L, H, N = (8, 8192, 768, 16) if getattr(args, "shape", None) is None else (int(v) for v in args.shape.split(","))
    split = bool(getattr(args, "global_batch", False))
    if split:  # the global batch's rows of this rank, from the one-rank draw
        if B % world:
            raise SystemExit(f"train: {B} videos do not split over {world} ranks")
        d, gy = train_inputs(0, "cpu", B, L, H, N)
        per = B // world
        rows = slice(rank * per, (rank + 1) * per)
        d = {k: (v[rows].contiguous() if k in ("u", "Bc", "Cc", "t") else v).to(dev) for k, v in d.items()}
        gy = gy[rows].contiguous().to(dev)
        B = per
    else:
        d, gy = train_inputs(rank, dev, B, L, H, N)
    leaves = {k: d[k].clone().requires_grad_(True) for k in ("u", "Bc", "Cc", "lam", "log_dt", "D")}
    eps = torch.tensor(0.12, device=dev, requires_grad=True)

    def step():
        y, gs, rs = fused_gated_scan(leaves["u"], leaves["Bc"], leaves["Cc"], d["t"], leaves["lam"],
                                     leaves["log_dt"], leaves["D"], eps, d["mean"], d["var"], 0.1, 1e-6)
        torch.autograd.backward([y], [gy])
        if world > 1:  # DDP: one bucket with the cell parameters' gradients, summed over the ranks
            grads = [torch.view_as_real(leaves["lam"].grad).reshape(-1), leaves["log_dt"].grad.reshape(-1),
                     leaves["D"].grad.reshape(-1), eps.grad.reshape(-1)]
            flat = torch.cat(grads)
            dist.all_reduce(flat)
            o = 0
            for t in grads:
                t.copy_(flat[o:o + t.numel()])
                o += t.numel()

    nsteps, warmup = max(3, args.steps // 10), 3
    for _ in range(warmup):
        step()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(nsteps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for k in range(nsteps):
        flush.zero_()
        ev[k][0].record()
        step()
        ev[k][1].record()
    torch.cuda.synchronize()
    st = [a.elapsed_time(b) for a, b in ev]
    total_ms = max_over_ranks(sum(st), dev, world)
    # the backward kernel on its own (autograd runs it on its own thread, where
    # the library's per-thread timing events are not set)
    det = {k: v.detach() for k, v in leaves.items()}
    _, gs_, rs_, stats_, prep = _train_fwd(det["u"], det["Bc"], det["Cc"], d["t"], det["lam"],
                                           det["log_dt"], det["D"], 0.12, d["mean"], d["var"], 0.1,
                                           1e-6, 1e-5, 1.0, "ste", 1e3)
    _, kt = timed(lambda: _train_bwd(prep, gs_, rs_, stats_, 0.12, 0.1, 1e-6, 1e-5, 1.0, 1e3, gy,
                                     None, None, None), nsteps, warmup, flush, True)
    upd = B * L * H * N
    with torch.no_grad():
        rate = float(gs_.mean())
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({
            "metric": "EACS gated cell training fwd+bwd Gstate-updates/s",
            "value": world * nsteps * upd / (total_ms / 1e3) / 1e9, "unit": UNIT, "n_gpus": world,
            "steps": nsteps, "warmup": warmup, "ms_per_step": total_ms / nsteps, "higher_is_better": True,
            "scaling": "strong" if split else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "GatedEACSCellFunction fwd+bwd (STE, T=0.1)"
                                   + ("; DDP all-reduce of the cell parameters' gradients" if world > 1 else ""),
                       "B_per_rank": B, "global_batch": B * world, "L": L, "H": H, "N": N, "u_dtype": "bf16",
                       "update_rate": rate,
                       "l2": "flushed between steps"},
            "backward_kernel_ms": statistics.median(kt),
            "backward_kernel_Gstate_updates_per_s": upd / (statistics.median(kt) / 1e3) / 1e9,
            "note": "backward_kernel_ms is the cluster backward kernel (train_bwd) alone, rank 0"}), flush=True)
    return 0


def wl_multiscale(args, dev, flush):
    """MultiScaleEACS, B=4 L=16384 H=1024 N=16: three gated branches (tau bands [0.5,4], [4,32], [32,256] s), each with its
    proj_out, and MultiScaleEACS's epilogue (fusion softmax, blend, LayerNorm) in one kernel."""
    from eacs_b200.ops.eacs_gated_scan import cell_forward_into, workspace_bytes
    from eacs_b200.ops.multiscale import branch_fuse, run_branches
    B, L, H, N = MULTISCALE_SHAPE
    bands = MULTISCALE_BANDS
    x, br = multiscale_inputs(dev)
    fusion = torch.nn.Linear(H, 3).to(dev)
    norm = torch.nn.LayerNorm(H).to(dev)
    proj_out = [torch.nn.Linear(H, H).to(dev, torch.bfloat16) for _ in bands]
    ys = [torch.empty(B, L, H, device=dev) for _ in bands]
    gts = [torch.empty(B, L, device=dev) for _ in bands]
    rss = [torch.empty(B, L, device=dev) for _ in bands]
    wss = [torch.empty(workspace_bytes(B, L, H, N), dtype=torch.uint8, device=dev) for _ in bands]
    dt_max = [max(1e3, 10 * tb[1]) for tb in bands]

    def cell(i, d):
        cell_forward_into(d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"],
                          d["mean"], d["var"], 0.12, 1e-6, 1e-5, 1.0, 1e-3, dt_max[i], None, "hard",
                          0.1, ys[i], gts[i], rss[i], wss[i])

    def cells():  # side by side on the branch streams, as multiscale_forward runs them
        run_branches(br, dev, cell)

    @torch.no_grad()
    def deltas():
        return [proj_out[i](ys[i].to(torch.bfloat16)) for i in range(3)]

    @torch.no_grad()
    def epilogue_torch(ds):  # multiscale.py:176-179 as the reference runs it under bf16 autocast
        with torch.autocast("cuda", torch.bfloat16):
            w = torch.softmax(fusion(x), dim=-1)
            fused = torch.einsum("bldn,bln->bld", torch.stack(ds, -1), w)
            return norm(x + fused)

    @torch.no_grad()
    def step():  # each branch's cell and proj_out on its stream (an EACSLayer forward each), then the epilogue
        def branch(i, d):
            cell(i, d)
            return proj_out[i](ys[i].to(torch.bfloat16))
        return branch_fuse(x, run_branches(br, dev, branch), fusion, norm)

    n = max(3, args.steps // 5)
    st, _ = timed(step, n, 2, flush, False)
    ct, _ = timed(cells, n, 2, flush, False)
    ds = deltas()
    pt, _ = timed(deltas, n, 2, flush, False)
    ft, _ = timed(lambda: branch_fuse(x, ds, fusion, norm), n, 2, flush, False)
    et, _ = timed(lambda: epilogue_torch(ds), n, 2, flush, False)
    upd = 3 * B * L * H * N
    med = statistics.median
    line("EACS MultiScaleEACS (3 branches) Gstate-updates/s", upd / (med(st) / 1e3) / 1e9,
         len(st), 2, med(st),
         {"workload": "MultiScaleEACS: 3 gated branches + proj_out (bf16 GEMM) + fused epilogue "
                      "(fusion softmax, blend, LayerNorm)", "B": B, "L": L, "H": H, "N": N,
          "u_dtype": "bf16", "update_rates": [float(v.mean()) for v in gts],
          "l2": "flushed between steps"},
         parts_ms={"cells": med(ct), "proj_out_gemms": med(pt), "epilogue_fused": med(ft),
                   "epilogue_torch_same_inputs": med(et)},
         note="input projections (LayerNorm, proj_u/B/C) are outside the timed step")


def wl_project(args, dev, flush):
    """EACS layer input projections inside a float16 autocast region:
    LayerNorm -> proj_u / proj_B / proj_C (eacs.py:376, :261-267) for config 1's
    rows and widths (8 x 4096 frames, d = H = 768, N = 16) and config 2's
    (4 x 16384, d = H = 1024), as one tcgen05 kernel (eacs_project, with its
    row-statistics pass) against the reference's autocast sequence on the same
    tensors.  Roofline: tensor, algorithmic flops 2 M d (H + 4N) per launch
    over the measured dense bf16 GEMM peak."""
    from eacs_b200.ops.projection import project
    peaks = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak, src = (json.load(open(peaks))["bf16_tflops"], "measured") if os.path.exists(peaks) else (1590.0, "fallback")
    out = []
    for (Bb, Ll, d, Hh, Nn) in ((8, 4096, 768, 768, 16), (4, 16384, 1024, 1024, 16)):
        torch.manual_seed(0)
        norm = torch.nn.LayerNorm(d).to(dev)
        lins = [torch.nn.Linear(d, o).to(dev) for o in (Hh, 2 * Nn, 2 * Nn)]
        x = torch.randn(Bb, Ll, d, generator=torch.Generator().manual_seed(1)).to(dev).half()

        def ours():
            project(x, norm, *lins, torch.float16)

        @torch.no_grad()
        def ref():
            with torch.autocast("cuda", torch.float16):
                xn = norm(x)
                u = lins[0](xn).float()
                b = lins[1](xn).float()
                c = lins[2](xn).float()
                return u, torch.complex(b[..., :Nn], b[..., Nn:]), torch.complex(c[..., :Nn], c[..., Nn:])
        n = max(5, args.steps // 5)
        st, kt = timed(ours, n, 3, flush, True)
        rt, _ = timed(ref, n, 3, flush, False)
        flops = 2 * Bb * Ll * d * (Hh + 4 * Nn)
        kms = statistics.median(kt)
        out.append({"rows": Bb * Ll, "d": d, "H": Hh, "N": Nn, "ms": statistics.median(st),
                    "kernel_ms": kms, "reference_autocast_ms": statistics.median(rt),
                    "roofline": {"bound": "tensor", "achieved": flops / (kms / 1e3) / 1e12, "peak": peak,
                                 "unit": "TFLOP/s", "frac": flops / (kms / 1e3) / 1e12 / peak,
                                 "peak_source": src, "alg_flops_per_launch": flops}})
    first = out[0]
    fl0 = first["roofline"]["alg_flops_per_launch"]
    line("EACS layer input projections (LayerNorm + proj_u/B/C, fp16 autocast) TFLOP/s", fl0 / (first["ms"] / 1e3) / 1e12,
         n, 3, first["ms"],
         {"workload": "LayerNorm + proj_u/B/C as one tcgen05 kernel (plus its row-statistics pass), "
                      "8 x 4096 rows, d = H = 768, N = 16", "cases": out, "l2": "flushed between steps"},
         unit="TFLOP/s", dtype="f16 x f16 -> f32",
         note="value: algorithmic flops / call time at config 1's rows and widths; cases[1] is config 2's widths; "
              "kernel_ms is the GEMM kernel alone; reference_autocast_ms the reference's sequence on the same tensors")
    return 0


def wl_query_train(args, dev, flush):
    """Training through per-frame commits and continuous-time queries
    (EACSLayer._commit_range + readout_from_commits under autograd,
    eacs.py:386-401, continuous_query.py:20-54) at config 1's widths: B = 8
    videos of L = 1024 frames, H = 768, N = 16 (--shape B,L,H,N), tau in [0.1, 1] s,
    Q = L query times per video, STE gate with the threshold at the median
    residual of an all-commit run (about half the frames commit).  One step =
    forward and backward of sum(y * gy) + sum(y_q * g_q) with respect to u,
    B, C, t, lam, log_dt, D, eps and the query times, from op-boundary tensors
    resident on the GPU.  The reference's own code (its step loop and
    autograd) runs on the same tensors on the same GPU when its package is
    present (one step: it takes seconds)."""
    import sys as _sys

    from eacs_b200.ops.continuous_query import QueryReadoutFunction, cell_commits_train, segment_index
    B, L, H, N = (8, 1024, 768, 16) if not args.shape else tuple(int(v) for v in args.shape.split(","))
    Q = L
    g = torch.Generator().manual_seed(0)
    d = cell_inputs(g, B, L, H, N, (0.1, 1.0), dev, torch.float32)
    tq = (d["t"][:, :1] - 0.2 + (d["t"][:, -1:] - d["t"][:, :1] + 0.4)
          * torch.rand(B, Q, generator=g).to(dev)).sort(1).values
    gy = torch.randn(B, L, H, generator=g).to(dev)
    gq = torch.randn(B, Q, H, generator=g).to(dev)
    from eacs_b200.ops.eacs_gated_scan import eacs_cell_forward
    _, _, r_all = eacs_cell_forward(d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"],
                                    d["mean"], d["var"], eps=0.0, eta=1e-6)
    eps0 = float(r_all.median())
    names = ("u", "Bc", "Cc", "t", "lam", "log_dt", "D")
    rate = []

    def ours():
        lv = {k: d[k].detach().requires_grad_(True) for k in names}
        eps = torch.tensor(eps0, device=dev, requires_grad=True)
        tqq = tq.detach().requires_grad_(True)
        ys, gs, rs, c = cell_commits_train(lv["lam"], lv["log_dt"], lv["u"], lv["Bc"], lv["Cc"], lv["t"],
                                           lv["D"], d["mean"], d["var"], eps, 1e-6, 0.1, "ste")
        yq = QueryReadoutFunction.apply(lv["lam"], lv["log_dt"], lv["D"], c["h"], c["t"], c["u"], c["B"],
                                        c["C"], tqq, segment_index(lv["t"].detach(), tq), 1e-3, 1e3)
        torch.autograd.backward([ys, yq], [gy, gq])
        if not rate:
            rate.append(float(gs.detach().mean()))

    n = max(3, min(args.steps, 10))
    st, _ = timed(ours, n, 2, flush, False)
    ms = statistics.median(st)
    updates = B * L * H * N
    ref_ms, ref_note = None, "reference package absent"
    root = None
    for cand in (os.environ.get("CST_SSM_REFERENCE"), os.path.join(ROOT, "baseline", "_ref")):
        if cand and os.path.isdir(os.path.join(cand, "cst_ssm")):
            root = cand
            break
    if root is not None:
        if root not in _sys.path:
            _sys.path.insert(0, root)
        from cst_ssm.modules.continuous_query import readout_from_commits
        from cst_ssm.modules.eacs import EACSLayer
        from cst_ssm.modules.event_gate import EventGate
        from cst_ssm.ops.spectral_init import BranchSpec
        torch.manual_seed(0)
        layer = EACSLayer(H, BranchSpec("short", N, 0.1, 1.0), gate=EventGate(init_eps=0.12)).to(dev).train()
        with torch.no_grad():
            layer.proj_out.weight.copy_(torch.eye(H))
            layer.proj_out.bias.zero_()
            layer.log_dt_scale.copy_(d["log_dt"])
            layer.D.copy_(d["D"])
            layer.obs_norm.running_mean.copy_(d["mean"])
            layer.obs_norm.running_var.copy_(d["var"])
        layer.gate.set_temperature(0.1)
        orig = layer.step_params

        def ref():
            lv = {k: d[k].detach().requires_grad_(True) for k in ("u", "Bc", "Cc", "t", "lam")}
            eps = torch.tensor(eps0, device=dev, requires_grad=True)

            def sp(lam, _o=orig):
                p = _o(lam)
                p.eps = eps
                return p
            layer.step_params = sp
            tqq = tq.detach().requires_grad_(True)
            state = (torch.zeros(B, H, N, dtype=torch.complex64, device=dev), lv["t"][:, 0] - layer.dt_init,
                     lv["u"][:, 0], lv["Bc"][:, 0], lv["Cc"][:, 0])
            ys, gs, rs, Hc, Tc, Uc, Bs, Cs = layer._commit_range(lv["lam"], state, lv["u"], lv["Bc"],
                                                                 lv["Cc"], lv["t"], 0, L)
            commits = dict(h=Hc, t=Tc, u=Uc, B=Bs, C=Cs, lam=lv["lam"], frame_t=lv["t"],
                           log_dt_scale=layer.log_dt_scale, dt_max=layer.dt_max)
            yq = readout_from_commits(layer, commits, tqq)
            torch.autograd.backward([ys, yq], [gy, gq])
        t0 = time.perf_counter()
        ref()
        torch.cuda.synchronize()
        ref_ms = (time.perf_counter() - t0) * 1e3
        ref_note = "the reference's _commit_range + readout_from_commits under autograd on the same GPU, one step (wall clock)"
    line("training through commits and queries (forward + backward), updates/s",
         updates / (ms / 1e3) / 1e9, n, 2, ms,
         {"workload": f"commit-training step, B={B} L={L} H={H} N={N}, Q={Q} query times a video, STE gate",
          "l2": "flushed between steps"},
         unit="Gupd/s", dtype="f32", update_rate=rate[0] if rate else None,
         reference_gpu_ms=ref_ms, speedup_vs_reference_gpu=(ref_ms / ms) if ref_ms else None,
         note="value: B*L*H*N / step time; " + ref_note)
    return 0


def wl_stream(args, dev, flush):
    """Streaming steps (temporal_step, streaming.py:45-85), one frame at a
    time through a MultiScaleEACS with config 2's three branch bands (tau in
    [0.5, 4], [4, 32], [32, 256] s, N = 16) at d = 1024, B = 4 videos, 64
    frames: inference (no autograd) and training (the STE gate, forward over
    the 64 frames then backward through the state), this library's
    temporal_step against the reference's own on the same module, inputs and
    GPU.  Needs the reference package (its module classes hold the
    parameters); timed on the device with CUDA events around the frame loop."""
    import sys as _sys
    root = None
    for cand in (os.environ.get("CST_SSM_REFERENCE"), os.path.join(ROOT, "baseline", "_ref")):
        if cand and os.path.isdir(os.path.join(cand, "cst_ssm")):
            root = cand
            break
    if root is None:
        print(json.dumps({"metric": "streaming frames/s", "unavailable": "reference package absent"}))
        return 0
    if root not in _sys.path:
        _sys.path.insert(0, root)
    from cst_ssm.modules.multiscale import MultiScaleEACS
    from cst_ssm.modules.streaming import initial_states
    from cst_ssm.modules.streaming import temporal_step as ref_step
    from cst_ssm.ops import eacs_gated_scan, scan_cuda
    from cst_ssm.ops.spectral_init import BranchSpec

    from eacs_b200.ops.streaming import temporal_step as our_step
    scan_cuda._EXT, scan_cuda._TRIED = None, True
    eacs_gated_scan._EXT, eacs_gated_scan._TRIED = None, True
    B, K, d = 4, 64, 1024
    torch.manual_seed(0)
    temporal = MultiScaleEACS(d, branches=[BranchSpec("short", 16, 0.5, 4.0), BranchSpec("mid", 16, 4.0, 32.0),
                                           BranchSpec("long", 16, 32.0, 256.0)],
                              gate_kwargs={"init_eps": 0.12}).to(dev)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(B, K, d, generator=g).to(dev)
    dt = 0.25 + 1.75 * torch.rand(B, K, generator=g)
    dt[torch.rand(B, K, generator=g) < 0.1] = 0.25
    t = torch.cumsum(dt, 1).to(dev)
    valid = torch.ones(B, K, dtype=torch.bool, device=dev)
    gy = torch.randn(B, K, d, generator=g).to(dev)

    def scan(step, train):
        states = initial_states(temporal, B, dev)
        ys, gs = [], []
        for k in range(K):
            y, gk, r, n, w, states = step(temporal, x[:, k], t[:, k], states, valid[:, k])
            ys.append(y)
            gs.append(gk)
        if train:
            (torch.stack(ys, 1) * gy).sum().backward()
        return torch.stack(gs, 1)

    def timed_scan(step, train, reps):
        temporal.train(train)
        out = []
        for i in range(reps + 1):
            temporal.zero_grad(set_to_none=True)
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            s0.record()
            with torch.set_grad_enabled(train):
                gates = scan(step, train)
            s1.record()
            torch.cuda.synchronize()
            if i:  # the first is a warm-up
                out.append(s0.elapsed_time(s1))
        return statistics.median(out), gates

    n = max(3, min(args.steps, 10))
    res = {}
    for train in (False, True):
        ours_ms, g_ours = timed_scan(our_step, train, n)
        ref_ms, g_ref = timed_scan(ref_step, train, 2)
        res["training" if train else "inference"] = {
            "ours_ms_per_frame": ours_ms / K, "reference_ms_per_frame": ref_ms / K,
            "speedup": ref_ms / ours_ms, "gates_equal": bool(torch.equal(g_ours.float(), g_ref.float())),
            "update_rate": float(g_ours.float().mean())}
    inf = res["inference"]
    line("streaming steps (temporal_step), frames/s over B videos", B / (inf["ours_ms_per_frame"] / 1e3), n, 1,
         inf["ours_ms_per_frame"] * K,
         {"workload": f"temporal_step frame by frame: MultiScaleEACS d={d}, three branches N=16 "
                      f"(config 2's bands), B={B} videos, {K} frames", "cases": res},
         unit="frames/s", dtype="f32",
         note="value: inference frames/s (B videos a frame); cases: per-frame device time of this "
              "library's temporal_step and of the reference's on the same module and GPU, inference "
              "and training (STE gate, forward over the frames then backward through the state)")
    return 0


def longvideo_inputs(rows, L, dev, seed, H=2048, N=32):
    """Long-video inputs (H=2048, N=32) for `rows` videos, drawn on the device from one seeded
    generator: fp16 u ~ N(0,1); B, C complex with N(0,1)/sqrt(N) parts;
    t = cumsum(dt), dt ~ Exp(mean 0.5 s) clipped to [1/30, 2] s; lambda with
    tau log-uniform on [0.5, 64] s and Im = pi*n; D ~ N(0,1)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    s = 1.0 / math.sqrt(N)

    def cplx(*shape):
        return torch.complex(torch.randn(*shape, device=dev, generator=g) * s,
                             torch.randn(*shape, device=dev, generator=g) * s)

    log_tau = torch.empty(H, N, device=dev).uniform_(math.log(0.5), math.log(64.0), generator=g)
    im = (math.pi * torch.arange(N, dtype=torch.float32, device=dev)).expand(H, N)
    dt = torch.empty(rows, L, device=dev).exponential_(1.0 / 0.5, generator=g).clamp_(1 / 30, 2.0)
    return dict(lam=torch.complex(-torch.exp(-log_tau), im.contiguous()),
                log_dt=torch.zeros(H, device=dev),
                u=torch.randn(rows, L, H, device=dev, dtype=torch.float16, generator=g),
                Bc=cplx(rows, L, N), Cc=cplx(rows, L, N), t=torch.cumsum(dt, 1),
                D=torch.randn(H, device=dev, generator=g), mean=torch.zeros(H, device=dev),
                var=torch.ones(H, device=dev))


def wl_longvideo(args):
    """Long-video gated cell: B=64 videos, H=2048, N=32, fp16 u,
    eps=0.12, L from --L (16384, 32768 or 65536).  The 64 videos are split
    over the ranks (strong scaling, no collective on the data path); time is
    device-measured, max over ranks."""
    import datetime
    import torch.distributed as dist
    from bench import ClockSampler, max_over_ranks
    from eacs_b200 import _lib
    from eacs_b200.ops.eacs_gated_scan import cell_forward_into, workspace_bytes
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    Bt, H, N = 64, 2048, 32
    L = args.L or 16384
    if getattr(args, "shape", None):  # a small case of the same kernel (for ncu)
        Bt, L, H, N = (int(v) for v in args.shape.split(","))
    if Bt % world:
        raise SystemExit(f"longvideo: {Bt} videos do not split over {world} ranks")
    rows = Bt // world
    d = longvideo_inputs(rows, L, dev, 4000 + rank, H, N)
    eps = 0.12 if args.eps is None else float(args.eps)
    y = torch.empty(rows, L, H, device=dev)
    gate = torch.empty(rows, L, device=dev)
    resid = torch.empty(rows, L, device=dev)
    ws = torch.empty(workspace_bytes(rows, L, H, N), dtype=torch.uint8, device=dev)

    def op():
        cell_forward_into(d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"], d["mean"],
                          d["var"], eps, 1e-6, 1e-5, 1.0, 1e-3, 1e3, None, "hard", 0.1, y, gate, resid, ws)

    steps = max(1, min(args.steps, 10))
    warmup = max(3, min(args.warmup, 5))
    sampler = ClockSampler(local)
    sampler.start()
    for _ in range(warmup):
        op()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    rate = float(gate.mean())
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in ev + kev:
        a.record()
        b.record()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.load = True
    launches0 = _lib.kernel_launches()
    for k in range(steps):
        ev[k][0].record()
        _lib.set_kernel_events(*kev[k])
        op()
        _lib.set_kernel_events(None, None)
        ev[k][1].record()
    torch.cuda.synchronize()
    sampler.load = False
    launches = _lib.kernel_launches() - launches0
    sampler.stop()
    total_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev), dev, world)
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
    assert _lib.device_status() == 0
    upd_rank = rows * L * H * N
    upd_job = Bt * L * H * N
    # algorithmic bytes of one launch: u fp16, Bc, Cc, t in; y fp32, gate, resid out
    alg = rows * L * (H * 2 + 2 * N * 8 + 4 + H * 4 + 8)
    peak, src = peak_hbm()
    achieved = alg / (kern_ms / 1e3) / 1e9
    # issue slots per update of cell_chain<SPEC> at H=2048, N=32 (ncu smsp__inst_executed.sum x 32
    # / updates on the 8 x 4096 case: 4,691,663,872 x 32 / 2,147,483,648); the kernel is issue-bound
    instr = 69.9 if (H, N) == (2048, 32) else None
    n_sm = torch.cuda.get_device_properties(dev).multi_processor_count
    issue_peak = n_sm * 4 * 32 * (sampler.summary().get("sm_mhz") or 1965.0) * 1e6
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({
            "metric": "EACS gated cell long-video Gstate-updates/s", "value": upd_job / (total_ms / 1e3 / steps) / 1e9,
            "unit": UNIT, "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": total_ms / steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded on the device)",
            "config": {"workload": "long-video gated cell (event gate + ZOH predict/update), videos split "
                       "over ranks", "B": Bt, "L": L, "H": H, "N": N, "u_dtype": "fp16", "eps": eps,
                       "update_rate": rate, "videos_per_rank": rows,
                       "l2": "inputs larger than L2 (no flush needed)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None, "peak_source": src,
                         "kernel": "cell_chain<SPEC> (rank 0)", "kernel_ms": kern_ms,
                         "alg_bytes_per_launch": alg,
                         "kernel_gupdates_per_s": upd_rank / (kern_ms / 1e3) / 1e9,
                         "issue": None if instr is None else {
                             "achieved_Tinstr_s": upd_rank / (kern_ms / 1e3) * instr / 1e12,
                             "peak_Tinstr_s": issue_peak / 1e12,
                             "frac": upd_rank / (kern_ms / 1e3) * instr / issue_peak,
                             "instr_per_update": instr,
                             "peak_basis": f"{n_sm} SMs x 128 lanes x median SM clock"}},
            "gpu_launches": launches, "clocks": sampler.summary()}), flush=True)
    return 0


def run_workload(args):
    if args.workload == "longvideo":
        return wl_longvideo(args)
    if args.workload == "train":
        return wl_train(args)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit(f"--workload {args.workload} runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    {"scan": wl_scan, "ssm": wl_ssm, "ssm_train": wl_ssm_train,
     "multiscale": wl_multiscale, "project": wl_project, "query_train": wl_query_train,
     "stream": wl_stream}[args.workload](
        args, dev, flush)
    from eacs_b200 import _lib
    assert _lib.device_status() == 0
    return 0
