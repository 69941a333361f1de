"""Parity at the full sizes the benchmarks time, on the benchmarks' own inputs.

Every workload of bench.py / bench_workloads.py is run here at its full shape
through the same entry points the benchmark times, and compared with the CPU
oracle (oracle/eacs_oracle.c, pinned to the reference's PyTorch code by
tests/golden/) over whole rows:

* gated cell inference, B=8 L=4096 H=768 N=16, fp16 u, eps=0.12, tau band
  [0.1, 1] s (bench.py's headline), through the device call and through the
  host-buffer call that bench.py's end-to-end figure times;
* the three MultiScaleEACS branches, B=4 L=16384 H=1024 N=16, bf16 u, tau
  bands [0.5,4], [4,32], [32,256] s, launched side by side as timed;
* the long-video cell, 64 videos x L in {16384, 32768, 65536}, H=2048, N=32,
  fp16 u: all 64 rows run on the device, the first and the last row (the
  largest offsets) compared in full;
* gated-cell training, 2 videos x L=8192, H=768, N=16, bf16 u: every gradient
  of GatedEACSCellFunction against the oracle's double-precision backward.

Tolerances: forward outputs 1e-4 relative (max |x - ref| / max |ref| per
row), gate masks bit-exact wherever the residual is more than 1e-5 from its
threshold, gradients 1e-3 relative per tensor.  du is returned in u's dtype
(bf16), so its bound adds bf16's rounding of each element (2^-8 |ref|).
"""
import numpy as np
import pytest
import torch

from golden_io import assert_cell_match, relerr
from oracle import oracle

pytestmark = pytest.mark.gpu

FWD_TOL = 1e-4
GRAD_TOL = 1e-3
DEV = "cuda:0"


def _np(x):
    x = x.detach()
    if x.is_complex():
        return x.cpu().numpy()
    return x.float().cpu().numpy()


def _oracle_cell(d, eps, dt_max=1e3, rows=None):
    h = {k: _np(v if rows is None or k not in ("u", "Bc", "Cc", "t") else v[rows]) for k, v in d.items()}
    oracle.set_threads(0)
    return oracle.cell_fwd(h["lam"], h["log_dt"], h["u"], h["Bc"], h["Cc"], h["t"], h["D"], h["mean"],
                           h["var"], eps, 1e-6, 1e-5, 1.0, 1e-3, dt_max)


def _device_cell(d, eps, dt_max=1e3):
    from eacs_b200.ops.eacs_gated_scan import cell_forward_into, workspace_bytes
    B, L, H = d["u"].shape
    N = d["lam"].shape[1]
    y = torch.empty(B, L, H, device=DEV)
    g = torch.empty(B, L, device=DEV)
    r = torch.empty(B, L, device=DEV)
    ws = torch.empty(workspace_bytes(B, L, H, N), dtype=torch.uint8, device=DEV)
    cell_forward_into(d["lam"], d["log_dt"], d["u"], d["Bc"], d["Cc"], d["t"], d["D"], d["mean"],
                      d["var"], eps, 1e-6, 1e-5, 1.0, 1e-3, dt_max, None, "hard", 0.1, y, g, r, ws)
    return y, g, r


def test_gated_cell_inference_b8_l4096_h768_n16():
    """bench.py's headline workload: the device call (value) and the
    host-buffer call (e2e) both equal the oracle over all 8 x 4096 frames."""
    import bench
    from eacs_b200 import _lib
    from eacs_b200.ops.eacs_gated_scan import eacs_cell_forward_host
    d, eps = bench.make_inputs(0, torch.device(DEV))
    assert d["u"].shape == (8, 4096, 768) and d["lam"].shape == (768, 16)
    ref = _oracle_cell(d, eps, bench.DT_MAX)
    got = [_np(x) for x in _device_cell(d, eps, bench.DT_MAX)]
    assert assert_cell_match(got, ref, eps, None) == 8 * 4096
    pin = {k: d[k].cpu().pin_memory() for k in ("u", "Bc", "Cc", "t")}
    out = [torch.empty(8, 4096, 768).pin_memory(), torch.empty(8, 4096).pin_memory(),
           torch.empty(8, 4096).pin_memory()]
    eacs_cell_forward_host(d["lam"], d["log_dt"], pin["u"], pin["Bc"], pin["Cc"], pin["t"], d["D"],
                           d["mean"], d["var"], eps, bench.ETA, bench.VAR_EPS, bench.DT_INIT,
                           bench.DT_MIN, bench.DT_MAX, chunk=bench.E2E_CHUNK, out=out)
    torch.cuda.synchronize()
    assert assert_cell_match([o.numpy() for o in out], ref, eps, None) == 8 * 4096
    assert _lib.device_status() == 0


def test_multiscale_branches_b4_l16384_h1024_n16():
    """The three branch cells of the multiscale workload, side by side on
    their streams as bench_workloads.wl_multiscale runs them."""
    from bench_workloads import MULTISCALE_BANDS, multiscale_inputs
    from eacs_b200 import _lib
    from eacs_b200.ops.multiscale import run_branches
    _, br = multiscale_inputs(torch.device(DEV))
    dt_max = [max(1e3, 10 * tb[1]) for tb in MULTISCALE_BANDS]
    outs = run_branches(br, torch.device(DEV), lambda i, d: _device_cell(d, 0.12, dt_max[i]))
    torch.cuda.synchronize()
    for i, (d, o) in enumerate(zip(br, outs)):
        ref = _oracle_cell(d, 0.12, dt_max[i])
        assert assert_cell_match([_np(x) for x in o], ref, 0.12, None) == 4 * 16384, f"branch {i}"
    assert _lib.device_status() == 0


@pytest.mark.parametrize("L", [16384, 32768, 65536])
def test_long_video_b64_h2048_n32(L):
    """All 64 videos run in one call (u alone is 64 x L x 2048 fp16: 17 GB at
    L=65536); rows 0 and 63 are compared with the oracle in full."""
    from bench_workloads import longvideo_inputs
    from eacs_b200 import _lib
    d = longvideo_inputs(64, L, torch.device(DEV), 4000)
    y, g, r = _device_cell(d, 0.12)
    torch.cuda.synchronize()
    rows = [0, 63]
    got = [_np(x[rows]) for x in (y, g, r)]
    del y, g, r
    ref = _oracle_cell(d, 0.12, rows=rows)
    assert assert_cell_match(got, ref, 0.12, None) == 2 * L
    assert _lib.device_status() == 0


def test_gated_cell_training_b2_l8192_h768_n16():
    """The training workload's first two videos at full length: forward
    values and all eight gradients of GatedEACSCellFunction (through
    fused_gated_scan, as timed) against the oracle's backward."""
    from bench_workloads import train_inputs
    from eacs_b200 import _lib
    from eacs_b200.ops.eacs_cell_train import fused_gated_scan
    d, gy = train_inputs(0, "cpu")
    d = {k: (v[:2].contiguous() if k in ("u", "Bc", "Cc", "t") else v) for k, v in d.items()}
    gy = gy[:2].contiguous()
    dev = {k: v.to(DEV) for k, v in d.items()}
    leaves = {k: dev[k].clone().requires_grad_(True) for k in ("u", "Bc", "Cc", "t", "lam", "log_dt", "D")}
    eps = torch.tensor(0.12, device=DEV, requires_grad=True)
    y, gs, rs = fused_gated_scan(leaves["u"], leaves["Bc"], leaves["Cc"], leaves["t"], leaves["lam"],
                                 leaves["log_dt"], leaves["D"], eps, dev["mean"], dev["var"], 0.1, 1e-6)
    order = ("u", "Bc", "Cc", "t", "lam", "log_dt", "D")
    grads = torch.autograd.grad([y], [leaves[k] for k in order] + [eps], [gy.to(DEV)])
    h = {k: _np(v) for k, v in d.items()}
    oracle.set_threads(0)
    y_ref, g_ref, _ = oracle.cell_fwd(h["lam"], h["log_dt"], h["u"], h["Bc"], h["Cc"], h["t"], h["D"],
                                      h["mean"], h["var"], 0.12, 1e-6, train_exp=True)
    assert relerr(_np(y), y_ref) < FWD_TOL
    assert np.array_equal(_np(gs), g_ref)
    ref = oracle.cell_bwd(h["lam"], h["log_dt"], h["u"], h["Bc"], h["Cc"], h["t"], h["D"], h["mean"],
                          h["var"], 0.12, 1e-6, 1e-5, 1.0, 1e3, 0.1, 0, _np(gs), _np(gy))
    names = ("du", "dBc", "dCc", "dt", "dlam", "dlog_dt", "dD", "deps")
    for k, v, rv in zip(names, grads, ref):
        v = _np(v).reshape(rv.shape)
        if k == "du":
            assert grads[0].dtype == torch.bfloat16
            bound = GRAD_TOL * np.abs(rv).max() + 2.0 ** -8 * np.abs(rv)
            assert np.all(np.abs(v - rv) <= bound), k
        else:
            assert relerr(v, rv) < GRAD_TOL, (k, relerr(v, rv))
    assert _lib.device_status() == 0
