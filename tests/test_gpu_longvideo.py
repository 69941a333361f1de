"""The gated cell at the long-video width (64 videos, H=2048, N=32, fp16 u,
eps=0.12, L=16384) against the oracle.

The full-size run is too long for the CPU oracle, so it is checked through
properties that hold at any size: the cell is causal (the first K steps of a
row depend only on that row's first K inputs, so the oracle on a prefix must
agree with the prefix of the full run) and rows are independent (a row run on
its own equals the same row inside the batch, bit for bit).  The skip and
repair path at this width is checked against the oracle on a short case with
a calibrated threshold.
"""
import numpy as np
import pytest
import torch

from golden_io import decisive, relerr
from inputs import cell_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
H, N = 2048, 32

if torch.cuda.is_available():
    from eacs_b200.ops.eacs_gated_scan import eacs_cell_forward


def _inputs(rows, L, seed):
    from bench_workloads import longvideo_inputs
    return longvideo_inputs(rows, L, torch.device(DEV), seed, H, N)


def _run(d, eps, sl=slice(None)):
    return eacs_cell_forward(d["lam"], d["log_dt"], d["u"][sl], d["Bc"][sl], d["Cc"][sl], d["t"][sl],
                             d["D"], d["mean"], d["var"], eps=eps, eta=1e-6)


def _host(d, rows, K):
    out = {}
    for k, v in d.items():
        if k in ("u", "Bc", "Cc", "t"):
            v = v[rows, :K]
        out[k] = v.float().cpu().numpy() if not v.is_complex() else v.cpu().numpy()
    return out


def test_longvideo_full_size_prefix_and_rows():
    B, L, K = 64, 16384, 96
    d = _inputs(B, L, 4000)
    y, g, r = _run(d, 0.12)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all() and torch.isfinite(r).all()
    rows = [0, 31, 63]
    ref = oracle.cell_fwd(**_host(d, rows, K), eps=0.12, eta=1e-6)
    yk, gk, rk = (x[rows, :K].cpu().numpy() for x in (y, g, r))
    keep = decisive(ref[2], 0.12, None)
    assert np.array_equal(gk[keep], ref[1][keep])
    assert relerr(yk, ref[0]) < 1e-4 and relerr(rk, ref[2]) < 1e-4
    # one row on its own: the same bits as inside the batch
    y1, g1, r1 = _run(d, 0.12, slice(7, 8))
    assert torch.equal(y1, y[7:8]) and torch.equal(g1, g[7:8]) and torch.equal(r1, r[7:8])


@pytest.mark.parametrize("rate", [0.5, 0.85])
def test_longvideo_width_with_skips(rate):
    from test_gpu_kernels import _calibrated_eps
    d = cell_inputs(2, 160, H, N, seed=int(rate * 100) + 7, tau=(0.5, 64.0))
    d["u"] = d["u"].astype(np.float16).astype(np.float32)
    eps = _calibrated_eps(d, rate)
    ref = oracle.cell_fwd(**d, eps=eps, eta=1e-6)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(DEV) for k, v in d.items()}
    t["u"] = t["u"].half()
    y, g, r = (x.cpu().numpy() for x in _run(t, eps))
    assert np.array_equal(g, ref[1])
    assert relerr(y, ref[0]) < 1e-4 and relerr(r, ref[2]) < 1e-4
    assert 0.0 < g.mean() < 1.0
