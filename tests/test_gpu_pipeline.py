"""The gated cell over host buffers in pipelined time chunks
(eacs_cell_fwd_host) against the device call on the whole sequence and the
oracle.

Rows resume from the carried state at every chunk boundary.  Where every frame
commits the result is bit-identical to one device call; with skips the repair
pass and the speculative pass sum the readout and residual in different
orders, so y and resid agree to 1e-5 relative and the gates exactly on every
step decided by more than 1e-5.
"""
import numpy as np
import pytest
import torch

from golden_io import relerr
from inputs import cell_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

if torch.cuda.is_available():
    from eacs_b200.ops.eacs_gated_scan import eacs_cell_forward, eacs_cell_forward_host


def _dev(d, k):
    return torch.from_numpy(np.ascontiguousarray(d[k])).to(DEV)


def _host(d, k, pinned=True):
    x = torch.from_numpy(np.ascontiguousarray(d[k]))
    return x.pin_memory() if pinned else x


def _run_host(d, eps, chunk, robust=None, u_dtype=torch.float32, pinned=True):
    u = _host(d, "u", pinned).to(u_dtype)
    u = u.pin_memory() if pinned else u
    out = eacs_cell_forward_host(_dev(d, "lam"), _dev(d, "log_dt"), u, _host(d, "Bc", pinned),
                                 _host(d, "Cc", pinned), _host(d, "t", pinned), _dev(d, "D"),
                                 _dev(d, "mean"), _dev(d, "var"), eps, 1e-6, robust=robust,
                                 chunk=chunk)
    torch.cuda.synchronize()
    return tuple(x.numpy() for x in out)


def _run_dev(d, eps, robust=None, u_dtype=torch.float32):
    out = eacs_cell_forward(_dev(d, "lam"), _dev(d, "log_dt"), _dev(d, "u").to(u_dtype), _dev(d, "Bc"),
                            _dev(d, "Cc"), _dev(d, "t"), _dev(d, "D"), _dev(d, "mean"),
                            _dev(d, "var"), eps=eps, eta=1e-6, robust=robust)
    return tuple(x.cpu().numpy() for x in out)


@pytest.mark.parametrize("B,L,H,N,chunk", [(3, 300, 96, 16, 64), (2, 256, 768, 16, 32),
                                           (2, 100, 40, 32, 512), (4, 97, 24, 5, 32),
                                           (8, 256, 768, 16, 64)])  # 8 rows of 768: wide speculative pass
def test_host_pipeline_all_commit_bit_exact(B, L, H, N, chunk):
    d = cell_inputs(B, L, H, N, seed=B * L + H)
    host = _run_host(d, 0.12, chunk)
    dev = _run_dev(d, 0.12)
    assert dev[1].min() == 1.0  # every frame commits
    for a, b in zip(host, dev):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("rate,robust,u_dtype", [(0.5, None, torch.float32),
                                                 (0.2, None, torch.bfloat16),
                                                 (0.6, (3, 2.0, 0.3), torch.float32),
                                                 (0.5, (1, 1.05, 0.5), torch.float32)])
def test_host_pipeline_with_skips(rate, robust, u_dtype):
    from test_gpu_kernels import _calibrated_eps
    B, L, H, N = 2, 200, 64, 16
    d = cell_inputs(B, L, H, N, seed=int(rate * 100))
    if u_dtype != torch.float32:
        d["u"] = torch.from_numpy(d["u"]).to(u_dtype).float().numpy()
    eps = _calibrated_eps(d, rate, robust)
    host = _run_host(d, eps, 32, robust, u_dtype)
    ref = oracle.cell_fwd(**d, eps=eps, eta=1e-6, robust=robust)
    dev = _run_dev(d, eps, robust, u_dtype)
    assert np.array_equal(host[1], ref[1]) and np.array_equal(dev[1], ref[1])
    assert relerr(host[0], ref[0]) < 1e-4 and relerr(host[2], ref[2]) < 1e-4
    assert relerr(host[0], dev[0]) < 1e-5 and relerr(host[2], dev[2]) < 1e-5
    assert 0.0 < host[1].mean() < 1.0


def test_host_pipeline_pageable():
    d = cell_inputs(2, 70, 32, 8, seed=9)
    host = _run_host(d, 0.12, 32, pinned=False)
    dev = _run_dev(d, 0.12)
    for a, b in zip(host, dev):
        assert np.array_equal(a, b)


def test_host_pipeline_wide_rows_with_skips():
    """H=2048, N=32 rows (too wide for the cluster repair pass): the one-CTA
    repair pass resumes them from the carried state at every chunk."""
    from test_gpu_kernels import _calibrated_eps
    d = cell_inputs(2, 64, 2048, 32, seed=21, tau=(0.5, 64.0))
    eps = _calibrated_eps(d, 0.5)
    host = _run_host(d, eps, 16)
    ref = oracle.cell_fwd(**d, eps=eps, eta=1e-6)
    dev = _run_dev(d, eps)
    assert np.array_equal(host[1], ref[1]) and np.array_equal(dev[1], ref[1])
    assert relerr(host[0], ref[0]) < 1e-4 and relerr(host[2], ref[2]) < 1e-4
    assert relerr(host[0], dev[0]) < 1e-5 and relerr(host[2], dev[2]) < 1e-5
    assert 0.0 < host[1].mean() < 1.0


def test_host_pipeline_one_cta_per_sm_with_skips():
    """8 rows of 768 channels (the speculative pass in one 11-warp CTA per SM)
    with skips: every chunk resumes from the carried state the wide pass or the
    repair pass left."""
    from test_gpu_kernels import _calibrated_eps
    B, L, H, N = 8, 96, 768, 16
    d = cell_inputs(B, L, H, N, seed=77)
    eps = _calibrated_eps(d, 0.5)
    host = _run_host(d, eps, 32)
    ref = oracle.cell_fwd(**d, eps=eps, eta=1e-6)
    dev = _run_dev(d, eps)
    assert np.array_equal(host[1], ref[1]) and np.array_equal(dev[1], ref[1])
    assert relerr(host[0], ref[0]) < 1e-4 and relerr(host[2], ref[2]) < 1e-4
    assert relerr(host[0], dev[0]) < 1e-5 and relerr(host[2], dev[2]) < 1e-5
    assert 0.0 < host[1].mean() < 1.0
