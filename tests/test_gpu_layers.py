"""Layer-level drop-ins on the GPU: EACSLayer's fused dispatch with robust_guard
(eacs_b200.ops.eacs_layer) and ContinuousSSMLayer.forward with the fused
ungated core (eacs_b200.ops.continuous_ssm.layer_forward), driven through
stand-in layer objects that carry the reference layers' attributes (the
reference package itself is not needed), against the oracle.

Tolerance: 1e-4 relative on the core outputs; gates bit-exact away from the
threshold; gradients 1e-3 relative.
"""
from dataclasses import dataclass

import numpy as np
import pytest
import torch
from torch import nn

from golden_io import relerr
from inputs import cell_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@dataclass
class EACSOutput:  # the reference's result type (cst_ssm/modules/eacs.py:33-38)
    y: torch.Tensor
    gates: torch.Tensor
    update_rate: torch.Tensor
    residual: torch.Tensor
    innovation: torch.Tensor = None


class _Std(nn.Module):
    def __init__(self, mean, var):
        super().__init__()
        self.register_buffer("running_mean", mean)
        self.register_buffer("running_var", var)
        self.eps = 1e-5


class _Gate(nn.Module):
    def __init__(self, eps):
        super().__init__()
        self.eps = torch.tensor(eps)
        self.norm_eta = 1e-6
        self.gate_kind = "event"
        self.cpi_modulation = 0.0


class StandInLayer(nn.Module):
    """Identity norm and projections so the core's inputs are the test's own."""

    def __init__(self, d, robust):
        super().__init__()
        self.N = d["lam"].shape[1]
        self.lam_c = torch.from_numpy(d["lam"]).to(DEV)
        self.log_dt_scale = torch.from_numpy(d["log_dt"]).to(DEV)
        self.D = torch.from_numpy(d["D"]).to(DEV)
        self.obs_norm = _Std(torch.from_numpy(d["mean"]).to(DEV), torch.from_numpy(d["var"]).to(DEV))
        self.gate = _Gate(d["eps"])
        self.disc_mode = "continuous"
        self.dt_init, self.dt_max = 1.0, 1e3
        self.robust_guard = robust is not None
        self.robust_k, self.robust_spike_ratio, self.robust_eps_factor = robust or (3, 2.0, 0.3)
        self.add_residual = False
        self.Bc = torch.from_numpy(d["Bc"]).to(DEV)
        self.Cc = torch.from_numpy(d["Cc"]).to(DEV)
        self.norm = nn.Identity()
        self.proj_out = nn.Identity()

    def lam(self):
        return self.lam_c

    def _project(self, x):
        return x.float(), self.Bc, self.Cc


@pytest.mark.parametrize("robust", [None, (3, 2.0, 0.3)])
def test_eacs_layer_forward_fused(robust):
    from eacs_b200.ops.eacs_layer import cuda_fused_ok, forward_fused
    from test_gpu_kernels import _calibrated_eps, assert_cell_match

    d = cell_inputs(2, 60, 64, 16, seed=31)
    eps = _calibrated_eps(d, 0.5, robust)
    layer = StandInLayer(dict(d, eps=eps), robust).eval()
    x = torch.from_numpy(d["u"]).to(DEV)
    t = torch.from_numpy(d["t"]).to(DEV)
    assert cuda_fused_ok(layer, x)
    out = forward_fused(layer, x, t)
    assert isinstance(out, EACSOutput)
    ref = oracle.cell_fwd(**d, eps=eps, eta=1e-6, robust=robust)
    got = tuple(v.cpu().numpy() for v in (out.y, out.gates, out.residual))
    assert_cell_match(got, ref, eps, robust)
    assert 0.0 < float(out.update_rate) < 1.0
    assert torch.equal(out.innovation, out.residual)


def test_continuous_ssm_layer_forward_and_grads():
    from eacs_b200.ops.continuous_ssm import layer_forward

    class UngatedStandIn(nn.Module):
        def __init__(self, d):
            super().__init__()
            self.N = d["lam"].shape[1]
            lam = torch.from_numpy(d["lam"])
            self.a_log_neg_real = nn.Parameter(torch.log(-lam.real).to(DEV))
            self.a_imag = nn.Parameter(lam.imag.clone().to(DEV))
            self.log_dt_scale = nn.Parameter(torch.from_numpy(d["log_dt"]).to(DEV))
            self.D = nn.Parameter(torch.from_numpy(d["D"]).to(DEV))
            self.Bc = torch.from_numpy(d["Bc"]).to(DEV)
            self.Cc = torch.from_numpy(d["Cc"]).to(DEV)
            self.norm = nn.Identity()
            self.proj_u = nn.Identity()
            self.proj_out = nn.Identity()
            self.add_residual = False
            N = self.N

            class _Split(nn.Module):
                def __init__(self, c):
                    super().__init__()
                    self.c = c

                def forward(self, x):
                    return torch.cat([self.c.real, self.c.imag], -1)

            self.proj_B = _Split(self.Bc)
            self.proj_C = _Split(self.Cc)
            assert N == self.Bc.shape[-1]

    B, L, H, N = 2, 130, 24, 8
    d = cell_inputs(B, L, H, N, seed=41, tau=(0.5, 64.0))
    layer = UngatedStandIn(d)
    x = torch.from_numpy(d["u"]).to(DEV).requires_grad_(True)
    t = torch.from_numpy(d["t"]).to(DEV)
    y = layer_forward(layer, x, t)
    y_ref = oracle.ssm_fwd(d["lam"], d["log_dt"], d["t"], d["Bc"], d["Cc"], d["u"], d["D"])
    assert relerr(y.detach().cpu().numpy(), y_ref) < 1e-4
    gy = np.random.default_rng(0).standard_normal((B, L, H)).astype(np.float32)
    y.backward(torch.from_numpy(gy).to(DEV))
    du, _, _, _, dlam, dlog, dD = oracle.ssm_bwd(d["lam"], d["log_dt"], d["t"], d["Bc"], d["Cc"],
                                                 d["u"], d["D"], gy)
    assert relerr(x.grad.cpu().numpy(), du) < 1e-3
    assert relerr(layer.log_dt_scale.grad.cpu().numpy(), dlog) < 1e-3
    assert relerr(layer.D.grad.cpu().numpy(), dD) < 1e-3
    # a_imag's gradient is Im(dlam); a_log_neg_real's is Re(dlam) * d(-exp(a))/da
    assert relerr(layer.a_imag.grad.cpu().numpy(), dlam.imag) < 1e-3
    lam_re = d["lam"].real
    assert relerr(layer.a_log_neg_real.grad.cpu().numpy(), dlam.real * lam_re) < 1e-3


def test_run_with_commits_and_continuous_query():
    from eacs_b200.ops.continuous_query import (continuous_query, readout_from_commits,
                                                run_with_commits)
    from test_gpu_kernels import _calibrated_eps

    d = cell_inputs(2, 50, 32, 16, seed=51)
    eps = _calibrated_eps(d, 0.5)
    layer = StandInLayer(dict(d, eps=eps), None).eval()
    x = torch.from_numpy(d["u"]).to(DEV)
    t = torch.from_numpy(d["t"]).to(DEV)
    out, commits = run_with_commits(layer, x, t)
    ref = oracle.cell_commits(**d, eps=eps, eta=1e-6)
    assert isinstance(out, EACSOutput) and out.innovation is None
    assert np.array_equal(out.gates.cpu().numpy(), ref[1])
    assert relerr(out.y.cpu().numpy(), ref[0]) < 1e-4
    for k, r in zip(("h", "t", "u", "B", "C"), ref[3:]):
        assert relerr(commits[k].cpu().numpy(), r) < 1e-4, k
    tq = t[:, :20] + 0.07
    yq = readout_from_commits(layer, commits, tq)
    yq_ref = oracle.query_readout(d["lam"], d["log_dt"], d["D"], *ref[3:], d["t"], tq.cpu().numpy())
    assert relerr(yq.cpu().numpy(), yq_ref) < 1e-4
    assert torch.equal(continuous_query(layer, x, t, tq), yq)
    # queries at the frame times themselves use each frame's own commits
    yf = readout_from_commits(layer, commits, commits["frame_t"])
    B, L = d["t"].shape
    idx = np.broadcast_to(np.arange(L, dtype=np.int32), (B, L))
    yf_ref = oracle.query_readout(d["lam"], d["log_dt"], d["D"], *ref[3:], d["t"], d["t"], idx=idx)
    assert relerr(yf.cpu().numpy(), yf_ref) < 1e-4
