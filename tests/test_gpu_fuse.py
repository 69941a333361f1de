"""Fused MultiScaleEACS branch epilogue (eacs_branch_fuse) against a plain
PyTorch float32 restatement of multiscale.py:176-179 on the same inputs.

Tolerances (max |x - ref| / max |ref|): float32 inputs 1e-5; float16 and
bfloat16 outputs are one rounding of the float32 result, so 2^-10 and 2^-7.
"""
from dataclasses import dataclass

import pytest
import torch
from torch import nn

from golden_io import relerr

pytestmark = pytest.mark.gpu
DEV = "cuda:0"

if torch.cuda.is_available():
    from eacs_b200.ops.multiscale import branch_fuse, multiscale_forward


@torch.no_grad()
def _ref(x, deltas, fusion, norm):
    x32 = x.float()
    w = torch.softmax(x32 @ fusion.weight.float().t() + (0 if fusion.bias is None else fusion.bias.float()), -1)
    fused = sum(w[..., s:s + 1] * deltas[s].float() for s in range(len(deltas)))
    v = x32 + fused
    y = torch.nn.functional.layer_norm(v, (x.shape[-1],), norm.weight.float() if norm.weight is not None else None,
                                       norm.bias.float() if norm.bias is not None else None, norm.eps)
    return y, w


@pytest.mark.parametrize("d,S,dtype,tol", [(64, 3, torch.float32, 1e-5), (1024, 3, torch.bfloat16, 2 ** -7),
                                           (2048, 2, torch.bfloat16, 2 ** -7), (768, 1, torch.float16, 2 ** -10),
                                           (1024, 8, torch.float32, 1e-5), (40, 3, torch.float16, 2 ** -10)])
def test_branch_fuse(d, S, dtype, tol):
    g = torch.Generator().manual_seed(d + S)
    B, L = 2, 37
    x = torch.randn(B, L, d, generator=g).to(DEV, dtype)
    deltas = [torch.randn(B, L, d, generator=g).to(DEV, dtype) for _ in range(S)]
    fusion = nn.Linear(d, S).to(DEV)
    norm = nn.LayerNorm(d).to(DEV)
    with torch.no_grad():
        norm.weight.normal_(1.0, 0.2)
        norm.bias.normal_(0.0, 0.2)
    y, w = branch_fuse(x, deltas, fusion, norm)
    y_ref, w_ref = _ref(x, deltas, fusion, norm)
    assert y.dtype == dtype and y.shape == x.shape and w.shape == (B, L, S)
    assert relerr(w.cpu().numpy(), w_ref.cpu().numpy()) < 1e-5
    assert relerr(y.float().cpu().numpy(), y_ref.cpu().numpy()) < tol


@dataclass
class _Out:  # the fields MultiScaleEACS.forward reads from each branch (eacs.py EACSOutput)
    y: torch.Tensor
    gates: torch.Tensor
    update_rate: torch.Tensor
    residual: torch.Tensor
    innovation: torch.Tensor = None


@dataclass
class MultiScaleOutput:  # cst_ssm/modules/multiscale.py:17-24
    y: torch.Tensor
    gates: torch.Tensor
    update_rate: torch.Tensor
    per_branch_update_rate: torch.Tensor
    fusion_weights: torch.Tensor
    residual: torch.Tensor
    innovation: torch.Tensor = None


class _Branch(nn.Module):
    def __init__(self, k):
        super().__init__()
        self.k = k

    def forward(self, x, t, cpi=None, frame_mask=None):
        g = (torch.arange(x.shape[1], device=x.device) % (self.k + 2) != 0).float().expand(x.shape[0], -1)
        return _Out(y=torch.tanh(x * (self.k + 1)), gates=g, update_rate=g.mean(),
                    residual=g * 0.5, innovation=g * 0.25)


class _Temporal(nn.Module):
    def __init__(self, d, S):
        super().__init__()
        self.branches = nn.ModuleList([_Branch(k) for k in range(S)])
        self.n_branch = S
        self.fusion = nn.Linear(d, S)
        self.out_norm = nn.LayerNorm(d)

    def _merge_ok(self, x):
        return False


def test_multiscale_forward_epilogue():
    B, L, d, S = 2, 30, 256, 3
    temporal = _Temporal(d, S).to(DEV)
    x = torch.randn(B, L, d, device=DEV)
    out = multiscale_forward(temporal, x, torch.zeros(B, L, device=DEV))
    outs = [br(x, None) for br in temporal.branches]
    deltas = torch.stack([o.y for o in outs], -1)
    w = torch.softmax(temporal.fusion(x), -1)
    y_ref = temporal.out_norm(x + torch.einsum("bldn,bln->bld", deltas, w))
    assert relerr(out.y.cpu().numpy(), y_ref.detach().cpu().numpy()) < 1e-5
    assert relerr(out.fusion_weights.cpu().numpy(), w.detach().cpu().numpy()) < 1e-5
    assert out.gates.shape == (B, S, L) and out.innovation.shape == (B, S, L)
    assert torch.allclose(out.per_branch_update_rate, torch.stack([o.update_rate for o in outs]))
