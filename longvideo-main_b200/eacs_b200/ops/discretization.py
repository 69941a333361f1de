"""ZOH discretisation on B200 (mirrors cst_ssm/ops/discretization.py:20-54).

`zoh_kernels(lam, dt)` returns (dA, dB_bar) like the reference function, from
one elementwise kernel; `zoh_discretize` applies B as zoh_apply_B does.  The
fused scan/cell kernels compute the same values in registers instead.
"""
from __future__ import annotations

import torch
from torch import Tensor

from .. import _lib
from ._check import cuda_tensors, require


@torch.no_grad()
def zoh_kernels(lam: Tensor, dt: Tensor, inv_lam: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """lam (H,N) complex, dt (*,H) -> dA, dB_bar (*,H,N) complex64.

    inv_lam is accepted for signature compatibility; the kernel forms 1/lam itself.
    """
    dev = cuda_tensors("zoh_kernels", lam, dt)
    require(lam.dim() == 2 and dt.shape[-1] == lam.shape[0], "zoh_kernels: lam (H,N), dt (*,H)")
    H, N = lam.shape
    lead = dt.shape[:-1]
    lam_c = lam.to(torch.complex64).contiguous()
    dt_c = dt.float().reshape(-1, H).contiguous()
    M = dt_c.shape[0]
    dA = torch.empty(*lead, H, N, dtype=torch.complex64, device=dev)
    dB = torch.empty_like(dA)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().eacs_zoh_kernels(lam_c.data_ptr(), dt_c.data_ptr(), dA.data_ptr(),
                                               dB.data_ptr(), M, H, N, _lib.stream_ptr(dev)),
                   "eacs_zoh_kernels")
    return dA, dB


def zoh_apply_B(dB_bar: Tensor, B: Tensor) -> Tensor:
    """dB = dB_bar * B (discretization.py:39-44)."""
    B_e = B.unsqueeze(-2)
    if not torch.is_complex(B_e):
        B_e = B_e.to(dB_bar.dtype)
    return dB_bar * B_e


def zoh_discretize(lam: Tensor, dt: Tensor, B: Tensor,
                   inv_lam: Tensor | None = None) -> tuple[Tensor, Tensor]:
    dA, dB_bar = zoh_kernels(lam, dt, inv_lam)
    return dA, zoh_apply_B(dB_bar, B)
