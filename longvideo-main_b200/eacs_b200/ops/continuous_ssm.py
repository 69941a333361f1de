"""Fused ungated continuous SSM core (cst_ssm/modules/continuous_ssm.py:44-55).

`ssm_forward` replaces, inside ContinuousSSMLayer.forward, the chain
dt -> effective_dt -> zoh_discretize -> dB*u -> selective_scan -> readout
with one kernel that keeps every (b, h, n) state in registers: no (B,L,H,N)
tensor is materialised.  Inference only (no autograd).
"""
from __future__ import annotations

import torch
from torch import Tensor

from .. import _lib
from ._check import cuda_tensors, require


@torch.no_grad()
def ssm_forward(lam: Tensor, log_dt_scale: Tensor, timestamps: Tensor, Bc: Tensor, Cc: Tensor,
                u: Tensor, D: Tensor, dt_min: float = 1e-3, dt_max: float = 1e3) -> Tensor:
    """y (B,L,H) fp32 = Re sum_n C_l h_l + D u with h the ZOH scan of (dB_bar B) u."""
    dev = cuda_tensors("ssm_forward", lam, log_dt_scale, timestamps, Bc, Cc, u, D)
    require(u.dim() == 3 and lam.dim() == 2, "ssm_forward: u (B,L,H), lam (H,N)")
    B, L, H = u.shape
    N = lam.shape[1]
    require(lam.shape[0] == H and Bc.shape == (B, L, N) and Cc.shape == (B, L, N)
            and timestamps.shape == (B, L), "ssm_forward: shape mismatch")
    if u.dtype not in _lib.DTYPE_CODES:
        u = u.float()
    lam_c = lam.to(torch.complex64).contiguous()
    log_c = log_dt_scale.float().contiguous()
    t_c = timestamps.float().contiguous()
    B_c = Bc.to(torch.complex64).contiguous()
    C_c = Cc.to(torch.complex64).contiguous()
    u_c = u.contiguous()
    D_c = D.float().contiguous()
    y = torch.empty(B, L, H, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().eacs_ssm_fwd(lam_c.data_ptr(), log_c.data_ptr(), t_c.data_ptr(),
                                           B_c.data_ptr(), C_c.data_ptr(), u_c.data_ptr(),
                                           _lib.DTYPE_CODES[u_c.dtype], D_c.data_ptr(),
                                           y.data_ptr(), B, L, H, N, float(dt_min), float(dt_max),
                                           _lib.stream_ptr(dev)),
                   "eacs_ssm_fwd")
    return y
