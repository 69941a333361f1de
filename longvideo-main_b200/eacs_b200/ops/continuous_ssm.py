"""Fused ungated continuous SSM core (cst_ssm/modules/continuous_ssm.py:44-55).

`ssm_forward` replaces, inside ContinuousSSMLayer.forward, the chain
dt -> effective_dt -> zoh_discretize -> dB*u -> selective_scan -> readout
with one kernel that keeps every (b, h, n) state in registers: no (B,L,H,N)
tensor is materialised.  It is differentiable: with autograd recording, the
forward also writes one state checkpoint every 8 steps and the backward
(eacs_ssm_bwd) recomputes each 8-step chunk from its checkpoint, returning
the gradients of lam, log_dt_scale, the timestamps, Bc, Cc, u and D.

`layer_forward(layer, x, timestamps)` is ContinuousSSMLayer.forward
(continuous_ssm.py:33-57) with the core routed through `ssm_forward`;
eacs_b200.install(..., fuse_ungated=True) binds it to the reference class.
"""
from __future__ import annotations

import torch
from torch import Tensor

from .. import _lib
from ._check import cuda_tensors, require

DT_MIN = 1e-3  # effective_dt defaults (ops/discretization.py:67-68)
DT_MAX = 1e3


def _prepare(lam, log_dt_scale, timestamps, Bc, Cc, u, D):
    dev = cuda_tensors("ssm_forward", lam, log_dt_scale, timestamps, Bc, Cc, u, D)
    require(u.dim() == 3 and lam.dim() == 2, "ssm_forward: u (B,L,H), lam (H,N)")
    B, L, H = u.shape
    N = lam.shape[1]
    require(lam.shape[0] == H and Bc.shape == (B, L, N) and Cc.shape == (B, L, N)
            and timestamps.shape == (B, L) and log_dt_scale.shape == (H,) and D.shape == (H,),
            "ssm_forward: shape mismatch")
    if u.dtype not in _lib.DTYPE_CODES:
        u = u.float()
    return dev, (lam.to(torch.complex64).contiguous(), log_dt_scale.float().contiguous(),
                 timestamps.float().contiguous(), Bc.to(torch.complex64).contiguous(),
                 Cc.to(torch.complex64).contiguous(), u.contiguous(), D.float().contiguous())


def _forward(prep, dev, dt_min, dt_max, with_ckpt):
    lam_c, log_c, t_c, B_c, C_c, u_c, D_c = prep
    B, L, H = u_c.shape
    N = lam_c.shape[1]
    y = torch.empty(B, L, H, dtype=torch.float32, device=dev)
    ckpt = None
    if y.numel() == 0:
        return y, ckpt
    L_ = _lib.lib()
    args = (lam_c.data_ptr(), log_c.data_ptr(), t_c.data_ptr(), B_c.data_ptr(), C_c.data_ptr(),
            u_c.data_ptr(), _lib.DTYPE_CODES[u_c.dtype], D_c.data_ptr(), y.data_ptr())
    with torch.cuda.device(dev):
        if with_ckpt:
            nbytes = int(L_.eacs_ssm_ckpt_size(B, L, H, N))
            require(nbytes > 0, f"eacs_ssm_train_fwd: unsupported sizes B={B} L={L} H={H} N={N}")
            ckpt = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            _lib.check(L_.eacs_ssm_train_fwd(*args, ckpt.data_ptr(), nbytes, B, L, H, N,
                                             float(dt_min), float(dt_max), _lib.stream_ptr(dev)),
                       "eacs_ssm_train_fwd")
        else:
            _lib.check(L_.eacs_ssm_fwd(*args, B, L, H, N, float(dt_min), float(dt_max),
                                       _lib.stream_ptr(dev)),
                       "eacs_ssm_fwd")
    return y, ckpt


def _backward(prep, ckpt, gy, dt_min, dt_max):
    lam_c, log_c, t_c, B_c, C_c, u_c, D_c = prep
    dev = u_c.device
    B, L, H = u_c.shape
    N = lam_c.shape[1]
    gy = gy.float().contiguous()
    du = torch.empty(B, L, H, dtype=torch.float32, device=dev)
    dBc = torch.empty(B, L, N, dtype=torch.complex64, device=dev)
    dCc = torch.empty_like(dBc)
    dt = torch.empty(B, L, dtype=torch.float32, device=dev)
    dlam = torch.empty(H, N, dtype=torch.complex64, device=dev)
    dlog = torch.empty(H, dtype=torch.float32, device=dev)
    dD = torch.empty(H, dtype=torch.float32, device=dev)
    if du.numel() == 0:
        return du, dBc.zero_(), dCc.zero_(), dt.zero_(), dlam.zero_(), dlog.zero_(), dD.zero_()
    L_ = _lib.lib()
    nbytes = int(L_.eacs_ssm_bwd_workspace_size(B, L, H, N))
    require(nbytes > 0, f"eacs_ssm_bwd: unsupported sizes B={B} L={L} H={H} N={N}")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(L_.eacs_ssm_bwd(
            lam_c.data_ptr(), log_c.data_ptr(), t_c.data_ptr(), B_c.data_ptr(), C_c.data_ptr(),
            u_c.data_ptr(), _lib.DTYPE_CODES[u_c.dtype], D_c.data_ptr(), gy.data_ptr(),
            ckpt.data_ptr(), ckpt.numel(), du.data_ptr(), dBc.data_ptr(), dCc.data_ptr(),
            dt.data_ptr(), dlam.data_ptr(), dlog.data_ptr(), dD.data_ptr(), ws.data_ptr(),
            ws.numel(), B, L, H, N, float(dt_min), float(dt_max), _lib.stream_ptr(dev)),
            "eacs_ssm_bwd")
    return du, dBc, dCc, dt, dlam, dlog, dD


class SSMCoreFunction(torch.autograd.Function):
    """y = Re sum_n C h + D u of the variable-step ZOH scan, with its VJP."""

    @staticmethod
    def forward(ctx, lam, log_dt_scale, timestamps, Bc, Cc, u, D, dt_min, dt_max):
        dev, prep = _prepare(lam, log_dt_scale, timestamps, Bc, Cc, u, D)
        y, ckpt = _forward(prep, dev, dt_min, dt_max, with_ckpt=True)
        ctx.save_for_backward(*prep, *(() if ckpt is None else (ckpt,)))
        ctx.has_ckpt = ckpt is not None
        ctx.dt = (dt_min, dt_max)
        ctx.dtypes = (lam.dtype, log_dt_scale.dtype, timestamps.dtype, Bc.dtype, Cc.dtype,
                      u.dtype, D.dtype)
        return y

    @staticmethod
    def backward(ctx, gy):
        saved = ctx.saved_tensors
        prep = saved[:7]
        if not ctx.has_ckpt:  # empty input
            return (None,) * 9
        grads = _backward(prep, saved[7], gy, *ctx.dt)
        du, dBc, dCc, dt, dlam, dlog, dD = grads
        order = (dlam, dlog, dt, dBc, dCc, du, dD)
        out = []
        for need, g, dtype in zip(ctx.needs_input_grad[:7], order, ctx.dtypes):
            if not need:
                out.append(None)
            elif g.is_complex() and not dtype.is_complex:
                out.append(g.real.to(dtype))
            else:
                out.append(g.to(dtype))
        return (*out, None, None)


def ssm_forward(lam: Tensor, log_dt_scale: Tensor, timestamps: Tensor, Bc: Tensor, Cc: Tensor,
                u: Tensor, D: Tensor, dt_min: float = DT_MIN, dt_max: float = DT_MAX) -> Tensor:
    """y (B,L,H) fp32 = Re sum_n C_l h_l + D u with h the ZOH scan of (dB_bar B) u.

    lam (H,N) complex, log_dt_scale (H), timestamps (B,L), Bc/Cc (B,L,N) complex,
    u (B,L,H) fp32/fp16/bf16, D (H).  Differentiable in all of them."""
    ts = (lam, log_dt_scale, timestamps, Bc, Cc, u, D)
    if torch.is_grad_enabled() and any(t.requires_grad for t in ts):
        return SSMCoreFunction.apply(*ts, dt_min, dt_max)
    dev, prep = _prepare(*ts)
    return _forward(prep, dev, dt_min, dt_max, with_ckpt=False)[0]


def layer_forward(layer, x: Tensor, timestamps: Tensor) -> Tensor:
    """ContinuousSSMLayer.forward (cst_ssm/modules/continuous_ssm.py:33-57) with
    the dt / discretisation / scan / readout core fused into one kernel."""
    x_in = x
    xn = layer.norm(x)
    u = layer.proj_u(xn)
    b = layer.proj_B(xn).float()
    Bc = torch.complex(b[..., :layer.N], b[..., layer.N:])
    c = layer.proj_C(xn).float()
    Cc = torch.complex(c[..., :layer.N], c[..., layer.N:])
    lam = torch.complex(-torch.exp(layer.a_log_neg_real.float()), layer.a_imag.float())
    y = ssm_forward(lam, layer.log_dt_scale, timestamps.float(), Bc, Cc, u, layer.D)
    y = layer.proj_out(y.to(x_in.dtype))
    return x_in + y if layer.add_residual else y
