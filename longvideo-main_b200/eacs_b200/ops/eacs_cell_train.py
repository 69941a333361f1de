"""Differentiable gated EACS cell on B200 (mirrors cst_ssm/ops/eacs_cell_train.py).

`GatedEACSCellFunction.apply(u, Bc, Cc, t, lam, log_dt, D, eps, mean, var, T,
eta, var_eps, dt_init, gate_mode, use_kernel, dt_max)` and `fused_gated_scan`
keep the reference signatures (eacs_cell_train.py:81-199).  The forward is the
gated cell kernel (hard gate values for "ste", the soft gate for "soft"); the
backward is the hand-derived VJP of the L-step scan (libeacs_b200.so,
eacs_cell_train_bwd) -- no Python loop and no (L,B,H,N) state list.  The
forward writes the checkpoints the backward recomputes from
(eacs_cell_train_fwd_ckpt / eacs_cell_train_bwd_ckpt).
`use_kernel` is accepted for signature compatibility; there is no other path.
"""
from __future__ import annotations

import torch
from torch import Tensor

from .. import _lib
from ._check import cuda_tensors, require
from .eacs_gated_scan import prepare, workspace_bytes


def _train_fwd(u, Bc, Cc, t, lam, log_dt, D, eps, mean, var, T, eta, var_eps, dt_init,
               gate_mode, dt_max, bwd_ws=None):
    """The gated forward for training.  With `bwd_ws` (a uint8 tensor of
    eacs_cell_train_bwd_workspace_size bytes) it also writes the backward's
    checkpoints there (eacs_cell_train_fwd_ckpt)."""
    dev, (lam_c, log_c, u_c, B_c, C_c, t_c, D_c, m_c, v_c) = prepare(
        lam, log_dt, u, Bc, Cc, t, D, mean, var)
    B, L, H = u_c.shape
    N = lam_c.shape[1]
    ys = torch.empty(B, L, H, dtype=torch.float32, device=dev)
    gs = torch.empty(B, L, dtype=torch.float32, device=dev)
    rs = torch.empty(B, L, dtype=torch.float32, device=dev)
    stats = torch.empty(B, L, 2, dtype=torch.float32, device=dev)
    if ys.numel():
        ws = torch.empty(workspace_bytes(B, L, H, N), dtype=torch.uint8, device=dev)
        args = (lam_c.data_ptr(), log_c.data_ptr(), u_c.data_ptr(), _lib.DTYPE_CODES[u_c.dtype],
                B_c.data_ptr(), C_c.data_ptr(), t_c.data_ptr(), D_c.data_ptr(), m_c.data_ptr(),
                v_c.data_ptr(), float(eps), float(eta), float(var_eps), float(dt_init), 1e-3,
                float(dt_max), 1 if gate_mode == "soft" else 0, float(T),
                ys.data_ptr(), gs.data_ptr(), rs.data_ptr(), stats.data_ptr(), ws.data_ptr(), ws.numel())
        with torch.cuda.device(dev):
            if bwd_ws is None:
                _lib.check(_lib.lib().eacs_cell_train_fwd(*args, B, L, H, N, _lib.stream_ptr(dev)),
                           "eacs_cell_train_fwd")
            else:
                _lib.check(_lib.lib().eacs_cell_train_fwd_ckpt(
                    *args, bwd_ws.data_ptr(), bwd_ws.numel(), B, L, H, N, _lib.stream_ptr(dev)),
                    "eacs_cell_train_fwd_ckpt")
    return ys, gs, rs, stats, (lam_c, log_c, u_c, B_c, C_c, t_c, D_c, m_c, v_c)


def _train_bwd(prep, gs, rs, stats, eps, T, eta, var_eps, dt_init, dt_max, g_ys, g_gs, g_rs, g_ns,
               bwd_ws=None):
    """The backward.  With `bwd_ws` holding the checkpoints a _train_fwd call
    with the same tensors wrote, its checkpoint pass is skipped."""
    lam_c, log_c, u_c, B_c, C_c, t_c, D_c, m_c, v_c = prep
    dev = u_c.device
    B, L, H = u_c.shape
    N = lam_c.shape[1]
    gy = (torch.zeros(B, L, H, dtype=torch.float32, device=dev) if g_ys is None
          else g_ys.float().contiguous())
    opt = [None if g is None else g.float().contiguous() for g in (g_gs, g_rs, g_ns)]
    du = torch.empty(B, L, H, dtype=torch.float32, device=dev)
    dBc = torch.empty(B, L, N, dtype=torch.complex64, device=dev)
    dCc = torch.empty_like(dBc)
    dt = torch.empty(B, L, dtype=torch.float32, device=dev)
    dlam = torch.empty(H, N, dtype=torch.complex64, device=dev)
    dlog = torch.empty(H, dtype=torch.float32, device=dev)
    dD = torch.empty(H, dtype=torch.float32, device=dev)
    deps = torch.empty(1, dtype=torch.float32, device=dev)
    L_ = _lib.lib()
    nbytes = int(L_.eacs_cell_train_bwd_workspace_size(B, L, H, N))
    require(nbytes > 0, f"eacs_cell_train_bwd: unsupported sizes B={B} L={L} H={H} N={N}")
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev) if bwd_ws is None else bwd_ws
    require(ws.numel() >= nbytes, "eacs_cell_train_bwd: checkpoint workspace too small")
    entry = L_.eacs_cell_train_bwd if bwd_ws is None else L_.eacs_cell_train_bwd_ckpt
    with torch.cuda.device(dev):
        _lib.check(entry(
            lam_c.data_ptr(), log_c.data_ptr(), u_c.data_ptr(), _lib.DTYPE_CODES[u_c.dtype],
            B_c.data_ptr(), C_c.data_ptr(), t_c.data_ptr(), D_c.data_ptr(), m_c.data_ptr(),
            v_c.data_ptr(), float(eps), float(eta), float(var_eps), float(dt_init), 1e-3,
            float(dt_max), float(T), gs.data_ptr(), rs.data_ptr(), stats.data_ptr(),
            gy.data_ptr(), *[_lib.ptr(g) for g in opt],
            du.data_ptr(), dBc.data_ptr(), dCc.data_ptr(), dt.data_ptr(), dlam.data_ptr(),
            dlog.data_ptr(), dD.data_ptr(), deps.data_ptr(), ws.data_ptr(), ws.numel(),
            B, L, H, N, _lib.stream_ptr(dev)), "eacs_cell_train_bwd" if bwd_ws is None else "eacs_cell_train_bwd_ckpt")
    return du, dBc, dCc, dt, dlam, dlog, dD, deps


class GatedEACSCellFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u, Bc, Cc, t, lam, log_dt, D, eps, mean, var,
                T, eta, var_eps, dt_init, gate_mode, use_kernel, dt_max):
        ctx.set_materialize_grads(False)
        cuda_tensors("GatedEACSCellFunction", u, Bc, Cc, t, lam, log_dt, D, mean, var)
        eps_v = float(eps)
        # When gradients are wanted, the forward also writes the checkpoints the
        # backward recomputes from (it computes those states anyway), into the
        # backward's workspace, held until the backward.
        bwd_ws = None
        if any(ctx.needs_input_grad[:8]) and u.numel():
            nbytes = int(_lib.lib().eacs_cell_train_bwd_workspace_size(*u.shape, lam.shape[1]))
            if nbytes:
                bwd_ws = torch.empty(nbytes, dtype=torch.uint8, device=u.device)
        ys, gs, rs, stats, prep = _train_fwd(u, Bc, Cc, t, lam, log_dt, D, eps_v, mean, var, T,
                                             eta, var_eps, dt_init, gate_mode, dt_max, bwd_ws)
        ctx.bwd_ws = bwd_ws
        ctx.prep = prep
        ctx.save_for_backward(gs, rs, stats)
        ctx.hp = (eps_v, float(T), float(eta), float(var_eps), float(dt_init), float(dt_max))
        ctx.dtypes = (u.dtype, Bc.dtype, Cc.dtype, t.dtype, lam.dtype, log_dt.dtype, D.dtype,
                      eps.dtype if torch.is_tensor(eps) else None,
                      eps.shape if torch.is_tensor(eps) else None)
        # the innovation has the residual's values (its gradient differs)
        return ys, gs, rs, rs.clone()

    @staticmethod
    def backward(ctx, g_ys, g_gs, g_rs, g_ns):
        gs, rs, stats = ctx.saved_tensors
        eps_v, T, eta, var_eps, dt_init, dt_max = ctx.hp
        du, dBc, dCc, dt, dlam, dlog, dD, deps = _train_bwd(
            ctx.prep, gs, rs, stats, eps_v, T, eta, var_eps, dt_init, dt_max, g_ys, g_gs, g_rs, g_ns,
            ctx.bwd_ws)
        u_t, B_t, C_t, t_t, lam_t, log_t, D_t, eps_t, eps_shape = ctx.dtypes
        deps_out = None
        if eps_t is not None:
            deps_out = deps.to(eps_t).reshape(eps_shape)
        return (du.to(u_t), dBc.to(B_t), dCc.to(C_t), dt.to(t_t), dlam.to(lam_t), dlog.to(log_t),
                dD.to(D_t), deps_out, None, None, None, None, None, None, None, None, None)


def fused_gated_scan(u: Tensor, Bc: Tensor, Cc: Tensor, t: Tensor,
                     lam: Tensor, log_dt: Tensor, D: Tensor, eps: Tensor,
                     mean: Tensor, var: Tensor, T: float, eta: float,
                     var_eps: float = 1e-5, dt_init: float = 1.0,
                     gate_mode: str = "ste", use_kernel: bool = True,
                     dt_max: float = 1e3, return_innovation: bool = False):
    """Return (y, gates, residual), optionally followed by the stop-target innovation."""
    outputs = GatedEACSCellFunction.apply(u, Bc, Cc, t, lam, log_dt, D, eps, mean, var,
                                          T, eta, var_eps, dt_init, gate_mode, use_kernel,
                                          dt_max)
    return outputs if return_innovation else outputs[:3]
