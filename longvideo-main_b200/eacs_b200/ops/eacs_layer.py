"""EACSLayer's inference dispatch on B200 (cst_ssm/modules/eacs.py:239-253, :365-378).

The reference sends an eval-mode CUDA input to its gated kernel only when
robust_guard is off (_fast_paths_ok, eacs.py:239-244), because its kernel has
no residual-spike fallback; robust layers run the Python step loop
(scan_range, eacs.py:145-173).  The B200 cell kernel implements robust_guard,
so `cuda_fused_ok` admits it and `forward_fused` passes the layer's
(robust_k, spike_ratio, eps_factor).  The innovation output of the step loop
(EventGate.residual of the detached target, eacs.py:104) has the values of the
residual and is returned as such.

Inside a float16 / bfloat16 autocast region, LayerNorm and the input
projections (eacs.py:376, :261-267) run as one tcgen05 kernel
(ops/projection.py) with autocast's rounding; outside one they run as the
reference writes them (float32 Linear layers).

install(..., layer_dispatch=True) binds both functions to the reference
class as `_cuda_fused_ok` and `_forward_fused`.
"""
from __future__ import annotations

import sys

import torch
from torch import Tensor


def fast_paths_ok(layer) -> bool:
    """eacs.py:239-244 without the robust_guard exclusion."""
    return (layer.disc_mode == "continuous"
            and getattr(layer.gate, "gate_kind", "event") == "event"
            and getattr(layer.gate, "cpi_modulation", 0.0) == 0)


def cuda_fused_ok(layer, x: Tensor) -> bool:
    """eacs.py:246-253: eval mode, CUDA input, a fused-compatible layer."""
    if layer.training or not x.is_cuda or not fast_paths_ok(layer):
        return False
    from .eacs_gated_scan import gated_kernel_available
    return gated_kernel_available()


@torch.no_grad()
def forward_fused(layer, x: Tensor, timestamps: Tensor):
    """eacs.py:365-378 with robust_guard honoured; returns the layer module's EACSOutput."""
    from .eacs_gated_scan import eacs_cell_forward

    x_in = x
    T = torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else None
    if T in (torch.float16, torch.bfloat16) and x.shape[-1] % 8 == 0:
        # LayerNorm + _project as autocast runs them, in one tensor-core kernel
        from .projection import project
        u, Bc, Cc = project(x, layer.norm, layer.proj_u, layer.proj_B, layer.proj_C, T)
    else:
        xn = layer.norm(x)
        u, Bc, Cc = layer._project(xn)
    robust = ((layer.robust_k, layer.robust_spike_ratio, layer.robust_eps_factor)
              if layer.robust_guard else None)
    ys, gates, resid = eacs_cell_forward(
        layer.lam(), layer.log_dt_scale, u, Bc, Cc, timestamps, layer.D,
        layer.obs_norm.running_mean, layer.obs_norm.running_var,
        eps=float(layer.gate.eps.item()), eta=layer.gate.norm_eta,
        var_eps=layer.obs_norm.eps, dt_init=layer.dt_init, dt_max=layer.dt_max, robust=robust)
    delta = layer.proj_out(ys.to(x_in.dtype))
    y = x_in + delta if layer.add_residual else delta
    EACSOutput = sys.modules[type(layer).__module__].EACSOutput
    return EACSOutput(y=y, gates=gates, update_rate=gates.mean(), residual=resid,
                      innovation=resid.clone())
