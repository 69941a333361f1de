"""EACS layer input projections on the tensor cores (eacs_project).

`project(x, norm, proj_u, proj_B, proj_C, dtype)` is LayerNorm followed by
the layer's `_project` (cst_ssm/modules/eacs.py:334 / :376 and :261-267) as
they run inside a float16 / bfloat16 autocast region, in one kernel:
LayerNorm in float32, rounded to `dtype`; the three Linear layers as one
tcgen05 GEMM over their stacked weights with float32 accumulation; bias
added and the result rounded to `dtype`.  Returns (u, Bc, Cc): u (B, L, H)
in `u_dtype` (default `dtype`), Bc and Cc (B, L, N) complex64.
"""
from __future__ import annotations

import torch
from torch import Tensor

from .. import _lib
from ._check import require

_ROWS = 256  # the kernel's output-column tile: stacked weights are padded to a multiple of it
_cache: dict = {}


def stacked_weight(proj_u, proj_B, proj_C, dtype: torch.dtype):
    """[proj_u.weight; proj_B.weight; proj_C.weight] in `dtype`, zero rows up
    to a multiple of 256, and the stacked float32 bias; cached per module
    parameter version."""
    params = [proj_u.weight, proj_B.weight, proj_C.weight, proj_u.bias, proj_B.bias, proj_C.bias]
    key = (tuple(id(p) for p in params), dtype)
    ver = tuple(p._version for p in params) + tuple(p.data_ptr() for p in params)
    hit = _cache.get(key)
    if hit is not None and hit[0] == ver:
        return hit[1], hit[2]
    with torch.no_grad():
        w = torch.cat([proj_u.weight, proj_B.weight, proj_C.weight], 0)
        rows = -(-w.shape[0] // _ROWS) * _ROWS
        wp = torch.zeros(rows, w.shape[1], dtype=dtype, device=w.device)
        wp[: w.shape[0]] = w.to(dtype)
        bias = torch.cat([proj_u.bias, proj_B.bias, proj_C.bias], 0).float().contiguous()
    _cache[key] = (ver, wp, bias)
    return wp, bias


@torch.no_grad()
def project(x: Tensor, norm, proj_u, proj_B, proj_C, dtype: torch.dtype, u_dtype: torch.dtype | None = None):
    require(x.is_cuda, "project: x must be a CUDA tensor")
    require(dtype in (torch.float16, torch.bfloat16), "project: dtype must be float16 or bfloat16")
    u_dtype = dtype if u_dtype is None else u_dtype
    d = x.shape[-1]
    H = proj_u.weight.shape[0]
    N = proj_B.weight.shape[0] // 2
    require(proj_C.weight.shape[0] == 2 * N, "project: proj_B and proj_C must both have 2N outputs")
    lead = x.shape[:-1]
    xc = x.reshape(-1, d)
    if xc.dtype not in _lib.DTYPE_CODES:
        xc = xc.float()
    xc = xc.contiguous()
    M = xc.shape[0]
    wp, bias = stacked_weight(proj_u, proj_B, proj_C, dtype)
    gamma = norm.weight.float().contiguous()
    beta = norm.bias.float().contiguous()
    u = torch.empty(M, H, dtype=u_dtype, device=x.device)
    Bc = torch.empty(M, N, dtype=torch.complex64, device=x.device)
    Cc = torch.empty(M, N, dtype=torch.complex64, device=x.device)
    ws = torch.empty(max(1, int(_lib.lib().eacs_project_workspace_size(M))), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        _lib.check(_lib.lib().eacs_project(
            xc.data_ptr(), _lib.DTYPE_CODES[xc.dtype], gamma.data_ptr(), beta.data_ptr(), float(norm.eps),
            wp.data_ptr(), _lib.DTYPE_CODES[dtype], wp.shape[0], bias.data_ptr(), u.data_ptr(),
            _lib.DTYPE_CODES[u_dtype], Bc.data_ptr(), Cc.data_ptr(), ws.data_ptr(), ws.numel(), M, d, H, N,
            _lib.stream_ptr(x.device)), "eacs_project")
    return u.view(*lead, H), Bc.view(*lead, N), Cc.view(*lead, N)
