"""MultiScaleEACS branch epilogue on B200 (cst_ssm/modules/multiscale.py:162-197).

`branch_fuse(x, deltas, fusion, out_norm)` computes
w = softmax(fusion(x)) and y = out_norm(x + sum_s w_s delta_s) in one kernel
(eacs_branch_fuse) instead of a GEMM, softmax, stack, einsum, add and
LayerNorm over (B, L, d) tensors.  `multiscale_forward` is
MultiScaleEACS.forward with that epilogue (the branches run as the reference
calls them, side by side on their own streams; with install() their cells are
the B200 kernels).  Inference
path; install(..., multiscale=True) keeps the reference's forward where
gradients are needed.
"""
from __future__ import annotations

import ctypes
import sys

import torch
from torch import Tensor

from .. import _lib
from ._check import cuda_tensors, require
from .eacs_gated_scan import side_by_side


def fuse_supported(x: Tensor, n_branch: int) -> bool:
    if not x.is_cuda or x.dtype not in _lib.DTYPE_CODES or not 1 <= n_branch <= 8:
        return False
    d = x.shape[-1]
    e = 4 if x.dtype == torch.float32 else 8
    return d % e == 0 and d <= 256 * e and n_branch * d * 4 <= 200 * 1024


@torch.no_grad()
def branch_fuse(x: Tensor, deltas, fusion, out_norm):
    """(y, w): y = out_norm(x + sum_s softmax(fusion(x))_s deltas[s]), w (..., S) fp32."""
    S = len(deltas)
    dev = cuda_tensors("branch_fuse", x, *deltas)
    require(fuse_supported(x, S), f"branch_fuse: unsupported d={x.shape[-1]} dtype={x.dtype} S={S}")
    d = x.shape[-1]
    xc = x.contiguous()
    ds = [t.to(x.dtype).contiguous() for t in deltas]
    require(all(t.shape == x.shape for t in ds), "branch_fuse: branch outputs must have x's shape")
    wf = fusion.weight.float().contiguous()
    bf = None if fusion.bias is None else fusion.bias.float().contiguous()
    g = None if out_norm.weight is None else out_norm.weight.float().contiguous()
    b = None if out_norm.bias is None else out_norm.bias.float().contiguous()
    y = torch.empty_like(xc)
    w = torch.empty(*x.shape[:-1], S, dtype=torch.float32, device=dev)
    ptrs = (ctypes.c_void_p * S)(*[t.data_ptr() for t in ds])
    rows = xc.numel() // d
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().eacs_branch_fuse(
            xc.data_ptr(), ptrs, S, _lib.DTYPE_CODES[x.dtype], wf.data_ptr(), _lib.ptr(bf),
            _lib.ptr(g), _lib.ptr(b), float(out_norm.eps), y.data_ptr(), w.data_ptr(), rows, d,
            _lib.stream_ptr(dev)), "eacs_branch_fuse")
    return y, w


_STREAMS: dict = {}


def branch_streams(dev: torch.device, n: int):
    """n side streams of `dev`, created once and reused."""
    key = (dev.index, n)
    if key not in _STREAMS:
        _STREAMS[key] = [torch.cuda.Stream(dev) for _ in range(n)]
    return _STREAMS[key]


def run_branches(branches, dev: torch.device, fn):
    """fn(i, branch) for every branch, each on its own stream, joined back to
    the current stream.  One branch's gated cell (B rows x H/16 channel tiles)
    fills a fraction of the SMs; side by side the branches share them, and
    the cells launched here are told how many run at once (side_by_side).
    Tensors the calls return are marked as used by the current stream."""
    cur = torch.cuda.current_stream(dev)
    outs = []
    with side_by_side(len(branches)):
        for i, (br, s) in enumerate(zip(branches, branch_streams(dev, len(branches)))):
            s.wait_stream(cur)
            with torch.cuda.stream(s):
                outs.append(fn(i, br))
    for s in branch_streams(dev, len(branches)):
        cur.wait_stream(s)
    for o in outs:
        for v in (vars(o).values() if hasattr(o, "__dict__") else o if isinstance(o, (tuple, list)) else (o,)):
            if isinstance(v, Tensor) and v.is_cuda:
                v.record_stream(cur)
    return outs


@torch.no_grad()
def multiscale_forward(temporal, x: Tensor, timestamps: Tensor, frame_mask=None, cpi=None):
    """MultiScaleEACS.forward (multiscale.py:162-193) with the fused epilogue;
    the branches run side by side on their own streams."""
    if temporal._merge_ok(x):
        outs = temporal._merged_branches(x, timestamps, cpi, frame_mask)
    elif x.is_cuda:
        outs = run_branches(list(temporal.branches), x.device,
                            lambda i, br: br(x, timestamps, cpi=cpi, frame_mask=frame_mask))
    else:
        outs = [br(x, timestamps, cpi=cpi, frame_mask=frame_mask) for br in temporal.branches]
    y, w = branch_fuse(x, [o.y for o in outs], temporal.fusion, temporal.out_norm)
    gates = torch.stack([o.gates for o in outs], dim=1)
    res = torch.stack([o.residual for o in outs], dim=1)
    innov = (torch.stack([o.innovation for o in outs], dim=1)
             if all(o.innovation is not None for o in outs) else None)
    if frame_mask is not None:
        m = frame_mask.to(gates.dtype).unsqueeze(1)
        denom = m.sum().clamp_min(1.0)
        update_rate = (gates * m).sum() / (denom * temporal.n_branch)
        pbur = (gates * m).sum(dim=(0, 2)) / denom
    else:
        update_rate = gates.mean()
        pbur = torch.stack([o.update_rate for o in outs])
    MultiScaleOutput = sys.modules[type(temporal).__module__].MultiScaleOutput
    return MultiScaleOutput(y=y, gates=gates, update_rate=update_rate, per_branch_update_rate=pbur,
                            fusion_weights=w.to(x.dtype), residual=res, innovation=innov)


def make_forward(original):
    def dispatch(self, x, timestamps, frame_mask=None, cpi=None):
        needs_grad = torch.is_grad_enabled() and (
            x.requires_grad or any(p.requires_grad for p in self.parameters()))
        if not needs_grad and fuse_supported(x, self.n_branch):
            return multiscale_forward(self, x, timestamps, frame_mask, cpi)
        return original(self, x, timestamps, frame_mask, cpi)
    dispatch.__wrapped__ = original
    return dispatch
