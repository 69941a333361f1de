"""Variable-step diagonal complex scan on B200 (mirrors cst_ssm/ops/scan_cuda.py).

`EXT` is a drop-in for the reference's JIT extension object (`_EXT` in
scan_cuda.py:14-29): `scan_fwd(a, b) -> [h]` and
`scan_bwd(a, h, grad_h) -> [grad_a, grad_b]` with the signatures bound at
cst_ssm/ops/csrc/eacs_scan_cuda.cu:98-101, running the TMA-pipelined kernels
of libeacs_b200.so.
"""
from __future__ import annotations

import torch
from torch import Tensor
from torch.autograd import Function

from .. import _lib
from ._check import cuda_tensors, require


class _ScanExt:
    """Object with the reference extension's methods."""

    @staticmethod
    def scan_fwd(a: Tensor, b: Tensor) -> list[Tensor]:
        dev = cuda_tensors("scan_fwd", a, b)
        require(a.dtype == torch.complex64 and b.dtype == torch.complex64,
                "scan_fwd: expects complex64")
        require(a.dim() == 4 and a.shape == b.shape, "scan_fwd: expects (B,L,H,N)")
        a = a.contiguous()
        b = b.contiguous()
        B, L, H, N = a.shape
        h = torch.empty_like(b)
        with torch.cuda.device(dev):
            _lib.check(_lib.lib().eacs_scan_fwd(a.data_ptr(), b.data_ptr(), h.data_ptr(),
                                                B, L, H, N, _lib.stream_ptr(dev)),
                       "eacs_scan_fwd")
        return [h]

    @staticmethod
    def scan_bwd(a: Tensor, h: Tensor, grad_h: Tensor) -> list[Tensor]:
        dev = cuda_tensors("scan_bwd", a, h, grad_h)
        require(a.dtype == torch.complex64 and h.dtype == torch.complex64
                and grad_h.dtype == torch.complex64, "scan_bwd: expects complex64")
        require(a.dim() == 4 and a.shape == h.shape == grad_h.shape,
                "scan_bwd: expects (B,L,H,N)")
        a = a.contiguous()
        h = h.contiguous()
        grad_h = grad_h.contiguous()
        B, L, H, N = a.shape
        grad_a = torch.empty_like(a)
        grad_b = torch.empty_like(a)
        with torch.cuda.device(dev):
            _lib.check(_lib.lib().eacs_scan_bwd(a.data_ptr(), h.data_ptr(), grad_h.data_ptr(),
                                                grad_a.data_ptr(), grad_b.data_ptr(),
                                                B, L, H, N, _lib.stream_ptr(dev)),
                       "eacs_scan_bwd")
        return [grad_a, grad_b]


EXT = _ScanExt()


def _load():
    """The extension object (raises if libeacs_b200.so is not built)."""
    _lib.lib()
    return EXT


def cuda_available() -> bool:
    if not torch.cuda.is_available():
        return False
    _lib.lib()
    return True


class _SelectiveScanCUDA(Function):
    @staticmethod
    def forward(ctx, a: Tensor, b: Tensor) -> Tensor:
        h = EXT.scan_fwd(a, b)[0]
        ctx.save_for_backward(a, h)
        return h

    @staticmethod
    def backward(ctx, grad_h: Tensor):
        a, h = ctx.saved_tensors
        grad_a, grad_b = EXT.scan_bwd(a, h, grad_h)
        return grad_a, grad_b


def selective_scan_cuda(a: Tensor, b: Tensor) -> Tensor:
    """Differentiable scan; a, b CUDA complex64 (B,L,H,N)."""
    return _SelectiveScanCUDA.apply(a, b)
