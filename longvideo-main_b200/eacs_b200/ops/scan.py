"""Unified scan entry (mirrors cst_ssm/ops/scan.py:64-78 selective_scan).

Always runs the B200 kernel; an initial state is folded into the first input
(b_0 + a_0 h_init), which is the first step of the reference's sequential
scan.  CPU tensors and backend="pytorch" raise: this package has no PyTorch
scan.
"""
from __future__ import annotations

from torch import Tensor

from .scan_cuda import selective_scan_cuda


def selective_scan(a: Tensor, b: Tensor, h_init: Tensor | None = None,
                   backend: str = "auto", chunk: int = 0) -> Tensor:
    if backend == "pytorch":
        raise ValueError("eacs_b200.selective_scan: there is no PyTorch backend")
    if not (a.is_cuda and b.is_cuda):
        raise RuntimeError("eacs_b200.selective_scan: expects CUDA tensors")
    if h_init is not None:
        b = b.clone()
        b[:, 0] = b[:, 0] + a[:, 0] * h_init
    return selective_scan_cuda(a, b)
