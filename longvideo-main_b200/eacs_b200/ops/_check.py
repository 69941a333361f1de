"""Argument checks shared by the operator modules (raise RuntimeError, as the
reference's TORCH_CHECKs do)."""
from __future__ import annotations

import torch


def require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def cuda_tensors(name: str, *ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        require(isinstance(t, torch.Tensor), f"{name}: expects tensors")
        require(t.is_cuda, f"{name}: expects CUDA tensors (eacs_b200 has no CPU path)")
        if dev is None:
            dev = t.device
        require(t.device == dev, f"{name}: tensors must be on one device")
    return dev
