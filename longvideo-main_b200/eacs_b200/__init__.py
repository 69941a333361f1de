"""eacs_b200 -- B200 (sm_100a) kernels for CST-SSM's EACS temporal hot path.

Modules under eacs_b200.ops mirror the reference's operator modules
(cst_ssm/ops/scan.py, scan_cuda.py, eacs_gated_scan.py, eacs_cell_train.py)
with the same function names and argument meaning; eacs_b200.install() points
an imported reference package at these kernels.
"""
from ._lib import LIB_PATH, device_status, version  # noqa: F401
from .install import install  # noqa: F401

__version__ = "0.1.0"
