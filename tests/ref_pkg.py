"""Location of the reference's Python package, for tests that run it as the
checker (never imported by the product).

Looked up in order: the CST_SSM_REFERENCE environment variable (a checkout
holding cst_ssm/), then baseline/_ref/ inside this repository, where
__graft_entry__.build() installs the reference package (pip --target) when
its checkout is present.  Both are optional: tests that need it skip without.
"""
from __future__ import annotations

import importlib
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

MODULES = ("ops.scan_cuda", "ops.eacs_gated_scan", "ops.eacs_cell_train", "ops.scan",
           "ops.spectral_init", "modules.continuous_ssm", "modules.eacs", "modules.event_gate",
           "modules.multiscale", "modules.continuous_query")


def reference_root() -> str | None:
    for cand in (os.environ.get("CST_SSM_REFERENCE"), os.path.join(REPO, "baseline", "_ref")):
        if cand and os.path.isdir(os.path.join(cand, "cst_ssm")):
            return cand
    return None


def import_reference():
    """The reference's modules by short name, or None when it is absent."""
    root = reference_root()
    if root is None:
        return None
    if root not in sys.path:
        sys.path.insert(0, root)
    try:
        return {n: importlib.import_module(f"cst_ssm.{n}") for n in MODULES}
    except ImportError:
        return None


def snapshot(mods):
    """Every attribute install() may replace, so a test can put them back."""
    e, q = mods["modules.eacs"].EACSLayer, mods["modules.continuous_query"]
    return [
        (mods["ops.scan_cuda"], "_EXT", mods["ops.scan_cuda"]._EXT),
        (mods["ops.scan_cuda"], "_TRIED", mods["ops.scan_cuda"]._TRIED),
        (mods["ops.eacs_gated_scan"], "_EXT", mods["ops.eacs_gated_scan"]._EXT),
        (mods["ops.eacs_gated_scan"], "_TRIED", mods["ops.eacs_gated_scan"]._TRIED),
        (mods["ops.eacs_cell_train"], "GatedEACSCellFunction",
         mods["ops.eacs_cell_train"].GatedEACSCellFunction),
        (mods["ops.eacs_cell_train"], "fused_gated_scan", mods["ops.eacs_cell_train"].fused_gated_scan),
        (mods["modules.continuous_ssm"].ContinuousSSMLayer, "forward",
         mods["modules.continuous_ssm"].ContinuousSSMLayer.forward),
        (e, "_cuda_fused_ok", e._cuda_fused_ok), (e, "_forward_fused", e._forward_fused),
        (e, "run_with_commits", e.run_with_commits),
        (q, "readout_from_commits", q.readout_from_commits), (q, "segment_index", q.segment_index),
        (mods["modules.multiscale"].MultiScaleEACS, "forward", mods["modules.multiscale"].MultiScaleEACS.forward),
    ]


def restore(saved):
    for owner, name, value in saved:
        setattr(owner, name, value)


def reference_only(mods):
    """Make the reference run its own PyTorch code: its CUDA extensions are
    marked as tried and absent, so nothing is compiled and its callers take
    their PyTorch paths (scan_cuda.py:20-29, eacs_gated_scan.py:13-28)."""
    mods["ops.scan_cuda"]._EXT, mods["ops.scan_cuda"]._TRIED = None, True
    mods["ops.eacs_gated_scan"]._EXT, mods["ops.eacs_gated_scan"]._TRIED = None, True
