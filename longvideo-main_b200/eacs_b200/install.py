"""Point an imported reference CST-SSM package at the B200 kernels.

The reference loads its CUDA extensions lazily through module globals and
imports its fused operators inside the calling functions
(cst_ssm/ops/scan_cuda.py:14-29, ops/eacs_gated_scan.py:16-28,
modules/eacs.py:250, :321, :367, ops/scan.py:69), so replacing those globals
makes ContinuousSSMLayer, EACSLayer and MultiScaleEACS run these kernels
without any change to the reference's code.
"""
from __future__ import annotations

import importlib


def install(package: str = "cst_ssm", fuse_ungated: bool = False,
            layer_dispatch: bool = False, queries: bool = False,
            streaming: bool = False, multiscale: bool = False) -> dict:
    """Patch `package` (already importable) and return what was replaced.

    fuse_ungated: also bind ContinuousSSMLayer.forward to the fused ungated
    core (eacs_b200.ops.continuous_ssm.layer_forward), which needs no
    (B,L,H,N) tensors, instead of only swapping its scan extension.
    layer_dispatch: also bind EACSLayer._cuda_fused_ok / _forward_fused to
    eacs_b200.ops.eacs_layer, so eval-mode layers with robust_guard run the
    fused kernel instead of the Python step loop.
    queries: also route EACSLayer.run_with_commits and the continuous-query
    functions (segment_index, readout_from_commits) through the commit and
    readout kernels, with gradients through the commits and the readouts
    (training); the reference's own code runs only for CPI-modulated or
    non-event gates and non-continuous discretisation.
    streaming: also route temporal_step (modules/streaming.py, and the name
    models/adaptive_path.py imported from it) through the streaming step
    kernel and its backward (gradients through the state from step to step);
    the reference's own code runs only for CPU tensors, non-event gates and
    non-continuous discretisation.
    multiscale: also route MultiScaleEACS.forward's epilogue (fusion softmax,
    blend, LayerNorm) through the one-pass branch-fuse kernel, under the same
    rule."""
    from .ops import eacs_gated_scan as ours_cell
    from .ops import scan_cuda as ours_scan

    patched = {}
    ref_scan = importlib.import_module(f"{package}.ops.scan_cuda")
    ref_scan._EXT = ours_scan._load()
    ref_scan._TRIED = True
    patched["scan_cuda._EXT"] = ref_scan._EXT

    ref_cell = importlib.import_module(f"{package}.ops.eacs_gated_scan")
    ref_cell._EXT = ours_cell._load()
    ref_cell._TRIED = True
    patched["eacs_gated_scan._EXT"] = ref_cell._EXT

    try:
        from .ops import eacs_cell_train as ours_train
    except ImportError:
        ours_train = None
    if ours_train is not None:
        ref_train = importlib.import_module(f"{package}.ops.eacs_cell_train")
        ref_train.GatedEACSCellFunction = ours_train.GatedEACSCellFunction
        ref_train.fused_gated_scan = ours_train.fused_gated_scan
        patched["eacs_cell_train.fused_gated_scan"] = ours_train.fused_gated_scan
    if fuse_ungated:
        from .ops import continuous_ssm as ours_ssm

        ref_layer = importlib.import_module(f"{package}.modules.continuous_ssm")
        ref_layer.ContinuousSSMLayer.forward = ours_ssm.layer_forward
        patched["continuous_ssm.ContinuousSSMLayer.forward"] = ours_ssm.layer_forward
    if queries:
        from .ops import continuous_query as ours_q

        ref_eacs = importlib.import_module(f"{package}.modules.eacs")
        ref_q = importlib.import_module(f"{package}.modules.continuous_query")
        for owner, name, make in ((ref_eacs.EACSLayer, "run_with_commits", ours_q.make_run_with_commits),
                                  (ref_q, "readout_from_commits", ours_q.make_readout_from_commits),
                                  (ref_q, "segment_index", ours_q.make_segment_index)):
            current = getattr(owner, name)
            if not hasattr(current, "__wrapped__"):  # installing twice keeps one wrapper
                setattr(owner, name, make(current))
            patched[f"{owner.__name__.split('.')[-1]}.{name}"] = getattr(owner, name)
    if streaming:
        from .ops import streaming as ours_s

        for mod_name in (f"{package}.modules.streaming", f"{package}.models.adaptive_path"):
            try:
                mod = importlib.import_module(mod_name)
            except ImportError:  # the model package may be absent
                continue
            current = mod.temporal_step
            if not hasattr(current, "__wrapped__"):
                mod.temporal_step = ours_s.make_temporal_step(current)
            patched[f"{mod_name.split('.')[-1]}.temporal_step"] = mod.temporal_step
    if multiscale:
        from .ops import multiscale as ours_ms

        ref_ms = importlib.import_module(f"{package}.modules.multiscale")
        current = ref_ms.MultiScaleEACS.forward
        if not hasattr(current, "__wrapped__"):
            ref_ms.MultiScaleEACS.forward = ours_ms.make_forward(current)
        patched["multiscale.MultiScaleEACS.forward"] = ref_ms.MultiScaleEACS.forward
    if layer_dispatch:
        from .ops import eacs_layer as ours_layer

        ref_eacs = importlib.import_module(f"{package}.modules.eacs")
        ref_eacs.EACSLayer._cuda_fused_ok = ours_layer.cuda_fused_ok
        ref_eacs.EACSLayer._forward_fused = ours_layer.forward_fused
        patched["eacs.EACSLayer._forward_fused"] = ours_layer.forward_fused
    return patched
