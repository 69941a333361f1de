"""eacs_b200.install() against an unmodified reference package (CPU only).

Runs only where the reference's Python package is importable (tests/ref_pkg.py:
CST_SSM_REFERENCE or baseline/_ref).  Checks that every hook the reference's
lazy loaders and dispatch go through is replaced, that the replaced layer
paths keep the reference's CPU behaviour where the reference falls back
(EACSLayer on CPU) and that the fused ungated layer refuses CPU tensors
instead of silently running elsewhere.
"""
import importlib
import sys

import pytest
import torch

from ref_pkg import import_reference, reference_root, restore, snapshot

pytestmark = pytest.mark.skipif(reference_root() is None, reason="reference package not present")


@pytest.fixture()
def ref_pkg():
    mods = import_reference()
    if mods is None:
        pytest.skip("reference not importable")
    saved = snapshot(mods)
    yield mods
    restore(saved)


def test_install_replaces_every_hook(ref_pkg):
    import eacs_b200
    from eacs_b200.ops import continuous_ssm, eacs_cell_train, eacs_layer
    from eacs_b200.ops import eacs_gated_scan as ours_cell
    from eacs_b200.ops import scan_cuda as ours_scan

    patched = eacs_b200.install("cst_ssm", fuse_ungated=True, layer_dispatch=True)
    assert ref_pkg["ops.scan_cuda"]._EXT is ours_scan.EXT and ref_pkg["ops.scan_cuda"]._TRIED
    assert ref_pkg["ops.eacs_gated_scan"]._EXT is ours_cell.EXT
    assert ref_pkg["ops.eacs_cell_train"].fused_gated_scan is eacs_cell_train.fused_gated_scan
    assert (ref_pkg["ops.eacs_cell_train"].GatedEACSCellFunction
            is eacs_cell_train.GatedEACSCellFunction)
    assert ref_pkg["modules.continuous_ssm"].ContinuousSSMLayer.forward is continuous_ssm.layer_forward
    assert ref_pkg["modules.eacs"].EACSLayer._forward_fused is eacs_layer.forward_fused
    assert len(patched) == 5
    # the extension objects expose the reference's method names
    for name in ("scan_fwd", "scan_bwd"):
        assert callable(getattr(ours_scan.EXT, name))
    assert callable(ours_cell.EXT.eacs_cell_fwd)


def test_robust_layer_on_cpu_keeps_reference_path(ref_pkg):
    """On CPU the patched dispatch declines (as the reference's does) and the
    reference's step loop runs, with robust_guard."""
    import eacs_b200
    from cst_ssm.ops.spectral_init import BranchSpec

    eacs_b200.install("cst_ssm", layer_dispatch=True)
    EACSLayer = ref_pkg["modules.eacs"].EACSLayer
    torch.manual_seed(0)
    layer = EACSLayer(16, BranchSpec("t", n_state=4, tau_min=0.5, tau_max=4.0), robust_guard=True).eval()
    x = torch.randn(2, 12, 16)
    t = torch.cumsum(torch.full((2, 12), 0.25), 1)
    assert not layer._cuda_fused_ok(x)
    out = layer(x, t)
    assert out.y.shape == (2, 12, 16) and out.gates.shape == (2, 12)
    assert torch.equal(out.innovation, out.residual)


def test_fused_ungated_layer_refuses_cpu(ref_pkg):
    import eacs_b200
    from cst_ssm.ops.spectral_init import BranchSpec

    eacs_b200.install("cst_ssm", fuse_ungated=True)
    layer = ref_pkg["modules.continuous_ssm"].ContinuousSSMLayer(
        16, BranchSpec("t", n_state=4, tau_min=0.5, tau_max=4.0))
    with pytest.raises(RuntimeError, match="CUDA"):
        layer(torch.randn(1, 5, 16), torch.cumsum(torch.full((1, 5), 0.25), 1))


def test_query_dispatch_keeps_reference_on_cpu_and_with_grad(ref_pkg):
    """Commits and query readouts: on CPU tensors (and wherever gradients must
    flow through the commits) the reference's own functions still run."""
    import eacs_b200
    from cst_ssm.ops.spectral_init import BranchSpec

    eacs_b200.install("cst_ssm", queries=True)
    eacs_b200.install("cst_ssm", queries=True)  # idempotent
    cq = ref_pkg["modules.continuous_query"]
    EACSLayer = ref_pkg["modules.eacs"].EACSLayer
    assert EACSLayer.run_with_commits.__wrapped__ is not None
    assert not hasattr(EACSLayer.run_with_commits.__wrapped__, "__wrapped__")
    torch.manual_seed(0)
    layer = EACSLayer(8, BranchSpec("t", n_state=4, tau_min=0.5, tau_max=4.0)).eval()
    x = torch.randn(2, 10, 8)
    t = torch.cumsum(torch.full((2, 10), 0.25), 1)
    tq = t[:, :5] + 0.1
    with torch.no_grad():
        out, commits = layer.run_with_commits(x, t)
        y = cq.readout_from_commits(layer, commits, tq)
        y2 = cq.continuous_query(layer, x, t, tq)
    assert commits["h"].shape == (2, 10, 8, 4) and y.shape == (2, 5, 8)
    assert torch.allclose(y, y2)
    assert torch.equal(cq.segment_index(t, tq), torch.arange(5).expand(2, 5))


def test_streaming_dispatch_keeps_reference_on_cpu(ref_pkg):
    import eacs_b200
    from cst_ssm.modules.multiscale import MultiScaleEACS
    from cst_ssm.ops.spectral_init import BranchSpec

    st_mod = importlib.import_module("cst_ssm.modules.streaming")
    saved = st_mod.temporal_step
    try:
        patched = eacs_b200.install("cst_ssm", streaming=True)
        assert "streaming.temporal_step" in patched
        assert st_mod.temporal_step.__wrapped__ is saved
        torch.manual_seed(0)
        temporal = MultiScaleEACS(8, branches=[BranchSpec("s", 4, 0.5, 4.0)]).eval()
        states = st_mod.initial_states(temporal, 2, "cpu")
        x = torch.randn(2, 8)
        with torch.no_grad():
            y, g, r, n, w, new = st_mod.temporal_step(temporal, x, torch.zeros(2), states,
                                                      torch.ones(2, dtype=torch.bool))
        assert y.shape == (2, 8) and bool(new[0].initialized.all())
    finally:
        st_mod.temporal_step = saved
        ap = sys.modules.get("cst_ssm.models.adaptive_path")
        if ap is not None and hasattr(ap.temporal_step, "__wrapped__"):
            ap.temporal_step = ap.temporal_step.__wrapped__


def test_multiscale_dispatch_keeps_reference_on_cpu(ref_pkg):
    import eacs_b200
    from cst_ssm.modules.multiscale import MultiScaleEACS
    from cst_ssm.ops.spectral_init import BranchSpec

    ms_mod = importlib.import_module("cst_ssm.modules.multiscale")
    saved = ms_mod.MultiScaleEACS.forward
    try:
        patched = eacs_b200.install("cst_ssm", multiscale=True)
        assert ms_mod.MultiScaleEACS.forward.__wrapped__ is saved
        assert "multiscale.MultiScaleEACS.forward" in patched
        torch.manual_seed(0)
        temporal = MultiScaleEACS(8, branches=[BranchSpec("a", 4, 0.5, 4.0),
                                               BranchSpec("b", 4, 4.0, 32.0)]).eval()
        with torch.no_grad():
            out = temporal(torch.randn(2, 6, 8), torch.cumsum(torch.full((2, 6), 0.25), 1))
        assert out.y.shape == (2, 6, 8) and out.fusion_weights.shape == (2, 6, 2)
    finally:
        ms_mod.MultiScaleEACS.forward = saved
