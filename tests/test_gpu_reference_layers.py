"""The reference's own layers on CUDA, unmodified, with and without install().

Each test builds a reference module (cst_ssm, imported from the reference
package: tests/ref_pkg.py) on the GPU and runs it twice on the same inputs:

* reference only: its CUDA extensions are marked absent, so the reference
  runs its own PyTorch code on the GPU (EACSLayer's step loop, MultiScaleEACS's
  merged loop, ContinuousSSMLayer's associative scan, GatedEACSCellFunction's
  Python forward and per-step autograd backward);
* after eacs_b200.install(): the same module objects, now reaching this
  library's kernels through the reference's own lazy imports.

The installed run must launch this library's kernels (its launch counter
grows: the reference's callers swallow extension errors and would otherwise
fall back silently, modules/eacs.py:308-311) and match the reference-only run:
forward outputs 1e-4 relative, gates bit-exact where the residual is more than
1e-5 from its threshold, gradients 1e-3 relative.
"""
import copy

import numpy as np
import pytest
import torch

from golden_io import decisive, relerr
from ref_pkg import import_reference, reference_only, reference_root, restore, snapshot

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(reference_root() is None, reason="reference package not present")]

FWD_TOL = 1e-4
GRAD_TOL = 1e-3
DEV = "cuda:0"


@pytest.fixture()
def ref():
    mods = import_reference()
    if mods is None:
        pytest.skip("reference not importable")
    saved = snapshot(mods)
    reference_only(mods)
    yield mods
    restore(saved)


def _launches():
    from eacs_b200 import _lib
    return _lib.kernel_launches()


def _install(**kw):
    import eacs_b200
    eacs_b200.install("cst_ssm", **kw)


def _video(B, L, d, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(B, L, d, generator=g) * scale).to(DEV)
    dt = 0.25 + 1.75 * torch.rand(B, L, generator=g)
    dt[torch.rand(B, L, generator=g) < 0.1] = 0.25
    return x, torch.cumsum(dt, 1).to(DEV)


def _rows_match(y, y_ref, g, g_ref, r_ref, eps):
    """Row by row up to the first step whose residual is within 1e-5 of eps."""
    dec = decisive(r_ref, eps, None)
    compared = 0
    for b in range(g_ref.shape[0]):
        bad = np.where(~dec[b])[0]
        stop = int(bad[0]) if bad.size else g_ref.shape[1]
        assert np.array_equal(g[b, :stop], g_ref[b, :stop]), f"row {b}: gates"
        assert relerr(y[b, :stop], y_ref[b, :stop]) < FWD_TOL, f"row {b}: y"
        compared += stop
    assert compared >= 0.9 * g_ref.size


@pytest.mark.parametrize("half_skip", [False, True])
def test_eacs_layer_eval(ref, half_skip):
    """EACSLayer.eval() at config 1's width (H=768, N=16, tau [0.1, 1] s).
    With half_skip the gate's threshold is lifted (eps_anneal) to the median
    residual, so about half the frames skip (the repair path)."""
    from cst_ssm.modules.event_gate import EventGate
    from cst_ssm.ops.spectral_init import BranchSpec
    torch.manual_seed(0)
    layer = ref["modules.eacs"].EACSLayer(768, BranchSpec("short", 16, 0.1, 1.0),
                                          gate=EventGate(init_eps=0.12)).to(DEV).eval()
    x, t = _video(2, 96, 768, 1)
    with torch.no_grad():
        if half_skip:  # bisect the threshold (through eps_anneal) to an update rate near 0.5
            base = float(layer.gate.eps) / float(layer.gate.eps_anneal)
            lo, hi = 0.0, 2.0
            for _ in range(14):
                mid = 0.5 * (lo + hi)
                layer.gate.set_eps_anneal(mid / base)
                rate = float(layer(x, t).gates.mean())
                lo, hi = (mid, hi) if rate > 0.5 else (lo, mid)
            eps = 0.5 * (lo + hi)
            for _ in range(200):  # then away from every residual, so each gate is decided
                layer.gate.set_eps_anneal(eps / base)
                if decisive(layer(x, t).residual.cpu().numpy(), eps, None, 2e-5).all():
                    break
                eps *= 1.00002
        n0 = _launches()
        out_ref = layer(x, t)
        assert _launches() == n0
        _install()
        out = layer(x, t)
        assert _launches() > n0
        eps = float(layer.gate.eps)
    g, g_ref = out.gates.cpu().numpy(), out_ref.gates.cpu().numpy()
    if half_skip:
        assert 0.2 < g_ref.mean() < 0.8
    _rows_match(out.y.cpu().numpy(), out_ref.y.cpu().numpy(), g, g_ref,
                out_ref.residual.cpu().numpy(), eps)


@pytest.mark.parametrize("T", [torch.float16, torch.bfloat16])
def test_eacs_layer_eval_autocast(ref, T):
    """EACSLayer.eval() inside an autocast region: after install(layer_dispatch=True)
    LayerNorm and the input projections run as the tensor-core kernel, the
    cell and proj_out follow.  The reference runs its own autocast path.  Both
    round the projections' outputs to T, in different summation orders, so
    the layer output is compared to 2e-3 of its largest value (a few units in
    the last place of float16 in the projected inputs) with identical gates."""
    from cst_ssm.modules.event_gate import EventGate
    from cst_ssm.ops.spectral_init import BranchSpec
    torch.manual_seed(0)
    layer = ref["modules.eacs"].EACSLayer(768, BranchSpec("short", 16, 0.1, 1.0),
                                          gate=EventGate(init_eps=0.12)).to(DEV).eval()
    x, t = _video(2, 96, 768, 7)
    with torch.no_grad(), torch.autocast("cuda", T):
        n0 = _launches()
        out_ref = layer(x, t)
        assert _launches() == n0
        _install(layer_dispatch=True)
        calls = dict(_lib_calls())
        out = layer(x, t)
        assert _launches() > n0 and _lib_calls().get("eacs_project", 0) > calls.get("eacs_project", 0)
    assert torch.equal(out.gates, out_ref.gates)
    assert relerr(out.y.float().cpu().numpy(), out_ref.y.float().cpu().numpy()) < 2e-3


def _lib_calls():
    from eacs_b200 import _lib
    return _lib.calls


def test_multiscale_eval(ref):
    """MultiScaleEACS with config 2's three branch bands (N=16 each), whose
    reference path is the merged sequential loop over the branches."""
    from cst_ssm.ops.spectral_init import BranchSpec
    torch.manual_seed(0)
    specs = [BranchSpec("short", 16, 0.5, 4.0), BranchSpec("mid", 16, 4.0, 32.0),
             BranchSpec("long", 16, 32.0, 256.0)]
    ms = ref["modules.multiscale"].MultiScaleEACS(256, branches=specs,
                                                  gate_kwargs={"init_eps": 0.12}).to(DEV).eval()
    x, t = _video(2, 80, 256, 2)
    with torch.no_grad():
        assert ms._merge_ok(x)
        n0 = _launches()
        out_ref = ms(x, t)
        assert _launches() == n0
        _install(multiscale=True)
        out = ms(x, t)
        assert _launches() > n0
    assert relerr(out.y.cpu().numpy(), out_ref.y.cpu().numpy()) < FWD_TOL
    assert relerr(out.fusion_weights.cpu().numpy(), out_ref.fusion_weights.cpu().numpy()) < FWD_TOL


def test_continuous_ssm_layer_forward_backward(ref):
    """ContinuousSSMLayer (config 0's shape: H=64, N=16): forward and every
    parameter gradient, the reference's associative scan against the fused
    ungated core."""
    from cst_ssm.ops.spectral_init import BranchSpec
    torch.manual_seed(0)
    layer = ref["modules.continuous_ssm"].ContinuousSSMLayer(64, BranchSpec("b", 16, 0.5, 64.0)).to(DEV)
    twin = copy.deepcopy(layer)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 256, 64, generator=g).to(DEV)
    dt = torch.empty(2, 256).exponential_(4.0, generator=g).clamp(1 / 30, 2.0)
    t = torch.cumsum(dt, 1).to(DEV)
    gy = torch.randn(2, 256, 64, generator=g).to(DEV)
    n0 = _launches()
    y_ref = layer(x, t)
    y_ref.backward(gy)
    assert _launches() == n0
    _install(fuse_ungated=True)
    y = twin(x, t)
    y.backward(gy)
    assert _launches() > n0
    assert relerr(y.detach().cpu().numpy(), y_ref.detach().cpu().numpy()) < FWD_TOL
    for (name, p), p_ref in zip(twin.named_parameters(), layer.parameters()):
        assert relerr(p.grad.cpu().numpy(), p_ref.grad.cpu().numpy()) < GRAD_TOL, name


def test_eacs_layer_fused_train(ref):
    """EACSLayer(fused_train=True) in training mode: the layer output, the
    innovation loss and every parameter gradient, the reference's
    GatedEACSCellFunction (Python forward, per-step autograd backward) against
    this library's checkpointed backward kernels."""
    from cst_ssm.modules.event_gate import EventGate
    from cst_ssm.ops.spectral_init import BranchSpec
    torch.manual_seed(0)
    layer = ref["modules.eacs"].EACSLayer(128, BranchSpec("short", 16, 0.5, 4.0),
                                          gate=EventGate(init_eps=0.12), fused_train=True).to(DEV).train()
    twin = copy.deepcopy(layer)
    x, t = _video(2, 48, 128, 4)
    gy = torch.randn(x.shape, generator=torch.Generator().manual_seed(5)).to(DEV)

    def run(m):
        out = m(x, t)
        loss = (out.y * gy).sum() + out.innovation.square().mean()
        loss.backward()
        return out

    n0 = _launches()
    out_ref = run(layer)
    assert _launches() == n0
    _install()
    out = run(twin)
    assert _launches() > n0
    assert torch.equal(out.gates, out_ref.gates)
    assert relerr(out.y.detach().cpu().numpy(), out_ref.y.detach().cpu().numpy()) < FWD_TOL
    assert relerr(out.residual.detach().cpu().numpy(), out_ref.residual.detach().cpu().numpy()) < FWD_TOL
    for (name, p), p_ref in zip(twin.named_parameters(), layer.parameters()):
        if p_ref.grad is None:
            assert p.grad is None or not p.grad.any(), name
            continue
        assert relerr(p.grad.cpu().numpy(), p_ref.grad.cpu().numpy()) < GRAD_TOL, name


@pytest.mark.parametrize("train", [True, False])
def test_continuous_query_gradients(ref, train):
    """continuous_query (modules/continuous_query.py:56-65) under autograd:
    run_with_commits (training mode: the STE gate; eval mode: r > eps) and
    readout_from_commits at query times between, on and around the frames.
    The loss's gradients with respect to the input and every parameter, the
    reference's own step loop and autograd against install(queries=True)'s
    commit and readout kernels (eacs_cell_train_commits_*,
    eacs_query_readout_bwd).  The threshold is bisected (eps_anneal) to an
    update rate near one half and moved away from every residual."""
    from cst_ssm.modules.event_gate import EventGate
    from cst_ssm.ops.spectral_init import BranchSpec
    cq = ref["modules.continuous_query"]
    torch.manual_seed(0)
    layer = ref["modules.eacs"].EACSLayer(96, BranchSpec("short", 16, 0.5, 4.0),
                                          gate=EventGate(init_eps=0.12)).to(DEV)
    x, t = _video(2, 40, 96, 12)
    g = torch.Generator().manual_seed(13)
    tq = (t[:, :1] - 0.2 + (t[:, -1:] - t[:, :1] + 0.5) * torch.rand(2, 33, generator=g).to(DEV)).sort(1).values
    tq[:, 3] = t[:, 7]
    gq = torch.randn(2, 33, 96, generator=g).to(DEV)
    layer.eval()
    with torch.no_grad():
        base = float(layer.gate.eps) / float(layer.gate.eps_anneal)
        lo, hi = 0.0, 4.0
        for _ in range(14):
            mid = 0.5 * (lo + hi)
            layer.gate.set_eps_anneal(mid / base)
            rate = float(layer.run_with_commits(x, t)[0].gates.mean())
            lo, hi = (mid, hi) if rate > 0.5 else (lo, mid)
        eps = 0.5 * (lo + hi)
        for _ in range(200):
            layer.gate.set_eps_anneal(eps / base)
            r = layer.run_with_commits(x, t)[0].residual.cpu().numpy()
            if decisive(r, eps, None, 2e-5).all():
                break
            eps *= 1.00002
    layer.train(train)
    twin = copy.deepcopy(layer)

    def run(m):
        xx = x.clone().requires_grad_(True)
        y = cq.continuous_query(m, xx, t, tq)
        (y * gq).sum().backward()
        return y.detach(), xx.grad

    n0 = _launches()
    y_ref, gx_ref = run(layer)
    assert _launches() == n0
    _install(queries=True)
    y, gx = run(twin)
    assert _launches() > n0
    rate = float(twin.run_with_commits(x, t)[0].gates.detach().float().mean())
    assert 0.2 < rate < 0.8, rate
    assert relerr(y.cpu().numpy(), y_ref.cpu().numpy()) < FWD_TOL
    assert relerr(gx.cpu().numpy(), gx_ref.cpu().numpy()) < GRAD_TOL
    for (name, p), p_ref in zip(twin.named_parameters(), layer.parameters()):
        if p_ref.grad is None:
            assert p.grad is None or not p.grad.any(), name
            continue
        assert relerr(p.grad.cpu().numpy(), p_ref.grad.cpu().numpy()) < GRAD_TOL, name
