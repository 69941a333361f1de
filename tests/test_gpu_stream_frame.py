"""One streaming frame of a MultiScaleEACS as eacs_stream_frame (S + 3 launches)
against the reference's own temporal_step (modules/streaming.py:45-85) on the
same module and inputs, frame after frame, without autograd: outputs 1e-4
relative, gates identical (every residual checked to be off its threshold),
states 1e-4.  Also the path the library's temporal_step takes by itself
without autograd."""
import copy

import numpy as np
import pytest
import torch

from golden_io import relerr
from ref_pkg import import_reference, reference_only, reference_root, restore, snapshot

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(reference_root() is None, reason="reference package not present")]

DEV = "cuda:0"
TOL = 1e-4


@pytest.fixture()
def ref():
    mods = import_reference()
    if mods is None:
        pytest.skip("reference not importable")
    import importlib
    mods["modules.streaming"] = importlib.import_module("cst_ssm.modules.streaming")
    saved = snapshot(mods)
    reference_only(mods)
    yield mods
    restore(saved)


def _module(ref, d, specs, seed, cpi_mod=0.0, soft=False, eps=0.6):
    from cst_ssm.ops.spectral_init import BranchSpec
    torch.manual_seed(seed)
    m = ref["modules.multiscale"].MultiScaleEACS(
        d, branches=[BranchSpec(f"b{i}", n, lo, hi) for i, (n, lo, hi) in enumerate(specs)],
        gate_kwargs=dict(init_eps=eps, eps_max=3.0, cpi_modulation=cpi_mod, use_ste=not soft,
                         temperature=0.3)).to(DEV)
    with torch.no_grad():  # non-trivial affines and standardiser buffers
        for br in m.branches:
            br.norm.weight.uniform_(0.5, 1.5)
            br.norm.bias.uniform_(-0.2, 0.2)
            br.obs_norm.running_mean.normal_(0.0, 0.1)
            br.obs_norm.running_var.uniform_(0.5, 1.5)
        m.out_norm.weight.uniform_(0.5, 1.5)
        m.out_norm.bias.uniform_(-0.2, 0.2)
    m.train(soft)  # soft gates need training mode; eval otherwise
    return m


def _frames(B, K, d, seed, cpi=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, K, d, generator=g)
    for k in range(2, K, 3):  # repeated frames: skips
        x[:, k] = x[:, k - 1] + 0.02 * torch.randn(B, d, generator=g)
    t = 1.0 + torch.cumsum(0.25 + 1.75 * torch.rand(B, K, generator=g), 1)
    valid = torch.ones(B, K, dtype=torch.bool)
    valid[0, 1] = False
    valid[-1, 0] = False
    c = (torch.rand(B, K, generator=g) * 1.4 - 0.2) if cpi else None
    return x.to(DEV), t.to(DEV), valid.to(DEV), None if c is None else c.to(DEV)


@pytest.mark.parametrize("B,d,specs,cpi,soft", [
    (4, 96, [(16, 0.5, 4.0), (16, 4.0, 32.0), (16, 32.0, 256.0)], False, False),  # config 2's bands
    (3, 64, [(8, 0.5, 4.0), (32, 4.0, 32.0)], True, False),                      # CPI-modulated threshold
    (8, 128, [(5, 0.5, 4.0)], False, True),                                       # soft gate, 8 rows, ragged N
    (2, 1024, [(16, 0.5, 4.0), (16, 4.0, 32.0), (16, 32.0, 256.0)], False, False),  # config 2's width
])
def test_stream_frame_matches_reference(ref, B, d, specs, cpi, soft):
    from eacs_b200 import _lib
    from eacs_b200.ops.streaming import frame_fusable, temporal_step_frame
    st_mod = ref["modules.streaming"]
    m = _module(ref, d, specs, seed=B + d, cpi_mod=0.5 if cpi else 0.0, soft=soft)
    x, t, valid, c = _frames(B, 6, d, seed=d, cpi=cpi)
    s_ref = st_mod.initial_states(m, B, DEV)
    s_ours = st_mod.initial_states(m, B, DEV)
    assert frame_fusable(m, x[:, 0], s_ours)
    gates = []
    with torch.no_grad():
        for k in range(x.shape[1]):
            ck = None if c is None else c[:, k]
            init_before = torch.stack([st.initialized for st in s_ref], 1)
            y_r, g_r, r_r, n_r, w_r, s_ref = st_mod.temporal_step(m, x[:, k], t[:, k], s_ref, valid[:, k], ck)
            n0 = _lib.kernel_launches()
            y, g, r, n, w, s_ours = temporal_step_frame(m, x[:, k], t[:, k], s_ours, valid[:, k], ck)
            assert _lib.kernel_launches() - n0 == len(specs) + 3
            if not soft:  # every gate decided by more than 1e-5
                eps = torch.tensor([float(b.gate.eps.detach()) for b in m.branches], device=DEV)
                if ck is not None:
                    mod = torch.tensor([b.gate.cpi_modulation for b in m.branches], device=DEV)
                    eps = torch.clamp_min(eps[None] * (1 - mod[None] * ck.clamp(0, 1)[:, None]), 1e-3)
                live = valid[:, k][:, None] & init_before
                assert float(((r_r - eps).abs() + (~live) * 1.0).min()) > 1e-5
                assert torch.equal(g, g_r)
            else:
                assert relerr(g.cpu().numpy(), g_r.cpu().numpy()) < TOL
            gates.append(g_r)
            for got, want in ((y, y_r), (r, r_r), (n, n_r), (w, w_r)):
                assert relerr(got.cpu().numpy(), want.cpu().numpy()) < TOL
            for a, b in zip(s_ours, s_ref):
                for f in ("h", "t", "u", "B", "C"):
                    assert relerr(getattr(a, f).cpu().numpy(), getattr(b, f).cpu().numpy()) < TOL, f
                assert torch.equal(a.initialized, b.initialized)
    if not soft:
        gm = torch.stack(gates).float().mean()
        assert 0.1 < float(gm) < 0.99, float(gm)
    assert _lib.device_status() == 0


def test_temporal_step_takes_the_frame_path_without_autograd(ref):
    """The library's temporal_step (what install(streaming=True) binds) runs a
    frame as eacs_stream_frame under no_grad and as the per-branch path with
    autograd; both give the same frame."""
    from eacs_b200 import _lib
    from eacs_b200.ops.streaming import temporal_step
    st_mod = ref["modules.streaming"]
    m = _module(ref, 64, [(16, 0.5, 4.0), (8, 4.0, 32.0)], seed=3)
    x, t, valid, _ = _frames(2, 3, 64, seed=4)
    s1 = st_mod.initial_states(m, 2, DEV)
    s2 = st_mod.initial_states(m, 2, DEV)
    for k in range(3):
        n0 = _lib.kernel_launches()
        with torch.no_grad():
            y1, g1, r1, *_, s1 = temporal_step(m, x[:, k], t[:, k], s1, valid[:, k])
        assert _lib.kernel_launches() - n0 == 5
        y2, g2, r2, *_, s2 = temporal_step(m, x[:, k], t[:, k], s2, valid[:, k])
        assert y2.requires_grad
        assert torch.equal(g1, g2.detach())
        assert relerr(y1.cpu().numpy(), y2.detach().cpu().numpy()) < TOL
        s2 = [type(s)(*(z.detach() for z in (s.h, s.t, s.u, s.B, s.C)), s.initialized) for s in s2]
