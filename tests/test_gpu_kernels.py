"""CUDA kernels (through the C ABI) against the CPU oracle and golden vectors.

Tolerances: forward outputs 1e-4 relative (max |x - ref| / max |ref|), gate
masks bit-exact on every step whose residual is more than 1e-5 from its
threshold, scan adjoints 1e-4 relative.
"""
import numpy as np
import pytest
import torch

from golden_io import assert_cell_match, cases, cell_args, decisive, relerr
from inputs import cell_inputs, scan_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from eacs_b200 import _lib
    from eacs_b200.ops.continuous_ssm import ssm_forward
    from eacs_b200.ops.eacs_gated_scan import eacs_cell_forward
    from eacs_b200.ops.scan_cuda import EXT as SCAN, selective_scan_cuda

FWD_TOL = 1e-4
DEV = "cuda:0"


def _t(x, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(DEV)
    return t if dtype is None else t.to(dtype)


def _status_ok():
    assert _lib.device_status() == 0


# ------------------------------------------------------------------ scan ----
@pytest.mark.parametrize("name", sorted(cases("scan")))
def test_scan_golden(name):
    d = cases("scan")[name]
    h = SCAN.scan_fwd(_t(d["a"]), _t(d["b"]))[0].cpu().numpy()
    assert relerr(h, d["h"]) < 1e-5
    ga, gb = SCAN.scan_bwd(_t(d["a"]), _t(d["h"]), _t(d["gh"]))
    assert relerr(ga.cpu().numpy(), d["ga"]) < 1e-5
    assert relerr(gb.cpu().numpy(), d["gb"]) < 1e-5
    _status_ok()


@pytest.mark.parametrize("shape", [(2, 1000, 64, 16), (3, 37, 5, 3), (1, 1, 2, 4), (2, 129, 33, 2),
                                   (1, 4096, 8, 16)])
def test_scan_vs_oracle(shape):
    a, b, g = scan_inputs(*shape, seed=sum(shape))
    h = SCAN.scan_fwd(_t(a), _t(b))[0].cpu().numpy()
    h_ref = oracle.scan_fwd(a, b)
    assert relerr(h, h_ref) < FWD_TOL
    ga, gb = SCAN.scan_bwd(_t(a), _t(h_ref), _t(g))
    ga_ref, gb_ref = oracle.scan_bwd(a, h_ref, g)
    assert relerr(ga.cpu().numpy(), ga_ref) < FWD_TOL
    assert relerr(gb.cpu().numpy(), gb_ref) < FWD_TOL
    _status_ok()


def test_scan_autograd_and_misaligned_views():
    a, b, g = scan_inputs(2, 50, 6, 8, seed=3)
    at = _t(a).requires_grad_(True)
    bt = _t(b).requires_grad_(True)
    h = selective_scan_cuda(at, bt)
    h.backward(_t(g))
    ga_ref, gb_ref = oracle.scan_bwd(a, oracle.scan_fwd(a, b), g)
    assert relerr(at.grad.cpu().numpy(), ga_ref) < FWD_TOL
    assert relerr(bt.grad.cpu().numpy(), gb_ref) < FWD_TOL
    # a view whose base is only 8-byte aligned takes the plain-load path
    big = _t(np.concatenate([a.reshape(-1), a.reshape(-1)[:1]]))
    a_off = big[1:].view(a.shape)
    h2 = SCAN.scan_fwd(a_off, _t(b))[0]
    a_np = np.ascontiguousarray(np.concatenate([a.reshape(-1), a.reshape(-1)[:1]])[1:]).reshape(a.shape)
    assert relerr(h2.cpu().numpy(), oracle.scan_fwd(a_np, b)) < FWD_TOL


def test_scan_repeatable():
    a, b, _ = scan_inputs(2, 300, 16, 16, seed=9)
    outs = [SCAN.scan_fwd(_t(a), _t(b))[0].cpu().numpy() for _ in range(3)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])


# ------------------------------------------------------------------- ssm ----
def _ssm(d, u_dtype=torch.float32):
    return ssm_forward(_t(d["lam"]), _t(d["log_dt"]), _t(d["t"]), _t(d["Bc"]), _t(d["Cc"]),
                       _t(d["u"]).to(u_dtype), _t(d["D"])).cpu().numpy()


@pytest.mark.parametrize("name", sorted(cases("ssm")))
def test_ssm_golden(name):
    d = cases("ssm")[name]
    assert relerr(_ssm(d), d["y"]) < FWD_TOL
    _status_ok()


@pytest.mark.parametrize("B,L,H,N", [(2, 512, 96, 16), (1, 300, 40, 32), (2, 130, 24, 20), (2, 77, 19, 64),
                                     (3, 64, 33, 3), (1, 40, 128, 8)])
@pytest.mark.parametrize("u_dtype", ["f32", "f16", "bf16"])
def test_ssm_vs_oracle(B, L, H, N, u_dtype):
    d = cell_inputs(B, L, H, N, seed=B * L + N, tau=(0.5, 64.0))
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[u_dtype]
    # the oracle sees exactly the values the kernel reads
    d["u"] = _t(d["u"]).to(tdt).float().cpu().numpy()
    y_ref = oracle.ssm_fwd(d["lam"], d["log_dt"], d["t"], d["Bc"], d["Cc"], d["u"], d["D"])
    assert relerr(_ssm(d, tdt), y_ref) < FWD_TOL


# ------------------------------------------------------------------ cell ----
def _cell(d, u_dtype=torch.float32, **kw):
    y, g, r = eacs_cell_forward(_t(d["lam"]), _t(d["log_dt"]), _t(d["u"]).to(u_dtype), _t(d["Bc"]),
                                _t(d["Cc"]), _t(d["t"]), _t(d["D"]), _t(d["mean"]), _t(d["var"]),
                                **kw)
    return y.cpu().numpy(), g.cpu().numpy(), r.cpu().numpy()


@pytest.mark.parametrize("name", sorted(cases("cell")))
def test_cell_golden(name):
    d = cases("cell")[name]
    a = cell_args(d)
    got = _cell(d, **a)
    assert_cell_match(got, (d["y"], d["gate"], d["resid"]), a["eps"], a["robust"])
    _status_ok()


def _calibrated_eps(d, rate, robust=None, margin=2e-4):
    """eps giving roughly `rate` updates on the oracle, then nudged until no
    residual lies within `margin` of a threshold."""
    lo, hi = 0.0, 4.0
    for _ in range(30):
        mid = 0.5 * (lo + hi)
        _, g, _ = oracle.cell_fwd(**d, eps=mid, eta=1e-6, robust=robust)
        lo, hi = (mid, hi) if g.mean() > rate else (lo, mid)
    eps = 0.5 * (lo + hi)
    for _ in range(200):
        _, _, r = oracle.cell_fwd(**d, eps=eps, eta=1e-6, robust=robust)
        if decisive(r, eps, robust, margin).all():
            return eps
        eps *= 1.0 + 3 * margin
    raise AssertionError("no eps away from the residuals")


@pytest.mark.parametrize("B,L,H,N,rate,robust", [
    (2, 96, 768, 16, None, None),        # config-1 channel count, all commit
    (2, 64, 768, 16, 0.5, None),         # gate-exercising
    (3, 80, 100, 32, 0.3, None),
    (2, 70, 50, 24, 0.5, None),          # 16 < N < 32: four chains a thread, padded chains
    (1, 41, 36, 17, None, None),
    (2, 50, 70, 64, 0.7, None),
    (2, 60, 45, 5, 0.5, (3, 2.0, 0.3)),
    (2, 60, 64, 16, 0.5, (1, 1.05, 0.5)),
    (1, 1, 16, 16, None, None),
    (4, 33, 8, 1, 0.6, None),
])
def test_cell_vs_oracle(B, L, H, N, rate, robust):
    d = cell_inputs(B, L, H, N, seed=B + L + H + N)
    eps = 0.12 if rate is None else _calibrated_eps(d, rate, robust)
    ref = oracle.cell_fwd(**d, eps=eps, eta=1e-6, robust=robust)
    got = _cell(d, eps=eps, eta=1e-6, robust=robust)
    assert_cell_match(got, ref, eps, robust)
    _status_ok()


@pytest.mark.parametrize("B,L,H,N,rate,robust,u_dtype", [
    (8, 48, 768, 16, None, None, torch.float16),         # config-1 rows: 18 tiles of 44 channels, last 20
    (8, 40, 768, 16, 0.5, None, torch.float16),          # skips: replay and repair after the wide pass
    (16, 40, 384, 16, 0.6, None, torch.float32),         # last tile 32 channels
    (6, 40, 975, 16, 0.5, None, torch.float16),          # odd H: synchronous staging
    (8, 40, 768, 12, 0.5, (3, 2.0, 0.3), torch.bfloat16),  # padded chains, robust_guard
])
def test_cell_wide_tiles(B, L, H, N, rate, robust, u_dtype):
    """Row counts whose four-warp tiles put three or more CTAs on an SM run the
    speculative pass as one 11-warp CTA per SM (44-channel tiles, B x tiles <=
    SM count); results are the oracle's like every other layout."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    if sms == 148:
        assert B * -(-H // 44) <= sms < B * -(-H // 16) / 2, "shape does not select the wide layout"
    d = cell_inputs(B, L, H, N, seed=B + L + H + N)
    d["u"] = _t(d["u"]).to(u_dtype).float().cpu().numpy()
    eps = 0.12 if rate is None else _calibrated_eps(d, rate, robust)
    ref = oracle.cell_fwd(**d, eps=eps, eta=1e-6, robust=robust)
    got = _cell(d, u_dtype=u_dtype, eps=eps, eta=1e-6, robust=robust)
    assert_cell_match(got, ref, eps, robust)
    _status_ok()


@pytest.mark.parametrize("u_dtype", [torch.float16, torch.bfloat16])
def test_cell_half_inputs(u_dtype):
    d = cell_inputs(2, 70, 96, 16, seed=5)
    d["u"] = _t(d["u"]).to(u_dtype).float().cpu().numpy()
    eps = _calibrated_eps(d, 0.6)
    ref = oracle.cell_fwd(**d, eps=eps, eta=1e-6)
    got = _cell(d, u_dtype=u_dtype, eps=eps, eta=1e-6)
    assert_cell_match(got, ref, eps, None)


def test_cell_soft_gate():
    d = cell_inputs(2, 40, 24, 8, seed=21)
    ref = oracle.cell_fwd(**d, eps=0.9, eta=1e-6, gate_mode=1, T=0.3)
    y, g, r = _cell(d, eps=0.9, eta=1e-6, gate_mode="soft", temperature=0.3)
    assert relerr(g, ref[1]) < FWD_TOL
    assert relerr(r, ref[2]) < FWD_TOL
    assert relerr(y, ref[0]) < FWD_TOL


def test_cell_repeatable_and_decreasing_time():
    d = cell_inputs(2, 64, 48, 16, seed=33)
    d["t"][0, 10] = d["t"][0, 9]           # dt = 0 -> dt_min
    d["t"][1, 20] = d["t"][1, 19] - 0.7    # decreasing -> clamp_min(0)
    eps = _calibrated_eps(d, 0.5)
    ref = oracle.cell_fwd(**d, eps=eps, eta=1e-6)
    outs = [_cell(d, eps=eps, eta=1e-6) for _ in range(3)]
    assert_cell_match(outs[0], ref, eps, None)
    for o in outs[1:]:
        for x, y in zip(outs[0], o):
            assert np.array_equal(x, y)


def test_cells_side_by_side():
    """Three cells of B=4, H=1024, N=16 launched side by side on their own
    streams (MultiScaleEACS's branches at config 2's width) are told so and
    run the speculative pass with four chains a thread, so their CTAs fit the
    GPU in one wave.  Each matches the oracle like a lone call, with and
    without skips, and a count below 1 is rejected."""
    from eacs_b200.ops.eacs_gated_scan import side_by_side
    from eacs_b200.ops.multiscale import run_branches
    B, L, H, N = 4, 48, 1024, 16
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    if sms == 148:
        assert 3 * B * (H // 16) > 4 * sms >= 3 * B * (H // 32), "shape does not select the layout"
    ds = [cell_inputs(B, L, H, N, seed=300 + k) for k in range(3)]
    epss = [0.12, _calibrated_eps(ds[1], 0.5), 0.12]
    refs = [oracle.cell_fwd(**d, eps=e, eta=1e-6) for d, e in zip(ds, epss)]
    outs = run_branches(list(range(3)), torch.device(DEV),
                        lambda i, _: eacs_cell_forward(
                            _t(ds[i]["lam"]), _t(ds[i]["log_dt"]), _t(ds[i]["u"]), _t(ds[i]["Bc"]),
                            _t(ds[i]["Cc"]), _t(ds[i]["t"]), _t(ds[i]["D"]), _t(ds[i]["mean"]),
                            _t(ds[i]["var"]), eps=epss[i], eta=1e-6))
    torch.cuda.synchronize()
    for o, ref, d, e in zip(outs, refs, ds, epss):
        got = tuple(x.cpu().numpy() for x in o)
        assert_cell_match(got, ref, e, None)
        alone = _cell(d, eps=e, eta=1e-6)
        assert np.array_equal(got[1], alone[1])
        assert relerr(got[0], alone[0]) < 1e-5 and relerr(got[2], alone[2]) < 1e-5
    assert 0.0 < refs[1][1].mean() < 1.0
    _status_ok()
    with side_by_side(0):  # clamped to 1 on the Python side: a lone call
        y = _cell(ds[0], eps=0.12, eta=1e-6)[0]
    assert np.array_equal(y, _cell(ds[0], eps=0.12, eta=1e-6)[0])
    args = ([None, None, None, 0] + [None] * 6 + [0.0] * 6 + [0, 3, 2.0, 0.3, 0, 0.1]
            + [None] * 4 + [0, 1, 1, 1, 1, 0, None])
    rc = _lib.lib().eacs_cell_fwd_side_by_side(*args)
    assert rc != 0 and b"cells_side_by_side" in _lib.lib().eacs_last_error()
