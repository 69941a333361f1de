"""eacs_cell_fwd_noalloc: the gated cell with the library's own scratch array.

Some callers cannot allocate device memory -- a host that binds only the C ABI
and has no device allocator, or a process whose device memory belongs to
another allocator's pool.  For them the library keeps the cell's scratch in a
file-scope device array.  This test calls that entry point through the C ABI
several times in a row (hard gate, soft gate, bf16 u, hard gate again) and
checks each result against eacs_cell_fwd with a caller workspace.  It sorts last so that a run stopping at the first failure has
already run every other test, and it needs no state from them.
"""
import numpy as np
import pytest
import torch

from inputs import cell_inputs

pytestmark = pytest.mark.gpu

TOL = 1e-4  # forward tolerance used by the other parity tests


def _relerr(x, ref):
    return float((x - ref).abs().max()) / max(float(ref.abs().max()), 1e-30)


def _call(lib_fn, d, eps, outs, ws=None, gate_mode=0, u_dtype=0):
    y, g, r = outs
    args = [d["lam"].data_ptr(), d["log_dt"].data_ptr(), d["u"].data_ptr(), u_dtype,
            d["Bc"].data_ptr(), d["Cc"].data_ptr(), d["t"].data_ptr(), d["D"].data_ptr(),
            d["mean"].data_ptr(), d["var"].data_ptr(), eps, 1e-6, 1e-5, 1.0, 1e-3, 1e3,
            0, 3, 2.0, 0.3, gate_mode, 0.3, y.data_ptr(), g.data_ptr(), r.data_ptr()]
    if ws is not None:
        args += [ws.data_ptr(), ws.numel()]
    B, L, H = d["u"].shape
    N = d["lam"].shape[1]
    args += [B, L, H, N, torch.cuda.current_stream().cuda_stream]
    return lib_fn(*args)


def test_noalloc_matches_workspace_entry_point():
    """Hard gate, soft gate (which clears and reuses the row state in the
    scratch) and bf16 u, each compared with eacs_cell_fwd on a caller
    workspace; the hard-gate call runs before and after the others, so stale
    scratch contents from a different call would show."""
    from eacs_b200 import _lib
    lib = _lib.lib()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    host = cell_inputs(2, 96, 256, 16, seed=77)
    d = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in host.items()}
    d_bf = dict(d, u=d["u"].to(torch.bfloat16))
    B, L, H = d["u"].shape
    N = d["lam"].shape[1]

    def outs():
        return (torch.empty(B, L, H, device=dev), torch.empty(B, L, device=dev),
                torch.empty(B, L, device=dev))

    ws = torch.empty(lib.eacs_cell_fwd_workspace_size(B, L, H, N), dtype=torch.uint8, device=dev)
    # a threshold near the median residual, so gates mix and the repair pass
    # (which uses most of the scratch) runs
    probe = outs()
    assert _call(lib.eacs_cell_fwd, d, 0.0, probe, ws) == 0
    eps = float(probe[2].median())
    cases = {"hard": (d, 0, 0), "soft": (d, 1, 0), "bf16": (d_bf, 0, 2)}
    refs = {}
    for name, (dd, gm, ud) in cases.items():
        ref = outs()
        assert _call(lib.eacs_cell_fwd, dd, eps, ref, ws, gm, ud) == 0, _lib.last_error()
        refs[name] = ref
    rate = float(refs["hard"][1].mean())
    assert 0.05 < rate < 0.95, rate

    for name in ("hard", "soft", "bf16", "hard"):  # the array keeps each call's contents
        dd, gm, ud = cases[name]
        ref = refs[name]
        got = outs()
        rc = _call(lib.eacs_cell_fwd_noalloc, dd, eps, got, None, gm, ud)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        if gm == 0:
            assert torch.equal(got[1], ref[1]), f"{name}: gates differ"
        else:
            assert _relerr(got[1], ref[1]) < TOL, name
        assert _relerr(got[2], ref[2]) < TOL, name
        assert _relerr(got[0], ref[0]) < TOL, name
    assert _lib.device_status() == 0


def test_noalloc_rejects_sizes_beyond_the_array():
    from eacs_b200 import _lib
    lib = _lib.lib()
    B, L, H, N = 64, 65536, 2048, 32  # far more scratch than the array holds
    assert lib.eacs_cell_fwd_workspace_size(B, L, H, N) > (32 << 20)
    p = 256  # never dereferenced: the size check comes first
    rc = lib.eacs_cell_fwd_noalloc(p, p, p, 0, p, p, p, p, p, p, 0.1, 1e-6, 1e-5, 1.0, 1e-3, 1e3,
                                   0, 3, 2.0, 0.3, 0, 0.1, p, p, p, B, L, H, N, None)
    assert rc == _lib.EACS_ERR_WORKSPACE
    assert "static array" in _lib.last_error()
