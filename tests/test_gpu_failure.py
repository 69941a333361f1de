"""Failure detection on the GPU without a fault: the bounded device-side waits.

The repair and training passes wait on mbarriers that other CTAs of their
cluster complete; every such wait gives up after a fixed number of polls,
records EACS_ERR_TIMEOUT in the device status word and lets the kernel run to
its end.  eacs_wait_selftest runs those same waits, with a small poll limit,
on a phase that nothing completes: the waits must expire, the kernel must
end, the status must read EACS_ERR_TIMEOUT exactly once, and the context must
stay usable for the next call.
"""
import ctypes

import numpy as np
import pytest
import torch

from golden_io import relerr
from inputs import cell_inputs
from oracle import oracle

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_and_reports_timeout():
    from eacs_b200 import _lib
    from eacs_b200.ops.eacs_gated_scan import eacs_cell_forward
    lib = _lib.lib()
    torch.cuda.set_device(0)
    assert _lib.device_status() == 0
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.eacs_wait_selftest(4096, stream) == 0, _lib.last_error()
    st = ctypes.c_int(-1)
    assert lib.eacs_device_status(ctypes.byref(st), stream) == 0
    assert st.value == _lib.EACS_ERR_TIMEOUT
    assert _lib.device_status() == 0  # read and cleared
    # the context is still usable: a gated cell call right after matches the oracle
    d = cell_inputs(2, 40, 64, 16, seed=3)
    T = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in d.items()}
    y, g, r = eacs_cell_forward(T["lam"], T["log_dt"], T["u"], T["Bc"], T["Cc"], T["t"], T["D"], T["mean"],
                                T["var"], eps=0.12, eta=1e-6)
    y_ref, g_ref, _ = oracle.cell_fwd(**d, eps=0.12, eta=1e-6)
    assert np.array_equal(g.cpu().numpy(), g_ref)
    assert relerr(y.cpu().numpy(), y_ref) < 1e-4
    assert _lib.device_status() == 0
