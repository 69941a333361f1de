"""C ABI checks that need no GPU: the library loads, exports every symbol the
header declares, and rejects bad arguments before touching the device."""
import ctypes
import os
import re

import pytest
import torch

from eacs_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "eacs_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"EACS_API\s+[\w\s\*]+?\b(eacs_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "eacs_cell_fwd" in syms and "eacs_scan_fwd" in syms and len(syms) >= 8


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing
    # the Python binding covers the same set
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_version_and_last_error():
    assert "sm_100a" in _lib.version()
    assert isinstance(_lib.last_error(), str)


def test_cell_rejects_unsupported_n_without_device():
    L = _lib.lib()
    rc = L.eacs_cell_fwd(*([None] * 3), 0, *([None] * 6), 0.1, 1e-6, 1e-5, 1.0, 1e-3, 1e3,
                         0, 0, 2.0, 0.3, 0, 0.1, None, None, None, None, 0, 2, 8, 4, 65, None)
    assert rc == _lib.EACS_ERR_UNSUPPORTED
    assert "N=65" in _lib.last_error()


def test_cell_rejects_missing_workspace_without_device():
    L = _lib.lib()
    p = 16  # any non-null pointer value; rejected before use
    rc = L.eacs_cell_fwd(p, p, p, 0, p, p, p, p, p, p, 0.1, 1e-6, 1e-5, 1.0, 1e-3, 1e3,
                         0, 0, 2.0, 0.3, 0, 0.1, p, p, p, None, 0, 2, 8, 4, 16, None)
    assert rc == _lib.EACS_ERR_WORKSPACE
    assert L.eacs_cell_fwd_workspace_size(2, 8, 4, 16) > 0
    assert L.eacs_cell_fwd_workspace_size(2, 8, 4, 65) == 0


def test_cell_rejects_bad_dtype_and_gate_mode():
    L = _lib.lib()
    p = 16
    rc = L.eacs_cell_fwd(p, p, p, 7, p, p, p, p, p, p, 0.1, 1e-6, 1e-5, 1.0, 1e-3, 1e3,
                         0, 0, 2.0, 0.3, 0, 0.1, p, p, p, p, 1 << 30, 2, 8, 4, 16, None)
    assert rc == _lib.EACS_ERR_INVALID
    rc = L.eacs_cell_fwd(p, p, p, 0, p, p, p, p, p, p, 0.1, 1e-6, 1e-5, 1.0, 1e-3, 1e3,
                         0, 0, 2.0, 0.3, 3, 0.1, p, p, p, p, 1 << 30, 2, 8, 4, 16, None)
    assert rc == _lib.EACS_ERR_INVALID


def test_train_fwd_ckpt_rejects_missing_backward_workspace_without_device():
    """The checkpoint-writing training forward needs the backward's workspace;
    it is checked before anything touches the device."""
    L = _lib.lib()
    p = 16  # any non-null pointer value; rejected before use
    B, Ln, H, N = 2, 16, 8, 16
    need = L.eacs_cell_train_bwd_workspace_size(B, Ln, H, N)
    assert need > 0
    for ws, nbytes in ((None, 0), (p, need - 1)):
        rc = L.eacs_cell_train_fwd_ckpt(p, p, p, 0, p, p, p, p, p, p, 0.1, 1e-6, 1e-5, 1.0, 1e-3, 1e3, 0, 0.1,
                                        p, p, p, p, p, 1 << 30, ws, nbytes, B, Ln, H, N, None)
        assert rc == _lib.EACS_ERR_WORKSPACE
        assert "backward workspace" in _lib.last_error()


def test_empty_shapes_are_noops():
    L = _lib.lib()
    assert L.eacs_scan_fwd(None, None, None, 0, 5, 3, 2, None) == _lib.EACS_OK
    assert L.eacs_scan_bwd(None, None, None, None, None, 2, 0, 3, 2, None) == _lib.EACS_OK
    assert L.eacs_ssm_fwd(None, None, None, None, None, None, 0, None, None, 2, 0, 3, 2,
                          1e-3, 1e3, None) == _lib.EACS_OK


def test_python_ops_reject_cpu_tensors():
    from eacs_b200.ops.eacs_gated_scan import eacs_cell_forward
    from eacs_b200.ops.scan_cuda import EXT
    a = torch.zeros(1, 2, 3, 4, dtype=torch.complex64)
    with pytest.raises(RuntimeError, match="CUDA"):
        EXT.scan_fwd(a, a)
    H, N = 3, 4
    z = torch.zeros(H)
    with pytest.raises(RuntimeError, match="CUDA"):
        eacs_cell_forward(torch.zeros(H, N, dtype=torch.complex64), z, torch.zeros(1, 2, H),
                          torch.zeros(1, 2, N, dtype=torch.complex64),
                          torch.zeros(1, 2, N, dtype=torch.complex64), torch.zeros(1, 2), z, z, z,
                          0.1, 1e-6)


def test_wait_selftest_rejects_bad_poll_counts_without_device():
    lib = _lib.lib()
    for polls in (0, -1, 65537):
        assert lib.eacs_wait_selftest(polls, None) == _lib.EACS_ERR_INVALID
    assert "polls" in _lib.last_error()


def test_project_rejects_bad_arguments_without_device():
    from eacs_b200 import _lib
    lib = _lib.lib()
    p = 256
    # d not a multiple of 8
    assert lib.eacs_project(p, 1, p, p, 1e-5, p, 1, 256, p, p, 1, p, p, p, 80, 10, 12, 8, 4, None) == _lib.EACS_ERR_UNSUPPORTED
    # too few weight rows
    assert lib.eacs_project(p, 1, p, p, 1e-5, p, 1, 0, p, p, 1, p, p, p, 80, 10, 16, 8, 4, None) == _lib.EACS_ERR_INVALID
    # float32 weight
    assert lib.eacs_project(p, 1, p, p, 1e-5, p, 0, 256, p, p, 1, p, p, p, 80, 10, 16, 8, 4, None) == _lib.EACS_ERR_INVALID
    # workspace too small (checked before any launch)
    assert lib.eacs_project(p, 1, p, p, 1e-5, p, 1, 256, p, p, 1, p, p, p, 8, 10, 16, 8, 4, None) == _lib.EACS_ERR_WORKSPACE
    assert lib.eacs_project_workspace_size(10) == 80


def test_commit_training_rejects_bad_arguments_without_device():
    """eacs_cell_train_commits_fwd/_bwd check the gate mode, the backward
    workspace and the commit buffers before anything touches the device."""
    L = _lib.lib()
    p = 256
    B, Ln, H, N = 2, 16, 8, 16
    need = L.eacs_cell_train_commits_workspace_size(B, Ln, H, N)
    assert need > 0 and L.eacs_cell_train_commits_workspace_size(B, Ln, H, 65) == 0
    head = (p, p, p, 0, p, p, p, p, p, p, 0.1, 1e-6, 1e-5, 1.0, 1e-3, 1e3)

    def fwd(gate_mode=0, commits=(p,) * 5, bws=p, bwn=None):
        return L.eacs_cell_train_commits_fwd(*head, gate_mode, 0.1, p, p, p, p, *commits, p, 1 << 30,
                                             bws, need if bwn is None else bwn, B, Ln, H, N, None)
    assert fwd(gate_mode=3) == _lib.EACS_ERR_INVALID and "gate_mode" in _lib.last_error()
    assert fwd(bws=None, bwn=0) == _lib.EACS_ERR_WORKSPACE
    assert fwd(bwn=need - 1) == _lib.EACS_ERR_WORKSPACE
    assert fwd(commits=(p, None, p, p, p)) == _lib.EACS_ERR_INVALID

    def bwd(gate_mode=0, ws=p, wn=None):
        return L.eacs_cell_train_commits_bwd(*head, gate_mode, 0.1, p, p, p, p, None, None, None, None, None,
                                             None, None, p, p, p, p, p, p, p, p, ws, need if wn is None else wn,
                                             B, Ln, H, N, None)
    assert bwd(gate_mode=-1) == _lib.EACS_ERR_INVALID
    assert bwd(ws=None, wn=0) == _lib.EACS_ERR_WORKSPACE


def test_query_readout_bwd_rejects_bad_arguments_without_device():
    L = _lib.lib()
    p = 256
    B, Ln, Q, H, N = 2, 16, 5, 8, 16
    need = L.eacs_query_readout_bwd_workspace_size(B, Ln, Q, H, N)
    assert need > 0 and L.eacs_query_readout_bwd_workspace_size(B, Ln, Q, H, 65) == 0

    def call(ptrs=(p,) * 20, ws=p, wn=None, n=N, b=B):
        return L.eacs_query_readout_bwd(*ptrs, ws, need if wn is None else wn, b, Ln, Q, H, n, 1e-3, 1e3, None)
    assert call(n=65) == _lib.EACS_ERR_UNSUPPORTED
    assert call(ptrs=(p,) * 10 + (None,) + (p,) * 9) == _lib.EACS_ERR_INVALID   # gy
    assert call(wn=need - 1) == _lib.EACS_ERR_WORKSPACE
    assert call(b=0) == _lib.EACS_OK


def test_stream_step_bwd_rejects_bad_arguments_without_device():
    L = _lib.lib()
    p = 256
    B, H, N = 2, 8, 16
    need = L.eacs_stream_step_bwd_workspace_size(B, H, N)
    assert need > 0 and L.eacs_stream_step_bwd_workspace_size(0, H, N) == 0

    def call(ptrs=(p,) * 41, wn=None, gate_mode=0, n=N, b=B):
        return L.eacs_stream_step_bwd(*ptrs, p, need if wn is None else wn, 0.1, 1e-6, 1e-5, 1.0, 1e-3, 1e3, 0.0,
                                      gate_mode, 0.1, b, H, n, None)
    assert call(gate_mode=3) == _lib.EACS_ERR_INVALID
    assert call(n=65) == _lib.EACS_ERR_UNSUPPORTED
    assert call(ptrs=(None,) + (p,) * 40) == _lib.EACS_ERR_INVALID
    assert call(wn=need - 1) == _lib.EACS_ERR_WORKSPACE
    assert call(b=0) == _lib.EACS_OK
