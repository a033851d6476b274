"""CPU tests of the C ABI boundary: libgsb200.so loads, exports exactly the
symbols include/gsb200.h declares, and rejects bad arguments on the host
(no CUDA call is made on these paths, so they run without a GPU)."""
import ctypes
import os
import re
import subprocess

import pytest

from gs_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gsb200.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^GS_API\s+[\w\s\*]+?\b(gs_\w+)\s*\(", src, flags=re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 17
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes table and header disagree"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r" T (gs_\w+)", out))
    assert exported == set(names)


def test_status_strings_and_version():
    lib = _lib.lib()
    assert lib.gs_status_string(0) == b"ok"
    assert b"capacity" in lib.gs_status_string(_lib.GS_ERR_CAPACITY)
    assert lib.gs_status_string(99) == b"unknown status"
    assert lib.gs_version() >> 16 == 1


def test_sizes():
    lib = _lib.lib()
    assert lib.gs_default_capacity(10) == 2560
    small = lib.gs_workspace_bytes(1000, 64, 48, 1000)
    big = lib.gs_workspace_bytes(1000, 64, 48, 256000)
    assert 0 < small < big
    assert big - small >= 4 * 4 * 254000  # double-buffered keys + ids (256-byte padding)
    assert lib.gs_workspace_bytes(-1, 64, 48, 0) == 0
    assert lib.gs_dssim_workspace_bytes(378, 504, 3) >= 3 * 378 * 504 * 3 * 4


def _render_forward(lib, n=10, W=64, H=48, cap=None, ws=None, ws_bytes=None, sh_k=16, deg=3):
    cap = lib.gs_default_capacity(n) if cap is None else cap
    need = lib.gs_workspace_bytes(max(n, 0), W, max(H, 1), cap)
    ws = ctypes.c_void_p(0x1000) if ws is None else ws  # never dereferenced: rejected first
    ws_bytes = need if ws_bytes is None else ws_bytes
    p = ctypes.c_void_p(0x2000)
    return lib.gs_render_forward(p, p, p, p, p, n, sh_k, None, p, W, H, 1.0, 1.0, 0.0, 0.0, None, deg,
                                 cap, ws, ws_bytes, p, p, p, p, None)


def test_host_side_argument_validation():
    lib = _lib.lib()
    E = _lib.GS_ERR_INVALID_ARGUMENT
    assert _render_forward(lib, n=-1) == E
    assert _render_forward(lib, W=0) == E
    assert _render_forward(lib, deg=4) == E
    assert _render_forward(lib, sh_k=4, deg=3) == E  # K < (deg+1)^2
    assert _render_forward(lib, cap=-5) == E
    assert _render_forward(lib, W=1 << 20, H=1 << 20) == E  # too many tiles for the key
    assert _render_forward(lib, ws_bytes=16) == _lib.GS_ERR_WORKSPACE_TOO_SMALL
    assert _render_forward(lib, ws=ctypes.c_void_p(0)) == _lib.GS_ERR_WORKSPACE_TOO_SMALL
    assert _render_forward(lib, ws=ctypes.c_void_p(0x1001)) == E  # misaligned workspace
    p = ctypes.c_void_p(0x2000)
    assert lib.gs_l1_loss(p, p, 10, 1.0, None, None, p, 4096, None) == E
    assert lib.gs_l1_loss(p, p, 10, 1.0, p, None, p, 16, None) == _lib.GS_ERR_WORKSPACE_TOO_SMALL
    assert lib.gs_mse_loss(p, p, -1, 1.0, p, None, p, 4096, None) == E
    assert lib.gs_mse_loss(p, p, 10, 1.0, None, None, p, 4096, None) == E
    assert lib.gs_mse_loss(p, p, 10, 1.0, p, None, p, 16, None) == _lib.GS_ERR_WORKSPACE_TOO_SMALL
    assert lib.gs_covariance_3d(p, p, -1, p, None) == E
    assert lib.gs_covariance_3d(None, p, 10, p, None) == E
    assert lib.gs_covariance_3d(p, p, 10, None, None) == E
    assert lib.gs_dssim_loss(p, p, 0, 4, 3, 1.0, p, None, None, p, 1 << 20, None) == E
    assert lib.gs_adam_step(p, p, p, p, 10, 16, None, None, 1, 0.9, 0.999, 1e-8, None) == E
    assert lib.gs_eval_sh(5, p, 10, 16, p, p, None) == E
    # entry points added for the captured and data-parallel steps
    assert lib.gs_train_step_metrics(None, None, 0.2, None, p, None) == E
    assert lib.gs_train_step_metrics(p, None, 0.2, None, None, None) == E
    assert lib.gs_check_extras(None, None) == E
    assert lib.gs_adam_step_flat_device(p, p, p, p, 10, 1e-3, 0.9, 0.999, 1e-8, None, None) == E
    assert lib.gs_adam_step_flat_device(p, p, p, p, -1, 1e-3, 0.9, 0.999, 1e-8, p, None) == E
    assert lib.gs_adam_step_flat(p, p, p, p, 10, 1e-3, 0, 0.9, 0.999, 1e-8, None) == E  # step >= 1
    ps = _lib.GsPeerSet()
    ps.world, ps.rank = 2, 0
    assert lib.gs_dp_barrier(ctypes.byref(ps), p, p, None) == E  # NULL rendezvous words
    ps.flags[0] = ps.flags[1] = 0x3000
    assert lib.gs_dp_barrier(ctypes.byref(ps), None, p, None) == E  # no epoch counter
    ps.rank = 2
    assert lib.gs_dp_barrier(ctypes.byref(ps), p, p, None) == E  # rank outside the group
    ps.world, ps.rank = 9, 0
    assert lib.gs_dp_barrier(ctypes.byref(ps), p, p, None) == E  # more ranks than GS_MAX_RANKS
    ps.world, ps.rank = 2, 0
    assert lib.gs_dp_publish_barrier(ctypes.byref(ps), p, 100, p, p, None) == E  # no inboxes
    ps.touched_in[0] = ps.touched_in[1] = 0x4000
    assert lib.gs_dp_publish_barrier(ctypes.byref(ps), None, 100, p, p, None) == E  # no flags to publish
    assert lib.gs_dp_publish_barrier(ctypes.byref(ps), p, 0, p, p, None) == E  # no Gaussians
    assert lib.gs_dp_publish_barrier(ctypes.byref(ps), p, 100, p, None, None) == E  # no status word


def test_product_fails_loudly_without_library(tmp_path):
    with pytest.raises(ImportError):
        _lib.load(str(tmp_path / "missing.so"))


def test_mirror_functions_refuse_host_tensors_and_bad_shapes():
    """The torch mirror has no CPU path: host tensors are refused before any
    library call, as are shapes the reference would not accept."""
    import torch
    from gs_b200.core.gaussians import get_covariance_3d
    from gs_b200.training.losses import l1_loss, mse_loss
    s, q = torch.zeros(4, 3), torch.zeros(4, 4)
    with pytest.raises(ValueError, match="CUDA"):
        get_covariance_3d(s, q)
    with pytest.raises(ValueError, match="expected"):
        get_covariance_3d(torch.zeros(4, 2), q)
    with pytest.raises(NotImplementedError):
        get_covariance_3d(s.requires_grad_(True), q)
    for fn in (l1_loss, mse_loss):
        with pytest.raises(ValueError, match="CUDA"):
            fn(torch.zeros(3), torch.zeros(3))
    from gs_b200.core.gaussians import Gaussians
    from gs_b200.core.camera import Camera
    from gs_b200.renderer.renderer import render_views
    g = Gaussians(torch.zeros(4, 3), torch.zeros(4, 3), torch.zeros(4, 4), torch.zeros(4, 1), torch.zeros(4, 16, 3))
    cam = Camera(8, 8, 1.0, 1.0, 4.0, 4.0, torch.eye(4), None)
    with pytest.raises(ValueError, match="w2cs"):
        render_views(g, cam, torch.eye(4))


def test_peer_set_fields_match_the_struct():
    """Every pointer array of GsPeerSet is one PeerSet knows, in the header's
    order (a missing one would reach the library as NULL; touched_in is left
    NULL on purpose when the untouched-row skip is off)."""
    from gs_b200 import _lib
    from gs_b200.training.trainer import PeerSet
    struct_fields = [name for name, _ in _lib.GsPeerSet._fields_ if name not in ("world", "rank")]
    assert list(PeerSet.FIELDS) == struct_fields
    header = open(os.path.join(ROOT, "include", "gsb200.h")).read()
    body = header[header.index("typedef struct GsPeerSet"):header.index("} GsPeerSet;")]
    assert re.findall(r"\*\s*(\w+)\[GS_MAX_RANKS\]", body) == struct_fields
