"""The seeded synthetic scenes that stand in for the reference's benchmark data
(gs_b200/synthetic.py): shapes, value distributions and cameras of the
benchmark configurations, and determinism by seed. CPU only."""
import math

import numpy as np
import pytest

from gs_b200 import synthetic as S


def _centre(w2c):
    R, t = w2c[:3, :3].astype(np.float64), w2c[:3, 3].astype(np.float64)
    return -R.T @ t  # Camera.center = -R^T t (camera.py:14-21)


def _looks_at_origin(w2c):
    c = _centre(w2c)
    fwd = w2c[2, :3].astype(np.float64)  # third row of R: the viewing axis
    return float(np.dot(fwd, -c / np.linalg.norm(c)))


def test_config1_shapes_and_distributions():
    sc = S.config1(0, n=20_000)
    assert sc.means.shape == (20_000, 3) and sc.sh.shape == (20_000, 16, 3) and sc.sh_degree == 0
    assert (sc.W, sc.H, sc.fx, sc.cx, sc.cy) == (504, 378, 400.0, 252.0, 189.0)
    assert np.all(sc.means[:, 2] >= 2) and np.all(sc.means[:, 2] <= 6)
    assert abs(sc.scales.mean() + 4.0) < 0.02 and abs(sc.scales.std() - 0.5) < 0.02
    np.testing.assert_allclose(np.linalg.norm(sc.quats, axis=1), 1.0, rtol=1e-5)
    assert not sc.sh[:, 1:].any()  # degree 0: only the DC term
    dc = sc.sh[:, 0] * S.C0 + 0.5
    assert dc.min() >= -1e-6 and dc.max() <= 1 + 1e-6
    np.testing.assert_array_equal(sc.w2cs[0], np.eye(4, dtype=np.float32))


def test_config2_capacity_padding_and_orbit():
    sc = S.config2(0, n_active=5_000, capacity=10_000)
    assert sc.active.sum() == 5_000 and sc.active[:5_000].all()
    pad = ~sc.active
    # padded slots as init_density_state pads them: zeros, identity rotation
    assert not sc.means[pad].any() and not sc.scales[pad].any() and not sc.opacities[pad].any()
    np.testing.assert_array_equal(sc.quats[pad], np.tile([1, 0, 0, 0], (pad.sum(), 1)).astype(np.float32))
    assert abs(sc.means[~pad].std() - 2.0) < 0.05
    assert abs(sc.opacities[~pad].mean() + 2.0) < 0.05
    assert sc.sh_degree == 3 and sc.sh[~pad, 1:].std() > 0.05
    assert len(sc.w2cs) == 20
    centres = np.array([_centre(w) for w in sc.w2cs])
    np.testing.assert_allclose(np.linalg.norm(centres, axis=1), 4.0, rtol=1e-5)
    az = np.degrees(np.arctan2(centres[:, 2], centres[:, 0]))
    assert abs((az.max() - az.min()) - 30.0) < 1e-3  # a 30 degree arc
    assert min(_looks_at_origin(w) for w in sc.w2cs) > 0.9999


def test_config3_sphere_views():
    sc = S.config3(0, n=20_000)
    assert (sc.W, sc.H, sc.fx, sc.cx, sc.cy) == (1920, 1080, 1200.0, 960.0, 540.0)
    assert len(sc.w2cs) == 64 and sc.active.all()
    assert sc.means.min() >= -5 and sc.means.max() <= 5
    assert abs(sc.scales.mean() + 3.5) < 0.02 and abs(sc.opacities.std() - 1.5) < 0.05
    centres = np.array([_centre(w) for w in sc.w2cs])
    np.testing.assert_allclose(np.linalg.norm(centres, axis=1), 12.0, rtol=1e-5)
    assert centres[:, 1].max() > 10 and centres[:, 1].min() < -10  # pole to pole
    assert min(_looks_at_origin(w) for w in sc.w2cs) > 0.9999


def test_config4_blobs_and_orbit():
    sc = S.config4(0, n=40_000, n_active=30_000, n_views=200)
    assert sc.active.sum() == 30_000 and (sc.W, sc.H) == (1600, 1064)
    assert sc.means.min() >= -10 and sc.means.max() <= 10
    assert len(sc.w2cs) == 200
    centres = np.array([_centre(w) for w in sc.w2cs])
    np.testing.assert_allclose(np.linalg.norm(centres, axis=1), 15.0, rtol=1e-5)
    az = np.sort(np.degrees(np.arctan2(centres[:, 2], centres[:, 0])))
    assert np.diff(az).max() < 2.0  # a full orbit, 1.8 degrees apart


def test_config5_surfels():
    p = S.config5(0, n=20_000)
    assert p["scales"].shape == (20_000, 2) and p["quaternions"].shape == (20_000, 4)
    assert p["means"].min() >= -3 and p["means"].max() <= 3
    assert abs(p["scales"].mean() + 3.5) < 0.02 and abs(p["scales"].std() - 0.5) < 0.02
    assert (p["W"], p["H"]) == (1264, 832) and len(p["w2cs"]) == 20


@pytest.mark.parametrize("gen", [lambda s: S.config1(s, n=2000),
                                 lambda s: S.config2(s, n_active=1000, capacity=2000),
                                 lambda s: S.config3(s, n=2000, n_views=8)])
def test_seeded_and_deterministic(gen):
    a, b, c = gen(3), gen(3), gen(4)
    for f in ("means", "scales", "quats", "opacities", "sh"):
        np.testing.assert_array_equal(getattr(a, f), getattr(b, f))
        assert getattr(a, f).dtype == np.float32
    assert not np.array_equal(a.means, c.means)


def test_target_image_is_uniform_and_seeded():
    t = S.target_image(0, 64, 48)
    assert t.shape == (64, 48, 3) and t.dtype == np.float32
    assert 0 <= t.min() and t.max() <= 1 and abs(t.mean() - 0.5) < 0.02
    np.testing.assert_array_equal(t, S.target_image(0, 64, 48))


def test_look_at_convention():
    w = S.look_at((0.0, 0.0, -5.0))
    R = w[:3, :3].astype(np.float64)
    # orthonormal up to the +1e-6 in the right vector's normalisation
    np.testing.assert_allclose(R @ R.T, np.eye(3), atol=1e-5)
    assert abs(np.linalg.det(R) - 1.0) < 1e-5
    # the origin lies on the optical axis, 5 units ahead
    p = w[:3, :3] @ np.zeros(3) + w[:3, 3]
    np.testing.assert_allclose(p, [0.0, 0.0, 5.0], atol=1e-5)
    assert math.isclose(_looks_at_origin(w), 1.0, rel_tol=1e-6)
