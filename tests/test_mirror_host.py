"""Host-side parts of the torch mirror that run without a GPU, against the
reference's own tests: tests/test_core.py:7-19 (init_gaussians_from_pcd) and
:40-52 (Camera), plus Camera.center (camera.py:14-21)."""
import numpy as np
import torch

from gs_b200.core.camera import Camera, camera_static
from gs_b200.core.gaussians import Gaussians, init_gaussians_from_pcd


def test_gaussians_initialization():
    rng = np.random.default_rng(0)
    points = torch.tensor(rng.uniform(-1, 1, (100, 3)), dtype=torch.float32)
    colors = torch.tensor(rng.uniform(0, 1, (100, 3)), dtype=torch.float32)
    g = init_gaussians_from_pcd(points, colors)
    assert isinstance(g, Gaussians)
    assert g.means.shape == (100, 3) and g.scales.shape == (100, 3)
    assert g.quaternions.shape == (100, 4) and g.opacities.shape == (100, 1)
    assert g.sh_coeffs.shape == (100, 16, 3)
    # gaussians.py:13-56: log-scale -3, identity rotation, logit 0, DC colour
    assert (g.scales == -3.0).all() and (g.opacities == 0.0).all()
    np.testing.assert_array_equal(g.quaternions.numpy(), np.tile([1, 0, 0, 0], (100, 1)))
    np.testing.assert_allclose(g.sh_coeffs[:, 0].numpy() * 0.28209479177387814 + 0.5, colors.numpy(), atol=1e-6)
    assert not g.sh_coeffs[:, 1:].any()


def test_black_point_cloud_gets_random_colours():
    # gaussians.py: colours that are all ~0 are replaced by uniform [0.1, 0.9]
    g = init_gaussians_from_pcd(torch.zeros((50, 3)), torch.zeros((50, 3)))
    dc = g.sh_coeffs[:, 0].numpy() * 0.28209479177387814 + 0.5
    assert dc.min() >= 0.1 - 1e-6 and dc.max() <= 0.9 + 1e-6 and dc.std() > 0.1


def test_camera_entity():
    cam = Camera(W=640, H=480, fx=500.0, fy=500.0, cx=320.0, cy=240.0, W2C=torch.eye(4), full_proj=torch.eye(4))
    assert cam.W == 640 and cam.H == 480 and cam.fx == 500.0
    assert cam.W2C.shape == (4, 4)
    assert camera_static(cam) == (640, 480, 500.0, 500.0, 320.0, 240.0)


def test_camera_center():
    w2c = torch.eye(4)
    c, s = np.cos(0.3), np.sin(0.3)
    w2c[:3, :3] = torch.tensor([[c, 0, s], [0, 1, 0], [-s, 0, c]], dtype=torch.float32)
    w2c[:3, 3] = torch.tensor([1.0, 2.0, 3.0])
    cam = Camera(W=8, H=8, fx=1.0, fy=1.0, cx=4.0, cy=4.0, W2C=w2c, full_proj=torch.eye(4))
    centre = cam.center
    # the centre maps to the camera origin
    np.testing.assert_allclose((w2c[:3, :3] @ centre + w2c[:3, 3]).numpy(), 0.0, atol=1e-6)
