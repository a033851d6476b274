"""The direct-path sort's bounded look-back wait, made to run out on purpose
(gs_test_set_sort_wait: every earlier key tile reads as unpublished, so each
wait gives up after a few polls -- a flag that nothing sets, no GPU stall).
The give-up must be reported (GsExtras.device_timeouts, gs_check_extras,
check_extras, the train step's metrics), the outputs must stay defined (every
tile range emptied: background image, zero gradients) and the library must
work normally once the setting is restored."""
import ctypes

import numpy as np
import pytest
import torch

from gs_b200 import _lib
from tests.helpers import oracle_render, random_scene, to_torch

pytestmark = pytest.mark.gpu


@pytest.fixture
def blind_sort():
    lib = _lib.lib()
    lib.gs_test_set_sort_wait(4, 1)
    try:
        yield
    finally:
        lib.gs_test_set_sort_wait(0, 0)


def _gaussians(sc, dev, grad=False):
    from gs_b200.core.gaussians import Gaussians
    t = to_torch(sc, dev)
    if grad:
        for key in ("means", "scales", "quats", "opac", "sh"):
            t[key].requires_grad_(True)
    g = Gaussians(means=t["means"], scales=t["scales"], quaternions=t["quats"], opacities=t["opac"],
                  sh_coeffs=t["sh"])
    return g, t


def _camera(sc, dev):
    from gs_b200.core.camera import Camera
    return Camera(sc["W"], sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"],
                  torch.as_tensor(sc["w2c"], device=dev), torch.eye(4, device=dev))


def test_sort_wait_give_up_is_reported_and_safe(blind_sort):
    from gs_b200.renderer.renderer import check_extras, render
    dev = torch.device("cuda", 0)
    sc = random_scene(7, 6000, 160, 120, sh_degree=3)  # 6000 < 2^18: the direct (waiting) path
    g, t = _gaussians(sc, dev, grad=True)
    bg = torch.tensor([0.25, 0.5, 0.75], device=dev)
    img, ex = render(g, _camera(sc, dev), background=bg, mask=t["active"], sh_degree=3)
    (img * torch.randn_like(img)).sum().backward()
    torch.cuda.synchronize(dev)
    assert int(ex["device_timeouts"]) > 0
    assert int(ex["n_interactions"]) > 2 * 2048  # several key tiles, so later tiles waited
    # every range emptied: the image is the background, no splat gets a gradient
    assert torch.equal(img.detach(), bg.expand_as(img))
    for key in ("means", "scales", "quats", "opac", "sh"):
        assert torch.count_nonzero(t[key].grad) == 0, key
    with pytest.raises(_lib.GsError) as e:
        check_extras(ex)
    assert e.value.status == _lib.GS_ERR_DEVICE_TIMEOUT
    # the same status through the C ABI, on the GsExtras block of a fresh render
    from gs_b200.renderer.renderer import _forward
    cam = (sc["W"], sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"])
    d = {key: v.detach() for key, v in t.items()}
    _, _, _, _, blk = _forward("gs_render_image", d["means"], d["scales"], d["quats"], d["opac"], d["sh"],
                               d["w2c"], None, d["active"].to(torch.uint8), cam, 3, 6000 * 256)
    assert _lib.lib().gs_check_extras(_lib.ptr(blk), _lib.stream(dev)) == _lib.GS_ERR_DEVICE_TIMEOUT


def test_sort_wait_restored_gives_the_oracle_image():
    from gs_b200.renderer.renderer import check_extras, render
    lib = _lib.lib()
    lib.gs_test_set_sort_wait(4, 1)
    lib.gs_test_set_sort_wait(0, 0)  # back to the default bound
    dev = torch.device("cuda", 0)
    sc = random_scene(7, 6000, 160, 120, sh_degree=3)
    g, t = _gaussians(sc, dev)
    with torch.no_grad():
        img, ex = render(g, _camera(sc, dev), mask=t["active"], sh_degree=3)
    torch.cuda.synchronize(dev)
    assert int(ex["device_timeouts"]) == 0
    check_extras(ex)
    oimg, _, _ = oracle_render(sc)
    assert float((img.cpu() - oimg).abs().max()) <= 1e-4


def test_train_step_reports_a_sort_give_up(blind_sort):
    from gs_b200.core.gaussians import Gaussians
    from gs_b200.training.trainer import AdamConfig, check_step, init_density_state, train_step
    dev = torch.device("cuda", 0)
    sc = random_scene(8, 6000, 160, 120, sh_degree=3)
    t = to_torch(sc, dev)
    g = Gaussians(means=t["means"], scales=t["scales"], quaternions=t["quats"], opacities=t["opac"],
                  sh_coeffs=t["sh"])
    state = init_density_state(g, AdamConfig(), 6000)
    tgt = torch.rand((sc["H"], sc["W"], 3), device=dev)
    cam = (sc["W"], sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"])
    _, loss, metrics = train_step(state, tgt, t["w2c"], cam, AdamConfig(), sh_degree=3)
    torch.cuda.synchronize(dev)
    assert float(metrics["device_timeouts"]) > 0
    with pytest.raises(_lib.GsError) as e:
        check_step(metrics)
    assert e.value.status == _lib.GS_ERR_DEVICE_TIMEOUT
    assert np.isfinite(float(loss))
