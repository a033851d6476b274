"""render_views: render() over a leading view axis on several streams gives,
view by view, the bits of one-at-a-time render() calls."""
import numpy as np
import pytest
import torch

from tests.helpers import random_scene, to_torch

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("streams", [1, 3])
def test_render_views_equals_per_view_render(streams):
    from gs_b200.core.camera import Camera
    from gs_b200.core.gaussians import Gaussians
    from gs_b200.renderer.renderer import render, render_views
    sc = random_scene(41, 1500, 112, 80, sh_degree=3, behind=0.05, mask_frac=0.1)
    t = to_torch(sc, "cuda")
    g = Gaussians(means=t["means"], scales=t["scales"], quaternions=t["quats"], opacities=t["opac"],
                  sh_coeffs=t["sh"])
    w2cs = []
    for i in range(5):
        w = t["w2c"].clone()
        w[0, 3] += 0.04 * i
        w[1, 3] -= 0.03 * i
        w2cs.append(w)
    cam = Camera(sc["W"], sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"], w2cs[0], None)
    bg = torch.tensor([0.1, 0.2, 0.3], device="cuda")
    with torch.no_grad():
        imgs, ex = render_views(g, cam, torch.stack(w2cs), background=bg, mask=t["active"], sh_degree=3,
                                streams=streams)
        torch.cuda.synchronize()
        assert imgs.shape == (5, sc["H"], sc["W"], 3)
        for i, w in enumerate(w2cs):
            img_i, ex_i = render(g, cam._replace(W2C=w), background=bg, mask=t["active"], sh_degree=3)
            np.testing.assert_array_equal(_np(imgs[i]), _np(img_i))
            np.testing.assert_array_equal(_np(ex["radii"][i]), _np(ex_i["radii"]))
            np.testing.assert_array_equal(_np(ex["valid_mask"][i]), _np(ex_i["valid_mask"]))
            for k in ("n_interactions", "max_interactions_per_tile", "radius_cap_violations"):
                assert int(ex[k][i]) == int(ex_i[k]), k
            assert float(ex["mean_interactions_per_tile"][i]) == float(ex_i["mean_interactions_per_tile"])
    assert int(ex["n_interactions"].min()) > 0
