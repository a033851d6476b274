"""Generate the golden fixtures under tests/golden/ from the CPU oracle.

JAX is not installed in this environment, so the reference cannot produce
fixtures itself; these pin the oracle (which the reference's own
known-answer tests pin in tests/test_oracle.py and tests/test_oracle_2d.py)
against drift, and give the GPU tests a fixed case.

  python tests/golden/make_golden.py [3d|2d|all]   (default all)

scene_small.npz: a 400-Gaussian SH-3 scene at 80x64 (3DGS render, its sorted
pairs, ranges, radii and the gradients of a weighted image sum).
scene_small_2d.npz: a 600-surfel 2DGS scene at 72x56 (image, depth, depth^2,
normal and accumulated-weight maps, and the gradients of a weighted sum of
all five).
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [ROOT, os.path.join(ROOT, "jax-gs_b200")]

from tests.helpers import oracle_render, random_scene  # noqa: E402


def main_3d():
    sc = random_scene(11, 400, 80, 64, sh_degree=3, behind=0.1, mask_frac=0.1)
    img, ex, t = oracle_render(sc, requires_grad=True)
    wimg = np.random.default_rng(5).standard_normal(img.shape).astype(np.float32)
    import torch
    (img * torch.tensor(wimg)).sum().backward()
    out = {}
    for k in ("means", "scales", "quats", "opac", "sh", "w2c", "active"):
        out["in_" + k] = np.asarray(sc[k])
    for k in ("W", "H", "sh_degree", "fx", "fy", "cx", "cy"):
        out["cfg_" + k] = np.asarray(sc[k])
    out["out_tiles"] = ex["sorted_tile_ids"]
    out["out_gids"] = ex["sorted_gaussian_ids"]
    out["out_ranges"] = ex["tile_ranges"]
    out["out_radii"] = ex["radii"].detach().numpy()
    out["out_image"] = img.detach().numpy()
    out["grad_weights"] = wimg
    for k in ("means", "scales", "quats", "opac", "sh"):
        out["grad_" + k] = t[k].grad.numpy()
    np.savez_compressed(os.path.join(os.path.dirname(__file__), "scene_small.npz"), **out)


def scene_2d(seed=21, n=600, W=72, H=56):
    """Seeded 2DGS scene: surfels in front of a slightly rotated camera, 5 %
    of them behind it or at the near plane."""
    rng = np.random.default_rng(seed)
    means = np.stack([rng.uniform(-1.2, 1.2, n), rng.uniform(-0.96, 0.96, n), rng.uniform(2.0, 6.0, n)], 1)
    means[: n // 20, 2] = rng.uniform(-2, 0.005, n // 20)
    p = {"means": means, "scales": rng.normal(-2.6, 0.4, (n, 2)), "quaternions": rng.normal(0, 1, (n, 4)),
         "opacities": rng.normal(0, 1.2, (n, 1)), "sh_coeffs": rng.normal(0, 0.5, (n, 16, 3))}
    p = {k: v.astype(np.float32) for k, v in p.items()}
    a, b = 0.12, -0.08
    Ry = np.array([[np.cos(a), 0, np.sin(a)], [0, 1, 0], [-np.sin(a), 0, np.cos(a)]])
    Rx = np.array([[1, 0, 0], [0, np.cos(b), -np.sin(b)], [0, np.sin(b), np.cos(b)]])
    w2c = np.eye(4, dtype=np.float32)
    w2c[:3, :3] = Rx @ Ry
    w2c[:3, 3] = [0.05, -0.02, 0.2]
    cam = dict(W=W, H=H, fx=0.9 * W, fy=0.92 * W, cx=W / 2 + 0.3, cy=H / 2 - 0.2)
    return p, w2c, cam


MAPS_2D = ("depth", "depth_sq", "normals", "accum_weight")


def render_2d_golden(p, w2c, cam, weights=None):
    """Oracle 2DGS render of the scene; with weights (image first, then
    MAPS_2D), also the gradients of the weighted sum of the five maps."""
    import torch
    from oracle import ref_restated_2d as R2
    t = {k: torch.tensor(v, requires_grad=weights is not None) for k, v in p.items()}
    img, ex = R2.render_2d(t["means"], t["scales"], t["quaternions"], t["opacities"], t["sh_coeffs"],
                           torch.tensor(w2c), cam["W"], cam["H"], cam["fx"], cam["fy"], cam["cx"], cam["cy"])
    if weights is not None:
        tot = (img * torch.tensor(weights[0])).sum()
        for k, w in zip(MAPS_2D, weights[1:]):
            tot = tot + (ex[k] * torch.tensor(w)).sum()
        tot.backward()
    return img, ex, t


def main_2d():
    p, w2c, cam = scene_2d()
    rng = np.random.default_rng(7)
    H, W = cam["H"], cam["W"]
    weights = [rng.standard_normal(s).astype(np.float32) for s in ((H, W, 3), (H, W, 1), (H, W, 1), (H, W, 3),
                                                                     (H, W, 1))]
    img, ex, t = render_2d_golden(p, w2c, cam, weights)
    out = {"in_" + k: v for k, v in p.items()}
    out["in_w2c"] = w2c
    for k, v in cam.items():
        out["cfg_" + k] = np.asarray(v)
    out["out_image"] = img.detach().numpy()
    for k in MAPS_2D:
        out["out_" + k] = ex[k].detach().numpy()
    for i, w in enumerate(weights):
        out["grad_weights_%d" % i] = w
    for k in p:
        out["grad_" + k] = t[k].grad.numpy()
    np.savez_compressed(os.path.join(os.path.dirname(__file__), "scene_small_2d.npz"), **out)


if __name__ == "__main__":
    which = sys.argv[1] if len(sys.argv) > 1 else "all"
    if which in ("3d", "all"):
        main_3d()
    if which in ("2d", "all"):
        main_2d()
