"""Generate tests/golden/scene_small.npz from the CPU oracle.

JAX is not installed in this environment, so the reference cannot produce
fixtures itself; these pin the oracle (which the reference's own
known-answer tests pin in tests/test_oracle.py) against drift, and give the
GPU tests a fixed case. Run: python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [ROOT, os.path.join(ROOT, "jax-gs_b200")]

from tests.helpers import oracle_render, random_scene  # noqa: E402


def main():
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


if __name__ == "__main__":
    main()
