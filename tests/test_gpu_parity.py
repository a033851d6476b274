"""GPU parity of the CUDA renderer against the CPU oracle, through the C ABI.

Bars: tile keys, sort order and per-tile ranges
bit-exact; images within 1e-4 max abs (fp32); per-Gaussian gradients within
1e-3 relative (measured against the array's largest oracle gradient, see
_grad_close), compared on active Gaussians.
"""

import numpy as np
import pytest
import torch

from oracle import ref_restated as R
from tests.helpers import oracle_render, random_scene, scene_from_synthetic, to_torch

pytestmark = pytest.mark.gpu

IMG_TOL = 1e-4
GRAD_RTOL = 1e-3


def gpu_gaussians(sc):
    from gs_b200.core.gaussians import Gaussians
    t = to_torch(sc, "cuda")
    g = Gaussians(means=t["means"], scales=t["scales"], quaternions=t["quats"], opacities=t["opac"],
                  sh_coeffs=t["sh"])
    return g, t


def gpu_camera(sc, device="cuda"):
    from gs_b200.core.camera import Camera
    return Camera(W=sc["W"], H=sc["H"], fx=sc["fx"], fy=sc["fy"], cx=sc["cx"], cy=sc["cy"],
                  W2C=torch.as_tensor(sc["w2c"], device=device), full_proj=torch.eye(4, device=device))


def gpu_render(sc, requires_grad=False, capacity=None, background=None):
    from gs_b200.renderer.renderer import render
    g, t = gpu_gaussians(sc)
    if requires_grad:
        for f in ("means", "scales", "quaternions", "opacities", "sh_coeffs"):
            getattr(g, f).requires_grad_(True)
    img, ex = render(g, gpu_camera(sc), background=background, mask=t["active"],
                     sh_degree=sc["sh_degree"], capacity=capacity)
    return img, ex, g


def _dense_faint():
    """1500 large, faint splats over a 48x32 image: every tile holds ~1000
    pairs and no pixel saturates, so every tile runs 4-5 full 256-splat
    batches on all four warps (long checkpoint chains, costly items first in
    the backward's order)."""
    sc = random_scene(5, 1500, 48, 32, sh_degree=3, scale_mu=-1.5, scale_sd=0.3, behind=0.0)
    sc["opac"][:] = -4.5
    return sc


SCENES = [
    ("dense_faint", _dense_faint),
    ("rot_sh3", lambda: random_scene(1, 600, 96, 80, sh_degree=3, behind=0.15, mask_frac=0.2)),
    ("rot_sh1", lambda: random_scene(2, 500, 83, 61, sh_degree=1, behind=0.1, mask_frac=0.0)),
    ("id_sh0", lambda: random_scene(3, 800, 128, 96, sh_degree=0, rotate=False, behind=0.0)),
    ("big_splats", lambda: random_scene(4, 150, 200, 150, sh_degree=2, scale_mu=-0.8, scale_sd=0.5)),
    ("config1_small", lambda: scene_from_synthetic(__import__("gs_b200.synthetic").synthetic.config1(0, 2000, 160, 120))),
]


def _np(t):
    return t.detach().cpu().numpy()


# ---------------------------------------------------------------- stage 1
@pytest.mark.parametrize("name,make", SCENES)
def test_projection_bit_exact(name, make):
    from gs_b200.renderer.projection import project_gaussians
    sc = make()
    g, t = gpu_gaussians(sc)
    m2, cov, radii, valid, z = project_gaussians(g, gpu_camera(sc), mask=t["active"])
    tc = to_torch(sc)
    rm2, rcov, rradii, rvalid, rz = R.project_gaussians(tc["means"], tc["scales"], tc["quats"], tc["w2c"],
                                                        sc["W"], sc["H"], sc["fx"], sc["fy"], sc["cx"],
                                                        sc["cy"], tc["active"])
    np.testing.assert_array_equal(_np(z), _np(rz))
    np.testing.assert_array_equal(_np(valid), _np(rvalid))
    np.testing.assert_array_equal(_np(m2), _np(rm2))
    np.testing.assert_array_equal(_np(cov), _np(rcov))
    np.testing.assert_array_equal(_np(radii), _np(rradii))


def test_projection_known_answer_gpu():
    # tests/test_renderer.py:11-33 through the CUDA path
    from gs_b200.core.gaussians import init_gaussians_from_pcd
    from gs_b200.renderer.projection import project_gaussians
    g = init_gaussians_from_pcd(torch.tensor([[0.0, 0.0, 5.0]], device="cuda"),
                                torch.tensor([[1.0, 1.0, 1.0]], device="cuda"))
    sc = dict(W=100, H=100, fx=50.0, fy=50.0, cx=50.0, cy=50.0, w2c=np.eye(4, dtype=np.float32))
    m2, cov, radii, valid, z = project_gaussians(g, gpu_camera(sc))
    assert torch.allclose(m2[0].cpu(), torch.tensor([50.0, 50.0]))
    assert bool(valid[0]) and float(z[0]) == 5.0 and float(radii[0]) > 0


# ---------------------------------------------------------------- stage 2
@pytest.mark.parametrize("name,make", SCENES)
def test_tile_interactions_bit_exact(name, make):
    """Stage 2 fed the oracle's own projection: keys, order, ranges exact."""
    from gs_b200.renderer.rasterizer import get_tile_interactions
    sc = make()
    tc = to_torch(sc)
    m2, _, radii, valid, z = R.project_gaussians(tc["means"], tc["scales"], tc["quats"], tc["w2c"], sc["W"],
                                                 sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"],
                                                 tc["active"])
    ref_t, ref_g, ref_n = R.get_tile_interactions_compact(_np(m2), _np(radii), _np(valid), _np(z),
                                                          sc["H"], sc["W"])
    T = ((sc["W"] + 15) // 16) * ((sc["H"] + 15) // 16)
    tiles, gids, n, ranges = get_tile_interactions(m2.cuda(), radii.cuda(), valid.cuda(), z.cuda(), sc["H"],
                                                   sc["W"], return_ranges=True)
    n = int(n)
    assert n == ref_n
    np.testing.assert_array_equal(_np(tiles)[:n], ref_t)
    np.testing.assert_array_equal(_np(gids)[:n], ref_g)
    assert (_np(tiles)[n:] == T).all() and (_np(gids)[n:] == 0).all()
    assert tiles.numel() == max(sc["means"].shape[0] * 256, 512)
    np.testing.assert_array_equal(_np(ranges), R.tile_ranges(ref_t, T))
    # literal N*256 layout: the valid segment is the same sequence
    full_t, full_g, full_n = R.get_tile_interactions(_np(m2), _np(radii), _np(valid), _np(z), sc["H"], sc["W"])
    seg = (full_t >= 0) & (full_t < T)
    lo = int(np.argmax(seg)) if seg.any() else 0
    np.testing.assert_array_equal(full_g[lo:lo + n], _np(gids)[:n])


def _padded(small, n_big, seed):
    """small's Gaussians at sorted random rows of an n_big array whose other
    rows are random but inactive."""
    rng = np.random.default_rng(seed)
    n = small["means"].shape[0]
    idx = np.sort(rng.choice(n_big, n, replace=False))
    filler = random_scene(seed + 1, n_big, small["W"], small["H"], sh_degree=small["sh_degree"])
    big = dict(small)
    for k in ("means", "scales", "quats", "opac", "sh"):
        a = filler[k].copy()
        a[idx] = small[k]
        big[k] = a
    big["active"] = np.zeros(n_big, bool)
    big["active"][idx] = small["active"]
    return big, idx


def test_presort_path_matches_direct_path():
    """From 2^19 Gaussians the pairs are sorted after a depth pre-sort of the
    Gaussians. The same visible Gaussians padded with inactive ones must give
    the direct path's pairs (ids mapped), ranges and a bit-identical image."""
    from gs_b200.renderer.rasterizer import get_tile_interactions
    small = random_scene(11, 3000, 200, 150, sh_degree=1, mask_frac=0.1)
    big, idx = _padded(small, 600_000, 12)
    out = []
    for sc in (small, big):
        g, t = gpu_gaussians(sc)
        from gs_b200.renderer.projection import project_gaussians
        m2, _, radii, valid, z = project_gaussians(g, gpu_camera(sc), mask=t["active"])
        out.append(get_tile_interactions(m2, radii, valid, z, sc["H"], sc["W"], return_ranges=True))
    (ts, gs_, ns, rs), (tb, gb, nb, rb) = out
    ns, nb = int(ns), int(nb)
    assert ns == nb > 0
    np.testing.assert_array_equal(_np(ts)[:ns], _np(tb)[:nb])
    np.testing.assert_array_equal(idx[_np(gs_)[:ns]], _np(gb)[:nb])
    np.testing.assert_array_equal(_np(rs), _np(rb))
    img_s, ex_s, g_s = gpu_render(small, requires_grad=True)
    img_b, ex_b, g_b = gpu_render(big, requires_grad=True)
    np.testing.assert_array_equal(_np(img_s), _np(img_b))
    for k in EXTRA_KEYS:
        assert int(ex_s[k]) == int(ex_b[k]), k
    w = torch.rand_like(img_s)
    (img_s * w).sum().backward()
    (img_b * w).sum().backward()
    # same pairs in the same order: the gradients differ only by the order in
    # which float atomics add them up (ill-conditioned for near-zero
    # quaternions, whose gradient scales as 1/|q|)
    for f in ("means", "scales", "quaternions", "opacities", "sh_coeffs"):
        a = _np(getattr(g_s, f).grad).astype(np.float64)
        b = _np(getattr(g_b, f).grad)[idx].astype(np.float64)
        assert np.all(np.abs(a - b) <= 1e-3 * np.abs(a) + 3e-3 * np.abs(a).max()), f


def test_tile_interactions_reference_case():
    # tests/test_renderer.py:35-51 (integer radii input)
    from gs_b200.renderer.rasterizer import get_tile_interactions
    m2 = torch.tensor([[16.0, 16.0], [0.0, 0.0]], device="cuda")
    radii = torch.tensor([4, 2], dtype=torch.int32, device="cuda")
    valid = torch.tensor([True, True], device="cuda")
    depths = torch.tensor([5.0, 10.0], device="cuda")
    tiles, gids, n = get_tile_interactions(m2, radii, valid, depths, 32, 32, 16)
    rt, rg, rn = R.get_tile_interactions_compact(_np(m2), _np(radii).astype(np.float32), _np(valid),
                                                 _np(depths), 32, 32)
    assert int(n) == rn > 0
    np.testing.assert_array_equal(_np(tiles)[:rn], rt)
    np.testing.assert_array_equal(_np(gids)[:rn], rg)


# ---------------------------------------------------------------- stage 3
def _analytic():
    from tests.test_oracle import analytic_case
    return analytic_case()


@pytest.mark.parametrize("fn", ["render_tiles", "render_tiles_tpu"])
def test_chunked_rasterization_matches_reference_gpu(fn):
    # tests/test_renderer.py:115-158 through the CUDA compositor
    from gs_b200.renderer import rasterizer, rasterizer_tpu
    means2D, cov2D, opac, colors, tiles, gids, ref = _analytic()
    c = lambda a: torch.as_tensor(a, device="cuda")  # noqa: E731
    if fn == "render_tiles":
        img = rasterizer.render_tiles(c(means2D), c(cov2D), c(opac), c(colors), c(tiles), c(gids), 16, 16, 16,
                                      torch.zeros(3, device="cuda"))
    else:
        img = rasterizer_tpu.render_tiles_tpu(c(means2D), c(cov2D), c(opac), c(colors), c(tiles), c(gids), 16,
                                              16, torch.zeros(3, device="cuda"))
    np.testing.assert_allclose(_np(img[8, 8]), ref, atol=1e-4, rtol=1e-4)
    oimg = R.render_tiles(torch.tensor(means2D), torch.tensor(cov2D), torch.tensor(opac),
                          torch.tensor(colors), tiles, gids, 16, 16, torch.zeros(3))
    assert np.abs(_np(img) - _np(oimg)).max() <= IMG_TOL


def test_rasterization_red_centre_gpu():
    # tests/test_renderer.py:53-76
    from gs_b200.renderer.rasterizer import render_tiles
    c = lambda a, dt=torch.float32: torch.tensor(a, dtype=dt, device="cuda")  # noqa: E731
    img = render_tiles(c([[16.0, 16.0]]), c([[[10.0, 0.0], [0.0, 10.0]]]), c([[10.0]]), c([[1.0, 0.0, 0.0]]),
                       c([0, 1, 2, 3], torch.int32), c([0, 0, 0, 0], torch.int32), 32, 32, 16, c([0.0, 0, 0]))
    assert img.shape == (32, 32, 3)
    assert float(img[16, 16, 0]) > 0.5 and float(img[16, 16, 1]) < 0.1


def test_full_render_red_centre_gpu():
    # tests/test_renderer.py:78-113
    from gs_b200.core.gaussians import init_gaussians_from_pcd
    from gs_b200.renderer.renderer import render
    g = init_gaussians_from_pcd(torch.tensor([[0.0, 0.0, 5.0]], device="cuda"),
                                torch.tensor([[1.0, 0.0, 0.0]], device="cuda"))
    g = g.replace(opacities=torch.tensor([[10.0]], device="cuda"),
                  scales=torch.tensor([[-1.0, -1.0, -1.0]], device="cuda"))
    sc = dict(W=64, H=64, fx=100.0, fy=100.0, cx=32.0, cy=32.0, w2c=np.eye(4, dtype=np.float32))
    img, extras = render(g, gpu_camera(sc))
    u8 = (_np(img) * 255).astype(np.uint8)
    assert u8.shape == (64, 64, 3) and u8[32, 32, 0] > 200 and u8[32, 32, 1] < 50


EXTRA_KEYS = ("n_interactions", "max_interactions_per_tile", "overflow_tiles", "overflow_interactions",
              "truncated_tiles", "truncated_interactions", "radius_cap_violations")


@pytest.mark.parametrize("name,make", SCENES)
def test_render_matches_oracle(name, make):
    sc = make()
    img, ex, _ = gpu_render(sc)
    oimg, oex, _ = oracle_render(sc)
    assert np.abs(_np(img) - _np(oimg)).max() <= IMG_TOL
    for k in EXTRA_KEYS:
        assert int(ex[k]) == oex[k], k
    assert float(ex["mean_interactions_per_tile"]) == pytest.approx(oex["mean_interactions_per_tile"], rel=1e-6)
    np.testing.assert_array_equal(_np(ex["radii"]), _np(oex["radii"]))
    np.testing.assert_array_equal(_np(ex["valid_mask"]), _np(oex["valid_mask"]))
    assert int(ex["capacity_overflow"]) == 0


@pytest.mark.parametrize("name,make", SCENES)
def test_render_image_equals_render_forward(name, make):
    """gs_render_image (no backward residuals; render() without gradients)
    and gs_render_forward (render() with gradients) give the same bits."""
    sc = make()
    img_f, ex_f, _ = gpu_render(sc, requires_grad=True)
    img_i, ex_i, _ = gpu_render(sc)
    np.testing.assert_array_equal(_np(img_f), _np(img_i))
    for k in tuple(EXTRA_KEYS) + ("capacity_overflow",):
        assert int(ex_f[k]) == int(ex_i[k]), k
    np.testing.assert_array_equal(_np(ex_f["radii"]), _np(ex_i["radii"]))


def test_render_background():
    sc = random_scene(5, 300, 70, 50, sh_degree=2)
    bg = [0.2, 0.5, 0.9]
    img, _, _ = gpu_render(sc, background=torch.tensor(bg, device="cuda"))
    from oracle import ref_restated as R_
    t = to_torch(sc)
    oimg, _ = R_.render(t["means"], t["scales"], t["quats"], t["opac"], t["sh"], t["w2c"], sc["W"], sc["H"],
                        sc["fx"], sc["fy"], sc["cx"], sc["cy"], background=torch.tensor(bg),
                        mask=t["active"], sh_degree=sc["sh_degree"])
    assert np.abs(_np(img) - _np(oimg)).max() <= IMG_TOL


# ---------------------------------------------------------------- stage 4
def _grad_close(g, r, name):
    """|g - r| <= 1e-3 * (|r| + max|r|): relative to the gradient itself and
    to the array's scale, since atomics reorder fp32 sums."""
    g, r = np.asarray(g, np.float64), np.asarray(r, np.float64)
    scale = np.abs(r).max() if r.size else 0.0
    err = np.abs(g - r)
    bound = GRAD_RTOL * (np.abs(r) + scale) + 1e-12
    bad = err > bound
    assert not bad.any(), (f"{name}: {bad.sum()} of {bad.size} over tolerance; "
                           f"max err {err.max():.3e} scale {scale:.3e}")


@pytest.mark.parametrize("name,make", SCENES)
def test_render_backward_matches_oracle(name, make):
    sc = make()
    rng = np.random.default_rng(17)
    w = rng.standard_normal((sc["H"], sc["W"], 3)).astype(np.float32)
    img, ex, g = gpu_render(sc, requires_grad=True)
    (img * torch.tensor(w, device="cuda")).sum().backward()
    oimg, oex, t = oracle_render(sc, requires_grad=True)
    (oimg * torch.tensor(w)).sum().backward()
    act = sc["active"]
    pairs = [("means", "means"), ("scales", "scales"), ("quaternions", "quats"), ("opacities", "opac"),
             ("sh_coeffs", "sh")]
    for gname, oname in pairs:
        gg = _np(getattr(g, gname).grad)[act]
        rr = _np(t[oname].grad)[act]
        rr = np.nan_to_num(rr)
        _grad_close(gg, rr, gname)
    # Gaussians without an interaction get exact zeros
    inactive = ~act
    if inactive.any():
        assert (_np(g.means.grad)[inactive] == 0).all()


@pytest.mark.parametrize("name,make", [s for s in SCENES if s[0] in ("rot_sh3", "big_splats", "config1_small")])
def test_render_backward_touched_flags(name, make):
    """gs_render_backward's optional touched output, which gs_dp_update reads
    to skip a rank's gradient rows over NVLink: 0 only where the Gaussian's
    whole gradient row is exact +0 (sign bit clear), and 1 on rows that hold
    nonzeros; the gradients are the same as without the output."""
    from gs_b200 import _lib
    from gs_b200.renderer.renderer import _f32, _forward, _u8
    sc = make()
    g, t = gpu_gaussians(sc)
    n, k = int(g.means.shape[0]), int(g.sh_coeffs.shape[1])
    cam = (int(sc["W"]), int(sc["H"]), float(sc["fx"]), float(sc["fy"]), float(sc["cx"]), float(sc["cy"]))
    w2c = _f32(torch.as_tensor(sc["w2c"]), "cuda")
    mask = _u8(t["active"], "cuda")
    cap = int(_lib.lib().gs_default_capacity(n))
    fields = [g.means, g.scales, g.quaternions, g.opacities, g.sh_coeffs]
    ws, img, radii, valid, ex = _forward("gs_render_forward", *fields, w2c, None, mask, cam, sc["sh_degree"], cap)
    rng = np.random.default_rng(3)
    gimg = torch.tensor(rng.standard_normal(tuple(img.shape)).astype(np.float32), device="cuda")
    P = _lib.ptr
    outs = []
    for with_touched in (False, True):
        grads = [torch.full_like(f, float("nan")) for f in fields]
        touched = torch.full((n,), 7, dtype=torch.uint8, device="cuda") if with_touched else None
        _lib.call("gs_render_backward", *[P(f) for f in fields], n, k, P(mask), P(w2c), *cam, None,
                  int(sc["sh_degree"]), cap, P(ws), ws.numel(), P(gimg), *[P(x) for x in grads], None,
                  P(touched), _lib.stream(torch.device("cuda")))
        outs.append((grads, touched))
    torch.cuda.synchronize()
    # the output changes no gradient (the compositor's atomic sums may differ
    # in the last bits between calls, exact zeros may not)
    for a, b in zip(outs[0][0], outs[1][0]):
        assert torch.equal(a == 0, b == 0)
        assert ((a - b).abs() <= GRAD_RTOL * (b.abs() + b.abs().max())).all()
    grads, touched = outs[1]
    rows = torch.cat([x.reshape(n, -1) for x in grads], dim=1)          # (n, 59) for SH 3
    bits = rows.view(torch.int32)
    assert set(touched.unique().tolist()) <= {0, 1}
    untouched = touched == 0
    assert (~untouched).any()
    if (mask == 0).any():
        assert untouched.any()
    assert (bits[untouched] == 0).all()                                # exact +0, every element
    # the converse is what makes the skip pay: touched rows hold nonzeros
    assert float((rows[~untouched] != 0).any(dim=1).float().mean()) >= 0.99
    assert not (touched.bool() & (mask == 0)).any()                    # inactive Gaussians are never touched


def test_render_tiles_backward_matches_oracle():
    sc = random_scene(8, 400, 90, 70, sh_degree=3, behind=0.1)
    tc = to_torch(sc)
    m2, cov, radii, valid, z = R.project_gaussians(tc["means"], tc["scales"], tc["quats"], tc["w2c"], sc["W"],
                                                   sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"])
    tiles, gids, _ = R.get_tile_interactions_compact(_np(m2), _np(radii), _np(valid), _np(z), sc["H"], sc["W"])
    rng = np.random.default_rng(3)
    colors = torch.tensor(rng.uniform(0, 1, (400, 3)), dtype=torch.float32)
    w = torch.tensor(rng.standard_normal((sc["H"], sc["W"], 3)), dtype=torch.float32)
    ins = [m2.detach().clone(), cov.detach().clone(), tc["opac"].clone(), colors]
    for a in ins:
        a.requires_grad_(True)
    oimg = R.render_tiles(*ins, tiles, gids, sc["H"], sc["W"], torch.zeros(3))
    (oimg * w).sum().backward()
    from gs_b200.renderer.rasterizer import render_tiles
    gins = [a.detach().cuda().requires_grad_(True) for a in ins]
    img = render_tiles(*gins, torch.as_tensor(tiles, device="cuda"), torch.as_tensor(gids, device="cuda"),
                       sc["H"], sc["W"], 16, torch.zeros(3, device="cuda"))
    assert np.abs(_np(img) - _np(oimg)).max() <= IMG_TOL
    (img * w.cuda()).sum().backward()
    for a, b, nm in zip(gins, ins, ("means2D", "cov2D", "opacities", "colors")):
        _grad_close(_np(a.grad), _np(b.grad), nm)


def test_golden_fixture_gpu():
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "scene_small.npz"))
    sc = {k: g["in_" + k] for k in ("means", "scales", "quats", "opac", "sh", "w2c", "active")}
    for k in ("W", "H", "sh_degree"):
        sc[k] = int(g["cfg_" + k])
    for k in ("fx", "fy", "cx", "cy"):
        sc[k] = float(g["cfg_" + k])
    img, ex, gg = gpu_render(sc, requires_grad=True)
    assert np.abs(_np(img) - g["out_image"]).max() <= IMG_TOL
    np.testing.assert_array_equal(_np(ex["radii"]), g["out_radii"])
    assert int(ex["n_interactions"]) == g["out_tiles"].shape[0]
    (img * torch.tensor(g["grad_weights"], device="cuda")).sum().backward()
    act = sc["active"]
    for f, k in (("means", "means"), ("scales", "scales"), ("quaternions", "quats"), ("opacities", "opac"),
                 ("sh_coeffs", "sh")):
        _grad_close(_np(getattr(gg, f).grad)[act], np.nan_to_num(g["grad_" + k][act]), f)


# ---------------------------------------------------------------- edge cases
def test_edge_empty_and_behind_camera():
    sc = random_scene(9, 200, 64, 48, behind=0.0)
    sc["active"] = np.zeros(200, bool)  # everything masked out
    img, ex, _ = gpu_render(sc)
    assert int(ex["n_interactions"]) == 0 and float(_np(img).max()) == 0.0
    sc = random_scene(9, 200, 64, 48, behind=1.0)  # everything behind the camera
    img, ex, _ = gpu_render(sc)
    oimg, oex, _ = oracle_render(sc)
    assert int(ex["n_interactions"]) == oex["n_interactions"]
    assert np.abs(_np(img) - _np(oimg)).max() <= IMG_TOL


def test_edge_nan_and_degenerate_inputs():
    sc = random_scene(10, 300, 64, 48, behind=0.0)
    sc["means"][0] = np.nan
    sc["quats"][1] = 0.0  # zero quaternion -> NaN covariance
    sc["scales"][2] = 50.0  # overflowing scale -> inf radius
    img, ex, g = gpu_render(sc, requires_grad=True)
    oimg, oex, _ = oracle_render(sc)
    assert np.isfinite(_np(img)).all()
    assert int(ex["n_interactions"]) == oex["n_interactions"]
    assert np.abs(_np(img) - _np(oimg)).max() <= IMG_TOL
    img.sum().backward()
    assert np.isfinite(_np(g.means.grad)[3:]).all()


@pytest.mark.parametrize("W,H", [(1, 1), (17, 5), (16, 16), (33, 100)])
def test_edge_image_sizes(W, H):
    sc = random_scene(12, 120, W, H, sh_degree=1, fov_f=60.0)
    img, ex, _ = gpu_render(sc)
    oimg, oex, _ = oracle_render(sc)
    assert img.shape == (H, W, 3)
    assert np.abs(_np(img) - _np(oimg)).max() <= IMG_TOL
    assert int(ex["n_interactions"]) == oex["n_interactions"]


def test_edge_tile_truncation_and_span_cap():
    """> MAX_TILE_INTERACTIONS splats on one tile, and splats wider than
    OFFSET_SIZE tiles (renderer.py:73-77 counters)."""
    n = 5000
    rng = np.random.default_rng(0)
    sc = random_scene(13, n, 300, 300, sh_degree=0, rotate=False, behind=0.0)
    sc["means"][:, 0] = rng.uniform(-0.02, 0.02, n)
    sc["means"][:, 1] = rng.uniform(-0.02, 0.02, n)
    sc["scales"][:] = -5.0
    sc["scales"][:5] = 1.5  # very wide splats: their clipped rectangles span > 16 tiles
    img, ex, _ = gpu_render(sc)
    oimg, oex, _ = oracle_render(sc)
    assert oex["truncated_tiles"] > 0 and oex["radius_cap_violations"] > 0
    for k in EXTRA_KEYS:
        assert int(ex[k]) == oex[k], k
    assert np.abs(_np(img) - _np(oimg)).max() <= IMG_TOL


def test_edge_capacity_overflow_is_reported_not_written():
    sc = random_scene(14, 500, 96, 80, sh_degree=0)
    _, oex, _ = oracle_render(sc)
    need = oex["n_interactions"]
    img, ex, _ = gpu_render(sc, capacity=need // 2)
    assert int(ex["n_interactions"]) == need
    assert int(ex["capacity_overflow"]) == need - need // 2
    assert np.isfinite(_np(img)).all()
    img2, ex2, _ = gpu_render(sc, capacity=need)
    assert int(ex2["capacity_overflow"]) == 0


def test_determinism_and_range():
    sc = random_scene(15, 3000, 200, 160, sh_degree=3)
    a, _, _ = gpu_render(sc)
    b, _, _ = gpu_render(sc)
    assert torch.equal(a, b)
    assert float(a.min()) >= 0.0 and float(a.max()) <= 1.0 + 1e-6


# ---------------------------------------------------------------- full-size properties
@pytest.mark.parametrize("which", ["config2", "config3"])
def test_full_size_sort_properties(which):
    """At BASELINE sizes (config 2: 200k capacity @ 504x378; config 3: 1M @
    1920x1080): the sorted interactions are exactly the per-Gaussian tile
    rectangles (count check against the oracle's rectangle code), ordered
    by (tile, depth key, Gaussian id), and the ranges bracket each tile."""
    from gs_b200 import synthetic
    from gs_b200.renderer.projection import project_gaussians
    from gs_b200.renderer.rasterizer import get_tile_interactions
    s = synthetic.config2(0) if which == "config2" else synthetic.config3(0, n_views=2)
    sc = scene_from_synthetic(s, 1)
    g, t = gpu_gaussians(sc)
    m2, cov, radii, valid, z = project_gaussians(g, gpu_camera(sc), mask=t["active"])
    tiles, gids, n, ranges = get_tile_interactions(m2, radii, valid, z, sc["H"], sc["W"], return_ranges=True)
    n = int(n)
    tx0, tx1, ty0, ty1, on = R._tile_rect(_np(m2), _np(radii), sc["H"], sc["W"])
    v = _np(valid) & on & (tx1 >= tx0) & (ty1 >= ty0)
    cnt = np.where(v, np.minimum(tx1 - tx0 + 1, 16) * np.minimum(ty1 - ty0 + 1, 16), 0)
    assert n == int(cnt.sum()) > 0
    tl = _np(tiles)[:n].astype(np.int64)
    gl = _np(gids)[:n].astype(np.int64)
    dq = (_np(z).view(np.int32) >> 18).astype(np.int64)[gl]
    key = (tl << 13) | dq
    assert (np.diff(key) >= 0).all()
    same = np.diff(key) == 0
    assert (np.diff(gl)[same] > 0).all()
    T = ((sc["W"] + 15) // 16) * ((sc["H"] + 15) // 16)
    np.testing.assert_array_equal(_np(ranges), np.searchsorted(tl, np.arange(T + 1)))
    assert np.array_equal(np.bincount(gl, minlength=len(cnt)), cnt)


def test_render_on_concurrent_streams_equals_sequential():
    """render() calls issued on four streams at once (each takes its scratch
    from the stream-aware allocator) give the images of one-at-a-time calls."""
    from gs_b200.core.camera import Camera
    from gs_b200.core.gaussians import Gaussians
    from gs_b200.renderer.renderer import render
    sc = random_scene(17, 4000, 160, 120, sh_degree=3, behind=0.05)
    t = to_torch(sc, "cuda")
    g = Gaussians(means=t["means"], scales=t["scales"], quaternions=t["quats"], opacities=t["opac"],
                  sh_coeffs=t["sh"])
    cams = []
    for i in range(8):
        w = t["w2c"].clone()
        w[0, 3] += 0.05 * i
        w[1, 3] -= 0.03 * i
        cams.append(Camera(sc["W"], sc["H"], sc["fx"], sc["fy"], sc["cx"], sc["cy"], w, None))
    with torch.no_grad():
        seq = [render(g, c, sh_degree=3)[0].clone() for c in cams]
        streams = [torch.cuda.Stream() for _ in range(4)]
        main = torch.cuda.current_stream()
        for s in streams:
            s.wait_stream(main)
        out = [None] * 8
        for i, c in enumerate(cams):
            with torch.cuda.stream(streams[i % 4]):
                out[i] = render(g, c, sh_degree=3)[0]
        for s in streams:
            main.wait_stream(s)
        torch.cuda.synchronize()
    for a, b in zip(seq, out):
        np.testing.assert_array_equal(_np(a), _np(b))
