"""The CPU oracle against the reference's own known answers (tests/golden/reference_kat.json)
and against independent numpy restatements of its integer stages."""

import numpy as np
import pytest

import oracle
from klartraum_b200 import GAUSSIAN2D_DTYPE, make_scene, orbit_camera, reference_key, workload_camera

from helpers import kat_bin_records, kat_project_scene, load_kat


def test_projection_known_answer():
    g, cam, k = kat_project_scene()
    cfg = oracle.config(*k["screen"], bin_size=128, sh_degree=1)
    out = oracle.project(cfg, cam, g)
    exp = np.array(k["expected_position"], np.float32)
    for i in range(4):
        for a in range(2):
            if k["exact"][i][a]:
                assert out["position"][i, a] == exp[i, a], (i, a, out["position"][i])
            else:
                assert abs(out["position"][i, a] - exp[i, a]) <= k["tolerance"], (i, a, out["position"][i])


def test_sort_known_answer():
    k = load_kat()["sort"]
    keys = reference_key(np.array(k["binMask"], np.uint64), np.array(k["z"], np.float32))
    sk, sv = oracle.sort_pairs(keys, np.arange(8, dtype=np.uint32), 64)
    assert list(sv) == k["expected_order"]
    z_sorted = np.array(k["z"], np.float32)[sv]
    assert list(z_sorted[:4]) == pytest.approx(k["expected_first4_z"])
    masks = np.array(k["binMask"])[sv][4:]
    assert np.all(np.diff(masks) >= 0)


def test_bin_known_answer():
    g, k = kat_bin_records()
    cfg = oracle.config(*k["screen"], bin_size=k["bin_size"], cull_z=-np.inf)
    counts = oracle.tile_counts(cfg, g)
    off, total = oracle.exclusive_scan(counts)
    keys, vals = oracle.emit_keys(cfg, g, off, total)
    bins = [sorted(int(b) for b in (keys[vals == i] >> np.uint64(32))) for i in range(len(g))]
    assert bins == k["expected_bins_no_cull"]
    masks = {1 << b[0] for b in bins}
    assert masks <= set(k["reference_mask_list"])
    cfg_cull = oracle.config(*k["screen"], bin_size=k["bin_size"])
    assert list(oracle.tile_counts(cfg_cull, g)) == k["expected_counts_with_cull"]


def overlaps_numpy(g2d, cfg, tx, ty):
    """All-bins evaluation of gsplat_binning.comp:53-81 in numpy float32."""
    ci = g2d["covInv"].astype(np.float32)
    det = ci[:, 0] * ci[:, 3] - ci[:, 2] * ci[:, 1]
    inv = np.float32(1) / det
    cxx = ci[:, 3] * inv
    cyy = ci[:, 0] * inv
    sx = np.sqrt(cxx) * np.float32(2.5)
    sy = np.sqrt(cyy) * np.float32(2.5)
    pos = g2d["position"].astype(np.float32)
    mnx, mxx, mny, mxy = pos[:, 0] - sx, pos[:, 0] + sx, pos[:, 1] - sy, pos[:, 1] + sy
    gx = np.arange(tx, dtype=np.float32)
    gy = np.arange(ty, dtype=np.float32)
    cw, ch = np.float32(cfg.bin_width), np.float32(cfg.bin_height)
    ox = ~((mxx[:, None] < gx * cw) | (mnx[:, None] > (gx + 1) * cw))
    oy = ~((mxy[:, None] < gy * ch) | (mny[:, None] > (gy + 1) * ch))
    keep = ~(g2d["z"] < np.float32(cfg.cull_z))
    return ox.sum(1) * oy.sum(1) * keep


@pytest.mark.parametrize("wname,n", [("plumbing", 4000), ("single_1m", 3000), ("stress_2m", 500)])
def test_tile_counts_match_all_bins_evaluation(wname, n):
    from klartraum_b200.scenes import WORKLOADS

    w = WORKLOADS[wname]
    g3d = make_scene(w, n=n)
    cam = workload_camera(w)
    cfg = oracle.config(w.width, w.height, bin_size=16, sh_degree=w.sh_degree)
    g2d = oracle.project(cfg, cam, g3d)
    tx, ty = oracle.tiles(cfg)
    assert np.array_equal(oracle.tile_counts(cfg, g2d), overlaps_numpy(g2d, cfg, tx, ty).astype(np.uint32))


def test_sort_is_a_stable_sort():
    rng = np.random.default_rng(3)
    for n, bits in [(0, 40), (1, 40), (5000, 45), (70000, 13), (100000, 64)]:
        keys = rng.integers(0, 1 << min(bits, 62), size=n, dtype=np.uint64) & np.uint64((1 << bits) - 1 if bits < 64 else -1 & 0xFFFFFFFFFFFFFFFF)
        if n > 10:
            keys[::7] = keys[0]  # many ties
        vals = np.arange(n, dtype=np.uint32)
        sk, sv = oracle.sort_pairs(keys, vals, bits)
        order = np.argsort(keys, kind="stable")
        assert np.array_equal(sk, keys[order]) and np.array_equal(sv, vals[order])


def test_ranges_follow_bin_bounds_shader():
    keys = (np.array([0, 0, 2, 2, 2, 5, 7, 7], np.uint64) << np.uint64(32)) | np.uint64(9)
    r = oracle.tile_ranges(keys, 8)
    exp = np.zeros((8, 2), np.uint32)
    exp[0] = [0, 2]
    exp[2] = [2, 5]
    exp[5] = [5, 6]
    exp[7] = [6, 8]
    assert np.array_equal(r, exp)


def test_scan_and_emission_agree():
    w = "plumbing"
    g3d = make_scene(w, n=2000)
    cam = workload_camera(w)
    cfg = oracle.config(256, 256, bin_size=16, sh_degree=0)
    g2d = oracle.project(cfg, cam, g3d)
    counts = oracle.tile_counts(cfg, g2d)
    off, total = oracle.exclusive_scan(counts)
    assert total == int(counts.sum())
    assert np.array_equal(off, np.concatenate([[0], np.cumsum(counts, dtype=np.uint64)[:-1]]))
    keys, vals = oracle.emit_keys(cfg, g2d, off, total)
    assert np.array_equal(np.bincount(vals, minlength=len(g2d)), counts)
    zb = g2d["z"].view(np.uint32) ^ np.uint32(0x80000000)
    assert np.array_equal(keys & np.uint64(0xFFFFFFFF), zb[vals].astype(np.uint64))


def test_rasterizer_batch_exit_semantics():
    """Opaque Gaussians saturate a pixel after the first; the reference still blends the rest
    of the 64-batch, then one tail element (gsplat_binned_splatting.comp:78-117)."""
    n = 70  # 64-batch + 6 tail elements, all at the pixel
    g = np.zeros(n, GAUSSIAN2D_DTYPE)
    g["position"] = [0.0, 0.0]
    g["covInv"] = [1.0, 0.0, 0.0, 1.0]
    g["alpha"] = 0.99999
    g["color"] = np.linspace(0.1, 0.9, n)[:, None]
    g["z"] = 2.0
    cfg = oracle.config(16, 16, bin_size=16, sh_degree=0)
    vals = np.arange(n, dtype=np.uint32)
    ranges = np.array([[0, n]], np.uint32)
    img0 = np.zeros((16, 16, 4), np.uint8)
    ref = oracle.rasterize(cfg, g, vals, ranges, img0)
    # pixel (0,0): manual replay of the shader loop in float32
    f = np.float32
    C = f(0)
    T = f(1)
    tmin = f(1.0 - 0.9999)
    for i in list(range(64)) + [64]:
        a = f(np.exp(f(-0.5) * f(0))) * g["alpha"][i]
        C = f(C + f(f(g["color"][i, 0] * a) * T))
        T = f(T * f(f(1) - a))
    out = np.uint8(np.rint(min(max(f(0) + f(C * f(f(1) - T)), 0), 1) * 255))
    assert ref[0, 0, 0] == out
    cfg_pe = oracle.config(16, 16, bin_size=16, sh_degree=0, exit_per_element=True)
    pe = oracle.rasterize(cfg_pe, g, vals, ranges, img0)
    assert pe[0, 0, 0] == np.uint8(np.rint(f(g["color"][0, 0] * g["alpha"][0]) * (f(1) - f(1 - g["alpha"][0])) * 255))
