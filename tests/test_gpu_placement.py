"""The pair placement's own device buffers against a direct model computed from the oracle.

The default binning path never sorts (bin, Gaussian) pairs: it sorts the Gaussians by depth and
then places the pairs by bin in two levels (klartraum_b200/csrc/place.cu). Its end product, the
pairs in bin order, is checked against the oracle in test_gpu_parity.py; this file checks the
intermediate device buffers stage by stage, so that a fault in one level shows at that level:

* DEPTH_ORDER   the depth sort's output: the indices of the Gaussians that meet a bin, stably
                sorted by floatBitsToUint(z) ^ 0x80000000 (the depth digits of
                shaders/gsplat/gsplat_radix_sort_include.glsl:51-63);
* COARSE_INFO   per coarse bin (4x4 bins): list start, entries, first segment;
* COARSE_LISTS  per coarse bin, (Gaussian, mask of the 4x4 bins met) in depth order;
* SEGMENT_COUNTS per 256-entry segment of a coarse list, the pairs of each of its 16 bins.

The model below is written from those definitions (numpy, vectorised), with the bin rectangles
and depths taken from the oracle, not from the GPU.
"""

import numpy as np
import pytest

import oracle
from klartraum_b200 import Renderer, make_scene, native as N, orbit_camera
from klartraum_b200.scenes import WORKLOADS

from helpers import background

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

COARSE = 4
SEG_LEN = 256


def span4(lo, hi):
    return ((1 << hi) - 1) & ~((1 << lo) - 1)


def placement_model(rects, depth_key, tx, rows):
    """Depth order, coarse lists, coarse info and segment counts from their definitions.
    rects: (n, 4) x0, x1, y0, y1 in bins, clipped to the binned rows, zeros for no bins;
    depth_key: the depth digits of every Gaussian."""
    n = len(rects)
    rb, re = rows
    visible = (rects[:, 1] > rects[:, 0]) & (rects[:, 3] > rects[:, 2])
    vis_idx = np.nonzero(visible)[0]
    order = vis_idx[np.argsort(depth_key[vis_idx], kind="stable")].astype(np.uint32)

    ctx, cty = (tx + 3) // 4, (re - rb + 3) // 4
    ncoarse = ctx * cty
    q = order
    x0, x1 = rects[q, 0].astype(np.int64), rects[q, 1].astype(np.int64)
    y0, y1 = rects[q, 2].astype(np.int64) - rb, rects[q, 3].astype(np.int64) - rb
    cx0, cx1 = x0 // 4, (x1 + 3) // 4
    cy0, cy1 = y0 // 4, (y1 + 3) // 4
    cw = cx1 - cx0
    ne = cw * (cy1 - cy0)
    first = np.cumsum(ne) - ne
    e = int(ne.sum())
    gi = np.repeat(np.arange(len(q)), ne)
    t = np.arange(e) - first[gi]
    dy, dx = t // cw[gi], t % cw[gi]
    ccx, ccy = cx0[gi] + dx, cy0[gi] + dy
    coarse = ccy * ctx + ccx
    bx, by = ccx * 4, ccy * 4
    clo = np.maximum(x0[gi], bx) - bx
    chi = np.minimum(x1[gi], bx + 4) - bx
    rlo = np.maximum(y0[gi], by) - by
    rhi = np.minimum(y1[gi], by + 4) - by
    cols = ((1 << chi) - 1) & ~((1 << clo) - 1)
    rws = ((1 << rhi) - 1) & ~((1 << rlo) - 1)
    spread = (rws & 1) | ((rws & 2) << 3) | ((rws & 4) << 6) | ((rws & 8) << 9)
    mask = (cols * spread).astype(np.uint32)
    by_bin = np.argsort(coarse, kind="stable")  # entries are generated in depth order
    clist = np.stack([q[gi[by_bin]].astype(np.uint32), mask[by_bin]], axis=1)
    tot = np.bincount(coarse, minlength=ncoarse).astype(np.int64)
    start = np.cumsum(tot) - tot
    nseg = (tot + SEG_LEN - 1) // SEG_LEN
    seg0 = np.cumsum(nseg) - nseg
    cinfo = np.stack([start, tot, seg0, np.zeros_like(tot)], axis=1).astype(np.uint32)
    bits = ((clist[:, 1][:, None] >> np.arange(16, dtype=np.uint32)) & 1).astype(np.int64)
    seg_cnt = np.zeros((int(nseg.sum()), 16), np.uint32)
    for c in np.nonzero(tot)[0]:
        for s in range(int(nseg[c])):
            a = int(start[c]) + s * SEG_LEN
            b = min(a + SEG_LEN, int(start[c] + tot[c]))
            seg_cnt[int(seg0[c]) + s] = bits[a:b].sum(0)
    return order, cinfo, clist, seg_cnt


# workload, n, (W, H), bin rows
CASES = [
    ("single_1m", 60000, (1920, 1080), None),   # 30 x 17 coarse bins, one placement band
    ("plumbing", None, (256, 256), (5, 11)),     # a band of bin rows: ragged coarse rows
    ("plumbing", 5000, (200, 120), None),        # ragged coarse columns
    ("single_1m", 150000, (3840, 2160), None),   # 60 x 34 coarse bins: two placement bands
    ("stress_2m", 8000, (1280, 720), None),      # large Gaussians: long coarse lists
    ("stress_2m", 200000, (640, 360), None),     # 60 coarse lists of ~60 segments: long runs, small bands
]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}-{c[2][0]}x{c[2][1]}" + ("-band" if c[3] else "")
                                             for c in CASES])
def test_placement_buffers_match_the_model(case):
    wname, n, (W, H), rows = case
    w = WORKLOADS[wname]
    g3d = make_scene(w, n=n)
    cam = orbit_camera(w.distance, W, H, fovy_deg=60.0, up="y")
    r = Renderer(W, H, bin_size=16, sh_degree=w.sh_degree, tile_rows=rows)
    r.set_gaussians(g3d)
    img = torch.from_numpy(background(H, W)).cuda()
    r.render(cam, img)
    st = r.stats()
    assert st["error_flags"] == 0

    cfg = oracle.config(W, H, bin_size=16, sh_degree=w.sh_degree, tile_rows=rows)
    g2d = oracle.project(cfg, cam, g3d)
    rects = oracle.tile_rects(cfg, g2d)
    depth_key = g2d["z"].view(np.uint32) ^ np.uint32(0x80000000)
    tx, ty = oracle.tiles(cfg)
    band = rows if rows else (0, ty)
    order, cinfo, clist, seg_cnt = placement_model(rects, depth_key, tx, band)

    assert np.array_equal(r.dump(N.STAGE_DEPTH_ORDER), order)
    assert np.array_equal(r.dump(N.STAGE_COARSE_INFO), cinfo)
    got_clist = r.dump(N.STAGE_COARSE_LISTS)
    assert got_clist.shape == clist.shape
    bad = np.nonzero((got_clist != clist).any(axis=1))[0]
    assert bad.size == 0, f"{bad.size} coarse entries differ, first at {bad[:5]}: {got_clist[bad[:3]]} vs {clist[bad[:3]]}"
    assert np.array_equal(r.dump(N.STAGE_SEGMENT_COUNTS), seg_cnt)
    # a slice through the windowed dump equals the same slice of the whole buffer
    k = len(clist)
    if k > 10:
        assert np.array_equal(r.dump(N.STAGE_COARSE_LISTS, first=k // 3, count=k // 3), clist[k // 3:2 * (k // 3)])
    # and the pairs that follow from them are the oracle's
    ref = oracle.render_frame(cfg, cam, g3d, background(H, W))
    assert np.array_equal(r.dump(N.STAGE_VALUES_SORTED), ref["vals"])


def test_placement_dumps_are_refused_on_the_keys_path():
    g3d = make_scene("plumbing", n=2000)
    r = Renderer(256, 256, bin_size=16, sh_degree=0, flags=N.FLAG_SORTED_KEYS)
    r.set_gaussians(g3d)
    img = torch.from_numpy(background(256, 256)).cuda()
    r.render(orbit_camera(1.5, 256, 256, fovy_deg=60.0, up="y"), img)
    with pytest.raises(N.KtError) as e:
        r.dump(N.STAGE_COARSE_LISTS)
    assert e.value.status == N.KT_ERR_STATE


def test_both_pair_placement_kernels_match_the_oracle():
    """The first frame of a path places pairs with a warp per segment; when the path's last frame
    had many segments per warp (here ~70k segments for ~9.5k warps), the next frames take runs of
    segments with the next one prefetched (kt_gs_stats.place_runs). Both must give the oracle's
    sorted pairs, ranges and image."""
    w = WORKLOADS["stress_2m"]
    g3d = make_scene(w, n=150000)
    cam = orbit_camera(w.distance, w.width, w.height, fovy_deg=60.0, up="y")
    cfg = oracle.config(w.width, w.height, bin_size=16, sh_degree=1)
    ref = oracle.render_frame(cfg, cam, g3d, background(w.height, w.width))
    r = Renderer(w.width, w.height, bin_size=16, sh_degree=1, key_capacity=ref["num_keys"] + 4096)
    r.set_gaussians(g3d)
    runs = []
    for frame in range(3):
        img = torch.from_numpy(background(w.height, w.width)).cuda()
        r.render(cam, img)
        st = r.stats()
        runs.append(st["place_runs"])
        assert st["num_keys"] == ref["num_keys"]
        assert np.array_equal(r.dump(N.STAGE_VALUES_SORTED), ref["vals"]), f"frame {frame}"
        assert np.array_equal(r.dump(N.STAGE_TILE_RANGES), ref["ranges"]), f"frame {frame}"
        assert np.abs(img.cpu().numpy().astype(int) - ref["image"].astype(int)).max() <= 1
    assert len(r.dump(N.STAGE_SEGMENT_COUNTS)) > 60000
    assert runs == [0, 1, 1], runs
    r.close()
