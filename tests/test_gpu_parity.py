"""CUDA renderer vs the CPU oracle on the same seeded inputs, through the C ABI.

Bars: projected records bit-exact (K1 is built with -fmad=false and IEEE division/sqrt);
tile counts, scan offsets, emitted and sorted keys/values and bin ranges bit-exact; the image
within 1/255 per channel and >= 50 dB PSNR (the rasteriser uses the hardware exp2)."""

import numpy as np
import pytest

import oracle
from klartraum_b200 import Renderer, make_scene, native as N, orbit_camera, workload_camera
from klartraum_b200.scenes import WORKLOADS

from helpers import background, compare_projected, kat_bin_records, kat_project_scene, log_divergence, psnr

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def device_image(host: np.ndarray):
    return torch.from_numpy(host.copy()).cuda()


# name, workload, n, (W, H) override, bin, sh, flags, rows, background, distance override
CASES = [
    ("plumbing_full", "plumbing", None, None, 16, None, 0, None, "black", None),
    ("single1m_sub", "single_1m", 60000, None, 16, None, 0, None, "black", None),
    ("stress_sub", "stress_2m", 6000, None, 16, None, 0, None, "random", None),
    ("ref512_grid", "single_1m", 20000, (512, 512), 128, None, 0, None, "black", None),
    ("odd_screen", "plumbing", 5000, (200, 120), 16, None, 0, None, "random", None),
    ("band_rows", "plumbing", None, None, 16, None, 0, (5, 11), "black", None),
    ("per_element_exit", "single_1m", 30000, (640, 360), 16, None, N.FLAG_EXIT_PER_ELEMENT, None, "black", None),
    ("sh1", "stress_2m", 3000, (640, 480), 16, 1, 0, None, "black", 1.5),
    ("sh2", "single_1m", 8000, (320, 240), 32, 2, 0, None, "black", None),
]


def run_case(name, wname, n, wh, bin_size, sh, flags, rows, bg_kind, dist):
    w = WORKLOADS[wname]
    W, H = wh if wh else (w.width, w.height)
    sh = w.sh_degree if sh is None else sh
    g3d = make_scene(w, n=n)
    if sh < w.sh_degree:
        ncoef = (sh + 1) ** 2 - 1
        for ch in ("shR", "shG", "shB"):
            g3d[ch][:, ncoef:] = 0
    cam = orbit_camera(dist or w.distance, W, H, fovy_deg=60.0, up="y")
    bg = background(H, W, bg_kind)
    r = Renderer(W, H, bin_size=bin_size, sh_degree=sh, flags=flags | N.FLAG_KEEP_UNSORTED, tile_rows=rows)
    r.set_gaussians(g3d)
    img = device_image(bg)
    r.render(cam, img)
    out = img.cpu().numpy()
    cfg = oracle.config(W, H, bin_size=bin_size, sh_degree=sh, exit_per_element=bool(flags & N.FLAG_EXIT_PER_ELEMENT),
                        tile_rows=rows)
    ref = oracle.render_frame(cfg, cam, g3d, bg)
    ref["cfg"], ref["cam"], ref["g3d"] = cfg, cam, g3d
    return r, out, ref, bg


@pytest.mark.parametrize("keys", [False, True], ids=["placed", "sorted_keys"])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_frame_parity(case, keys):
    """Every stage buffer against the oracle, for the default path (pairs placed in bin order)
    and the reference-structured one (scan, key emission, radix sort, boundary search). On the
    default path OFFSETS and the unsorted keys/values are rebuilt on the host from the device's
    counts and rectangles (no device buffer holds them), so their equalities check the counts and
    rectangles, not a kernel of their own; the placement's device buffers are checked in
    test_gpu_placement.py. The image is also measured against the double-precision oracle."""
    case = list(case)
    if keys:
        case[6] |= N.FLAG_SORTED_KEYS
    r, out, ref, bg = run_case(*case)
    st = r.stats()
    assert st["error_flags"] == 0
    assert st["num_keys"] == ref["num_keys"]
    compare_projected(r.dump(N.STAGE_PROJECTED), ref["g2d"], ref["counts"])
    assert np.array_equal(r.dump(N.STAGE_TILE_COUNTS), ref["counts"])
    assert np.array_equal(r.dump(N.STAGE_OFFSETS), ref["offsets"])
    assert np.array_equal(r.dump(N.STAGE_KEYS_UNSORTED), ref["keys_unsorted"])
    assert np.array_equal(r.dump(N.STAGE_VALUES_UNSORTED), ref["vals_unsorted"])
    assert np.array_equal(r.dump(N.STAGE_KEYS_SORTED), ref["keys"])
    assert np.array_equal(r.dump(N.STAGE_VALUES_SORTED), ref["vals"])
    assert np.array_equal(r.dump(N.STAGE_TILE_RANGES), ref["ranges"])
    diff = np.abs(out.astype(np.int16) - ref["image"].astype(np.int16))
    assert diff.max() <= 1, f"max abs diff {diff.max()} at {np.unravel_index(diff.argmax(), diff.shape)}"
    assert psnr(out, ref["image"]) >= 50.0
    if st["num_keys"]:
        assert not np.array_equal(out, bg), "nothing was drawn"
    f64, _ = oracle.render_frame_f64(ref["cfg"], ref["cam"], ref["g3d"], bg)
    log_divergence(f"{case[0]}-{'sorted_keys' if keys else 'placed'}", out, ref["image"], f64)


def test_projection_known_answer_on_gpu():
    g, cam, k = kat_project_scene()
    r = Renderer(*k["screen"], bin_size=128, sh_degree=1)
    r.set_gaussians(g)
    img = device_image(background(512, 512))
    r.render(cam, img)
    p = r.dump(N.STAGE_PROJECTED)
    exp = np.array(k["expected_position"], np.float32)
    for i in range(4):
        for a in range(2):
            if k["exact"][i][a]:
                assert p["position"][i, a] == exp[i, a]
            else:
                assert abs(p["position"][i, a] - exp[i, a]) <= k["tolerance"]
    cfg = oracle.config(512, 512, bin_size=128, sh_degree=1)
    compare_projected(p, oracle.project(cfg, cam, g), r.dump(N.STAGE_TILE_COUNTS))


def test_bin_known_answer_on_gpu():
    g, k = kat_bin_records()
    r = Renderer(*k["screen"], bin_size=k["bin_size"], cull_z=-np.inf, flags=N.FLAG_KEEP_UNSORTED)
    img = device_image(background(512, 512))
    r.render_projected(g, img)
    keys = r.dump(N.STAGE_KEYS_UNSORTED)
    vals = r.dump(N.STAGE_VALUES_UNSORTED)
    bins = [sorted(int(b) for b in (keys[vals == i] >> np.uint64(32))) for i in range(len(g))]
    assert bins == k["expected_bins_no_cull"]
    # the same records with the reference's z-cull are all dropped
    r2 = Renderer(*k["screen"], bin_size=k["bin_size"])
    img2 = device_image(background(512, 512))
    r2.render_projected(g, img2)
    assert list(r2.dump(N.STAGE_TILE_COUNTS)) == k["expected_counts_with_cull"]
    assert np.array_equal(img2.cpu().numpy(), background(512, 512))


def test_render_projected_matches_oracle():
    w = WORKLOADS["single_1m"]
    g3d = make_scene(w, n=20000)
    cam = workload_camera(w)
    cfg = oracle.config(w.width, w.height, bin_size=16, sh_degree=3)
    g2d = oracle.project(cfg, cam, g3d)
    bg = background(w.height, w.width, "random")
    r = Renderer(w.width, w.height, bin_size=16)
    img = device_image(bg)
    r.render_projected(g2d, img)
    ref = oracle.render_projected(cfg, g2d, bg)
    assert np.array_equal(r.dump(N.STAGE_KEYS_SORTED), ref["keys"])
    assert np.array_equal(r.dump(N.STAGE_VALUES_SORTED), ref["vals"])
    out = img.cpu().numpy()
    assert np.abs(out.astype(int) - ref["image"].astype(int)).max() <= 1


def test_empty_scene_leaves_background():
    r = Renderer(256, 256, bin_size=16)
    r.set_gaussians(make_scene("plumbing", n=0))
    bg = background(256, 256, "random")
    img = device_image(bg)
    r.render(workload_camera("plumbing"), img)
    assert r.stats()["num_keys"] == 0
    assert np.array_equal(img.cpu().numpy(), bg)


def test_all_culled_scene_leaves_background():
    # camera 0.5 away from a point cloud behind it: every clip z is below 1.0
    g = make_scene("plumbing", n=5000)
    g["position"][:, 0] = np.abs(g["position"][:, 0]) + 3.0
    cam = orbit_camera(1.0, 256, 256, fovy_deg=60.0, up="y")
    r = Renderer(256, 256, bin_size=16, sh_degree=0)
    r.set_gaussians(g)
    bg = background(256, 256, "random")
    img = device_image(bg)
    r.render(cam, img)
    st = r.stats()
    assert st["num_keys"] == 0 and st["num_visible"] == 0
    assert np.array_equal(img.cpu().numpy(), bg)


def test_single_gaussian():
    g = make_scene("plumbing", n=1)
    g["position"] = [0, 0, 0]
    g["scale"] = 0.05
    g["alpha"] = 0.9
    cam = workload_camera("plumbing")
    r = Renderer(256, 256, bin_size=16, sh_degree=0)
    r.set_gaussians(g)
    bg = background(256, 256)
    img = device_image(bg)
    r.render(cam, img)
    cfg = oracle.config(256, 256, bin_size=16, sh_degree=0)
    ref = oracle.render_frame(cfg, cam, g, bg)
    assert r.stats()["num_keys"] == ref["num_keys"] > 0
    assert np.abs(img.cpu().numpy().astype(int) - ref["image"].astype(int)).max() <= 1


def test_capacity_growth_and_overflow_error():
    w = WORKLOADS["single_1m"]
    g3d = make_scene(w, n=50000)
    cam = workload_camera(w)
    bg = background(w.height, w.width)
    # auto-grow from a deliberately small capacity gives the same frame
    r = Renderer(w.width, w.height, bin_size=16, key_capacity=4096)
    r.set_gaussians(g3d)
    img = device_image(bg)
    r.render(cam, img)
    st = r.stats()
    assert st["key_capacity"] >= st["num_keys"] > 4096
    r_big = Renderer(w.width, w.height, bin_size=16)
    r_big.set_gaussians(g3d)
    img_big = device_image(bg)
    r_big.render(cam, img_big)
    assert torch.equal(img, img_big)
    # without auto-grow the call fails with KT_ERR_CAPACITY and draws nothing
    r_small = Renderer(w.width, w.height, bin_size=16, key_capacity=4096, flags=N.FLAG_NO_AUTOGROW)
    r_small.set_gaussians(g3d)
    img_small = device_image(bg)
    with pytest.raises(N.KtError) as e:
        r_small.render(cam, img_small)
    assert e.value.status == N.KT_ERR_CAPACITY
    assert r_small.stats()["num_keys"] == st["num_keys"]
    assert np.array_equal(img_small.cpu().numpy(), bg)


def test_deterministic_replay():
    w = WORKLOADS["stress_2m"]
    g3d = make_scene(w, n=20000)
    cam = workload_camera(w)
    r = Renderer(w.width, w.height, bin_size=16, sh_degree=1)
    r.set_gaussians(g3d)
    outs = []
    for _ in range(2):
        img = device_image(background(w.height, w.width))
        r.render(cam, img)
        outs.append((img.cpu().numpy(), r.dump(N.STAGE_VALUES_SORTED), r.dump(N.STAGE_TILE_RANGES)))
    for a, b in zip(outs[0], outs[1]):
        assert np.array_equal(a, b)


def host_image(a, kind):
    """A host image holding `a`: a pageable numpy array (the runtime stages its copies) or a
    page-locked torch tensor (copied by DMA)."""
    if kind == "pageable":
        return a.copy()
    t = torch.empty(a.shape, dtype=torch.uint8, pin_memory=True)
    t.copy_(torch.from_numpy(a))
    return t


def host_array(h):
    return h if isinstance(h, np.ndarray) else h.numpy()


@pytest.mark.parametrize("kind", ["pageable", "pinned"])
def test_render_host_matches_device_render(kind):
    w = WORKLOADS["plumbing"]
    g3d = make_scene(w)
    cam = workload_camera(w)
    bg = background(w.height, w.width, "random")
    r = Renderer(w.width, w.height, bin_size=16, sh_degree=0)
    r.set_gaussians(g3d)
    host = host_image(bg, kind)
    r.render_host(cam, host)
    img = device_image(bg)
    r.render(cam, img)
    assert np.array_equal(host_array(host), img.cpu().numpy())


def test_unaligned_images_are_refused():
    """RGBA8 pixels are written as 4-byte words: an image address that is not 4-byte aligned is
    refused before anything is launched."""
    r = Renderer(64, 64, bin_size=16, sh_degree=0)
    r.set_gaussians(make_scene("plumbing", n=100))
    img = torch.zeros(64 * 64 * 4 + 4, dtype=torch.uint8, device="cuda")
    with pytest.raises(N.KtError) as e:
        r.render(workload_camera("plumbing"), img.data_ptr() + 1)
    assert e.value.status == N.KT_ERR_ARG
    r.close()


def test_render_batch_matches_single_views():
    from klartraum_b200 import orbit_views

    g3d = make_scene("plumbing", n=8000)
    cams = orbit_views(4, 1.5, 256, 256)
    r = Renderer(256, 256, bin_size=16, sh_degree=0)
    r.set_gaussians(g3d)
    imgs = [device_image(background(256, 256)) for _ in range(4)]
    r.render_batch(cams, imgs)
    for v in range(4):
        single = device_image(background(256, 256))
        r.render(cams[v], single)
        assert torch.equal(single, imgs[v])


def test_multiple_paths_are_independent():
    g3d = make_scene("plumbing", n=8000)
    cam = workload_camera("plumbing")
    r = Renderer(256, 256, bin_size=16, sh_degree=0, num_paths=2)
    r.set_gaussians(g3d)
    a, b = device_image(background(256, 256)), device_image(background(256, 256))
    r.render(cam, a, path=0)
    r.render(cam, b, path=1)
    assert torch.equal(a, b)
    assert r.stats(0)["num_keys"] == r.stats(1)["num_keys"]


def test_sh_degree_detection():
    g3d = make_scene("single_1m", n=1000)
    r = Renderer(320, 240, bin_size=16, sh_degree=-1)
    r.set_gaussians(g3d)
    assert r.sh_degree == 3
    g0 = make_scene("plumbing", n=1000)
    r0 = Renderer(320, 240, bin_size=16, sh_degree=-1)
    r0.set_gaussians(g0)
    assert r0.sh_degree == 0


def test_async_frames_report_overflow_at_sync_only_once():
    w = WORKLOADS["single_1m"]
    g3d = make_scene(w, n=50000)
    cam = workload_camera(w)
    bg = background(w.height, w.width)
    # a checked frame that had to grow its buffers leaves nothing for a later sync
    r = Renderer(w.width, w.height, bin_size=16, key_capacity=4096)
    r.set_gaussians(g3d)
    img = device_image(bg)
    r.render(cam, img)
    r.sync()
    # an async frame that overflows draws nothing and is reported by the next sync, once
    r2 = Renderer(w.width, w.height, bin_size=16, key_capacity=4096, flags=N.FLAG_ASYNC | N.FLAG_NO_AUTOGROW)
    r2.set_gaussians(g3d)
    img2 = device_image(bg)
    r2.render(cam, img2)
    r2.render(cam, img2)
    with pytest.raises(N.KtError) as e:
        r2.sync()
    assert e.value.status == N.KT_ERR_CAPACITY
    assert np.array_equal(img2.cpu().numpy(), bg)
    r2.set_flags(N.FLAG_NO_AUTOGROW)
    with pytest.raises(N.KtError):
        r2.render(cam, img2)
    r2.sync()  # the failed checked frame was reported by render() itself


def test_counters_accumulate_frames_and_keys():
    g3d = make_scene("plumbing", n=8000)
    cam = workload_camera("plumbing")
    r = Renderer(256, 256, bin_size=16, sh_degree=0, flags=N.FLAG_TIMING)
    r.set_gaussians(g3d)
    img = device_image(background(256, 256))
    r.render(cam, img)
    r.counters()
    r.stage_times_total()
    r.set_flags(N.FLAG_TIMING | N.FLAG_ASYNC)
    for _ in range(20):
        r.render(cam, img)
    r.sync()
    c = r.counters()
    st = r.stats()
    assert c["frames"] == 20 and c["keys"] == 20 * st["num_keys"]
    assert st["sort_passes"] == 0 and c["key_passes"] == 0  # pairs placed in bin order directly
    # 4 B per pair and 8 B per (Gaussian, coarse bin) entry; entries <= pairs
    assert 4 * c["keys"] < c["sort_bytes"] <= 12 * c["keys"] and (c["sort_bytes"] - 4 * c["keys"]) % 8 == 0
    ms, frames = r.stage_times_total()
    assert frames == 20 and ms["frame"] > 0 and ms["fine_place"] > 0
    assert r.counters()["frames"] == 0


@pytest.mark.parametrize("wname,n,wh", [("single_1m", 200000, (1280, 720)), ("stress_2m", 20000, (960, 540))])
def test_sorted_keys_path_draws_the_same_image(wname, n, wh):
    """The two binning paths order the pairs identically, so their images are identical."""
    w = WORKLOADS[wname]
    g3d = make_scene(w, n=n)
    cam = orbit_camera(w.distance, *wh, fovy_deg=60.0, up="y")
    bg = background(wh[1], wh[0], "random")
    imgs, keys = [], []
    for flags in (0, N.FLAG_SORTED_KEYS):
        r = Renderer(*wh, bin_size=16, sh_degree=w.sh_degree, flags=flags)
        r.set_gaussians(g3d)
        img = device_image(bg)
        r.render(cam, img)
        imgs.append(img.cpu().numpy())
        keys.append((r.dump(N.STAGE_KEYS_SORTED), r.dump(N.STAGE_VALUES_SORTED), r.dump(N.STAGE_TILE_RANGES)))
        assert r.stats()["sort_passes"] == (0 if flags == 0 else r.stats()["sort_passes"])
        r.close()
    assert np.array_equal(imgs[0], imgs[1])
    for a, b in zip(keys[0], keys[1]):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("kind", ["pageable", "pinned"])
def test_render_host_clear_equals_a_cleared_image(kind):
    """kt_gs_render_host_clear: the device image set to the clear colour, then the frame; the
    same as kt_gs_render_host given an image of that colour, on both binning paths, bands (whose
    rows outside the band stay cleared) and a graph replay, into pageable and pinned images."""
    g3d = make_scene("plumbing", n=6000)
    cam = workload_camera("plumbing")
    for flags, rows in [(0, None), (N.FLAG_SORTED_KEYS, None), (0, (3, 9)), (N.FLAG_GRAPH, (0, 5))]:
        r = Renderer(256, 256, bin_size=16, sh_degree=0, flags=flags, tile_rows=rows)
        r.set_gaussians(g3d)
        for clear in [(0, 0, 0, 255), (10, 200, 30, 0)]:
            host = host_image(np.full((256, 256, 4), 77, np.uint8), kind)  # overwritten entirely
            r.render_host_clear(cam, host, clear=clear)
            expect = np.empty((256, 256, 4), np.uint8)
            expect[:] = clear
            r.render_host(cam, expect)
            assert np.array_equal(host_array(host), expect)
        r.close()
