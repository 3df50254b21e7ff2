"""Sharding across ranks: view split, bin-row bands, strip gather.

CPU tests run two gloo ranks as spawned processes; each renders its band with the oracle and the
gathered frame must equal the oracle's full frame. The GPU test renders the bands through the
C ABI on one GPU and checks that they tile the full frame bit for bit.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from klartraum_b200.multigpu import band_pixel_rows, band_rows, gather_strips, row_pair_counts, view_shard

from helpers import background


def test_view_shard_partitions_views():
    for n_views in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            seen = [v for r in range(world) for v in view_shard(n_views, world, r)]
            assert sorted(seen) == list(range(n_views))
            sizes = [len(view_shard(n_views, world, r)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        view_shard(4, 2, 2)


@pytest.mark.parametrize("tiles_y", [1, 2, 5, 68, 135])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_band_rows_cover_rows(tiles_y, world):
    rng = np.random.default_rng(tiles_y * 10 + world)
    for weights in (None, rng.integers(0, 1000, tiles_y), np.zeros(tiles_y), np.r_[np.zeros(tiles_y - 1), 5]):
        bands = band_rows(tiles_y, world, weights)
        assert len(bands) == world
        assert bands[0][0] == 0 and bands[-1][1] == tiles_y
        for (a0, a1), (b0, b1) in zip(bands, bands[1:]):
            assert a1 == b0
        for a, b in bands:
            assert a <= b
            if tiles_y >= world:
                assert b > a


def test_band_rows_balance_weights():
    w = np.r_[np.full(60, 1.0), np.full(8, 100.0)]  # heavy bottom rows
    bands = band_rows(68, 2, w)
    loads = [w[a:b].sum() for a, b in bands]
    assert max(loads) / sum(loads) < 0.55
    eq = band_rows(68, 2)
    assert eq == [(0, 34), (34, 68)]


def test_rebalance_bands_follows_measured_time():
    """Bands balanced on pairs, but the pairs of the top half cost three times as much (say,
    larger Gaussians there): after one rebalance on the measured times each band's predicted
    time is about equal, and a second rebalance with times that match the prediction keeps it."""
    from klartraum_b200.multigpu import rebalance_bands

    ty, world = 120, 4
    pairs = np.full(ty, 100.0)
    cost = np.r_[np.full(60, 3.0), np.full(60, 1.0)]  # time per pair, unknown to the splitter
    bands = band_rows(ty, world, pairs)
    times = [float((pairs * cost)[a:b].sum()) for a, b in bands]
    assert max(times) / min(times) > 2.0
    new = rebalance_bands(pairs, bands, times)
    t2 = [float((pairs * cost)[a:b].sum()) for a, b in new]
    assert max(t2) / min(t2) < 1.15
    assert new[0][0] == 0 and new[-1][1] == ty and all(a1 == b0 for (_, a1), (b0, _) in zip(new, new[1:]))
    again = rebalance_bands(pairs, new, t2)
    t3 = [float((pairs * cost)[a:b].sum()) for a, b in again]
    assert max(t3) / min(t3) < 1.15
    with pytest.raises(ValueError):
        rebalance_bands(pairs, bands, times[:2])


def test_band_pixel_rows_clip_last_band():
    assert band_pixel_rows((0, 34), 16, 1080) == (0, 544)
    assert band_pixel_rows((34, 68), 16, 1080) == (544, 1080)


def test_row_pair_counts():
    ranges = np.array([[0, 3], [3, 3], [3, 10], [10, 11]], dtype=np.uint32)
    assert row_pair_counts(ranges, 2, 2).tolist() == [3, 8]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


W, H, BIN = 96, 80, 16


def _scene():
    from klartraum_b200 import make_scene, orbit_camera

    g3d = make_scene("plumbing", n=3000, seed=11)
    cam = orbit_camera(3.0, W, H, fovy_deg=45.0, azimuth=0.3, elevation=0.2)
    return g3d, cam


def _band_worker(rank: int, world: int, port: int, out_path: str, weighted: bool):
    import torch.distributed as dist

    import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch

        g3d, cam = _scene()
        bg = background(H, W, "random")
        ty = (H + BIN - 1) // BIN
        weights = None
        if weighted:
            # balance on the pair counts of a previous full frame, as a renderer would
            full = oracle.render_frame(oracle.config(W, H, bin_size=BIN, sh_degree=0), cam, g3d, bg)
            weights = row_pair_counts(full["ranges"], (W + BIN - 1) // BIN, ty)
        bands = band_rows(ty, world, weights)
        px = [band_pixel_rows(b, BIN, H) for b in bands]
        cfg = oracle.config(W, H, bin_size=BIN, sh_degree=0, tile_rows=bands[rank])
        img = oracle.render_frame(cfg, cam, g3d, bg)["image"]
        r0, r1 = px[rank]
        frame = gather_strips(torch.from_numpy(np.ascontiguousarray(img[r0:r1])), px, W, H, dist, rank)
        if rank == 0:
            np.save(out_path, frame.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("weighted", [False, True])
def test_banded_frame_gathers_to_full_frame_gloo(tmp_path, weighted):
    """Two gloo ranks render a band each (oracle) and all-gather the strips; the assembled frame
    equals the oracle's full frame byte for byte."""
    import torch.multiprocessing as mp

    import oracle

    out = str(tmp_path / "frame.npy")
    mp.start_processes(_band_worker, args=(2, _free_port(), out, weighted), nprocs=2, join=True,
                       start_method="spawn")
    g3d, cam = _scene()
    bg = background(H, W, "random")
    full = oracle.render_frame(oracle.config(W, H, bin_size=BIN, sh_degree=0), cam, g3d, bg)["image"]
    assert np.array_equal(np.load(out), full)


def _view_worker(rank: int, world: int, port: int, out_path: str):
    import torch
    import torch.distributed as dist

    import oracle

    from klartraum_b200 import orbit_views

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g3d, _ = _scene()
        cams = orbit_views(5, 3.0, W, H, fovy_deg=45.0)
        bg = background(H, W)
        cfg = oracle.config(W, H, bin_size=BIN, sh_degree=0)
        mine = view_shard(len(cams), world, rank)
        imgs = torch.zeros((len(cams), H, W, 4), dtype=torch.uint8)
        for v in mine:
            imgs[v] = torch.from_numpy(oracle.render_frame(cfg, cams[v], g3d, bg)["image"])
        # each view is rendered by exactly one rank: a sum over ranks assembles the batch
        flat = imgs.to(torch.int32)
        dist.all_reduce(flat)
        if rank == 0:
            np.save(out_path, flat.to(torch.uint8).numpy())
    finally:
        dist.destroy_process_group()


def test_multiview_shard_covers_batch_gloo(tmp_path):
    import torch.multiprocessing as mp

    import oracle

    from klartraum_b200 import orbit_views

    out = str(tmp_path / "views.npy")
    mp.start_processes(_view_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    g3d, _ = _scene()
    cams = orbit_views(5, 3.0, W, H, fovy_deg=45.0)
    cfg = oracle.config(W, H, bin_size=BIN, sh_degree=0)
    got = np.load(out)
    for v in range(len(cams)):
        assert np.array_equal(got[v], oracle.render_frame(cfg, cams[v], g3d, background(H, W))["image"])


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 3, 4])
def test_bands_tile_full_frame_gpu(world):
    """Banded renders through the C ABI (one context per band, as ranks would hold) cover the
    full-frame render exactly; balanced on the full frame's per-row pair counts."""
    import torch

    from klartraum_b200 import Renderer, make_scene, native as N, orbit_camera

    w, h = 640, 360
    g3d = make_scene("single_1m", n=60000, seed=5)
    cam = orbit_camera(4.0, w, h, fovy_deg=50.0, azimuth=0.7, elevation=0.25)
    bg = torch.from_numpy(background(h, w, "random")).cuda()
    full = bg.clone()
    r = Renderer(w, h, bin_size=16, sh_degree=3)
    r.set_gaussians(g3d)
    r.render(cam, full)
    torch.cuda.synchronize()
    ty = (h + 15) // 16
    weights = row_pair_counts(r.dump(N.STAGE_TILE_RANGES), (w + 15) // 16, ty)
    r.close()
    for bands in (band_rows(ty, world), band_rows(ty, world, weights)):
        out = torch.zeros_like(bg)
        for b in bands:
            rb = Renderer(w, h, bin_size=16, sh_degree=3, tile_rows=b)
            rb.set_gaussians(g3d)
            strip = bg.clone()
            rb.render(cam, strip)
            torch.cuda.synchronize()
            y0, y1 = band_pixel_rows(b, 16, h)
            out[y0:y1] = strip[y0:y1]
            rb.close()
        assert torch.equal(out, full)
