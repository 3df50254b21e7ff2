"""Work sharding across the GPUs of one box: one process per GPU (``torch.distributed``).

Two splits, both without communication inside a frame's compute:

* multi-view: views are independent; rank r renders views r, r + N, r + 2N, ... of a batch,
  each with the full (replicated) scene. The only collective is an optional gather of images.
* banded: one large frame is split into horizontal bands of bin rows; every rank projects the
  whole scene but bins and draws only its band (``kt_gs_config.tile_row_begin/end``), so the
  bands together are exactly the full frame. One exchange step gathers the strips (NCCL over
  NVLink on GPUs, gloo on CPU). Band boundaries can follow the per-row pair counts of the
  previous frame so that every rank gets a similar amount of work.
"""

from __future__ import annotations

import numpy as np


def view_shard(n_views: int, world: int, rank: int) -> list[int]:
    """Views rendered by `rank`: round-robin, so the counts differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    return list(range(rank, n_views, world))


def band_rows(tiles_y: int, world: int, weights=None) -> list[tuple[int, int]]:
    """Split bin rows [0, tiles_y) into `world` contiguous bands [y0, y1).

    Without weights the bands have equal row counts (+-1). With per-row weights (e.g. the pairs
    per bin row of the previous frame) the cuts put about the same total weight in every band;
    every band keeps at least one row when tiles_y >= world.
    """
    if world <= 0:
        raise ValueError("world must be positive")
    if weights is None:
        cuts = [(tiles_y * k) // world for k in range(world + 1)]
    else:
        w = np.asarray(weights, dtype=np.float64)
        if w.shape != (tiles_y,):
            raise ValueError("one weight per bin row")
        w = np.maximum(w, 0.0) + 1e-9  # empty rows still count a little
        c = np.concatenate([[0.0], np.cumsum(w)])
        cuts = [0]
        for k in range(1, world):
            target = c[-1] * k / world
            y = int(np.searchsorted(c, target))
            lo = cuts[-1] + 1 if tiles_y >= world else cuts[-1]
            hi = tiles_y - (world - k) if tiles_y >= world else tiles_y
            cuts.append(min(max(y, lo), hi))
        cuts.append(tiles_y)
    return [(cuts[k], cuts[k + 1]) for k in range(world)]


def rebalance_bands(row_weights, bands: list[tuple[int, int]], band_ms) -> list[tuple[int, int]]:
    """New cuts from the measured time of each band: the rows of band k are weighted by
    band_ms[k] / (its summed row weight), i.e. by the measured cost per unit of weight of the rank
    that drew them, and the rows are split again so that every band gets the same predicted
    time. With per-row pair counts as weights this balances on time, not on pairs."""
    w = np.asarray(row_weights, dtype=np.float64)
    t = np.asarray(band_ms, dtype=np.float64)
    if len(t) != len(bands):
        raise ValueError("one time per band")
    scale = np.ones_like(w)
    for k, (y0, y1) in enumerate(bands):
        total = w[y0:y1].sum()
        scale[y0:y1] = t[k] / total if total > 0 else 0.0
    return band_rows(len(w), len(bands), w * scale)


def band_pixel_rows(band: tuple[int, int], bin_h: int, height: int) -> tuple[int, int]:
    """Pixel rows [r0, r1) covered by a band of bin rows."""
    y0, y1 = band
    return min(y0 * bin_h, height), min(y1 * bin_h, height)


def gather_strips(strip, band_px: list[tuple[int, int]], width: int, height: int, dist, rank: int,
                  device=None):
    """All-gather the ranks' image strips (uint8 H_band x W x 4 tensors) into the full frame.

    Strips are padded to the tallest band so that one all_gather moves them (the collective
    wants equal sizes); every rank receives the assembled frame. `dist` is torch.distributed
    (NCCL for CUDA tensors, gloo for CPU tensors).
    """
    import torch

    world = len(band_px)
    tallest = max(r1 - r0 for r0, r1 in band_px)
    pad = torch.zeros((tallest, width, 4), dtype=torch.uint8, device=device)
    r0, r1 = band_px[rank]
    if tuple(strip.shape) != (r1 - r0, width, 4):
        raise ValueError(f"strip of rank {rank} is {tuple(strip.shape)}, band needs {(r1 - r0, width, 4)}")
    pad[: r1 - r0] = strip
    out = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(out, pad)
    frame = torch.empty((height, width, 4), dtype=torch.uint8, device=device)
    for k, (a, b) in enumerate(band_px):
        frame[a:b] = out[k][: b - a]
    return frame


def row_pair_counts(ranges: np.ndarray, tiles_x: int, tiles_y: int) -> np.ndarray:
    """Pairs per bin row from a frame's bin ranges ({start, end} per bin), for balancing."""
    r = np.asarray(ranges, dtype=np.int64).reshape(tiles_y, tiles_x, 2)
    return (r[..., 1] - r[..., 0]).sum(axis=1)


class StripGather:
    """Preallocated all-gather of band strips into the full frame, for a frame loop.

    `__call__(img)` takes this rank's full-size H x W x 4 image whose band rows are rendered and
    returns the assembled frame (a buffer reused by every call). NCCL moves the padded strips in
    one all_gather_into_tensor; other backends use the list form.
    """

    def __init__(self, band_px: list[tuple[int, int]], width: int, height: int, dist, rank: int, device=None):
        import torch

        self.band_px, self.dist, self.rank = band_px, dist, rank
        self.world = len(band_px)
        self.tallest = max(max(r1 - r0 for r0, r1 in band_px), 1)
        self.pad = torch.zeros((self.tallest, width, 4), dtype=torch.uint8, device=device)
        self.out = torch.empty((self.world, self.tallest, width, 4), dtype=torch.uint8, device=device)
        self.frame = torch.empty((height, width, 4), dtype=torch.uint8, device=device)
        self.fused = dist.get_backend() == "nccl"

    @property
    def bytes_per_frame(self) -> int:
        """Bytes each rank receives per frame (the padded strips of all ranks)."""
        return self.out.numel()

    def __call__(self, img):
        r0, r1 = self.band_px[self.rank]
        self.pad[: r1 - r0].copy_(img[r0:r1])
        if self.fused:
            self.dist.all_gather_into_tensor(self.out, self.pad)
        else:
            self.dist.all_gather(list(self.out.unbind(0)), self.pad)
        for k, (a, b) in enumerate(self.band_px):
            self.frame[a:b].copy_(self.out[k, : b - a])
        return self.frame


def broadcast_scene(g3d, dist, rank: int, device):
    """Rank 0's Gaussian3D records (numpy, 236 B each) as a device byte tensor on every rank.

    One broadcast at scene load replaces a per-rank file read; the renderer then takes the records
    from device memory (kt_gs_set_gaussians_device). Returns (tensor, n)."""
    import torch

    meta = torch.zeros(2, dtype=torch.int64, device=device)
    if rank == 0:
        meta[0], meta[1] = len(g3d), g3d.dtype.itemsize
    dist.broadcast(meta, 0)
    n, rec = int(meta[0].item()), int(meta[1].item())
    buf = torch.empty(n * rec, dtype=torch.uint8, device=device)
    if rank == 0:
        buf.copy_(torch.from_numpy(np.ascontiguousarray(g3d).view(np.uint8).reshape(-1)))
    dist.broadcast(buf, 0)
    return buf, n
