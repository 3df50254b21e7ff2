"""Model of the two-level pair placement (klartraum_b200/csrc/place.cu), run on the CPU.

The kernels are checked on the GPU against the oracle (test_gpu_parity.py). This test checks the
design on its own: the same index arithmetic in Python (coarse bins of 4x4 bins, chunks of depth
order, 32-entry steps numbered in lane order with owner slots found by ballot / OR-reduction, lane
ranks per coarse bin, 4x4 bin masks, segments of the coarse lists, segment prefixes), on random
rectangles, bands of bin rows and ragged grid edges, against a stable sort of the (bin, Gaussian)
pairs by bin: the reference's order (shaders/gsplat/gsplat_radix_sort_include.glsl:51-63 with the
Gaussians already in depth order).
"""

from __future__ import annotations

import numpy as np
import pytest

COARSE = 4


def popc(x: int) -> int:
    return bin(x & 0xFFFFFFFF).count("1")


def span4(lo: int, hi: int) -> int:
    return ((1 << hi) - 1) & ~((1 << lo) - 1)


def divmod_small(a: int, w: int) -> tuple[int, int]:
    inv = np.float32(1) / np.float32(w)
    q = int(np.float32(np.float32(a) * inv))
    if q * w > a:
        q -= 1
    if (q + 1) * w <= a:
        q += 1
    return q, a - q * w


def place(rects, order, tx, row_begin, row_end, chunk_len, band_max=1024, seg_len=512):
    """rects: per depth position (x0, x1, y0, y1) in absolute bins, or None; order: Gaussian index
    per depth position. Returns {bin: [Gaussian, ...]} as the kernels lay the pairs out."""
    n = len(rects)
    rows = row_end - row_begin
    ctx, cty = (tx + 3) // 4, (rows + 3) // 4
    ncoarse = ctx * cty
    br = band_max // ctx
    nbands = (cty + br - 1) // br
    band_rows = (cty + nbands - 1) // nbands
    local = []
    for r in rects:  # clipped to the binned rows, rows relative to row_begin (local_rect)
        if r is None:
            local.append(None)
            continue
        x0, x1, y0, y1 = r
        y0, y1 = max(y0, row_begin), min(y1, row_end)
        local.append(None if (x0 >= x1 or y0 >= y1) else (x0, x1, y0 - row_begin, y1 - row_begin))
    nchunks = (n + chunk_len - 1) // chunk_len
    # k_coarse_count + k_coarse_scan: entries per (chunk, coarse bin), prefixes, list starts
    table = np.zeros((nchunks, ncoarse), np.int64)
    for p, r in enumerate(local):
        if r is None:
            continue
        x0, x1, y0, y1 = r
        for cy in range(y0 // 4, (y1 + 3) // 4):
            for cx in range(x0 // 4, (x1 + 3) // 4):
                table[p // chunk_len, cy * ctx + cx] += 1
    tot = table.sum(0)
    pref = np.cumsum(table, 0) - table
    cstart = np.cumsum(tot) - tot
    clist = [None] * int(tot.sum())
    # k_coarse_place
    for band in range(nbands):
        cb0, cb1 = band * band_rows, min(band * band_rows + band_rows, cty)
        nb, bin0 = (cb1 - cb0) * ctx, cb0 * ctx
        for chunk in range(nchunks):
            cur = [int(pref[chunk, bin0 + i] + cstart[bin0 + i]) for i in range(nb)]
            q0, q1 = chunk * chunk_len, min(chunk * chunk_len + chunk_len, n)
            for qb in range(q0, q1, 32):
                e, first, slots = [0] * 32, [0] * 32, []
                for lane in range(32):
                    q = qb + lane
                    r = local[q] if q < q1 else None
                    if r is not None:
                        x0, x1, y0, y1 = r
                        cy0, cy1 = max(y0 // 4, cb0), min((y1 + 3) // 4, cb1)
                        if cy0 < cy1:
                            e[lane] = ((x1 + 3) // 4 - x0 // 4) * (cy1 - cy0)
                total, acc = sum(e), 0
                for lane in range(32):
                    first[lane] = acc
                    acc += e[lane]
                    if e[lane]:
                        slots.append((first[lane], local[qb + lane], int(order[qb + lane])))
                for t0 in range(0, total, 32):
                    before = sum(1 for j in range(32) if e[j] and first[j] <= t0) - 1
                    starts = 0
                    for j in range(32):
                        if e[j] and t0 < first[j] < t0 + 32:
                            starts |= 1 << (first[j] - t0)
                    step = []
                    for lane in range(32):
                        t = t0 + lane
                        if t >= total:
                            break
                        f0, (x0, x1, y0, y1), g = slots[before + popc(starts & (((2 << lane) & 0xFFFFFFFF) - 1))]
                        cx0, cw = x0 // 4, (x1 + 3) // 4 - x0 // 4
                        dy, dx = divmod_small(t - f0, cw)
                        ccx, ccy = cx0 + dx, max(y0 // 4, cb0) + dy
                        cl = (ccy - cb0) * ctx + ccx
                        assert 0 <= cl < nb
                        bx, by = ccx * 4, ccy * 4
                        cols = span4(max(x0, bx) - bx, min(x1, bx + 4) - bx)
                        rws = span4(max(y0, by) - by, min(y1, by + 4) - by)
                        spread = (rws & 1) | ((rws & 2) << 3) | ((rws & 4) << 6) | ((rws & 8) << 9)
                        step.append((cl, cols * spread, g))
                    seen: dict[int, int] = {}
                    for cl, mask, g in step:  # ranks by lane among equal coarse bins
                        k = seen.get(cl, 0)
                        seen[cl] = k + 1
                        clist[cur[cl] + k] = (g, mask)
                    for cl, k in seen.items():
                        cur[cl] += k
    assert all(x is not None for x in clist)
    # k_fine_count: per segment and bin of the 4x4; totals; ranges
    segs = []  # (coarse bin, e0, e1)
    for c in range(ncoarse):
        for e0 in range(int(cstart[c]), int(cstart[c] + tot[c]), seg_len):
            segs.append((c, e0, min(e0 + seg_len, int(cstart[c] + tot[c]))))
    seg_cnt = [[sum((clist[e][1] >> f) & 1 for e in range(e0, e1)) for f in range(16)] for _, e0, e1 in segs]
    fine_tot = {}
    for (c, _, _), cnt in zip(segs, seg_cnt):
        cy, cx = divmod(c, ctx)
        for f in range(16):
            bx, by = cx * 4 + (f & 3), row_begin + cy * 4 + (f >> 2)
            if cnt[f]:
                assert bx < tx and by < row_end
                fine_tot[by * tx + bx] = fine_tot.get(by * tx + bx, 0) + cnt[f]
    start, acc = {}, 0
    for b in range(row_begin * tx, row_end * tx):
        start[b] = acc
        acc += fine_tot.get(b, 0)
    pairs = [None] * acc
    # k_fine_place: cursors = bin start + earlier segments of the coarse list, ballots per bin
    for si, (c, e0, e1) in enumerate(segs):
        cy, cx = divmod(c, ctx)
        off = []
        for f in range(16):
            bx, by = cx * 4 + (f & 3), row_begin + cy * 4 + (f >> 2)
            earlier = sum(seg_cnt[sj][f] for sj in range(si) if segs[sj][0] == c)
            off.append(start.get(by * tx + bx, 0) + earlier)
        for w0 in range(e0, e1, 32):
            wave = clist[w0:min(w0 + 32, e1)]
            for f in range(16):
                k = 0
                for g, mask in wave:
                    if (mask >> f) & 1:
                        pairs[off[f] + k] = g
                        k += 1
                off[f] += k
    assert all(x is not None for x in pairs)
    out = {}
    for b in range(row_begin * tx, row_end * tx):
        n_b = fine_tot.get(b, 0)
        if n_b:
            out[b] = pairs[start[b]:start[b] + n_b]
    return out


def stable_by_bin(rects, order, tx, row_begin, row_end):
    ref: dict[int, list[int]] = {}
    for p, r in enumerate(rects):
        if r is None:
            continue
        x0, x1, y0, y1 = r
        for y in range(max(y0, row_begin), min(y1, row_end)):
            for x in range(x0, x1):
                ref.setdefault(y * tx + x, []).append(int(order[p]))
    return ref


@pytest.mark.parametrize("tx,ty,rows,n,chunk,band_max", [
    (30, 17, (0, 17), 1500, 256, 1024),    # 1080p-like coarse grid, one band
    (13, 9, (2, 7), 800, 100, 1024),        # a band of bin rows, ragged coarse edges
    (7, 5, (0, 5), 300, 64, 1024),          # tiny grid
    (150, 70, (3, 70), 1200, 512, 1024),    # ctx 38 -> several placement bands
    (40, 40, (0, 40), 900, 128, 40),        # a band per coarse row
])
def test_two_level_placement_is_the_stable_sort_by_bin(tx, ty, rows, n, chunk, band_max):
    rng = np.random.default_rng(tx * 1000 + n)
    rects = []
    for _ in range(n):
        if rng.random() < 0.1:
            rects.append(None)  # culled: no bins
            continue
        x0 = int(rng.integers(0, tx))
        y0 = int(rng.integers(0, ty))
        big = rng.random() < 0.03
        w = int(rng.integers(1, 40 if big else 9))
        h = int(rng.integers(1, 30 if big else 7))
        rects.append((x0, min(x0 + w, tx), y0, min(y0 + h, ty)))
    order = rng.permutation(n)  # Gaussian index of each depth position
    got = place(rects, order, tx, rows[0], rows[1], chunk, band_max=band_max, seg_len=64)
    assert got == stable_by_bin(rects, order, tx, rows[0], rows[1])


def test_owner_slots_match_a_search_over_first_entries():
    """The owner of entry t in a 32-entry step: slots starting at or before the step (minus one)
    plus the slots starting inside it up to t; the same lane as a search over first entries."""
    rng = np.random.default_rng(7)
    for _ in range(3000):
        e = rng.integers(0, 6, 32) * (rng.random(32) < rng.random())
        if rng.random() < 0.1:
            e[rng.integers(0, 32)] = rng.integers(20, 200)
        first = np.cumsum(e) - e
        total = int(e.sum())
        nonempty = [j for j in range(32) if e[j]]
        for t0 in range(0, total, 32):
            before = sum(1 for j in range(32) if e[j] and first[j] <= t0) - 1
            starts = sum(1 << int(first[j] - t0) for j in range(32) if e[j] and t0 < first[j] < t0 + 32)
            for lane in range(min(32, total - t0)):
                t = t0 + lane
                slot = before + popc(starts & (((2 << lane) & 0xFFFFFFFF) - 1))
                owner = max(j for j in range(32) if e[j] and first[j] <= t)
                assert nonempty[slot] == owner
