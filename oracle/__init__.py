"""CPU oracle for the Gaussian-splatting hot path (TEST INFRASTRUCTURE ONLY).

A ctypes wrapper of ``oracle/libkt_oracle.so``, a plain C restatement of klartraum's gsplat
compute shaders (see kt_oracle.h for the per-stage citations). Only the tests,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` use it, and only as the
checker or the timed CPU baseline - never as part of the renderer.

Parity pinning: the reference's own test expectations (tests/test_gaussian_splatting.cpp)
are checked against this oracle in tests/test_oracle_golden.py; the reference itself cannot
run on these machines (its hot path is Vulkan GLSL).
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libkt_oracle.so")

# same record layouts as the renderer's C ABI
G3D = np.dtype([("position", "<f4", (3,)), ("rotation", "<f4", (4,)), ("scale", "<f4", (3,)),
                ("color", "<f4", (3,)), ("alpha", "<f4"), ("shR", "<f4", (15,)), ("shG", "<f4", (15,)),
                ("shB", "<f4", (15,))])
G2D = np.dtype([("position", "<f4", (2,)), ("z", "<f4"), ("binMask", "<u4"), ("covInv", "<f4", (4,)),
                ("color", "<f4", (3,)), ("alpha", "<f4")])
CAM = np.dtype([("model", "<f4", (16,)), ("view", "<f4", (16,)), ("proj", "<f4", (16,))])


class OracleConfig(C.Structure):
    _fields_ = [("width", C.c_uint32), ("height", C.c_uint32), ("bin_width", C.c_uint32),
                ("bin_height", C.c_uint32), ("sh_degree", C.c_int32), ("cull_z", C.c_float),
                ("exit_per_element", C.c_uint32), ("row_begin", C.c_uint32), ("row_end", C.c_uint32)]


def build() -> str:
    """Compile the oracle with its Makefile (gcc) if needed."""
    src = os.path.join(HERE, "kt_oracle.c")
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(src),
                                                              os.path.getmtime(os.path.join(HERE, "kt_oracle.h"))):
        subprocess.run(["make", "-C", HERE, "ORACLE_CC=gcc"], check=True, capture_output=True)
    return LIB


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB)
        vp, u64, u32 = C.c_void_p, C.c_uint64, C.c_uint32
        cfgp = C.POINTER(OracleConfig)
        sigs = {
            "ko_set_threads": (None, [C.c_int]),
            "ko_get_threads": (C.c_int, []),
            "ko_tiles_x": (u32, [cfgp]),
            "ko_tiles_y": (u32, [cfgp]),
            "ko_project": (None, [cfgp, vp, vp, u64, vp]),
            "ko_tile_counts": (None, [cfgp, vp, u64, vp]),
            "ko_exclusive_scan": (u64, [vp, u64, vp]),
            "ko_emit_keys": (None, [cfgp, vp, u64, vp, vp, vp]),
            "ko_sort_pairs": (None, [vp, vp, u64, u32]),
            "ko_tile_ranges": (None, [vp, u64, u32, vp]),
            "ko_rasterize": (None, [cfgp, vp, vp, vp, vp]),
            "ko_tile_rects": (None, [cfgp, vp, u64, vp]),
            "ko_project_f64": (None, [cfgp, vp, vp, u64, vp]),
            "ko_render_frame_f64": (u64, [cfgp, vp, vp, u64, vp, vp]),
            "ko_render_frame": (u64, [cfgp, vp, vp, u64, vp, vp, vp, vp, vp, vp, u64, vp]),
            "ko_render_projected": (u64, [cfgp, vp, u64, vp, vp, vp, u64, vp]),
        }
        for name, (res, args) in sigs.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def config(width=512, height=512, bin_size=128, sh_degree=3, cull_z=1.0, exit_per_element=False,
           tile_rows=None) -> OracleConfig:
    bw, bh = (bin_size, bin_size) if isinstance(bin_size, int) else bin_size
    rb, re = tile_rows if tile_rows is not None else (0, 0)
    return OracleConfig(width, height, bw, bh, sh_degree, cull_z, int(bool(exit_per_element)), rb, re)


def set_threads(n: int) -> None:
    lib().ko_set_threads(n)


def _p(a: np.ndarray) -> int:
    return a.ctypes.data if a.size else 0


def tiles(cfg: OracleConfig) -> tuple[int, int]:
    return lib().ko_tiles_x(C.byref(cfg)), lib().ko_tiles_y(C.byref(cfg))


def project(cfg, cam, g3d) -> np.ndarray:
    g3d = np.ascontiguousarray(g3d, G3D)
    cam = np.ascontiguousarray(cam, CAM)
    out = np.zeros(len(g3d), G2D)
    lib().ko_project(C.byref(cfg), cam.ctypes.data, _p(g3d), len(g3d), _p(out))
    return out


def tile_counts(cfg, g2d) -> np.ndarray:
    g2d = np.ascontiguousarray(g2d, G2D)
    out = np.zeros(len(g2d), np.uint32)
    lib().ko_tile_counts(C.byref(cfg), _p(g2d), len(g2d), _p(out))
    return out


def exclusive_scan(counts) -> tuple[np.ndarray, int]:
    counts = np.ascontiguousarray(counts, np.uint32)
    out = np.zeros(len(counts), np.uint64)
    total = lib().ko_exclusive_scan(_p(counts), len(counts), _p(out))
    return out, int(total)


def emit_keys(cfg, g2d, offsets, total) -> tuple[np.ndarray, np.ndarray]:
    g2d = np.ascontiguousarray(g2d, G2D)
    offsets = np.ascontiguousarray(offsets, np.uint64)
    keys = np.zeros(total, np.uint64)
    vals = np.zeros(total, np.uint32)
    lib().ko_emit_keys(C.byref(cfg), _p(g2d), len(g2d), _p(offsets), _p(keys), _p(vals))
    return keys, vals


def sort_pairs(keys, vals, key_bits=64) -> tuple[np.ndarray, np.ndarray]:
    keys = np.array(keys, np.uint64, copy=True)
    vals = np.array(vals, np.uint32, copy=True)
    lib().ko_sort_pairs(_p(keys), _p(vals), len(keys), key_bits)
    return keys, vals


def tile_ranges(keys, ntiles) -> np.ndarray:
    keys = np.ascontiguousarray(keys, np.uint64)
    out = np.zeros((ntiles, 2), np.uint32)
    lib().ko_tile_ranges(_p(keys), len(keys), ntiles, out.ctypes.data)
    return out


def rasterize(cfg, g2d, vals, ranges, image) -> np.ndarray:
    g2d = np.ascontiguousarray(g2d, G2D)
    vals = np.ascontiguousarray(vals, np.uint32)
    ranges = np.ascontiguousarray(ranges, np.uint32)
    img = np.array(image, np.uint8, copy=True)
    lib().ko_rasterize(C.byref(cfg), _p(g2d), _p(vals), ranges.ctypes.data, img.ctypes.data)
    return img


G2D_F64 = np.dtype([("position", "<f8", (2,)), ("z", "<f8"), ("covInv", "<f8", (4,)), ("color", "<f8", (3,)),
                    ("alpha", "<f8")])


def tile_rects(cfg, g2d) -> np.ndarray:
    """(x0, x1, y0, y1) bin rectangle per Gaussian, half-open; zeros when culled."""
    g2d = np.ascontiguousarray(g2d, G2D)
    out = np.zeros((len(g2d), 4), np.uint32)
    lib().ko_tile_rects(C.byref(cfg), _p(g2d), len(g2d), out.ctypes.data)
    return out


def project_f64(cfg, cam, g3d) -> np.ndarray:
    g3d = np.ascontiguousarray(g3d, G3D)
    cam = np.ascontiguousarray(cam, CAM)
    out = np.zeros(len(g3d), G2D_F64)
    lib().ko_project_f64(C.byref(cfg), cam.ctypes.data, _p(g3d), len(g3d), _p(out))
    return out


def render_frame_f64(cfg, cam, g3d, image) -> tuple[np.ndarray, int]:
    """Whole frame in double precision; returns (RGBA float64 in [0, 1], pair count)."""
    g3d = np.ascontiguousarray(g3d, G3D)
    cam = np.ascontiguousarray(cam, CAM)
    img = np.ascontiguousarray(image, np.uint8)
    out = np.zeros(img.shape, np.float64)
    k = lib().ko_render_frame_f64(C.byref(cfg), cam.ctypes.data, _p(g3d), len(g3d), img.ctypes.data,
                                  out.ctypes.data)
    if k == 2**64 - 1:
        raise MemoryError("double-precision oracle: allocation failed")
    return out, int(k)


def divergence(img_u8, ref_f64, rows=None) -> dict:
    """Distance of an RGBA8 image from the double-precision image, in units of 1/255:
    max_abs = max |u8 - 255 * ref|, mean_abs, and PSNR against 255 * ref (dB)."""
    a = np.asarray(img_u8, np.float64)
    b = np.asarray(ref_f64, np.float64) * 255.0
    if rows is not None:
        a, b = a[rows[0]:rows[1]], b[rows[0]:rows[1]]
    d = np.abs(a - b)
    mse = float(np.mean(d * d))
    return {"max_abs": float(d.max()) if d.size else 0.0, "mean_abs": float(d.mean()) if d.size else 0.0,
            "psnr_db": float("inf") if mse == 0.0 else float(10.0 * np.log10(255.0 * 255.0 / mse))}


def render_frame(cfg, cam, g3d, image) -> dict:
    """Every stage of one frame; returns the stage buffers and the image."""
    g2d = project(cfg, cam, g3d)
    counts = tile_counts(cfg, g2d)
    offsets, total = exclusive_scan(counts)
    keys_u, vals_u = emit_keys(cfg, g2d, offsets, total)
    tx, ty = tiles(cfg)
    key_bits = 32 + int(tx * ty - 1).bit_length()
    keys, vals = sort_pairs(keys_u, vals_u, key_bits)
    ranges = tile_ranges(keys, tx * ty)
    img = rasterize(cfg, g2d, vals, ranges, image)
    return dict(g2d=g2d, counts=counts, offsets=offsets, num_keys=total, keys_unsorted=keys_u,
                vals_unsorted=vals_u, keys=keys, vals=vals, ranges=ranges, image=img)


def render_frame_fast(cfg, cam, g3d, image) -> tuple[np.ndarray, int]:
    """Whole frame inside C (the timed CPU baseline); returns (image, K)."""
    g3d = np.ascontiguousarray(g3d, G3D)
    cam = np.ascontiguousarray(cam, CAM)
    img = np.array(image, np.uint8, copy=True)
    k = lib().ko_render_frame(C.byref(cfg), cam.ctypes.data, _p(g3d), len(g3d), img.ctypes.data,
                              None, None, None, None, None, 0, None)
    return img, int(k)


def render_projected(cfg, g2d, image) -> dict:
    counts = tile_counts(cfg, g2d)
    offsets, total = exclusive_scan(counts)
    keys_u, vals_u = emit_keys(cfg, g2d, offsets, total)
    tx, ty = tiles(cfg)
    keys, vals = sort_pairs(keys_u, vals_u, 32 + int(tx * ty - 1).bit_length())
    ranges = tile_ranges(keys, tx * ty)
    img = rasterize(cfg, g2d, vals, ranges, image)
    return dict(counts=counts, offsets=offsets, num_keys=total, keys=keys, vals=vals, ranges=ranges, image=img)
