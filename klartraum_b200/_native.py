"""ctypes binding of ``libkt_gs.so`` (the C ABI declared in include/kt_gs.h).

The library is the only compute path: importing this module fails loudly when it has not
been built (``python -m klartraum_b200.build``); there is no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
import os

import numpy as np

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libkt_gs.so")

KT_OK = 0
STATUS_NAMES = {
    0: "KT_OK", 1: "KT_ERR_ARG", 2: "KT_ERR_CUDA", 3: "KT_ERR_CAPACITY", 4: "KT_ERR_TIMEOUT",
    5: "KT_ERR_NCCL", 6: "KT_ERR_IO", 7: "KT_ERR_STATE", 8: "KT_ERR_NOMEM",
}
KT_ERR_ARG, KT_ERR_CUDA, KT_ERR_CAPACITY, KT_ERR_TIMEOUT = 1, 2, 3, 4
KT_ERR_NCCL, KT_ERR_IO, KT_ERR_STATE, KT_ERR_NOMEM = 5, 6, 7, 8

FLAG_EXIT_PER_ELEMENT = 0x1
FLAG_NO_AUTOGROW = 0x2
FLAG_ASYNC = 0x4
FLAG_KEEP_UNSORTED = 0x8
FLAG_TIMING = 0x10
FLAG_SORTED_KEYS = 0x20
FLAG_GRAPH = 0x40

STAGE_PROJECTED = 0
STAGE_TILE_COUNTS = 1
STAGE_OFFSETS = 2
STAGE_KEYS_UNSORTED = 3
STAGE_VALUES_UNSORTED = 4
STAGE_KEYS_SORTED = 5
STAGE_VALUES_SORTED = 6
STAGE_TILE_RANGES = 7
STAGE_DEPTH_ORDER = 8
STAGE_COARSE_INFO = 9
STAGE_COARSE_LISTS = 10
STAGE_SEGMENT_COUNTS = 11
# dumps of the default binning path that are rebuilt on the host (no device buffer holds them)
HOST_REBUILT_STAGES = (STAGE_OFFSETS, STAGE_KEYS_UNSORTED, STAGE_VALUES_UNSORTED)
NSTAGES = 7
STAGE_NAMES = ["project_count", "depth_sort", "coarse_count", "coarse_place", "fine_place", "rasterize", "frame"]
# the same timer slots when KT_GS_FLAG_SORTED_KEYS selects the reference-structured binning
STAGE_NAMES_KEYS = ["project_count", "scan_emit", "key_sort", "bin_ranges", "totals", "rasterize", "frame"]

# every entry point include/kt_gs.h declares
EXPORTED_SYMBOLS = [
    "kt_gs_config_default", "kt_gs_abi_version", "kt_gs_status_string", "kt_gs_create",
    "kt_gs_destroy", "kt_gs_last_error", "kt_gs_get_config", "kt_gs_set_gaussians",
    "kt_gs_set_gaussians_device", "kt_gs_load_spz", "kt_gs_render", "kt_gs_render_host",
    "kt_gs_render_batch", "kt_gs_render_projected", "kt_gs_sync", "kt_gs_frame_stats",
    "kt_gs_debug_dump", "kt_gs_stage_times", "kt_gs_stage_times_total", "kt_gs_radix_sort_pairs",
    "kt_gs_set_flags", "kt_gs_counters_take", "kt_gs_spz_decode", "kt_gs_load_ply", "kt_gs_ply_decode",
    "kt_gs_debug_dump_range", "kt_gs_radix_sort_pairs_static", "kt_gs_radix_sort_status",
    "kt_gs_radix_sort_static_timeout_probe", "kt_gs_render_host_clear",
]


class KtError(RuntimeError):
    """A non-OK kt_status (the reference raises std::runtime_error on the same conditions)."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


class Config(C.Structure):
    _fields_ = [
        ("width", C.c_uint32), ("height", C.c_uint32),
        ("bin_width", C.c_uint32), ("bin_height", C.c_uint32),
        ("sh_degree", C.c_int32), ("cull_z", C.c_float),
        ("flags", C.c_uint32), ("num_paths", C.c_uint32),
        ("key_capacity", C.c_uint64),
        ("tile_row_begin", C.c_uint32), ("tile_row_end", C.c_uint32),
    ]


class Stats(C.Structure):
    _fields_ = [
        ("num_gaussians", C.c_uint64), ("num_keys", C.c_uint64),
        ("key_capacity", C.c_uint64), ("num_visible", C.c_uint64),
        ("tiles_x", C.c_uint32), ("tiles_y", C.c_uint32),
        ("key_bits", C.c_uint32), ("depth_bits", C.c_uint32),
        ("sort_passes", C.c_uint32), ("error_flags", C.c_uint32),
        ("depth_min_bits", C.c_uint32), ("depth_max_bits", C.c_uint32),
        ("status_bytes", C.c_uint32), ("launches", C.c_uint32),
        ("packed", C.c_uint32), ("idx_bits", C.c_uint32),
        ("place_chunks", C.c_uint32), ("place_bands", C.c_uint32),
        ("place_runs", C.c_uint32),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class Counters(C.Structure):
    _fields_ = [("frames", C.c_uint64), ("keys", C.c_uint64), ("key_passes", C.c_uint64),
                ("visible", C.c_uint64), ("sort_bytes", C.c_uint64), ("depth_sort_bytes", C.c_uint64)]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


assert C.sizeof(Config) == 48
assert C.sizeof(Stats) == 96
assert C.sizeof(Counters) == 48

_lib = None


def lib_path() -> str:
    return _LIB_PATH


def load() -> C.CDLL:
    """Load the renderer library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        raise RuntimeError(f"{_LIB_PATH} is missing; build it with `python -m klartraum_b200.build`")
    lib = C.CDLL(_LIB_PATH)
    vp, u32, u64, i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int32
    sig = {
        "kt_gs_config_default": (None, [C.POINTER(Config)]),
        "kt_gs_abi_version": (C.c_int, []),
        "kt_gs_status_string": (C.c_char_p, [C.c_int]),
        "kt_gs_create": (C.c_int, [C.POINTER(Config), C.c_int, C.POINTER(vp)]),
        "kt_gs_destroy": (C.c_int, [vp]),
        "kt_gs_last_error": (C.c_char_p, [vp]),
        "kt_gs_get_config": (C.c_int, [vp, C.POINTER(Config)]),
        "kt_gs_set_gaussians": (C.c_int, [vp, vp, u64]),
        "kt_gs_set_gaussians_device": (C.c_int, [vp, vp, u64, vp]),
        "kt_gs_load_spz": (C.c_int, [vp, C.c_char_p]),
        "kt_gs_spz_decode": (C.c_int, [C.c_char_p, vp, C.c_uint64, C.POINTER(C.c_uint64), C.POINTER(u32)]),
        "kt_gs_load_ply": (C.c_int, [vp, C.c_char_p]),
        "kt_gs_ply_decode": (C.c_int, [C.c_char_p, vp, C.c_uint64, C.POINTER(C.c_uint64)]),
        "kt_gs_render": (C.c_int, [vp, vp, vp, u32, vp]),
        "kt_gs_render_host": (C.c_int, [vp, vp, vp, u32, vp]),
        "kt_gs_render_host_clear": (C.c_int, [vp, vp, C.POINTER(C.c_uint8), vp, u32, vp]),
        "kt_gs_render_batch": (C.c_int, [vp, vp, u32, vp, vp]),
        "kt_gs_render_projected": (C.c_int, [vp, vp, u64, vp, u32, vp]),
        "kt_gs_sync": (C.c_int, [vp, u32]),
        "kt_gs_frame_stats": (C.c_int, [vp, u32, C.POINTER(Stats)]),
        "kt_gs_debug_dump": (C.c_int, [vp, u32, C.c_int, vp, u64, C.POINTER(u64)]),
        "kt_gs_debug_dump_range": (C.c_int, [vp, u32, C.c_int, u64, u64, vp, u64, C.POINTER(u64)]),
        "kt_gs_stage_times": (C.c_int, [vp, u32, C.POINTER(C.c_float)]),
        "kt_gs_stage_times_total": (C.c_int, [vp, u32, C.POINTER(C.c_double), C.POINTER(u64)]),
        "kt_gs_radix_sort_pairs": (C.c_int, [vp, vp, vp, vp, u64, u32, vp, C.POINTER(C.c_size_t), vp]),
        "kt_gs_radix_sort_pairs_static": (C.c_int, [vp, vp, vp, vp, u64, u32, vp]),
        "kt_gs_radix_sort_status": (C.c_int, [vp, vp]),
        "kt_gs_radix_sort_static_timeout_probe": (C.c_int, [u32, vp]),
        "kt_gs_set_flags": (C.c_int, [vp, u32]),
        "kt_gs_counters_take": (C.c_int, [vp, u32, C.POINTER(Counters)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    del i32
    _lib = lib
    return lib


def default_config() -> Config:
    cfg = Config()
    load().kt_gs_config_default(C.byref(cfg))
    return cfg


def check(status: int, ctx=None) -> None:
    if status != KT_OK:
        msg = ""
        if ctx:
            raw = load().kt_gs_last_error(ctx)
            msg = raw.decode() if raw else ""
        raise KtError(status, msg)


def as_ptr(a) -> int:
    """Address of a numpy array, a torch tensor or an int."""
    if a is None:
        return 0
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    raise TypeError(f"cannot take the address of {type(a)}")


def radix_sort_pairs(keys_in, vals_in, keys_out, vals_out, n: int, key_bits: int, temp=None,
                     stream: int = 0) -> int:
    """kt_gs_radix_sort_pairs; returns the scratch size when temp is None."""
    lib = load()
    size = C.c_size_t(0)
    if temp is None:
        check(lib.kt_gs_radix_sort_pairs(None, None, None, None, n, key_bits, None, C.byref(size), None))
        return size.value
    size.value = temp.numel() if hasattr(temp, "numel") else int(temp.nbytes)
    check(lib.kt_gs_radix_sort_pairs(as_ptr(keys_in), as_ptr(vals_in), as_ptr(keys_out), as_ptr(vals_out),
                                     n, key_bits, as_ptr(temp), C.byref(size), stream or None))
    return size.value


def spz_decode(path: str):
    """Decode an .spz file on the host (kt_gs_spz_decode): (Gaussian3D records, SH degree)."""
    import numpy as np

    from .types import GAUSSIAN3D_DTYPE

    lib = load()
    n, deg = C.c_uint64(0), C.c_uint32(0)
    check(lib.kt_gs_spz_decode(path.encode(), None, 0, C.byref(n), C.byref(deg)))
    out = np.zeros(n.value, GAUSSIAN3D_DTYPE)
    if n.value:
        check(lib.kt_gs_spz_decode(path.encode(), out.ctypes.data, n.value, C.byref(n), C.byref(deg)))
    return out, deg.value


def ply_decode(path: str):
    """Decode a 3D Gaussian Splatting .ply file on the host (kt_gs_ply_decode)."""
    import numpy as np

    from .types import GAUSSIAN3D_DTYPE

    lib = load()
    n = C.c_uint64(0)
    check(lib.kt_gs_ply_decode(path.encode(), None, 0, C.byref(n)))
    out = np.zeros(n.value, GAUSSIAN3D_DTYPE)
    if n.value:
        check(lib.kt_gs_ply_decode(path.encode(), out.ctypes.data, n.value, C.byref(n)))
    return out
