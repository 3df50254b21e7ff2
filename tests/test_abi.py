"""The C ABI library: it loads, exports every entry point include/kt_gs.h declares, and its
structs match the header. No kernel runs here."""

import ctypes as C
import os
import re

import numpy as np
import pytest

from klartraum_b200 import _native as N
from klartraum_b200 import GAUSSIAN2D_DTYPE, GAUSSIAN3D_DTYPE, CAMERA_DTYPE

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not h.endswith(".h"):
            continue
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names += re.findall(r"\b(kt_\w+)\s*\(", src)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    lib = N.load()
    declared = declared_functions()
    assert declared, "no declarations found"
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing
    assert set(N.EXPORTED_SYMBOLS) <= set(declared)


def test_abi_version_and_status_strings():
    lib = N.load()
    assert lib.kt_gs_abi_version() == 3
    for code, name in N.STATUS_NAMES.items():
        assert lib.kt_gs_status_string(code).decode() == name


def test_config_defaults_are_the_reference_constants():
    cfg = N.default_config()
    # src/vulkan_gaussian_splatting.cpp:20-23: 512x512 screen, 4x4 grid of 128-px bins
    assert (cfg.width, cfg.height, cfg.bin_width, cfg.bin_height) == (512, 512, 128, 128)
    assert cfg.cull_z == 1.0 and cfg.sh_degree == 3 and cfg.num_paths == 1


def test_record_sizes_match_header():
    assert GAUSSIAN3D_DTYPE.itemsize == 236
    assert GAUSSIAN2D_DTYPE.itemsize == 48
    assert CAMERA_DTYPE.itemsize == 192
    assert C.sizeof(N.Config) == 48 and C.sizeof(N.Stats) == 96


def test_invalid_configs_are_rejected_before_touching_a_device():
    lib = N.load()
    ctx = C.c_void_p()
    for field, value in [("width", 0), ("bin_width", 24), ("sh_degree", 4), ("num_paths", 0)]:
        cfg = N.default_config()
        setattr(cfg, field, value)
        assert lib.kt_gs_create(C.byref(cfg), 0, C.byref(ctx)) == N.KT_ERR_ARG
    assert lib.kt_gs_create(None, 0, C.byref(ctx)) == N.KT_ERR_ARG


def test_sort_scratch_size_query_needs_no_device():
    size = N.radix_sort_pairs(None, None, None, None, 1 << 20, 45)
    assert size >= (1 << 20) * 12


def test_null_context_calls_fail_cleanly():
    lib = N.load()
    assert lib.kt_gs_render(None, None, None, 0, None) == N.KT_ERR_ARG
    assert lib.kt_gs_destroy(None) == 0
    assert lib.kt_gs_last_error(None) == b"null context"


def test_create_without_gpu_reports_cuda_error():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = N.load()
    cfg = N.default_config()
    ctx = C.c_void_p()
    assert lib.kt_gs_create(C.byref(cfg), 0, C.byref(ctx)) == N.KT_ERR_CUDA
