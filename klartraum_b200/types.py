"""numpy views of the C ABI's records (include/kt_gs.h)."""

from __future__ import annotations

import numpy as np

# klartraum::Gaussian3D (include/klartraum/vulkan_gaussian_splatting_types.hpp:24-33), 236 B
GAUSSIAN3D_DTYPE = np.dtype([
    ("position", "<f4", (3,)),
    ("rotation", "<f4", (4,)),   # x, y, z, w
    ("scale", "<f4", (3,)),      # already exp()'d
    ("color", "<f4", (3,)),      # raw SH DC coefficient
    ("alpha", "<f4"),            # already sigmoid()'ed
    ("shR", "<f4", (15,)),
    ("shG", "<f4", (15,)),
    ("shB", "<f4", (15,)),
])
assert GAUSSIAN3D_DTYPE.itemsize == 236

# GLSL Gaussian2D in scalar layout (shaders/gsplat/gsplat_types.glsl:12-19), 48 B
GAUSSIAN2D_DTYPE = np.dtype([
    ("position", "<f4", (2,)),
    ("z", "<f4"),
    ("binMask", "<u4"),
    ("covInv", "<f4", (4,)),     # column-major [0][0], [0][1], [1][0], [1][1]
    ("color", "<f4", (3,)),
    ("alpha", "<f4"),
])
assert GAUSSIAN2D_DTYPE.itemsize == 48

# CameraMVP (include/klartraum/camera.hpp:44-48): model, view, proj; each column-major 4x4
CAMERA_DTYPE = np.dtype([("model", "<f4", (16,)), ("view", "<f4", (16,)), ("proj", "<f4", (16,))])
assert CAMERA_DTYPE.itemsize == 192


def camera_record(model: np.ndarray, view: np.ndarray, proj: np.ndarray) -> np.ndarray:
    """Pack three 4x4 matrices given as m[col][row] (glm's indexing) into a CameraMVP record."""
    cam = np.zeros((), dtype=CAMERA_DTYPE)
    cam["model"] = np.asarray(model, np.float32).reshape(16)
    cam["view"] = np.asarray(view, np.float32).reshape(16)
    cam["proj"] = np.asarray(proj, np.float32).reshape(16)
    return cam


def reference_key(bins: np.ndarray, z: np.ndarray) -> np.ndarray:
    """bin << 32 | (floatBitsToUint(z) ^ 0x80000000) (gsplat_radix_sort_include.glsl:51-63)."""
    zb = np.asarray(z, np.float32).view(np.uint32) ^ np.uint32(0x80000000)
    return (np.asarray(bins, np.uint64) << np.uint64(32)) | zb.astype(np.uint64)
