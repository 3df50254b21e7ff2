"""Python mirror of klartraum's ``VulkanGaussianSplatting`` graph node over the C ABI.

Reference interface (include/klartraum/vulkan_gaussian_splatting.hpp:23-83,
src/vulkan_gaussian_splatting.cpp:13-316):

* the node is constructed with an image source (input slot 0), a camera UBO (slot 1) and a
  scene; ``checkInput`` raises on a wrong input type or a slot index above 1;
* ``_setup(numberPaths)`` prepares per-path state; ``_record(commandBuffer, pathId)`` records
  the frame for one path; ``getType()`` is ``"GaussianSplatting"``.

Here the "command buffer" is a CUDA stream, the image source is a headless RGBA8 device
buffer per path and the camera UBO is a host CameraMVP per path. :class:`Renderer` is the
thin wrapper of one ``kt_gs_ctx``; :class:`GaussianSplattingNode` adds the node interface.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from .types import CAMERA_DTYPE, GAUSSIAN2D_DTYPE, GAUSSIAN3D_DTYPE


class Renderer:
    """One renderer context (``kt_gs_ctx``) on one CUDA device."""

    def __init__(self, width: int = 512, height: int = 512, *, bin_size: int | tuple = 128,
                 sh_degree: int = 3, cull_z: float = 1.0, flags: int = 0, num_paths: int = 1,
                 key_capacity: int = 0, tile_rows: tuple | None = None, device: int = 0):
        self._lib = N.load()
        cfg = N.default_config()
        cfg.width, cfg.height = width, height
        bw, bh = (bin_size, bin_size) if isinstance(bin_size, int) else bin_size
        cfg.bin_width, cfg.bin_height = bw, bh
        cfg.sh_degree = sh_degree
        cfg.cull_z = cull_z
        cfg.flags = flags
        cfg.num_paths = num_paths
        cfg.key_capacity = key_capacity
        if tile_rows is not None:
            cfg.tile_row_begin, cfg.tile_row_end = tile_rows
        self.config = cfg
        self._flags = flags
        ctx = C.c_void_p()
        N.check(self._lib.kt_gs_create(C.byref(cfg), device, C.byref(ctx)))
        self._ctx = ctx
        self.width, self.height = width, height
        self.device = device

    # ------------------------------------------------------------------ lifetime
    def close(self) -> None:
        if getattr(self, "_ctx", None):
            self._lib.kt_gs_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, status: int) -> None:
        N.check(status, self._ctx)

    # ---------------------------------------------------------------- scene
    def set_gaussians(self, g: np.ndarray) -> None:
        g = np.ascontiguousarray(g, dtype=GAUSSIAN3D_DTYPE)
        self._check(self._lib.kt_gs_set_gaussians(self._ctx, g.ctypes.data, len(g)))

    def set_gaussians_device(self, dev_ptr: int, n: int, stream: int = 0) -> None:
        self._check(self._lib.kt_gs_set_gaussians_device(self._ctx, dev_ptr, n, stream or None))

    def load_spz(self, path: str) -> None:
        self._check(self._lib.kt_gs_load_spz(self._ctx, path.encode()))

    def load_ply(self, path: str) -> None:
        self._check(self._lib.kt_gs_load_ply(self._ctx, path.encode()))

    @property
    def sh_degree(self) -> int:
        cfg = N.Config()
        self._check(self._lib.kt_gs_get_config(self._ctx, C.byref(cfg)))
        return cfg.sh_degree

    # ---------------------------------------------------------------- frames
    @staticmethod
    def _cam(cam: np.ndarray) -> np.ndarray:
        cam = np.ascontiguousarray(cam, dtype=CAMERA_DTYPE)
        assert cam.size == 1 or cam.ndim >= 1
        return cam

    def render(self, cam: np.ndarray, image, path: int = 0, stream: int = 0) -> None:
        """Render into a device RGBA8 image (torch tensor or device address)."""
        cam = self._cam(cam)
        self._check(self._lib.kt_gs_render(self._ctx, cam.ctypes.data, N.as_ptr(image), path, stream or None))

    def render_host(self, cam: np.ndarray, image, path: int = 0, stream: int = 0):
        """Render into a host RGBA8 image (H x W x 4 uint8 numpy array, pinned torch tensor or
        host address), in place; returns it."""
        if isinstance(image, np.ndarray):
            assert image.dtype == np.uint8 and image.flags.c_contiguous
            assert image.size == self.width * self.height * 4
        cam = self._cam(cam)
        self._check(self._lib.kt_gs_render_host(self._ctx, cam.ctypes.data, N.as_ptr(image), path, stream or None))
        return image

    def render_host_clear(self, cam: np.ndarray, image, clear=(0, 0, 0, 255), path: int = 0, stream: int = 0):
        """Render into a host RGBA8 image with the device image first cleared to `clear` (the
        render pass's clear colour) instead of copied in; returns the image."""
        if isinstance(image, np.ndarray):
            assert image.dtype == np.uint8 and image.flags.c_contiguous
            assert image.size == self.width * self.height * 4
        cam = self._cam(cam)
        col = (C.c_uint8 * 4)(*[int(v) for v in clear])
        self._check(self._lib.kt_gs_render_host_clear(self._ctx, cam.ctypes.data, col, N.as_ptr(image), path,
                                                      stream or None))
        return image

    def render_batch(self, cams: np.ndarray, images: list, stream: int = 0) -> None:
        cams = np.ascontiguousarray(cams, dtype=CAMERA_DTYPE)
        ptrs = (C.c_void_p * len(images))(*[N.as_ptr(i) for i in images])
        self._check(self._lib.kt_gs_render_batch(self._ctx, cams.ctypes.data, len(images), ptrs, stream or None))

    def render_projected(self, g2d: np.ndarray, image, path: int = 0, stream: int = 0) -> None:
        g2d = np.ascontiguousarray(g2d, dtype=GAUSSIAN2D_DTYPE)
        self._check(self._lib.kt_gs_render_projected(self._ctx, g2d.ctypes.data, len(g2d), N.as_ptr(image),
                                                     path, stream or None))

    def set_flags(self, flags: int) -> None:
        self._check(self._lib.kt_gs_set_flags(self._ctx, flags))
        self.config.flags = flags
        self._flags = flags

    @property
    def stage_names(self) -> list:
        """Names of the stage timer slots for the binning path the flags select."""
        return N.STAGE_NAMES_KEYS if self._flags & N.FLAG_SORTED_KEYS else N.STAGE_NAMES

    def counters(self, path: int = 0) -> dict:
        """Frame totals accumulated on the device since the previous call (then reset)."""
        c = N.Counters()
        self._check(self._lib.kt_gs_counters_take(self._ctx, path, C.byref(c)))
        return c.as_dict()

    def sync(self, path: int = 0) -> None:
        self._check(self._lib.kt_gs_sync(self._ctx, path))

    # ------------------------------------------------------------- inspection
    def stats(self, path: int = 0) -> dict:
        s = N.Stats()
        self._check(self._lib.kt_gs_frame_stats(self._ctx, path, C.byref(s)))
        return s.as_dict()

    def stage_times(self, path: int = 0) -> dict:
        ms = (C.c_float * N.NSTAGES)()
        self._check(self._lib.kt_gs_stage_times(self._ctx, path, ms))
        return dict(zip(self.stage_names, list(ms)))

    def stage_times_total(self, path: int = 0) -> tuple[dict, int]:
        """Summed stage milliseconds of all timed frames since the last call, and their count."""
        ms = (C.c_double * N.NSTAGES)()
        frames = C.c_uint64(0)
        self._check(self._lib.kt_gs_stage_times_total(self._ctx, path, ms, C.byref(frames)))
        return dict(zip(self.stage_names, list(ms))), frames.value

    _STAGE_DTYPES = {
        N.STAGE_PROJECTED: GAUSSIAN2D_DTYPE,
        N.STAGE_TILE_COUNTS: np.dtype(np.uint32),
        N.STAGE_OFFSETS: np.dtype(np.uint64),
        N.STAGE_KEYS_UNSORTED: np.dtype(np.uint64),
        N.STAGE_VALUES_UNSORTED: np.dtype(np.uint32),
        N.STAGE_KEYS_SORTED: np.dtype(np.uint64),
        N.STAGE_VALUES_SORTED: np.dtype(np.uint32),
        N.STAGE_TILE_RANGES: np.dtype(np.uint32),
        N.STAGE_DEPTH_ORDER: np.dtype(np.uint32),
        N.STAGE_COARSE_INFO: np.dtype(np.uint32),
        N.STAGE_COARSE_LISTS: np.dtype(np.uint32),
        N.STAGE_SEGMENT_COUNTS: np.dtype(np.uint32),
    }
    # u32 words per element of the stages whose elements are small records
    _STAGE_WIDTH = {N.STAGE_TILE_RANGES: 2, N.STAGE_COARSE_INFO: 4, N.STAGE_COARSE_LISTS: 2,
                    N.STAGE_SEGMENT_COUNTS: 16}

    def dump(self, stage: int, path: int = 0, first: int = 0, count: int | None = None) -> np.ndarray:
        """A stage buffer of the last frame on `path` (kt_gs_debug_dump), or elements
        [first, first + count) of it (kt_gs_debug_dump_range)."""
        need = C.c_uint64(0)
        whole = first == 0 and count is None
        cnt = (1 << 64) - 1 if count is None else count

        def call(ptr, nbytes, out_len):
            if whole:
                return self._lib.kt_gs_debug_dump(self._ctx, path, stage, ptr, nbytes, out_len)
            return self._lib.kt_gs_debug_dump_range(self._ctx, path, stage, first, cnt, ptr, nbytes, out_len)

        self._check(call(None, 0, C.byref(need)))
        dt = self._STAGE_DTYPES[stage]
        out = np.zeros(need.value // dt.itemsize, dtype=dt)
        wrote = C.c_uint64(0)
        self._check(call(out.ctypes.data if out.size else None, out.nbytes, C.byref(wrote)))
        if stage in self._STAGE_WIDTH:
            out = out.reshape(-1, self._STAGE_WIDTH[stage])
        return out


class CameraUBO:
    """Per-path host CameraMVP, the counterpart of ``UniformBufferObject<CameraMVP>``
    (include/klartraum/computegraph/uniformbufferobject.hpp:22-199)."""

    def __init__(self, num_paths: int = 1):
        self.ubo = np.zeros((), dtype=CAMERA_DTYPE)
        self._paths = np.zeros(num_paths, dtype=CAMERA_DTYPE)

    def update(self, path: int) -> None:
        self._paths[path] = self.ubo

    def get(self, path: int) -> np.ndarray:
        return self._paths[path]

    def get_type(self) -> str:
        return "UniformBufferObject"


class ImageBuffer:
    """Headless RGBA8 image per path (what ImageViewSrc provides in the reference,
    include/klartraum/computegraph/imageviewsrc.hpp:13-55); device tensors, cleared to
    (0,0,0,1) like the reference's render pass (renderpass.hpp:170)."""

    def __init__(self, width: int, height: int, num_paths: int = 1, device: int = 0):
        import torch

        self.width, self.height = width, height
        self.images = [torch.zeros((height, width, 4), dtype=torch.uint8, device=f"cuda:{device}")
                       for _ in range(num_paths)]
        for im in self.images:
            im[..., 3] = 255

    def get_image(self, path: int):
        return self.images[path]

    def get_type(self) -> str:
        return "ImageViewSrc"


class GaussianSplattingNode:
    """Graph-node view of the renderer: input 0 = ImageBuffer, input 1 = CameraUBO."""

    def __init__(self, image: ImageBuffer, camera: CameraUBO, gaussians: np.ndarray | str, **cfg):
        self.inputs: dict[int, object] = {}
        self.set_input(image, 0)
        self.set_input(camera, 1)
        self._cfg = dict(cfg)
        self._scene = gaussians
        self.renderer = self._make_renderer(self._cfg.pop("num_paths", 1))
        self.number_of_paths = 0

    def _make_renderer(self, num_paths: int) -> Renderer:
        image = self.inputs[0]
        r = Renderer(image.width, image.height, num_paths=num_paths, **self._cfg)
        if isinstance(self._scene, str):
            r.load_spz(self._scene)
        else:
            r.set_gaussians(self._scene)
        return r

    def check_input(self, inp, index: int = 0) -> None:
        # src/vulkan_gaussian_splatting.cpp:220-232
        if index == 0 and not isinstance(inp, ImageBuffer):
            raise RuntimeError("input is not an ImageViewSrc!")
        if index == 1 and not isinstance(inp, CameraUBO):
            raise RuntimeError("input is not a CameraUboType!")
        if index > 1:
            raise RuntimeError("input index out of range!")

    def set_input(self, inp, index: int = 0) -> None:
        self.check_input(inp, index)
        self.inputs[index] = inp

    def setup(self, number_paths: int) -> None:
        """_setup(ctx, numberPaths) (src/vulkan_gaussian_splatting.cpp:234-236): one renderer path
        (its own device workspace) per graph path, so paths can be in flight together."""
        if number_paths > self.renderer.config.num_paths:
            self.renderer.close()
            self.renderer = self._make_renderer(number_paths)
        self.number_of_paths = number_paths

    def record(self, stream: int, path: int) -> None:
        """Enqueue the frame of `path` on `stream` (the reference records a command buffer)."""
        if path >= max(self.number_of_paths, 1):
            raise RuntimeError("path index out of range!")
        image, camera = self.inputs[0], self.inputs[1]
        self.renderer.render(camera.get(path), image.get_image(path), path=path, stream=stream)

    def get_type(self) -> str:
        return "GaussianSplatting"
