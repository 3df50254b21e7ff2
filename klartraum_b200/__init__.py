"""B200-native Gaussian-splatting renderer: the hot path behind klartraum's
VulkanGaussianSplatting node (projection -> binning -> sort -> bin ranges -> splatting),
as hand-written sm_100a CUDA kernels behind a C ABI (include/kt_gs.h).
"""

from . import _native as native
from .camera import orbit_camera, orbit_views
from .scenes import WORKLOADS, Workload, make_scene, workload_camera
from .splatting import CameraUBO, GaussianSplattingNode, ImageBuffer, Renderer
from .types import CAMERA_DTYPE, GAUSSIAN2D_DTYPE, GAUSSIAN3D_DTYPE, camera_record, reference_key

__all__ = [
    "native", "orbit_camera", "orbit_views", "WORKLOADS", "Workload", "make_scene", "workload_camera",
    "CameraUBO", "GaussianSplattingNode", "ImageBuffer", "Renderer", "CAMERA_DTYPE", "GAUSSIAN2D_DTYPE",
    "GAUSSIAN3D_DTYPE", "camera_record", "reference_key",
]
