"""The Python mirror of klartraum's VulkanGaussianSplatting node (klartraum_b200.splatting):
input slots and checkInput's errors (src/vulkan_gaussian_splatting.cpp:220-232), _setup's path
count (:234-236), and frames recorded per path equal to Renderer.render's frames."""

import numpy as np
import pytest

from klartraum_b200 import Renderer, make_scene, orbit_views
from klartraum_b200.splatting import CameraUBO, GaussianSplattingNode, ImageBuffer

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def test_node_records_the_renderers_frames_on_two_paths():
    g3d = make_scene("plumbing", n=6000)
    cams = orbit_views(4, 1.5, 256, 256)
    image = ImageBuffer(256, 256, num_paths=2)
    camera = CameraUBO(num_paths=2)
    node = GaussianSplattingNode(image, camera, g3d, bin_size=16, sh_degree=0)
    assert node.get_type() == "GaussianSplatting"
    node.setup(2)
    assert node.renderer.config.num_paths == 2
    streams = [torch.cuda.Stream() for _ in range(2)]
    ref = Renderer(256, 256, bin_size=16, sh_degree=0)
    ref.set_gaussians(g3d)
    for frame in range(4):
        path = frame % 2
        camera.ubo = cams[frame]
        camera.update(path)
        image.get_image(path)[:] = 0
        image.get_image(path)[..., 3] = 255
        node.record(streams[path].cuda_stream, path)
        streams[path].synchronize()
        expect = torch.zeros((256, 256, 4), dtype=torch.uint8, device="cuda")
        expect[..., 3] = 255
        ref.render(cams[frame], expect)
        assert torch.equal(image.get_image(path), expect), f"frame {frame} on path {path}"
        assert not torch.equal(expect[..., :3], torch.zeros_like(expect[..., :3]))
    # both paths in flight at once on their own streams, then compared
    for path in range(2):
        camera.ubo = cams[path + 2]
        camera.update(path)
        image.get_image(path)[:] = 0
        image.get_image(path)[..., 3] = 255
    torch.cuda.synchronize()
    for path in range(2):
        node.record(streams[path].cuda_stream, path)
    torch.cuda.synchronize()
    for path in range(2):
        expect = torch.zeros((256, 256, 4), dtype=torch.uint8, device="cuda")
        expect[..., 3] = 255
        ref.render(cams[path + 2], expect)
        assert torch.equal(image.get_image(path), expect)
    with pytest.raises(RuntimeError, match="path index out of range"):
        node.record(0, 2)
    node.renderer.close()
    ref.close()


def test_node_check_input_errors():
    image = ImageBuffer(64, 64)
    camera = CameraUBO()
    node = GaussianSplattingNode(image, camera, make_scene("plumbing", n=100), bin_size=16, sh_degree=0)
    with pytest.raises(RuntimeError, match="input is not an ImageViewSrc!"):
        node.set_input(camera, 0)
    with pytest.raises(RuntimeError, match="input is not a CameraUboType!"):
        node.set_input(image, 1)
    with pytest.raises(RuntimeError, match="input index out of range!"):
        node.set_input(image, 2)
    node.set_input(image, 0)
    node.set_input(camera, 1)
    assert node.inputs[0] is image and node.inputs[1] is camera
    assert image.get_type() == "ImageViewSrc" and camera.get_type() == "UniformBufferObject"
    node.renderer.close()
