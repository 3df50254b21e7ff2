"""The header-only C++ node interface (include/kt_gs_node.hpp): it compiles, and a frame
rendered through klartraum-style graph code equals the C ABI's frame."""

import os
import subprocess

import numpy as np
import pytest

from klartraum_b200 import Renderer, make_scene, workload_camera
from klartraum_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = "/usr/local/cuda"


def compile_demo(out_dir: str) -> str:
    exe = os.path.join(out_dir, "node_demo")
    lib_dir = os.path.dirname(N.lib_path())
    cmd = ["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"), "-I", f"{CUDA}/include",
           os.path.join(ROOT, "tests", "cpp", "node_demo.cpp"), "-o", exe, "-L", lib_dir, "-lkt_gs",
           f"-Wl,-rpath,{lib_dir}", "-L", f"{CUDA}/lib64", "-lcudart", f"-Wl,-rpath,{CUDA}/lib64"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_node_header_compiles(tmp_path):
    N.load()
    compile_demo(str(tmp_path))


@pytest.mark.gpu
def test_node_frame_equals_c_abi_frame(tmp_path):
    import torch

    exe = compile_demo(str(tmp_path))
    g3d = make_scene("plumbing", n=6000)
    cam = workload_camera("plumbing")
    (tmp_path / "scene.bin").write_bytes(g3d.tobytes())
    (tmp_path / "cam.bin").write_bytes(np.ascontiguousarray(cam).tobytes())
    out = tmp_path / "out.rgba"
    r = subprocess.run([exe, str(tmp_path / "scene.bin"), str(tmp_path / "cam.bin"), "256", "256", str(out)],
                       capture_output=True, text=True)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    got = np.frombuffer(out.read_bytes(), np.uint8).reshape(256, 256, 4)
    rr = Renderer(256, 256, bin_size=16, sh_degree=0)
    rr.set_gaussians(g3d)
    img = torch.zeros((256, 256, 4), dtype=torch.uint8, device="cuda")
    img[..., 3] = 255
    rr.render(cam, img)
    assert np.array_equal(got, img.cpu().numpy())
