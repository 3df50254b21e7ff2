"""3D Gaussian Splatting .ply reader (kt_gs_ply_decode / kt_gs_load_ply), loadPLYModel semantics
(src/vulkan_gaussian_splatting.cpp:367-417): clip box +-1.5, alpha = sigmoid(opacity), scale = exp,
colour = 0.5 + 0.282095 f_dc, rotation (rot_1, rot_2, rot_3, rot_0) = (x, y, z, w)."""

import ctypes as C

import numpy as np
import pytest

from klartraum_b200 import GAUSSIAN3D_DTYPE, _native as N

FIELDS = ["x", "y", "z", "nx", "ny", "nz", "f_dc_0", "f_dc_1", "f_dc_2"] + [f"f_rest_{i}" for i in range(45)] + \
         ["opacity", "scale_0", "scale_1", "scale_2", "rot_0", "rot_1", "rot_2", "rot_3"]


def _vertices(n, seed):
    rng = np.random.default_rng(seed)
    v = np.zeros(n, [(f, np.float32) for f in FIELDS])
    for f in ("x", "y", "z"):
        v[f] = rng.uniform(-2.0, 2.0, n)  # some outside the clip box
    for f in FIELDS[6:]:
        v[f] = rng.normal(0.0, 1.0, n)
    for i in range(3):
        v[f"scale_{i}"] = rng.normal(-4.0, 0.5, n)
    return v


def _write(path, v, ascii=False, extra_face=False):
    head = ["ply", "format ascii 1.0" if ascii else "format binary_little_endian 1.0", f"element vertex {len(v)}"]
    head += [f"property float {f}" for f in v.dtype.names]
    if extra_face:
        head += ["element face 0", "property list uchar int vertex_indices"]
    head.append("end_header")
    with open(path, "wb") as fh:
        fh.write(("\n".join(head) + "\n").encode())
        if ascii:
            for row in v:
                fh.write((" ".join(repr(float(x)) for x in row) + "\n").encode())
        else:
            fh.write(v.tobytes())


def _expected(v):
    f32 = np.float32
    keep = np.ones(len(v), bool)
    for f in ("x", "y", "z"):
        keep &= (v[f] >= -1.5) & (v[f] <= 1.5)
    k = v[keep]
    g = np.zeros(len(k), GAUSSIAN3D_DTYPE)
    g["position"] = np.stack([k["x"], k["y"], k["z"]], -1)
    g["rotation"] = np.stack([k["rot_1"], k["rot_2"], k["rot_3"], k["rot_0"]], -1)
    g["alpha"] = (1.0 / (1.0 + np.exp(-k["opacity"].astype(np.float64)))).astype(f32)
    g["color"] = (0.5 + 0.282095 * np.stack([k["f_dc_0"], k["f_dc_1"], k["f_dc_2"]], -1).astype(np.float64)).astype(f32)
    g["scale"] = np.exp(np.stack([k["scale_0"], k["scale_1"], k["scale_2"]], -1).astype(f32))
    return g


@pytest.mark.parametrize("ascii", [False, True], ids=["binary", "ascii"])
def test_ply_decode_matches_load_ply_model(tmp_path, ascii):
    v = _vertices(500, seed=4)
    p = str(tmp_path / "s.ply")
    _write(p, v, ascii=ascii, extra_face=True)
    got = N.ply_decode(p)
    exp = _expected(v)
    assert len(got) == len(exp) and 0 < len(got) < 500
    for f in ("position", "rotation", "color", "alpha"):
        assert np.array_equal(got[f], exp[f]), f
    assert np.allclose(got["scale"], exp["scale"], rtol=2e-6, atol=0)
    assert not got["shR"].any() and not got["shG"].any() and not got["shB"].any()


def test_ply_errors(tmp_path):
    lib = N.load()
    n = C.c_uint64(0)
    assert lib.kt_gs_ply_decode(str(tmp_path / "none.ply").encode(), None, 0, C.byref(n)) == 6
    bad = tmp_path / "bad.ply"
    bad.write_bytes(b"not a ply\n")
    assert lib.kt_gs_ply_decode(str(bad).encode(), None, 0, C.byref(n)) == 6
    v = _vertices(10, seed=5)
    missing = v[[f for f in v.dtype.names if f != "opacity"]]
    p = str(tmp_path / "missing.ply")
    _write(p, np.ascontiguousarray(missing))
    assert lib.kt_gs_ply_decode(p.encode(), None, 0, C.byref(n)) == 6
    p2 = str(tmp_path / "short.ply")
    _write(p2, v)
    with open(p2, "rb") as fh:
        data = fh.read()
    with open(p2, "wb") as fh:
        fh.write(data[:-10])
    assert lib.kt_gs_ply_decode(p2.encode(), None, 0, C.byref(n)) == 6
