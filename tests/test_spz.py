""".spz reader (kt_gs_spz_decode / kt_gs_load_spz).

The reference reads .spz through nianticlabs/spz, which is not vendored (empty submodule) and has
no test vectors in the reference's tests: parity of the decode is unpinned. These tests restate
the published format in tests/spz_format.py, write files with it and check the C reader's records
(and loadSPZModel's activations) against the restated decode."""

import ctypes as C

import numpy as np
import pytest

from klartraum_b200 import _native as N

import spz_format


def _random_scene(n, deg, seed):
    rng = np.random.default_rng(seed)
    pos = rng.uniform(-3.0, 3.0, (n, 3))
    log_scale = rng.normal(-4.0, 0.8, (n, 3))
    quat = rng.normal(size=(n, 4))
    opacity = rng.uniform(0.0, 1.0, n)
    dc = rng.normal(0.0, 0.6, (n, 3))
    sh = rng.normal(0.0, 0.2, (n, (deg + 1) ** 2 - 1, 3))
    return pos, log_scale, quat, opacity, dc, sh


def _close(a, b, rtol=2e-6, atol=0.0):
    return np.allclose(a, b, rtol=rtol, atol=atol, equal_nan=False)


@pytest.mark.parametrize("version", [1, 2, 3])
@pytest.mark.parametrize("deg", [0, 1, 3])
def test_decode_matches_restated_format(tmp_path, version, deg):
    pos, log_scale, quat, opacity, dc, sh = _random_scene(300, deg, seed=version * 10 + deg)
    qz = spz_format.quantize(pos, log_scale, quat, opacity, dc, sh, frac_bits=14, version=version)
    path = str(tmp_path / "scene.spz")
    spz_format.write(path, qz, deg)
    got, got_deg = N.spz_decode(path)
    exp = spz_format.expected(qz, deg)
    assert got_deg == deg and len(got) == 300
    # arithmetic without transcendental functions: bit-exact
    for f in ("position", "color", "shR", "shG", "shB"):
        assert np.array_equal(got[f], exp[f]), f
    assert np.array_equal(got["rotation"], exp["rotation"]) or _close(got["rotation"], exp["rotation"], atol=1e-7)
    # exp / log: the C library and numpy may differ in the last place
    assert _close(got["scale"], exp["scale"])
    assert _close(got["alpha"], exp["alpha"], atol=1e-7)
    # and the round trip recovers the inputs to quantisation precision
    assert np.abs(got["position"] - pos).max() <= (0.5 if version == 1 else 1.0) / (1 << 14) + 2e-3 * (version == 1)
    assert np.abs(np.log(got["scale"]) - log_scale).max() <= 1.0 / 32 + 1e-5
    assert np.abs(got["alpha"] - opacity).max() <= 0.5 / 255 + 1e-6
    q = quat / np.linalg.norm(quat, axis=1, keepdims=True)
    dots = np.abs((got["rotation"] * q).sum(axis=1))
    assert dots.min() > 0.995


def test_size_query_and_errors(tmp_path):
    lib = N.load()
    n, deg = C.c_uint64(0), C.c_uint32(0)
    assert lib.kt_gs_spz_decode(str(tmp_path / "missing.spz").encode(), None, 0, C.byref(n), C.byref(deg)) == 6
    pos, log_scale, quat, opacity, dc, sh = _random_scene(10, 1, seed=3)
    qz = spz_format.quantize(pos, log_scale, quat, opacity, dc, sh)
    good = str(tmp_path / "good.spz")
    spz_format.write(good, qz, 1)
    assert lib.kt_gs_spz_decode(good.encode(), None, 0, C.byref(n), C.byref(deg)) == 0
    assert n.value == 10 and deg.value == 1
    from klartraum_b200 import GAUSSIAN3D_DTYPE

    small = np.zeros(5, GAUSSIAN3D_DTYPE)
    assert lib.kt_gs_spz_decode(good.encode(), small.ctypes.data, 5, C.byref(n), C.byref(deg)) == 3  # capacity
    # bad magic, unknown version, truncated arrays
    import gzip
    import struct

    raw = gzip.open(good).read()
    for name, data in [("magic", b"XXXX" + raw[4:]),
                       ("version", raw[:4] + struct.pack("<I", 9) + raw[8:]),
                       ("degree", raw[:12] + bytes([4]) + raw[13:]),
                       ("truncated", raw[:-7])]:
        p = str(tmp_path / f"{name}.spz")
        with gzip.open(p, "wb") as f:
            f.write(data)
        assert lib.kt_gs_spz_decode(p.encode(), None, 0, C.byref(n), C.byref(deg)) == 6, name


@pytest.mark.gpu
def test_load_spz_renders_the_decoded_records(tmp_path):
    """kt_gs_load_spz uploads exactly the decoded records: same image as kt_gs_set_gaussians."""
    torch = pytest.importorskip("torch")
    from klartraum_b200 import Renderer, orbit_camera

    pos, log_scale, quat, opacity, dc, sh = _random_scene(5000, 3, seed=11)
    pos *= 0.15
    log_scale -= 0.5
    qz = spz_format.quantize(pos, log_scale, quat, opacity, dc, sh, frac_bits=16, version=3)
    path = str(tmp_path / "scene.spz")
    spz_format.write(path, qz, 3)
    cam = orbit_camera(2.0, 320, 240, fovy_deg=60.0, up="y")
    imgs = []
    for use_file in (True, False):
        r = Renderer(320, 240, bin_size=16, sh_degree=3)
        if use_file:
            r.load_spz(path)
        else:
            r.set_gaussians(N.spz_decode(path)[0])
        img = torch.zeros((240, 320, 4), dtype=torch.uint8, device="cuda")
        r.render(cam, img)
        imgs.append(img.cpu().numpy())
        assert r.stats()["num_keys"] > 0
        r.close()
    assert np.array_equal(imgs[0], imgs[1])
