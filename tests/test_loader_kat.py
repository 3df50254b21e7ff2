"""Known answers for the scene loaders, with every input byte written out here and every expected
value computed by hand from the format's definition (not by a writer of this repository).

The reference reads .spz and .ply files through nianticlabs/spz (not vendored in the reference:
3rdparty/spz is an empty submodule) and applies the activations of loadSPZModel / loadPLYModel
(src/vulkan_gaussian_splatting.cpp:322-365, 367-417). The byte layouts restated here:

.spz (gzip stream): header <magic "NGSP" = 0x5053474e, version, count> (u32 each), SH degree,
fractional bits, flags, reserved (u8 each); then positions (v1: 3 half floats; v2/v3: 3 x 24-bit
signed fixed point / 2^fractional_bits), alphas (sigmoid * 255), colours ((dc * 0.15 + 0.5) * 255),
scales ((log scale + 10) * 16), rotations (v1/v2: x, y, z as (v + 1) * 127.5, w >= 0 from the
norm; v3: 2-bit index of the largest component, then the other three, last index first from bit
0, as 9-bit magnitude over sqrt(1/2) plus a sign bit), SH ((v * 128) + 128, coefficient-major).

.ply: ASCII header, x y z, f_dc_0..2, opacity (logit), scale_0..2 (log), rot_0..3 (w, x, y, z);
loadPLYModel keeps |x|, |y|, |z| <= 1.5 and stores colour = 0.5 + 0.282095 f_dc.
"""

import gzip
import math
import struct

import numpy as np
import pytest

from klartraum_b200 import _native as N

SQRT1_2 = math.sqrt(0.5)


def spz_file(path, version, deg, frac, pos_bytes, alpha, colour, scale, rot_bytes, sh_bytes):
    n = len(alpha)
    head = struct.pack("<IIIBBBB", 0x5053474E, version, n, deg, frac, 0, 0)
    body = bytes(pos_bytes) + bytes(alpha) + bytes(colour) + bytes(scale) + bytes(rot_bytes) + bytes(sh_bytes)
    with gzip.open(path, "wb") as f:
        f.write(head + body)


# two points, SH degree 1 (3 coefficients x 3 channels per point)
ALPHA = [191, 1]
COLOUR = [38, 128, 217, 255, 0, 64]
SCALE = [96, 112, 160, 0, 255, 168]
SH = [192, 128, 64, 0, 255, 128, 130, 126, 128,
      128, 128, 128, 1, 2, 3, 250, 251, 252]


def expected_common(g):
    # alpha: loadSPZModel's sigmoid of the stored logit = the stored byte / 255
    assert np.allclose(g["alpha"], [191 / 255, 1 / 255], rtol=1e-6, atol=0)
    # colour: (byte / 255 - 0.5) / 0.15, the raw DC coefficient
    exp_col = [[(38 / 255 - 0.5) / 0.15, (128 / 255 - 0.5) / 0.15, (217 / 255 - 0.5) / 0.15],
               [(255 / 255 - 0.5) / 0.15, (0 / 255 - 0.5) / 0.15, (64 / 255 - 0.5) / 0.15]]
    assert np.allclose(g["color"], exp_col, rtol=1e-6, atol=1e-6)  # float32 (byte / 255 - 0.5): 4e-7 absolute
    # scale: exp(byte / 16 - 10)
    exp_scale = [[math.exp(-4.0), math.exp(-3.0), math.exp(0.0)],
                 [math.exp(-10.0), math.exp(255 / 16 - 10), math.exp(0.5)]]
    assert np.allclose(g["scale"], exp_scale, rtol=2e-6, atol=0)
    # SH: (byte - 128) / 128, coefficient-major R, G, B
    assert np.allclose(g["shR"][:, :3], [[0.5, -1.0, 2 / 128], [0.0, -127 / 128, 122 / 128]])
    assert np.allclose(g["shG"][:, :3], [[0.0, 127 / 128, -2 / 128], [0.0, -126 / 128, 123 / 128]])
    assert np.allclose(g["shB"][:, :3], [[-0.5, 0.0, 0.0], [0.0, -125 / 128, 124 / 128]])
    assert not g["shR"][:, 3:].any() and not g["shG"][:, 3:].any() and not g["shB"][:, 3:].any()


def test_spz_v2_fixed_point_and_three_byte_rotations(tmp_path):
    # 24-bit little-endian fixed point with 12 fractional bits
    pos = [0x00, 0x18, 0x00,  0x00, 0xFC, 0xFF,  0x01, 0x00, 0x00,   # 6144, -1024, 1 (/4096)
           0xFF, 0xFF, 0x7F,  0x00, 0x00, 0x80,  0x00, 0x00, 0x00]   # 2^23-1, -2^23, 0
    rot = [128, 128, 128,  255, 128, 0]
    p = str(tmp_path / "v2.spz")
    spz_file(p, 2, 1, 12, pos, ALPHA, COLOUR, SCALE, rot, SH)
    g, deg = N.spz_decode(p)
    assert deg == 1 and len(g) == 2
    assert np.array_equal(g["position"], np.array([[1.5, -0.25, 1 / 4096],
                                                   [(2**23 - 1) / 4096, -(2**23) / 4096, 0.0]], np.float32))
    x = 128 / 127.5 - 1
    r1 = [255 / 127.5 - 1, 128 / 127.5 - 1, 0 / 127.5 - 1]
    exp_rot = [[x, x, x, math.sqrt(1 - 3 * x * x)],
               [r1[0], r1[1], r1[2], math.sqrt(max(0.0, 1 - sum(v * v for v in r1)))]]
    assert np.allclose(g["rotation"], exp_rot, rtol=1e-6, atol=1e-7)
    expected_common(g)


def test_spz_v1_half_float_positions(tmp_path):
    # half floats: 0x3E00 = 1.5, 0xB400 = -0.25, 0x0001 = 2^-24 (subnormal), 0x7BFF = 65504,
    # 0x8000 = -0.0, 0x3C01 = 1 + 2^-10
    halves = [0x3E00, 0xB400, 0x0001, 0x7BFF, 0x8000, 0x3C01]
    pos = list(struct.pack("<6H", *halves))
    rot = [128, 128, 128,  255, 128, 0]
    p = str(tmp_path / "v1.spz")
    spz_file(p, 1, 1, 0, pos, ALPHA, COLOUR, SCALE, rot, SH)
    g, _ = N.spz_decode(p)
    assert np.array_equal(g["position"], np.array([[1.5, -0.25, 2.0**-24], [65504.0, -0.0, 1 + 2.0**-10]],
                                                  np.float32))
    assert np.signbit(g["position"][1, 1])
    expected_common(g)


def test_spz_v3_smallest_three_rotations(tmp_path):
    pos = [0] * 18
    # point 0: largest = w (3); x magnitude 511, y and z 0:
    #   bits 0-9 z, 10-19 y, 20-29 x, 30-31 largest -> 0xDFF00000
    # point 1: largest = x (0); bits 0-9 w (100), 10-19 z (0), 20-29 y (256 with the sign bit)
    #   -> (0x300 << 20) | 100 = 0x30000064
    rot = list(struct.pack("<II", 0xDFF00000, 0x30000064))
    p = str(tmp_path / "v3.spz")
    spz_file(p, 3, 1, 12, pos, ALPHA, COLOUR, SCALE, rot, SH)
    g, _ = N.spz_decode(p)
    w1 = SQRT1_2 * 100 / 511
    y1 = -SQRT1_2 * 256 / 511
    exp_rot = [[SQRT1_2, 0.0, 0.0, math.sqrt(1 - 0.5)],
               [math.sqrt(1 - y1 * y1 - w1 * w1), y1, 0.0, w1]]
    assert np.allclose(g["rotation"], exp_rot, rtol=1e-6, atol=1e-7)
    assert not g["position"].any()
    expected_common(g)


PLY_ROWS = [
    # x, y, z, f_dc_0..2, opacity, scale_0..2, rot_0 (w), rot_1..3 (x, y, z)
    (0.5, -1.0, 1.5, 1.0, 0.0, -1.0, 0.0, 0.0, math.log(2.0), -math.log(2.0), 1.0, 0.0, 0.0, 0.0),
    (1.6, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0),   # outside the box: dropped
    (-1.5, 0.0, 0.0, 2.0, 0.5, 0.0, math.log(3.0), -4.0, -4.0, -4.0, 0.5, 0.5, 0.5, 0.5),
    (0.0, -1.50001, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0),  # just outside
]
PLY_NAMES = ["x", "y", "z", "f_dc_0", "f_dc_1", "f_dc_2", "opacity", "scale_0", "scale_1", "scale_2",
             "rot_0", "rot_1", "rot_2", "rot_3"]


def check_ply(g):
    assert len(g) == 2
    assert np.allclose(g["position"], [[0.5, -1.0, 1.5], [-1.5, 0.0, 0.0]])
    assert np.allclose(g["alpha"], [0.5, 0.75], rtol=1e-6)                  # sigmoid(0), sigmoid(ln 3)
    assert np.allclose(g["scale"], [[1.0, 2.0, 0.5], [math.exp(-4)] * 3], rtol=2e-6)
    assert np.allclose(g["color"], [[0.5 + 0.282095, 0.5, 0.5 - 0.282095],
                                    [0.5 + 2 * 0.282095, 0.5 + 0.5 * 0.282095, 0.5]], rtol=1e-6)
    assert np.allclose(g["rotation"], [[0, 0, 0, 1], [0.5, 0.5, 0.5, 0.5]])  # (x, y, z, w)
    assert not g["shR"].any() and not g["shG"].any() and not g["shB"].any()


def test_ply_ascii_known_answer(tmp_path):
    head = ["ply", "format ascii 1.0", "comment hand-written", f"element vertex {len(PLY_ROWS)}"]
    head += [f"property float {n}" for n in PLY_NAMES] + ["end_header"]
    text = "\n".join(head) + "\n" + "\n".join(" ".join(repr(v) for v in row) for row in PLY_ROWS) + "\n"
    p = tmp_path / "kat_ascii.ply"
    p.write_text(text)
    check_ply(N.ply_decode(str(p)))


def test_ply_binary_known_answer_with_mixed_types(tmp_path):
    # opacity stored as double, the rest as float, an extra uchar property in the middle
    names = PLY_NAMES[:6] + ["red"] + PLY_NAMES[6:]
    types = ["float"] * 6 + ["uchar", "double"] + ["float"] * 7
    fmt = "<" + "".join({"float": "f", "double": "d", "uchar": "B"}[t] for t in types)
    head = ["ply", "format binary_little_endian 1.0", f"element vertex {len(PLY_ROWS)}"]
    head += [f"property {t} {n}" for t, n in zip(types, names)] + ["end_header"]
    body = b"".join(struct.pack(fmt, *(row[:6] + (200,) + row[6:])) for row in PLY_ROWS)
    p = tmp_path / "kat_binary.ply"
    p.write_bytes(("\n".join(head) + "\n").encode() + body)
    check_ply(N.ply_decode(str(p)))


@pytest.mark.gpu
def test_load_ply_renders_the_decoded_records(tmp_path):
    """kt_gs_load_ply uploads exactly the records kt_gs_ply_decode returns: the same image as
    kt_gs_set_gaussians with them."""
    torch = pytest.importorskip("torch")
    from klartraum_b200 import Renderer, orbit_camera

    rng = np.random.default_rng(21)
    n = 4000
    rows = np.zeros((n, len(PLY_NAMES)), np.float32)
    rows[:, 0:3] = rng.uniform(-0.6, 0.6, (n, 3))
    rows[:, 3:6] = rng.normal(0, 1, (n, 3))
    rows[:, 6] = rng.normal(0, 1.5, n)
    rows[:, 7:10] = rng.normal(-4.5, 0.5, (n, 3))
    q = rng.normal(0, 1, (n, 4))
    rows[:, 10:14] = q / np.linalg.norm(q, axis=1, keepdims=True)
    rows[:5, 0] = 2.0  # outside the clip box
    head = ["ply", "format binary_little_endian 1.0", f"element vertex {n}"]
    head += [f"property float {nm}" for nm in PLY_NAMES] + ["end_header"]
    p = str(tmp_path / "scene.ply")
    with open(p, "wb") as f:
        f.write(("\n".join(head) + "\n").encode() + rows.tobytes())
    cam = orbit_camera(2.0, 320, 240, fovy_deg=60.0, up="y")
    imgs = []
    for use_file in (True, False):
        r = Renderer(320, 240, bin_size=16, sh_degree=0)
        if use_file:
            r.load_ply(p)
        else:
            g = N.ply_decode(p)
            assert len(g) == n - 5
            r.set_gaussians(g)
        img = torch.zeros((240, 320, 4), dtype=torch.uint8, device="cuda")
        img[..., 3] = 255
        r.render(cam, img)
        imgs.append(img.cpu().numpy())
        assert r.stats()["num_keys"] > 0
        r.close()
    assert np.array_equal(imgs[0], imgs[1])
