"""Writer of .spz files for the loader tests: the published layout of nianticlabs/spz (gzip stream of
a 16-byte header and per-attribute arrays), restated with numpy. Expected decodes are computed
here too, in float32 in the same operation order as the C reader."""

from __future__ import annotations

import gzip
import struct

import numpy as np

MAGIC = 0x5053474E


def quantize(pos, log_scale, quat_xyzw, opacity, dc, sh, frac_bits=12, version=2):
    """Quantized arrays of n Gaussians (inputs: pos (n,3), log_scale (n,3), unit quat (n,4) in
    x,y,z,w order, opacity in [0,1] (n,), dc (n,3), sh (n,k,3) with k = (d+1)^2 - 1)."""
    n = len(pos)
    fixed = np.clip(np.round(pos * (1 << frac_bits)), -(1 << 23), (1 << 23) - 1).astype(np.int64)
    if version == 1:
        p = pos.astype(np.float16).view(np.uint8).reshape(n, 6)
    else:
        u = (fixed & 0xFFFFFF).astype(np.uint32)
        p = np.stack([(u >> s) & 0xFF for s in (0, 8, 16)], axis=-1).astype(np.uint8).reshape(n, 9)
    alpha = np.clip(np.round(opacity * 255.0), 0, 255).astype(np.uint8)
    col = np.clip(np.round((dc * 0.15 + 0.5) * 255.0), 0, 255).astype(np.uint8)
    scl = np.clip(np.round((log_scale + 10.0) * 16.0), 0, 255).astype(np.uint8)
    q = quat_xyzw / np.linalg.norm(quat_xyzw, axis=1, keepdims=True)
    if version == 3:
        rot = np.zeros((n, 4), np.uint8)
        for i in range(n):
            big = int(np.argmax(np.abs(q[i])))
            v = q[i] if q[i, big] >= 0 else -q[i]
            comp = big
            for k in range(4):
                if k == big:
                    continue
                mag = int(round(abs(v[k]) / np.sqrt(0.5) * 511))
                comp = (comp << 10) | (min(mag, 511)) | ((1 if v[k] < 0 else 0) << 9)
            rot[i] = np.frombuffer(struct.pack("<I", comp & 0xFFFFFFFF), np.uint8)
    else:
        v = np.where(q[:, 3:4] < 0, -q, q)  # w >= 0 is implied
        rot = np.clip(np.round((v[:, :3] + 1.0) * 127.5), 0, 255).astype(np.uint8)
    shq = np.clip(np.round(sh * 128.0 + 128.0), 0, 255).astype(np.uint8)
    return dict(pos=p, alpha=alpha, col=col, scale=scl, rot=rot, sh=shq, frac=frac_bits, version=version)


def write(path, qz, sh_degree, flags=0):
    n = len(qz["alpha"])
    head = struct.pack("<IIIBBBB", MAGIC, qz["version"], n, sh_degree, qz["frac"], flags, 0)
    body = b"".join(np.ascontiguousarray(qz[k]).tobytes() for k in ("pos", "alpha", "col", "scale", "rot", "sh"))
    with gzip.open(path, "wb") as f:
        f.write(head + body)


def expected(qz, sh_degree):
    """Gaussian3D values the reader must produce (loadSPZModel's activations applied)."""
    from klartraum_b200 import GAUSSIAN3D_DTYPE

    n = len(qz["alpha"])
    g = np.zeros(n, GAUSSIAN3D_DTYPE)
    f32 = np.float32
    if qz["version"] == 1:
        g["position"] = qz["pos"].view(np.float16).reshape(n, 3).astype(f32)
    else:
        b = qz["pos"].reshape(n, 3, 3).astype(np.int64)
        v = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16)
        v = np.where(v & 0x800000, v - (1 << 24), v)
        g["position"] = v.astype(f32) * (f32(1.0) / f32(1 << qz["frac"]))
    g["scale"] = np.exp(qz["scale"].astype(f32) / f32(16.0) - f32(10.0))
    if qz["version"] == 3:
        for i in range(n):
            comp = int(struct.unpack("<I", qz["rot"][i].tobytes())[0])
            big = comp >> 30
            q = np.zeros(4, f32)
            ss = f32(0)
            for k in (3, 2, 1, 0):
                if k == big:
                    continue
                mag, neg = comp & 511, (comp >> 9) & 1
                comp >>= 10
                val = f32(0.70710678118654752) * f32(mag) / f32(511)
                q[k] = -val if neg else val
                ss = f32(ss + q[k] * q[k])
            q[big] = np.sqrt(max(f32(0), f32(1) - ss))
            g["rotation"][i] = q
    else:
        xyz = qz["rot"].astype(f32) / f32(127.5) - f32(1.0)
        ss = (xyz[:, 0] * xyz[:, 0] + xyz[:, 1] * xyz[:, 1]) + xyz[:, 2] * xyz[:, 2]
        g["rotation"][:, :3] = xyz
        g["rotation"][:, 3] = np.sqrt(np.maximum(f32(0), f32(1) - ss))
    a = qz["alpha"].astype(f32) / f32(255.0)
    with np.errstate(divide="ignore"):
        logit = np.log(a / (f32(1.0) - a))
    g["alpha"] = (1.0 / (1.0 + np.exp(-logit.astype(np.float64)))).astype(f32)
    g["color"] = (qz["col"].astype(f32) / f32(255.0) - f32(0.5)) / f32(0.15)
    k = (sh_degree + 1) ** 2 - 1
    s = (qz["sh"].reshape(n, k, 3).astype(f32) - f32(128.0)) / f32(128.0)
    g["shR"][:, :k] = s[..., 0]
    g["shG"][:, :k] = s[..., 1]
    g["shB"][:, :k] = s[..., 2]
    return g
