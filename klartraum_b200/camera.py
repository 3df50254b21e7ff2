"""Orbit camera producing CameraMVP records, as klartraum's InterfaceCameraOrbit::update does
(src/interface_camera_orbit.cpp:19-56): view = lookAt((d,0,0), 0, up) * rotate(elevation)
* rotate(azimuth) [* translate(position)], proj = perspective(fovy, aspect, near, far) with
proj[1][1] negated for Vulkan's downward y. Matrices are float32, indexed m[col][row].

lookAt, rotate and perspective are the standard right-handed formulas (glm's
``lookAtRH``, ``rotate`` and ``perspectiveRH_NO``), evaluated in float32.
"""

from __future__ import annotations

import math

import numpy as np

from .types import camera_record

F = np.float32


def _normalize(v: np.ndarray) -> np.ndarray:
    v = v.astype(F)
    return (v / F(np.sqrt(F(np.dot(v, v))))).astype(F)


def identity() -> np.ndarray:
    return np.eye(4, dtype=F)


def matmul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """a * b for m[col][row] matrices, products summed in ascending k in float32."""
    r = np.zeros((4, 4), F)
    for c in range(4):
        for k in range(4):
            s = F(a[0][k] * b[c][0])
            for j in range(1, 4):
                s = F(s + F(a[j][k] * b[c][j]))
            r[c][k] = s
    return r


def look_at(eye, center, up) -> np.ndarray:
    eye, center, up = (np.asarray(x, F) for x in (eye, center, up))
    f = _normalize(center - eye)
    s = _normalize(np.cross(f, up).astype(F))
    u = np.cross(s, f).astype(F)
    m = identity()
    m[0][0], m[1][0], m[2][0] = s
    m[0][1], m[1][1], m[2][1] = u
    m[0][2], m[1][2], m[2][2] = -f
    m[3][0] = -F(np.dot(s, eye))
    m[3][1] = -F(np.dot(u, eye))
    m[3][2] = F(np.dot(f, eye))
    return m


def rotate(m: np.ndarray, angle: float, axis) -> np.ndarray:
    a = F(angle)
    c, s = F(math.cos(a)), F(math.sin(a))
    axis = _normalize(np.asarray(axis, F))
    temp = (F(1) - c) * axis
    R = np.zeros((3, 3), F)
    R[0][0] = c + temp[0] * axis[0]
    R[0][1] = temp[0] * axis[1] + s * axis[2]
    R[0][2] = temp[0] * axis[2] - s * axis[1]
    R[1][0] = temp[1] * axis[0] - s * axis[2]
    R[1][1] = c + temp[1] * axis[1]
    R[1][2] = temp[1] * axis[2] + s * axis[0]
    R[2][0] = temp[2] * axis[0] + s * axis[1]
    R[2][1] = temp[2] * axis[1] - s * axis[0]
    R[2][2] = c + temp[2] * axis[2]
    out = np.zeros((4, 4), F)
    for col in range(3):
        out[col] = m[0] * R[col][0] + m[1] * R[col][1] + m[2] * R[col][2]
    out[3] = m[3]
    return out


def translate(m: np.ndarray, v) -> np.ndarray:
    out = m.copy()
    v = np.asarray(v, F)
    out[3] = m[0] * v[0] + m[1] * v[1] + m[2] * v[2] + m[3]
    return out


def perspective(fovy: float, aspect: float, near: float, far: float) -> np.ndarray:
    t = F(math.tan(F(fovy) / F(2)))
    m = np.zeros((4, 4), F)
    m[0][0] = F(1) / (F(aspect) * t)
    m[1][1] = F(1) / t
    m[2][2] = -(F(far) + F(near)) / (F(far) - F(near))
    m[2][3] = F(-1)
    m[3][2] = -(F(2) * F(far) * F(near)) / (F(far) - F(near))
    return m


def orbit_camera(distance: float, width: int, height: int, *, fovy_deg: float = 45.0,
                 azimuth: float = 0.0, elevation: float = 0.0, up: str = "z",
                 near: float = 0.1, far: float = 10.0, position=(0.0, 0.0, 0.0)) -> np.ndarray:
    """CameraMVP record of InterfaceCameraOrbit::update for the given orbit state."""
    model = identity()
    if up == "y":
        view = matmul(matmul(look_at((distance, 0, 0), (0, 0, 0), (0, 1, 0)),
                             rotate(identity(), elevation, (0, 0, 1))),
                      rotate(identity(), azimuth, (0, 1, 0)))
        view = matmul(view, translate(identity(), position))
    elif up == "z":
        view = matmul(matmul(look_at((distance, 0, 0), (0, 0, 0), (0, 0, 1)),
                             rotate(identity(), elevation, (0, 1, 0))),
                      rotate(identity(), azimuth, (0, 0, 1)))
    else:
        raise ValueError("up must be 'y' or 'z'")
    proj = perspective(math.radians(fovy_deg), width / float(height), near, far)
    proj[1][1] *= F(-1)
    return camera_record(model, view, proj)


def orbit_views(n_views: int, distance: float, width: int, height: int, *, fovy_deg: float = 60.0,
                elev_range_deg=(-30.0, 30.0), up: str = "y") -> np.ndarray:
    """n_views cameras at azimuth 2*pi*k/n and elevations spread linearly over the range."""
    cams = []
    lo, hi = elev_range_deg
    for k in range(n_views):
        el = lo + (hi - lo) * (k / max(1, n_views - 1))
        cams.append(orbit_camera(distance, width, height, fovy_deg=fovy_deg,
                                 azimuth=2.0 * math.pi * k / n_views, elevation=math.radians(el), up=up))
    return np.stack(cams)
