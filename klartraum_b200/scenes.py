"""Seeded synthetic scenes (numpy PCG64) for the renderer's workloads.

No public dataset is used; each workload is generated from the distributions below:

* ``plumbing``  16,384 Gaussians, SH0, 256x256: positions U[-0.5,0.5]^3, log-scales
  N(-4, 0.5), normalised N(0,1)^4 quaternions, opacity sigmoid(N(0,1.5)), DC N(0,0.5).
* ``single_1m``  1,000,000 Gaussians, SH3, 1920x1080: positions from a 64-component
  Gaussian mixture (centres U[-0.5,0.5]^3, sigma U[0.02,0.2]), log-scales N(-5, 0.6),
  DC N(0,0.5), bands 1-3 N(0,0.08), opacity sigmoid(N(0,1.5)).
* ``large_6m``  6,000,000 Gaussians, same distributions, 3840x2160.
* ``multiview_3m``  3,000,000 Gaussians, same distributions, 64 orbit views at 1920x1080.
* ``stress_2m``  2,000,000 Gaussians, SH1, log-scales N(-3, 0.8), opacity sigmoid(N(2,1)),
  positions U[-0.5,0.5]^3, 3840x2160, camera at distance 1.0.

All cameras: orbit of radius 1.5 (1.0 for the stress scene), 60 degree vertical FOV, y up,
16x16-pixel bins. Scales are stored exp()'d and opacities sigmoid()'ed, as klartraum's
loader leaves them.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .types import GAUSSIAN3D_DTYPE


@dataclass(frozen=True)
class Workload:
    name: str
    n: int
    sh_degree: int
    width: int
    height: int
    distance: float = 1.5
    fovy_deg: float = 60.0
    log_scale_mean: float = -5.0
    log_scale_std: float = 0.6
    opacity_mean: float = 0.0
    opacity_std: float = 1.5
    mixture: bool = True
    views: int = 1
    bin_size: int = 16
    seed: int = 20241201
    extra: dict = field(default_factory=dict)


WORKLOADS = {
    "plumbing": Workload("plumbing", 16384, 0, 256, 256, log_scale_mean=-4.0, log_scale_std=0.5,
                         mixture=False),
    "single_1m": Workload("single_1m", 1_000_000, 3, 1920, 1080),
    "large_6m": Workload("large_6m", 6_000_000, 3, 3840, 2160),
    "multiview_3m": Workload("multiview_3m", 3_000_000, 3, 1920, 1080, views=64),
    "stress_2m": Workload("stress_2m", 2_000_000, 1, 3840, 2160, distance=1.0, log_scale_mean=-3.0,
                          log_scale_std=0.8, opacity_mean=2.0, opacity_std=1.0, mixture=False),
}


def _sigmoid(x: np.ndarray) -> np.ndarray:
    return 1.0 / (1.0 + np.exp(-x))


def make_scene(w: Workload | str, n: int | None = None, seed: int | None = None) -> np.ndarray:
    """Array of ``n`` Gaussian3D records drawn from the workload's distributions."""
    if isinstance(w, str):
        w = WORKLOADS[w]
    n = w.n if n is None else n
    rng = np.random.Generator(np.random.PCG64(w.seed if seed is None else seed))
    g = np.zeros(n, dtype=GAUSSIAN3D_DTYPE)
    if w.mixture:
        k = 64
        centres = rng.uniform(-0.5, 0.5, size=(k, 3))
        sig = rng.uniform(0.02, 0.2, size=k)
        comp = rng.integers(0, k, size=n)
        pos = centres[comp] + rng.standard_normal((n, 3)) * sig[comp, None]
    else:
        pos = rng.uniform(-0.5, 0.5, size=(n, 3))
    g["position"] = pos
    q = rng.standard_normal((n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    g["rotation"] = q
    g["scale"] = np.exp(rng.normal(w.log_scale_mean, w.log_scale_std, size=(n, 3)))
    g["alpha"] = _sigmoid(rng.normal(w.opacity_mean, w.opacity_std, size=n))
    g["color"] = rng.normal(0.0, 0.5, size=(n, 3))
    ncoef = (w.sh_degree + 1) ** 2 - 1
    if ncoef:
        for ch in ("shR", "shG", "shB"):
            g[ch][:, :ncoef] = rng.normal(0.0, 0.08, size=(n, ncoef))
    return g


def workload_camera(w: Workload | str, view: int = 0) -> np.ndarray:
    """CameraMVP of view ``view`` of the workload."""
    from .camera import orbit_camera, orbit_views

    if isinstance(w, str):
        w = WORKLOADS[w]
    if w.views > 1:
        return orbit_views(w.views, w.distance, w.width, w.height, fovy_deg=w.fovy_deg)[view]
    return orbit_camera(w.distance, w.width, w.height, fovy_deg=w.fovy_deg, up="y")
