"""Shared helpers of the test suite: fixtures, oracle comparison, image metrics."""

from __future__ import annotations

import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load_kat() -> dict:
    with open(os.path.join(HERE, "golden", "reference_kat.json")) as f:
        return json.load(f)


def kat_project_scene():
    """Inputs of the reference's `project` test as Gaussian3D records + its camera."""
    from klartraum_b200 import GAUSSIAN3D_DTYPE, orbit_camera

    k = load_kat()["project"]
    g = np.zeros(len(k["gaussians"]), GAUSSIAN3D_DTYPE)
    for i, d in enumerate(k["gaussians"]):
        g[i]["position"] = d["position"]
        g[i]["rotation"] = d["rotation"]
        g[i]["scale"] = d["scale"]
        g[i]["color"] = d["color"]
        g[i]["alpha"] = d["alpha"]
        g[i]["shR"][0] = d["shR0"]
        g[i]["shG"][0] = d["shG0"]
        g[i]["shB"][0] = d["shB0"]
    c = k["camera"]
    cam = orbit_camera(c["distance"], *k["screen"], fovy_deg=c["fovy_deg"], up=c["up"], near=c["near"],
                       far=c["far"])
    return g, cam, k


def kat_bin_records():
    from klartraum_b200 import GAUSSIAN2D_DTYPE

    k = load_kat()["bin"]
    g = np.zeros(len(k["records"]), GAUSSIAN2D_DTYPE)
    for i, r in enumerate(k["records"]):
        g[i]["position"] = r["position"]
        g[i]["z"] = r["z"]
        g[i]["covInv"] = r["covInv"]
        g[i]["color"] = [1.0, 1.0, 1.0]
        g[i]["alpha"] = 0.5
    return g, k


def psnr(a: np.ndarray, b: np.ndarray) -> float:
    d = a.astype(np.float64) - b.astype(np.float64)
    mse = float(np.mean(d * d))
    if mse == 0.0:
        return float("inf")
    return 10.0 * np.log10(255.0 * 255.0 / mse)


def background(h: int, w: int, kind: str = "black", seed: int = 7) -> np.ndarray:
    img = np.zeros((h, w, 4), np.uint8)
    if kind == "black":
        img[..., 3] = 255  # render pass clear colour (0,0,0,1) (renderpass.hpp:170)
    elif kind == "random":
        img[:] = np.random.default_rng(seed).integers(0, 256, size=img.shape, dtype=np.uint8)
    return img


def bits(a: np.ndarray) -> np.ndarray:
    """float32 fields as uint32 bit patterns for exact comparison."""
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def compare_projected(gpu: np.ndarray, ref: np.ndarray, counts: np.ndarray) -> None:
    """Projected records bit for bit. The colour is compared for Gaussians that meet a bin
    (counts > 0); the projection stores 0 for the others, whose colour no later stage reads."""
    counts = np.asarray(counts)
    for f in ("position", "z", "covInv", "color", "alpha"):
        g, r = bits(gpu[f]), bits(ref[f])
        if f == "color":
            assert not g[counts == 0].any(), "colour of Gaussians without bins is not 0"
            g, r = g[counts > 0], r[counts > 0]
        bad = np.nonzero((g != r).reshape(len(g), -1).any(axis=1))[0]
        assert bad.size == 0, f"{f}: {bad.size} records differ, first {bad[:5]}: gpu {gpu[f][bad[:3]]} ref {ref[f][bad[:3]]}"


# Divergence of float32 images from the double-precision oracle, collected over the session and
# printed by tests/conftest.py at the end of the run.
DIVERGENCE: list[dict] = []


def log_divergence(case: str, gpu_img: np.ndarray, f32_img: np.ndarray, f64_img: np.ndarray,
                   rows: tuple | None = None) -> dict:
    """Measure the GPU image and the float32 oracle's image against the double-precision
    oracle's (in units of 1/255), record both, and check that the GPU drifts no further from the
    double-precision result than the float32 oracle does plus one quantisation step."""
    import oracle

    g = oracle.divergence(gpu_img, f64_img, rows)
    f = oracle.divergence(f32_img, f64_img, rows)
    entry = {"case": case, "gpu": g, "f32_oracle": f}
    DIVERGENCE.append(entry)
    assert g["max_abs"] <= f["max_abs"] + 1.0, entry
    return entry
