"""Write tests/golden/reference_kat.json: the known-answer vectors of klartraum's own
Gaussian-splatting tests (tests/test_gaussian_splatting.cpp in the reference repository),
restated in this renderer's record layout.

The reference's tests cannot run here (they open a GLFW window and a Vulkan device) and
several are stale (see the notes in each entry), so the expected values below are taken
from the test source as literals, each with its file:line. Run:

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))


def kat() -> dict:
    return {
        "source": "klartraum tests/test_gaussian_splatting.cpp",
        "project": {
            "cite": "tests/test_gaussian_splatting.cpp:65-162",
            "note": ("4 unit Gaussians; InterfaceCameraOrbit with default up = Z, distance 5 "
                     "(:126-129), perspective(45 deg, 512/512, 0.1, 10) with proj[1][1] negated "
                     "(src/interface_camera_orbit.cpp:52-55); 512x512 screen (backend_config.hpp)"),
            "screen": [512, 512],
            "camera": {"distance": 5.0, "up": "z", "fovy_deg": 45.0, "near": 0.1, "far": 10.0},
            "gaussians": [
                {"position": [0, 0, 0], "rotation": [0, 0, 0, 1], "scale": [1, 1, 1], "color": [1, 1, 1],
                 "alpha": 1.0, "shR0": 1.01, "shG0": 1.02, "shB0": 1.03},
                {"position": [1, 0, 0], "rotation": [0, 0, 0, 1], "scale": [1, 1, 1], "color": [1, 0, 0],
                 "alpha": 1.0, "shR0": 1.0, "shG0": 1.0, "shB0": 1.0},
                {"position": [0, 1, 0], "rotation": [0, 0, 0, 1], "scale": [1, 1, 1], "color": [0, 1, 0],
                 "alpha": 1.0, "shR0": 1.0, "shG0": 1.0, "shB0": 1.0},
                {"position": [0, 0, 1], "rotation": [0, 0, 0, 1], "scale": [1, 1, 1], "color": [0, 0, 1],
                 "alpha": 1.0, "shR0": 1.0, "shG0": 1.0, "shB0": 1.0},
            ],
            # :148-159 (EXPECT_EQ where exact, EXPECT_NEAR(.., 0.1) otherwise)
            "expected_position": [[256.0, 256.0], [256.0, 256.0], [379.6, 256.0], [256.0, 132.39]],
            "exact": [[True, True], [True, True], [False, True], [True, False]],
            "tolerance": 0.1,
        },
        "sort": {
            "cite": "tests/test_gaussian_splatting.cpp:164-238",
            "note": ("records (position, z, binMask); the sort key is binMask[15:0] << 32 | "
                     "(floatBitsToUint(z) ^ 0x80000000) (gsplat_radix_sort_include.glsl:51-63). "
                     "The test zeroes the element count it sorts by (:205-206), so it is stale; its "
                     "expectations still hold for the stable key order"),
            "z": [-0.5, 0.2, 0.8, 0.1, -0.5, 0.2, 0.8, 0.1],
            "binMask": [0, 0, 0, 0, 4, 2, 1, 16],
            "expected_first4_z": [-0.5, 0.1, 0.2, 0.8],          # :227-230
            "expected_last4_binMask_nondecreasing": True,         # :233-235
            "expected_order": [0, 3, 1, 2, 6, 5, 4, 7],           # implied by the two above
        },
        "bin": {
            "cite": "tests/test_gaussian_splatting.cpp:240-342",
            "note": ("4 Gaussians, one per quadrant of a 512x512 screen with a 4x4 grid; the test "
                     "stores a covariance in the covInv slot (:253-286). Its z values (0.2..0.5) are "
                     "culled by the current shader (gsplat_binning.comp:113) and its 44-byte host "
                     "struct is read with the shader's 48-byte stride, so its list 1,2,8,4096,32768 "
                     "(:334-338) is stale. With culling disabled and aligned records the four "
                     "Gaussians fall in bins 0, 3, 12, 15 = masks 1, 8, 4096, 32768, all in that list"),
            "screen": [512, 512],
            "bin_size": 128,
            "records": [
                {"position": [115.0, 100.0], "z": 0.2, "covInv": [250.0, 0.0, 0.0, 50.0]},
                {"position": [400.0, 100.0], "z": 0.3, "covInv": [60.0, 0.0, 0.0, 60.0]},
                {"position": [100.0, 400.0], "z": 0.4, "covInv": [40.0, 0.0, 0.0, 40.0]},
                {"position": [400.0, 400.0], "z": 0.5, "covInv": [70.0, 0.0, 0.0, 70.0]},
            ],
            "expected_bins_no_cull": [[0], [3], [12], [15]],
            "expected_counts_with_cull": [0, 0, 0, 0],
            "reference_mask_list": [1, 2, 8, 4096, 32768],
        },
    }


def main() -> None:
    path = os.path.join(HERE, "reference_kat.json")
    with open(path, "w") as f:
        json.dump(kat(), f, indent=1)
        f.write("\n")
    print(path)


if __name__ == "__main__":
    main()
