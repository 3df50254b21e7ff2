import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: full-size workloads")


def pytest_terminal_summary(terminalreporter):
    """Log how far the float32 images (GPU and float32 oracle) are from the double-precision
    oracle for every case that measured it."""
    try:
        from helpers import DIVERGENCE
    except ImportError:
        return
    if not DIVERGENCE:
        return
    tr = terminalreporter
    tr.section("divergence from the double-precision oracle (units of 1/255)")
    tr.write_line(f"{'case':<44} {'gpu max':>8} {'gpu mean':>9} {'gpu dB':>7} {'f32 max':>8} {'f32 mean':>9} "
                  f"{'f32 dB':>7}")
    for e in DIVERGENCE:
        g, f = e["gpu"], e["f32_oracle"]
        tr.write_line(f"{e['case']:<44} {g['max_abs']:8.3f} {g['mean_abs']:9.4f} {g['psnr_db']:7.2f} "
                      f"{f['max_abs']:8.3f} {f['mean_abs']:9.4f} {f['psnr_db']:7.2f}")
