import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "ada-mla_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

# North-star parity bar on O* (fp16 in, fp32 accumulate).
MAX_ABS_TOL = 1e-2
MEAN_ABS_TOL = 1e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def assert_close_parity(got, ref, max_tol=MAX_ABS_TOL, mean_tol=MEAN_ABS_TOL, what=""):
    """max-abs and mean-abs error bars of the north star."""
    import numpy as np

    g = np.asarray(got, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    assert g.shape == r.shape, (what, g.shape, r.shape)
    assert np.isfinite(g).all(), f"{what}: non-finite output"
    d = np.abs(g - r)
    mx, mean = float(d.max()) if d.size else 0.0, float(d.mean()) if d.size else 0.0
    assert mx <= max_tol and mean <= mean_tol, f"{what}: max-abs {mx:.3g} mean-abs {mean:.3g}"
    return mx, mean
