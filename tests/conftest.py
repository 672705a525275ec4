import json
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "qwen-flash-next-8gb_b200")
ORACLE = os.path.join(REPO, "oracle")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device (B200)")
    # The oracle is test infrastructure; build it if this checkout has no binary yet.
    sys.path.insert(0, ORACLE)
    import build as oracle_build  # oracle/build.py
    oracle_build.build()
    sys.modules.pop("build", None)
    sys.path.remove(ORACLE)


@pytest.fixture(scope="session")
def golden():
    with open(os.path.join(GOLDEN, "golden.json")) as f:
        meta = json.load(f)

    class G:
        cases = meta["cases"]

        @staticmethod
        def load(name):
            return np.load(os.path.join(GOLDEN, name + ".npy"))

    return G


def rel_err(a, ref):
    """max |a - ref| / RMS(ref), in float64."""
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref * ref))
    return float(np.max(np.abs(a - ref)) / rms)


def sha(a):
    import hashlib
    a = np.ascontiguousarray(a)
    if a.dtype == np.float32:
        a = a.copy()
        a[np.isnan(a)] = np.float32("nan")
    return hashlib.sha256(a.tobytes()).hexdigest()


def bf16_steps(a, b):
    """Distance in bf16 rounding steps between arrays of bf16 values held as
    fp32 (|difference of the top 16 bits of the patterns|; same-sign values)."""
    a = np.ascontiguousarray(a, np.float32).view(np.int32) >> 16
    b = np.ascontiguousarray(b, np.float32).view(np.int32) >> 16
    return np.abs(a.astype(np.int64) - b.astype(np.int64))
