"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on a CPU-only machine."""
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(REPO, "birdnet-neon-engine_b200"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

from bnneon_b200 import synth  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def pkg_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("packages")


@pytest.fixture(scope="session")
def mini_pkg(pkg_dir):
    """The 4-block v2.4-architecture package (seed 1, 61 classes -> 64 outputs)."""
    path = str(pkg_dir / "v24_mini.bnpk")
    synth.make_package(path, seed=1, mini=True)
    return path


@pytest.fixture(scope="session")
def full_pkg(pkg_dir):
    """The full v2.4-architecture package (seed 0, 6522 classes -> 6528 outputs)."""
    path = str(pkg_dir / "v24_full.bnpk")
    synth.make_package(path, seed=0, mini=False)
    return path


def gpu_visible():
    """A GPU device node exists (any index: a GPU box may expose only, say, /dev/nvidia3)."""
    import glob  # pylint: disable=import-outside-toplevel
    return bool(glob.glob("/dev/nvidia[0-9]*"))


def bits_equal(a, b):
    """Bit-exact equality of float arrays; any NaN equals any NaN (payloads are not modelled)."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    if a.shape != b.shape:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    if not np.array_equal(na, nb):
        return False
    return np.array_equal(a.view(np.int32)[~na], b.view(np.int32)[~nb])


def mismatch_report(a, b):
    a = np.asarray(a, np.float32).reshape(-1)
    b = np.asarray(b, np.float32).reshape(-1)
    bad = np.nonzero(a.view(np.int32) != b.view(np.int32))[0]
    if bad.size == 0:
        return "identical"
    i = bad[0]
    return (f"{bad.size} of {a.size} differ; first at {i}: {a[i]!r} vs {b[i]!r}; "
            f"max abs diff {np.nanmax(np.abs(a - b)):.3g}")
