"""CPU tests: the package writer and the oracle against the reference's own fixtures and compiler output."""
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import REPO
from bnneon_b200 import synth
from oracle import oracle

GOLDEN = os.path.join(REPO, "tests", "golden")


def sha256(path):
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


@pytest.mark.parametrize("name", ["v24_mini", "v24_full"])
def test_package_bytes_match_reference_compiler(name, mini_pkg, full_pkg):
    """Our writer emits the reference compiler's bytes (sha256 recorded by tests/golden/make_golden.py)."""
    with open(os.path.join(GOLDEN, "packages.json"), encoding="utf-8") as f:
        want = json.load(f)[name]
    path = mini_pkg if name == "v24_mini" else full_pkg
    assert os.path.getsize(path) == want["size"]
    assert sha256(path) == want["sha256"]


def test_s8_packing_matches_reference_packer():
    """s8_tensors of the reference (lower.py:883-914) on fixed matrices, recorded in s8_packing.npz."""
    z = np.load(os.path.join(GOLDEN, "s8_packing.npz"))
    for i in range(4):
        lw = synth._Int8Lowering([])  # pylint: disable=protected-access
        tl, shp = lw.s8("t", z[f"w{i}"], z[f"bias{i}"])
        assert tuple(shp) == tuple(z[f"shape{i}"])
        for j, suffix in enumerate(("q", "sw", "cs", "b")):
            got, want = lw.tensors[tl[j]][1], z[f"{suffix}{i}"]
            assert got.dtype == want.dtype and np.array_equal(got, want), (i, suffix)


def test_s8_rounding_reference_vectors():
    """The reference's own packing test (tests/test_lower_units.py:139-156), restated."""
    lw = synth._Int8Lowering([])  # pylint: disable=protected-access
    w = np.array([[0.5, -1.0, 0.25], [0.0, 0.0, 0.0]], np.float32)
    tl, shp = lw.s8("t", w, np.array([1.0, 2.0], np.float32))
    assert shp == (2, 3, 16, 8)
    q = lw.tensors[tl[0]][1]
    assert q.shape == (2, 1, 4, 16)
    assert q[0, 0, 0, :3].tolist() == [64, -127, 32]  # 63.5 -> 64 and 31.75 -> 32: ties away from zero
    assert not q[0, 0, 1].any()
    assert lw.tensors[tl[2]][1][:2].tolist() == [64 - 127 + 32, 0]
    sw = lw.tensors[tl[1]][1]
    assert np.isclose(sw[0], 1 / 127) and sw[1] == 1.0


def f32(x):
    return np.float32(x)


def test_frecpe_arm_values():
    """FRECPE on values whose estimates the Arm pseudocode fixes (RecipEstimate of the top 8 mantissa bits)."""
    assert oracle.lib().bnno_frecpe(1.0) == f32(0.998046875)
    assert oracle.lib().bnno_frecpe(2.0) == f32(0.4990234375)
    assert oracle.lib().bnno_frecpe(0.5) == f32(1.99609375)
    assert oracle.lib().bnno_frecpe(1.5) == f32(0.666015625)
    assert oracle.lib().bnno_frecpe(-4.0) == f32(-0.24951171875)
    assert np.isinf(oracle.lib().bnno_frecpe(0.0))
    assert oracle.lib().bnno_frecpe(float("inf")) == 0.0
    # the estimate is within 2^-8 of 1/x across a binade
    xs = np.float32(1.0) + np.arange(256, dtype=np.float32) / 256
    est = oracle.fn("bnno_frecpe", xs)
    assert np.all(np.abs(est * xs - 1) < 2 ** -8)


def test_silu_sigmoid_close_to_exact():
    x = np.linspace(-30, 30, 2001).astype(np.float32)
    s = oracle.fn("bnno_silu", x)
    exact = x / (1 + np.exp(-x.astype(np.float64)))
    assert np.max(np.abs(s - exact) / np.maximum(np.abs(exact), 1e-3)) < 1e-4
    g = oracle.fn("bnno_sigmoid", x)
    assert np.max(np.abs(g - 1 / (1 + np.exp(-x.astype(np.float64))))) < 1e-6


def test_fe_pow_polynomials_close_to_exact():
    x = np.logspace(-20, 10, 300).astype(np.float32)
    assert np.max(np.abs(oracle.fn("bnno_log2_acc", x) - np.log2(x.astype(np.float64)))) < 1e-5
    t = np.linspace(-100, 100, 301).astype(np.float32)
    e = oracle.fn("bnno_exp2_acc", t)
    assert np.max(np.abs(e / np.exp2(t.astype(np.float64)) - 1)) < 1e-6


def quant(rows, K, Kp, gate=None):
    x = np.ascontiguousarray(rows, np.float32)
    M = x.shape[0]
    q, sa, za = np.zeros((M, Kp), np.int8), np.zeros(M, np.float32), np.zeros(M, np.int32)
    oracle.lib().bnno_quant_rows(oracle.ptr(x), x.shape[1], M, K, Kp, oracle.ptr(gate), oracle.ptr(q), oracle.ptr(sa),
                                 oracle.ptr(za))
    return q, sa, za


def test_quant_rows_rules():
    """s8n_quant_rows (gemm_s8n.c:15-51): asymmetric into [-127, 127], constant rows symmetric, pads = zero point."""
    x = np.array([[-1.0, 0.0, 1.0, 3.0, 0.5, 0.25, -0.5, 2.0, 1.5, -1.0, 0.0, 0.0]], np.float32)
    q, sa, za = quant(x, 12, 16)
    assert q.min() == -127 and q.max() == 127
    assert sa[0] == np.float32(np.float32(4.0) / np.float32(254.0))
    assert all(v == za[0] for v in q[0, 12:])
    q, sa, za = quant(np.full((1, 8), 2.5, np.float32), 8, 16)
    assert za[0] == 0 and sa[0] == np.float32(np.float32(2.5) / np.float32(127.0)) and np.all(q[0, :8] == 127)
    q, sa, za = quant(np.zeros((1, 8), np.float32), 8, 16)
    assert za[0] == 0 and np.all(q == 0)


def test_oracle_package_runs(mini_pkg):
    p = oracle.Package(mini_pkg)
    assert p.n_ops == 20
    pcm = synth.audio(1, seed=11)[0]
    a, ea = p.run(pcm)
    b, eb = p.run(pcm)
    assert a.shape == (64,) and ea.shape == (1024,)
    assert np.all(np.isfinite(a)) and np.array_equal(a, b) and np.array_equal(ea, eb)
