"""FE_LOGMEL, the framed log-mel front end of compiled models (Perch): packages written as the reference compiler writes
them (tests/golden/logmel_packages.json, made by tests/golden/make_golden.py with the reference's lower.py), the
oracle against an independent float64 DFT, the loader's record checks, and (GPU) the kernel bit for bit against the
oracle through the per-op C ABI and through packages."""
import hashlib
import json
import os
import struct

import numpy as np
import pytest

from conftest import bits_equal, mismatch_report, gpu_visible
from bnneon_b200 import BnnError, Model, load_library, pkgread, synth
from oracle import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "logmel_packages.json"), encoding="utf-8") as fh:
    PACKAGES = json.load(fh)


def frontend(g):
    return synth.logmel_frontend(g["nsamp"], g["frame"], g["hop"], g["pad"], g["nfft"], g["nmel"], floor=g["floor"],
                                 scale=g["scale"])


def signal(n, nsamp, seed):
    rng = np.random.default_rng(seed)
    t = np.arange(nsamp) / synth.PERCH_SAMPLE_RATE
    x = 0.05 * rng.standard_normal((n, nsamp)) + 0.3 * np.sin(2 * np.pi * rng.uniform(200, 8000, (n, 1)) * t)
    return x.astype(np.float32)


def dft_reference(x, fe):
    """log(max(mel |rfft(window * frame)|, floor)) * scale in float64 (an independent check of the oracle)."""
    n, nsamp = x.shape
    pad, frame, hop, nfft = fe["pad"], fe["frame"], fe["hop"], fe["nfft"]
    nfr = synth.logmel_frames(fe)
    y = np.zeros((n, nsamp + 2 * pad + nfft + 64))
    y[:, pad:pad + nsamp] = x
    w = np.zeros(nfft)
    w[:frame] = fe["window"]
    out = np.zeros((n, nfr, fe["mel"].shape[0]))
    for t in range(nfr):
        mag = np.abs(np.fft.rfft(y[:, t * hop:t * hop + nfft] * w, axis=1))
        out[:, t] = np.log(np.maximum(mag @ fe["mel"].T.astype(np.float64), fe["floor"])) * fe["scale"]
    return out


@pytest.mark.parametrize("name", sorted(PACKAGES))
def test_logmel_package_bytes_match_reference_compiler(tmp_path, name):
    g = PACKAGES[name]
    path = str(tmp_path / f"{name}.bnpk")
    synth.write_logmel_package(path, frontend(g))
    with open(path, "rb") as f:
        data = f.read()
    assert len(data) == g["size"] and hashlib.sha256(data).hexdigest() == g["sha256"]


@pytest.mark.parametrize("name", sorted(PACKAGES))
def test_oracle_against_float64_dft(name):
    g = PACKAGES[name]
    fe = frontend(g)
    x = signal(2, g["nsamp"], 3)
    got = oracle.logmel(x, fe["frame"], fe["hop"], fe["pad"], fe["nfft"], fe["window"], fe["mel"], fe["floor"],
                        fe["scale"])
    want = dft_reference(x, fe)
    assert got.shape == want.shape and np.abs(got - want).max() < 2e-5 * max(1.0, g["scale"] * 10)


def init_error(path):
    with pytest.raises(BnnError) as e:
        Model(path, mode=4)
    return e.value


def test_logmel_validation_errors(tmp_path):
    """logmel_init's checks (src/rt_ops_f32.c:364-380): nfft a power of two in 16..2048, frame <= nfft."""
    g = PACKAGES["logmel_small"]
    path = str(tmp_path / "lm.bnpk")
    synth.write_logmel_package(path, frontend(g))
    if not gpu_visible():
        e = init_error(path)
        assert e.kind == "CPU" and "no CUDA device" in str(e)
    off = pkgread.op_offsets(path)[0]
    with open(path, "rb") as f:
        data = bytearray(f.read())
    _, _, nb, nt, ni, _ = struct.unpack("<6H", bytes(data[off:off + 12]))
    ints = off + 12 + 4 * (nb + nt)
    for k, val, text in ((4, 513, "(p[4] & (p[4] - 1)) == 0"), (4, 500, "tensor argument 1"), (1, 600, "p[4] >= p[1]"),
                         (2, 0, "p[2] > 0")):
        d = bytearray(data)
        d[ints + 4 * k:ints + 4 * k + 4] = struct.pack("<i", val)
        p = tmp_path / f"i{k}.bnpk"
        p.write_bytes(bytes(d))
        e = init_error(str(p))
        assert e.kind == "PACKAGE" and text in str(e) and "op 0 fe_logmel" in str(e), (k, str(e))


# ------------------------------------------------------------------ GPU

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    h = load_library()
    torch.cuda.init()
    assert h.bnn_cuda_device_init() == 0, h.bnn_last_error()
    return h


def run_op(h, fe, x):
    op = h.bnn_logmel_new(fe["nsamp"], fe["frame"], fe["hop"], fe["pad"], fe["nfft"], fe["mel"].shape[0],
                          fe["window"].ctypes.data, np.ascontiguousarray(fe["mel"]).ctypes.data, fe["floor"],
                          fe["scale"])
    assert op, h.bnn_last_error()
    try:
        nfr, nmel = h.bnn_logmel_frames(op), fe["mel"].shape[0]
        d_x = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        d_s = torch.full((x.shape[0], nfr * nmel + 5), 7.0, dtype=torch.float32, device="cuda")
        assert h.bnn_logmel_run(op, x.shape[0], d_x.data_ptr(), x.shape[1], d_s.data_ptr(), nfr * nmel + 5, None) == 0
        torch.cuda.synchronize()
        out = d_s.cpu().numpy()
        assert (out[:, nfr * nmel:] == 7.0).all()
        return out[:, :nfr * nmel].reshape(x.shape[0], nfr, nmel)
    finally:
        h.bnn_logmel_free(op)


GEOMETRIES = [  # (nsamp, frame, hop, pad, nfft, nmel, floor, scale)
    (4000, 400, 160, 0, 512, 40, 1e-5, 1.0),
    (3001, 255, 100, 64, 256, 20, 1e-3, 0.5),
    (2000, 16, 16, 0, 16, 3, 1e-5, 1.0),
    (1000, 13, 7, 5, 32, 5, 1e-5, 2.0),
    (9000, 2048, 512, 1024, 2048, 128, 1e-6, 1.0),
    (6000, 1000, 333, 0, 1024, 64, 1e-4, 1.0),
    (5000, 128, 64, 0, 128, 16, 1e-5, 1.0),
]


@pytest.mark.gpu
@pytest.mark.parametrize("geom", GEOMETRIES, ids=[f"nfft{g[4]}_frame{g[1]}_pad{g[3]}" for g in GEOMETRIES])
def test_logmel_op(lib, geom):
    nsamp, frame, hop, pad, nfft, nmel, floor, scale = geom
    fe = synth.logmel_frontend(nsamp, frame, hop, pad, nfft, nmel, floor=floor, scale=scale)
    x = signal(3, nsamp, nfft)
    got = run_op(lib, fe, x)
    want = oracle.logmel(x, frame, hop, pad, nfft, fe["window"], fe["mel"], floor, scale)
    assert bits_equal(got, want), mismatch_report(got, want)


@pytest.mark.gpu
def test_logmel_edge_values(lib):
    """Silence (every band at the floor), huge samples (|X|^2 overflows to inf), a negative floor (log2_acc of a
    negative sum), a window with negative taps; a NaN and an infinite sample: the frames that do not read them are
    bit-exact (the frames that do carry a NaN whose payload the GPU does not model, and the log2 polynomial reads the
    payload's bits into a finite number)."""
    fe = synth.logmel_frontend(3000, 256, 128, 32, 256, 24, floor=1e-5)
    x = signal(5, 3000, 1)
    x[0] = 0.0
    x[1, 700] = np.nan
    x[2, 100] = np.inf
    x[3] *= 1e18
    got = run_op(lib, fe, x)
    want = oracle.logmel(x, fe["frame"], fe["hop"], fe["pad"], fe["nfft"], fe["window"], fe["mel"], fe["floor"],
                         fe["scale"])
    for w, bad in ((0, None), (1, 700), (2, 100), (3, None), (4, None)):
        keep = np.ones(got.shape[1], bool)
        if bad is not None:
            st = np.arange(got.shape[1]) * fe["hop"] - fe["pad"]
            keep = ~((st <= bad) & (bad < st + fe["nfft"]))
            assert keep.sum() > 0 and not keep.all()
        assert bits_equal(got[w][keep], want[w][keep]), (w, mismatch_report(got[w][keep], want[w][keep]))
    assert (want[0] == want[0][0, 0]).all()  # silence: every band at the floor
    fe2 = dict(fe, floor=-1.0, window=(fe["window"] - 0.25).astype(np.float32))
    got = run_op(lib, fe2, x[3:5])
    want = oracle.logmel(x[3:5], fe2["frame"], fe2["hop"], fe2["pad"], fe2["nfft"], fe2["window"], fe2["mel"],
                         fe2["floor"], fe2["scale"])
    assert bits_equal(got, want), mismatch_report(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(PACKAGES))
def test_logmel_package(lib, name, tmp_path):
    g = PACKAGES[name]
    path = str(tmp_path / f"{name}.bnpk")
    nfr, nmel = synth.write_logmel_package(path, frontend(g))
    x = signal(7, g["nsamp"], 5)
    with Model(path, mode=4, batch=3) as m:
        got, _ = m.infer_batch(x)
        assert m.launches_per_batch == 1
    want, _ = oracle.run_many(path, x, threads=4)
    assert got.shape == (7, nfr * nmel) and bits_equal(got, want), mismatch_report(got, want)


@pytest.mark.gpu
def test_logmel_perch_geometry(lib):
    """The Perch-like front end (5 s at 32 kHz, 20 ms frames, 10 ms hop, 1024-point FFT, 128 mel bins)."""
    p = synth.PERCH_FE
    fe = synth.logmel_frontend(p["nsamp"], p["frame"], p["hop"], p["pad"], p["nfft"], p["nmel"], p["fmin"], p["fmax"],
                               p["floor"], p["scale"])
    x = signal(4, p["nsamp"], 9)
    got = run_op(lib, fe, x)
    want = oracle.logmel(x, fe["frame"], fe["hop"], fe["pad"], fe["nfft"], fe["window"], fe["mel"], fe["floor"],
                         fe["scale"])
    assert got.shape == (4, 499, 128) and bits_equal(got, want), mismatch_report(got, want)
