"""FE_DBIMG, the dB-image front end of the v3.0 models (src/fe_dbimg.c driven by src/rt_ops_f32x.c:15-86): packages
written as the reference compiler writes them (tests/golden/dbimg_packages.json, made by tests/golden/make_golden.py
with the reference's lower.py l_fe_dbimg), the oracle (oracle/oracle_dbimg.c) against the reference's own runtime
(oracle/_ref) bit for bit, the loader's record checks, and (GPU) the kernels against the oracle through the per-op
C ABI and through packages.

The logarithm. The reference calls the C library's logf. The B200 kernel rounds the double-precision log once to
float (correctly rounded); this host's glibc logf is not correctly rounded on some inputs (one unit in the last place).
The oracle runs either: log mode 0 (this host's logf: bit for bit with the reference build) and log mode 1 (the
correctly rounded log: bit for bit with the GPU). GPU images against log mode 0 are held to a tolerance: at most
2e-6 relative to the image's range plus 1e-6 of the value (IMAGE_RTOL, IMAGE_ATOL).
"""
import json
import os
import struct

import numpy as np
import pytest

from conftest import bits_equal, mismatch_report, gpu_visible
from bnneon_b200 import BnnError, Model, load_library, pkgread, synth
from oracle import oracle, ref

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "dbimg_packages.json"), encoding="utf-8") as fh:
    PACKAGES = json.load(fh)
MODE_INT8 = 4
IMAGE_RTOL, IMAGE_ATOL = 1e-6, 2e-6  # GPU (correctly rounded log) against the reference's logf, per pixel


def frontend(g):
    g = dict(g)
    if g.get("post") is not None:
        g["post"] = [(int(c), float(v)) for c, v in g["post"]]
    if g.get("chan") is not None:
        g["chan"] = [(int(c), np.asarray(v, np.float32)) for c, v in g["chan"]]
    if "rows" in g:
        g["rows"] = list(g["rows"])
    return synth.dbimg_frontend(**g)


def signal(n, nsamp, seed):
    rng = np.random.default_rng(seed)
    t = np.arange(nsamp) / synth.V3_SAMPLE_RATE
    x = 0.02 * rng.standard_normal((n, nsamp)) + 0.3 * np.sin(2 * np.pi * rng.uniform(200, 12000, (n, 1)) * t)
    x *= (1.0 + 0.5 * np.sin(2 * np.pi * rng.uniform(0.5, 3.0, (n, 1)) * t))
    return x.astype(np.float32)


def oracle_op(fe, halo=0):
    tens, ints, _, _ = synth.dbimg_record(fe, halo)
    return oracle.DbImg(ints, tens["window"], tens["mel"], tens["rows"], tens["consts"])


def close_to(got, want):
    """|got - want| <= IMAGE_ATOL * range + IMAGE_RTOL * |want| per pixel (NaN where both are NaN)"""
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    both = np.isnan(got) & np.isnan(want)
    fin = np.isfinite(want)
    rng = np.ptp(want[fin]) if fin.any() else 0.0
    ok = both | (got == want) | (np.abs(got - want) <= IMAGE_ATOL * max(rng, 1.0) + IMAGE_RTOL * np.abs(want))
    return bool(ok.all()), int((~ok).sum())


GEOMS = {  # name: (frontend kwargs, halo)
    "small": (PACKAGES["dbimg_small"]["frontend"], 0),
    "zero_pad": (PACKAGES["dbimg_zero"]["frontend"], 0),
    "no_pad": (PACKAGES["dbimg_none"]["frontend"], 0),
    "small_halo1": (PACKAGES["dbimg_small"]["frontend"], 1),
    "zero_halo3": (PACKAGES["dbimg_zero"]["frontend"], 3),
    "nfft2048_c64": (dict(nsamp=12000, nfft=2048, hop=480, pad=1024, pad_mode="reflect", nmel=96,
                          rows=list(range(0, 96, 2)), Ho=30, Wo=17, C=64, top_db=60.0, norm=1), 0),
    "nfft8192": (dict(nsamp=16384, nfft=8192, hop=4096, pad=0, pad_mode="none", nmel=32, rows=list(range(32)), Ho=64,
                      Wo=5, C=2, top_db=80.0, norm=2), 2),
    "upsample": (dict(nsamp=3000, nfft=128, hop=128, pad=64, pad_mode="zero", nmel=12, rows=[11, 5, 0, 7], Ho=37,
                      Wo=91, C=3, top_db=None, norm=1, post=[(3, 1.0), (4, 0.5), (1, 3.0)]), 1),
}


# ------------------------------------------------------------------ CPU

@pytest.mark.parametrize("name", sorted(PACKAGES))
def test_dbimg_package_bytes_match_reference_compiler(tmp_path, name):
    import hashlib  # pylint: disable=import-outside-toplevel
    g = PACKAGES[name]
    path = str(tmp_path / f"{name}.bnpk")
    synth.write_dbimg_package(path, frontend(g["frontend"]))
    with open(path, "rb") as f:
        data = f.read()
    assert len(data) == g["size"] and hashlib.sha256(data).hexdigest() == g["sha256"]


@pytest.fixture(scope="module")
def reflib():
    if ref.reference_checkout() is not None:
        ref.build()
    if not ref.available():
        pytest.skip("no reference build (oracle/_ref) and no reference checkout to build it from")
    return ref.lib()


def reference_images(tmp_path, fe, x, halo=0):
    path = str(tmp_path / "db.bnpk")
    n_out = synth.write_dbimg_package(path, fe, halo=halo)
    out, _, rc = ref.run_many(path, MODE_INT8, x, threads=min(4, x.shape[0]))
    assert (rc == 0).all() and out.shape[1] == n_out
    return out, path


@pytest.mark.parametrize("geom", ["small", "zero_pad", "no_pad", "small_halo1", "zero_halo3", "upsample"])
def test_oracle_matches_reference_runtime(reflib, tmp_path, geom):
    """the oracle in log mode 0 against the reference's fe_db_run (through its bnn_init / bnn_infer) bit for bit, and
    the oracle's package runner against both"""
    kw, halo = GEOMS[geom]
    fe = frontend(kw)
    x = signal(3, fe["nsamp"], 11)
    want, path = reference_images(tmp_path, fe, x, halo)
    got = oracle_op(fe, halo).run(x, 0)
    assert bits_equal(got, want), mismatch_report(got, want)
    oracle.set_log_mode(0)
    pk, _ = oracle.run_many(path, x, threads=2)
    assert bits_equal(pk, want), mismatch_report(pk, want)


def test_oracle_matches_reference_runtime_v3(reflib, tmp_path):
    """the BirdNET v3.0 geometry (5 s at 32 kHz, 1024-point FFT, 501 frames, 96 of 128 mel rows to 224 x 468 x 3)"""
    fe = frontend(PACKAGES["dbimg_v3"]["frontend"])
    x = signal(2, fe["nsamp"], 12)
    want, _ = reference_images(tmp_path, fe, x)
    got = oracle_op(fe).run(x, 0)
    assert got.shape == (2, 224 * 468 * 4) and bits_equal(got, want), mismatch_report(got, want)


def edge_signals(nsamp):
    x = signal(4, nsamp, 5)
    x[0] = 0.0                 # silence: every band at the floor, max - min = 0
    x[1, nsamp // 3] = np.nan  # a NaN sample: NaN in the frames that read it
    x[2] *= 1e19               # the power overflows to inf
    x[3, ::7] = np.inf
    return x


def test_oracle_edge_signals_match_reference_runtime(reflib, tmp_path):
    fe = frontend(GEOMS["small"][0])
    x = edge_signals(fe["nsamp"])
    want, _ = reference_images(tmp_path, fe, x, 1)
    got = oracle_op(fe, 1).run(x, 0)
    assert bits_equal(got, want), mismatch_report(got, want)


def test_log_modes_differ_by_one_ulp_at_most():
    """every float in [0.5, 2) and 2^20 random positive floats: the correctly rounded log and this host's logf differ
    by at most one unit in the last place"""
    x = np.concatenate([np.arange(0x3f000000, 0x40000000, dtype=np.uint32).view(np.float32),
                        np.random.default_rng(0).integers(1, 0x7f800000, 1 << 20, dtype=np.uint32).view(np.float32)])
    a, b = oracle.log_f32(x, 0), oracle.log_f32(x, 1)
    d = np.abs(a.view(np.int32).astype(np.int64) - b.view(np.int32).astype(np.int64))
    assert d.max() <= 1
    assert np.array_equal(np.isnan(a), np.isnan(b))


@pytest.mark.parametrize("geom", ["small", "zero_pad", "upsample"])
def test_log_modes_images_close(geom):
    kw, halo = GEOMS[geom]
    fe = frontend(kw)
    x = signal(3, fe["nsamp"], 13)
    op = oracle_op(fe, halo)
    ok, bad = close_to(op.run(x, 1), op.run(x, 0))
    assert ok, f"{bad} pixels outside the tolerance"


def init_error(path):
    with pytest.raises(BnnError) as e:
        Model(path, mode=MODE_INT8)
    return e.value


def test_dbimg_validation_errors(tmp_path):
    """fe_db_init's checks (src/rt_ops_f32x.c:24-49) with the reference's messages"""
    fe = frontend(GEOMS["small"][0])
    path = str(tmp_path / "db.bnpk")
    synth.write_dbimg_package(path, fe)
    if not gpu_visible():
        e = init_error(path)
        assert e.kind == "CPU" and "no CUDA device" in str(e)
    off = pkgread.op_offsets(path)[0]
    with open(path, "rb") as f:
        data = bytearray(f.read())
    _, _, nb, nt, ni, _ = struct.unpack("<6H", bytes(data[off:off + 12]))
    assert (nb, nt, ni) == (2, 4, 21)
    ints = off + 12 + 4 * (nb + nt)
    for k, val, text in ((1, 1000, "(N & (N - 1)) == 0"), (5, 77, "nfr == (nsamp + 2 * pad - N) / hop + 1"),
                         (4, 0, "(padmode || !pad)"), (13, 0, "p[13] == 1"), (19, 2, "ld >= C"),
                         (20, 4, "h <= 3"), (10, 5, "p[10] <= 4"), (6, 50, "tensor argument 1"),
                         (14, 47, "buffer argument 1 (buffer #1, image): expected 47 x 64, ld 4, halo 0; found 48 x 64")):
        d = bytearray(data)
        d[ints + 4 * k:ints + 4 * k + 4] = struct.pack("<i", val)
        p = tmp_path / f"i{k}.bnpk"
        p.write_bytes(bytes(d))
        e = init_error(str(p))
        assert e.kind == "PACKAGE" and text in str(e) and "op 0 fe_dbimg" in str(e), (k, str(e))
    bad = dict(fe, rows=np.array([0, 3, 40], np.int32))
    p = str(tmp_path / "rows.bnpk")
    synth.write_dbimg_package(p, bad)
    e = init_error(p)
    assert e.kind == "PACKAGE" and "row table entry 2 = 40 outside 0..39" in str(e), str(e)


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


def run_op(h, fe, x, halo=0, batch=None):
    tens, ints, _, _ = synth.dbimg_record(fe, halo)
    p = np.array(ints, np.int32)
    arrs = [np.ascontiguousarray(tens[k]) for k in ("window", "mel", "rows", "consts")]
    op = h.bnn_dbimg_new(p.ctypes.data, 21, *[a.ctypes.data for a in arrs], batch or x.shape[0])
    assert op, h.bnn_last_error()
    try:
        elems = h.bnn_dbimg_image_elems(op)
        d_x = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        d_i = torch.full((x.shape[0], elems + 5), 7.0, dtype=torch.float32, device="cuda")
        assert h.bnn_dbimg_run(op, x.shape[0], d_x.data_ptr(), x.shape[1], d_i.data_ptr(), elems + 5, None) == 0, \
            h.bnn_last_error()
        torch.cuda.synchronize()
        out = d_i.cpu().numpy()
        assert (out[:, elems:] == 7.0).all()
        return out[:, :elems]
    finally:
        h.bnn_dbimg_free(op)


@pytest.mark.gpu
@pytest.mark.parametrize("geom", sorted(GEOMS))
def test_dbimg_op(lib, geom):
    """the per-op C ABI: bit for bit against the oracle with the correctly rounded log, within the tolerance against
    the oracle with the reference's logf"""
    kw, halo = GEOMS[geom]
    fe = frontend(kw)
    x = signal(5, fe["nsamp"], len(geom))
    got = run_op(lib, fe, x, halo)
    op = oracle_op(fe, halo)
    want = op.run(x, 1)
    assert bits_equal(got, want), mismatch_report(got, want)
    ok, bad = close_to(got, op.run(x, 0))
    assert ok, f"{bad} pixels outside the tolerance against the reference's logf"


@pytest.mark.gpu
def test_dbimg_edge_signals(lib):
    fe = frontend(GEOMS["small"][0])
    x = edge_signals(fe["nsamp"])
    got = run_op(lib, fe, x, 1)
    want = oracle_op(fe, 1).run(x, 1)
    assert bits_equal(got, want), mismatch_report(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["dbimg_small", "dbimg_zero", "dbimg_none"])
def test_dbimg_package(lib, name, tmp_path):
    """the reference compiler's package bytes through bnn_infer_batch (chunks of 3 windows)"""
    fe = frontend(PACKAGES[name]["frontend"])
    path = str(tmp_path / f"{name}.bnpk")
    n_out = synth.write_dbimg_package(path, fe)
    x = signal(7, fe["nsamp"], 5)
    with Model(path, mode=MODE_INT8, batch=3) as m:
        got, _ = m.infer_batch(x)
        assert m.launches_per_batch == 3
    oracle.set_log_mode(1)
    try:
        want, _ = oracle.run_many(path, x, threads=4)
    finally:
        oracle.set_log_mode(0)
    assert got.shape == (7, n_out) and bits_equal(got, want), mismatch_report(got, want)


@pytest.mark.gpu
def test_dbimg_v3_geometry_batch64(lib):
    """the v3.0 front end at batch 64, eight sampled windows against the oracle"""
    fe = frontend(PACKAGES["dbimg_v3"]["frontend"])
    x = signal(64, fe["nsamp"], 21)
    got = run_op(lib, fe, x)
    idx = [0, 1, 17, 31, 32, 50, 62, 63]
    op = oracle_op(fe)
    want = op.run(x[idx], 1)
    assert bits_equal(got[idx], want), mismatch_report(got[idx], want)
    ok, bad = close_to(got[idx], op.run(x[idx], 0))
    assert ok, f"{bad} pixels outside the tolerance against the reference's logf"


@pytest.mark.gpu
def test_device_log_correctly_rounded(lib):
    """bnn_cuda_fn 9 (the kernel's logarithm) against the oracle's correctly rounded log on every float in [0.5, 2),
    2^22 random positive floats, subnormals, zero, inf and NaN; and the count of inputs where it differs from this
    host's logf"""
    rng = np.random.default_rng(1)
    x = np.concatenate([np.arange(0x3f000000, 0x40000000, dtype=np.uint32).view(np.float32),
                        rng.integers(1, 0x7f800000, 1 << 22, dtype=np.uint32).view(np.float32),
                        np.arange(1, 4096, dtype=np.uint32).view(np.float32),
                        np.array([0.0, -0.0, np.inf, -1.0, np.nan, 1e-45, 3.4e38], np.float32)])
    d_x = torch.from_numpy(x).cuda()
    d_y = torch.empty_like(d_x)
    assert lib.bnn_cuda_fn(9, x.size, d_x.data_ptr(), d_y.data_ptr(), None) == 0
    torch.cuda.synchronize()
    got = d_y.cpu().numpy()
    want = oracle.log_f32(x, 1)
    assert bits_equal(got, want), mismatch_report(got, want)
    glibc = oracle.log_f32(x, 0)
    diff = int((got.view(np.int32) != glibc.view(np.int32)).sum() - (np.isnan(got) & np.isnan(glibc)).sum())
    print(f"device log vs this host's logf: {diff} of {x.size} inputs differ (one ulp)")
