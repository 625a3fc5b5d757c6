"""The oracle pinned to the reference's own code: oracle/liboracle.so (our C restatement, the checker of every GPU test)
against oracle/_ref/libbnneon_ref.so (the reference's unmodified C runtime compiled for this host by oracle/ref.mk,
NEON intrinsics through the scalar stand-in oracle/neon/arm_neon.h), bit for bit.

* whole packages through the reference's own C API (bnn_init / bnn_infer, src/bnneon.c:310-330): logits and
  embeddings of the v2.4-architecture neon-int8 packages (mini and full), the neon-fp16 packages (mini with an fp16 and
  with an fp32 head), the Perch-architecture neon-fp16 + int8-head package, the one-op PROTO_S8 and FE_LOGMEL packages;
* every buffer every op writes, for one window, from the reference's BNN_DUMP (src/rt_pkg.c:512-526) against the
  oracle's buffer after the same op: the int8 rows, scales and zero points of every PW_S8, every activation, channel
  sum and gate;
* the exported kernels on edge inputs: s8n_quant_rows / s8n_quant_rows_gate (src/gemm_s8n.c:15-63) on NaN, infinite,
  constant and huge rows; dw3x3_f32 (src/gemm_f32.c:378-411) on odd shapes; the SiLU of silu_rows_f32
  (src/gemm_f32.c:303-320) on special and random floats.

CPU only. Skipped when neither the built library nor a reference checkout to build it from is present.
"""
import ctypes
import json
import os

import numpy as np
import pytest

from conftest import bits_equal, mismatch_report
from bnneon_b200 import pkgread, synth
from oracle import oracle, ref

HERE = os.path.dirname(os.path.abspath(__file__))
MODE_FP16, MODE_INT8 = 3, 4


@pytest.fixture(scope="module")
def reflib():
    if ref.reference_checkout() is not None:
        ref.build()
    if not ref.available():
        pytest.skip("no reference build (oracle/_ref) and no reference checkout to build it from")
    h = ref.lib()
    P, I, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    # src/gemm_s8n.h:16-19, src/gemm_f32.h:48-49, src/gemm_f32.c:303
    h.s8n_quant_rows.restype, h.s8n_quant_rows.argtypes = None, [P, I, I, I, I, I, P, P, P]
    h.s8n_quant_rows_gate.restype, h.s8n_quant_rows_gate.argtypes = None, [P, I, I, I, I, I, P, P, P, P]
    h.dw3x3_f32.restype, h.dw3x3_f32.argtypes = None, [P, I, I, I, I, P, P, P, I, I, P]
    h.silu_rows_f32.restype, h.silu_rows_f32.argtypes = None, [P, SZ, I, P]
    return h


def compare_windows(pkg, mode, path_name, pcm):
    want, wemb = oracle.run_many(pkg, pcm, threads=min(8, pcm.shape[0]), path_name=path_name)
    got, gemb, rc = ref.run_many(pkg, mode, pcm, threads=min(8, pcm.shape[0]))
    assert not rc.any(), rc
    assert bits_equal(got, want), "logits: " + mismatch_report(got, want)
    assert bits_equal(gemb, wemb), "embeddings: " + mismatch_report(gemb, wemb)


def compare_ops(pkg, mode, path_name, pcm):
    """every buffer every op writes, right after the op, for one window"""
    dumps, (rc, _, _) = ref.dump_ops(pkg, mode, pcm)
    assert rc == 0
    ops, bufs = pkgread.read_ops(pkg, path_name)
    p = oracle.Package(pkg, path_name)
    checked = 0
    for i, (code, bl, _, prm) in enumerate(ops):
        p.run_range(pcm, i, i + 1)
        for a, b in enumerate(bl):
            if (i, a) not in dumps or (code not in (22, 23) and a in pkgread.SCRATCH.get(code, ())):
                continue  # im2col / GEMM / cell scratch (POSTPC, STEM, PROTO), not an op result
            _, dt = p.buf_info(b)
            got = np.frombuffer(dumps[(i, a)], dt)
            want = p.get(b)
            assert got.size == want.size, (i, a, got.size, want.size)
            if code == 23 and a >= 2:  # GEMV_S8 quantizes one row into q [4][Kp], sa [4], za [4] (rt_ops_s8n.c:136)
                got, want = got[:prm[2] if a == 2 else 1], want[:prm[2] if a == 2 else 1]
            _, H, W, _, ld, halo, _, elems = bufs[b]
            if H > 0 and W > 0 and (H + 2 * halo) * (W + 2 * halo) * ld < elems:
                # rows past the map: the reference's 8-row GEMM tiles store rows there that nothing reads
                n = (H + 2 * halo) * (W + 2 * halo) * ld
                got, want = got[:n], want[:n]
            if dt in (np.float32,):
                ok = bits_equal(got, want)
                msg = mismatch_report(got, want)
            else:
                ok = np.array_equal(got.view(np.uint8), want.view(np.uint8))
                msg = f"{int(np.sum(got != want))} of {got.size} differ"
            assert ok, f"op {i} ({pkgread.NAMES.get(code, code)}) argument {a} (buffer {b}): {msg}"
            checked += 1
    assert checked >= len(ops)  # every op wrote at least one buffer
    return checked


@pytest.fixture(scope="module")
def f16_mini(pkg_dir):
    path = str(pkg_dir / "v24_mini_f16_100.bnpk")
    synth.make_package(path, seed=1, mini=True, n_classes=100, path=synth.PATH_F16)
    return path


@pytest.fixture(scope="module")
def perch_mini(pkg_dir):
    path = str(pkg_dir / "perch_mini.bnpk")
    _, _, ns = synth.make_perch_package(path, seed=1, mini=True)
    return path, ns


def test_int8_mini_windows(reflib, mini_pkg):
    pcm = synth.audio(6, seed=31)
    pcm[4] = 0.0                       # silence: constant rows everywhere (the quantizer's degenerate branch)
    pcm[5] = np.sign(pcm[5]) * 0.999   # a clipped, square-wave window
    compare_windows(mini_pkg, MODE_INT8, synth.PATH, pcm)


def test_int8_mini_every_op(reflib, mini_pkg):
    compare_ops(mini_pkg, MODE_INT8, synth.PATH, synth.audio(1, seed=32)[0])


def test_int8_full_windows_and_every_op(reflib, full_pkg):
    compare_windows(full_pkg, MODE_INT8, synth.PATH, synth.audio(3, seed=33))
    compare_ops(full_pkg, MODE_INT8, synth.PATH, synth.audio(1, seed=34)[0])


def test_fp16_mini_windows_and_every_op(reflib, f16_mini):
    compare_windows(f16_mini, MODE_FP16, synth.PATH_F16, synth.audio(2, seed=35))
    compare_ops(f16_mini, MODE_FP16, synth.PATH_F16, synth.audio(1, seed=36)[0])


def test_fp16_mini_fp32_head(reflib, pkg_dir):
    path = str(pkg_dir / "v24_mini_f16_61.bnpk")
    synth.make_package(path, seed=1, mini=True, path=synth.PATH_F16)  # 61 classes: the fp32 DENSE head
    compare_windows(path, MODE_FP16, synth.PATH_F16, synth.audio(2, seed=37))


def test_perch_mini_windows_and_every_op(reflib, perch_mini):
    path, ns = perch_mini
    pcm = synth.audio(2, seed=38, n_samples=ns, rate=synth.PERCH_SAMPLE_RATE)
    compare_windows(path, MODE_FP16, synth.PATH_F16, pcm)
    compare_ops(path, MODE_FP16, synth.PATH_F16, pcm[0])


def load_golden(name):
    with open(os.path.join(HERE, "golden", name), encoding="utf-8") as f:
        return json.load(f)


@pytest.mark.parametrize("name", sorted(load_golden("proto_packages.json")))
def test_proto_packages(reflib, pkg_dir, name):
    """the PROTO_S8 heads written as the reference compiler writes them (tests/golden/proto_packages.json), windows
    of cells with ties, zeros and a NaN"""
    g = load_golden("proto_packages.json")[name]
    head = synth.proto_head(g["seed"], g["cells"], g["channels"], g["classes"], g["ppc"], g["eps"])
    path = str(pkg_dir / f"ref_{name}.bnpk")
    synth.write_proto_package(path, head, g["ld"])
    rng = np.random.default_rng(g["seed"])
    pcm = rng.standard_normal((4, g["cells"] * g["ld"])).astype(np.float32)
    pcm[1, : g["ld"]] = 0.0
    pcm[2] = np.round(pcm[2] * 4) / 4
    want, _ = oracle.run_many(path, pcm[:3], threads=3)
    got, _, rc = ref.run_many(path, MODE_INT8, pcm[:3], threads=3)
    assert not rc.any()
    assert bits_equal(got, want), mismatch_report(got, want)
    pcm[3, 5] = np.nan  # a failed window in both: non-finite logits (src/bnneon.c:313-325)
    with ref.Context(path, MODE_INT8) as c:
        assert c.infer(pcm[3])[0] != 0


@pytest.mark.parametrize("name", sorted(load_golden("logmel_packages.json")))
def test_logmel_packages(reflib, pkg_dir, name):
    """the FE_LOGMEL front ends written as the reference compiler writes them (tests/golden/logmel_packages.json)"""
    g = load_golden("logmel_packages.json")[name]
    fe = synth.logmel_frontend(g["nsamp"], g["frame"], g["hop"], g["pad"], g["nfft"], g["nmel"], floor=g["floor"],
                               scale=g["scale"])
    path = str(pkg_dir / f"ref_{name}.bnpk")
    synth.write_logmel_package(path, fe)
    rng = np.random.default_rng(7)
    t = np.arange(g["nsamp"]) / synth.PERCH_SAMPLE_RATE
    pcm = (0.05 * rng.standard_normal((3, g["nsamp"])) + 0.3 * np.sin(2 * np.pi * 1000.0 * t)).astype(np.float32)
    pcm[2] = 0.0
    want, _ = oracle.run_many(path, pcm, threads=3)
    got, _, rc = ref.run_many(path, MODE_INT8, pcm, threads=3)
    assert not rc.any()
    assert bits_equal(got, want), mismatch_report(got, want)


def test_quant_rows_edges(reflib):
    """s8n_quant_rows / _gate on rows the packages never produce"""
    rng = np.random.default_rng(40)
    K, Kp = 40, 48
    rows = [np.zeros(K), np.full(K, 3.5), np.full(K, -1e-38), rng.standard_normal(K) * 1e30,
            rng.standard_normal(K) * 1e-30, rng.standard_normal(K), np.linspace(-1, 1, K)]
    r = rng.standard_normal(K); r[7] = np.nan; rows.append(r)
    r = rng.standard_normal(K); r[3] = np.inf; rows.append(r)
    r = rng.standard_normal(K); r[3] = -np.inf; r[9] = np.inf; rows.append(r)
    r = np.full(K, 1.0); r[0] = 1.0000001; rows.append(r)
    r = rng.standard_normal(K); r[5] = 3.4e38; r[6] = -3.4e38; rows.append(r)
    x = np.ascontiguousarray(np.stack(rows).astype(np.float32))
    M = x.shape[0]
    gate = rng.uniform(-2, 2, K).astype(np.float32)
    for g in (None, gate):
        q1, sa1, za1 = np.zeros((M, Kp), np.int8), np.zeros(M, np.float32), np.zeros(M, np.int32)
        q2, sa2, za2 = np.zeros((M, Kp), np.int8), np.zeros(M, np.float32), np.zeros(M, np.int32)
        if g is None:
            reflib.s8n_quant_rows(oracle.ptr(x), K, 0, M, K, Kp, oracle.ptr(q1), oracle.ptr(sa1), oracle.ptr(za1))
        else:
            reflib.s8n_quant_rows_gate(oracle.ptr(x), K, 0, M, K, Kp, oracle.ptr(g), oracle.ptr(q1), oracle.ptr(sa1),
                                       oracle.ptr(za1))
        oracle.lib().bnno_quant_rows(oracle.ptr(x), K, M, K, Kp, oracle.ptr(g), oracle.ptr(q2), oracle.ptr(sa2),
                                     oracle.ptr(za2))
        assert np.array_equal(q1, q2), np.argwhere(q1 != q2)[:5]
        assert bits_equal(sa1, sa2), mismatch_report(sa1, sa2)
        assert np.array_equal(za1, za2), (za1, za2)


@pytest.mark.parametrize("H,W,C,s", [(5, 7, 16, 1), (9, 5, 40, 2), (6, 16, 72, 1), (3, 8, 24, 2), (1, 1, 8, 1)])
def test_dw3_shapes(reflib, H, W, C, s):
    rng = np.random.default_rng(H * 100 + W * 10 + C + s)
    Ho, Wo = (H - 1) // s + 1, (W - 1) // s + 1
    xp = np.zeros((H + 2, W + 2, C), np.float32)
    xp[1:-1, 1:-1] = rng.standard_normal((H, W, C)).astype(np.float32) * 2
    w = (rng.standard_normal((9, C)) * 0.5).astype(np.float32)
    b = (rng.standard_normal(C) * 0.1).astype(np.float32)
    o1, c1 = np.zeros(Ho * Wo * C, np.float32), np.zeros(C, np.float32)
    o2, c2 = np.zeros(Ho * Wo * C, np.float32), np.zeros(C, np.float32)
    reflib.dw3x3_f32(oracle.ptr(xp), H, W, C, s, oracle.ptr(w), oracle.ptr(b), oracle.ptr(o1), Ho, Wo, oracle.ptr(c1))
    oracle.lib().bnno_dw3(oracle.ptr(xp), H, W, C, s, oracle.ptr(w), oracle.ptr(b), oracle.ptr(o2), Ho, Wo,
                          oracle.ptr(c2))
    assert bits_equal(o1, o2), mismatch_report(o1, o2)
    assert bits_equal(c1, c2), mismatch_report(c1, c2)


def test_silu_special_floats(reflib):
    rng = np.random.default_rng(41)
    sp = np.array([0.0, -0.0, 1e-45, -1e-45, 1e-30, -1e-30, 60.0, -60.0, 61.0, -61.0, 87.5, -87.5, 88.7, -103.9,
                   126.0, -126.0, 127.5, 1e30, -1e30, 3.4e38, -3.4e38], np.float32)
    u = rng.integers(0, 2 ** 32, 20000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    x = np.concatenate([sp, u[np.isfinite(u)], (rng.standard_normal(4000) * 10).astype(np.float32)])
    x = np.ascontiguousarray(x[: x.size // 32 * 32])
    y = x.copy()
    reflib.silu_rows_f32(oracle.ptr(y), y.size, 8, None)
    want = oracle.fn("bnno_silu", x)
    assert bits_equal(y, want), mismatch_report(y, want)
