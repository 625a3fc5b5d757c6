"""The int8 prototype head (PROTO_S8) without a GPU: the packer and the oracle against the reference's own packer and
lowering (tests/golden/proto_packing.npz, proto_packages.json, made by tests/golden/make_golden.py from the reference
compiler), the oracle's quantizer rules, and the loader's checks of PROTO_S8 records."""
import hashlib
import json
import os
import struct

import numpy as np
import pytest

from conftest import gpu_visible

from bnneon_b200 import BnnError, Model, pkgread, synth
from oracle import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
PACKING = np.load(os.path.join(HERE, "golden", "proto_packing.npz"))
with open(os.path.join(HERE, "golden", "proto_packages.json"), encoding="utf-8") as fh:
    PACKAGES = json.load(fh)
N_MATS = len([k for k in PACKING.files if k.startswith("qp")])


def proto_pkg(tmp_path, name):
    g = PACKAGES[name]
    head = synth.proto_head(g["seed"], g["cells"], g["channels"], g["classes"], g["ppc"], g["eps"])
    path = str(tmp_path / f"{name}.bnpk")
    synth.write_proto_package(path, head, g["ld"])
    return path, head, g


@pytest.mark.parametrize("i", range(N_MATS))
def test_proto_packing_matches_reference_packer(i):
    w = PACKING[f"w{i}"]
    qp, sw, n4, q = synth.pack_proto_s8(w)
    assert np.array_equal(q, PACKING[f"q{i}"])
    assert np.array_equal(sw.view(np.int32), PACKING[f"sw{i}"].view(np.int32))
    assert np.array_equal(n4, PACKING[f"n4_{i}"])
    assert np.array_equal(qp, PACKING[f"qp{i}"])
    assert np.array_equal(oracle.proto_unpack(PACKING[f"qp{i}"]), PACKING[f"q{i}"])


@pytest.mark.parametrize("i", (0, 4))
def test_sdot_packing_matches_reference_packer(i):
    """PROTO variant 2's prototype tensors (lower.py proto_s8: [Np/12][K/4][12][4], Np = N rounded up to 12)."""
    qp, sw, q = synth.pack_proto_s8_sdot(PACKING[f"w{i}"])
    assert np.array_equal(qp, PACKING[f"sdot_qp{i}"])
    assert np.array_equal(sw.view(np.int32), PACKING[f"sdot_sw{i}"].view(np.int32))
    rows = np.empty(q.shape, np.int8)
    oracle.lib().bnno_proto_unpack12(oracle.ptr(np.ascontiguousarray(qp)), q.shape[0], q.shape[1], oracle.ptr(rows))
    assert np.array_equal(rows, q)


def test_proto_rounding_reference_vectors():
    """Ties go away from zero and nothing maps to -128 (the reference's tests/test_lower_s8.py rules)."""
    q = PACKING["q2"]
    assert q[0, 1] == 127 and q[0, 0] == 3 and q[0, 2] == 1 and q[0, 3] == 1  # 127 * 2.5 / 127 = 2.5 -> 3
    for i in range(N_MATS):
        assert PACKING[f"q{i}"].min() >= -127


def test_n4_check_matches_reference_flags():
    """Panels the reference packer flags pass the loader's lane check; a flag planted on a panel whose lanes exceed
    258 is caught (oracle and library restate pc_proto_n4_check)."""
    h = oracle.lib()
    for i in range(N_MATS):
        qp = np.ascontiguousarray(PACKING[f"qp{i}"])
        n4 = np.ascontiguousarray(PACKING[f"n4_{i}"]).astype(np.uint8)
        kp = qp.shape[1] * 16
        assert h.bnno_proto_n4_check(oracle.ptr(qp), kp, oracle.ptr(n4), n4.size) == -1
    qp = np.ascontiguousarray(PACKING["qp4"])
    n4 = PACKING["n4_4"].astype(np.uint8).copy()
    assert n4[0] == 0
    n4[0] = 1
    assert h.bnno_proto_n4_check(oracle.ptr(qp), 128, oracle.ptr(n4), n4.size) == 0
    # -128 counts 128 (vabsq_s8 wraps, then the lane is read unsigned): 2 x 128 + 2 x 1 = 258 passes, 259 does not
    qp = np.zeros((1, 2, 4, 16), np.int8)
    qp[0, 0, 0, 0] = -128
    qp[0, 0, 0, 8] = -128
    qp[0, 1, 0, 0] = 1
    qp[0, 1, 0, 8] = 1
    one = np.ones(1, np.uint8)
    assert h.bnno_proto_n4_check(oracle.ptr(qp), 32, oracle.ptr(one), 1) == -1
    qp[0, 1, 0, 8] = 2
    assert h.bnno_proto_n4_check(oracle.ptr(qp), 32, oracle.ptr(one), 1) == 0
    qp = np.zeros((1, 3, 4, 16), np.int8)  # Kp 48: the n4 loop is never used, nothing is checked
    qp[:] = 127
    assert h.bnno_proto_n4_check(oracle.ptr(qp), 48, oracle.ptr(one), 1) == -1


@pytest.mark.parametrize("name", sorted(PACKAGES))
def test_proto_package_bytes_match_reference_compiler(tmp_path, name):
    path, _, g = proto_pkg(tmp_path, name)
    with open(path, "rb") as f:
        data = f.read()
    assert len(data) == g["size"] and hashlib.sha256(data).hexdigest() == g["sha256"]


def test_oracle_quantizer_rules():
    """pc_quant_cells_f32: q = FCVTAS(x * (127 / max|x|)) clamped to [-127, 127], zero past C; sx = max|x| / (127
    (||x|| + eps)); an all-zero cell gets max 1e-30; a cell with NaN gets max 1e-30 too (NaN fails mx > 0)."""
    rng = np.random.default_rng(5)
    P, C, ld, Kp = 8, 40, 44, 48
    x = (rng.standard_normal((P, ld)) * 3).astype(np.float32)
    x[1] = 0.0
    x[2, :C] = 0.0
    x[2, 0], x[2, 1], x[2, 2] = 127.0, 2.5, -2.5  # ties at .5 after scaling by 127 / 127
    x[3, 5] = np.nan
    x[4, 7] = np.float32(1e-38)
    x[4, :7] = 0.0
    x[4, 8:] = 0.0
    qa = np.full((P, Kp), 99, np.int8)
    sx = np.zeros(P, np.float32)
    oracle.lib().bnno_proto_quant_cells(oracle.ptr(x), P, C, ld, np.float32(1e-6), oracle.ptr(qa), Kp, oracle.ptr(sx))
    assert (qa[:, C:] == 0).all() and qa.min() >= -127
    assert qa[2, 0] == 127 and qa[2, 1] == 3 and qa[2, 2] == -3
    assert (qa[1] == 0).all() and sx[1] == np.float32(1e-30) / np.float32(127 * 1e-6)
    for p in (0, 5, 6, 7):
        r = x[p, :C]
        mx = np.abs(r).max()
        v = r * (np.float32(127.0) / mx)
        want = np.clip(np.sign(v) * np.floor(np.abs(v) + np.float32(0.5)), -127, 127)
        assert np.array_equal(qa[p, :C], want.astype(np.int8)), p
        assert abs(sx[p] - mx / (127 * (np.sqrt((r.astype(np.float64) ** 2).sum()) + 1e-6))) < 1e-6 * sx[p]
    assert np.isnan(sx[3])
    assert qa[4, 7] == 127 and (qa[4, :7] == 0).all()


def init_error(path):
    with pytest.raises(BnnError) as e:
        Model(path, mode=4)
    return e.value


def test_proto_package_loads_until_device_check(tmp_path):
    if gpu_visible():
        pytest.skip("a GPU is present")
    path, _, _ = proto_pkg(tmp_path, "proto_small")
    e = init_error(path)
    assert e.kind == "CPU" and "no CUDA device" in str(e)


def test_proto_validation_errors(tmp_path):
    """The loader refuses PROTO_S8 records as proto8n_init / rt_proto_geom do: a planted n4 flag on an unsafe panel, a
    prototype count that is not classes x prototypes per class, Kp that is not K rounded up to 16."""
    name = "proto_mid"
    g = PACKAGES[name]
    head = synth.proto_head(g["seed"], g["cells"], g["channels"], g["classes"], g["ppc"], g["eps"])
    head["P"][:4, :32] = 40.0  # the first panel's lanes exceed 258, so the packer does not flag it
    path = str(tmp_path / "unsafe.bnpk")
    synth.write_proto_package(path, head, g["ld"])
    ops, _ = pkgread.read_ops(path)
    assert ops[0][0] == synth.OPC_PROTO_S8
    with open(path, "rb") as f:
        data = bytearray(f.read())
    n4_name = b"s8n/proto.0.n4"
    toff = pkgread.tensor_offset(path, n4_name.decode())
    assert data[toff] == 0
    data[toff] = 1
    bad = tmp_path / "n4.bnpk"
    bad.write_bytes(bytes(data))
    e = init_error(str(bad))
    assert e.kind == "PACKAGE" and "prototype panel 0 is flagged for 4 products per int16 lane" in str(e)
    assert "op 0 proto_s8n" in str(e)
    off = pkgread.op_offsets(path)[0]
    code, _, nb, nt, ni, _ = struct.unpack("<6H", bytes(data[off:off + 12]))
    ints = off + 12 + 4 * (nb + nt)
    for k, val, text in ((7, g["classes"] - 1, "nc * ppc == (size_t)N"), (2, 272, "Kp == ((K + 15) & ~15)"),
                         (4, 62, "P % 4 == 0")):
        d = bytearray(data)
        d[toff] = 0
        d[ints + 4 * k:ints + 4 * k + 4] = struct.pack("<i", val)
        p = tmp_path / f"i{k}.bnpk"
        p.write_bytes(bytes(d))
        e = init_error(str(p))
        assert e.kind == "PACKAGE" and text in str(e), (k, str(e))
