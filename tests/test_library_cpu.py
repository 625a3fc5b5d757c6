"""CPU tests of libbnneon.so: exports, probe / metadata / labels, and the loader's and validator's error contract
(fault injection by package mutation, as the reference's tests/test_errors.py does). No GPU is needed: a valid
package passes validation and then stops at the device check."""
import os
import re
import struct

import pytest

from conftest import REPO, gpu_visible
from bnneon_b200 import BnnError, Model, load_library, pkgread, probe, probe_meta, synth, verify_labels


def declared_functions():
    names = set()
    for h in ("bnneon.h", "bnneon_cuda.h"):
        with open(os.path.join(REPO, "include", h), encoding="utf-8") as f:
            text = f.read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(bnn_\w+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_exports_every_declared_function():
    h = load_library()
    names = declared_functions()
    assert len(names) >= 30
    missing = [n for n in sorted(names) if not hasattr(h, n)]
    assert not missing, missing


def test_api_version_and_families():
    h = load_library()
    assert h.bnn_api_version() == 2
    assert h.bnn_cpu_supported(24) == 1 and h.bnn_cpu_supported(120) == 1 and h.bnn_cpu_supported(99) == 0


def test_probe_and_metadata(mini_pkg):
    i = probe(mini_pkg)
    assert (i.model, i.format_version, i.sample_rate, i.n_samples, i.n_classes, i.emb_dim, i.post) == \
        (24, 1, 48000, 144000, 64, 1024, 1)
    assert i.path == b"neon-int8" and i.has_labels_sha == 1 and i.logit_scale == 1.0
    assert probe_meta(mini_pkg, "model_id") == b"birdnet_v2.4_synthetic"
    assert probe_meta(mini_pkg, "licence") == probe_meta(mini_pkg, "license")  # either spelling
    assert probe_meta(mini_pkg, "labels") == synth.labels_for(64)
    assert probe_meta(mini_pkg, "n_classes") == b"64"
    assert probe_meta(mini_pkg, "no_such_key") is None


def test_struct_size_handshake(mini_pkg):
    import ctypes  # pylint: disable=import-outside-toplevel
    from bnneon_b200 import Info  # pylint: disable=import-outside-toplevel
    h = load_library()
    info = Info()
    info.struct_size = 24  # an old host that knows the first fields only
    assert h.bnn_probe(mini_pkg.encode(), ctypes.byref(info)) == 0
    assert info.struct_size == 24 and info.n_samples == 144000 and info.n_classes == 0
    info.struct_size = 4
    assert h.bnn_probe(mini_pkg.encode(), ctypes.byref(info)) == -1 and h.bnn_last_error_kind() == 6


def test_verify_labels(mini_pkg, tmp_path):
    good = tmp_path / "labels.txt"
    good.write_bytes(synth.labels_for(64))
    verify_labels(mini_pkg, str(good))
    bad = tmp_path / "bad.txt"
    bad.write_bytes(synth.labels_for(63))
    with pytest.raises(BnnError) as e:
        verify_labels(mini_pkg, str(bad))
    assert e.value.kind == "LABELS" and "is not the label file" in str(e.value)


def init_error(path, mode=0):
    with pytest.raises(BnnError) as e:
        Model(path, mode=mode)
    return e.value


def test_valid_package_stops_at_device_check(mini_pkg):
    """On a machine without a GPU a valid package passes every check and then reports the missing device."""
    if gpu_visible():
        pytest.skip("a GPU is present")
    e = init_error(mini_pkg)
    assert e.kind == "CPU" and "no CUDA device" in str(e)


def mutate(src, dst, at, data):
    with open(src, "rb") as f:
        b = bytearray(f.read())
    if at is None:
        b = b[:data]
    else:
        b[at:at + len(data)] = data
    with open(dst, "wb") as f:
        f.write(b)
    return str(dst)


def test_loader_errors(mini_pkg, tmp_path):
    size = os.path.getsize(mini_pkg)
    cases = [
        (0, b"NOTAPKG!", "PACKAGE", "not a bnneon weights file"),
        (8, struct.pack("<I", 0x04030201), "PACKAGE", "byte-order mark"),
        (14, struct.pack("<H", 2), "PACKAGE", "needs reader version 2"),
        (None, size - 100, "PACKAGE", "package truncated"),
        (0, b"BN24ENG1", "PACKAGE", "legacy BirdNET v2.4"),
    ]
    for k, (at, data, kind, text) in enumerate(cases):
        p = mutate(mini_pkg, tmp_path / f"m{k}.bnpk", at, data)
        e = init_error(p)
        assert e.kind == kind and text in str(e), (k, str(e))
        with pytest.raises(BnnError):
            probe(p)


def op_field(pkg, op, field):
    """File offset of int field `field` of op record `op` (header 12 bytes, then buffers, tensors, ints)."""
    off = pkgread.op_offsets(pkg)[op]
    with open(pkg, "rb") as f:
        f.seek(off)
        code, _, nb, nt, ni, _ = struct.unpack("<6H", f.read(12))
    return off, code, nb, nt, ni


def test_validation_errors(mini_pkg, tmp_path):
    ops, _ = pkgread.read_ops(mini_pkg)
    i = next(k for k, o in enumerate(ops) if o[0] == 22)  # the first PW_S8 (p0)
    off, code, nb, nt, ni = op_field(mini_pkg, i, 0)
    act_at = off + 12 + 4 * (nb + nt) + 4 * 6  # int param 6 = act
    p = mutate(mini_pkg, tmp_path / "act.bnpk", act_at, struct.pack("<i", 7))
    e = init_error(p)
    assert e.kind == "PACKAGE" and f"op {i} pw_s8n (ONNX node 'v24/p0')" in str(e) and "act <= 2" in str(e)
    assert "int params: [" in str(e)
    p = mutate(mini_pkg, tmp_path / "k.bnpk", off + 12 + 4 * (nb + nt) + 4, struct.pack("<i", 32))  # K 48 -> 32
    e = init_error(p)
    assert "expected Np = N rounded up to 8, Kp = K rounded up to 16" in str(e)
    p = mutate(mini_pkg, tmp_path / "op.bnpk", off, struct.pack("<H", 29))  # WINO_S8 (dotprod family): no GPU kernel
    e = init_error(p)  # the path picker skips paths with ops this library has no kernel for
    assert e.kind == "CPU" and "runs none of the package's paths" in str(e)
    p = mutate(mini_pkg, tmp_path / "buf.bnpk", off + 12, struct.pack("<i", 9999))
    e = init_error(p)
    assert "names buffer #9999" in str(e)
    p = mutate(mini_pkg, tmp_path / "req.bnpk", off + 12 + 4, struct.pack("<i", -1))  # the output: required
    e = init_error(p)
    assert "required by the kernel but absent" in str(e)


def test_mode_errors(mini_pkg):
    e = init_error(mini_pkg, mode=1)
    assert e.kind == "USAGE" and "mode 1" in str(e)
    e = init_error(mini_pkg, mode=3)
    assert e.kind == "CPU" and "path neon-fp16 is not in this package" in str(e)
    e = init_error(mini_pkg, mode=9)
    assert e.kind == "USAGE"


def test_missing_file():
    e = init_error("/nonexistent/model.bnpk")
    assert e.kind == "PACKAGE" and "cannot open" in str(e)
