"""The fp16 body of a Perch-v2-architecture package (neon-fp16 with the int8 prototype head) on the CPU: the oracle's
whole model against a float64 forward pass of the same weights, and the library's loader on its records (the checks
and messages of src/rt_ops_f16.c and src/rt_ops_f32.c) before any device is touched.

Parity of the new fp16 ops is pinned like the rest of the fp16 path: by construction (every fp16 operation rounded
once, in the order of src/pc_kern_f16.c) and by tolerance against float64.
"""
import struct

import numpy as np
import pytest

from bnneon_b200 import synth
from oracle import oracle


@pytest.fixture(scope="module")
def perch_mini(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("perch") / "perch_mini.bnpk")
    ir = synth.perch_ir(0, mini=True)
    synth.write_perch_package(path, ir)
    return path, ir


def sqnr_db(got, want):
    return 10 * np.log10(np.sum(want ** 2) / max(np.sum((got - want) ** 2), 1e-300))


def f64_forward(ir, spec):
    """the Perch IR in float64 numpy from the front end's spectrogram [frames][nmel]: (logits, embedding, cells)"""
    ops, vshape = ir[0], ir[1]
    vals = {ops[0]["out"]: spec.astype(np.float64)[:, :, None]}
    swish = lambda v: v / (1.0 + np.exp(-v))  # noqa: E731
    for o in ops[1:]:
        x = vals[o["ins"][0]]
        if o["op"] == "CONV" and o["k"] != [1, 1]:  # the VALID stem
            k, s = o["k"][0], o["s"][0]
            ho, wo = vshape[o["out"]]
            y = np.zeros((ho, wo, o["w"].shape[0])) + o["b"]
            for ky in range(k):
                for kx in range(k):
                    y += x[ky:ky + s * (ho - 1) + 1:s, kx:kx + s * (wo - 1) + 1:s, :] @ o["w"][:, :, ky, kx].T
            vals[o["out"]] = swish(y)
        elif o["op"] == "CONV":
            y = x @ o["w"][:, :, 0, 0].T.astype(np.float64) + o["b"]
            y = swish(y) if o.get("act") == "swish" else y
            vals[o["out"]] = y + (vals[o["res"]] if o.get("res") else 0)
        elif o["op"] == "DWCONV":
            k, s = o["k"][0], o["s"][0]
            pt, pl, pb, pr = o["pads"]
            xp = np.pad(x, ((pt, pb), (pl, pr), (0, 0)))
            ho, wo = vshape[o["out"]]
            y = np.zeros((ho, wo, x.shape[2])) + o["b"]
            for ky in range(k):
                for kx in range(k):
                    y += xp[ky:ky + s * (ho - 1) + 1:s, kx:kx + s * (wo - 1) + 1:s, :] * o["w"][:, 0, ky, kx]
            vals[o["out"]] = swish(y)
        elif o["op"] == "SE":
            m = x.mean((0, 1))
            g = 1.0 / (1.0 + np.exp(-(o["w2"] @ swish(o["w1"] @ m + o["b1"]) + o["b2"])))
            vals[o["out"]] = x * g
        elif o["op"] == "MEAN":
            vals[o["out"]] = x.mean((0, 1))
        elif o["op"] == "PROTO":
            cells = x.reshape(-1, x.shape[2])
            a = cells / (np.sqrt((cells ** 2).sum(1, keepdims=True)) + o["eps"])
            sims = (a @ o["P"].T.astype(np.float64)).max(0)
            nc, ppc = o["cw"].shape
            vals[o["out"]] = (sims.reshape(nc, ppc) * o["cw"]).sum(1) + o["cb"]
    return vals[ir[2]], vals[ir[3]]


def test_perch_oracle_tracks_float64_model(perch_mini):
    """The oracle's mini Perch model (fp32 stem, fp16 body, int8 prototype head) against float64 on the same
    spectrogram. Tolerance: the embedding (the fp16 body's output) within 50 dB SQNR -- the reference compiler's own
    screen for an fp16 layer (lower.py:69-71 need_db = 50.0) -- and the logits, which also carry the int8
    quantization of cells and prototypes, within 30 dB. (Measured: 58 dB on the embedding, 38 dB on the logits.)"""
    path, ir = perch_mini
    pcm = synth.audio(1, seed=5, n_samples=ir[4]["nsamp"], rate=synth.PERCH_SAMPLE_RATE)[0]
    p = oracle.Package(path, "neon-fp16")
    p.run_range(pcm, 0, 1)
    spec = p.get(1)[:ir[1][ir[0][0]["out"]][0] * ir[1][ir[0][0]["out"]][1]]
    spec = spec.reshape(ir[1][ir[0][0]["out"]])
    got, emb = p.run(pcm)
    want, wemb = f64_forward(ir, spec)
    print("embedding", sqnr_db(emb, wemb), "logits", sqnr_db(got, want))
    assert sqnr_db(emb, wemb) >= 50, sqnr_db(emb, wemb)
    assert sqnr_db(got, want) >= 30, sqnr_db(got, want)


def test_perch_package_ops_and_loader(tmp_path, perch_mini):
    """Every op kind of the Perch body is in the mini package; the library accepts its records (with no GPU it stops
    only at the device) and checks each new record as the reference does (the same messages)."""
    from conftest import gpu_visible  # pylint: disable=import-outside-toplevel
    from bnneon_b200 import BnnError, Model, pkgread  # pylint: disable=import-outside-toplevel
    path, _ = perch_mini
    ops, _ = pkgread.read_ops(path, synth.PATH_F16)
    codes = [o[0] for o in ops]
    for c in (8, 0x109, 0x103, 0x104, 0x105, 0x10A, 0x10B, 0x10C, 0x20D):
        assert c in codes, hex(c)
    assert any(o[0] == 0x10A and o[3][3] == 5 for o in ops)  # a 5x5 depthwise conv
    assert any(o[0] == 0x10A and o[3][3] == 3 and o[3][2] > 2048 for o in ops)  # DWK 3x3 above 2048 channels
    if not gpu_visible():
        with pytest.raises(BnnError) as e:
            Model(path, mode=3)
        assert e.value.kind == "CPU" and "no CUDA device" in str(e.value)
    offs = pkgread.op_offsets(path, synth.PATH_F16)
    with open(path, "rb") as f:
        data = f.read()
    first = {code: i for i, (code, _, _, _) in reversed(list(enumerate(ops)))}
    cases = [(0x109, 8, 2, "K == k * k", "stem_f32to16"), (0x109, 10, 3, "p[10] >= 0 && p[10] <= 2", "stem_f32to16"),
             (0x10A, 3, 4, "k % 2 == 1 && k >= 1 && k <= 7", "dwk_f16"),
             (0x10A, 5, 3, "pt >= 0 && pt <= h && pl >= 0 && pl <= h", "dwk_f16"),
             (0x10A, 2, 12, "C % 8 == 0", "dwk_f16"),
             (0x10B, 4, 4, "p[4] >= 1 && p[4] <= 3", "pad_f16"), (0x10B, 3, 8, "p[3] >= p[2]", "pad_f16"),
             (0x10C, 1, 6, "p[1] % 4 == 0", "mean_f16"),
             (0x20D, 3, 12, "P % 8 == 0 && Np % 12 == 0 && Np >= N", "proto_s8"),
             (0x20D, 1, 1544, "K == C", "proto_s8")]
    for code, k, val, text, kname in cases:
        i = first[code]
        _, _, nb, nt, _, _ = struct.unpack_from("<6H", data, offs[i])
        at = offs[i] + 12 + 4 * (nb + nt + k)
        d = bytearray(data)
        d[at:at + 4] = struct.pack("<i", val)
        p = tmp_path / f"c{code:x}_{k}.bnpk"
        p.write_bytes(bytes(d))
        with pytest.raises(BnnError) as e:
            Model(str(p), mode=3)
        assert e.value.kind == "PACKAGE" and text in str(e.value) and f"op {i} {kname}" in str(e.value), str(e.value)


def test_perch_path_needs_dotprod_flag(tmp_path, perch_mini):
    """The int8 prototype head (opcode 0x20d) in a path that declares only fp16 is refused, as src/rt_pkg.c:449-455
    refuses it."""
    from bnneon_b200 import BnnError, Model  # pylint: disable=import-outside-toplevel
    path, _ = perch_mini
    with open(path, "rb") as f:
        data = bytearray(f.read())
    path_off = struct.unpack_from("<4Q", data, 32)[2]
    assert struct.unpack_from("<I", data, path_off + 24)[0] == 3
    struct.pack_into("<I", data, path_off + 24, 1)
    p = tmp_path / "nodot.bnpk"
    p.write_bytes(bytes(data))
    with pytest.raises(BnnError) as e:
        Model(str(p), mode=3)
    assert "dotprod kernel (opcode 0x20d)" in str(e.value), str(e.value)


def test_dwk_and_stem_entry_points_check_shapes_without_a_device():
    """bnn_cuda_dwk_f16 / bnn_cuda_stem_f16 refuse shapes the reference's checks refuse before touching a device"""
    from bnneon_b200 import load_library  # pylint: disable=import-outside-toplevel
    h = load_library()
    cases = [  # (args, text in the message)
        ((1, 1, 0, 8, 8, 12, 3, 1, 1, 1, 1, 1, 1, 1, 0, 8, 8, 1, 0, None), "C % 8 == 0"),
        ((1, 1, 0, 8, 8, 8, 4, 1, 1, 1, 1, 1, 1, 1, 0, 8, 8, 1, 0, None), "k odd"),
        ((1, 1, 0, 8, 8, 8, 3, 3, 1, 1, 1, 1, 1, 1, 0, 3, 3, 1, 0, None), "s 1|2"),
        ((1, 1, 0, 8, 8, 8, 3, 1, 2, 1, 1, 1, 1, 1, 0, 8, 8, 1, 0, None), "pt and pl"),
        ((1, 1, 0, 8, 8, 8, 3, 1, 1, 1, 1, 1, 1, 1, 0, 9, 8, 1, 0, None), "taps inside the halo"),
        ((1, 1, 0, 8, 4000, 8, 3, 1, 1, 1, 1, 1, 1, 1, 0, 8, 4000, 1, 0, None), "768 pixel groups"),
    ]
    for args, text in cases:
        assert h.bnn_cuda_dwk_f16(*args) == -1
        assert text in h.bnn_last_error().decode(), h.bnn_last_error()
    assert h.bnn_cuda_stem_f16(1, 1, 0, 8, 8, 3, 1, 7, 6, 1, 1, 8, 12, 1, 1, 0, 8, 0, None) == -1
    assert "VALID conv" in h.bnn_last_error().decode()
    assert h.bnn_cuda_stem_f16(1, 1, 0, 8, 8, 3, 1, 6, 6, 1, 1, 8, 8, 1, 1, 0, 8, 0, None) == -1  # Kp < k k
    assert h.bnn_cuda_stem_f16(1, 1, 0, 200, 200, 3, 1, 6, 6, 1, 1, 1024, 12, 1, 1, 0, 1024, 0, None) == -1  # > 48 KB
    assert "48 KB" in h.bnn_last_error().decode()
    # two windows whose strides are shorter than a window
    assert h.bnn_cuda_dwk_f16(2, 1, 100, 8, 8, 8, 3, 1, 1, 1, 1, 1, 1, 1, 512, 8, 8, 1, 8, None) == -1
    assert "at least one window" in h.bnn_last_error().decode()
    assert h.bnn_cuda_stem_f16(2, 1, 50, 8, 8, 3, 1, 6, 6, 1, 1, 8, 12, 1, 1, 288, 8, 0, None) == -1
    assert "at least one window" in h.bnn_last_error().decode()



def op_macs(code, p):
    """(class, MACs per window) of one op record of the Perch package"""
    if code == 0x103:  # PW: M K N
        return "1x1", p[4] * p[1] * p[0]
    if code == 0x104:  # DW3: Ho Wo C 9
        return "dw3x3", p[4] * p[5] * p[2] * 9
    if code == 0x10A:  # DWK: Ho Wo C k k
        return f"dw{p[3]}x{p[3]}", p[7] * p[8] * p[2] * p[3] * p[3]
    if code == 0x109:  # STEM: Ho Wo N K
        return "stem", p[6] * p[7] * p[0] * p[1]
    if code == 0x20D:  # PROTO: cells K prototypes
        return "proto", p[3] * p[1] * p[0]
    return None, 0


def test_perch_package_has_perch_v2_work(tmp_path):
    """The full synthetic package does Perch v2's work: per window, the MACs of its op records against the reference's
    published table for the Perch v2 graph (results/perch_mac_table.txt:2-13: 1x1 convs 1096.3 + head conv 37.7, dw 5x5
    56.2, dw 3x3 36.0, stem 5.6 MMAC, body 1233 MMAC, prototype head 5817.6 MMAC)."""
    from bnneon_b200 import pkgread  # pylint: disable=import-outside-toplevel
    path = str(tmp_path / "perch_full.bnpk")
    synth.make_perch_package(path, seed=0)
    ops, _ = pkgread.read_ops(path, synth.PATH_F16)
    mac, body = {}, 0.0
    for code, _, _, p in ops:
        k, m = op_macs(code, p)
        if k:
            mac[k] = mac.get(k, 0.0) + m / 1e6
            body += m / 1e6 if k != "proto" else 0.0
    assert abs(mac["1x1"] - (1096.3 + 37.7)) / 1134.0 < 0.005, mac
    assert abs(mac["dw5x5"] - 56.2) / 56.2 < 0.01, mac
    assert abs(mac["dw3x3"] - 36.0) / 36.0 < 0.01, mac
    assert abs(mac["stem"] - 5.6) / 5.6 < 0.02, mac
    assert abs(body - 1233.0) / 1233.0 < 0.005, (body, mac)
    assert abs(mac["proto"] - 5817.6) / 5817.6 < 1e-4, mac
