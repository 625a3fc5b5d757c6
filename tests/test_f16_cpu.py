"""The neon-fp16 path on the CPU: package bytes against the reference compiler (tests/golden/f16_packages.json, made
by tests/golden/make_golden.py with the reference's lower.py), the oracle's fp16 arithmetic against exact rational
arithmetic and numpy, its SiLU table against the reference's header and against x * sigmoid(x), and the oracle's
whole fp16 model against a float64 forward pass of the same weights.

The reference's fp16 kernels are AArch64 assembly (FMLA .8h) that cannot run here, so the fp16 oracle is pinned by
construction (every fp16 operation rounded once, in the reference's order, read from src/gemm_f16.c, src/kern_f16.c,
src/v24_fast.c) and by tolerance: its logits must stay within the stated SQNR of the float64 model.
"""
import hashlib
import json
import os
from fractions import Fraction

import numpy as np
import pytest

from bnneon_b200 import synth
from oracle import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "f16_packages.json"), encoding="utf-8") as fh:
    GOLD = json.load(fh)
MODELS = sorted(k for k in GOLD if k != "silu_lut")


def model_ir(g):
    return synth.v24_ir(g["seed"], g["head_classes"], synth.V24_BLOCKS if g["blocks"] == "full" else synth.MINI_BLOCKS)


@pytest.fixture(scope="module")
def f16_mini(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("f16") / "v24_mini_f16.bnpk")
    synth.write_f16_package(path, model_ir(GOLD["v24_mini_f16"]))
    return path


@pytest.mark.parametrize("name", [m for m in MODELS if "full" not in m])
def test_f16_package_bytes_match_reference_compiler(tmp_path, name):
    g = GOLD[name]
    path = str(tmp_path / f"{name}.bnpk")
    nc, emb = synth.write_f16_package(path, model_ir(g))
    with open(path, "rb") as f:
        data = f.read()
    assert (nc, emb) == (g["n_classes"], g["emb_dim"])
    assert len(data) == g["size"] and hashlib.sha256(data).hexdigest() == g["sha256"]


def test_f16_full_package_bytes_match_reference_compiler(tmp_path):
    g = GOLD["v24_full_f16"]
    path = str(tmp_path / "full.bnpk")
    synth.write_f16_package(path, model_ir(g))
    with open(path, "rb") as f:
        assert hashlib.sha256(f.read()).hexdigest() == g["sha256"]


def test_silu_table_is_the_reference_table():
    assert oracle.silu_table() == GOLD["silu_lut"]


# ------------------------------------------------------------------ fp16 arithmetic

def exact(h):
    """the exact value of fp16 bits h as a Fraction (finite only)"""
    s, e, m = h >> 15, (h >> 10) & 31, h & 1023
    v = Fraction(m, 1 << 24) if e == 0 else Fraction(m | 1024, 1) * Fraction(2) ** (e - 25)
    return -v if s else v


def round_half(x, neg_zero=False):
    """x (a Fraction) rounded to fp16 bits, nearest even"""
    if x == 0:
        return 0x8000 if neg_zero else 0
    s, a = (0x8000, -x) if x < 0 else (0, x)
    e = -14
    while a >= Fraction(2) ** (e + 1):
        e += 1
    q = round(a / Fraction(2) ** (e - 10))  # Fraction rounding: half to even
    if q == 2048:
        e, q = e + 1, 1024
    if e > 15:
        return s | 0x7C00
    return s | (((e + 14) << 10) + q) if q >= 1024 else s | q


def finite_halves(rng, n):
    h = rng.integers(0, 1 << 16, n, dtype=np.uint32).astype(np.uint16)
    h = h[(h & 0x7C00) != 0x7C00]
    small = rng.integers(0, 40, n // 4).astype(np.uint16) | (rng.integers(0, 2, n // 4).astype(np.uint16) << 15)
    return np.concatenate([h, small, np.array([0, 0x8000, 0x3C00, 0xBC00, 0x7BFF, 0xFBFF, 1, 0x8001], np.uint16)])


def test_h_fma_is_correctly_rounded():
    rng = np.random.default_rng(5)
    a, b, c = (finite_halves(rng, 1500) for _ in range(3))
    n = min(len(a), len(b), len(c))
    got = oracle.h_op("bnno_h_fma", a[:n], b[:n], c[:n])
    for i in range(n):
        p, cc = exact(int(a[i])) * exact(int(b[i])), exact(int(c[i]))
        x = p + cc
        neg0 = x == 0 and (p < 0 or (p == 0 and (int(a[i]) ^ int(b[i])) & 0x8000)) and bool(int(c[i]) & 0x8000)
        want = round_half(x, neg0)
        if want & 0x7C00 == 0x7C00:  # overflow: infinity of the sign
            assert got[i] == want, (hex(a[i]), hex(b[i]), hex(c[i]))
            continue
        if x == 0 or abs(x) < Fraction(1, 1 << 25):  # a zero result takes the sign of the exact value / IEEE sum rule
            assert got[i] & 0x7FFF == 0, (hex(a[i]), hex(b[i]), hex(c[i]))
            continue
        assert got[i] == want, (hex(a[i]), hex(b[i]), hex(c[i]), hex(got[i]), hex(want))


def test_h_add_mul_and_rounding_match_numpy():
    rng = np.random.default_rng(6)
    a, b = finite_halves(rng, 4000), finite_halves(rng, 4000)
    n = min(len(a), len(b))
    a, b = a[:n], b[:n]
    with np.errstate(over="ignore", invalid="ignore"):
        assert (oracle.h_op("bnno_h_add", a, b) == (a.view(np.float16) + b.view(np.float16)).view(np.uint16)).all()
        assert (oracle.h_op("bnno_h_mul", a, b) == (a.view(np.float16) * b.view(np.float16)).view(np.uint16)).all()
    x = np.concatenate([rng.standard_normal(3000) * 10.0 ** rng.integers(-9, 6, 3000), [65519.99, 65520.0, 2.0 ** -25,
                        2.0 ** -25 * 1.0000001, -2.0 ** -26, 1e-30, 0.0, -0.0]])
    got = np.array([oracle.lib().bnno_d2h(float(v)) for v in x], np.uint16)
    with np.errstate(over="ignore"):
        assert (got == x.astype(np.float16).view(np.uint16)).all()


def test_silu_table_tracks_x_sigmoid_x():
    """every finite fp16 input: the table SiLU is within the reference's stated accuracy of x * sigmoid(x) (max abs
    error 4.2e-3 on [-8, 8], src/silu_lut.h:6-7); beyond, 1 % relative plus the tail of the clamp at |x| = 15.4
    (q(15.4) ~ 3e-7 is applied to any larger |x|)"""
    h = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    h = h[(h & 0x7C00) != 0x7C00]
    got = oracle.h_op("bnno_h_silu", h).view(np.float16).astype(np.float64)
    x = h.view(np.float16).astype(np.float64)
    with np.errstate(over="ignore"):
        want = x / (1.0 + np.exp(-x))
    err = np.abs(got - want)
    inside = np.abs(x) <= 8
    assert err[inside].max() <= 4.3e-3
    assert (err[~inside] <= 1e-2 * np.abs(want[~inside]) + 4.3e-3 + 4e-7 * np.abs(x[~inside])).all()


# ------------------------------------------------------------------ the model against float64

def f64_forward(ir, img):
    """the v2.4 IR in float64 numpy, from the front end's image [96][511][2]: (logits, embedding)"""
    ops = ir[0]
    vals = {ops[0]["out"]: img.astype(np.float64)}
    swish = lambda v: v / (1.0 + np.exp(-v))  # noqa: E731

    def conv(x, w, b, s, pads):
        (pt, pl, pb, pr), (co, ci, kh, kw) = pads, w.shape
        xp = np.pad(x, ((pt, pb), (pl, pr), (0, 0)))
        ho, wo = (xp.shape[0] - kh) // s + 1, (xp.shape[1] - kw) // s + 1
        y = np.zeros((ho, wo, co))
        for ky in range(kh):
            for kx in range(kw):
                y += xp[ky:ky + s * (ho - 1) + 1:s, kx:kx + s * (wo - 1) + 1:s, :] @ w[:, :, ky, kx].T.astype(np.float64)
        return y + b

    i = 1
    while i < len(ops):
        o = ops[i]
        x = vals[o["ins"][0]]
        if o["op"] == "CONV" and o["k"] == [4, 8]:
            y = np.maximum(conv(x, o["w"], o["b"], 2, (1, 3, 1, 4)), 0)
            vals[o["out"]] = np.concatenate([np.maximum(y[:, 0::2], y[:, 1::2]), (y[:, 0::2] + y[:, 1::2]) / 2], 2)
        elif o["op"] == "CONV" and o["k"] == [1, 1]:
            y = x @ o["w"][:, :, 0, 0].T.astype(np.float64) + o["b"]
            y = swish(y) if o.get("act") == "swish" else y
            vals[o["out"]] = y + (vals[o["res"]] if o.get("res") else 0)
        elif o["op"] == "DWCONV":
            c, s = x.shape[2], o["s"][0]
            xp = np.pad(x, ((1, 1), (1, 1), (0, 0)))
            ho, wo = ir[1][o["out"]]
            y = np.zeros((ho, wo, c)) + o["b"]
            for ky in range(3):
                for kx in range(3):
                    y += xp[ky:ky + s * (ho - 1) + 1:s, kx:kx + s * (wo - 1) + 1:s, :] * o["w"][:, 0, ky, kx]
            vals[o["out"]] = swish(y)
        elif o["op"] == "SE":
            m = x.mean((0, 1))
            g = 1.0 / (1.0 + np.exp(-(o["w2"] @ swish(o["w1"] @ m + o["b1"]) + o["b2"])))
            vals[o["out"]] = x * g
        elif o["op"] == "AFFINE":
            vals[o["out"]] = np.maximum(x * o["s"] + o["t"], 0)
        elif o["op"] == "CONV":  # the 3x3 valid pc conv
            vals[o["out"]] = np.maximum(conv(x, o["w"], o["b"], 1, (0, 0, 0, 0)), 0)
        elif o["op"] == "MEAN":
            vals[o["out"]] = x.mean((0, 1))
        elif o["op"] == "DENSE":
            vals[o["out"]] = o["w"].astype(np.float64) @ x + o["b"]
        i += 1
    return vals[ir[2]], vals[ir[3]]


def sqnr_db(got, want):
    return 10 * np.log10(np.sum(want ** 2) / max(np.sum((got - want) ** 2), 1e-300))


def test_f16_oracle_tracks_float64_model(f16_mini):
    """The fp16 path of the mini v2.4 model against a float64 forward pass of the same weights, from the same front-end
    image (FE_STFT2 is fp32 on both paths). Tolerance: SQNR >= 50 dB on the logits and on the embedding -- the
    reference compiler's own screen for an fp16 layer (lower.py:69-71 need_db = 50.0) -- and the logits' max-abs error
    below 1 % of their range. (Measured: 61-62 dB on the logits, 63-64 dB on the embedding.)"""
    ir = model_ir(GOLD["v24_mini_f16"])
    pcm = synth.audio(2, seed=3)
    p = oracle.Package(f16_mini, "neon-fp16")
    for w in range(2):
        p.run_range(pcm[w], 0, 1)
        img = p.get(1).reshape(96, 511, 2)
        got, emb = p.run(pcm[w])
        want, wemb = f64_forward(ir, img)
        assert sqnr_db(emb, wemb) >= 50, sqnr_db(emb, wemb)
        assert sqnr_db(got, want) >= 50, sqnr_db(got, want)
        assert np.abs(got - want).max() <= 0.01 * (want.max() - want.min())


def test_f16_oracle_runs_the_fp32_head(tmp_path):
    """61 classes: the compiler puts the head on the exact fp32 GEMV (DENSE variant 0)"""
    g = GOLD["v24_mini_f16_h32"]
    path = str(tmp_path / "h32.bnpk")
    synth.write_f16_package(path, model_ir(g))
    p = oracle.Package(path, "neon-fp16")
    assert p.op_code(p.n_ops - 1) == 7
    out, emb = p.run(synth.audio(1, seed=4)[0])
    assert out.shape == (61,) and np.isfinite(out).all() and np.isfinite(emb).all()


# ------------------------------------------------------------------ the library's loader on the fp16 path

def test_f16_path_selection_and_validation(tmp_path, f16_mini):
    """Mode 4 names a path the package does not have; the fp16 records are checked as rt_ops_f16.c checks them (the
    same messages), before any device is touched."""
    from conftest import gpu_visible  # pylint: disable=import-outside-toplevel
    from bnneon_b200 import BnnError, Model  # pylint: disable=import-outside-toplevel
    import struct  # pylint: disable=import-outside-toplevel
    from bnneon_b200 import pkgread  # pylint: disable=import-outside-toplevel
    with pytest.raises(BnnError) as e:
        Model(f16_mini, mode=4)
    assert e.value.kind == "CPU" and "path neon-int8 is not in this package" in str(e.value)
    if not gpu_visible():
        with pytest.raises(BnnError) as e:
            Model(f16_mini, mode=3)
        assert e.value.kind == "CPU" and "no CUDA device" in str(e.value)
    ops, _ = pkgread.read_ops(f16_mini, synth.PATH_F16)
    offs = pkgread.op_offsets(f16_mini, synth.PATH_F16)
    with open(f16_mini, "rb") as f:
        data = f.read()
    first = {code: i for i, (code, _, _, _) in reversed(list(enumerate(ops)))}
    cases = [(0x103, 5, 16, "lda >= Kp", "pw_f16"), (0x103, 6, 3, "act >= 0 && act <= 2", "pw_f16"),
             (0x104, 6, 2, "pt >= 0 && pt <= 1 && pl >= 0 && pl <= 1", "dw3_f16"),
             (0x104, 2, 4096, "p[2] <= 2048", "dw3_f16"),
             (0x105, 0, 12, "C > 0 && C % 8 == 0 && C <= 4096", "se_f16"),
             (0x102, 0, 16, "GEMM shape N 16 K 64 Kp 64 Np 24", "c0pool_f16"),
             (0x106, 0, 512, "GEMM shape N 512", "postpc_f16"),
             (0x107, 0, 0, "N > 0", "dense_f16")]
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
