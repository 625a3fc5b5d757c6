"""The fp32 ops beyond the v2.4 path: BirdNET v3.0's CONVK, CONVW (Winograd F(4x4, 3x3)), GEM, SED and VADD
(src/rt_ops_f32x.c:88-436) and Perch's fp32 body ops STEM, DWK, PAD and MEAN (src/rt_ops_f32.c:387-520).

Each op runs in a small package (synth.write_ops_package: the window itself is the op's input, declared in the layout
the op reads; a VADD of the window makes a second input where an op needs one). The checker is the reference's own
runtime compiled for this host (oracle/_ref, oracle/ref.mk), run on the same package and windows:

* CPU: the reference accepts each package and scores it; the B200 library's loader accepts it too (its record checks
  are the reference's) and refuses corrupted records with the reference's messages;
* GPU: bnn_infer_batch of the B200 library against the reference bit for bit, except GEM, whose last step is libm
  powf (the device rounds the double-precision pow once): within one unit in the last place there.
"""
import struct

import numpy as np
import pytest

from conftest import bits_equal, mismatch_report, gpu_visible
from bnneon_b200 import BnnError, Model, pkgread, synth
from oracle import ref

F32 = synth.F32
VADD, GEM, SED, CONVK, CONVW, SED_S8 = 20, 18, 19, 17, 21, 24
STEM, DWK, PAD, MEAN = 9, 10, 11, 12


def r8(n):
    return (n + 7) & ~7


# ------------------------------------------------------------------ op packages

def pkg_vadd(path, n=1000):
    bufs = [(F32, 1, 1, n, n, 0, n), (F32, 1, 1, n, n, 0, n)]
    synth.write_ops_package(path, bufs, [], [(VADD, [0, 0, 1], [], [n])], 1)
    return n, None


def pkg_gem(path, P=37, C=24, ld=28, eps=1e-6, p=3.0, q=1.0 / 3.0):
    bufs = [(F32, 1, P, C, ld, 0, P * ld), (F32, 1, 1, C, C, 0, C)]
    consts = np.array([eps, p, q], np.float32)
    synth.write_ops_package(path, bufs, [("gem.0.consts", consts)], [(GEM, [0, 1], [0], [P, C, ld])], 1)
    return P * ld, None


def pkg_mean(path, P=50, C=16, ld=20):
    bufs = [(F32, 1, P, C, ld, 0, P * ld), (F32, 1, 1, C, C, 0, C)]
    synth.write_ops_package(path, bufs, [], [(MEAN, [0, 1], [], [P, C, ld])], 1)
    return P * ld, None


def pkg_pad(path, H=5, W=7, C=8, ld=12, h=2):
    bufs = [(F32, H, W, C, ld, 0, H * W * ld), (F32, H, W, C, C, h, (H + 2 * h) * (W + 2 * h) * C)]
    synth.write_ops_package(path, bufs, [], [(PAD, [0, 1], [], [H, W, C, ld, h])], 1)
    return H * W * ld, None


def halo_mask(H, W, ld, h, extra=0):
    """1 inside the image, 0 on the halo ring (and on the slack past it), for a window [H + 2h][W + 2h][ld]"""
    m = np.zeros((H + 2 * h, W + 2 * h, ld), np.float32)
    m[h:h + H, h:h + W, :] = 1
    return np.concatenate([m.reshape(-1), np.zeros(extra, np.float32)])


def pkg_dwk(path, H=11, W=14, C=16, k=5, s=2, act=1, seed=0):
    """TF-same padding: Ho = ceil(H / s), the total pad split top / bottom with the larger part at the bottom"""
    rng = np.random.default_rng(seed)
    h = (k - 1) // 2
    Ho, Wo = -(-H // s), -(-W // s)
    pt = max((Ho - 1) * s + k - H, 0) // 2
    pl = max((Wo - 1) * s + k - W, 0) // 2
    n_in = (H + 2 * h) * (W + 2 * h) * C
    bufs = [(F32, H, W, C, C, h, n_in), (F32, Ho, Wo, C, C, 0, Ho * Wo * C), (F32, 1, 1, C, C, 0, C)]
    w = (rng.standard_normal((k * k, C)) * 0.3).astype(np.float32)
    b = (rng.standard_normal(C) * 0.1).astype(np.float32)
    rec = (DWK, [0, 1, 2], [0, 1], [H, W, C, k, s, pt, pl, Ho, Wo, act])
    synth.write_ops_package(path, bufs, [("dwk.w", w), ("dwk.b", b)], [rec], 1, emb_buf=2)
    return n_in, halo_mask(H, W, C, h)


def pkg_stem(path, H=29, W=23, k=3, s=2, N=40, act=1, opad=1, seed=1):
    rng = np.random.default_rng(seed)
    Ho, Wo = (H - k) // s + 1, (W - k) // s + 1
    K, Kp = k * k, (k * k + 3) & ~3
    panels, bias, (_, _, _, Np) = synth.pack_f32(rng.standard_normal((N, K)) * 0.4, rng.standard_normal(N) * 0.1, Kp)
    bufs = [(F32, H, W, 1, 1, 0, H * W), (F32, Ho, Wo, N, Np, opad, (Ho + 2 * opad) * (Wo + 2 * opad) * Np),
            (F32, 1, 1, r8(Ho * Wo) * Kp, r8(Ho * Wo) * Kp, 0, r8(Ho * Wo) * Kp)]
    rec = (STEM, [0, 1, 2], [0, 1], [N, K, Kp, Np, H, W, Ho, Wo, k, s, act, Np, opad])
    synth.write_ops_package(path, bufs, [("stem.w", panels), ("stem.b", bias)], [rec], 1)
    return H * W, None


def pkg_convk(path, H=9, W=13, C=8, N=20, kh=3, kw=3, s=1, act=1, opad=1, res=True, seed=2):
    rng = np.random.default_rng(seed)
    h = 1
    Ho, Wo = (H - 1) // s + 1, (W - 1) // s + 1
    K = kh * kw * C
    panels, bias, (_, _, _, Np) = synth.pack_f32(rng.standard_normal((N, K)) * 0.15, rng.standard_normal(N) * 0.1, K)
    Wp = W + 2 * h
    last = ((0 + (Ho - 1) * s + kh - 1) * Wp + 0 + (((Wo + 7) & ~7) - 1) * s + kw) * C + 4
    base = (H + 2 * h) * Wp * C
    n_in = max(base, last, Ho * Wo * Np)
    bufs = [(F32, H, W, C, C, h, n_in), (F32, Ho, Wo, N, Np, opad, (Ho + 2 * opad) * (Wo + 2 * opad) * Np)]
    recs = []
    rb = -1
    if res:
        bufs.append((F32, Ho, Wo, Np, Np, 0, Ho * Wo * Np))
        rb = 2
        recs.append((VADD, [0, 0, 2], [], [Ho * Wo * Np]))
    recs.append((CONVK, [0, 1, rb], [0, 1], [N, K, K, Np, H, W, Ho, Wo, kh, kw, s, 0, 0, act, Np, opad]))
    synth.write_ops_package(path, bufs, [("convk.w", panels), ("convk.b", bias)], recs, 1)
    return n_in, halo_mask(H, W, C, h, n_in - base)


def pkg_pw(path, M=300, K=40, Kp=None, lda=None, N=24, act=0, gated=True, res=True, ow=0, opad=0, seed=5):
    """PW (the fp32 1x1 conv of the neon-int8 Perch body, pw_run, src/rt_ops_f32.c:193-206): the window is the
    [M8][lda] input; a MEAN of it over the M rows makes the [K] input-channel gate, a VADD of it the residual"""
    rng = np.random.default_rng(seed)
    Kp = Kp or (K + 3) & ~3
    lda = lda or Kp
    panels, bias, (_, _, _, Np) = synth.pack_f32(rng.standard_normal((N, K)) * 0.2, rng.standard_normal(N) * 0.1, Kp)
    n_in = max(r8(M) * lda, M * Np)
    if opad:
        out = (F32, M // ow, ow, N, Np, opad, (M // ow + 2 * opad) * (ow + 2 * opad) * Np)
    else:
        out = (F32, 1, M, N, Np, 0, M * Np)
    bufs = [(F32, 1, r8(M), K, lda, 0, n_in), out]
    recs = []
    rb = gb = -1
    if res:
        bufs.append((F32, 1, M, Np, Np, 0, M * Np))
        rb = len(bufs) - 1
        recs.append((VADD, [0, 0, rb], [], [M * Np]))
    if gated:
        bufs.append((F32, 1, 1, K, K, 0, K))
        gb = len(bufs) - 1
        recs.append((MEAN, [0, gb], [], [M, K, lda]))
    recs.append((3, [0, 1, rb] + ([gb] if gated else []), [0, 1], [N, K, Kp, Np, M, lda, act, Np, ow, opad, Np]))
    synth.write_ops_package(path, bufs, [("pw.w", panels), ("pw.b", bias)], recs, 1)
    mask = np.zeros(n_in, np.float32)
    mask.reshape(-1)[:r8(M) * lda].reshape(r8(M), lda)[:, :K] = 1
    return n_in, mask


def pkg_convw(path, H=10, W=14, C=8, N=12, act=1, opad=1, res=True, seed=3):
    rng = np.random.default_rng(seed)
    h, Np = 1, r8(N)
    U = (rng.standard_normal((36, Np // 8, C, 8)) * 0.2).astype(np.float32)
    if N % 8:
        U[:, N // 8, :, N % 8:] = 0.0  # the pad channels carry zero weights, as compiled
    bias = np.zeros(Np + 8, np.float32)
    bias[:N] = rng.standard_normal(N) * 0.1
    base = (H + 2 * h) * (W + 2 * h) * C
    n_in = max(base, H * W * Np)
    bufs = [(F32, H, W, C, C, h, n_in), (F32, H, W, N, Np, opad, (H + 2 * opad) * (W + 2 * opad) * Np)]
    recs = []
    rb = -1
    if res:
        bufs.append((F32, H, W, Np, Np, 0, H * W * Np))
        rb = 2
        recs.append((VADD, [0, 0, 2], [], [H * W * Np]))
    recs.append((CONVW, [0, 1, rb], [0, 1], [C, N, Np, H, W, act, Np, opad, 8, 64]))
    synth.write_ops_package(path, bufs, [("convw.U", U), ("convw.b", bias)], recs, 1)
    return n_in, halo_mask(H, W, C, h, n_in - base)


def pkg_sed(path, red=3, H=12, W=5, C=16, ld=16, hid=24, NC=10, pk=3, dk=3, hc=1, seed=4):
    rng = np.random.default_rng(seed)
    L = H if red == 3 else W
    L8 = r8(L)
    Cp = (C + 7) & ~7
    fcw, fcb, (_, _, fkp, fnp) = synth.pack_f32(rng.standard_normal((hid, C)) * 0.3, rng.standard_normal(hid) * 0.1,
                                                Cp)
    atw, atb, (_, _, akp, anp) = synth.pack_f32(rng.standard_normal((NC, hid)) * 0.3, rng.standard_normal(NC) * 0.1,
                                                fnp)
    clw, clb, (_, _, ckp, cnp) = synth.pack_f32(rng.standard_normal((NC, hid)) * 0.3, rng.standard_normal(NC) * 0.1,
                                                fnp)
    dw = (rng.standard_normal((max(dk, 1), C)) * 0.3).astype(np.float32)
    db = (rng.standard_normal(C) * 0.1).astype(np.float32)
    consts = np.array([-1.5, 1.5, 0.7], np.float32)
    bufs = [(F32, H, W, C, ld, 0, H * W * ld), (F32, 1, 1, NC, NC, 0, NC),
            (F32, L8, 1, Cp, Cp, 0, L8 * Cp), (F32, L8, 1, Cp, Cp, 0, L8 * Cp),
            (F32, L8, 1, fnp, fnp, 0, L8 * fnp), (F32, L8, 1, anp, anp, 0, L8 * anp), (F32, L8, 1, cnp, cnp, 0, L8 * cnp)]
    tens = [("sed.dw", dw), ("sed.db", db), ("sed.fc.w", fcw), ("sed.fc.b", fcb), ("sed.att.w", atw),
            ("sed.att.b", atb), ("sed.cla.w", clw), ("sed.cla.b", clb), ("sed.consts", consts)]
    ints = [hid, C, fkp, fnp, NC, hid, akp, anp, NC, hid, ckp, cnp, red, H, W, C, ld, L, pk, dk, hc]
    synth.write_ops_package(path, bufs, tens, [(SED, [0, 1, 2, 3, 4, 5, 6], list(range(9)), ints)], 1)
    return H * W * ld, None


def s8_tensors(tag, w, b):
    """the reference packer's int8 GEMM tensors (s8_tensors, lower.py:883-914) as synth writes them for PW_S8"""
    lw = synth._Int8Lowering([])  # pylint: disable=protected-access
    tl, shp = lw.s8(tag, np.asarray(w, np.float64), np.asarray(b, np.float32))
    return [lw.tensors[i] for i in tl], shp


def pkg_sed_s8(path, red=3, H=12, W=5, C=20, ld=24, hid=40, NC=12, pk=3, dk=3, hc=1, seed=5):
    """SED_S8 (rt_ops_s8n.c:160-210): the SED head with int8 fc / att / cla GEMMs on per-row quantized rows"""
    rng = np.random.default_rng(seed)
    L = H if red == 3 else W
    L8, Cp = r8(L), r8(C)
    fc, (_, _, fkp, fnp) = s8_tensors("sed.fc", rng.standard_normal((hid, C)) * 0.3, rng.standard_normal(hid) * 0.1)
    at, (_, _, akp, anp) = s8_tensors("sed.att", rng.standard_normal((NC, hid)) * 0.3, rng.standard_normal(NC) * 0.1)
    cl, (_, _, ckp, cnp) = s8_tensors("sed.cla", rng.standard_normal((NC, hid)) * 0.3, rng.standard_normal(NC) * 0.1)
    dw = (rng.standard_normal((max(dk, 1), C)) * 0.3).astype(np.float32)
    db = (rng.standard_normal(C) * 0.1).astype(np.float32)
    consts = np.array([-2.0, 2.0, 0.5], np.float32)
    kq = max(fkp, akp)
    bufs = [(F32, H, W, C, ld, 0, H * W * ld), (F32, 1, 1, NC, NC, 0, NC),
            (F32, L8, 1, Cp, Cp, 0, L8 * Cp), (F32, L8, 1, Cp, Cp, 0, L8 * Cp),
            (F32, L8, 1, fnp, fnp, 0, L8 * fnp), (F32, L8, 1, anp, anp, 0, L8 * anp), (F32, L8, 1, cnp, cnp, 0, L8 * cnp),
            (synth.I8, L8, 1, kq, kq, 0, L8 * kq), (F32, L8, 1, 1, 1, 0, L8), (synth.I32, L8, 1, 1, 1, 0, L8)]
    tens = [("sed.dw", dw), ("sed.db", db)] + fc + at + cl + [("sed.consts", consts)]
    ints = [hid, C, fkp, fnp, NC, hid, akp, anp, NC, hid, ckp, cnp, red, H, W, C, ld, L, pk, dk, hc]
    synth.write_ops_package(path, bufs, tens, [(SED_S8, list(range(10)), list(range(15)), ints)], 1)
    return H * W * ld, None


CASES = {
    "vadd": (pkg_vadd, {}),
    "gem": (pkg_gem, {}),
    "gem_p1": (pkg_gem, dict(P=5, C=8, ld=8, p=1.0, q=1.0)),
    "mean": (pkg_mean, {}),
    "pad": (pkg_pad, {}),
    "dwk_k5_s2": (pkg_dwk, {}),
    "dwk_k3_s1": (pkg_dwk, dict(k=3, s=1, H=9, W=10, C=24)),
    "dwk_k7_s1_linear": (pkg_dwk, dict(k=7, s=1, H=12, W=9, C=8, act=0)),
    # 32 channel pairs per CTA with a ragged last CTA, several chunks of rows per window
    "dwk_k5_s1_c72": (pkg_dwk, dict(k=5, s=1, H=13, W=11, C=72)),
    "dwk_k3_s2_c40": (pkg_dwk, dict(k=3, s=2, H=17, W=19, C=40)),
    # short rows, several rows per thread and chunk, two chunks of 28 rows
    "dwk_k5_s1_tall": (pkg_dwk, dict(k=5, s=1, H=40, W=8, C=64)),
    "stem": (pkg_stem, {}),
    "stem_relu_nohalo": (pkg_stem, dict(act=2, opad=0, N=16, k=5, s=1, H=12, W=11)),
    "convk_s1_res": (pkg_convk, {}),
    "convk_s2": (pkg_convk, dict(s=2, res=False, act=2, N=16)),
    "convk_1x3": (pkg_convk, dict(kh=1, kw=3, act=0, opad=0)),
    # fp32 PW at every tile width of the tiled GEMM (32, 64, 128 columns), ragged rows and K steps, padded output
    "pw_gated_n24_res": (pkg_pw, {}),
    "pw_silu_n136_pad": (pkg_pw, dict(M=300, K=50, Kp=52, lda=56, N=136, act=1, gated=False, res=False, ow=20,
                                      opad=1)),
    "pw_gated_n384_res": (pkg_pw, dict(M=129, K=144, N=384, act=0)),
    "pw_relu_n60": (pkg_pw, dict(M=77, K=20, Kp=24, lda=28, N=60, act=2, gated=False, res=False)),
    "pw_gated_n232_silu": (pkg_pw, dict(M=70, K=96, N=232, act=1, res=False)),
    "convw_res": (pkg_convw, {}),
    "convw_edge": (pkg_convw, dict(H=7, W=5, C=12, N=20, act=2, opad=0, res=False)),
    "sed_time": (pkg_sed, {}),
    "sed_freq_nopool": (pkg_sed, dict(red=2, H=6, W=9, pk=0, dk=5, hc=0, C=12, ld=16)),
    "sed_pool_only": (pkg_sed, dict(pk=5, dk=0)),
    "sed_s8_time": (pkg_sed_s8, {}),
    "sed_s8_freq": (pkg_sed_s8, dict(red=2, H=7, W=10, pk=0, dk=5, hc=0, C=16, ld=16, NC=9)),
}


def windows(n_in, mask, n, seed):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((n, n_in)) * 0.7).astype(np.float32)
    if mask is not None:
        x *= mask[None, :n_in]
    return x


@pytest.fixture(scope="module")
def reflib():
    if ref.reference_checkout() is not None:
        ref.build()
    if not ref.available():
        pytest.skip("no reference build (oracle/_ref) and no reference checkout to build it from")
    return ref.lib()


def build(tmp_path, name):
    fn, kw = CASES[name]
    path = str(tmp_path / f"{name}.bnpk")
    n_in, mask = fn(path, **kw)
    return path, n_in, mask


@pytest.mark.parametrize("name", sorted(CASES))
def test_reference_and_loader_accept_package(reflib, tmp_path, name):
    path, n_in, mask = build(tmp_path, name)
    x = windows(n_in, mask, 2, 1)
    out, emb, rc = ref.run_many(path, 4, x, threads=1)
    assert (rc == 0).all() and np.isfinite(out).all()
    if not gpu_visible():
        with pytest.raises(BnnError) as e:
            Model(path, mode=4)
        assert e.value.kind == "CPU" and "no CUDA device" in str(e.value), str(e.value)


def corrupt(path, op_index, k, val, dst):
    off = pkgread.op_offsets(path)[op_index]
    with open(path, "rb") as f:
        data = bytearray(f.read())
    _, _, nb, nt, _, _ = struct.unpack("<6H", bytes(data[off:off + 12]))
    ints = off + 12 + 4 * (nb + nt)
    data[ints + 4 * k:ints + 4 * k + 4] = struct.pack("<i", val)
    with open(dst, "wb") as f:
        f.write(bytes(data))


@pytest.mark.parametrize("name, op, k, val, text", [
    ("convk_s2", 0, 10, 3, "st >= 1 && st <= 2"),
    ("convk_s1_res", 1, 13, 3, "act >= 0 && act <= 2"),
    ("convw_res", 1, 2, 17, "Np == ((N + 7) & ~7)"),
    ("convw_res", 1, 9, 12, "Nb % 8 == 0"),
    ("gem", 0, 1, 6, "C % 4 == 0"),
    ("sed_time", 0, 12, 1, "red == 2 || red == 3"),
    ("sed_time", 0, 18, 2, "(pk == 0 || pk % 2)"),
    ("dwk_k5_s2", 0, 3, 4, "k % 2 == 1"),
    ("stem", 0, 10, 5, "p[10] >= 0 && p[10] <= 2"),
    ("vadd", 0, 0, 0, "p[0] > 0"),
    ("sed_s8_time", 0, 2, 24, "Kp = K rounded up to 16"),
])
def test_record_checks(tmp_path, name, op, k, val, text):
    path, _, _ = build(tmp_path, name)
    bad = str(tmp_path / "bad.bnpk")
    corrupt(path, op, k, val, bad)
    with pytest.raises(BnnError) as e:
        Model(bad, mode=4)
    assert e.value.kind == "PACKAGE" and text in str(e.value), str(e.value)


# ------------------------------------------------------------------ GPU

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    torch.cuda.init()


def ulp_diff(a, b):
    a = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    a = np.where(a < 0, -(a & 0x7fffffff), a)
    b = np.where(b < 0, -(b & 0x7fffffff), b)
    return np.abs(a - b)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(CASES))
def test_op_against_reference(cuda, reflib, tmp_path, name):
    path, n_in, mask = build(tmp_path, name)
    x = windows(n_in, mask, 11, 7)
    want, wemb, rc = ref.run_many(path, 4, x, threads=4)
    assert (rc == 0).all()
    with Model(path, mode=4, batch=4) as m:
        for call in range(2):
            got, gemb = m.infer_batch(x)
            if name.startswith("gem"):
                d = ulp_diff(got, want)
                assert d.max() <= 1, f"call {call}: {int((d > 0).sum())} outputs differ, max {int(d.max())} ulp"
            else:
                assert bits_equal(got, want), f"call {call}: " + mismatch_report(got, want)
            if wemb.shape[1]:
                assert bits_equal(gemb, wemb), f"call {call} (second output): " + mismatch_report(gemb, wemb)
