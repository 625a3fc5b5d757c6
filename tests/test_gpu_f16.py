"""GPU parity of the neon-fp16 path: every op and whole packages bit for bit against the CPU oracle, through the C ABI.

The packages are the reference compiler's bytes for the v2.4 architecture (tests/golden/f16_packages.json pins them):
the mini model with an fp16 head (100 classes) and with the fp32 head the compiler gives 64 classes or fewer, and the
full model (6522 classes). Device memory for the debug entry points comes from the library itself.
"""
import numpy as np
import pytest

from conftest import bits_equal, mismatch_report
from bnneon_b200 import BnnError, Model, load_library, pkgread, synth
from oracle import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
PATH = synth.PATH_F16
MODELS = {"mini": (1, synth.MINI_BLOCKS, 100), "mini_h32": (1, synth.MINI_BLOCKS, 61), "full": (0, synth.V24_BLOCKS, 6522)}


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    h = load_library()
    torch.cuda.init()
    assert h.bnn_cuda_device_init() == 0, h.bnn_last_error()
    return h


@pytest.fixture(scope="module")
def f16_pkgs(tmp_path_factory):
    d = tmp_path_factory.mktemp("f16pkg")
    out = {}
    for name, (seed, blocks, nc) in MODELS.items():
        out[name] = str(d / f"{name}.bnpk")
        synth.write_f16_package(out[name], synth.v24_ir(seed, nc, blocks))
    return out


@pytest.mark.parametrize("which", ["mini", "mini_h32", "full"])
def test_f16_every_op(lib, which, f16_pkgs):
    """Op by op: the GPU op on the oracle's inputs against the oracle's outputs (the oracle advances op by op, so an
    op that works in place -- SE -- gets its input as it was before the op)."""
    pkg = f16_pkgs[which]
    ops, _ = pkgread.read_ops(pkg, PATH)
    B = 2
    pcm = synth.audio(B, seed=5)
    states = [oracle.Package(pkg, PATH) for _ in range(B)]
    with Model(pkg, mode=3, batch=B) as m:
        assert m.info.path == b"neon-fp16" and m.info.precision == b"fp16"
        for i, (code, bl, _, _) in enumerate(ops):
            ins, outs = pkgread.op_io(code, bl)
            for b in set(ins + outs):
                if b != 0:
                    m.set_buffer(b, np.stack([s.get(b) for s in states]))
            for w, s in enumerate(states):
                s.run_range(pcm[w], i, i + 1)
            m.run_ops(pcm, i, i + 1)
            for b in outs:
                elems, dt = states[0].buf_info(b)
                got = m.get_buffer(b, B, dt, elems)
                for w in range(B):
                    want = states[w].get(b)
                    g = got[w].view(np.uint16).astype(np.float32) if dt == np.float16 else got[w]
                    h = want.view(np.uint16).astype(np.float32) if dt == np.float16 else want
                    if dt == np.float16:  # fp16: bit patterns, any NaN equal to any NaN
                        gn, hn = np.isnan(got[w].astype(np.float32)), np.isnan(want.astype(np.float32))
                        ok = np.array_equal(gn, hn) and np.array_equal(g[~gn], h[~hn])
                    else:
                        ok = bits_equal(g, h)
                    assert ok, (f"op {i} {pkgread.NAMES[code]} buffer {b} window {w}: "
                                + mismatch_report(got[w].astype(np.float32), want.astype(np.float32)))


@pytest.mark.parametrize("which,n", [("mini", 5), ("mini_h32", 3), ("full", 3)])
def test_f16_end_to_end(lib, which, n, f16_pkgs):
    pkg = f16_pkgs[which]
    pcm = synth.audio(n, seed=9)
    want, wemb = oracle.run_many(pkg, pcm, threads=4, path_name=PATH)
    with Model(pkg, mode=3, batch=2) as m:  # 2 windows per launch: exercises chunking and graph replay
        got, gemb = m.infer_batch(pcm)
        again, _ = m.infer_batch(pcm)
        one, oemb = m.infer(pcm[1])
    assert bits_equal(got, want), mismatch_report(got, want)
    assert bits_equal(gemb, wemb), mismatch_report(gemb, wemb)
    assert bits_equal(again, want)
    assert bits_equal(one, want[1]) and bits_equal(oemb, wemb[1])


def test_f16_batch_split_invariance(lib, f16_pkgs):
    pcm = synth.audio(7, seed=21)
    with Model(f16_pkgs["mini"], mode=0, batch=7) as m:
        assert m.info.path == b"neon-fp16"
        a, ea = m.infer_batch(pcm)
        m.set_batch(3)
        b, eb = m.infer_batch(pcm)
    assert bits_equal(a, b) and bits_equal(ea, eb)


def test_f16_overflow_fails_the_window(lib, tmp_path):
    """fp16 overflow: a post-BN scale of 1e8 sends the fp16 post activations to infinity, the pc conv makes them
    NaN, and v24k16_postpc finds non-finite features and returns -2 (src/v24_fast.c:305-310); every window is reported
    failed (BNN_ERR_WINDOW, the first failed window named), as the oracle reports it."""
    ops, vshape, lv, ev = synth.v24_ir(1, 100, synth.MINI_BLOCKS)
    for o in ops:
        if o["op"] == "AFFINE":
            o["s"] = (o["s"] * 1e8).astype(np.float32)
    pkg = str(tmp_path / "overflow.bnpk")
    synth.write_f16_package(pkg, (ops, vshape, lv, ev))
    pcm = synth.audio(3, seed=2)
    p = oracle.Package(pkg, PATH)
    with pytest.raises(RuntimeError):
        p.run(pcm[0])
    with Model(pkg, mode=3, batch=4) as m:
        with pytest.raises(BnnError) as e:
            m.infer_batch(pcm)
        assert e.value.kind == "WINDOW" and "postpc_f16" in str(e.value) and "window 0" in str(e.value)


# ------------------------------------------------------------------ the fp16 1x1 conv through its own C ABI

PW_CASES = [  # (Mw, B, N, K, act, ow, opad, residual): shapes the v2.4 model never has, and its own
    (37, 3, 24, 48, 0, 0, 0, False),      # ragged row tiles, N 24 (4-channel thread tiles)
    (100, 2, 8, 8, 1, 0, 0, False),       # N 8: a channel tile wider than N
    (64, 2, 72, 24, 1, 16, 1, False),     # padded output rows (the depthwise conv's input)
    (50, 2, 40, 136, 2, 0, 0, True),      # two K blocks of 72 and 64, ReLU, residual
    (20, 5, 136, 264, 1, 0, 0, False),    # N 136 (a ragged second channel tile), three K blocks of 88
    (33, 2, 288, 72, 1, 11, 2, False),    # halo 2
    (7, 3, 1536, 1536, 0, 0, 0, True),    # twelve K blocks of 128
    (6, 4, 1024, 1728, 2, 0, 0, False),   # the pc conv's shape: fourteen blocks
    (1, 9, 16, 1000, 1, 0, 0, False),     # K not a multiple of 8: Kp 1000 -> 1000, 8 K blocks of 128 - (ragged 104)
]


def half_bits(a):
    return np.ascontiguousarray(a, np.float16).view(np.uint16)


def f16_equal(got, want):
    g, w = np.asarray(got, np.uint16), np.asarray(want, np.uint16)
    gn = (g & 0x7C00) == 0x7C00
    gn &= (g & 0x3FF) != 0
    wn = ((w & 0x7C00) == 0x7C00) & ((w & 0x3FF) != 0)
    return np.array_equal(gn, wn) and np.array_equal(g[~gn], w[~wn])


@pytest.mark.parametrize("case", PW_CASES, ids=[f"M{c[0]}xB{c[1]}_N{c[2]}_K{c[3]}_act{c[4]}" for c in PW_CASES])
def test_pw_f16_op(lib, case):
    Mw, B, N, K, act, ow, opad, residual = case
    rng = np.random.default_rng(N * 31 + K)
    Kp = (K + 7) & ~7
    w = (rng.standard_normal((N, K)) * (2.0 / np.sqrt(K))).astype(np.float32)
    w[0, :] = 0.0  # a zero channel
    b = (rng.standard_normal(N) * 0.2).astype(np.float32)
    panels, b32, b16, shp = synth.pack_h16(w, b, Kp)
    Np = shp[3]
    lda, ldo, ldr = Kp + 8, Np + 4, Np + 8
    x = (rng.standard_normal((B, Mw, lda)) * 3.0).astype(np.float16)
    x[:, :, Kp:] = 0
    x[0, 0, :4] = [60000.0, -60000.0, 6e-8, -0.0]  # overflow toward infinity, a subnormal, -0
    res = (rng.standard_normal((B, Mw, ldr)) * 0.5).astype(np.float16) if residual else None
    orows = ((Mw // ow) + 2 * opad) * (ow + 2 * opad) if opad else Mw
    op = lib.bnn_pw_f16_new(N, K, Kp, Np, panels.ctypes.data, b32.ctypes.data, b16.ctypes.data)
    assert op, lib.bnn_last_error()
    try:
        d_x = torch.from_numpy(half_bits(x).astype(np.int16)).cuda()
        d_out = torch.full((B, orows, ldo), 0x7777, dtype=torch.int16, device="cuda")
        d_res = torch.from_numpy(half_bits(res).astype(np.int16)).cuda() if residual else None
        rc = lib.bnn_pw_f16_run(op, B, Mw, d_x.data_ptr(), Mw * lda, lda, act, d_out.data_ptr(), orows * ldo, ldo, ow,
                                opad, d_res.data_ptr() if residual else None, Mw * ldr if residual else 0,
                                ldr if residual else 0, None)
        assert rc == 0, lib.bnn_last_error()
        torch.cuda.synchronize()
        got = d_out.cpu().numpy().view(np.uint16)
    finally:
        lib.bnn_pw_f16_free(op)
    for wi in range(B):
        want = oracle.gemm_f16(x[wi], panels, b32, b16, Kp, Np, act, Mw, ldo=ldo, ow=ow, opad=opad,
                               res=None if res is None else res[wi], ldr=ldr).view(np.uint16)
        if opad:  # the halo is not written: the sentinel stays
            keep = np.zeros((orows,), bool)
            for m in range(Mw):
                keep[((m // ow) + opad) * (ow + 2 * opad) + m % ow + opad] = True
            assert (got[wi][~keep] == 0x7777).all()
            g, wv = got[wi][keep][:, :Np], want[keep][:, :Np]
        else:
            g, wv = got[wi][:, :Np], want[:, :Np]
        assert (got[wi][:, Np:] == 0x7777).all()
        assert f16_equal(g, wv), (wi, int(np.sum(g != wv)))


def test_pw_f16_op_refuses_bad_arguments(lib):
    panels, b32, b16, _ = synth.pack_h16(np.ones((8, 8), np.float32), np.zeros(8, np.float32), 8)
    assert not lib.bnn_pw_f16_new(8, 8, 12, 8, panels.ctypes.data, b32.ctypes.data, b16.ctypes.data)
    assert "Kp % 8 == 0" in lib.bnn_last_error().decode()
    op = lib.bnn_pw_f16_new(8, 8, 8, 8, panels.ctypes.data, b32.ctypes.data, b16.ctypes.data)
    try:
        d = torch.zeros(64, dtype=torch.int16, device="cuda")
        assert lib.bnn_pw_f16_run(op, 1, 4, d.data_ptr(), 32, 4, 0, d.data_ptr(), 32, 8, 0, 0, None, 0, 0, None) == -1
        assert "lda 4" in lib.bnn_last_error().decode()
    finally:
        lib.bnn_pw_f16_free(op)


# ------------------------------------------------------------------ the fp16 depthwise conv through its own C ABI

DW_CASES = [  # (B, H, W, C, s, pt, pl): the v2.4 shapes and the record's other geometries
    (2, 24, 64, 72, 1, 1, 1), (2, 48, 128, 72, 2, 1, 1), (3, 12, 32, 288, 1, 1, 1), (2, 6, 16, 864, 2, 1, 1),
    (2, 3, 8, 1536, 1, 1, 1),
    (2, 9, 14, 16, 1, 0, 0),    # pt = pl = 0 and an odd output width (one pixel per group)
    (3, 10, 11, 8, 2, 0, 1),    # stride 2, pt 0, C 8
    (1, 5, 7, 2048, 2, 1, 0),   # the widest C the record allows
]


@pytest.mark.parametrize("case", DW_CASES, ids=[f"H{c[1]}W{c[2]}C{c[3]}s{c[4]}pt{c[5]}pl{c[6]}" for c in DW_CASES])
def test_dw3_f16_op(lib, case):
    B, H, W, C, s, pt, pl = case
    # the largest output the taps allow: (Ho - 1) s - pt + 1 + 3 <= H + 2
    Ho, Wo = (H + 2 - 4 + pt) // s + 1, (W + 2 - 4 + pl) // s + 1
    rng = np.random.default_rng(H * 7 + C)
    xp = np.zeros((B, H + 2, W + 2, C), np.float16)
    xp[:, 1:H + 1, 1:W + 1] = (rng.standard_normal((B, H, W, C)) * 2.0).astype(np.float16)
    xp[0, 1, 1, :2] = [60000.0, -0.0]
    w = (rng.standard_normal((9, C)) * 0.5).astype(np.float16)
    bias = (rng.standard_normal(C) * 0.1).astype(np.float16)
    xws, ows = (H + 2) * (W + 2) * C, Ho * Wo * C
    d_x = torch.from_numpy(half_bits(xp).astype(np.int16)).cuda()
    d_w = torch.from_numpy(half_bits(w).astype(np.int16)).cuda()
    d_b = torch.from_numpy(half_bits(bias).astype(np.int16)).cuda()
    d_o = torch.full((B, ows), 0x7777, dtype=torch.int16, device="cuda")
    d_c = torch.full((B, C), 7.0, dtype=torch.float32, device="cuda")
    assert lib.bnn_cuda_dw3_f16(B, d_x.data_ptr(), xws, H, W, C, s, pt, pl, d_w.data_ptr(), d_b.data_ptr(),
                                d_o.data_ptr(), ows, Ho, Wo, d_c.data_ptr(), C, None) == 0, lib.bnn_last_error()
    torch.cuda.synchronize()
    assert lib.bnn_cuda_op_error() == 0
    got, chs = d_o.cpu().numpy().view(np.uint16), d_c.cpu().numpy()
    for wi in range(B):
        out = np.zeros((Ho * Wo, C), np.uint16)
        cs = np.zeros(C, np.float32)
        oracle.lib().bnno_dw3_f16(half_bits(xp[wi]).ctypes.data, H, W, C, s, pt, pl, half_bits(w).ctypes.data,
                                  half_bits(bias).ctypes.data, out.ctypes.data, Ho, Wo, cs.ctypes.data)
        assert f16_equal(got[wi].reshape(Ho * Wo, C), out), (wi, int(np.sum(got[wi].reshape(Ho * Wo, C) != out)))
        assert bits_equal(chs[wi], cs), mismatch_report(chs[wi], cs)
