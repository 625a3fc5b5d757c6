"""GPU parity: every kernel of the v2.4 neon-int8 path against the CPU oracle, bit for bit, through the C ABI.

Device memory comes from torch (plumbing only); every compute call goes through libbnneon.so's entry points
(include/bnneon.h, include/bnneon_cuda.h).
"""
import ctypes

import numpy as np
import pytest

from conftest import bits_equal, mismatch_report
from bnneon_b200 import Model, load_library, pkgread, synth
from oracle import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    h = load_library()
    torch.cuda.init()
    assert h.bnn_cuda_device_init() == 0, h.bnn_last_error()
    return h


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


# ------------------------------------------------------------------ elementwise functions

def special_floats():
    return np.array([0.0, -0.0, 1.0, -1.0, 1e-30, -1e-30, 1e-45, -1e-45, 60.0, -60.0, 61.0, -61.0, 87.5, -87.5, 88.7,
                     89.0, -103.9, -104.0, 126.0, -126.0, 127.5, 1e30, -1e30, 3.4e38, -3.4e38, np.inf, -np.inf],
                    np.float32)


def sample_floats(n, seed):
    rng = np.random.default_rng(seed)
    u = rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32).view(np.float32)
    u = u[np.isfinite(u)]
    return np.concatenate([special_floats(), u, (rng.standard_normal(n) * 10).astype(np.float32)])


@pytest.mark.parametrize("fn,name", [(0, "bnno_silu"), (1, "bnno_silu"), (2, "bnno_sigmoid"), (3, "bnno_frecpe"),
                                     (4, "bnno_log2_acc"), (5, "bnno_exp2_acc"), (6, "bnno_expf")])
def test_elementwise(lib, fn, name):
    x = sample_floats(20000, fn)
    if fn == 4:
        x = np.abs(x[np.isfinite(x) & (np.abs(x) >= 1e-30)])  # the front end's log2 takes max(|m|, 1e-30)
    if fn in (1, 5):
        # the table estimate serves finite SiLU inputs; exp2_acc builds its result from the bits of its polynomial,
        # so a NaN's payload (which differs between AArch64 and CUDA) would leak into the bits: finite inputs only
        x = x[np.isfinite(x)]
    y = torch.empty(x.size, dtype=torch.float32, device="cuda")
    xd = dev(x)
    assert lib.bnn_cuda_fn(fn, x.size, xd.data_ptr(), y.data_ptr(), None) == 0
    got, want = host(y), oracle.fn(name, x)
    assert bits_equal(got, want), mismatch_report(got, want)


def test_paired_fp32(lib):
    """sm_100's paired fp32 fma rounds each lane once, as fmaf; the paired SiLU equals the reference's SiLU."""
    x = sample_floats(20000, 8)
    x = x[np.isfinite(x)]
    xd = dev(x)
    y = torch.empty(x.size, dtype=torch.float32, device="cuda")
    ok = np.abs(x) < 1e30  # the double product is exact there, so rounding the double sum once equals fmaf
    fused = (x[ok].astype(np.float64) * np.float64(np.float32(1.7)) + np.float64(np.float32(0.3))).astype(np.float32)
    assert lib.bnn_cuda_fn(8, x.size, xd.data_ptr(), y.data_ptr(), None) == 0
    got = host(y)[ok]
    assert bits_equal(got, fused), mismatch_report(got, fused)
    assert lib.bnn_cuda_fn(7, x.size, xd.data_ptr(), y.data_ptr(), None) == 0
    got, want = host(y), oracle.fn("bnno_silu", x)
    assert bits_equal(got, want), mismatch_report(got, want)


def test_expf_matches_libm_exhaustive_slice(lib):
    """glibc expf restated on the GPU against the host libm over a dense slice of the floats around the SE range."""
    u = np.arange(0xC2D00000, 0xC2D00000 + 2 ** 22, dtype=np.uint32)  # [-104, ...]
    x = np.concatenate([u.view(np.float32), np.arange(0, 2 ** 22, dtype=np.uint32).view(np.float32) * 1e30,
                        np.linspace(-90, 90, 2 ** 20, dtype=np.float32)])
    x = x[np.isfinite(x)]
    y = torch.empty(x.size, dtype=torch.float32, device="cuda")
    assert lib.bnn_cuda_fn(6, x.size, dev(x).data_ptr(), y.data_ptr(), None) == 0
    got = host(y)
    want = np.exp(x.astype(np.float64)).astype(np.float32)  # close, but libm is the reference:
    libm = ctypes.CDLL("libm.so.6")
    libm.expf.restype = ctypes.c_float
    libm.expf.argtypes = [ctypes.c_float]
    idx = np.random.default_rng(3).choice(x.size, 20000, replace=False)
    ref = np.array([libm.expf(float(v)) for v in x[idx]], np.float32)
    assert bits_equal(got[idx], ref), mismatch_report(got[idx], ref)
    assert np.allclose(got, want, rtol=1e-6, atol=0)


# ------------------------------------------------------------------ the quantizer

@pytest.mark.parametrize("K,lda", [(24, 24), (36, 40), (48, 48), (72, 72), (108, 112), (288, 288), (864, 864),
                                   (1536, 1536), (1024, 1024), (13, 16), (3, 3)])
def test_quant_rows(lib, K, lda):
    rng = np.random.default_rng(K)
    B, Mw = 3, 37
    x = (rng.standard_normal((B, Mw, lda)) * rng.uniform(0.01, 10, (B, Mw, 1))).astype(np.float32)
    x[0, 0, :] = 1.25             # constant row
    x[0, 1, :] = 0.0              # zero row
    x[1, 2, :K] = np.float32(3.0) + np.arange(K, dtype=np.float32) * np.float32(2 ** -22)  # a very narrow row
    if K > 8:
        x[1, 3, 5] = np.nan       # NaN
        x[2, 4, 1] = np.inf
    gate = (rng.uniform(0, 1, (B, K))).astype(np.float32)
    for use_gate in (False, True):
        Kq = (K + 31) // 32 * 32
        q = torch.zeros(B * Mw * Kq, dtype=torch.int8, device="cuda")
        sa = torch.zeros(B * Mw, dtype=torch.float32, device="cuda")
        za = torch.zeros(B * Mw, dtype=torch.int32, device="cuda")
        xd, gd = dev(x), dev(gate)
        rc = lib.bnn_cuda_quant_rows(B * Mw, Mw, xd.data_ptr(), Mw * lda, lda, K, Kq, gd.data_ptr() if use_gate else None,
                                     K, q.data_ptr(), sa.data_ptr(), za.data_ptr(), None)
        assert rc == 0, lib.bnn_last_error()
        gq, gsa, gza = host(q).reshape(B * Mw, Kq), host(sa), host(za)
        Kp = (K + 15) // 16 * 16
        for w in range(B):
            oq, osa, oza = (np.zeros((Mw, Kp), np.int8), np.zeros(Mw, np.float32), np.zeros(Mw, np.int32))
            g = gate[w] if use_gate else None
            oracle.lib().bnno_quant_rows(oracle.ptr(x[w]), lda, Mw, K, Kp, oracle.ptr(g), oracle.ptr(oq),
                                         oracle.ptr(osa), oracle.ptr(oza))
            rows = slice(w * Mw, (w + 1) * Mw)
            assert np.array_equal(gq[rows, :Kp], oq), (K, use_gate, w)
            assert bits_equal(gsa[rows], osa) and np.array_equal(gza[rows], oza)


# ------------------------------------------------------------------ PW_S8 / GEMV_S8 (quantizer + tcgen05 GEMM)

def make_pw(rng, N, K):
    w = (rng.standard_normal((N, K)) * 0.3).astype(np.float32)
    lw = synth._Int8Lowering([])  # pylint: disable=protected-access
    tl, (n, k, kp, np_) = lw.s8("t", w, (rng.standard_normal(N) * 0.1).astype(np.float32))
    return [lw.tensors[t][1] for t in tl], (n, k, kp, np_)


PW_CASES = [  # (N, K, Mw, B, act, residual, padded output (ow), gated)
    (24, 48, 6144, 2, 0, False, 0, False),     # p0
    (72, 24, 6144, 1, 1, False, 128, False),   # b1.1 pw: haloed output
    (36, 72, 1536, 2, 0, False, 0, False),     # b1.1 pwl
    (36, 72, 1536, 2, 0, True, 0, False),      # b1.2 pwl + residual
    (288, 36, 1536, 2, 1, False, 64, False),   # b2.1 pw
    (72, 288, 384, 3, 0, True, 0, True),       # b2.2 pwl: SE gate + residual
    (864, 72, 384, 2, 1, False, 32, False),    # b3.1 pw
    (108, 864, 96, 3, 0, True, 0, True),       # b3 pwl
    (1536, 108, 96, 2, 1, False, 16, False),   # b4.1 pw
    (192, 1536, 24, 5, 0, True, 0, True),      # b4 pwl
    (1536, 192, 24, 3, 1, False, 8, False),    # b4 pw
    (6522, 1024, 1, 300, 0, False, 0, False),  # the head (GEMV_S8 batched: M = windows)
    (10, 20, 7, 3, 2, True, 0, False),         # ragged: ReLU, residual, N and M not multiples of anything
    (40, 36, 100, 2, 1, True, 0, True),        # SiLU + residual + gate (the C ABI allows what v2.4 never uses)
    (5, 3, 129, 1, 1, False, 0, False),        # tiny K
    # a gated small-K layer with SiLU and residual over a partial last tile (288 rows), K = 256 gated over 160 rows,
    # K = 16 with ReLU, K = 40 (the last 16-element chunk ragged) with a haloed output
    (40, 36, 96, 3, 1, True, 0, True),
    (64, 256, 32, 5, 0, False, 0, True),
    (16, 16, 64, 1, 2, False, 0, False),
    (24, 40, 64, 3, 1, True, 8, False),
    # linear layers of K <= 72 take the one-launch form (the quantizer inside the GEMM): 32-, 64- and 128-byte K
    # blocks, several N tiles, ragged last tiles, residual and padded outputs
    (600, 64, 200, 3, 0, True, 0, False),
    (40, 8, 333, 2, 0, False, 9, False),
    (96, 72, 130, 1, 0, True, 0, False),
    (8, 4, 50, 4, 0, False, 0, False),
]


@pytest.mark.parametrize("case", PW_CASES, ids=[f"N{c[0]}K{c[1]}M{c[2]}B{c[3]}" for c in PW_CASES])
def test_pw_s8(lib, case):
    N, K, Mw, B, act, use_res, ow, gated = case
    rng = np.random.default_rng(N * 7 + K)
    (wq, sw, cs, bb), (n, k, kp, np_) = make_pw(rng, N, K)
    lda = (K + 7) // 8 * 8
    ldo = np_
    x = (rng.standard_normal((B, Mw, lda)) * 0.7).astype(np.float32)
    gate = rng.uniform(0, 1, (B, K)).astype(np.float32) if gated else None
    opad = 1 if ow else 0
    oh = Mw // ow if ow else 0
    oelems = ((oh + 2) * (ow + 2) if ow else Mw) * ldo
    res = (rng.standard_normal((B, Mw, ldo)) * 0.5).astype(np.float32) if use_res else None
    h = lib.bnn_pw_s8_new(n, k, kp, np_, wq.ctypes.data, sw.ctypes.data, cs.ctypes.data, bb.ctypes.data, B * Mw)
    assert h, lib.bnn_last_error()
    try:
        out = torch.zeros(B * oelems, dtype=torch.float32, device="cuda")
        xd = dev(x)
        gd = dev(gate) if gated else None
        rd = dev(res) if use_res else None
        rc = lib.bnn_pw_s8_run(h, B, Mw, xd.data_ptr(), Mw * lda, lda, gd.data_ptr() if gated else None, K, act,
                               out.data_ptr(), oelems, ldo, ow, opad, rd.data_ptr() if use_res else None, Mw * ldo, ldo,
                               0, 0, None)
        assert rc == 0, lib.bnn_last_error()
        got = host(out).reshape(B, oelems)
        assert lib.bnn_pw_s8_error(h) == 0
    finally:
        lib.bnn_pw_s8_free(h)
    for w in range(B):
        want = np.zeros(oelems, np.float32)
        q, sa, za = np.zeros((Mw, kp), np.int8), np.zeros(Mw, np.float32), np.zeros(Mw, np.int32)
        oracle.lib().bnno_pw_s8(oracle.ptr(x[w]), lda, Mw, n, k, kp, np_, oracle.ptr(None if gate is None else gate[w]),
                                oracle.ptr(wq), oracle.ptr(sw), oracle.ptr(cs), oracle.ptr(bb), act, oracle.ptr(want),
                                ldo, ow, opad, oh, oracle.ptr(None if res is None else res[w]), ldo, 0, 0,
                                oracle.ptr(q), oracle.ptr(sa), oracle.ptr(za))
        assert bits_equal(got[w], want), f"window {w}: " + mismatch_report(got[w], want)


def test_pw_s8_special_rows(lib):
    """rows with NaN, infinities, huge and tiny values, constant and all-zero rows and ties through the quantizer and
    the GEMM epilogue, against the oracle"""
    N, K, Mw, B = 48, 40, 64, 2
    rng = np.random.default_rng(99)
    (wq, sw, cs, bb), (n, k, kp, np_) = make_pw(rng, N, K)
    x = (rng.standard_normal((B, Mw, K)) * 0.7).astype(np.float32)
    x[0, 0, 3] = np.nan
    x[0, 1, 5] = np.inf
    x[0, 2, 7] = -np.inf
    x[0, 3] = 0.0
    x[0, 4] = 2.5
    x[0, 5] *= 1e30
    x[0, 6] *= 1e-30
    x[0, 7, :] = np.arange(K) - 20.0  # exact ties at .5 after scaling
    x[1, 9, 0] = 3.4e38
    x[1, 9, 1] = -3.4e38
    h = lib.bnn_pw_s8_new(n, k, kp, np_, wq.ctypes.data, sw.ctypes.data, cs.ctypes.data, bb.ctypes.data, B * Mw)
    assert h, lib.bnn_last_error()
    try:
        out = torch.zeros(B * Mw * np_, dtype=torch.float32, device="cuda")
        xd = dev(x)
        assert lib.bnn_pw_s8_run(h, B, Mw, xd.data_ptr(), Mw * K, K, None, 0, 1, out.data_ptr(), Mw * np_, np_, 0, 0,
                                 None, 0, 0, 0, 0, None) == 0, lib.bnn_last_error()
        got = host(out).reshape(B, Mw * np_)
        assert lib.bnn_pw_s8_error(h) == 0
    finally:
        lib.bnn_pw_s8_free(h)
    for w in range(B):
        want = np.zeros(Mw * np_, np.float32)
        q, sa, za = np.zeros((Mw, kp), np.int8), np.zeros(Mw, np.float32), np.zeros(Mw, np.int32)
        oracle.lib().bnno_pw_s8(oracle.ptr(x[w]), K, Mw, n, k, kp, np_, None, oracle.ptr(wq), oracle.ptr(sw),
                                oracle.ptr(cs), oracle.ptr(bb), 1, oracle.ptr(want), np_, 0, 0, 0, None, np_, 0, 0,
                                oracle.ptr(q), oracle.ptr(sa), oracle.ptr(za))
        assert bits_equal(got[w], want), f"window {w}: " + mismatch_report(got[w], want)


# ------------------------------------------------------------------ DW3

@pytest.mark.parametrize("H,W,C,s", [(48, 128, 72, 2), (24, 64, 72, 1), (24, 64, 288, 2), (12, 32, 288, 1),
                                     (12, 32, 864, 2), (6, 16, 864, 1), (6, 16, 1536, 2), (3, 8, 1536, 1),
                                     (5, 7, 16, 1), (9, 5, 40, 2)])
def test_dw3(lib, H, W, C, s):
    rng = np.random.default_rng(H * W + C)
    B = 3
    Ho, Wo = (H - 1) // s + 1, (W - 1) // s + 1
    xp = np.zeros((B, H + 2, W + 2, C), np.float32)
    xp[:, 1:-1, 1:-1, :] = rng.standard_normal((B, H, W, C)).astype(np.float32)
    wt = (rng.standard_normal((9, C)) * 0.4).astype(np.float32)
    bias = (rng.standard_normal(C) * 0.1).astype(np.float32)
    out = torch.zeros(B * Ho * Wo * C, dtype=torch.float32, device="cuda")
    cs = torch.zeros(B * C, dtype=torch.float32, device="cuda")
    xd, wd, bd = dev(xp), dev(wt), dev(bias)
    rc = lib.bnn_cuda_dw3(B, xd.data_ptr(), (H + 2) * (W + 2) * C, H, W, C, s, wd.data_ptr(), bd.data_ptr(),
                          out.data_ptr(), Ho * Wo * C, Ho, Wo, cs.data_ptr(), C, None)
    assert rc == 0, lib.bnn_last_error()
    got, gcs = host(out).reshape(B, -1), host(cs).reshape(B, C)
    for w in range(B):
        o, c = np.zeros(Ho * Wo * C, np.float32), np.zeros(C, np.float32)
        oracle.lib().bnno_dw3(oracle.ptr(xp[w]), H, W, C, s, oracle.ptr(wt), oracle.ptr(bias), oracle.ptr(o), Ho, Wo,
                              oracle.ptr(c))
        assert bits_equal(got[w], o), mismatch_report(got[w], o)
        assert bits_equal(gcs[w], c), mismatch_report(gcs[w], c)


@pytest.mark.parametrize("H,W,C,s,B", [(24, 64, 72, 1, 3), (48, 128, 72, 2, 2), (24, 64, 72, 1, 256), (13, 9, 16, 1, 5)])
def test_dw3_without_channel_sums(lib, H, W, C, s, B):
    """d_chsum NULL (the whole-package form for a DW3 whose sums no op reads): the output rows are cut into bands over
    several CTAs per window; the outputs stay the reference's bit for bit (B = 256: the benchmarked batch of the
    v2.4 block-1 layers)"""
    rng = np.random.default_rng(H * W + C + B)
    Ho, Wo = (H - 1) // s + 1, (W - 1) // s + 1
    xp = np.zeros((B, H + 2, W + 2, C), np.float32)
    xp[:, 1:-1, 1:-1, :] = rng.standard_normal((B, H, W, C)).astype(np.float32)
    wt = (rng.standard_normal((9, C)) * 0.4).astype(np.float32)
    bias = (rng.standard_normal(C) * 0.1).astype(np.float32)
    out = torch.zeros(B * Ho * Wo * C, dtype=torch.float32, device="cuda")
    xd, wd, bd = dev(xp), dev(wt), dev(bias)
    rc = lib.bnn_cuda_dw3(B, xd.data_ptr(), (H + 2) * (W + 2) * C, H, W, C, s, wd.data_ptr(), bd.data_ptr(),
                          out.data_ptr(), Ho * Wo * C, Ho, Wo, None, C, None)
    assert rc == 0, lib.bnn_last_error()
    got = host(out).reshape(B, -1)
    for w in sorted({0, 1, B // 2, B - 1}):
        o, c = np.zeros(Ho * Wo * C, np.float32), np.zeros(C, np.float32)
        oracle.lib().bnno_dw3(oracle.ptr(xp[w]), H, W, C, s, oracle.ptr(wt), oracle.ptr(bias), oracle.ptr(o), Ho, Wo,
                              oracle.ptr(c))
        assert bits_equal(got[w], o), f"window {w}: " + mismatch_report(got[w], o)


# ------------------------------------------------------------------ every op of the packages, one at a time

def oracle_states(pkg, pcm):
    """The oracle's buffers after each window's run (every buffer has memory of its own there)."""
    states = []
    for w in range(pcm.shape[0]):
        p = oracle.Package(pkg)
        p.run_range(pcm[w], 0, p.n_ops)
        states.append(p)
    return states


@pytest.mark.parametrize("which", ["mini", "full"])
def test_every_op(lib, which, mini_pkg, full_pkg):
    pkg = mini_pkg if which == "mini" else full_pkg
    ops, bufs = pkgread.read_ops(pkg)
    B = 2
    pcm = synth.audio(B, seed=5)
    states = oracle_states(pkg, pcm)
    m = Model(pkg, batch=B)
    try:
        for i, (code, bl, _, _) in enumerate(ops):
            ins, outs = pkgread.op_io(code, bl)
            for b in ins:
                if b == 0:
                    continue
                m.set_buffer(b, np.stack([s.get(b) for s in states]))
            m.run_ops(pcm, i, i + 1)
            for b in outs:
                if code == 6 and b != bl[1]:
                    continue  # POSTPC's im2col / GEMM rows stay in the runtime's own scratch
                elems, dt = states[0].buf_info(b)
                got = m.get_buffer(b, B, dt, elems)
                for w in range(B):
                    want = states[w].get(b)
                    assert bits_equal(got[w], want), (f"op {i} {pkgread.NAMES[code]} buffer {b} window {w}: "
                                                      + mismatch_report(got[w], want))
    finally:
        m.close()


# ------------------------------------------------------------------ end to end

@pytest.mark.parametrize("which,n", [("mini", 5), ("full", 3)])
def test_end_to_end(lib, which, n, mini_pkg, full_pkg):
    pkg = mini_pkg if which == "mini" else full_pkg
    pcm = synth.audio(n, seed=9)
    want, wemb = oracle.run_many(pkg, pcm, threads=4)
    with Model(pkg, batch=2) as m:  # 2 windows per launch: exercises chunking
        got, gemb = m.infer_batch(pcm)
        one, oemb = m.infer(pcm[1])
    assert bits_equal(got, want), mismatch_report(got, want)
    assert bits_equal(gemb, wemb), mismatch_report(gemb, wemb)
    assert bits_equal(one, want[1]) and bits_equal(oemb, wemb[1])


def test_batch_split_invariance(lib, mini_pkg):
    """Per-window results do not depend on the batch they are scored in (the reference's thread-count guarantee)."""
    pcm = synth.audio(7, seed=21)
    with Model(mini_pkg, batch=7) as m:
        a, ea = m.infer_batch(pcm)
        m.set_batch(3)
        b, eb = m.infer_batch(pcm)
    assert bits_equal(a, b) and bits_equal(ea, eb)


def test_graph_replay(lib, mini_pkg):
    """Launch sequences are replayed from CUDA graphs from the second call with the same windows and input buffer on:
    four calls with different audio (the 1st eager, the 2nd captured, the 3rd and 4th replayed; both upload buffers),
    each against the oracle; then the device entry point the same way."""
    n = 6
    with Model(mini_pkg, mode=4, batch=3) as m:  # chunks of 3 windows alternate between the two upload buffers
        for call in range(4):
            pcm = synth.audio(n, seed=100 + call)
            want, wemb = oracle.run_many(mini_pkg, pcm, threads=4)
            got, gemb = m.infer_batch(pcm)
            assert bits_equal(got, want) and bits_equal(gemb, wemb), (call, mismatch_report(got, want))
        d_out = torch.zeros((3, m.info.n_classes), dtype=torch.float32, device="cuda")
        d_emb = torch.zeros((3, m.info.emb_dim), dtype=torch.float32, device="cuda")
        d_pcm = torch.zeros((3, synth.NSAMP), dtype=torch.float32, device="cuda")
        for call in range(3):
            pcm = synth.audio(3, seed=200 + call)
            d_pcm.copy_(torch.from_numpy(pcm))
            m.infer_device(3, d_pcm.data_ptr(), d_out.data_ptr(), d_emb.data_ptr())
            want, wemb = oracle.run_many(mini_pkg, pcm, threads=3)
            assert bits_equal(host(d_out), want) and bits_equal(host(d_emb), wemb), call


def test_device_entry_point(lib, mini_pkg):
    pcm = synth.audio(4, seed=2)
    with Model(mini_pkg, batch=4) as m:
        want, wemb = m.infer_batch(pcm)
        d_pcm = dev(pcm)
        d_out = torch.zeros((4, m.info.n_classes), dtype=torch.float32, device="cuda")
        d_emb = torch.zeros((4, m.info.emb_dim), dtype=torch.float32, device="cuda")
        m.infer_device(4, d_pcm.data_ptr(), d_out.data_ptr(), d_emb.data_ptr())
        assert bits_equal(host(d_out), want) and bits_equal(host(d_emb), wemb)


def test_two_gpus_in_one_context(lib, mini_pkg):
    """bnn_set_threads(ctx, 2) spreads a batch over two GPUs in one process; outputs equal one GPU's bit for bit."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two visible GPUs")
    pcm = synth.audio(9, seed=5)
    with Model(mini_pkg, mode=4, batch=4) as m1:
        out1, emb1 = m1.infer_batch(pcm)
    with Model(mini_pkg, mode=4, batch=4) as m2:
        m2.set_threads(2)
        out2, emb2 = m2.infer_batch(pcm)
    assert bits_equal(out1, out2), mismatch_report(out1, out2)
    assert bits_equal(emb1, emb2), mismatch_report(emb1, emb2)
