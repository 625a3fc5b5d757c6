"""GPU parity of a Perch-v2-architecture package (neon-fp16 body with the int8 SDOT prototype head, bnc.py compile
--paths neon-fp16 --proto-s8): every op and whole packages bit for bit against the CPU oracle, through the C ABI.

The mini model has every op kind and geometry of the full one (DW3 on the stem output, PAD + DWK 3x3, every strided
depthwise form, 5x5 depthwise convs, DWK above 2048 channels, the prototype head, the embedding mean) on 2.5 s
windows; the full model is Perch v2's backbone and head (59180 prototypes) on 5 s windows.
"""
import numpy as np
import pytest

from conftest import bits_equal, mismatch_report
from bnneon_b200 import Model, load_library, pkgread, synth
from oracle import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
PATH = synth.PATH_F16


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    h = load_library()
    torch.cuda.init()
    assert h.bnn_cuda_device_init() == 0, h.bnn_last_error()
    return h


@pytest.fixture(scope="module")
def perch_pkgs(tmp_path_factory):
    d = tmp_path_factory.mktemp("perchpkg")
    out = {}
    for name, mini in (("mini", True), ("full", False)):
        out[name] = str(d / f"perch_{name}.bnpk")
        ns = synth.write_perch_package(out[name], synth.perch_ir(0, mini=mini))[2]
        out[name + "_ns"] = ns
    return out


def pcm_for(pkgs, which, n, seed):
    return synth.audio(n, seed=seed, n_samples=pkgs[which + "_ns"], rate=synth.PERCH_SAMPLE_RATE)


def test_perch_every_op(lib, perch_pkgs):
    """Op by op on the mini model: the GPU op on the oracle's inputs against the oracle's outputs (fp16 buffers as bit
    patterns, any NaN equal to any NaN; fp32 buffers bit for bit)."""
    pkg = perch_pkgs["mini"]
    ops, _ = pkgread.read_ops(pkg, PATH)
    B = 2
    pcm = pcm_for(perch_pkgs, "mini", B, 5)
    states = [oracle.Package(pkg, PATH) for _ in range(B)]
    with Model(pkg, mode=3, batch=B) as m:
        assert m.info.path == b"neon-fp16"
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
                    if dt == np.float16:
                        g, h = got[w].view(np.uint16), want.view(np.uint16)
                        gn, hn = np.isnan(got[w].astype(np.float32)), np.isnan(want.astype(np.float32))
                        ok = np.array_equal(gn, hn) and np.array_equal(g[~gn], h[~hn])
                    else:
                        ok = bits_equal(got[w], want)
                    assert ok, (f"op {i} {pkgread.NAMES[code]} buffer {b} window {w}: "
                                + mismatch_report(got[w].astype(np.float32), want.astype(np.float32)))


@pytest.mark.parametrize("which,n", [("mini", 5), ("full", 2)])
def test_perch_end_to_end(lib, which, n, perch_pkgs):
    """Logits and the 1536-d embedding of whole windows, bit for bit; batches of 2 windows per launch (chunking and
    graph replay) and a single window."""
    pkg = perch_pkgs[which]
    pcm = pcm_for(perch_pkgs, which, n, 9)
    want, wemb = oracle.run_many(pkg, pcm, threads=max(2, n), path_name=PATH)
    with Model(pkg, mode=3, batch=2) as m:
        got, gemb = m.infer_batch(pcm)
        again, _ = m.infer_batch(pcm)
        one, oemb = m.infer(pcm[1])
    assert bits_equal(got, want), mismatch_report(got, want)
    assert bits_equal(gemb, wemb), mismatch_report(gemb, wemb)
    assert bits_equal(again, want)
    assert bits_equal(one, want[1]) and bits_equal(oemb, wemb[1])


def test_perch_batch_split_invariance(lib, perch_pkgs):
    pcm = pcm_for(perch_pkgs, "mini", 7, 21)
    with Model(perch_pkgs["mini"], mode=0, batch=7) as m:
        assert m.info.path == b"neon-fp16"
        a, ea = m.infer_batch(pcm)
        m.set_batch(3)
        b, eb = m.infer_batch(pcm)
    assert bits_equal(a, b) and bits_equal(ea, eb)


# ------------------------------------------------------------------ DWK f16 and STEM f16 through their own C ABI

# (H, W, C, k, s, pt, pl, act, extra window stride in halves): every k the kernels take, both strides, every pad,
# rows ending in a pair and a single pixel, tall and wide maps, 2304 channels, and a window stride that is not a
# multiple of 4 halves (the channel-pair form)
DWK_CASES = [(13, 11, 16, 3, 1, 1, 1, 1, 0), (13, 11, 16, 3, 2, 1, 0, 1, 0), (17, 9, 24, 5, 1, 2, 2, 1, 0),
             (17, 10, 24, 5, 2, 2, 1, 0, 0), (11, 13, 8, 7, 1, 3, 3, 1, 0), (15, 15, 8, 7, 2, 1, 2, 1, 0),
             (9, 7, 32, 1, 1, 0, 0, 1, 0), (9, 7, 32, 1, 2, 0, 0, 1, 0), (300, 6, 8, 3, 1, 1, 1, 1, 0),
             (12, 11, 40, 5, 1, 2, 2, 1, 2), (8, 4, 2304, 3, 1, 1, 1, 1, 0), (20, 300, 8, 3, 1, 1, 1, 1, 0)]


def h16_equal(got, want):
    gn, hn = np.isnan(got.astype(np.float32)), np.isnan(want.astype(np.float32))
    return np.array_equal(gn, hn) and np.array_equal(got.view(np.uint16)[~gn], want.view(np.uint16)[~hn])


@pytest.mark.parametrize("case", DWK_CASES, ids=lambda c: "x".join(map(str, c)))
def test_dwk_f16_shapes(lib, case):
    H, W, C, k, s, pt, pl, act, extra = case
    h = (k - 1) // 2
    Ho, Wo = (H + h + pt - k) // s + 1, (W + h + pl - k) // s + 1
    B = 3
    rng = np.random.default_rng(hash(case) % 2 ** 32)
    xp = np.zeros((B, H + 2 * h, W + 2 * h, C), np.float16)
    xp[:, h:h + H, h:h + W] = rng.standard_normal((B, H, W, C)).astype(np.float16)
    w = (rng.standard_normal((k * k, C)) * 0.3).astype(np.float16)
    b = (rng.standard_normal(C) * 0.1).astype(np.float16)
    xws = (H + 2 * h) * (W + 2 * h) * C + extra
    flat = np.zeros(B * xws, np.float16)
    for i in range(B):
        flat[i * xws:i * xws + xp[i].size] = xp[i].ravel()
    d_x = torch.from_numpy(flat.view(np.int16)).cuda()
    d_w, d_b = torch.from_numpy(w.view(np.int16)).cuda(), torch.from_numpy(b.view(np.int16)).cuda()
    d_out = torch.zeros(B * Ho * Wo * C, dtype=torch.int16, device="cuda")
    d_cs = torch.zeros(B * C, dtype=torch.float32, device="cuda")
    assert lib.bnn_cuda_dwk_f16(B, d_x.data_ptr(), xws, H, W, C, k, s, pt, pl, d_w.data_ptr(), d_b.data_ptr(), act,
                                d_out.data_ptr(), Ho * Wo * C, Ho, Wo, d_cs.data_ptr(), C, None) == 0, lib.bnn_last_error()
    torch.cuda.synchronize()
    got = d_out.cpu().numpy().view(np.float16).reshape(B, Ho * Wo * C)
    gcs = d_cs.cpu().numpy().reshape(B, C)
    for i in range(B):
        want = np.zeros(Ho * Wo * C, np.uint16)
        wcs = np.zeros(C, np.float32)
        xi = np.ascontiguousarray(xp[i]).view(np.uint16)
        oracle.lib().bnno_dwk_f16(oracle.ptr(xi), H, W, C, k, s, pt, pl, oracle.ptr(w.view(np.uint16)),
                                  oracle.ptr(b.view(np.uint16)), act, oracle.ptr(want), Ho, Wo, oracle.ptr(wcs))
        assert h16_equal(got[i], want.view(np.float16)), f"window {i}: " + mismatch_report(
            got[i].astype(np.float32), want.view(np.float16).astype(np.float32))
        assert bits_equal(gcs[i], wcs), mismatch_report(gcs[i], wcs)


# (H, W, k, s, N, Kp, act, ldo, opad): the 3x3 form (Perch's stem), other k on the general form, partial panels, channel
# strides above Np, halos 0..2
STEM_CASES = [(40, 24, 3, 2, 40, 12, 1, 40, 1), (21, 19, 5, 1, 20, 28, 2, 24, 0), (30, 17, 3, 1, 16, 16, 0, 32, 2),
              (25, 25, 1, 3, 8, 4, 1, 8, 0), (33, 20, 3, 2, 12, 12, 1, 16, 1)]


@pytest.mark.parametrize("case", STEM_CASES, ids=lambda c: "x".join(map(str, c)))
def test_stem_f16_shapes(lib, case):
    """the stem's fp16 outputs bit for bit; channels N..ldo and the halo keep what was there (a sentinel)"""
    H, W, k, s, N, Kp, act, ldo, opad = case
    Ho, Wo = (H - k) // s + 1, (W - k) // s + 1
    B = 2
    rng = np.random.default_rng(sum(case))
    img = (rng.standard_normal((B, H, W)) * 3).astype(np.float32)
    wt = (rng.standard_normal((N, k * k)) * 0.5).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float32)
    panels, bb, (_, _, kp, np_) = synth._Int8Lowering.pack_f32(wt, bias, Kp)  # pylint: disable=protected-access
    assert kp == Kp
    pw = np.ascontiguousarray(panels[:np_ * Kp])
    ows = (Ho + 2 * opad) * (Wo + 2 * opad) * ldo
    sentinel = np.full(B * ows, 0x7bff, np.uint16)
    d_img = torch.from_numpy(img).cuda()
    d_w, d_b = torch.from_numpy(pw).cuda(), torch.from_numpy(bb).cuda()
    d_out = torch.from_numpy(sentinel.view(np.int16)).cuda()
    assert lib.bnn_cuda_stem_f16(B, d_img.data_ptr(), H * W, H, W, k, s, Ho, Wo, d_w.data_ptr(), d_b.data_ptr(), N, Kp,
                                 act, d_out.data_ptr(), ows, ldo, opad, None) == 0, lib.bnn_last_error()
    torch.cuda.synchronize()
    got = d_out.cpu().numpy().view(np.uint16).reshape(B, Ho + 2 * opad, Wo + 2 * opad, ldo)
    for i in range(B):
        want = np.full((Ho + 2 * opad, Wo + 2 * opad, ldo), 0x7bff, np.uint16)
        oracle.lib().bnno_stem_f16(oracle.ptr(np.ascontiguousarray(img[i])), H, W, k, s, Ho, Wo, oracle.ptr(pw),
                                   oracle.ptr(bb), N, Kp, act, oracle.ptr(want), ldo, opad)
        assert np.array_equal(got[i], want), f"window {i}: " + mismatch_report(
            got[i].view(np.float16).astype(np.float32), want.view(np.float16).astype(np.float32))


def test_dwk_and_stem_refuse_bad_shapes(lib):
    assert lib.bnn_cuda_dwk_f16(1, 1, 0, 8, 8, 12, 3, 1, 1, 1, 1, 1, 1, 1, 0, 8, 8, 1, 0, None) == -1
    assert "C % 8 == 0" in lib.bnn_last_error().decode()
    assert lib.bnn_cuda_dwk_f16(1, 1, 0, 8, 8, 8, 4, 1, 1, 1, 1, 1, 1, 1, 0, 8, 8, 1, 0, None) == -1
    assert lib.bnn_cuda_stem_f16(1, 1, 0, 8, 8, 3, 1, 7, 6, 1, 1, 8, 12, 1, 1, 0, 8, 0, None) == -1
    assert "VALID conv" in lib.bnn_last_error().decode()


def test_perch_nonfinite_logits_fail_the_window(lib, tmp_path):
    """class weights of 1e38 send the logits past 3e38: pc_proto_logits returns -2 (src/pc_kern_f32.c:364-376), the
    oracle refuses the window, and the library reports every window failed (BNN_ERR_WINDOW, the prototype head and
    the first failed window named), as the reference's rt_run / bnn_infer report it"""
    from bnneon_b200 import BnnError  # pylint: disable=import-outside-toplevel
    ops, vshape, lv, ev, fe = synth.perch_ir(4, mini=True)
    for o in ops:
        if o["op"] == "PROTO":
            o["cw"] = np.full_like(o["cw"], 1e38)
    pkg = str(tmp_path / "perch_overflow.bnpk")
    synth.write_perch_package(pkg, (ops, vshape, lv, ev, fe))
    pcm = synth.audio(3, seed=6, n_samples=fe["nsamp"], rate=synth.PERCH_SAMPLE_RATE)
    with pytest.raises(RuntimeError):
        oracle.Package(pkg, PATH).run(pcm[0])
    with Model(pkg, mode=3, batch=4) as m:
        with pytest.raises(BnnError) as e:
            m.infer_batch(pcm)
        assert e.value.kind == "WINDOW" and "proto_s8" in str(e.value) and "window 0" in str(e.value), str(e.value)
