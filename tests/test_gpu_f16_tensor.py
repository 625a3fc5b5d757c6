"""The neon-fp16 path's tensor mode (bnn_set_fp16_tensor): its 1x1 convs (PW f16) run as tcgen05 kind::f16 GEMMs
with fp32 accumulators instead of the reference's fp16 FMA chains (src/gemm_f16.c:109-169). The sums are exact products
added in fp32, so results differ from the reference's (and the oracle's) in the last fp16 bits; parity is by
tolerance, stated here:

* op by op, each PW f16 of the packages on the oracle's inputs: SQNR >= 50 dB against the oracle's output (the
  reference compiler's own screen for an fp16 layer, lower.py:69-71 need_db = 50.0); all but one in 10^4 elements
  within 2^-6 max(|want|, rms(want)) (about two fp16 units in the last place at that magnitude: what the reference's
  own fp16 chains, one rounding per k-step for up to 128 steps, drift from an exact sum) and every element within
  2^-4 max(|want|, rms(want)) (outputs whose sum cancels carry the chain's error of its larger partial sums);
* whole models: logits and embeddings within 40 dB SQNR of the bit-exact mode on the full v2.4 package (C3, batch
  1024, sampled windows) and the Perch package (C4, batch 512, sampled windows), and on the mini model no further
  from a float64 forward pass of the same weights than the reference's own fp16 arithmetic is (within 1 dB), and
  >= 50 dB from it;
* every other op stays bit-exact, and switching the mode off gives the bit-exact results again.
"""
import numpy as np
import pytest

from conftest import bits_equal, mismatch_report
from bnneon_b200 import Model, load_library, pkgread, synth
from oracle import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
PATH = synth.PATH_F16
PW_F16 = 0x103


def sqnr_db(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return 10 * np.log10(np.sum(want ** 2) / max(np.sum((got - want) ** 2), 1e-300))


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    h = load_library()
    torch.cuda.init()
    assert h.bnn_cuda_device_init() == 0, h.bnn_last_error()
    return h


@pytest.fixture(scope="module")
def pkgs(tmp_path_factory):
    d = tmp_path_factory.mktemp("tc16")
    out = {}
    for name, (seed, blocks, nc) in {"mini": (1, synth.MINI_BLOCKS, 100), "full": (0, synth.V24_BLOCKS, 6522)}.items():
        out[name] = str(d / f"{name}.bnpk")
        synth.write_f16_package(out[name], synth.v24_ir(seed, nc, blocks))
    out["perch"] = str(d / "perch.bnpk")
    out["perch_ns"] = synth.write_perch_package(out["perch"], synth.perch_ir(0, mini=True))[2]
    return out


@pytest.mark.parametrize("which", ["mini", "full", "perch"])
def test_tensor_mode_op_by_op(lib, which, pkgs):
    pkg = pkgs[which]
    ops, _ = pkgread.read_ops(pkg, PATH)
    B = 2
    pcm = synth.audio(B, seed=5, **({} if which != "perch" else
                                     dict(n_samples=pkgs["perch_ns"], rate=synth.PERCH_SAMPLE_RATE)))
    states = [oracle.Package(pkg, PATH) for _ in range(B)]
    n_pw = 0
    with Model(pkg, mode=3, batch=B, fp16_tensor=True) as m:
        assert m.fp16_tensor
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
                    g, h = got[w].astype(np.float64), want.astype(np.float64)
                    where = f"op {i} {pkgread.NAMES[code]} buffer {b} window {w}"
                    if code == PW_F16:
                        assert np.isfinite(g).all() and np.isfinite(h).all(), where
                        rms = np.sqrt(np.mean(h ** 2))
                        assert sqnr_db(g, h) >= 50, f"{where}: {sqnr_db(g, h):.1f} dB"
                        scale = np.maximum(np.abs(h), rms)
                        bad = np.abs(g - h) > 2.0 ** -6 * scale
                        assert bad.sum() <= bad.size // 10000, (f"{where}: {int(bad.sum())} of {bad.size} beyond "
                                                                f"2^-6, worst {np.abs(g - h).max():.3g} at rms {rms:.3g}")
                        assert (np.abs(g - h) <= 2.0 ** -4 * scale).all(), (
                            f"{where}: worst {np.abs(g - h).max():.3g} at rms {rms:.3g} beyond 2^-4")
                    elif dt == np.float16:
                        gn, hn = np.isnan(g), np.isnan(h)
                        gb = got[w].view(np.uint16)
                        hb = want.view(np.uint16)
                        assert np.array_equal(gn, hn) and np.array_equal(gb[~gn], hb[~hn]), where
                    else:
                        assert bits_equal(got[w], want), where + ": " + mismatch_report(got[w], want)
            n_pw += code == PW_F16
    assert n_pw > 0


def test_tensor_mode_tracks_float64_like_the_reference(lib, pkgs):
    from test_f16_cpu import GOLD, f64_forward, model_ir  # pylint: disable=import-outside-toplevel
    ir = model_ir(GOLD["v24_mini_f16"])
    pcm = synth.audio(3, seed=3)
    ref_logits, ref_emb = oracle.run_many(pkgs["mini"], pcm, threads=3, path_name=PATH)
    with Model(pkgs["mini"], mode=3, batch=3, fp16_tensor=True) as m:
        got, gemb = m.infer_batch(pcm)
    for w in range(3):
        p = oracle.Package(pkgs["mini"], PATH)
        p.run_range(pcm[w], 0, 1)
        want, wemb = f64_forward(ir, p.get(1).reshape(96, 511, 2))
        for name, g, r, x in (("logits", got[w], ref_logits[w], want), ("embedding", gemb[w], ref_emb[w], wemb)):
            s_tc, s_ref = sqnr_db(g, x), sqnr_db(r, x)
            assert s_tc >= 50, f"window {w} {name}: tensor mode {s_tc:.1f} dB from float64"
            assert s_tc >= s_ref - 1.0, f"window {w} {name}: tensor mode {s_tc:.1f} dB, reference arithmetic {s_ref:.1f} dB"


@pytest.mark.parametrize("which,batch,k", [("full", 1024, 16), ("perch", 512, 8)])
def test_tensor_mode_at_benchmarked_batch(lib, which, batch, k, tmp_path):
    if which == "full":
        pkg = str(tmp_path / "full.bnpk")
        synth.make_package(pkg, seed=0, path=PATH)
        pcm = synth.audio(batch, seed=4000)
    else:
        pkg = str(tmp_path / "perch.bnpk")
        _, _, ns = synth.write_perch_package(pkg, synth.perch_ir(0))
        pcm = synth.audio(batch, seed=4100, n_samples=ns, rate=synth.PERCH_SAMPLE_RATE)
    idx = np.unique(np.concatenate([[0, 1, batch // 4 - 1, batch // 4, batch // 2, batch - 2, batch - 1],
                                    np.random.default_rng(1).choice(batch, k - 7, replace=False)]))
    with Model(pkg, mode=3, batch=batch) as m:
        exact, eemb = m.infer_batch(pcm)
        m.set_fp16_tensor(True)
        got, gemb = m.infer_batch(pcm)
        m.set_fp16_tensor(False)
        back, bemb = m.infer_batch(pcm)
    assert bits_equal(back, exact) and bits_equal(bemb, eemb)
    want, wemb = oracle.run_many(pkg, np.ascontiguousarray(pcm[idx]), threads=8, path_name=PATH)
    assert bits_equal(exact[idx], want), mismatch_report(exact[idx], want)
    for j, w in enumerate(idx):
        assert np.isfinite(got[w]).all() and np.isfinite(gemb[w]).all()
        assert sqnr_db(got[w], want[j]) >= 40, f"window {w}: logits {sqnr_db(got[w], want[j]):.1f} dB"
        assert sqnr_db(gemb[w], wemb[j]) >= 40, f"window {w}: embedding {sqnr_db(gemb[w], wemb[j]):.1f} dB"
