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
