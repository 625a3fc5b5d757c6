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
