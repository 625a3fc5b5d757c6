"""The Perch-v2-architecture model on the neon-int8 path (the reference ships perch_v2-neon-int8.bnpk): FE_LOGMEL, the
fp32 STEM, DW3 / PAD + DWK, SE_GATE, PW_S8 for the expansions and the 1536-channel top conv, the SE-gated fp32 PW for
the projections, MEAN and the int8 prototype head PROTO_S8 — the reference compiler's default int8 policy.

* CPU: synth.write_perch_int8_package writes the reference compiler's bytes (tests/golden/perch_int8_packages.json,
  made by tests/golden/make_golden.py with the reference's lower.py); the reference runtime (oracle/_ref) and the B200
  loader both accept the package.
* GPU: bnn_infer_batch against the reference runtime run on the same package and windows, bit for bit (logits and the
  1536-d embedding), on the mini model (every op kind and geometry of the full one) and on sampled windows of the full
  model at batch 64.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import bits_equal, mismatch_report, gpu_visible
from bnneon_b200 import BnnError, Model, synth
from oracle import ref

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "perch_int8_packages.json"), encoding="utf-8") as fh:
    PACKAGES = json.load(fh)
MODE_INT8 = 4


@pytest.fixture(scope="module")
def mini_int8(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("perch8") / "perch_v2_int8_mini.bnpk")
    _, _, ns = synth.write_perch_int8_package(path, synth.perch_ir(0, mini=True))
    return path, ns


@pytest.fixture(scope="module")
def reflib():
    if ref.reference_checkout() is not None:
        ref.build()
    if not ref.available():
        pytest.skip("no reference build (oracle/_ref) and no reference checkout to build it from")
    return ref.lib()


def test_mini_package_bytes_match_reference_compiler(mini_int8):
    path, _ = mini_int8
    g = PACKAGES["perch_v2_int8_mini"]
    with open(path, "rb") as f:
        data = f.read()
    assert len(data) == g["size"] and hashlib.sha256(data).hexdigest() == g["sha256"]


def test_reference_and_loader_accept(reflib, mini_int8):
    path, ns = mini_int8
    pcm = synth.audio(2, seed=5, n_samples=ns, rate=synth.PERCH_SAMPLE_RATE)
    out, emb, rc = ref.run_many(path, MODE_INT8, pcm, threads=2)
    assert (rc == 0).all() and np.isfinite(out).all() and emb.shape == (2, 1536)
    if not gpu_visible():
        with pytest.raises(BnnError) as e:
            Model(path, mode=MODE_INT8)
        assert e.value.kind == "CPU" and "no CUDA device" in str(e.value), str(e.value)


# ------------------------------------------------------------------ GPU

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    torch.cuda.init()


@pytest.mark.gpu
def test_mini_against_reference(cuda, reflib, mini_int8):
    path, ns = mini_int8
    pcm = synth.audio(10, seed=21, n_samples=ns, rate=synth.PERCH_SAMPLE_RATE)
    want, wemb, rc = ref.run_many(path, MODE_INT8, pcm, threads=min(10, os.cpu_count() or 1))
    assert (rc == 0).all()
    with Model(path, mode=MODE_INT8, batch=4) as m:
        assert m.info.path.decode() == "neon-int8"
        for call in range(3):  # eager, captured, replayed
            got, gemb = m.infer_batch(pcm)
            assert bits_equal(got, want), f"call {call} logits: " + mismatch_report(got, want)
            assert bits_equal(gemb, wemb), f"call {call} embedding: " + mismatch_report(gemb, wemb)


@pytest.mark.gpu
def test_full_sampled_batch64(cuda, reflib, tmp_path):
    path = str(tmp_path / "perch_v2_int8.bnpk")
    _, _, ns = synth.write_perch_int8_package(path, synth.perch_ir(0))
    B = 64
    pcm = synth.audio(B, seed=4200, n_samples=ns, rate=synth.PERCH_SAMPLE_RATE)
    idx = np.array([0, 15, 16, 63])
    want, wemb, rc = ref.run_many(path, MODE_INT8, np.ascontiguousarray(pcm[idx]), threads=4)
    assert (rc == 0).all()
    with Model(path, mode=MODE_INT8, batch=B) as m:
        got, gemb = m.infer_batch(pcm)
    assert bits_equal(got[idx], want), mismatch_report(got[idx], want)
    assert bits_equal(gemb[idx], wemb), mismatch_report(gemb[idx], wemb)
