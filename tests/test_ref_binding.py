"""The reference's own Python binding (python/bnneon/binding.py, installed unchanged under baseline/_ref) drives this
libbnneon.so: the reference's compatibility check for hosts (its binding is how Python hosts call the library).
Skipped when the reference package is not installed in baseline/_ref.

Probe, metadata and label checks need no GPU; inference through the reference binding is compared bit for bit with
this repository's batched entry point.
"""
import importlib.util
import os

import numpy as np
import pytest

from conftest import REPO, bits_equal, mismatch_report
from bnneon_b200 import DEFAULT_LIB, synth

REF_BINDING = os.path.join(REPO, "baseline", "_ref", "bnneon", "binding.py")


@pytest.fixture(scope="module")
def refb():
    if not os.path.exists(REF_BINDING):
        pytest.skip("the reference package is not installed in baseline/_ref")
    spec = importlib.util.spec_from_file_location("ref_binding", REF_BINDING)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_binding_probe_and_meta(refb, mini_pkg):
    info = refb.probe(mini_pkg, lib=DEFAULT_LIB)
    assert info.n_samples == 144000 and info.n_classes == 64 and info.emb_dim == 1024
    assert info.path == b"neon-int8"
    assert refb.probe_meta(mini_pkg, "model_id", lib=DEFAULT_LIB) is not None


@pytest.mark.gpu
def test_reference_binding_infer_matches(refb, mini_pkg):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    from bnneon_b200 import Model  # pylint: disable=import-outside-toplevel
    pcm = synth.audio(3, seed=77)
    with refb.Model(mini_pkg, mode=4, lib=DEFAULT_LIB) as m:
        assert m.info.path == b"neon-int8"
        got = [m.infer(pcm[i]) for i in range(3)]
        labels = m.labels()
    with Model(mini_pkg, mode=4, batch=4) as ours:
        out, emb = ours.infer_batch(pcm)
    for i in range(3):
        assert bits_equal(got[i][0], out[i]), mismatch_report(got[i][0], out[i])
        assert bits_equal(got[i][1], emb[i]), mismatch_report(got[i][1], emb[i])
    assert labels is not None and len(labels) == 64


@pytest.fixture(scope="module")
def perch_mini_pkg(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("refb_perch") / "perch_mini.bnpk")
    synth.make_perch_package(path, seed=3, mini=True)
    return path


def test_reference_binding_probes_a_perch_package(refb, perch_mini_pkg):
    """the reference's binding probes a Perch-architecture fp16 package through this library (no GPU needed)"""
    info = refb.probe(perch_mini_pkg, lib=DEFAULT_LIB)
    assert info.n_samples == 80000 and info.n_classes == 61 and info.emb_dim == 1536
    assert info.path == b"neon-fp16"


@pytest.mark.gpu
def test_reference_binding_runs_a_perch_package(refb, perch_mini_pkg):
    """mode 3 (neon-fp16) through the reference's binding: logits and the 1536-d embedding bit for bit against this
    repository's batched entry point"""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    from bnneon_b200 import Model  # pylint: disable=import-outside-toplevel
    pcm = synth.audio(2, seed=78, n_samples=80000, rate=synth.PERCH_SAMPLE_RATE)
    with refb.Model(perch_mini_pkg, mode=3, lib=DEFAULT_LIB) as m:
        assert m.info.path == b"neon-fp16"
        got = [m.infer(pcm[i]) for i in range(2)]
    with Model(perch_mini_pkg, mode=3, batch=2) as ours:
        out, emb = ours.infer_batch(pcm)
    for i in range(2):
        assert bits_equal(got[i][0], out[i]), mismatch_report(got[i][0], out[i])
        assert bits_equal(got[i][1], emb[i]), mismatch_report(got[i][1], emb[i])
