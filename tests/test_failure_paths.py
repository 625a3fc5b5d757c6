"""Failure paths in the forms that fault no GPU.

* Allocation failure (the reference maps every failed allocation to BNN_ERR_OOM, src/bnneon.h:90-92, its kernels'
  rt_oom): bnn_debug_fail_alloc makes the k-th host or device allocation of the library fail as if memory had run
  out. Host allocations run on the CPU (the context, the op list: before any device is touched); device allocations
  (activation arena, scratch, weights) on the GPU. The failed bnn_init frees what it had and the next one works.
* A bounded wait that runs out (every mbarrier wait of the tensor-core kernels has a deadline): bnn_debug_stall_next_gemm
  makes the next int8 GEMM's producer issue no TMA load and no MMA and shortens its waits to 200 us, so every consumer
  wait runs out with nothing in flight. The call fails with BNN_ERR_WINDOW ("a GPU kernel's bounded wait ran out"),
  the error word is cleared, and the same context then scores the same windows bit-exactly.
"""
import numpy as np
import pytest

from conftest import bits_equal, mismatch_report, gpu_visible
from bnneon_b200 import BnnError, Model, load_library, synth
from oracle import oracle


@pytest.fixture
def lib():
    h = load_library()
    yield h
    h.bnn_debug_fail_alloc(0, 0)


def init_error(path, **kw):
    with pytest.raises(BnnError) as e:
        Model(path, mode=4, **kw)
    return e.value


@pytest.mark.parametrize("k, what", [(1, "context"), (2, "op list")])
def test_host_allocation_failure_is_oom(lib, mini_pkg, k, what):
    assert lib.bnn_debug_fail_alloc(k, 0) == 0
    e = init_error(mini_pkg)
    assert e.kind == "OOM" and "out of memory" in str(e) and what in str(e), str(e)
    # the hook is spent: the next init goes on as usual
    if not gpu_visible():
        e = init_error(mini_pkg)
        assert e.kind == "CPU" and "no CUDA device" in str(e), str(e)


def test_fail_alloc_usage(lib):
    assert lib.bnn_debug_fail_alloc(-1, 0) == -1
    assert lib.bnn_debug_fail_alloc(0, 0) == 0


# ------------------------------------------------------------------ GPU

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    torch.cuda.init()


@pytest.mark.gpu
@pytest.mark.parametrize("k", [1, 2, 4, 8, 16, 40])
def test_device_allocation_failure_is_oom(cuda, lib, full_pkg, k):
    """the k-th device allocation of bnn_init fails: OOM with the batch hint; the next context on the same device
    works and scores bit-exactly"""
    assert lib.bnn_debug_fail_alloc(0, k) == 0
    e = init_error(full_pkg, batch=16)
    assert e.kind == "OOM" and "lower the batch" in str(e), str(e)
    lib.bnn_debug_fail_alloc(0, 0)
    pcm = synth.audio(3, seed=k)
    want, wemb = oracle.run_many(full_pkg, pcm, threads=3)
    with Model(full_pkg, mode=4, batch=16) as m:
        got, gemb = m.infer_batch(pcm)
    assert bits_equal(got, want), mismatch_report(got, want)
    assert bits_equal(gemb, wemb), mismatch_report(gemb, wemb)


@pytest.mark.gpu
def test_stalled_gemm_wait_runs_out(cuda, lib, mini_pkg):
    pcm = synth.audio(5, seed=31)
    want, wemb = oracle.run_many(mini_pkg, pcm, threads=5)
    with Model(mini_pkg, mode=4, batch=8) as m:
        lib.bnn_debug_stall_next_gemm()
        with pytest.raises(BnnError) as e:
            m.infer_batch(pcm)
        assert e.value.kind == "WINDOW" and "bounded wait ran out" in str(e.value), str(e.value)
        for call in range(3):  # eager, captured, replayed: the context and the GPU answer as before
            got, gemb = m.infer_batch(pcm)
            assert bits_equal(got, want), (call, mismatch_report(got, want))
            assert bits_equal(gemb, wemb), (call, mismatch_report(gemb, wemb))
