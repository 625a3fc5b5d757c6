"""GPU parity at the benchmarked configurations: the packages the benchmark times, at the batch it times them, through
the calls it times (bnn_infer_batch with its default chunking and CUDA-graph replay, bnn_infer_device), bit for bit
against the CPU oracle.

Per-window semantics to reproduce: rt_run (src/rt_pkg.c:528-542) runs every op of the path on one window; a batch
must give each window exactly those bits, whatever chunk, tile schedule or grid shape it lands in.

* config 2: the full v2.4-architecture neon-int8 package, batch 256, all 256 windows (chunks of 64 + 192);
* config 3: the v2.4-architecture neon-fp16 package, batch 1024, 16 sampled windows (chunks of 256 + 768: the first
  and last window, both sides of the chunk boundary, a few more);
* config 4: the Perch-v2-architecture neon-fp16 + int8-head package, batch 512, 8 sampled windows (chunks 128 + 384);
* the largest int8 layers at batch 256 op by op (p0 over 1.57 M rows, b1.1 pw / dw / pwl), sampled windows.
"""
import os

import numpy as np
import pytest

from conftest import bits_equal, mismatch_report
from bnneon_b200 import Model, pkgread, synth
from oracle import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

CORES = os.cpu_count() or 1


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    torch.cuda.init()


def chunk_edges(n, batch):
    """The first window of every chunk bnn_infer_batch cuts a call of n windows into (next_chunk in bnn_api.c): a
    quarter of the batch first (rounded up to 8, from 64 windows on), then full batches."""
    edges, w, prev = [], 0, 0
    while w < n:
        rem = n - w
        first = min(rem, batch)
        s = batch if prev else ((first // 4 + 7) // 8 * 8 if first >= 64 else first)
        s = min(s, rem)
        if 0 < rem - s < s // 2 and rem <= batch:
            s = rem
        edges.append(w)
        w, prev = w + s, s
    return edges


def sample_windows(n, batch, extra, seed):
    edges = chunk_edges(n, batch)
    idx = {0, n - 1}
    for e in edges[1:]:
        idx.update((e - 1, e))
    rng = np.random.default_rng(seed)
    while len(idx) < extra:
        idx.add(int(rng.integers(0, n)))
    return np.array(sorted(idx))


def check(got, gemb, want, wemb, idx, what):
    for j, w in enumerate(idx):
        assert bits_equal(got[w], want[j]), f"{what}: window {w} logits: " + mismatch_report(got[w], want[j])
        if wemb is not None:
            assert bits_equal(gemb[w], wemb[j]), f"{what}: window {w} embedding: " + mismatch_report(gemb[w], wemb[j])


def run_config(pkg, mode, pcm, batch, idx, path_name):
    """bnn_infer_batch three times (eager, captured, replayed graphs) and bnn_infer_device once on the whole batch;
    every call's sampled windows against the oracle"""
    want, wemb = oracle.run_many(pkg, np.ascontiguousarray(pcm[idx]), threads=min(CORES, len(idx)),
                                 path_name=path_name)
    n = pcm.shape[0]
    with Model(pkg, mode=mode, batch=batch) as m:
        assert m.batch == batch
        for call in range(3):
            got, gemb = m.infer_batch(pcm)
            check(got, gemb, want, wemb, idx, f"bnn_infer_batch call {call}")
        d_pcm = torch.from_numpy(pcm).cuda()
        d_out = torch.full((n, m.info.n_classes), float("nan"), dtype=torch.float32, device="cuda")
        d_emb = torch.full((n, m.info.emb_dim), float("nan"), dtype=torch.float32, device="cuda")
        m.infer_device(n, d_pcm.data_ptr(), d_out.data_ptr(), d_emb.data_ptr())
        torch.cuda.synchronize()
        check(d_out.cpu().numpy(), d_emb.cpu().numpy(), want, wemb, idx, "bnn_infer_device")


def test_config2_int8_batch256_all_windows(cuda, full_pkg):
    """config 2 as timed (the benchmark's own audio seed for rank 0), every window of the batch"""
    B = 256
    pcm = synth.audio(B, seed=1000)
    assert chunk_edges(B, B) == [0, 64]
    run_config(full_pkg, 4, pcm, B, np.arange(B), synth.PATH)


def test_config3_fp16_batch1024_sampled(cuda, pkg_dir):
    B = 1024
    pkg = str(pkg_dir / "v24_full_f16.bnpk")
    if not os.path.exists(pkg):
        synth.make_package(pkg, seed=0, path=synth.PATH_F16)
    pcm = synth.audio(B, seed=4000)
    idx = sample_windows(B, B, 16, seed=3)
    assert {0, 255, 256, 1023} <= set(idx.tolist()) and len(idx) == 16
    run_config(pkg, 3, pcm, B, idx, synth.PATH_F16)


def test_config4_perch_batch512_sampled(cuda, pkg_dir):
    B = 512
    pkg = str(pkg_dir / "perch_v2_f16s8.bnpk")
    _, _, ns = synth.make_perch_package(pkg, seed=0)
    pcm = synth.audio(B, seed=4100, n_samples=ns, rate=synth.PERCH_SAMPLE_RATE)
    idx = sample_windows(B, B, 8, seed=4)
    assert {0, 127, 128, 511} <= set(idx.tolist()) and len(idx) == 8
    run_config(pkg, 3, pcm, B, idx, synth.PATH_F16)


def test_largest_int8_layers_at_batch256(cuda, full_pkg):
    """FE, C0POOL, p0 (6144 rows per window: 1.57 M rows at batch 256), b1.1 pw / dw / pwl run on the GPU at batch 256
    from the audio on (no oracle buffers injected), one after the other; every buffer they write is compared for
    sampled windows"""
    B = 256
    ops, _ = pkgread.read_ops(full_pkg)
    names = [pkgread.NAMES[c] for c, _, _, _ in ops[:6]]
    assert names == ["FE_STFT2", "C0POOL", "PW_S8", "PW_S8", "DW3", "PW_S8"], names
    pcm = synth.audio(B, seed=77)
    idx = [0, 1, 63, 64, 128, 200, 254, 255]
    states = []
    for w in idx:
        p = oracle.Package(full_pkg)
        p.run_range(pcm[w], 0, 6)
        states.append(p)

    def compare(m, i):
        code, bl, _, _ = ops[i]
        for b in pkgread.op_io(code, bl)[1]:
            elems, dt = states[0].buf_info(b)
            got = m.get_buffer(b, B, dt, elems)
            for j, w in enumerate(idx):
                want = states[j].get(b)
                assert bits_equal(got[w], want), (f"op {i} {names[i]} buffer {b} window {w}: "
                                                  + mismatch_report(got[w], want))

    # each op's outputs are read right after it runs: buffers whose lifetimes do not overlap share memory (the
    # package's slot plan), so a later op may overwrite them
    with Model(full_pkg, mode=4, batch=B) as m:
        m.run_ops(pcm, 0, 1)
        compare(m, 0)
        m.run_ops(pcm, 1, 2)  # C0POOL as the last op of a range writes its fp32 rows
        compare(m, 1)
        m.run_ops(pcm, 1, 3)  # as scored: C0POOL quantizes p0's rows itself (no fp32 rows that nothing else reads)
        compare(m, 2)
        for i in (3, 4, 5):
            m.run_ops(pcm, i, i + 1)
            compare(m, i)


def test_int8_pw_pairs_fused_quantizer(cuda, full_pkg, monkeypatch):
    """BNN_PW_FUSE=1: the pwl GEMMs quantize their stored rows for the expand layer after them (13 quantizer launches
    fewer per batch at batch 256); logits and embeddings stay bit-exact"""
    B = 256
    pcm = synth.audio(B, seed=1000)
    idx = sample_windows(B, B, 12, seed=5)
    want, wemb = oracle.run_many(full_pkg, np.ascontiguousarray(pcm[idx]), threads=min(CORES, len(idx)),
                                 path_name=synth.PATH)
    with Model(full_pkg, mode=4, batch=B) as m:
        base = m.launches_per_batch
    monkeypatch.setenv("BNN_PW_FUSE", "1")
    with Model(full_pkg, mode=4, batch=B) as m:
        assert m.launches_per_batch == base - 13, (base, m.launches_per_batch)
        for call in range(2):
            got, gemb = m.infer_batch(pcm)
            check(got, gemb, want, wemb, idx, f"fused quantizer, call {call}")
