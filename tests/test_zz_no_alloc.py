"""bnn_pw_s8_run_static: the PW_S8 entry point that allocates nothing (its quantized activations live in a static
device array) gives the same bits as bnn_pw_s8_run, call after call, through the C ABI.

Collected last so that it also runs after every other GPU test in one process; it passes alone too.
"""
import numpy as np
import pytest

from bnneon_b200 import load_library, synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

MAX_ROWS = 32768          # BNN_PW_S8_STATIC_MAX_ROWS
MAX_QBYTES = 4 << 20      # BNN_PW_S8_STATIC_MAX_QBYTES
BNN_ERR_USAGE = 6


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    h = load_library()
    torch.cuda.init()
    assert h.bnn_cuda_device_init() == 0, h.bnn_last_error()
    return h


def make_op(lib, rng, N, K, rows_cap):
    w = (rng.standard_normal((N, K)) * 0.3).astype(np.float32)
    lw = synth._Int8Lowering([])  # pylint: disable=protected-access
    tl, (n, k, kp, np_) = lw.s8("t", w, (rng.standard_normal(N) * 0.1).astype(np.float32))
    wq, sw, cs, bb = [lw.tensors[t][1] for t in tl]
    h = lib.bnn_pw_s8_new(n, k, kp, np_, wq.ctypes.data, sw.ctypes.data, cs.ctypes.data, bb.ctypes.data, rows_cap)
    assert h, lib.bnn_last_error()
    return h, np_


class Call:
    """one PW_S8 invocation's device buffers: (N, K, Mw, B, act, residual, padded output width, gated)"""

    def __init__(self, lib, seed, N, K, Mw, B, act, use_res, ow, gated):
        rng = np.random.default_rng(seed)
        self.h, np_ = make_op(lib, rng, N, K, B * Mw)
        self.B, self.Mw, self.K, self.act, self.ow = B, Mw, K, act, ow
        self.lda = (K + 7) // 8 * 8
        self.ldo = np_
        oh = Mw // ow if ow else 0
        self.oelems = ((oh + 2) * (ow + 2) if ow else Mw) * self.ldo
        self.x = torch.from_numpy((rng.standard_normal((B, Mw, self.lda)) * 0.7).astype(np.float32)).cuda()
        self.gate = (torch.from_numpy(rng.uniform(0, 1, (B, K)).astype(np.float32)).cuda() if gated else None)
        self.res = (torch.from_numpy((rng.standard_normal((B, Mw, self.ldo)) * 0.5).astype(np.float32)).cuda()
                    if use_res else None)

    def run(self, fn, out, B=None):
        return fn(self.h, self.B if B is None else B, self.Mw, self.x.data_ptr(), self.Mw * self.lda, self.lda,
                  None if self.gate is None else self.gate.data_ptr(), self.K, self.act, out.data_ptr(), self.oelems,
                  self.ldo, self.ow, 1 if self.ow else 0, None if self.res is None else self.res.data_ptr(),
                  self.Mw * self.ldo, self.ldo, 0, 0, None)

    def out(self):
        return torch.zeros(self.B * self.oelems, dtype=torch.float32, device="cuda")


CALLS = [  # two layers of the v2.4 int8 path, run back to back on the shared static array
    (72, 288, 384, 3, 0, True, 0, True),     # b2.2 pwl: SE gate + residual
    (72, 24, 6144, 2, 1, False, 128, False),  # b1.1 pw: SiLU, haloed output, 12288 rows
    # both limits reached exactly: 4 x 8192 = 32768 rows of Kq = 128 bytes = 4 MiB of quantized rows, so the q
    # region's tensor map is used to its last row and the sa / za regions to their last entry
    (36, 128, 8192, 4, 1, True, 0, False),
]


def test_static_matches_run_on_consecutive_calls(lib):
    assert lib.bnn_pw_s8_run_static(None, 0, 1, None, 0, 1, None, 0, 0, None, 0, 1, 0, 0, None, 0, 0, 0, 0,
                                    None) == -1  # no op: usage error, nothing launched
    calls = [Call(lib, 11 + i, *c) for i, c in enumerate(CALLS)]
    try:
        for c in calls:  # B = 0: the per-device set-up only
            assert c.run(lib.bnn_pw_s8_run_static, c.out(), B=0) == 0, lib.bnn_last_error()
        want = []
        for c in calls:
            o = c.out()
            assert c.run(lib.bnn_pw_s8_run, o) == 0, lib.bnn_last_error()
            want.append(o)
        torch.cuda.synchronize()
        for rep in range(2):  # two rounds of both layers in a row: the second call of each reuses the array
            got = []
            for c in calls:
                o = c.out()
                assert c.run(lib.bnn_pw_s8_run_static, o) == 0, lib.bnn_last_error()
                got.append(o)
            torch.cuda.synchronize()
            for i, (g, w) in enumerate(zip(got, want)):
                gi, wi = g.view(torch.int32).cpu(), w.view(torch.int32).cpu()
                bad = int((gi != wi).sum())
                assert bad == 0, f"round {rep} call {i}: {bad} of {gi.numel()} outputs differ from bnn_pw_s8_run"
        for c in calls:
            assert lib.bnn_pw_s8_error(c.h) == 0
    finally:
        for c in calls:
            lib.bnn_pw_s8_free(c.h)


def test_static_allocates_nothing(lib):
    c = Call(lib, 5, *CALLS[1])
    try:
        o = c.out()
        assert c.run(lib.bnn_pw_s8_run_static, o) == 0, lib.bnn_last_error()  # set-up and first launches
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        for _ in range(3):
            assert c.run(lib.bnn_pw_s8_run_static, o) == 0, lib.bnn_last_error()
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0
    finally:
        lib.bnn_pw_s8_free(c.h)


def test_static_rejects_sizes_beyond_the_array(lib):
    rng = np.random.default_rng(3)
    h, np_ = make_op(lib, rng, 16, 256, 64)
    try:
        # rows over the row limit, then rows within it whose quantized bytes (rows x 256) are over the byte limit
        for B, Mw in ((MAX_ROWS + 1, 1), (1, MAX_QBYTES // 256 + 1)):
            rc = lib.bnn_pw_s8_run_static(h, B, Mw, None, 0, 256, None, 0, 0, None, 0, np_, 0, 0, None, 0, 0, 0, 0,
                                          None)
            assert rc == -1
            assert lib.bnn_last_error_kind() == BNN_ERR_USAGE
            assert b"exceed the static scratch" in lib.bnn_last_error()
    finally:
        lib.bnn_pw_s8_free(h)
