"""GPU parity of the int8 prototype head (PROTO_S8) against the CPU oracle, bit for bit, through the C ABI: the per-op
entry point (include/bnneon_cuda.h bnn_proto_s8_*) on edge shapes and values, one-op packages written as the
reference compiler writes them (tests/golden/proto_packages.json) through bnn_infer_batch, the Perch v2 head shape
(64 cells x 1536 channels -> 59180 prototypes) on sampled windows of a larger batch, and PROTO variant 2 (fp16 cells,
SDOT-packed prototypes, bnn_proto_s8h_*)."""
import ctypes

import numpy as np
import pytest

from conftest import bits_equal, mismatch_report
from bnneon_b200 import BnnError, Model, load_library, synth
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


def p(a):
    return a.ctypes.data


class ProtoOp:
    """bnn_proto_s8_new on a packed head; run() returns (qa, sx, colmax, logits, status) of B windows."""

    def __init__(self, h, head, P, C, cap):
        self.h = h
        self.qp, self.sw, self.n4, self.rows = synth.pack_proto_s8(head["P"])
        self.cw = np.ascontiguousarray(head["cw"], np.float32)
        self.cb = np.ascontiguousarray(head["cb"], np.float32)
        self.nc, self.ppc = self.cw.shape
        self.Np, self.Kp = self.rows.shape
        self.P, self.C, self.eps = P, C, np.float32(head["eps"])
        self.op = h.bnn_proto_s8_new(self.nc * self.ppc, C, self.Kp, self.Np, p(self.qp), p(self.sw), p(self.n4),
                                     p(self.cw), p(self.cb), self.nc, self.ppc, float(self.eps), P, cap)
        assert self.op, h.bnn_last_error()

    def run(self, x, colmax_stride=None):
        B, P, ld = x.shape
        cws = colmax_stride or self.Np
        d_x = dev(x)
        d_lg = torch.full((B, self.nc + 3), 7.0, dtype=torch.float32, device="cuda")
        d_cm = torch.full((B, cws), 7.0, dtype=torch.float32, device="cuda")
        d_st = torch.full((B,), 7, dtype=torch.int32, device="cuda")
        rc = self.h.bnn_proto_s8_run(self.op, B, d_x.data_ptr(), P * ld, ld, d_lg.data_ptr(), self.nc + 3,
                                     d_cm.data_ptr(), cws, d_st.data_ptr(), None)
        assert rc == 0, self.h.bnn_last_error()
        torch.cuda.synchronize()
        qa = np.zeros((B, P, self.Kp), np.int8)
        sx = np.zeros((B, P), np.float32)
        assert self.h.bnn_proto_s8_read_scratch(self.op, B, p(qa), p(sx)) == 0
        assert self.h.bnn_proto_s8_error(self.op) == 0
        lg = host(d_lg)
        assert (lg[:, self.nc:] == 7.0).all()  # nothing past nc written
        return qa, sx, host(d_cm)[:, :self.Np], lg[:, :self.nc], host(d_st)

    def close(self):
        self.h.bnn_proto_s8_free(self.op)


def check(got, want, what):
    qa, sx, cm, lg, st = got
    wqa, wsx, wcm, wlg, wst = want
    assert np.array_equal(qa, wqa), f"{what}: quantized cells differ ({int((qa != wqa).sum())} bytes)"
    assert bits_equal(sx, wsx), f"{what}: cell scales: {mismatch_report(sx, wsx)}"
    assert bits_equal(cm, wcm), f"{what}: column maxima: {mismatch_report(cm, wcm)}"
    assert bits_equal(lg, wlg), f"{what}: logits: {mismatch_report(lg, wlg)}"
    assert np.array_equal(st, wst), f"{what}: status {st} vs {wst}"


# (B, P, C, ld, classes, prototypes per class, eps, what it covers)
CASES = [
    (3, 8, 40, 40, 10, 3, 1e-6, "Kp 48: one ragged K block; Np 32 > N 30"),
    (5, 12, 64, 72, 25, 4, 1e-3, "P % 8 == 4: 4-column TMEM loads; ld > C"),
    (2, 300, 96, 96, 9, 2, 1e-6, "P > 256: windows split in chunks"),
    (9, 64, 256, 256, 130, 4, 1e-6, "4 windows per cell tile, a partial last tile; 5 prototype tiles"),
    (4, 4, 8, 8, 7, 1, 1e-6, "K 8 -> Kp 16, P 4, one prototype per class"),
    (70, 4, 136, 140, 33, 3, 1e-6, "64 windows per cell tile, 2 cell tiles; Kp 144"),
    (3, 520, 48, 48, 5, 4, 0.0, "P > 512: 3 chunks per window; eps 0"),
    (2, 16, 1544, 1544, 40, 4, 1e-6, "K 1544: 13 K blocks, the last ragged"),
]


@pytest.mark.parametrize("case", CASES, ids=[c[-1].split(":")[0] for c in CASES])
def test_proto_op(lib, case):
    B, P, C, ld, nc, ppc, eps, what = case
    head = synth.proto_head(len(what), P, C, nc, ppc, eps)
    x = synth.cells(B, P, ld, seed=B * 1000 + P)
    op = ProtoOp(lib, head, P, C, B)
    try:
        got = op.run(x)
    finally:
        op.close()
    want = oracle.proto_s8(x, op.rows, op.sw, op.cw, op.cb, op.eps, C, op.Kp)
    check(got, want, what)


def test_proto_edge_values(lib):
    """Zero cells, tiny and huge magnitudes, ties, NaN and infinity (the reference's vcvtaq / vqmovn / max -127 rules,
    the 1e-30 floor, NaN propagation through the maxima), and windows whose logits fail the finite check."""
    B, P, C, ld, nc, ppc = 6, 16, 64, 64, 12, 3
    head = synth.proto_head(99, P, C, nc, ppc, 1e-6)
    x = synth.cells(B, P, ld, seed=7)
    x[0, 0] = 0.0                                   # an all-zero cell
    x[0, 1, :] = 0.0
    x[0, 1, 3] = 1e-38                              # a denormal-sized maximum
    x[0, 2, :4] = [127.0, 2.5, -2.5, 0.5]           # exact ties after scaling
    x[1, 5, 9] = np.nan                             # NaN: max 1e-30, scale NaN -> this window's maxima NaN
    x[2, 3, 0] = np.inf                             # infinity: the sum of squares overflows
    x[3] *= 1e19                                    # squares overflow in the sum
    x[4, :, :] = -3.0                               # every value equal and negative
    x[5, 7] = 1e-30
    op = ProtoOp(lib, head, P, C, B)
    try:
        got = op.run(x)
    finally:
        op.close()
    want = oracle.proto_s8(x, op.rows, op.sw, op.cw, op.cb, op.eps, C, op.Kp)
    check(got, want, "edge values")
    assert (want[4] != 0).any(), "no window failed the finite check: the case does not test the status"


def test_colmax_window_stride(lib):
    """colmax at a window stride wider than Np (the runtime's buffer slots), logits likewise."""
    B, P, C, nc, ppc = 5, 8, 32, 20, 4
    head = synth.proto_head(3, P, C, nc, ppc, 1e-6)
    x = synth.cells(B, P, C, seed=3)
    op = ProtoOp(lib, head, P, C, 8)
    try:
        got = op.run(x, colmax_stride=op.Np + 40)
    finally:
        op.close()
    check(got, oracle.proto_s8(x, op.rows, op.sw, op.cw, op.cb, op.eps, C, op.Kp), "strided colmax")


@pytest.mark.parametrize("name", ["proto_small", "proto_ld", "proto_wide", "proto_mid"])
def test_proto_package(lib, name, tmp_path):
    """One-op packages as the reference compiler writes them, through bnn_infer_batch, against the oracle's package
    executor; batches split into chunks and windows of the call numbered across them."""
    import json  # pylint: disable=import-outside-toplevel
    import os  # pylint: disable=import-outside-toplevel
    with open(os.path.join(os.path.dirname(__file__), "golden", "proto_packages.json"), encoding="utf-8") as f:
        g = json.load(f)[name]
    head = synth.proto_head(g["seed"], g["cells"], g["channels"], g["classes"], g["ppc"], g["eps"])
    path = str(tmp_path / f"{name}.bnpk")
    synth.write_proto_package(path, head, g["ld"])
    n = 11
    x = synth.cells(n, g["cells"], g["ld"], seed=42).reshape(n, -1)
    with Model(path, mode=4, batch=4) as m:
        out, _ = m.infer_batch(x)
        assert m.launches_per_batch == 3 + (g["cells"] > 256)
    want, _ = oracle.run_many(path, x, threads=4)
    assert bits_equal(out, want), mismatch_report(out, want)


def test_failed_window_is_reported(lib, tmp_path):
    """A window whose logits are not finite fails the call as bnn_infer does (code -2, kind WINDOW), naming the first
    failed window of the call; the other windows are still scored."""
    g = dict(seed=5, cells=8, channels=40, classes=10, ppc=3, ld=40, eps=1e-6)
    head = synth.proto_head(g["seed"], g["cells"], g["channels"], g["classes"], g["ppc"], g["eps"])
    path = str(tmp_path / "fail.bnpk")
    synth.write_proto_package(path, head, g["ld"])
    n = 9
    x = synth.cells(n, g["cells"], g["ld"], seed=8)
    x[6, 2, :] = np.nan  # a NaN cell: its window's maxima and logits are NaN
    x[7, 1, 0] = np.nan
    xr = x.reshape(n, -1)
    h = load_library()
    with Model(path, mode=4, batch=4) as m:
        out = np.zeros((n, g["classes"]), np.float32)
        rc = h.bnn_infer_batch(m.ctx, n, p(xr), p(out), None)
        assert rc == -2
        msg = h.bnn_last_error().decode()
        assert h.bnn_last_error_kind() == 4 and "window 6 of the call" in msg and "op 0 proto_s8n" in msg, msg
        ok, _ = m.infer_batch(xr[:6])  # the failure does not stick to the next call
    want = np.stack([oracle.proto_s8(x[i:i + 1], *proto_args(head, g))[3][0] for i in range(6)])
    assert bits_equal(out[:6], want) and bits_equal(ok, want)
    with pytest.raises(BnnError):
        Model(path, mode=4, batch=4).infer(xr[7])


def proto_args(head, g):
    qp, sw, _, rows = synth.pack_proto_s8(head["P"])
    del qp
    return rows, sw, head["cw"], head["cb"], np.float32(head["eps"]), g["channels"], rows.shape[1]


class ProtoOpH(ProtoOp):
    """bnn_proto_s8h_new on the SDOT-packed head (PROTO variant 2); run() takes fp16 cells."""

    def __init__(self, h, head, P, C, cap):  # pylint: disable=super-init-not-called
        self.h = h
        self.qp, self.sw, self.rows = synth.pack_proto_s8_sdot(head["P"])
        self.cw = np.ascontiguousarray(head["cw"], np.float32)
        self.cb = np.ascontiguousarray(head["cb"], np.float32)
        self.nc, self.ppc = self.cw.shape
        self.Np, self.K = self.rows.shape
        self.Kq = (self.K + 15) // 16 * 16
        self.P, self.C, self.eps = P, C, np.float32(head["eps"])
        self.op = h.bnn_proto_s8h_new(self.nc * self.ppc, C, self.Np, p(self.qp), p(self.sw), p(self.cw), p(self.cb),
                                      self.nc, self.ppc, float(self.eps), P, cap)
        assert self.op, h.bnn_last_error()

    def run(self, x, colmax_stride=None):
        B, P, ld = x.shape
        d_x = dev(np.ascontiguousarray(x, np.float16).view(np.uint16))
        d_lg = torch.full((B, self.nc), 7.0, dtype=torch.float32, device="cuda")
        d_cm = torch.full((B, self.Np), 7.0, dtype=torch.float32, device="cuda")
        d_st = torch.full((B,), 7, dtype=torch.int32, device="cuda")
        rc = self.h.bnn_proto_s8h_run(self.op, B, d_x.data_ptr(), P * ld, ld, d_lg.data_ptr(), self.nc,
                                      d_cm.data_ptr(), self.Np, d_st.data_ptr(), None)
        assert rc == 0, self.h.bnn_last_error()
        torch.cuda.synchronize()
        qa = np.zeros((B, P, self.Kq), np.int8)
        sx = np.zeros((B, P), np.float32)
        assert self.h.bnn_proto_s8_read_scratch(self.op, B, p(qa), p(sx)) == 0
        assert self.h.bnn_proto_s8_error(self.op) == 0
        assert (qa[:, :, self.K:] == 0).all()
        return qa[:, :, :self.K], sx, host(d_cm), host(d_lg), host(d_st)


# (B, P, C, ld, classes, prototypes per class, what it covers) for PROTO variant 2
CASES_H = [
    (3, 8, 40, 40, 10, 3, "K 40 (rows padded to 48), Np 36 > N 30"),
    (4, 16, 64, 72, 25, 4, "ld > C"),
    (2, 264, 96, 96, 9, 2, "P > 256: chunked windows"),
    (9, 64, 256, 256, 130, 4, "Np 528, 4 windows per cell tile"),
]


@pytest.mark.parametrize("case", CASES_H, ids=[c[-1].split(":")[0] for c in CASES_H])
def test_proto_variant2(lib, case):
    B, P, C, ld, nc, ppc, what = case
    head = synth.proto_head(len(what) + 100, P, C, nc, ppc, 1e-6)
    x = synth.cells(B, P, ld, seed=B * 7 + P).astype(np.float16)
    x[0, 1, 3] = np.float16(-np.inf)  # a cell with -inf: its bytes saturate to -128 (no -127 clamp here)
    x[0, 2, :] = 0                     # a zero cell
    op = ProtoOpH(lib, head, P, C, B)
    try:
        got = op.run(x)
    finally:
        op.close()
    want = oracle.proto_s8h(x, op.rows, op.sw, op.cw, op.cb, op.eps, C)
    check(got, want, what)
    assert got[0][0, 1].min() == -128 or got[0][0, 1].min() == 0  # -inf: -128 unless the cell's scale is infinite


def test_perch_head_shape(lib):
    """The Perch v2 head (results/perch_graph_compact.txt: 64 cells x 1536 channels, 14795 classes x 4 prototypes)
    over 130 windows (33 cell tiles, the last one partial), sampled windows against the oracle."""
    B, P, C, nc, ppc = 130, 64, 1536, 14795, 4
    head = synth.proto_head(2024, P, C, nc, ppc, 1e-6)
    x = synth.cells(B, P, C, seed=11)
    op = ProtoOp(lib, head, P, C, B)
    try:
        qa, sx, cm, lg, st = op.run(x)
    finally:
        op.close()
    sample = [0, 3, 64, 127, 129]
    want = oracle.proto_s8(x[sample], op.rows, op.sw, op.cw, op.cb, op.eps, C, op.Kp)
    check((qa[sample], sx[sample], cm[sample], lg[sample], st[sample]), want, "Perch head")
    assert (st == 0).all()
