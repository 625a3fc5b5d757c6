"""Config 1 of the benchmark: one int8 pointwise GEMM on given int8 rows, through bnn_pw_s8_gemm (the reference's
s8n_gemm_range on the rows s8n_quant_rows writes), against the CPU oracle bit for bit.

Inputs as the config states them: activations int8 [M = 4096][K = 256] seeded uniform in [-127, 127] with scale 0.05
and zero point 0; weights N(0, 0.02) [N = 512][K = 256] quantized per output channel by the package rule
(scale max|w| / 127); an int32 bias mapped to the reference's fp32 bias b = f32(bias * f32(sw * 0.05)); then the
harness's requantization to int8 (round half away from zero, clamp to +-127) of the fp32 outputs.
"""
import numpy as np
import pytest

from conftest import bits_equal, mismatch_report
from bnneon_b200 import load_library, synth
from oracle import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

M, K, N, SA, S_OUT = 4096, 256, 512, np.float32(0.05), np.float32(0.125)


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a visible CUDA device")
    h = load_library()
    torch.cuda.init()
    assert h.bnn_cuda_device_init() == 0, h.bnn_last_error()
    return h


def c1_inputs():
    a = np.random.default_rng(1).integers(-127, 128, (M, K)).astype(np.int8)
    w = np.random.default_rng(2).normal(0.0, 0.02, (N, K)).astype(np.float32)
    bias = np.random.default_rng(3).integers(-2 ** 15, 2 ** 15, N).astype(np.int32)
    lw = synth._Int8Lowering([])  # pylint: disable=protected-access
    tl, (n, k, kp, np_) = lw.s8("c1", w, np.zeros(N, np.float32))
    wq, sw, cs, _ = [lw.tensors[t][1] for t in tl]
    b = (bias.astype(np.float32) * (sw[:N] * SA).astype(np.float32)).astype(np.float32)  # f32(bias * f32(sw * sa))
    bb = np.zeros(np_, np.float32)
    bb[:N] = b
    q = np.zeros((M, kp), np.int8)
    q[:, :K] = a
    return q, wq, sw, cs, bb, (n, k, kp, np_)


def requant(y):
    """the harness extension: int8 = clamp(round_half_away(y / s_out), -127, 127)"""
    t = (y / S_OUT).astype(np.float32)
    r = np.sign(t) * np.floor(np.abs(t) + np.float32(0.5))
    return np.clip(r, -127, 127).astype(np.int8)


def test_c1_gemm_bit_exact(lib):
    q, wq, sw, cs, bb, (n, k, kp, np_) = c1_inputs()
    sa = np.full(M, SA, np.float32)
    za = np.zeros(M, np.int32)
    h = lib.bnn_pw_s8_new(n, k, kp, np_, wq.ctypes.data, sw.ctypes.data, cs.ctypes.data, bb.ctypes.data, M)
    assert h, lib.bnn_last_error()
    try:
        qd, sad, zad = (torch.from_numpy(v).cuda() for v in (q, sa, za))
        out = torch.zeros(M * np_, dtype=torch.float32, device="cuda")
        rc = lib.bnn_pw_s8_gemm(h, 1, M, qd.data_ptr(), kp, sad.data_ptr(), zad.data_ptr(), 0, out.data_ptr(), M * np_,
                                np_, 0, 0, None, 0, 0, 0, 0, None)
        assert rc == 0, lib.bnn_last_error()
        torch.cuda.synchronize()
        got = out.cpu().numpy().reshape(M, np_)
        assert lib.bnn_pw_s8_error(h) == 0
    finally:
        lib.bnn_pw_s8_free(h)
    want = np.zeros((M, np_), np.float32)
    oracle.lib().bnno_s8_gemm(oracle.ptr(q), oracle.ptr(sa), oracle.ptr(za), M, n, kp, np_, oracle.ptr(wq),
                              oracle.ptr(sw), oracle.ptr(cs), oracle.ptr(bb), 0, oracle.ptr(want), np_, 0, 0, None, 0,
                              0, 0)
    assert bits_equal(got, want), mismatch_report(got, want)
    assert np.array_equal(requant(got[:, :N]), requant(want[:, :N]))
    assert (requant(got[:, :N]) != 0).mean() > 0.5  # the requant scale exercises the int8 range
