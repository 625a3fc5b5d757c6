"""The one-add rounding the row quantizers use for rows whose scaled values stay below 2^22 in magnitude.

For |t| < 2^22 the fp32 sum t + 1.5 * 2^23 lies in (2^23, 2^24), where the fp32 grid is the integers, so the one
rounded add rounds t to the nearest integer, ties to even, exactly as FCVTNS (and lrintf) do, and the sum's bits are
0x4B400000 + round(t). The kernels (emu.cuh quant_word_fast) rely on this identity and fall back to the conversion
instructions for any row whose bound max(|lo|, |hi|) * inv reaches 2^22. This checks the identity with IEEE fp32
arithmetic on the host: random values, exact ties, values next to the bound, and the bound's own edge.
"""
import numpy as np

MAGIC = np.float32(12582912.0)  # 1.5 * 2^23
BITS = 0x4B400000


def one_add_round(t):
    s = (t.astype(np.float32) + MAGIC).astype(np.float32)
    return (s.view(np.uint32).astype(np.int64) - BITS).astype(np.int64)


def test_one_add_rounding_matches_round_half_even():
    rng = np.random.default_rng(5)
    t = np.concatenate([
        rng.uniform(-4194303.0, 4194303.0, 200000),        # the whole admitted range
        rng.uniform(-300.0, 300.0, 200000),                # the range quantized rows actually use
        np.arange(-1000, 1000) + np.float32(0.5),          # exact ties
        np.arange(-1000, 1000) - np.float32(0.5),
        np.float32(4194303.5) - np.arange(64, dtype=np.float32) * np.float32(0.5),  # next to the bound
        -(np.float32(4194303.5) - np.arange(64, dtype=np.float32) * np.float32(0.5)),
        np.array([0.0, -0.0, 0.49999997, -0.49999997, 1.5, 2.5, -1.5, -2.5], np.float32),
    ]).astype(np.float32)
    assert np.all(np.abs(t) < 4194304.0)
    want = np.rint(t.astype(np.float64)).astype(np.int64)  # round half to even
    np.testing.assert_array_equal(one_add_round(t), want)


def test_bound_check_rejects_what_the_identity_does_not_cover():
    # the kernels' test: fmaxf(|lo|, |hi|) * inv < 2^22; a row whose bound reaches 2^22 (or is NaN / infinite) keeps
    # the conversion instructions. Past 2^22 the identity breaks: the sum passes 2^24, where the grid spacing is 2,
    # so an odd integer such as 2^22 + 1 comes back even.
    t = np.float32(4194305.0)
    assert one_add_round(np.array([t]))[0] != np.rint(np.float64(t))
    bound = np.float32(np.float32(3.0e6) * np.float32(1.5))  # 4.5e6 >= 2^22: rejected
    assert not bound < np.float32(4194304.0)
    with np.errstate(invalid="ignore"):
        assert not np.float32(np.nan) < np.float32(4194304.0)
        assert not np.float32(np.inf) * np.float32(0.0) < np.float32(4194304.0)
