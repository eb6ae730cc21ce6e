"""Exactness of the integer-in-float identities the staged tensor-core kernels rely on
(hearth_b200/csrc/hx_prefill_tc.cu): the accumulator starts at the bit pattern of 1.5 * 2^23, the
tensor cores add the nibble dot X of a Q4 block, and the drain recovers isum = X - 8 * sum(q) with one
f32 subtraction of cm = 12582912 + 8 * sum(q). Checked here in IEEE single precision (numpy float32),
exhaustively over X and sum(q)."""
import numpy as np

MAGIC = 0x4B400000
MAGIC_F = np.float32(12582912.0)
X_MAX = 64 * 15 * 127        # |sum(nib * q)| over one 64-weight block (nib 0..15, |q| <= 127)
S_MAX = 64 * 127             # |sum(q)| over one activation block


def test_magic_word_is_exact_for_every_block_dot():
    x = np.arange(-X_MAX, X_MAX + 1, dtype=np.int64)
    words = (MAGIC + x).astype(np.uint32)
    as_float = words.view(np.float32)
    # the word read back is 12582912 + X exactly: X changes only the low mantissa bits
    assert np.array_equal(as_float.astype(np.float64), 12582912.0 + x.astype(np.float64))
    assert np.all((words >> 23) == (MAGIC >> 23))


def test_cm_is_exact_for_every_activation_sum():
    s = np.arange(-S_MAX, S_MAX + 1, dtype=np.int64)
    cm = (12582912 + 8 * s).astype(np.float32)   # what __int2float_rn(kMagicI + 8 * sum) stores
    assert np.array_equal(cm.astype(np.int64), 12582912 + 8 * s)


def test_one_subtraction_gives_the_signed_block_dot():
    # every X against a grid of sums (and every sum against a grid of X), in float32 arithmetic
    x_all = np.arange(-X_MAX, X_MAX + 1, dtype=np.int64)
    s_all = np.arange(-S_MAX, S_MAX + 1, dtype=np.int64)
    for x, s in ((x_all, s_all[::127]), (x_all[::251], s_all)):
        X, S = np.meshgrid(x, s, indexing="ij")
        got = (MAGIC + X).astype(np.uint32).view(np.float32) - (12582912 + 8 * S).astype(np.float32)
        assert got.dtype == np.float32
        assert np.array_equal(got.astype(np.int64), X - 8 * S)


def test_extremes():
    for x in (-X_MAX, X_MAX, 0):
        for s in (-S_MAX, S_MAX, 0):
            w = np.array([MAGIC + x], dtype=np.int64).astype(np.uint32).view(np.float32)[0]
            cm = np.float32(12582912 + 8 * s)
            assert int(np.float32(w - cm)) == x - 8 * s
