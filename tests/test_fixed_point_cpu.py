"""The fixed-point scheme of the tcgen05 KIVI kernel (csrc/kivi_tc.cuh), restated in numpy.

The kernel folds scales into exact integer tensor-core operands. These properties hold for the
scheme itself; the GPU tests check the kernel against the oracle:

* balanced limbs: x + 0x808080 (three limbs) or x + 0x80808080 (four limbs) has bytes b_k
  with x = sum (b_k - 128) 256^k, so byte ^ 0x80 is the signed int8 limb;
* packed INT4 bytes: a byte is lo + 16 hi, so sum lo a + hi b = sum byte (b / 16) + lo (a - b / 16)
  when b is a multiple of 16; with v = round(x_odd / 16) the odd channels keep their precision
  when x has 26 bits;
* ranges: |x_even - v| and p'_even - v stay inside four balanced limbs, and the int32 limb
  sums of one chunk times the 256-chunk flush interval stay below 2^31.
"""
import numpy as np


def limbs(x, n):
    """Signed int8 limbs of int64 x (|x| inside the n-limb balanced range), as the kernel
    builds them: bytes of x + 0x80..80, each XOR 0x80."""
    bias = sum(0x80 << (8 * k) for k in range(n))
    u = (x.astype(np.int64) + bias).astype(np.uint64)
    out = []
    for k in range(n):
        b = ((u >> np.uint64(8 * k)) & np.uint64(0xFF)).astype(np.int64)
        out.append(((b ^ 0x80) + 128) % 256 - 128)   # the byte read as int8
    return np.stack(out)


def unlimb(ls):
    return sum(ls[k].astype(np.int64) * (256 ** k) for k in range(ls.shape[0]))


def test_balanced_limbs_round_trip():
    rng = np.random.default_rng(0)
    for n, lo, hi in ((3, -0x808080, 0x7F7F7F), (4, -0x80808080, 0x7F7F7F7F)):
        x = np.concatenate([rng.integers(lo, hi + 1, 100000), [lo, hi, 0, -1, 1]])
        ls = limbs(x, n)
        assert ls.min() >= -128 and ls.max() <= 127
        assert np.array_equal(unlimb(ls), x)


def test_packed_nibble_identity():
    rng = np.random.default_rng(1)
    for _ in range(200):
        lo = rng.integers(0, 16, 64)
        hi = rng.integers(0, 16, 64)
        byte = lo + 16 * hi
        a = rng.integers(-(1 << 26), 1 << 26, 64)
        v = rng.integers(-(1 << 22), 1 << 22, 64)
        b = 16 * v
        assert int((lo * a + hi * b).sum()) == int((byte * v + lo * (a - v)).sum())


def test_int4_key_quantisation_keeps_22_bits():
    """x = round(q' 2^ek), |x| < 2^26; the odd channels enter as 16 round(x / 16). The largest
    error per channel is 8 units of 2^-ek = 2^-22 of the largest |q'| -- the same as three-limb
    x with |x| < 2^22 rounded to an integer. Both operands fit four balanced limbs."""
    rng = np.random.default_rng(2)
    qs = rng.standard_normal((1000, 128)) * np.exp(rng.standard_normal((1000, 1)) * 3)
    qm = np.abs(qs).max(axis=1, keepdims=True)
    ek = 25 - np.floor(np.log2(qm)).astype(np.int64)
    scaled = qs * np.exp2(ek)
    assert np.abs(scaled).max() < 2 ** 26
    x = np.rint(scaled).astype(np.int64)
    x_even, x_odd = x[:, 0::2], scaled[:, 1::2]
    v = np.rint(x_odd / 16).astype(np.int64)
    err_odd = np.abs(16 * v - x_odd) / np.exp2(ek)
    assert (err_odd <= 8.0 * np.exp2(-ek) + 1e-12).all()
    assert (err_odd / qm <= 2.0 ** -22 + 1e-12).all()
    d = x_even - v
    for w in (v, d):
        assert np.abs(w).max() < 0x7F7F7F7F
        assert np.array_equal(unlimb(limbs(w.ravel(), 4)), w.ravel())


def test_int4_value_operands_and_accumulator_headroom():
    """p' < 2^30 (one bit more headroom than the 2^31 of unpacked values): v = round(p'_odd/16)
    and p'_even - v fit four balanced limbs, and 256 chunks of limb sums fit int32."""
    rng = np.random.default_rng(3)
    p = rng.uniform(0, 2 ** 30 - 1, (10000, 2))
    v = np.rint(p[:, 1] / 16).astype(np.int64)
    d = np.rint(p[:, 0]).astype(np.int64) - v
    assert d.min() > -0x80808080 and d.max() < 0x7F7F7F7F
    # per chunk and output column: 64 packed pair rows (bytes <= 255) and 64 low-nibble rows
    # (<= 15) against limbs of magnitude <= 128
    per_chunk = 64 * 255 * 128 + 64 * 15 * 128
    assert 256 * per_chunk < 2 ** 31
    # keys: one page slot, 64 packed bytes + 64 low nibbles against limbs <= 128
    assert 64 * 255 * 128 + 64 * 15 * 128 < 2 ** 31
