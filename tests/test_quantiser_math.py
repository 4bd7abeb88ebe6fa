"""The arithmetic behind the fused kernel's activation quantisation (CPU).

The kernel turns x * (32767 / amax) into int16 values X without a float-to-int
conversion: adding 1.5 * 2^23 rounds the product into the low mantissa bits,
so the sum's bits are 0x4B400000 + X and its two low bytes are X's.  This
checks that identity, in float32 with round-to-nearest-even like the GPU,
against the conversion it replaces (round, clamp to +-32767, NaN -> 0), and
that the group sums follow from sums of the bits.
"""
import numpy as np

MAGIC = np.float32(12582912.0)  # 1.5 * 2^23
BIAS = 0x4B400000


def _groups(rng, n):
    g = rng.standard_normal((n, 32)).astype(np.float32)
    g[0::7] *= np.float32(1e-30)
    g[1::7] *= np.float32(1e30)
    g[2::7] = (rng.integers(-5, 5, (len(g[2::7]), 32)) * 0.5).astype(np.float32)  # ties
    g[3::7, 5] = np.nan
    g[4::7] = 0.0
    g[5::7, :] = np.float32(-2.5)
    return g


def test_magic_rounding_matches_convert_and_clamp():
    rng = np.random.default_rng(0)
    g = _groups(rng, 7000)
    with np.errstate(all="ignore"):
        amax = np.nanmax(np.abs(g), axis=1)
        amax = np.where(np.isnan(amax), np.float32(0), amax).astype(np.float32)
        inv = np.where(amax > 0, np.float32(32767.0) / amax, np.float32(0)).astype(np.float32)
        keep = inv < np.float32(3.0e38)  # the kernel falls back to the conversion otherwise
        y = (g * inv[:, None]).astype(np.float32)
        # the replaced conversion: round half to even, NaN -> 0, clamp
        ref = np.where(np.isnan(y), 0, np.rint(y))
        ref = np.clip(ref, -32767, 32767).astype(np.int64)
        # the kernel's form
        y0 = np.where(np.isnan(y), np.float32(0), y).astype(np.float32)
        bits = (y0 + MAGIC).astype(np.float32).view(np.uint32).astype(np.int64)
    assert keep.sum() == len(g)
    assert np.array_equal(bits & 0xFF, ref & 0xFF)  # low byte
    assert np.array_equal((bits >> 8) & 0xFF, (ref >> 8) & 0xFF)  # high byte
    assert np.array_equal(bits - BIAS, ref)  # the whole value
    # the clamp never fires: |x| <= amax keeps rn(x * 32767 / amax) inside +-32767
    assert np.all(np.abs(ref) <= 32767)
    # group half sums from the bits (32-bit wrap-around, as on the GPU)
    for lo, hi in ((0, 16), (16, 32)):
        s_bits = (bits[:, lo:hi].sum(axis=1) - 16 * BIAS) & 0xFFFFFFFF
        s_bits = np.where(s_bits >= 2**31, s_bits - 2**32, s_bits)
        assert np.array_equal(s_bits, ref[:, lo:hi].sum(axis=1))


def test_tiny_groups_overflow_the_scale():
    # amax below ~1e-34 makes 32767 / amax overflow: those groups take the
    # conversion-and-clamp path in the kernel
    with np.errstate(over="ignore"):
        inv = np.float32(32767.0) / np.float32(1e-38)
    assert not inv < np.float32(3.0e38)
