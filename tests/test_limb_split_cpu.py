"""The staged histogram kernels form each row's limbs in float arithmetic
(tree.cu, LimbSplit): q = rint(v * s) with s a power of two, l1 = rint(q *
2^-L), l0 = q - l1 * 2^L in one fused multiply-add; the three-limb form
(LimbSplit3) first takes l2 = rint(q * 2^-2L) and splits the remainder the
same way. These checks restate that arithmetic in float32 and confirm the
facts the kernels' exactness and their normalisation intervals rest on, for
every limb width they use and values up to the widest each takes: every step
is exact, the limbs sum to q, |l0| (and |l1| with three limbs) <= 2^(L-1),
and the top limb <= 2^(bits - L) (two limbs) or 2^(bits - 2L) (three)."""
import numpy as np
import pytest


def _split(q32, L):
    inv = np.float32(2.0 ** -L)
    two = np.float32(2.0 ** L)
    scaled = (q32 * inv).astype(np.float32)
    hi = np.rint(scaled).astype(np.float32)
    # The fused multiply-add's exact value; it is representable (|l0| < 2^24),
    # so the single rounding of the FMA leaves it unchanged.
    l0 = q32.astype(np.float64) - hi.astype(np.float64) * float(two)
    return scaled, hi, l0


@pytest.mark.parametrize("L", [17, 18, 19, 20, 21])
def test_float_limb_split_is_exact_and_bounded(L):
    rng = np.random.default_rng(L)
    for bits in range(1, 2 * L + 1):
        mag = rng.integers(0, 1 << bits, 20000, dtype=np.int64)
        sign = rng.choice(np.array([-1, 1], dtype=np.int64), mag.size)
        # rint(v * s) of a float v and a power-of-two s: an integer-valued float.
        q32 = (mag * sign).astype(np.float32)
        scaled, hi, l0 = _split(q32, L)
        q = q32.astype(np.float64)
        assert np.array_equal(scaled.astype(np.float64), q * 2.0 ** -L)  # exact scaling
        assert np.all(np.abs(l0) <= 2.0 ** (L - 1))
        assert np.all(np.abs(l0) < 2.0 ** 24)
        assert np.all(np.abs(hi) <= max(1.0, 2.0 ** (bits - L)))
        assert np.array_equal(l0 + hi.astype(np.float64) * 2.0 ** L, q)


def test_ties_round_to_even_and_stay_in_bounds():
    L = 19
    half = 2 ** (L - 1)
    q32 = np.array([half, -half, 3 * half, -3 * half, 5 * half], dtype=np.float32)
    _, hi, l0 = _split(q32, L)
    assert np.all(np.abs(l0) <= half)
    assert np.array_equal(l0 + hi.astype(np.float64) * 2.0 ** L, q32.astype(np.float64))


def _split3(q32, L):
    """The three-limb split (tree.cu, LimbSplit3) in float32, each fused
    multiply-add taken at its exact value (representable, so the FMA's one
    rounding leaves it unchanged; checked below)."""
    top = np.rint((q32 * np.float32(2.0 ** (-2 * L))).astype(np.float32)).astype(np.float32)
    r = q32.astype(np.float64) - top.astype(np.float64) * 2.0 ** (2 * L)
    r32 = r.astype(np.float32)
    assert np.array_equal(r32.astype(np.float64), r)  # the first FMA is exact
    mid = np.rint((r32 * np.float32(2.0 ** -L)).astype(np.float32)).astype(np.float32)
    l0 = r - mid.astype(np.float64) * 2.0 ** L
    assert np.array_equal(l0.astype(np.float32).astype(np.float64), l0)  # and the second
    return l0, mid.astype(np.float64), top.astype(np.float64)


@pytest.mark.parametrize("L", [12, 15, 17, 21])
def test_float_three_limb_split_is_exact_and_bounded(L):
    rng = np.random.default_rng(100 + L)
    for bits in range(1, min(3 * L - 1, 63) + 1):
        mag = rng.integers(0, 1 << min(bits, 62), 20000, dtype=np.int64)
        if bits == 63:
            mag = mag * 2 + 1
        sign = rng.choice(np.array([-1, 1], dtype=np.int64), mag.size)
        q32 = (mag.astype(np.float64) * sign).astype(np.float32)  # a float q: <= 24 significant bits
        l0, l1, l2 = _split3(q32, L)
        assert np.all(np.abs(l0) <= 2.0 ** (L - 1)) and np.all(np.abs(l1) <= 2.0 ** (L - 1))
        assert np.all(np.abs(l2) <= max(1.0, 2.0 ** (bits - 2 * L)))
        total = l0 + l1 * 2.0 ** L + l2 * 2.0 ** (2 * L)  # exact in binary64 for these magnitudes
        exact = [int(a) + int(b) * 2 ** L + int(c) * 2 ** (2 * L) for a, b, c in zip(l0[:200], l1[:200], l2[:200])]
        assert exact == [int(v) for v in q32[:200].astype(np.float64)]
        assert np.array_equal(total, q32.astype(np.float64))


def test_three_limb_width_rule():
    """limb3_width: L = ceil((bits + 1) / 3), within [12, 21], so that every
    limb of a bits-wide value stays within 2^(L-1) below 63 bits."""
    for bits in range(0, 64):
        L = min(max((bits + 3) // 3, 12), 21)
        if bits < 63:
            assert bits - 2 * L <= L - 1
        # the normalisation interval covers a whole 12-warp CTA step (384 rows)
        per_row = max(L - 1, bits - 2 * L)
        assert ((2 ** 31 - 1 - 2 ** 26) >> per_row) >= 384
