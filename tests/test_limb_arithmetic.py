"""The integer formulation of the tensor-core GEMM / GEMV (umma.cuh), restated
in numpy and checked on its own terms (no GPU):

- an activation row is scaled by 2^s so that its largest magnitude lies in
  [2^21, 2^22) and rounded to an integer X with |X| <= 2^22;
- X is cut into balanced base-256 digits X = 65536 t + 256 m + l with
  m, l in [-128, 127] and |t| <= 64 (three signed 8-bit limbs);
- each limb times the signed levels q (|q| <= qmax <= 127) is summed in
  int32: exact up to K = 131072;
- the limb sums combine in int64, convert to fp32 once and take 2^-s.

The device kernels are checked against the oracle in the GPU tests; this file
pins the arithmetic those kernels rely on."""
import numpy as np

X_BITS = 22
MAX_K = 131072


def fixed(v, s):
    """rint(v * 2^s) clamped to +-2^22 (the device's ug_fixed for finite v)."""
    f = np.rint(np.ldexp(v.astype(np.float64), s))
    return np.clip(f, -(1 << X_BITS), 1 << X_BITS).astype(np.int64)


def digits(x):
    """Balanced base-256 digits (t, m, l) of x (the device's ug_digits)."""
    l = ((x & 0xFF) ^ 0x80) - 0x80
    x1 = (x - l) >> 8
    m = ((x1 & 0xFF) ^ 0x80) - 0x80
    t = (x1 - m) >> 8
    return t, m, l


def row_shift(row):
    amax = np.abs(row).max()
    return 0 if amax == 0 else (X_BITS - 1) - int(np.floor(np.log2(amax)))


def test_digits_rebuild_and_stay_in_range():
    rng = np.random.RandomState(0)
    x = np.concatenate([rng.randint(-(1 << X_BITS), (1 << X_BITS) + 1, size=200000),
                        [0, 1, -1, 127, 128, -128, -129, 255, 256, (1 << X_BITS), -(1 << X_BITS),
                         (1 << X_BITS) - 1, -(1 << X_BITS) + 1, 32767, -32768, 8355711, -8355712 // 2]])
    x = np.clip(x, -(1 << X_BITS), 1 << X_BITS).astype(np.int64)
    t, m, l = digits(x)
    np.testing.assert_array_equal(65536 * t + 256 * m + l, x)
    assert m.min() >= -128 and m.max() <= 127 and l.min() >= -128 and l.max() <= 127
    assert np.abs(t).max() <= 64


def test_int32_limb_sums_cannot_overflow_at_max_k():
    worst = MAX_K * 128 * 127          # |limb| <= 128, |q| <= 127
    assert worst < 2 ** 31 - 1
    assert 2 * worst > 2 ** 31 - 1     # twice the limit could overflow: the limit is near tight


def test_scaling_puts_the_row_maximum_in_range():
    rng = np.random.RandomState(1)
    for e in (-30, -5, 0, 7, 20):
        row = (rng.randn(4096) * 2.0 ** e).astype(np.float32)
        s = row_shift(row)
        top = np.abs(np.ldexp(row.astype(np.float64), s)).max()
        assert 2 ** 21 <= top < 2 ** 22


def test_product_error_within_the_stated_bound():
    """sum_k X q via three int32 limb sums equals the exact integer product;
    against float64 x . level the error per row is at most
    2^-22 * max|x| * sum_k |q| (each element's rounding is at most half an
    ulp of 2^-s), plus the final fp32 rounding."""
    rng = np.random.RandomState(2)
    K, N, qmax = 3000, 64, 127
    q = rng.randint(-qmax, qmax + 1, size=(K, N)).astype(np.int64)
    for e in (-12, 0, 9):
        x = (rng.randn(K) * 2.0 ** e * np.exp(rng.randn(K))).astype(np.float32)
        s = row_shift(x)
        X = fixed(x, s)
        t, m, l = digits(X)
        acc = [(limb[:, None] * q).sum(axis=0) for limb in (t, m, l)]
        for a in acc:
            assert np.abs(a).max() < 2 ** 31
        total = 65536 * acc[0] + 256 * acc[1] + acc[2]
        np.testing.assert_array_equal(total, (X[:, None] * q).sum(axis=0))
        y = np.ldexp(total.astype(np.float32).astype(np.float64), -s)
        ref = (x.astype(np.float64)[:, None] * q).sum(axis=0)
        bound = np.ldexp(0.5, -s) * np.abs(q).sum(axis=0) + np.abs(ref) * 2.0 ** -23 + 1e-300
        assert np.all(np.abs(y - ref) <= bound * 1.0001), np.abs(y - ref).max()


def _byte_perm(x, y, sel):
    """PTX prmt (default mode) on uint32 arrays: byte i of the result is
    byte (sel >> 4i) & 7 of the 8-byte value y:x."""
    out = np.zeros_like(x)
    for i in range(4):
        b = (sel >> (4 * i)) & 7
        src = x if b < 4 else y
        out |= ((src >> np.uint32(8 * (b & 3))) & np.uint32(0xFF)) << np.uint32(8 * i)
    return out


def test_byte_permute_digits_equal_balanced_digits():
    """The decode matvec (qmvi.cuh) builds the limb words of four k at once:
    with Y = X + 0x8080 the balanced digits are byte 0 of Y - 128, byte 1 of
    Y - 128 and Y >> 16, so the low / mid / top words are byte permutes of
    the four Y (the first two with every byte's top bit flipped). Checked
    against the digit arithmetic over random X and the range's edges."""
    rng = np.random.RandomState(3)
    edges = np.array([-(1 << 22), 1 << 22, 0, -1, 1, 127, 128, -128, -129, 255, 256, 32767, 32768, -32768,
                      -32769, (1 << 22) - 1, -(1 << 22) + 1], np.int64)
    xs = np.concatenate([rng.randint(-(1 << 22), (1 << 22) + 1, size=40000), np.tile(edges, 4)])
    xs = xs[: len(xs) // 4 * 4].reshape(-1, 4)
    Y = ((xs + 0x8080) & 0xFFFFFFFF).astype(np.uint32)
    pair = lambda sel: _byte_perm(_byte_perm(Y[:, 0], Y[:, 1], sel), _byte_perm(Y[:, 2], Y[:, 3], sel), 0x5410)
    l4 = pair(0x0040) ^ np.uint32(0x80808080)
    m4 = pair(0x0051) ^ np.uint32(0x80808080)
    t4 = pair(0x0062)
    t, m, l = digits(xs)
    pack = lambda d: sum(((d[:, b] & 0xFF).astype(np.uint32) << np.uint32(8 * b)) for b in range(4)).astype(np.uint32)
    np.testing.assert_array_equal(l4, pack(l))
    np.testing.assert_array_equal(m4, pack(m))
    np.testing.assert_array_equal(t4, pack(t))
