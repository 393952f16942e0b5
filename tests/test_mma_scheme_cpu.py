"""The arithmetic of the tensor-core decode of 4-bit group-scaled cells,
restated in numpy (no GPU): per 128-column group, the code bytes masked with
0x0F / 0xF0 times int8 pieces of y = x_even and z = x_odd / 16 under one
power-of-two exponent, summed exactly in integers, then
scale * (sum_n D_n 128^-n / S - 8 sum x).  Checks the identity against a
float64 dot product of (code - 8) * scale * x at a tight tolerance for x with
a wide range, the bound on the integer sums that the kernel's exact
int-to-float conversion needs (|D| < 2^21), and that a non-finite x gives a
NaN row.  The GPU kernel itself is checked against the oracle in
tests/test_gpu_kernels.py::test_gemv_flat_mma."""
import numpy as np

PIECES = 4


def split_group(x):
    """int8 pieces (4, 64) of y and z for one group of 128 columns, and 1 / S."""
    y = x[0::2].astype(np.float32)
    z = (x[1::2] * np.float32(0.0625)).astype(np.float32)
    m = float(max(np.abs(y).max(), np.abs(z).max()))
    if not np.isfinite(m):
        return np.zeros((PIECES, 64), np.int64), np.zeros((PIECES, 64), np.int64), float("nan")
    k = 0 if m == 0.0 else min(6 - int(np.frexp(m)[1]), 126)
    S = np.float32(2.0 ** k)
    out = []
    for v in (y, z):
        r = (v * S).astype(np.float32)
        p = []
        for _ in range(PIECES):
            i = np.rint(r)
            p.append(i.astype(np.int64))
            r = ((r - i) * np.float32(128)).astype(np.float32)
        out.append(np.stack(p))
    return out[0], out[1], float(2.0 ** -k)


def gemv_scheme(codes, scales, x):
    rows, cols = codes.shape
    lo = codes[:, 0::2].astype(np.int64)           # masked byte & 0x0F
    hi16 = 16 * codes[:, 1::2].astype(np.int64)    # masked byte & 0xF0
    out = np.zeros(rows, np.float64)
    dmax = 0
    for G in range(cols // 128):
        xs = x[G * 128:(G + 1) * 128]
        py, pz, invS = split_group(xs)
        b = slice(G * 64, (G + 1) * 64)
        D = lo[:, b] @ py.T + hi16[:, b] @ pz.T     # [rows][piece], exact integers
        dmax = max(dmax, int(np.abs(D).max()))
        v = sum(D[:, n].astype(np.float64) * 128.0 ** -n for n in range(PIECES))
        out += scales[:, G] * (v * invS - 8.0 * float(xs.astype(np.float64).sum()))
    return out, dmax


def test_scheme_matches_f64_dot_and_bounds_the_sums():
    rng = np.random.default_rng(7)
    rows, cols = 16, 1024
    codes = rng.integers(0, 16, (rows, cols))
    scales = rng.uniform(1e-3, 1e-2, (rows, cols // 128))
    for spike in (1.0, 1e4):
        x = rng.standard_normal(cols).astype(np.float32)
        x[rng.integers(0, cols, 3)] *= np.float32(spike)
        got, dmax = gemv_scheme(codes, scales, x)
        w = (codes - 8) * np.repeat(scales, 128, axis=1)
        ref = w @ x.astype(np.float64)
        assert dmax < 2 ** 21
        assert np.max(np.abs(got - ref)) <= 1e-6 * np.max(np.abs(ref)), spike


def test_non_finite_x_gives_nan_rows():
    rng = np.random.default_rng(8)
    codes = rng.integers(0, 16, (4, 256))
    scales = np.ones((4, 2))
    x = rng.standard_normal(256).astype(np.float32)
    x[200] = np.inf
    got, _ = gemv_scheme(codes, scales, x)
    assert np.all(np.isnan(got))
