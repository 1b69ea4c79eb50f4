"""The exact re-rank's fast path, restated on the CPU.

The kernels score a candidate row with Store.dotRow (src/store/store.ts:114-130)
by summing the exact f64 products in a warp-parallel order and accepting the
result only when the error bound B = 4 (K + 1) 2^-53 sum|x q| proves that the
reference's sequential f64 sum rounds to the same f32; otherwise they run the
sequence itself.  This test restates that order and check in numpy (IEEE f64,
round to nearest) and confirms, against the oracle's sequential dotRow, that
every accepted fast result is the reference's, on random rows and on rows built
to put the sum on an f32 rounding boundary (where the orders disagree).
"""
import numpy as np

from oracle import oracle as O


def fast_dot(x, q, nacc=4):
    """The warp orders of dot_row_exact_warp (nacc 4: four interleaved partial sums per lane) and
    dot_rows2_exact_warp (nacc 2): lane l takes i = l + 32t, then a butterfly."""
    dim = x.size
    p = x.astype(np.float64) * q.astype(np.float64)  # exact products
    lanes_s, lanes_a = [], []
    for lane in range(32):
        s = [0.0] * nacc
        a = [0.0] * nacc
        i = lane
        while i + 32 * (nacc - 1) < dim:
            for r in range(nacc):
                s[r] = s[r] + p[i + 32 * r]
                a[r] = a[r] + abs(p[i + 32 * r])
            i += 32 * nacc
        while i < dim:
            s[0] = s[0] + p[i]
            a[0] = a[0] + abs(p[i])
            i += 32
        if nacc == 4:
            lanes_s.append((s[0] + s[1]) + (s[2] + s[3]))
            lanes_a.append((a[0] + a[1]) + (a[2] + a[3]))
        else:
            lanes_s.append(s[0] + s[1])
            lanes_a.append(a[0] + a[1])
    off = 16
    while off:
        lanes_s = [lanes_s[l] + lanes_s[l ^ off] for l in range(32)]
        lanes_a = [lanes_a[l] + lanes_a[l ^ off] for l in range(32)]
        off >>= 1
    assert len(set(np.float64(v).tobytes() for v in lanes_s)) == 1  # every lane holds the same sum
    s, a = lanes_s[0], lanes_a[0]
    B = a * float(dim // 4 + 13) * 2.0 ** -51
    B = np.nextafter(B, np.inf)
    lo = np.float32(np.nextafter(s - B, -np.inf))
    hi = np.float32(np.nextafter(s + B, np.inf))
    if lo == lo and lo.view(np.uint32) == hi.view(np.uint32):
        return lo
    return None  # the kernel would run the reference's sequence


def test_fast_path_agrees_with_dot_row():
    rng = np.random.default_rng(0)
    accepted = 0
    for dim in (1, 3, 4, 7, 31, 32, 100, 127, 128, 129, 384, 768, 1000):
        for _ in range(40):
            x = rng.standard_normal(dim).astype(np.float32)
            q = rng.standard_normal(dim).astype(np.float32)
            want = np.float32(O.dot_row(x, q)).view(np.uint32)
            for nacc in (4, 2):
                got = fast_dot(x, q, nacc)
                if got is not None:
                    accepted += 1
                    assert got.view(np.uint32) == want
    assert accepted > 1000  # the fast path is the common case


def test_rounding_boundary_rows_fall_back():
    # exact sum just above the f32 midpoint 1 + 2^-24, but the reference's f64
    # sequence loses the small term and rounds the tie to even (1.0)
    q = np.array([1, 1, 1, 1, 0, 0, 0, 0], np.float32)
    for tiny in (2.0 ** -60, 2.0 ** -80, 2.0 ** -100):
        for pos in (2, 3):
            x = np.zeros(8, np.float32)
            x[0], x[1], x[pos] = 1.0, 2.0 ** -24, tiny
            ref = np.float32(O.dot_row(x, q))
            assert ref == np.float32(1.0)
            assert fast_dot(x, q, 4) is None and fast_dot(x, q, 2) is None  # the interval straddles the midpoint
