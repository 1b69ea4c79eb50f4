"""normalizeInPlace (src/store/store.ts:209-217) on the host: the product's
vectorised normalize_rows against the oracle's sequential restatement, bit for
bit, including zero rows, tiny and huge magnitudes and odd dimensions."""
import numpy as np

from browservec_b200.index import normalize_rows
from oracle import oracle as O


def test_normalize_rows_matches_oracle():
    rng = np.random.default_rng(0)
    for d in (1, 3, 4, 17, 96, 384, 768, 1000):
        m = rng.standard_normal((50, d)).astype(np.float32)
        m[0] = 0.0
        m[1] *= np.float32(1e-20)
        m[2] *= np.float32(1e18)
        m[3, :] = np.float32(3.0)
        want = O.normalize_rows(m)
        got = normalize_rows(m)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), d
