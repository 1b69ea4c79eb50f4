"""IVF x quant candidate-list scan (src/index/ivfquant.ts:468-490) against the
oracle: each query is scored over only its candidate rows (any order, lists of
0 .. 15,000 rows), the best F by (score desc, earlier candidate), exact re-rank,
best k -- candidates, quantized scores, rows and exact scores bit-exact, for
every width and scoring, with F on both sides of the one-launch finish."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _rows(n, d, seed):
    rng = np.random.default_rng(seed)
    return O.normalize_rows(rng.standard_normal((n, d)).astype(np.float32))


@pytest.mark.parametrize("bits,scoring,mode,d,fetch", [
    (8, "asym", O.MODE_ASYM, 384, 40), (8, "int", O.MODE_INT, 96, 40), (4, "asym", O.MODE_ASYM, 384, 300),
    (4, "int", O.MODE_INT, 128, 80), (1, "hamming", O.MODE_HAMMING, 768, 320), (1, "asym", O.MODE_ASYM, 256, 40)])
def test_candidate_scan_matches_oracle(bits, scoring, mode, d, fetch):
    from browservec_b200.index import AddonQuantIndex

    n, k = 20000, 10
    x = _rows(n, d, bits + d)
    rng = np.random.default_rng(5)
    sizes = [0, 7, 1000, 5000, 15000, 3]
    lists = [rng.permutation(n)[:m].astype(np.uint32) for m in sizes]
    qs = _rows(len(sizes), d, 99)
    idx = AddonQuantIndex(d, bits=bits, scoring=scoring)
    try:
        idx.append(x, n)
        corpus = O.Corpus(x, d, bits)
        rows, scores, counts, crows, cscores, ccounts = idx.search_candidates(qs, lists, k, fetch,
                                                                              with_candidates=True)
        for i, lst in enumerate(lists):
            wr, ws, wcr, wcs = corpus.query_candidates(qs[i], lst, k, fetch, mode)
            assert int(ccounts[i]) == wcr.size, i
            assert np.array_equal(crows[i, :wcr.size], wcr), i
            assert np.array_equal(cscores[i, :wcr.size].view(np.uint32), wcs.view(np.uint32)), i
            assert int(counts[i]) == wr.size, i
            assert np.array_equal(rows[i, :wr.size], wr), i
            assert np.array_equal(scores[i, :wr.size].view(np.uint32), ws.view(np.uint32)), i
        # the same lists again: scratch reuse leaves no trace
        rows2, scores2, counts2 = idx.search_candidates(qs, lists, k, fetch)
        assert np.array_equal(rows2, rows) and np.array_equal(counts2, counts)
    finally:
        idx.destroy()


def test_candidate_outside_index_is_rejected():
    from browservec_b200 import _lib
    from browservec_b200.index import AddonQuantIndex

    idx = AddonQuantIndex(64, bits=8)
    try:
        idx.append(_rows(100, 64, 1), 100)
        with pytest.raises(_lib.BvError, match="outside the index"):
            idx.search_candidates(_rows(1, 64, 2), [np.array([3, 100], np.uint32)], 2, 4)
        rows, _, counts = idx.search_candidates(_rows(1, 64, 2), [np.array([5, 9, 7], np.uint32)], 2, 4)
        assert int(counts[0]) == 2 and set(rows[0].tolist()) <= {5, 7, 9}
    finally:
        idx.destroy()
