"""CUDA path vs the C oracle, bit for bit, through the C ABI (libbvcuda.so).

Checked per case: GPU-encoded codes and scales (encode.ts arithmetic), the F
approximate candidates (rows and quantized scores, canonical arithmetic and
tie rule) and the final top-k after the exact re-rank (rows bit-exact; the
fp32 re-rank scores must agree within 1e-5 relative and are in fact
bit-identical, since both sides add the same exact f64 products in the same
order).
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

RERANK_RTOL = 1e-5  # north_star tolerance for the fp32 re-rank scores


def _normal_rows(n, d, seed):
    rng = np.random.default_rng(seed)
    return O.normalize_rows(rng.standard_normal((n, d)).astype(np.float32))


def _index(d, bits, scoring="asym", seed=O.DEFAULT_SEED, rounds=2):
    from browservec_b200.index import AddonQuantIndex
    return AddonQuantIndex(d, seed=seed, rounds=rounds, bits=bits, scoring=scoring)


MODES = {"asym": O.MODE_ASYM, "int": O.MODE_INT, "hamming": O.MODE_HAMMING}


def _check_queries(idx, corpus, qs, k, fetch, scoring, mask=None, rerank=True):
    rows, scores, counts, crows, cscores, ccounts = idx.search_arrays(qs, k, fetch, rerank, mask)
    for i, q in enumerate(qs):
        wr, ws, wcr, wcs = corpus.query(q, k, fetch, MODES[scoring], mask, rerank)
        nc = int(ccounts[i])
        assert nc == wcr.size, (i, nc, wcr.size)
        assert np.array_equal(crows[i, :nc], wcr), f"candidate rows differ for query {i}"
        assert np.array_equal(cscores[i, :nc].view(np.uint32), wcs.view(np.uint32)), \
            f"candidate scores differ for query {i}"
        n = int(counts[i])
        assert n == wr.size
        assert np.array_equal(rows[i, :n], wr), f"final rows differ for query {i}"
        np.testing.assert_allclose(scores[i, :n], ws, rtol=RERANK_RTOL, atol=0)
        assert np.array_equal(scores[i, :n].view(np.uint32), ws.view(np.uint32))


@pytest.mark.parametrize("bits", [8, 4, 1])
@pytest.mark.parametrize("dim", [1, 5, 33, 64, 100, 384, 768, 1000])
def test_encoder_bit_exact(bits, dim):
    if bits == 4 and O.pad_to_pow2(dim) < 8:
        pytest.skip("int4 needs paddedDim >= 8")
    if bits == 1 and O.pad_to_pow2(dim) < 32:
        pytest.skip("1-bit needs paddedDim >= 32")
    n = 777
    x = (O.mulberry32(dim * 10 + bits, n * dim) * 2 - 1).astype(np.float32).reshape(n, dim) * 3
    idx = _index(dim, bits)
    try:
        idx.append(x[:300], 300)
        idx.append(x[300:], n - 300)  # exercises capacity growth + copy
        words, scales = idx.export_codes()
        w2, s2, _ = O.encode(x, dim, bits)
        assert np.array_equal(words, w2)
        assert np.array_equal(scales.view(np.uint32), s2.view(np.uint32))
    finally:
        idx.destroy()


@pytest.mark.parametrize("bits,scoring", [(8, "asym"), (8, "int"), (4, "asym"), (4, "int"),
                                          (1, "asym"), (1, "int"), (1, "hamming")])
@pytest.mark.parametrize("dim", [64, 384, 768])
def test_scan_parity(bits, scoring, dim):
    n = 9000 + dim  # not a multiple of any tile
    x = _normal_rows(n, dim, 1000 + dim + bits)
    qs = _normal_rows(6, dim, 2000 + dim)
    qs[0] = x[17]  # a stored row: must come back first after re-rank
    idx = _index(dim, bits, scoring)
    try:
        idx.append(x, n)
        corpus = O.Corpus(x, dim, bits)
        k = 10
        fetch = O.fetch_count(n, k, {8: 4, 4: 16, 1: 32}[bits])
        _check_queries(idx, corpus, qs, k, fetch, scoring)
        rows, _, _, _, _, _ = idx.search_arrays(qs[:1], k, fetch)
        assert rows[0, 0] == 17
    finally:
        idx.destroy()


@pytest.mark.parametrize("bits,dim", [(8, 4), (8, 8), (8, 16), (4, 8), (4, 16), (4, 2048), (8, 2048),
                                      (8, 4096), (1, 32), (1, 64), (1, 4096), (8, 128),
                                      (8, 37), (4, 250), (1, 70)])
def test_scan_parity_shapes(bits, dim):
    """Every lane layout: chunk bytes 4/8/16, lanes 1..32, chunks per lane 1..8; dimensions that are
    not a multiple of 4 (re-rank rows read from global memory instead of staged by bulk copies)."""
    n = 3000
    x = _normal_rows(n, dim, 3000 + dim + bits)
    qs = _normal_rows(3, dim, 4000 + dim)
    for scoring in (["asym", "int"] + (["hamming"] if bits == 1 else [])):
        idx = _index(dim, bits, scoring)
        try:
            idx.append(x, n)
            _check_queries(idx, O.Corpus(x, dim, bits), qs, 5, 20, scoring)
        finally:
            idx.destroy()


def test_mask_and_edges():
    dim, n = 96, 5000
    x = _normal_rows(n, dim, 5)
    qs = _normal_rows(4, dim, 6)
    idx = _index(dim, 8)
    corpus = O.Corpus(x, dim, 8)
    try:
        # empty index returns [] (quant.ts:184)
        rows, scores, counts, *_ = idx.search_arrays(qs, 10, 40)
        assert (counts == 0).all()
        idx.append(x, n)
        rng = np.random.default_rng(7)
        for frac in (0.5, 0.01, 0.001):
            bits = rng.random(n) < frac
            from browservec_b200.filter import pack_mask
            mask = pack_mask(bits)
            _check_queries(idx, corpus, qs, 10, 40, "asym", mask=mask)
        # mask that keeps only 3 rows: fewer candidates than fetch
        bits = np.zeros(n, bool)
        bits[[5, 77, 4999]] = True
        _check_queries(idx, corpus, qs, 10, 40, "asym", mask=pack_mask(bits))
        # no re-rank: the approximate top-k
        _check_queries(idx, corpus, qs, 10, 10, "asym", rerank=False)
        # k and fetch above n-ish sizes, fetch at the fused limit
        _check_queries(idx, corpus, qs[:1], 64, 256, "asym")
        # short mask is rejected with the reference's message (scoreMask.ts:68-70)
        from browservec_b200._lib import BvError
        with pytest.raises(ValueError, match="mask has 1 words, need 157 for 5000 rows"):
            idx.search(qs[:1], 10, 40, mask=np.zeros(1, np.uint32))
        with pytest.raises(BvError, match="mask has 1 words, need 157 for 5000 rows"):
            idx.search_arrays(qs[:1], 10, 40, True, np.zeros(1, np.uint32))
        with pytest.raises(BvError, match="exceeds"):
            idx.search(qs[:1], 10, 2000)
    finally:
        idx.destroy()


def test_tiny_corpus_and_ties():
    dim = 48
    x = _normal_rows(7, dim, 9)
    x = np.concatenate([x, x, x])  # exact duplicates: ties broken by lower row
    idx = _index(dim, 8)
    try:
        idx.append(x, x.shape[0])
        corpus = O.Corpus(x, dim, 8)
        qs = _normal_rows(3, dim, 10)
        _check_queries(idx, corpus, qs, 5, 21, "asym")
        rows, scores, counts, *_ = idx.search_arrays(x[2:3], 3, 21)
        assert rows[0, :3].tolist() == [2, 9, 16]
    finally:
        idx.destroy()


def test_query_rows_exact():
    dim, n = 200, 3000
    x = _normal_rows(n, dim, 11)
    idx = _index(dim, 8)
    try:
        idx.append(x, n)
        q = _normal_rows(1, dim, 12)[0]
        sel = np.random.default_rng(3).choice(n, 4096 if n >= 4096 else 1234, replace=False).astype(np.uint32)
        sel.sort()
        got = idx.query_rows_exact(q, sel, 10)
        wr, ws = O.query_rows_exact(x, dim, sel, q, 10)
        assert [h.row for h in got] == wr.tolist()
        assert np.array_equal(np.array([h.score for h in got], np.float32).view(np.uint32), ws.view(np.uint32))
    finally:
        idx.destroy()


def test_c2_shape_parity():
    """BASELINE config 2 shape (100k x 768 int8, k=10, F=40) on a few queries."""
    dim, n = 768, 100_000
    x = _normal_rows(n, dim, 2)
    qs = _normal_rows(4, dim, 102)
    for scoring in ("asym", "int"):
        idx = _index(dim, 8, scoring)
        try:
            idx.append(x, n)
            corpus = O.Corpus(x, dim, 8)
            _check_queries(idx, corpus, qs, 10, 40, scoring)
        finally:
            idx.destroy()


@pytest.mark.parametrize("scoring", ["asym", "int"])
def test_rerank_rounding_boundaries(scoring):
    """Rows whose exact dot sits on an f32 rounding boundary: the kernels' fast
    re-rank order must defer to the reference's sequential f64 sum (store.ts:114-130)."""
    dim = 8
    rng = np.random.default_rng(21)
    rows = [rng.standard_normal(dim).astype(np.float32) for _ in range(20)]
    for tiny in (2.0 ** -60, 2.0 ** -80):
        for pos in (2, 3):
            x = np.zeros(dim, np.float32)
            x[0], x[1], x[pos] = 1.0, 2.0 ** -24, tiny
            rows.append(x)
    x = np.stack(rows)
    n = x.shape[0]
    q = np.array([[1, 1, 1, 1, 0, 0, 0, 0]], np.float32)
    idx = _index(dim, 8, scoring)
    try:
        idx.append(x, n)
        _check_queries(idx, O.Corpus(x, dim, 8), q, n, n, scoring)
        out_rows, out_scores, counts, *_ = idx.search_arrays(q, n, n)
        for r, s in zip(out_rows[0, :counts[0]], out_scores[0, :counts[0]]):
            assert np.float32(s).view(np.uint32) == np.float32(O.dot_row(x[r], q[0])).view(np.uint32)
    finally:
        idx.destroy()
