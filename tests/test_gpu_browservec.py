"""BrowserVec's filtered queries (src/index.ts:343-436, :473-517) on the GPU.

The filter's mask comes from the device predicate over device copies of the
metadata columns, cached per (filter, store version).  Checked against the
oracle: at most 4096 matches -> the exact scan of the matching rows
(queryRowsExact, src/index.ts:445-464); more -> the masked quantized search
(same rows and exact scores as the oracle's masked query); deletes bump the
version and drop their rows; a filtered query_batch equals query() per query.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

N, D = 12000, 64
LANGS = ["en", "fr", "de", "es"]


def _store(scoring):
    from browservec_b200.index import BrowserVec

    rng = np.random.default_rng(7)
    x = rng.standard_normal((N, D)).astype(np.float32)
    lang = rng.integers(0, 4, N)
    year = rng.integers(1990, 2030, N)
    recs = [{"id": f"r{i}", "vector": x[i], "metadata": {"lang": LANGS[lang[i]], "year": int(year[i])}}
            for i in range(N)]
    db = BrowserVec.create({"dimension": D, "quantBits": 8, "scoring": scoring})
    db.add_batch(recs)
    return db, O.normalize_rows(x), lang, year


def _want(db, xn, q, k, keep, mode):
    """The oracle's answer: exact scan of <= 4096 matches, else the masked
    quantized query with the reference fetch rule, as (ids, scores)."""
    from browservec_b200.filter import pack_mask

    rows = np.flatnonzero(keep).astype(np.uint32)
    qn = O.normalize_rows(q[None, :])[0]
    if rows.size == 0:
        return [], []
    if rows.size <= 4096:
        r, s = O.query_rows_exact(xn, D, rows, qn, k)
    else:
        k_eff = min(N, k)
        fetch = min(N, max(k_eff, k_eff * db.rerank_factor))
        r, s, _, _ = O.Corpus(xn, D, 8).query(qn, k_eff, fetch, mode, mask=pack_mask(keep))
    return [f"r{i}" for i in r[:k]], list(s[:k])


@pytest.mark.parametrize("scoring,mode", [("asym", O.MODE_ASYM), ("int", O.MODE_INT)])
def test_filtered_queries_match_oracle(scoring, mode):
    db, xn, lang, year = _store(scoring)
    try:
        rng = np.random.default_rng(11)
        qs = rng.standard_normal((70, D)).astype(np.float32)
        deleted = np.zeros(N, bool)
        filters = [({"lang": "en"}, lang == 0),                                   # ~3000: exact rows
                   ({"year": {"$gte": 2000}}, year >= 2000),                       # ~9000: masked search
                   ({"lang": {"$in": ["en", "fr"]}, "year": {"$lt": 2025}}, (lang <= 1) & (year < 2025))]
        for rnd in range(2):
            for flt, keep in filters:
                keep = keep & ~deleted
                for qi in (0, 1):
                    got = db.query(qs[qi], k=10, filter=flt)
                    wi, ws = _want(db, xn, qs[qi], 10, keep, mode)
                    assert [g.id for g in got] == wi, (flt, rnd, qi)
                    assert np.array_equal(np.array([g.score for g in got], np.float32).view(np.uint32),
                                          np.array(ws, np.float32).view(np.uint32))
                batch = db.query_batch(qs, k=10, filter=flt)  # 70 queries: one call (a batch for int)
                for qi in (0, 33, 69):
                    one = db.query(qs[qi], k=10, filter=flt)
                    assert [g.id for g in batch[qi]] == [g.id for g in one], (flt, qi)
                    assert [g.score for g in batch[qi]] == [g.score for g in one]
            # deletes bump the store version: the cached masks are rebuilt without those rows
            for i in range(0, N, 7):
                db.delete(f"r{i}")
                deleted[i] = True
        assert db.query(qs[0], k=5, filter={"lang": "xx"}) == []
        assert db.query_batch(qs[:3], k=5, filter={"year": {"$gt": 3000}}) == [[], [], []]
    finally:
        db.destroy()


def test_filter_errors_are_the_reference_errors():
    db, *_ = _store("asym")
    try:
        q = np.ones(D, np.float32)
        with pytest.raises(ValueError, match='filter: \\$gt on "year" expects a number, got string'):
            db.query(q, 5, filter={"year": {"$gt": "x"}})
        with pytest.raises(ValueError, match='filter: unknown operator "\\$regex" on field "lang"'):
            db.query_batch([q], 5, filter={"lang": {"$regex": "e"}})
    finally:
        db.destroy()


@pytest.mark.parametrize("bits", [8, 1, 0])
def test_snapshot_round_trip_bulk_load(bits):
    """export -> import (src/index.ts:608-700): the snapshot holds the live rows
    only; the imported store, loaded in one bulk append encoded on the GPU,
    answers exactly as a store built record by record from those rows."""
    from browservec_b200.index import BrowserVec

    rng = np.random.default_rng(3)
    n, d = 3000, 48
    x = rng.standard_normal((n, d)).astype(np.float32)
    recs = [{"id": f"r{i}", "vector": x[i], "metadata": {"g": int(i % 5)}} for i in range(n)]
    a = BrowserVec.create({"dimension": d, "quantBits": bits})
    b = c = None
    try:
        a.add_batch(recs)
        for i in range(0, n, 11):
            a.delete(f"r{i}")
        snap = a.export()
        b = BrowserVec.import_(snap, {"quantBits": bits})
        live = [r for i, r in enumerate(recs) if i % 11]
        c = BrowserVec.create({"dimension": d, "quantBits": bits})
        c.add_batch(live)
        assert b.count == c.count == len(live)
        qs = rng.standard_normal((4, d)).astype(np.float32)
        for q in qs:
            for flt in (None, {"g": 2}):
                rb, rc = b.query(q, 10, filter=flt), c.query(q, 10, filter=flt)
                assert [h.id for h in rb] == [h.id for h in rc]
                assert [h.score for h in rb] == [h.score for h in rc]
                assert [h.metadata for h in rb] == [h.metadata for h in rc]
    finally:
        for s in (a, b, c):
            if s is not None:
                s.destroy()
