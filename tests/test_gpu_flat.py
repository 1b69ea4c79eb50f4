"""Exact fp32 flat index (bits 0) against the reference's CPU scan.

The reference scores an exact flat query with the WASM-SIMD f32 dot of
src/fallback/kernel.wat (restated by the oracle as bvo_wasm_dot); the CUDA
flat kernel computes the same lanes in the same order, so every score is
bit-identical and the top k equals the oracle's canonical top k (score desc,
row asc).  Cases cover dimension tails (dim % 4), rows around the 128-row CTA
block, k up to 1000 and a mask.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _rows(n, d, seed):
    rng = np.random.default_rng(seed)
    return O.normalize_rows(rng.standard_normal((n, d)).astype(np.float32))


@pytest.mark.parametrize("n,d,k", [(1, 4, 1), (127, 5, 10), (128, 384, 10), (129, 3, 5), (20000, 384, 10),
                                   (5000, 1001, 100), (3000, 768, 1000), (700, 1, 3)])
def test_flat_matches_wasm_scan(n, d, k):
    from browservec_b200.index import AddonQuantIndex

    x = _rows(n, d, n + d)
    qs = _rows(4, d, 7)
    idx = AddonQuantIndex(d, bits=0)
    try:
        idx.append(x, n)
        rows, scores, counts, *_ = idx.search_arrays(qs, k, k, False)
        for i in range(qs.shape[0]):
            sc = O.wasm_dot(x, qs[i], d)
            wr, ws = O.topk(sc, k)
            c = int(counts[i])
            assert c == wr.size
            assert np.array_equal(rows[i, :c].astype(np.uint32), wr)
            assert np.array_equal(scores[i, :c].view(np.uint32), ws.view(np.uint32))
    finally:
        idx.destroy()


def test_flat_mask_and_browservec():
    from browservec_b200.index import AddonQuantIndex, BrowserVec

    n, d, k = 4000, 96, 10
    x = _rows(n, d, 3)
    q = _rows(1, d, 4)[0]
    rng = np.random.default_rng(5)
    keep = rng.random(n) < 0.3
    mask = np.packbits(np.concatenate([keep, np.zeros((-n) % 32, bool)]), bitorder="little").view(np.uint32)
    idx = AddonQuantIndex(d, bits=0)
    try:
        idx.append(x, n)
        hits = idx.query_masked(q, k, mask)
        wr, ws = O.topk(O.wasm_dot(x, q, d), k, mask)
        assert [h.row for h in hits] == wr.tolist()
    finally:
        idx.destroy()
    db = BrowserVec.create({"dimension": d, "quantBits": 0})
    try:
        db.add_batch([{"id": f"v{i}", "vector": x[i]} for i in range(n)])
        res = db.query(x[17], k=5)
        assert res[0].id == "v17"
        wr, _ = O.topk(O.wasm_dot(x, O.normalize(x[17]), d), 5)
        assert [r.id for r in res] == [f"v{r}" for r in wr.tolist()]
    finally:
        db.destroy()
