"""Exact fp32 flat index (bits 0) against the reference's CPU scan.

The reference scores an exact flat query with the WASM-SIMD f32 dot of
src/fallback/kernel.wat (restated by the oracle as bvo_wasm_dot); the CUDA
flat kernel computes the same lanes in the same order, so every score is
bit-identical and the top k equals the oracle's canonical top k (score desc,
row asc).  Cases cover dimension tails (dim % 4, the per-row kernel), column
tails of the TMA-fed kernel (dim % 32), rows around the 128-row block, k up to
1000 and a mask.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _rows(n, d, seed):
    rng = np.random.default_rng(seed)
    return O.normalize_rows(rng.standard_normal((n, d)).astype(np.float32))


@pytest.mark.parametrize("n,d,k", [(1, 4, 1), (127, 5, 10), (128, 384, 10), (129, 3, 5), (20000, 384, 10),
                                   (5000, 1001, 100), (3000, 768, 1000), (700, 1, 3), (129, 100, 10),
                                   (257, 36, 256), (50000, 64, 40), (3000, 2052, 7)])
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
        # one query per call (a grid over every CTA slot) gives the same answer
        r1, s1, c1, *_ = idx.search_arrays(qs[:1], k, k, False)
        assert np.array_equal(r1[0, :c1[0]], rows[0, :counts[0]])
        assert np.array_equal(s1[0, :c1[0]].view(np.uint32), scores[0, :counts[0]].view(np.uint32))
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


def test_async_n_matches_per_call():
    """bv_search_async_n over several indexes gives each entry's bv_search_async answer."""
    import torch
    from browservec_b200.index import AddonQuantIndex, AsyncSearchList

    dev = torch.device("cuda", 0)
    n, d, k = 3000, 96, 10
    idxs, xs = [], []
    for r, bits in enumerate((0, 8, 0)):
        x = _rows(n, d, 40 + r)
        ix = AddonQuantIndex(d, bits=bits, scoring="int" if bits else "asym")
        ix.append(x, n)
        idxs.append(ix)
        xs.append(x)
    try:
        qs = torch.from_numpy(_rows(6, d, 50)).to(dev)
        o_r = torch.zeros(6, k, dtype=torch.int32, device=dev)
        o_s = torch.zeros(6, k, device=dev)
        o_c = torch.zeros(6, dtype=torch.int32, device=dev)
        lst = AsyncSearchList([(idxs[i % 3], qs[i].data_ptr(), k, 40, True, o_r[i].data_ptr(), o_s[i].data_ptr(),
                                o_c[i:].data_ptr()) for i in range(6)])
        torch.cuda.synchronize()
        lst.submit(0)  # NULL stream: each entry on its index's own stream
        torch.cuda.synchronize()
        for i in range(6):
            rows, scores, counts, *_ = idxs[i % 3].search_arrays(qs[i:i + 1].cpu().numpy(), k, 40, True)
            c = int(counts[0])
            assert int(o_c[i]) == c
            assert np.array_equal(o_r[i, :c].cpu().numpy().astype(np.uint32), rows[0, :c])
            assert np.array_equal(o_s[i, :c].cpu().numpy().view(np.uint32), scores[0, :c].view(np.uint32))
    finally:
        for ix in idxs:
            ix.destroy()
