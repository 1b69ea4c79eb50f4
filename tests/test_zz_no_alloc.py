"""bv_search_noalloc through the C ABI against bv_search_async.

bv_search_noalloc serves hosts that cannot allocate device memory while they
run (their device memory is reserved up front by their own pool, or a budget
forbids cudaMalloc and the synchronisation of cudaFree on the query path): its
scan and tail kernels keep their scratch in a fixed array inside the library.
Two calls in a row must give the same rows and the same scores, within the
re-rank tolerance of the other GPU tests, as the allocating entry point; the
second call also shows that what the first left in the shared array does not
leak into the next result.  The file name sorts last so that a run stopping at
its first failure has run every other test before this one.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RERANK_RTOL = 1e-5  # same tolerance as the other re-rank checks


def _rows(n, d, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, d)).astype(np.float64)
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x.astype(np.float32)


def _search(fn, idx, q, k, fetch, stream):
    import torch
    from browservec_b200 import _lib

    nq = q.shape[0]
    dev = q.device
    rows = torch.zeros((nq, k), dtype=torch.int32, device=dev)
    scores = torch.zeros((nq, k), dtype=torch.float32, device=dev)
    counts = torch.zeros(nq, dtype=torch.int32, device=dev)
    crows = torch.zeros((nq, fetch), dtype=torch.int32, device=dev)
    cscores = torch.zeros((nq, fetch), dtype=torch.float32, device=dev)
    ccounts = torch.zeros(nq, dtype=torch.int32, device=dev)
    args = _lib.BvSearchArgs(queries=q.data_ptr(), nq=nq, k=k, fetch=fetch, rerank=1, mask=None,
                             mask_words=0, out_rows=rows.data_ptr(), out_scores=scores.data_ptr(),
                             out_counts=counts.data_ptr(), cand_rows=crows.data_ptr(),
                             cand_scores=cscores.data_ptr(), cand_counts=ccounts.data_ptr())
    _lib.check(fn(idx._h, C.byref(args), C.c_void_p(stream.cuda_stream)))
    stream.synchronize()
    return [t.cpu().numpy() for t in (rows, scores, counts, crows, cscores, ccounts)]


@pytest.mark.parametrize("bits,scoring,fetch", [(8, "asym", 40), (8, "int", 40), (4, "asym", 160),
                                                 (1, "hamming", 256)])
def test_noalloc_matches_search_async(bits, scoring, fetch):
    import torch
    from browservec_b200.index import AddonQuantIndex

    n, d, k, nq = 20000, 384, 10, 6
    idx = AddonQuantIndex(d, seed=0x9E3779B9, rounds=2, bits=bits, scoring=scoring)
    try:
        idx.append(_rows(n, d, 11), n)
        stream = torch.cuda.Stream()
        L = idx._L
        for call in range(2):
            q = torch.from_numpy(_rows(nq, d, 100 + call)).cuda()
            want = _search(L.bv_search_async, idx, q, k, fetch, stream)
            got = _search(L.bv_search_noalloc, idx, q, k, fetch, stream)
            wr, ws, wc, wcr, wcs, wcc = want
            gr, gs, gc, gcr, gcs, gcc = got
            assert np.array_equal(gc, wc) and np.all(wc == k), (call, gc, wc)
            assert np.array_equal(gcc, wcc), (call, gcc, wcc)
            assert np.array_equal(gr, wr), f"rows differ on call {call}"
            np.testing.assert_allclose(gs, ws, rtol=RERANK_RTOL, atol=0)
            for i in range(nq):
                m = int(wcc[i])
                assert np.array_equal(gcr[i, :m], wcr[i, :m]), (call, i)
                np.testing.assert_allclose(gcs[i, :m], wcs[i, :m], rtol=RERANK_RTOL, atol=0)
    finally:
        idx.destroy()


@pytest.mark.parametrize("bits,scoring,mode", [(8, "asym", 0), (8, "int", 1), (1, "hamming", 2)])
def test_noalloc_small_grid_many_queries_matches_oracle(bits, scoring, mode):
    """About 2,000 rows give a scan grid of a few CTAs, so several of the
    call's queries are in flight at once and share tile counters in turn;
    70 queries also wrap the counter rotation once.  Checked against the
    CPU oracle (rows and exact scores) and against bv_search_async."""
    import torch
    from browservec_b200.index import AddonQuantIndex
    from oracle import oracle as O

    n, d, k, fetch, nq = 2048, 64, 10, 40, 70
    x = _rows(n, d, 21)
    idx = AddonQuantIndex(d, seed=0x9E3779B9, rounds=2, bits=bits, scoring=scoring)
    try:
        idx.append(x, n)
        corpus = O.Corpus(x, d, bits)
        stream = torch.cuda.Stream()
        for call in range(2):
            qn = _rows(nq, d, 300 + call)
            q = torch.from_numpy(qn).cuda()
            want = _search(idx._L.bv_search_async, idx, q, k, fetch, stream)
            got = _search(idx._L.bv_search_noalloc, idx, q, k, fetch, stream)
            for a, b in zip(got, want):
                assert np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32)), call
            gr, gs, gc, gcr, gcs, gcc = got
            for i in range(0, nq, 7):
                wr, ws, wcr, wcs = corpus.query(qn[i], k, fetch, mode)
                assert int(gcc[i]) == wcr.size and np.array_equal(gcr[i, : wcr.size].astype(np.uint32), wcr)
                assert np.array_equal(gcs[i, : wcr.size].view(np.uint32), wcs.view(np.uint32)), (call, i)
                assert int(gc[i]) == wr.size and np.array_equal(gr[i, : wr.size].astype(np.uint32), wr)
                np.testing.assert_allclose(gs[i, : wr.size], ws, rtol=RERANK_RTOL, atol=0)
    finally:
        idx.destroy()


def test_noalloc_rejects_exact_index():
    """An exact fp32 index (bits 0) holds no codes: refused before any launch."""
    import torch
    from browservec_b200 import _lib
    from browservec_b200.index import AddonQuantIndex

    idx = AddonQuantIndex(64, seed=1, rounds=2, bits=0, scoring="asym")
    try:
        idx.append(_rows(500, 64, 5), 500)
        q = torch.from_numpy(_rows(1, 64, 6)).cuda()
        with pytest.raises(_lib.BvError, match="quantized indexes only"):
            _search(idx._L.bv_search_noalloc, idx, q, 10, 40, torch.cuda.Stream())
    finally:
        idx.destroy()


def test_noalloc_rejects_fetch_above_limit():
    import torch
    from browservec_b200 import _lib
    from browservec_b200.index import AddonQuantIndex

    idx = AddonQuantIndex(64, seed=1, rounds=2, bits=8, scoring="asym")
    try:
        idx.append(_rows(1000, 64, 3), 1000)
        q = torch.from_numpy(_rows(1, 64, 4)).cuda()
        with pytest.raises(_lib.BvError, match="fixed scratch limit of 256"):
            _search(idx._L.bv_search_noalloc, idx, q, 10, 300, torch.cuda.Stream())
    finally:
        idx.destroy()
