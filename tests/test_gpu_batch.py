"""Batched tensor-core search (bv_search_batch) against the per-query scans.

The batch scores with exact int8 contractions, so every candidate (rows and
quantized scores), every exact re-rank score and every final row must be
bit-identical to bv_search_async over the same queries, and to the oracle.
Cases cover the three code widths, both integer scorings, paddedDim below and
above one 128-byte K block, query counts across the 128-query tile, row counts
off the 256-row tile, masks, wide F, and a corpus sorted by score that forces
the candidate-buffer overflow fallback.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

MODES = {"int": O.MODE_INT, "hamming": O.MODE_HAMMING}


def _rows(n, d, seed):
    rng = np.random.default_rng(seed)
    return O.normalize_rows(rng.standard_normal((n, d)).astype(np.float32))


def _run(idx, fn_name, q, k, fetch, mask=None):
    import torch

    nq = q.shape[0]
    dev = q.device
    out = [torch.zeros((nq, k), dtype=torch.int32, device=dev), torch.zeros((nq, k), dtype=torch.float32, device=dev),
           torch.zeros(nq, dtype=torch.int32, device=dev), torch.zeros((nq, fetch), dtype=torch.int32, device=dev),
           torch.zeros((nq, fetch), dtype=torch.float32, device=dev), torch.zeros(nq, dtype=torch.int32, device=dev),
           torch.zeros((nq, fetch), dtype=torch.float32, device=dev)]
    m = None if mask is None else torch.from_numpy(mask.view(np.int32)).to(dev)
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    fn = idx.search_batch_device if fn_name == "batch" else idx.search_device_cand
    fn(q.data_ptr(), nq, k, fetch, True, out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr(),
       mask_ptr=0 if m is None else m.data_ptr(), mask_words=0 if m is None else m.numel(),
       stream=stream.cuda_stream, cand_rows_ptr=out[3].data_ptr(), cand_scores_ptr=out[4].data_ptr(),
       cand_counts_ptr=out[5].data_ptr(), cand_exact_ptr=out[6].data_ptr())
    stream.synchronize()
    return [t.cpu().numpy() for t in out]


def _compare(got, want, nq, k, fetch):
    gr, gs, gc, gcr, gcs, gcc, gce = got
    wr, ws, wc, wcr, wcs, wcc, wce = want
    assert np.array_equal(gc, wc) and np.array_equal(gcc, wcc)
    for i in range(nq):
        n, m = int(wc[i]), int(wcc[i])
        assert np.array_equal(gcr[i, :m], wcr[i, :m]), f"candidate rows differ, query {i}"
        assert np.array_equal(gcs[i, :m].view(np.uint32), wcs[i, :m].view(np.uint32)), f"candidate scores, query {i}"
        assert np.array_equal(gce[i, :m].view(np.uint32), wce[i, :m].view(np.uint32)), f"exact scores, query {i}"
        assert np.array_equal(gr[i, :n], wr[i, :n]), f"final rows differ, query {i}"
        assert np.array_equal(gs[i, :n].view(np.uint32), ws[i, :n].view(np.uint32)), f"final scores, query {i}"


@pytest.mark.parametrize("bits,scoring,n,d,nq,k,fetch", [
    (8, "int", 5000, 384, 5, 10, 40),
    (8, "int", 20011, 768, 130, 10, 40),
    (8, "int", 3000, 64, 70, 5, 20),       # paddedDim 64 < one K block
    (4, "int", 30000, 384, 200, 10, 80),
    (4, "int", 7777, 100, 33, 10, 160),    # P = 128
    (1, "hamming", 40000, 768, 64, 100, 1000),
    (1, "int", 12000, 256, 129, 10, 320),
    (1, "hamming", 5000, 96, 17, 10, 40),  # P = 128, 96 real dims
])
def test_batch_matches_per_query(bits, scoring, n, d, nq, k, fetch):
    import torch

    from browservec_b200.index import AddonQuantIndex

    x = _rows(n, d, bits * 31 + nq)
    qs = _rows(nq, d, 5 + nq)
    idx = AddonQuantIndex(d, bits=bits, scoring=scoring)
    try:
        idx.append(x[: n // 3], n // 3)
        q = torch.from_numpy(qs).cuda()
        _compare(_run(idx, "batch", q, k, fetch), _run(idx, "single", q, k, fetch), nq, k, fetch)
        idx.append(x[n // 3:], n - n // 3)  # rows appended after a batch: the tiles are extended
        got = _run(idx, "batch", q, k, fetch)
        _compare(got, _run(idx, "single", q, k, fetch), nq, k, fetch)
        corpus = O.Corpus(x, d, bits)
        for i in range(min(nq, 4)):
            wr, ws, wcr, wcs = corpus.query(qs[i], k, fetch, MODES[scoring])
            assert np.array_equal(got[3][i, :wcr.size].view(np.uint32), wcr)
            assert np.array_equal(got[4][i, :wcs.size].view(np.uint32), wcs.view(np.uint32))
            assert np.array_equal(got[0][i, :wr.size].view(np.uint32), wr)
            assert np.array_equal(got[1][i, :ws.size].view(np.uint32), ws.view(np.uint32))
    finally:
        idx.destroy()


@pytest.mark.parametrize("keep_frac", [0.1, 0.6, 0.0, 0.0005])
def test_batch_mask(keep_frac):
    """A mask keeping at most half the rows is served by compacting the kept
    rows into their own tiles; above half the GEMM masks in its epilogue.
    Bits past the last row are set on purpose: they must be ignored."""
    import torch

    from browservec_b200.index import AddonQuantIndex

    n, d, nq, k, fetch = 9001, 128, 100, 10, 40
    x = _rows(n, d, 3)
    rng = np.random.default_rng(4)
    keep = rng.random(n) < keep_frac
    mask = np.packbits(np.concatenate([keep, np.ones((-n) % 32, bool)]), bitorder="little").view(np.uint32)
    idx = AddonQuantIndex(d, bits=8, scoring="int")
    try:
        idx.append(x, n)
        q = torch.from_numpy(_rows(nq, d, 5)).cuda()
        got = _run(idx, "batch", q, k, fetch, mask)
        _compare(got, _run(idx, "single", q, k, fetch, mask), nq, k, fetch)
        assert int(got[2].min()) == min(k, int(keep.sum()))
        for i in range(nq):
            assert all(keep[r] for r in got[0][i, :int(got[2][i])].tolist())
    finally:
        idx.destroy()


def test_batch_overflow_fallback():
    """Rows along one direction with a growing norm (a raw index, not
    normalised): the score factor and the score both grow with the row, so the
    first round -- tiles scattered over the factor order -- misses the best
    rows, the next round's candidates overflow their buffers and the batch is
    redone round by round.  The result must not change."""
    import torch

    from browservec_b200.index import AddonQuantIndex

    n, d, nq, k, fetch = 300_000, 64, 8, 10, 40
    rng = np.random.default_rng(9)
    u = rng.standard_normal(d).astype(np.float64)
    u /= np.linalg.norm(u)
    x = (np.linspace(1.0, 2.0, n)[:, None] * u[None, :]).astype(np.float32)
    qs = O.normalize_rows((u + 0.01 * rng.standard_normal((nq, d))).astype(np.float32))
    idx = AddonQuantIndex(d, bits=8, scoring="int", metric="dot")
    try:
        idx.append(x, n)
        q = torch.from_numpy(qs).cuda()
        got = _run(idx, "batch", q, k, fetch)
        launches = idx.last_launches()
        _compare(got, _run(idx, "single", q, k, fetch), nq, k, fetch)
        assert got[0][0, 0] == n - 1  # the largest row scores highest
        # fast path: prep + (gemm + select) per round + tail; the fallback adds more
        T = (n + 255) // 256
        rounds, seen = 0, 0
        grow = (4096 - fetch) / (2.0 * fetch)
        while seen < T:
            size = 16 if seen == 0 else max(1, int(seen * grow))
            seen = min(T, seen + size)
            rounds += 1
        assert launches > 2 + 2 * rounds, (launches, rounds)
    finally:
        idx.destroy()


def test_batch_rejects_asym():
    import torch

    from browservec_b200 import _lib
    from browservec_b200.index import AddonQuantIndex

    idx = AddonQuantIndex(64, bits=8, scoring="asym")
    try:
        idx.append(_rows(100, 64, 1), 100)
        q = torch.from_numpy(_rows(2, 64, 2)).cuda()
        with pytest.raises(_lib.BvError, match="integer modes"):
            _run(idx, "batch", q, 5, 10)
    finally:
        idx.destroy()


@pytest.mark.parametrize("bits,scoring,n,d,nq,k,fetch", [
    (8, "int", 20011, 768, 130, 10, 40),
    (4, "int", 30000, 384, 385, 10, 80),    # an odd number of query tiles (4): the last pair is half empty
    (1, "hamming", 40000, 768, 300, 100, 1000),
])
def test_pair_gemm_matches_per_query(bits, scoring, n, d, nq, k, fetch, monkeypatch):
    """The CTA-pair GEMM (cta_group::2, chosen with BV_GEMM_PAIR=1 when a batch
    has two or more query tiles) gives the same bits as the per-query scans."""
    import torch

    from browservec_b200.index import AddonQuantIndex

    monkeypatch.setenv("BV_GEMM_PAIR", "1")
    x = _rows(n, d, bits * 37 + nq)
    qs = _rows(nq, d, 9 + nq)
    idx = AddonQuantIndex(d, bits=bits, scoring=scoring)
    try:
        idx.append(x, n)
        q = torch.from_numpy(qs).cuda()
        _compare(_run(idx, "batch", q, k, fetch), _run(idx, "single", q, k, fetch), nq, k, fetch)
    finally:
        idx.destroy()
