"""Failure detection without a GPU fault.

Every wait in the kernels is a bounded mbarrier poll: when it runs out the
kernel raises the index's timeout flag and returns, and the host reports
BV_ERR_TIMEOUT.  bv_check_wait_timeout runs that path on a barrier nothing
completes (one thread, no copies in flight); the status and message must be
the ones a search reports, and the same index must then answer a search
exactly as the CPU oracle does.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _rows(n, d, seed):
    rng = np.random.default_rng(seed)
    return O.normalize_rows(rng.standard_normal((n, d)).astype(np.float32))


@pytest.mark.parametrize("polls", [1, 64, 4096])
def test_wait_budget_runs_out_and_index_stays_usable(polls):
    from browservec_b200 import _lib
    from browservec_b200.index import AddonQuantIndex

    n, d, k, fetch = 3000, 96, 10, 40
    x = _rows(n, d, 1)
    idx = AddonQuantIndex(d, bits=8, scoring="asym")
    try:
        idx.append(x, n)
        with pytest.raises(_lib.BvError, match=r"wait ran out of budget \(flag 0x1\)") as ei:
            _lib.check(idx._L.bv_check_wait_timeout(idx._h, polls))
        assert ei.value.status == _lib.BV_ERR_TIMEOUT
        # the flag was cleared and the context is intact: a search is exact
        q = _rows(2, d, 2)
        rows, scores, counts, crows, cscores, ccounts = idx.search_arrays(q, k, fetch, True)
        corpus = O.Corpus(x, d, 8)
        for i in range(2):
            wr, ws, _, _ = corpus.query(q[i], k, fetch)
            assert np.array_equal(rows[i, :counts[i]].astype(np.uint32), wr)
            assert np.array_equal(scores[i, :counts[i]].view(np.uint32), ws.view(np.uint32))
    finally:
        idx.destroy()


def test_wait_probe_rejects_bad_budget():
    from browservec_b200 import _lib
    from browservec_b200.index import AddonQuantIndex

    idx = AddonQuantIndex(32, bits=8)
    try:
        for polls in (0, (1 << 22) + 1):
            with pytest.raises(_lib.BvError, match="polls must be"):
                _lib.check(idx._L.bv_check_wait_timeout(idx._h, polls))
    finally:
        idx.destroy()
