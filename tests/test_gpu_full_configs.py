"""Parity at the full shapes of BASELINE configurations 3, 4 and 5.

Each corpus is generated on the GPU as the benchmark generates it (1M x 384
int4 mixture; 10M x 768 1-bit mixture; 50M x 128 int8 with the {lang, year}
filter) and searched as a batch on the tensor cores.  The CPU oracle then
scores every row of the codes the GPU holds (the integer scoring restated in
C), selects the best F (score desc, row asc, masked rows excluded) and
re-ranks them with the f64 dot of store.ts:114-130; candidates, their
quantized scores, final rows and exact scores must match bit for bit.  A block
of rows is re-encoded by the oracle to check the codes themselves.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

CONFIGS = {
    "c3": dict(bits=4, n=1_000_000, dim=384, kind="mixture", seed=3, k=10, rf=8, filter=False),
    "c4": dict(bits=1, n=10_000_000, dim=768, kind="mixture", seed=4, k=100, rf=10, filter=False),
    "c5": dict(bits=8, n=50_000_000, dim=128, kind="iid", seed=5, k=10, rf=4, filter=True),
}


def _score_rows_threaded(words, scales, q, dim, bits):
    """O.score_rows over row blocks on all host threads (the C call releases the GIL)."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    n = scales.size
    out = np.empty(n, np.float32)
    step = -(-n // (4 * (os.cpu_count() or 1)))

    def part(a):
        out[a:a + step] = O.score_rows(words[a:a + step], scales[a:a + step], q, dim, bits, O.MODE_INT)

    with ThreadPoolExecutor(os.cpu_count() or 1) as ex:
        list(ex.map(part, range(0, n, step)))
    return out


@pytest.mark.parametrize("name", ["c3", "c4", "c5"])
def test_full_config_batch_matches_oracle(name):
    import torch

    from browservec_b200 import datagen
    from browservec_b200.filter import DeviceColumns
    from browservec_b200.index import AddonQuantIndex

    cfg = CONFIGS[name]
    n, dim, bits, k = cfg["n"], cfg["dim"], cfg["bits"], cfg["k"]
    F = k * cfg["rf"]
    nq = 130  # two query tiles
    dev = torch.device("cuda", 0)
    x = datagen.rows(torch, dev, cfg["kind"], cfg["seed"], 0, n, dim)
    qs = datagen.rows(torch, dev, cfg["kind"], cfg["seed"], 0, nq, dim, stream=datagen.STREAM_QUERIES)
    mask_dev = None
    if cfg["filter"]:
        year, lang = datagen.metadata(torch, dev, cfg["seed"], 0, n)
        dc = DeviceColumns(dev)
        dc.set_number_column("year", year)
        dc.set_string_column("lang", lang, [f"lang{i}" for i in range(8)])
        mask_dev = dc.mask({"lang": "lang0", "year": {"$gte": 2020}})
        del year, lang, dc
    idx = AddonQuantIndex(dim, bits=bits, scoring="int", device=0)
    try:
        idx.append_device(x.data_ptr(), n, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        out = [torch.zeros((nq, k), dtype=torch.int32, device=dev), torch.zeros((nq, k), dtype=torch.float32, device=dev),
               torch.zeros(nq, dtype=torch.int32, device=dev), torch.zeros((nq, F), dtype=torch.int32, device=dev),
               torch.zeros((nq, F), dtype=torch.float32, device=dev), torch.zeros(nq, dtype=torch.int32, device=dev)]
        st = torch.cuda.Stream()
        idx.search_batch_device(qs.data_ptr(), nq, k, F, True, out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr(),
                                mask_ptr=0 if mask_dev is None else mask_dev.data_ptr(),
                                mask_words=0 if mask_dev is None else mask_dev.numel(), stream=st.cuda_stream,
                                cand_rows_ptr=out[3].data_ptr(), cand_scores_ptr=out[4].data_ptr(),
                                cand_counts_ptr=out[5].data_ptr())
        st.synchronize()
        rows, scores, counts, crows, cscores, ccounts = [t.cpu().numpy() for t in out]
        words, scales = idx.export_codes()
        # the codes themselves: a block of rows re-encoded by the oracle
        r0 = n // 3
        ow, osc, _ = O.encode(x[r0:r0 + 4096].cpu().numpy(), dim, bits)
        assert np.array_equal(ow, words[r0:r0 + 4096]) and np.array_equal(osc.view(np.uint32),
                                                                       scales[r0:r0 + 4096].view(np.uint32))
        mask = None if mask_dev is None else mask_dev.cpu().numpy().view(np.uint32)
        qn = qs.cpu().numpy()
        for i in (0, 129):
            sc = _score_rows_threaded(words, scales, qn[i], dim, bits)
            wr, ws = O.topk(sc, F, mask)
            m = int(ccounts[i])
            assert m == wr.size, (name, i)
            assert np.array_equal(crows[i, :m].view(np.uint32), wr), (name, i)
            assert np.array_equal(cscores[i, :m].view(np.uint32), ws.view(np.uint32)), (name, i)
            orig = x[torch.from_numpy(wr.astype(np.int64)).to(dev)].cpu().numpy()
            ex = np.array([np.float32(O.dot_row(orig[j], qn[i])) for j in range(wr.size)], np.float32)
            order = np.argsort(O.keys(ex, wr))[::-1][:k]
            c = int(counts[i])
            assert c == min(k, wr.size)
            assert np.array_equal(rows[i, :c].view(np.uint32), wr[order]), (name, i)
            assert np.array_equal(scores[i, :c].view(np.uint32), ex[order].view(np.uint32)), (name, i)
    finally:
        idx.destroy()
        del x
        torch.cuda.empty_cache()
