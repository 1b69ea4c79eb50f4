"""Device metadata predicate (bv_filter_mask) against the reference semantics.

The host mirror (FilterColumns, vectorised compileFilter of
src/store/filter.ts:18-68) is itself checked against the row-by-row predicate;
the device mask must equal it bit for bit for every operator and every value
type (numbers, strings, booleans, null, missing fields), with tombstones.
Filtered batched searches then compact the kept rows (tested beside the
per-query masked scan in test_gpu_batch.py).
"""
import numpy as np
import pytest

from browservec_b200.filter import DeviceColumns, FilterColumns, compile_filter, pack_mask

FILTERS = [
    {"lang": "en"}, {"lang": {"$ne": "en"}}, {"year": {"$gte": 2020}}, {"year": {"$gt": 2000, "$lt": 2010}},
    {"lang": {"$in": ["en", "fr", 5]}}, {"flag": True}, {"flag": {"$ne": False}}, {"year": None},
    {"nofield": {"$ne": 1}}, {"nofield": 1}, {"lang": "en", "year": {"$gte": 2020}}, {"year": "2020"},
    {"year": 2020.0}, {"lang": {"$in": []}}, {"lang": "zz"}, {"year": {"$lte": 1995}, "flag": {"$ne": True}},
    {"score": {"$lt": 0.25}}, {"year": {"$in": [1990, 2029, None, "2020"]}},
    # Set.has is SameValueZero (filter.ts:29-30): NaN in $in finds stored NaN; $eq NaN finds nothing
    {"score": {"$in": [float("nan"), 0.5]}}, {"score": float("nan")}, {"score": {"$ne": float("nan")}},
    # more values than one device term holds (an OR of calls) and more terms than one call holds (an AND)
    {"year": {"$in": list(range(1990, 2030, 1))}},
    {"year": {"$gte": 1990, "$lte": 2029, "$ne": 2001, "$gt": 1989, "$lt": 2030, "$in": list(range(1990, 2030))},
     "lang": {"$ne": "zz", "$in": ["en", "fr", "de", "es", 5], "$eq": "en"},
     "score": {"$gte": 0.0, "$lte": 1.0, "$ne": 0.5, "$gt": -1, "$lt": 2},
     "flag": {"$ne": None, "$in": [True, False], "$eq": True}},
]


def _records(n, seed):
    rng = np.random.default_rng(seed)
    langs = ["en", "fr", "de", "es", 5, None]
    out = []
    for i in range(n):
        m = {}
        r = rng.random()
        if r < 0.7:
            m["year"] = int(rng.integers(1990, 2030))
        elif r < 0.8:
            m["year"] = "2020"
        elif r < 0.85:
            m["year"] = None
        elif r < 0.9:
            m["year"] = bool(rng.integers(2))
        if rng.random() < 0.9:
            m["lang"] = langs[int(rng.integers(len(langs)))]
        if rng.random() < 0.5:
            m["flag"] = bool(rng.integers(2))
        if rng.random() < 0.6:
            m["score"] = float(rng.random()) if rng.random() < 0.9 else float("nan")
        out.append(m if m or rng.random() < 0.5 else None)
    return out


def test_host_columns_match_row_predicate():
    recs = _records(700, 1)
    fc = FilterColumns()
    fc.append(recs)
    for flt in FILTERS:
        pred = compile_filter(flt)
        want = np.array([pred(m) for m in recs])
        assert np.array_equal(fc.match(flt), want), flt


def test_compile_errors_match_reference():
    import torch

    fc = FilterColumns()
    fc.append(_records(10, 2))
    dc = DeviceColumns.from_host(fc, torch.device("cpu"))
    with pytest.raises(ValueError, match='filter: \\$gt on "year" expects a number, got string'):
        dc.units({"year": {"$gt": "x"}})
    with pytest.raises(ValueError, match='filter: \\$in on "lang" expects an array, got string'):
        dc.units({"lang": {"$in": "en"}})
    with pytest.raises(ValueError, match='filter: unknown operator "\\$regex" on field "lang"'):
        dc.units({"lang": {"$regex": "e"}})


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 31, 32, 1000, 4099])
def test_device_mask_matches_host(n):
    import torch

    recs = _records(n, n)
    fc = FilterColumns()
    fc.append(recs)
    dc = DeviceColumns.from_host(fc, torch.device("cuda"))
    rng = np.random.default_rng(n + 1)
    live = rng.random(n) < 0.8
    live_w = torch.from_numpy(pack_mask(live).view(np.int32)).cuda()
    for flt in FILTERS:
        want = pack_mask(fc.match(flt))
        got = dc.mask(flt).cpu().numpy().view(np.uint32)
        assert np.array_equal(got, want), flt
        got_live = dc.mask(flt, live=live_w).cpu().numpy().view(np.uint32)
        assert np.array_equal(got_live, pack_mask(fc.match(flt) & live)), flt


@pytest.mark.gpu
def test_typed_columns_c5_filter():
    """The config-5 shape: an integer 'year' and a categorical 'lang' held as
    device columns; {lang: <top>, year: {$gte: 2020}}."""
    import torch

    n = 100_003
    rng = np.random.default_rng(5)
    year = rng.integers(1990, 2030, n)
    lang = rng.integers(0, 8, n)
    words = [f"l{i}" for i in range(8)]
    dc = DeviceColumns(torch.device("cuda"))
    dc.set_number_column("year", torch.from_numpy(year).cuda())
    dc.set_string_column("lang", torch.from_numpy(lang).cuda(), words)
    flt = {"lang": "l0", "year": {"$gte": 2020}}
    got = dc.mask(flt).cpu().numpy().view(np.uint32)
    assert np.array_equal(got, pack_mask((lang == 0) & (year >= 2020)))
