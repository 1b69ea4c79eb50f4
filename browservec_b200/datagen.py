"""Seeded synthetic corpora of the benchmark configurations, generated on the GPU.

Rows are produced in fixed chunks of ``CHUNK`` rows; chunk c of stream s is
drawn from a Philox generator seeded with ``(seed, s, c)``, so any row range
(one shard of a row-sharded corpus) is generated alone and identically for
every shard count.  Rows are L2-normalised with an f64 sum of squares and an
f64 division, rounded to f32 (the normalisation of src/store/store.ts:209-217
up to the summation order of the f64 reduction).

* ``iid``: N(0,1) components.
* ``mixture``: ``centres`` centres drawn N(0,1) from ``(seed, centres)``; a
  row picks a centre uniformly and adds ``sigma``*N(0,1) noise.
"""
from __future__ import annotations

CHUNK = 1 << 16
STREAM_ROWS, STREAM_QUERIES, STREAM_CENTRES, STREAM_META = 0, 1, 2, 3


def _gen(torch, device, seed: int, stream: int, chunk: int):
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1_000_003 + stream * 7_919 + chunk * 104_729) & 0x7FFF_FFFF_FFFF_FFFF)
    return g


def normalize_(torch, x):
    """In-place f64-accumulated L2 normalisation of float32 rows."""
    n = x.double().pow(2).sum(1, keepdim=True).sqrt()
    n[n == 0] = 1.0
    x.copy_((x.double() / n).float())
    return x


def centres(torch, device, seed: int, n_centres: int, dim: int):
    return torch.randn((n_centres, dim), generator=_gen(torch, device, seed, STREAM_CENTRES, 0),
                       device=device, dtype=torch.float32)


def rows(torch, device, kind: str, seed: int, lo: int, hi: int, dim: int, stream: int = STREAM_ROWS,
         n_centres: int = 1024, sigma: float = 0.3, out=None):
    """Rows [lo, hi) of the corpus (or query set, stream=STREAM_QUERIES)."""
    n = hi - lo
    if out is None:
        out = torch.empty((n, dim), dtype=torch.float32, device=device)
    cen = centres(torch, device, seed, n_centres, dim) if kind == "mixture" else None
    c0, c1 = lo // CHUNK, (hi + CHUNK - 1) // CHUNK
    for c in range(c0, c1):
        a, b = max(lo, c * CHUNK), min(hi, (c + 1) * CHUNK)
        g = _gen(torch, device, seed, stream, c)
        if kind == "iid":
            blk = torch.randn((CHUNK, dim), generator=g, device=device, dtype=torch.float32)
        elif kind == "mixture":
            pick = torch.randint(0, n_centres, (CHUNK,), generator=g, device=device)
            noise = torch.randn((CHUNK, dim), generator=g, device=device, dtype=torch.float32)
            blk = cen[pick] + sigma * noise
        else:
            raise ValueError(kind)
        out[a - lo:b - lo] = blk[a - c * CHUNK:b - c * CHUNK]
        normalize_(torch, out[a - lo:b - lo])
    return out


def metadata(torch, device, seed: int, lo: int, hi: int, years=(1990, 2029), n_lang: int = 8,
             zipf_s: float = 1.1):
    """Per-row integer 'year' uniform in [years] and categorical 'lang' code in
    [0, n_lang) with Zipf(zipf_s) frequencies (code 0 the most common)."""
    n = hi - lo
    year = torch.empty(n, dtype=torch.int32, device=device)
    lang = torch.empty(n, dtype=torch.uint8, device=device)
    w = torch.tensor([1.0 / (i + 1) ** zipf_s for i in range(n_lang)], dtype=torch.float64, device=device)
    w = w / w.sum()
    c0, c1 = lo // CHUNK, (hi + CHUNK - 1) // CHUNK
    for c in range(c0, c1):
        a, b = max(lo, c * CHUNK), min(hi, (c + 1) * CHUNK)
        g = _gen(torch, device, seed, STREAM_META, c)
        y = torch.randint(years[0], years[1] + 1, (CHUNK,), generator=g, device=device, dtype=torch.int32)
        l = torch.multinomial(w, CHUNK, replacement=True, generator=g).to(torch.uint8)
        year[a - lo:b - lo] = y[a - c * CHUNK:b - c * CHUNK]
        lang[a - lo:b - lo] = l[a - c * CHUNK:b - c * CHUNK]
    return year, lang
