"""The reference's own known-answer tests, restated against the C oracle.

Each test names the reference test it restates (tests/unit/*.test.ts in
sharma-open-source/browservec).  These pin the oracle before it is trusted as
the parity checker for the CUDA path.  CPU only.
"""
import numpy as np
import pytest

from oracle import np_ref
from oracle import oracle as O


def random_vec(n, seed, scale=1.0):
    """tests/unit/rotator.test.ts:5-10 / codec.test.ts:5-10: (rng()*2-1)*scale as f32."""
    r = O.mulberry32(seed, n)
    return ((r * 2 - 1) * scale).astype(np.float32)


# ----------------------------------------------------------- prng.test.ts
def test_mulberry32_deterministic_and_range():
    # prng.test.ts:5-35
    a = O.mulberry32(42, 100)
    assert np.array_equal(a, O.mulberry32(42, 100))
    assert not np.array_equal(O.mulberry32(1, 20), O.mulberry32(2, 20))
    v = O.mulberry32(0xDEADBEEF, 10_000)
    assert (v >= 0).all() and (v < 1).all()
    m = O.mulberry32(7, 50_000).mean()
    assert 0.48 < m < 0.52


def test_mulberry32_matches_independent_restatement():
    for seed in (0, 1, 42, 0x9E3779B9, 0xFFFFFFFF, 123456789):
        rng = np_ref.Mulberry32(seed)
        want = np.array([rng() for _ in range(257)])
        assert np.array_equal(O.mulberry32(seed, 257), want)


def test_random_signs():
    # prng.test.ts:38-50
    s = O.random_signs(1024, 123)
    assert set(np.abs(s).tolist()) == {1.0}
    a, b = O.random_signs(256, 9), O.random_signs(256, 9)
    assert np.array_equal(a, b) and (a == 1).any() and (a == -1).any()
    assert np.array_equal(a, np_ref.random_signs(256, 9))


# -------------------------------------------------------- rotator.test.ts
def test_pad_to_pow2():
    # rotator.test.ts:18-28
    for n, p in [(1, 4), (4, 4), (5, 8), (384, 512), (768, 1024), (1024, 1024), (1536, 2048)]:
        assert O.pad_to_pow2(n) == p


def test_fwht_involution_and_impulse():
    # rotator.test.ts:31-46
    v = random_vec(64, 1)
    twice = O.fwht(O.fwht(v))
    np.testing.assert_allclose(twice, v * 64, atol=5e-4)
    e0 = np.zeros(8, np.float32)
    e0[0] = 1
    assert (O.fwht(e0) == 1).all()


def test_fwht_matches_independent_restatement():
    for n in (4, 32, 1024):
        v = random_vec(n, n)
        assert np.array_equal(O.fwht(v), np_ref.fwht(v))


def test_rotator_orthonormal():
    # rotator.test.ts:50-60
    dim = 100
    a, b = random_vec(dim, 2), random_vec(dim, 3)
    ra, rb = O.rotate(a, dim, 12345), O.rotate(b, dim, 12345)
    assert ra.size == 128
    assert abs(float(np.dot(ra.astype(np.float64), rb)) - float(np.dot(a.astype(np.float64), b))) < 5e-4
    assert abs(float(np.dot(ra.astype(np.float64), ra)) - float(np.dot(a.astype(np.float64), a))) < 5e-4


def test_rotator_seed_and_rounds():
    # rotator.test.ts:62-76
    v = random_vec(384, 4)
    assert np.array_equal(O.rotate(v, 384, 99, 2), O.rotate(v, 384, 99, 2))
    w = random_vec(64, 5)
    r1, r2, r3 = O.rotate(w, 64, 1), O.rotate(w, 64, 2), O.rotate(w, 64, 1, 3)
    assert not np.array_equal(r1, r2) and not np.array_equal(r1, r3)


@pytest.mark.parametrize("dim,seed,rounds", [(6, 1, 2), (100, 12345, 2), (384, 0x9E3779B9, 2),
                                             (768, 0x9E3779B9, 2), (64, 1, 3), (5, 7, 1)])
def test_rotation_matches_independent_restatement(dim, seed, rounds):
    v = random_vec(dim, seed % 1000 + 3)
    assert np.array_equal(O.rotate(v, dim, seed, rounds), np_ref.rotate(v, dim, seed, rounds))


# ---------------------------------------------------------- codec.test.ts
def test_int8_codec():
    # codec.test.ts:20-52
    v = random_vec(64, 1, 3.0)
    w, s = O.quantize_row(v, 8)
    back = O.dequant_row(w, s, 8)
    assert (np.abs(back - v) <= s / 127 / 2 + 1e-6).all()
    w, s = O.quantize_row(np.array([0.5, -2.5, 1, 0], np.float32), 8)
    assert s == 2.5
    assert abs(O.dequant_row(w, s, 8)[1] + 2.5) < 1e-4
    assert O.quantize_row(random_vec(32, 2, 3.0), 8)[0].size == 8
    w, s = O.quantize_row(np.zeros(16, np.float32), 8)
    assert s == 1 and (O.dequant_row(w, s, 8) == 0).all()
    with pytest.raises(ValueError, match="multiple of 4"):
        O.quantize_row(np.zeros(7, np.float32), 8)


def test_int4_codec():
    # codec.test.ts:54-73
    v = random_vec(64, 3, 3.0)
    w, s = O.quantize_row(v, 4)
    back = O.dequant_row(w, s, 4)
    assert (np.abs(back - v) <= s / 7 / 2 + 1e-6).all()
    assert O.quantize_row(random_vec(64, 4, 3.0), 4)[0].size == 8
    with pytest.raises(ValueError, match="multiple of 8"):
        O.quantize_row(np.zeros(12, np.float32), 4)


def test_1bit_codec():
    # codec.test.ts:75-103
    v = random_vec(64, 5, 3.0)
    w, s = O.quantize_row(v, 1)
    assert abs(s - np.abs(v.astype(np.float64)).sum() / 64) < 1e-5
    back = O.dequant_row(w, s, 1)
    assert np.allclose(back, np.where(v >= 0, 1, -1) * s, atol=1e-5)
    assert O.quantize_row(random_vec(64, 6, 3.0), 1)[0].size == 2
    with pytest.raises(ValueError, match="multiple of 32"):
        O.quantize_row(np.zeros(48, np.float32), 1)
    w, _ = O.quantize_row(np.zeros(32, np.float32), 1)
    assert int(w[0]) == 0xFFFFFFFF


@pytest.mark.parametrize("bits", [8, 4, 1])
def test_codecs_match_independent_restatement(bits):
    for seed in range(6):
        v = random_vec(128, 100 + seed, 3.0)
        if seed == 0:  # exact .5 ties exercise Math.round's half-up rule
            v = np.array([(i % 9 - 4) * 0.5 for i in range(128)], np.float32) * (1 / 127 * 4)
        w, s = O.quantize_row(v, bits)
        w2, s2 = np_ref.quantize_row(v, bits)
        assert np.array_equal(w, w2)
        assert np.float32(s) == np.float32(s2)


def test_math_round_half_up():
    # snormByte uses Math.round (half toward +inf): -0.5*... -> 0, 0.5 -> 1.
    v = np.array([0.5 / 127, -0.5 / 127, 1.5 / 127, -1.5 / 127], np.float32)
    v = np.concatenate([v, np.array([1.0], np.float32)])
    v = np.concatenate([v, np.zeros(3, np.float32)])
    w, _ = O.quantize_row(v, 8)
    b = w.view(np.int8)
    want = [np_ref.js_round(float(np.float32(x)) * 127) for x in v[:4]]
    assert b[:4].tolist() == [int(x) for x in want]


# --------------------------------------------------------- encode.test.ts
def test_batch_encoder_matches_rotate_quantize():
    # encode.test.ts:15-46
    dim, rows = 48, 5
    data = ((O.mulberry32(1, rows * dim) * 2 - 1)).astype(np.float32).reshape(rows, dim)
    words, scales, _ = O.encode(data, dim, 8, seed=11, rounds=2)
    for r in range(rows):
        w, s = O.quantize_row(O.rotate(data[r], dim, 11, 2), 8)
        assert np.array_equal(words[r], w) and scales[r] == np.float32(s)
    dim = 40
    data = ((O.mulberry32(2, 3 * dim) * 2 - 1)).astype(np.float32).reshape(3, dim)
    for bits in (4, 1):
        words, _, _ = O.encode(data, dim, bits, seed=5, rounds=2)
        w, _ = O.quantize_row(O.rotate(data[0], dim, 5, 2), bits)
        assert np.array_equal(words[0], w)


def test_words_per_row():
    # encode.test.ts:48-52
    P = O.pad_to_pow2(384)
    assert [O.words_per_row(P, b) for b in (8, 4, 1)] == [128, 64, 16]
    # 1-bit at d=768 pads to P=1024: 32 words = 128 bytes of sign bits per row.
    assert O.words_per_row(O.pad_to_pow2(768), 1) * 4 == 128


def test_encode_returns_rotated_rows():
    # encode.test.ts:55-66
    dim = 20
    data = ((O.mulberry32(3, 2 * dim) * 2 - 1)).astype(np.float32).reshape(2, dim)
    _, _, rot = O.encode(data, dim, 8, seed=3, rounds=2, want_rotated=True)
    assert rot.shape == (2, 32)
    assert np.array_equal(rot[1], O.rotate(data[1], dim, 3, 2))


def test_encode_validates_length():
    # encode.test.ts:68-71
    with pytest.raises(ValueError, match="expected 16 floats"):
        O.encode(np.zeros(15, np.float32), 8, 8)


# ----------------------------------------------------------- topk.test.ts
def _full_sort(scores, k):
    order = sorted(range(len(scores)), key=lambda r: (-float(scores[r]), r))
    return order[:k]


def test_topk_matches_full_sort():
    # topk.test.ts:14-33 (both the canonical and the reference heap)
    rng = np_ref.Mulberry32(1)
    for n, k in [(100, 10), (1000, 1), (1000, 50), (17, 17)]:
        s = np.array([rng() * 200 - 100 for _ in range(n)], np.float32)
        want = _full_sort(s, k)
        rows, sc = O.topk(s, k)
        assert rows.tolist() == want and np.array_equal(sc, s[want])
        rows, sc = O.topk_ref(s, k)
        assert rows.tolist() == want


def test_topk_edges():
    # topk.test.ts:35-54
    assert O.topk(np.array([3, 1, 2], np.float32), 10)[0].tolist() == [0, 2, 1]
    assert O.topk_ref(np.array([3, 1, 2], np.float32), 10)[0].tolist() == [0, 2, 1]
    assert O.topk(np.array([1, 2], np.float32), 0)[0].size == 0
    assert O.topk(np.zeros(0, np.float32), 5)[0].size == 0
    rows, sc = O.topk(np.array([-5, -1, -3], np.float32), 2)
    assert rows.tolist() == [1, 2] and sc.tolist() == [-1, -3]
    for fn in (O.topk, O.topk_ref):
        rows, sc = fn(np.array([1, 1, 1, 0], np.float32), 3)
        assert sc.tolist() == [1, 1, 1] and set(rows.tolist()) == {0, 1, 2}


def test_topk_tie_rule_lower_row_wins():
    # The canonical rule keeps the lower row on a boundary tie.
    s = np.array([5, 5, 5, 9], np.float32)
    assert O.topk(s, 2)[0].tolist() == [3, 0]


def test_topk_mask():
    s = np.arange(64, dtype=np.float32)
    mask = np.array([0x0000FFFF, 0x0], np.uint32)
    rows, _ = O.topk(s, 3, mask)
    assert rows.tolist() == [15, 14, 13]


def test_merge_partials_ref():
    # gpuTopk.ts:160-189: fillers (-3.4e38 as f64) and out-of-range rows are skipped.
    scores = np.array([1.0, 5.0, 3.0, 4.0], np.float32)
    rows = np.array([0, 1, 2, 99], np.uint32)
    r, s = O.merge_partials_ref(scores, rows, n=10, k=2)
    assert r.tolist() == [1, 2] and s.tolist() == [5.0, 3.0]


# ----------------------------------------------- store.test.ts / cpu.test.ts
def test_dot_row_and_normalize():
    # store.test.ts:88-106 (dotRow) and store.ts:209-217
    a = random_vec(33, 9)
    b = random_vec(33, 10)
    want = sum(float(x) * float(y) for x, y in zip(a[:32:4], b[:32:4]))  # lane 0 only
    assert isinstance(O.dot_row(a, b), float)
    exact = float(np.dot(a.astype(np.float64), b.astype(np.float64)))
    assert abs(O.dot_row(a, b) - exact) < 1e-12
    assert want != 0
    n = O.normalize(a)
    assert abs(float(np.dot(n.astype(np.float64), n)) - 1.0) < 1e-6
    assert (O.normalize(np.zeros(4, np.float32)) == 0).all()


def test_wasm_dot_matches_brute_force():
    # cpu.test.ts:47-72: SIMD == brute force on rows, scores to 3 decimals.
    dim, rows = 33, 500
    data = (O.mulberry32(1, rows * dim) * 2 - 1).astype(np.float32)
    q = (O.mulberry32(2, dim) * 2 - 1).astype(np.float32)
    sc = O.wasm_dot(data, q, dim)
    ref = data.reshape(rows, dim).astype(np.float64) @ q.astype(np.float64)
    assert np.allclose(sc, ref, atol=1e-3)
    r1, _ = O.topk_ref(sc, 10)
    r2, _ = O.topk_ref(ref.astype(np.float32), 10)
    assert r1.tolist() == r2.tolist()
    ro, so = O.cpu_index_query_batch(data, dim, np.stack([q, q]), 10, threads=2)
    assert ro[0].tolist() == r1.tolist() and ro[1].tolist() == r1.tolist()
