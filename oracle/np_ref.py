"""Independent numpy / pure-Python restatement of the reference's encoder.

TEST INFRASTRUCTURE ONLY.  A second, independently written restatement used to
cross-check the C oracle (oracle/bv_oracle.c) on small inputs: the two share no
code, so agreement pins the C oracle's reading of the TypeScript.  Pure-Python
loops: small cases only.
"""
from __future__ import annotations

import math

import numpy as np

M32 = 0xFFFFFFFF


def _imul(a: int, b: int) -> int:
    return (a * b) & M32


class Mulberry32:
    """prng.ts:5-14, written from the JS semantics (ToInt32 / >>> 0 as mod 2^32)."""

    def __init__(self, seed: int):
        self.a = seed & M32

    def next_u32(self) -> int:
        self.a = (self.a + 0x6D2B79F5) & M32
        a = self.a
        t = _imul(a ^ (a >> 15), 1 | a)
        t = ((t + _imul(t ^ (t >> 7), 61 | t)) & M32) ^ t
        return (t ^ (t >> 14)) & M32

    def __call__(self) -> float:
        return self.next_u32() / 4294967296.0


def random_signs(n: int, seed: int) -> np.ndarray:
    """prng.ts:17-22"""
    rng = Mulberry32(seed)
    return np.array([-1.0 if rng() < 0.5 else 1.0 for _ in range(n)], np.float32)


def pad_to_pow2(n: int) -> int:
    p = 4
    while p < n:
        p <<= 1
    return p


def fwht(a: np.ndarray) -> np.ndarray:
    """rotator.ts:46-58 -- stage-at-a-time with numpy f32 add/sub."""
    a = a.astype(np.float32).copy()
    n = a.size
    length = 1
    while length < n:
        v = a.reshape(-1, 2, length)
        x = v[:, 0, :].copy()
        y = v[:, 1, :].copy()
        v[:, 0, :] = x + y
        v[:, 1, :] = x - y
        length <<= 1
    return a


def rotator_signs(dim: int, seed: int, rounds: int) -> np.ndarray:
    P = pad_to_pow2(dim)
    inv = 1.0 / math.sqrt(P)
    out = []
    for r in range(rounds):
        rs = (seed ^ ((0x9E3779B9 * (r + 1)) & M32)) & M32
        s = random_signs(P, rs).astype(np.float64) * inv
        out.append(s.astype(np.float32))
    return np.stack(out) if out else np.zeros((0, P), np.float32)


def rotate(x: np.ndarray, dim: int, seed: int, rounds: int) -> np.ndarray:
    P = pad_to_pow2(dim)
    s = rotator_signs(dim, seed, rounds)
    d = np.zeros(P, np.float32)
    d[:dim] = x
    for r in range(rounds):
        d = (d * s[r]).astype(np.float32)
        d = fwht(d)
    return d


def js_round(x: float) -> float:
    r = math.floor(x)
    return r + 1 if x - r >= 0.5 else r


def quantize_row(rot: np.ndarray, bits: int):
    """codec.ts:32-54 / :85-108 / :135-154 in Python floats (f64)."""
    rot = rot.astype(np.float32)
    n = rot.size
    if bits == 1:
        s = 0.0
        for v in rot:
            s += abs(float(v))
        scale = float(np.float32(s / n)) if s > 0 else 1.0
        words = []
        for g in range(n // 32):
            w = 0
            for j in range(32):
                if rot[g * 32 + j] >= 0:
                    w |= 1 << j
            words.append(w)
        return np.array(words, np.uint32), scale
    levels, per, width, mask = (127.0, 4, 8, 0xFF) if bits == 8 else (7.0, 8, 4, 0xF)
    m = 0.0
    for v in rot:
        if abs(float(v)) > m:
            m = abs(float(v))
    scale = m if m > 0 else 1.0
    inv = 1.0 / scale
    words = []
    for g in range(n // per):
        w = 0
        for j in range(per):
            c = float(rot[g * per + j]) * inv
            c = -1.0 if c < -1 else (1.0 if c > 1 else c)
            b = int(max(-levels, min(levels, js_round(c * levels))))
            w |= (b & mask) << (width * j)
        words.append(w)
    return np.array(words, np.uint32), scale
