"""Deterministic test inputs, restated from the reference's generators so the golden
hashes it ships can be reproduced:

- vector inputs (tests/vector_inputs.h:8-50 of the reference): xorshift64 (13, 7, 17)
  draws, an approximately Gaussian integer as the sum of four 10-bit uniforms, scaled by
  integer channel and token factors and 2^-12 (exact in float), rounded to fp16;
- position-addressable sequence inputs (tests/test_state.c:33-70): a SplitMix64-style
  mix of (seed, variant, pos, index, side) to a small integer times 2^-12.

Integer arithmetic only, so the values do not depend on libm or the platform.
"""
import numpy as np

M64 = (1 << 64) - 1


class XorShift:
    def __init__(self, seed):
        self.s = seed & M64

    def next(self):
        s = self.s
        s ^= (s << 13) & M64
        s ^= s >> 7
        s ^= (s << 17) & M64
        self.s = s
        return (s >> 11) & 0xFFFFFFFF

    def gauss(self):
        a = 0
        for _ in range(4):
            a += (self.next() & 1023) - 512
        return a


def _f16(vals):
    return np.asarray(vals, dtype=np.float32).astype(np.float16).view(np.uint16)


def fill_group(D, G, seed):
    """One (group, head) seal input: (K, V) as [G][D] fp16 bit patterns."""
    rng = XorShift(0x9E3779B97F4A7C15 ^ seed)
    out = []
    for _side in range(2):
        chf = []
        for _d in range(D):
            if rng.next() % 100 < 3:
                chf.append(24 + (rng.next() & 7))
            else:
                chf.append(1 + (rng.next() & 3))
        ints = np.zeros((G, D), dtype=np.int64)
        for t in range(G):
            tf = 1 + (rng.next() & 3)
            for d in range(D):
                ints[t, d] = rng.gauss() * chf[d] * tf
        # int -> float is exact (|v| < 2^24) and the 2^-12 scaling is exact; numpy's
        # float32 -> float16 cast rounds to nearest even like the codec's converter
        out.append(_f16(ints.astype(np.float32) * np.float32(1.0 / 4096.0)))
    return out[0], out[1]


def fill_rows(rows, n):
    """Rotated float rows for the staging codec; the last row is all zeros."""
    rng = XorShift(0xD1B54A32D192ED03)
    x = np.zeros((rows, n), dtype=np.float32)
    for r in range(rows):
        tf = 1 + (rng.next() & 7)
        ints = np.array([rng.gauss() * tf for _ in range(n)], dtype=np.int64)
        x[r] = ints.astype(np.float32) * np.float32(1.0 / 4096.0)
    x[rows - 1] = 0.0
    return x


def gauss_ints(rng, n):
    return np.array([rng.gauss() for _ in range(n)], dtype=np.int64)


# ---- position-addressable sequence inputs ----

def _mix(x):
    x = (x + 0x9E3779B97F4A7C15) & M64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & M64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & M64
    return x ^ (x >> 31)


def _mix_np(x):
    x = x + np.uint64(0x9E3779B97F4A7C15)
    x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return x ^ (x >> np.uint64(31))


def seq_row(seed, variant, pos, n, side):
    """Values val(seed, variant, pos, i, side) for i in [0, n): float32 [n]."""
    i = np.arange(n, dtype=np.uint64)
    key = (np.uint64((seed << 40) & M64) ^ np.uint64((variant << 36) & M64) ^ np.uint64((pos << 16) & M64)
           ^ (i << np.uint64(1)) ^ np.uint64(side))
    with np.errstate(over="ignore"):
        h = _mix_np(key)
    g = (h & np.uint64(1023)).astype(np.int64) + ((h >> np.uint64(10)) & np.uint64(1023)).astype(np.int64) - 1024
    scale = np.where((i % np.uint64(41)) == 0, 24, 1 + ((h >> np.uint64(20)) & np.uint64(3)).astype(np.int64))
    return (g * scale).astype(np.float32) * np.float32(1.0 / 4096.0)


def edge_tiles(D, G=128, seed=7):
    """Seal inputs (K, V as fp16 bits [G][D]) at the edges of the balancing arithmetic: signed zeros, fp16
    subnormals, values near the fp16 maximum, constant and all-zero rows and columns. Every value is finite
    (the reference's quantiser casts rint() of the balanced value to an integer, so an Inf or NaN input has no
    platform-independent result)."""
    rng = np.random.default_rng(seed)
    sub = np.array([1, 2, 3, 0x1FF, 0x3FF], np.uint16)             # fp16 subnormal encodings
    out = []
    # 1: zeros of both signs with a few subnormals and normals
    k = np.where(rng.random((G, D)) < 0.5, 0x8000, 0x0000).astype(np.uint16)
    m = rng.random((G, D)) < 0.1
    k[m] = rng.choice(sub, m.sum()) | np.where(rng.random(m.sum()) < 0.5, 0x8000, 0).astype(np.uint16)
    v = _f16(rng.standard_normal((G, D)))
    v[:, 3] = 0x8000                                                  # a column of -0
    v[5] = 0                                                          # a row of +0
    out.append(("zeros+subnormals", k, v))
    # 2: a wide dynamic range: values near 65504 next to subnormals
    x = rng.standard_normal((G, D)) * np.exp(rng.uniform(-16, 10, (G, D)))
    k = _f16(np.clip(x, -65504, 65504))
    k[0, 0], k[1, 1], k[2, 2] = 0x7BFF, 0xFBFF, 0x0001
    v = _f16(np.clip(rng.standard_normal((G, D)) * 3e4, -65504, 65504))
    out.append(("wide range", k, v))
    # 3: constant rows and columns (zero standard deviation: the 1e-3 clamp) and an all-zero tile
    k = np.tile(_f16(rng.standard_normal(D)), (G, 1))
    v = np.tile(_f16(rng.standard_normal((G, 1))), (1, D))
    out.append(("constant rows / columns", k, v))
    out.append(("all zero", np.zeros((G, D), np.uint16), np.full((G, D), 0x8000, np.uint16)))
    return out
