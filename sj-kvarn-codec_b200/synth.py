"""Seeded synthetic K/V/Q streams with the distributions of the benchmark configurations
(no public dataset is involved):

  K = X * s[h, d]   X ~ N(0, 1) (Student-t with nu = 4 when heavy=True), s ~ LogNormal(0, 1) per
                    (KV head, channel), and 4 outlier channels per head whose scale is multiplied by 8
  V ~ N(0, 1)
  Q ~ N(0, 1), rounded to fp16 (the decode-time query precision of the configs)

Values are in the model basis; the cache write rotates them (per-head Hadamard). numpy's PCG64 generator
seeded with the config seed; each position's rows are a pure function of (seed, position), so any range
of positions can be produced independently and in any order.
"""
import numpy as np


class KVStream:
    def __init__(self, seed, n_layers, H, D, heavy=False):
        self.seed, self.nl, self.H, self.D, self.heavy = seed, n_layers, H, D, heavy
        rng = np.random.default_rng([seed, 0xC0FFEE])
        self.scale = np.exp(rng.standard_normal((n_layers, H, D))).astype(np.float32)
        for il in range(n_layers):
            for h in range(H):
                out = rng.choice(D, size=4, replace=False)
                self.scale[il, h, out] *= 8.0

    def rows(self, pos0, n, layer=None):
        """(K, V) float32 of positions [pos0, pos0+n): [n_layers][n][H][D] (or [n][H][D] for one layer)."""
        layers = range(self.nl) if layer is None else [layer]
        ks, vs = [], []
        for il in layers:
            rng = np.random.default_rng([self.seed, 1 + il, pos0, n])
            shape = (n, self.H, self.D)
            if self.heavy:
                x = rng.standard_t(4, size=shape)
            else:
                x = rng.standard_normal(shape)
            ks.append((x * self.scale[il][None]).astype(np.float32))
            vs.append(rng.standard_normal(shape).astype(np.float32))
        if layer is not None:
            return ks[0], vs[0]
        return np.stack(ks), np.stack(vs)


def queries(seed, n_layers, n_q, n_head, D):
    """Q rows [n_layers][n_q][n_head][D], N(0,1) rounded to fp16, returned as float32."""
    rng = np.random.default_rng([seed, 0xABCD])
    return rng.standard_normal((n_layers, n_q, n_head, D)).astype(np.float16).astype(np.float32)
