"""The seeded input generator of the benchmark configurations (host side, sj-kvarn-codec_b200/csrc/sjk_synth.h):
accuracy of its own ln / exp / cos / sin, its fp16 rounding, the distributions it draws, and that every position
range is generated independently of how the positions are split up or how many threads draw them. The device side
is checked bit-for-bit against this one in tests/test_gpu_configs.py."""
import ctypes as C
import math

import numpy as np
import pytest

import refcache


@pytest.fixture(scope="module")
def G(oracle_lib):
    return refcache._gen(oracle_lib.lib())


def _ulps(a, b):
    a, b = np.float64(a), np.float64(b)
    if a == b:
        return 0
    return abs(int(np.array(a).view(np.int64)) - int(np.array(b).view(np.int64)))


def test_ln_exp_cossin_accuracy(G):
    rng = np.random.default_rng(5)
    u = np.concatenate([rng.random(20000), [1.0, 0.5, 2.0 ** -53, 1e-300, 0.7071067811865476, 0.7071067811865475]])
    u = u[u > 0]
    worst = max(_ulps(G.sjk_synth_ln(float(x)), math.log(x)) for x in u)
    assert worst <= 4, worst
    x = rng.standard_normal(20000) * 3
    worst = max(_ulps(G.sjk_synth_exp(float(t)), math.exp(t)) for t in x)
    assert worst <= 4, worst
    c, s = C.c_double(), C.c_double()
    worst = 0.0
    for v in np.concatenate([rng.random(20000), [0.0, 0.125, 0.25, 0.5, 0.75, 1.0]]):
        G.sjk_synth_cossin(float(v), C.byref(c), C.byref(s))
        worst = max(worst, abs(c.value - math.cos(2 * math.pi * v)), abs(s.value - math.sin(2 * math.pi * v)))
    assert worst < 1e-15, worst


def test_f16_rounding_matches_numpy(G):
    rng = np.random.default_rng(6)
    x = np.concatenate([rng.standard_normal(50000).astype(np.float32) * np.float32(8),
                        (rng.standard_normal(20000) * 1e-5).astype(np.float32),
                        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 6.1035156e-05, 5.9604645e-08, 2.9802322e-08,
                                  2.9802326e-08, -1.0, 1.0 + 2 ** -11, 1.0 + 3 * 2 ** -11], np.float32)])
    got = np.array([G.sjk_synth_f16(float(v)) for v in x], np.uint16)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


def test_distributions(oracle_lib):
    lib = oracle_lib.lib()
    H, D = 4, 256
    sc = refcache.synth_scales(0, 0, 2, H, D, lib=lib)
    for il in range(2):
        for h in range(H):
            ln = np.log(sc[il, h].astype(np.float64))
            big = np.sort(ln)[-4:]
            # 4 outlier channels x 8 (ln 8 = 2.08 above their LogNormal draw)
            assert len(set(np.argsort(ln)[-4:])) == 4 and big.min() > 0
    k, v = refcache.synth_kv(0, 0, H, D, False, sc[0], 0, 4096, lib=lib)
    assert abs(v.mean()) < 0.01 and abs(v.std() - 1) < 0.01
    x = (k / sc[0][None]).astype(np.float64)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1) < 0.01
    kt, _ = refcache.synth_kv(2, 0, H, D, True, sc[0], 0, 4096, lib=lib)
    t = (kt / sc[0][None]).astype(np.float64).ravel()
    # Student-t(4): variance nu / (nu - 2) = 2, excess kurtosis infinite (heavy tails)
    assert 1.8 < t.var() < 2.3
    assert (np.abs(t) > 6).mean() > 20 * (np.abs(x.ravel()) > 6).mean()
    q = refcache.synth_q(1, 0, 4, 16, D, lib=lib)
    assert np.array_equal(q, q.astype(np.float16).astype(np.float32))
    assert abs(q.std() - 1) < 0.05


def test_position_addressable_and_thread_independent(oracle_lib):
    lib = oracle_lib.lib()
    H, D = 4, 256
    sc = refcache.synth_scales(3, 5, 1, H, D, lib=lib)[0]
    k, v = refcache.synth_kv(3, 5, H, D, True, sc, 1000, 300, n_threads=1, lib=lib)
    k8, v8 = refcache.synth_kv(3, 5, H, D, True, sc, 1000, 300, n_threads=8, lib=lib)
    ka, va = refcache.synth_kv(3, 5, H, D, True, sc, 1000, 77, lib=lib)
    kb, vb = refcache.synth_kv(3, 5, H, D, True, sc, 1077, 223, lib=lib)
    assert np.array_equal(k.view(np.uint32), k8.view(np.uint32)) and np.array_equal(v.view(np.uint32), v8.view(np.uint32))
    assert np.array_equal(k.view(np.uint32), np.concatenate([ka, kb]).view(np.uint32))
    assert np.array_equal(v.view(np.uint32), np.concatenate([va, vb]).view(np.uint32))
    # other layers and seeds draw other values
    k2, _ = refcache.synth_kv(3, 6, H, D, True, sc, 1000, 300, lib=lib)
    assert not np.array_equal(k, k2)


def test_reference_build_draws_the_same(oracle_lib):
    """The compiled reference library carries the same generator: identical bytes to the oracle's."""
    if not refcache.available():
        pytest.skip("oracle/_ref not built")
    R = refcache.ref()
    sc_o = refcache.synth_scales(4, 0, 1, 4, 256, lib=oracle_lib.lib())
    sc_r = refcache.synth_scales(4, 0, 1, 4, 256, lib=R)
    assert np.array_equal(sc_o.view(np.uint32), sc_r.view(np.uint32))
    a = refcache.synth_kv(4, 0, 4, 256, True, sc_o[0], 12345, 64, lib=oracle_lib.lib())
    b = refcache.synth_kv(4, 0, 4, 256, True, sc_r[0], 12345, 64, lib=R)
    assert all(np.array_equal(x.view(np.uint32), y.view(np.uint32)) for x, y in zip(a, b))
