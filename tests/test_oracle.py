"""The CPU oracle against the reference's golden vectors (CPU only, no GPU)."""
import os
import re

import numpy as np
import pytest

import inputs
import seqbuild

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _vector_lines():
    out = []
    for ln in open(os.path.join(GOLDEN, "expected_vectors.txt")):
        m = re.match(r"seal D=(\d+) bk=(\d) bv=(\d) body=(\d) bytes=(\d+) rec=([0-9a-f]+) dec=([0-9a-f]+)", ln)
        if m:
            out.append(tuple(map(int, m.groups()[:5])) + (int(m.group(6), 16), int(m.group(7), 16)))
    return out


_INPUTS = {}


def group_inputs(D):
    if D not in _INPUTS:
        _INPUTS[D] = inputs.fill_group(D, 128, 1)
    return _INPUTS[D]


@pytest.mark.parametrize("D,bk,bv,body,nbytes,erec,edec", _vector_lines())
def test_seal_golden(oracle_lib, D, bk, bv, body, nbytes, erec, edec):
    o = oracle_lib
    K, V = group_inputs(D)
    lay = o.layout(D, bk, bv, body)
    assert lay.bytes == nbytes
    rec = o.seal(lay, K, V)
    assert o.fnv(rec) == erec
    k, v = o.decode(lay, rec)
    h = o.fnv(np.stack([k, v], axis=1))   # row order: K row t, then V row t
    assert h == edec


def test_tq6_golden(oracle_lib):
    o = oracle_lib
    for ln in open(os.path.join(GOLDEN, "expected_vectors.txt")):
        m = re.match(r"tq6 rows=(\d+) n=(\d+) enc=([0-9a-f]+) dec=([0-9a-f]+)", ln)
        if not m:
            continue
        rows, n = int(m.group(1)), int(m.group(2))
        x = inputs.fill_rows(rows, n)
        enc = o.tq6_encode(x)
        dec = o.tq6_decode(enc, rows * n)
        assert o.fnv(enc) == int(m.group(3), 16)
        assert o.fnv(dec) == int(m.group(4), 16)


def test_state_golden(oracle_lib):
    o = oracle_lib
    exp = {}
    for ln in open(os.path.join(GOLDEN, "expected_state.txt")):
        m = re.match(r"state (\S+) v1 hash=([0-9a-f]+)", ln)
        if m:
            exp[m.group(1)] = int(m.group(2), 16)
    assert len(exp) == 5
    for name, bk, bv, tr, st, sf, fc in seqbuild.GOLDEN_CFGS:
        s = seqbuild.OracleSeq(bk, bv, tr, st, sf, fc)
        seqbuild.grow(s, 23, 0, 1500, 4)
        assert o.fnv(s.state()) == exp[name], name
        s.close()


def test_fp16_roundtrip_exhaustive(oracle_lib):
    """Every non-NaN half decodes and re-encodes to itself (reference tests/test_fp16.c:26-33)."""
    o = oracle_lib
    h = np.arange(65536, dtype=np.uint32)
    nan = ((h & 0x7C00) == 0x7C00) & ((h & 0x3FF) != 0)
    bad = 0
    for x in h[~nan][::7]:
        f = o.lib().ora_h2f(int(x))
        bad += o.lib().ora_f2h(f) != int(x)
    assert bad == 0


def test_fp16_rne_sweep(oracle_lib):
    """f32 -> f16 rounds to nearest even over the half range, ties and subnormals included,
    compared with numpy's IEEE conversion (the reference checks the same rule in
    tests/test_fp16.c:34-40)."""
    o = oracle_lib
    i = np.arange(20000, dtype=np.uint64)
    w = (0x33000000 + i * ((0x47800000 - 0x33000000) // 20000) + (i & 0x1FFF)).astype(np.uint32)
    f = w.view(np.float32)
    want = f.astype(np.float16).view(np.uint16)
    got = np.array([o.lib().ora_f2h(float(x)) for x in f], dtype=np.uint16)
    assert np.array_equal(got, want)
    got_neg = np.array([o.lib().ora_f2h(float(-x)) for x in f[::13]], dtype=np.uint16)
    assert np.array_equal(got_neg, (-f[::13]).astype(np.float16).view(np.uint16))
    # NaN, infinities and the overflow threshold
    assert o.lib().ora_f2h(float("nan")) & 0x7FFF == 0x7E00
    assert o.lib().ora_f2h(float("inf")) == 0x7C00
    assert o.lib().ora_f2h(65519.99) == 0x7BFF
    assert o.lib().ora_f2h(65520.0) == 0x7C00


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(__file__), "..", "oracle", "_ref", "libsjref.so")),
                    reason="reference not compiled here")
def test_oracle_matches_compiled_reference_fp16(oracle_lib):
    """Oracle conversion == the compiled reference's sj_kvarn_f32_to_f16 on a dense sweep."""
    import ctypes as C
    import oracle
    r = oracle.ref()
    r.sj_kvarn_f32_to_f16.argtypes = [C.c_float]
    r.sj_kvarn_f32_to_f16.restype = C.c_uint16
    rng = np.random.default_rng(0)
    w = rng.integers(0, 2 ** 32, size=20000, dtype=np.uint64).astype(np.uint32)
    for x in w.view(np.float32):
        assert r.sj_kvarn_f32_to_f16(float(x)) == oracle_lib.lib().ora_f2h(float(x))


def test_window_and_layout_offsets(oracle_lib):
    """Record offsets of the three headline bodies at D=256 (reference README, Formats)."""
    o = oracle_lib
    assert o.layout(256, 4, 4, 0).bytes == 35072
    assert o.layout(256, 3, 3, 1).bytes == 26880
    assert o.layout(256, 3, 2, 1).bytes == 22784
    assert o.layout(256, 2, 2, 1).bytes == 18688


EDGE_BODIES = [(4, 4, 0), (3, 2, 1), (3, 3, 1), (2, 2, 1), (4, 2, 0)]


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(__file__), "..", "oracle", "_ref", "libsjref.so")),
                    reason="reference not compiled here")
@pytest.mark.parametrize("bk,bv,body", EDGE_BODIES)
def test_oracle_seal_edges_match_compiled_reference(oracle_lib, bk, bv, body):
    """Oracle seal == the compiled reference's sj_kvarn_seal_group on edge tiles (signed zeros, fp16 subnormals,
    values near the fp16 maximum, constant and all-zero tiles): pins the oracle where no golden vector reaches."""
    import ctypes as C
    import inputs
    import oracle
    import sjk
    r = oracle.ref()
    lay = sjk.Layout()
    assert r.sj_kvarn_layout_init(C.byref(lay), 256, 128, bk, bv, body) == 0
    r.sjref_seal_batch.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_int,
                                   C.c_void_p, C.c_int]
    ol = oracle_lib.layout(256, bk, bv, body == 1)
    assert ol.bytes == lay.bytes
    for name, k, v in inputs.edge_tiles(256):
        want = np.zeros(lay.bytes, np.uint8)
        r.sjref_seal_batch(C.byref(lay), k.ctypes.data, v.ctypes.data, 256, 1, 1, 16, want.ctypes.data, 1)
        got = oracle_lib.seal(ol, k, v)
        assert np.array_equal(got, want), name


REF_BUILT = os.path.exists(os.path.join(os.path.dirname(__file__), "..", "oracle", "_ref", "libsjref.so"))


def _small_builds(oracle_lib, bits=(4, 4), heavy=False, npos=1500, seed=9, H=2):
    """The same small cache (D 256, sink 128, tail 256 -> 512, ubatch 128) built through the policy in the oracle and
    in the compiled reference, from the seeded generator's rows."""
    import refcache
    D, tail, tail_max, n_ub = 256, 256, 512, 128
    trellis = bits != (4, 4) and bits != (4, 2)
    oc = oracle_lib.OracleCache(D, H, bits[0], bits[1], trellis, 16, 0, True, 128, tail, tail_max, n_ub, npos + 256)
    rl = refcache.RefLayer(D, H, npos + 256, n_ub, bits_k=bits[0], bits_v=bits[1], tail=tail, tail_max=tail_max)
    O = oracle_lib.lib()
    pol = oracle_lib.Policy()
    O.ora_policy_init(pol, 128, tail, tail_max, 128, 0)
    scale = refcache.synth_scales(seed, 0, 1, H, D)[0]
    for pos in range(0, npos, n_ub):
        n = min(n_ub, npos - pos)
        O.ora_policy_begin(pol, pos, n)
        if pol.B_pending > pol.B:
            oc.seal(pol.B, pol.B_pending)
        O.ora_policy_commit(pol)
        rl.begin_ubatch(pos, n, threaded=False)
        k, v = refcache.synth_kv(seed, 0, H, D, heavy, scale, pos, n)
        rl.store(pos, k, v)
        kr, vr = oracle_lib.fwht_rows(k), oracle_lib.fwht_rows(v)
        for i in range(n):
            oc.store(pos + i, kr[i], vr[i])
    assert pol.B == rl.pol.B
    return oc, rl, pol.B


@pytest.mark.skipif(not REF_BUILT, reason="reference not compiled here")
@pytest.mark.parametrize("bits,heavy", [((4, 4), False), ((3, 2), True)])
def test_oracle_cache_and_attend_row_match_compiled_reference(oracle_lib, bits, heavy):
    """A policy-driven build in the oracle equals one through the compiled reference (sink, ring, records), and the
    oracle's attention loop ora_attend_row equals sj_kvarn_layer_attend_row bit for bit over every region."""
    import ctypes as C
    import refcache
    oc, rl, B = _small_builds(oracle_lib, bits, heavy)
    N = 1500
    ng = (B - 128) // 128
    assert np.array_equal(oc.body_bytes(ng), rl.records(0, ng))
    assert np.array_equal(oc.ring_bytes(), rl.ring_bytes())
    assert np.array_equal(oc.sink_bytes(), rl.sink_bytes())
    q = rl.rotate(refcache.synth_q(9, 0, 3, 4, 256))
    out = np.zeros(256, np.float32)
    for iq in range(3):
        for hq in range(4):
            for qpos in (N - 3 + iq, 200, B + 5):
                want = rl.attend_row(B, N, q[iq, hq], hq // 2, qpos, 1.0 / 16)
                oracle_lib.lib().ora_attend_row(C.byref(oc.c), B, N, np.ascontiguousarray(q[iq, hq]), hq // 2, qpos,
                                                1.0 / 16, out)
                assert np.array_equal(out.view(np.uint32), want.view(np.uint32)), (iq, hq, qpos)
    oc.close()
    rl.close()


@pytest.mark.skipif(not REF_BUILT, reason="reference not compiled here")
def test_reference_seal_harness_matches_layer_seal():
    """The threaded harness that the CPU baselines and the configuration tests use (sjref_layer_seal_mt: per record,
    unstage the ring rows, round to fp16, sj_kvarn_seal_group with a per-thread workspace) writes exactly the records
    of the reference's own sj_kvarn_layer_seal."""
    import refcache
    D, H = 256, 4
    for bits, heavy in (((4, 4), False), ((3, 2), True)):
        a = refcache.RefLayer(D, H, 2048, 512, bits_k=bits[0], bits_v=bits[1], tail=512, tail_max=1024)
        b = refcache.RefLayer(D, H, 2048, 512, bits_k=bits[0], bits_v=bits[1], tail=512, tail_max=1024)
        scale = refcache.synth_scales(5, 0, 1, H, D)[0]
        k, v = refcache.synth_kv(5, 0, H, D, heavy, scale, 0, 128 + 3 * 128)
        a.store(0, k, v)
        b.store(0, k, v)
        a.seal(128, 512, threaded=True)
        b.seal(128, 512, threaded=False)
        assert np.array_equal(a.records(0, 3), b.records(0, 3)), bits
        a.close()
        b.close()
