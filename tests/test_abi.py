"""The C-ABI library on the CPU: it loads, exports every symbol include/sjk.h declares, and its host-only
logic (layout, policy, status strings, state-stream validation) matches the oracle. No GPU calls."""
import ctypes as C
import random

import numpy as np
import pytest

import sjk


@pytest.fixture(scope="module")
def L():
    import build
    build.build()
    return sjk.lib()


def test_exports_every_header_symbol(L):
    names = sjk.exported_symbols_in_header()
    assert len(names) > 60
    missing = [n for n in names if not hasattr(L, n)]
    assert missing == []
    # and the binding covers all of them
    assert sorted(set(names) - set(sjk.SIGNATURES)) == []


def test_layout_matches_oracle(L, oracle_lib):
    o = oracle_lib
    for D in (128, 256):
        for bk in (2, 3, 4):
            for bv in (2, 3, 4):
                for body in (0, 1):
                    lay = sjk.Layout()
                    rc = L.sj_kvarn_layout_init(C.byref(lay), D, 128, bk, bv, body)
                    ol = o.Layout()
                    orc = o.lib().ora_layout_init(C.byref(ol), D, 128, bk, bv, body)
                    assert (rc == 0) == (orc == 0)
                    if rc:
                        continue
                    assert lay.bytes == ol.bytes == L.sj_kvarn_record_bytes(D, 128, bk, bv)
                    for t in (0, 5, 17, 127):
                        for d in (0, 3, 16, 31, D - 1):
                            for is_v in (0, 1):
                                assert L.sj_kvarn_code_bit(C.byref(lay), t, d, is_v) == o.lib().ora_code_bit(C.byref(ol), t, d, is_v)
                    for d in range(D):
                        assert L.sj_kvarn_k_ch_idx(C.byref(lay), d) == o.lib().ora_k_ch(C.byref(ol), d)
                        assert L.sj_kvarn_v_ch_idx(C.byref(lay), d) == o.lib().ora_v_ch(C.byref(ol), d)


def test_fp16_host_matches_oracle(L, oracle_lib):
    rng = np.random.default_rng(1)
    w = rng.integers(0, 2 ** 32, size=5000, dtype=np.uint64).astype(np.uint32)
    for x in w.view(np.float32):
        assert L.sj_kvarn_f32_to_f16(float(x)) == oracle_lib.lib().ora_f2h(float(x))
    for h in range(0, 65536, 3):
        a, b = L.sj_kvarn_f16_to_f32(h), oracle_lib.lib().ora_h2f(h)
        assert (a == b) or (a != a and b != b)


def _policy_pair(L, o, sink, tail, tail_max, group, flush):
    p = sjk.Policy()
    q = o.Policy()
    L.sj_kvarn_policy_init(C.byref(p), sink, tail, tail_max, group, flush)
    o.lib().ora_policy_init(C.byref(q), sink, tail, tail_max, group, flush)
    return p, q


def _same(p, q):
    return (p.B, p.B_prev, p.B_pending, p.draining) == (q.B, q.B_prev, q.B_pending, q.draining)


def test_policy_fuzz_against_oracle(L, oracle_lib):
    """Random ubatches / idles / truncations: the library's policy and the oracle's stay identical
    (the reference fuzzes its rule the same way, tests/test_policy.c:31-98)."""
    o = oracle_lib
    rng = random.Random(7)
    for trial in range(40):
        sink = rng.choice([64, 128, 192])
        group = 128
        tail = group * rng.randint(1, 8)
        tail_max = rng.choice([0, tail, tail + 128 * rng.randint(1, 8)])
        flush = rng.choice([0, 0, 1, 2])
        p, q = _policy_pair(L, o, sink, tail, tail_max, group, flush)
        pos = 0
        for step in range(400):
            r = rng.random()
            if r < 0.8:
                n = rng.choice([1, 1, 2, 4, 16, 64, 512])
                a = L.sj_kvarn_policy_begin_ubatch(C.byref(p), pos, n)
                b = o.lib().ora_policy_begin(C.byref(q), pos, n)
                assert a == b
                L.sj_kvarn_policy_commit(C.byref(p)); o.lib().ora_policy_commit(C.byref(q))
                pos += n
            elif r < 0.9:
                keep = rng.choice([0, 10, 300, 5000])
                a = L.sj_kvarn_policy_idle(C.byref(p), pos, keep)
                b = o.lib().ora_policy_idle(C.byref(q), pos, keep)
                assert a == b
                L.sj_kvarn_policy_commit(C.byref(p)); o.lib().ora_policy_commit(C.byref(q))
            else:
                cut = rng.randint(0, pos + 10)
                da, db = C.c_uint32(), C.c_uint32()
                a = L.sj_kvarn_policy_truncate(C.byref(p), cut, C.byref(da))
                b = o.lib().ora_policy_truncate(C.byref(q), cut, C.byref(db))
                assert a == b and da.value == db.value
                if a != 0xFFFFFFFF:
                    pos = min(pos, a)
            assert _same(p, q), (trial, step)


def test_ring_capacity_and_slots(L, oracle_lib):
    for tail, tmax, ub in [(4096, 8192, 512), (256, 512, 64), (4096, 0, 1)]:
        assert L.sj_kvarn_ring_capacity(tail, tmax, 128, ub) == oracle_lib.lib().ora_ring_capacity(tail, tmax, 128, ub)
    assert L.sj_kvarn_ring_capacity(4096, 8192, 128, 512) == 9344
    assert L.sj_kvarn_ring_slot(128, 9344, 128 + 9344 + 5) == 5


def test_strerror_and_config(L):
    assert L.sj_kvarn_strerror(0) == b"ok"
    assert b"checksum" in L.sj_kvarn_strerror(-107)
    assert L.sj_kvarn_strerror(-130) != b"unknown SJ-KVaRN status code"
    c = sjk.config(256, 4, 100000, 512)
    assert (c.bits_k, c.bits_v, c.sink, c.tail, c.tail_max, c.iters, c.group) == (4, 4, 128, 4096, 8192, 16, 128)
    cfg = sjk.config(128, 2, 2304, 64, bits_k=3, bits_v=3, tail=256, tail_max=512)
    assert L.sj_kvarn_state_size_max(C.byref(cfg), 2) > 128


def test_state_peek_rejects_damage_without_gpu(L, oracle_lib):
    """A stream written by the oracle parses with the library's peek; damage is rejected with the
    reference's codes (tests/test_state.c:273-348)."""
    import seqbuild
    s = seqbuild.OracleSeq(3, 3, 1, 0, 1, 1)
    seqbuild.grow(s, 31, 0, 700, 2)
    st = s.state()
    info = sjk.StateInfo()
    buf = C.create_string_buffer(st.tobytes(), len(st))
    assert L.sj_kvarn_state_peek(buf, len(st), C.byref(info)) == 0
    assert info.n == 700 and info.B == s.pol.B and info.n_layers == 2 and info.cfg.body == 1
    bad = bytearray(st.tobytes()); bad[0] = ord("X")
    assert L.sj_kvarn_state_peek(bytes(bad), len(bad), C.byref(info)) == -104
    bad = bytearray(st.tobytes()); bad[8] = 2
    assert L.sj_kvarn_state_peek(bytes(bad), len(bad), C.byref(info)) == -105
    bad = bytearray(st.tobytes()); bad[len(bad) // 2] ^= 0x10
    assert L.sj_kvarn_state_peek(bytes(bad), len(bad), C.byref(info)) == -107
    assert L.sj_kvarn_state_peek(st.tobytes(), len(st) - 1, C.byref(info)) == -103
    assert L.sj_kvarn_state_peek(st.tobytes(), 4, C.byref(info)) == -103
    s.close()


def test_desc_fill_entries_and_checks(L):
    """The descriptor of the descriptor-driven calls: the reference's entry order (INTEGRATION_LLAMACPP.md:54-69),
    values from the view, and the same checks the kernels apply (host-only, no GPU)."""
    v = sjk.View()
    v.lay = sjk.layout(256, 3, 3, 1)
    v.n_head_kv, v.staging, v.sink_type, v.S, v.cap, v.stage_bytes = 4, 0, 0, 128, 1152, 196
    d = sjk.desc_fill(v, 128 + 256, 128 + 512, 900, 899)
    assert list(d) == [128, 1152, 640, 900, 899, 128, 256, v.lay.bytes, 4, 384, 0, 0, 1, 0, 0, 0]
    assert sjk.DESC_B_OLD == 9 and sjk.DESC_SINK_TYPE == 13 and sjk.DESC_N_ENTRIES == 16
    # sink-only, empty ubatch seal
    assert list(sjk.desc_fill(v, 128, 128, 50, 49))[:5] == [128, 1152, 128, 50, 49]
    bad = [(128, 128 + 100, 900, 0),       # B off a group boundary
           (128 + 256, 128, 900, 0),       # B_OLD > B
           (100, 128, 900, 0),             # B_OLD inside the sink
           (128, 64, 100, 0),              # B inside the sink
           (128, 256, 256 + 1153, 0),      # more staged positions than the ring holds
           (128, 256, 2 ** 31, 0)]         # not an int32
    for args in bad:
        with pytest.raises(sjk.SjkError):
            sjk.desc_fill(v, *args)
