"""Batched attention over a paged record pool (sjk_attend_batch) through the C-ABI.

Several sequences share one pool (interleaved block ids) and are built with the product's sequence API through the
adaptive-tail policy; the same rotated rows build oracle caches through the oracle's policy. One batched call per
layer must equal, per sequence, the oracle's attention loop (the reference's sj_kvarn_layer_attend_row restated,
sj_kvarn.h:1535-1564) within the tensor-core bound, and the per-sequence sjk_attend of the same cache. The cases
cover a sequence that ends inside the sink (no body), a query over a prefix that ends inside a record, ring tails
that wrapped, decode widths 1 and 4, and the per-sequence route taken by scalar bodies."""
import ctypes as C

import numpy as np
import pytest

import gpu_util as gu
import seqbuild
import sjk

pytestmark = pytest.mark.gpu

ATTN_TOL_TIGHT = 1e-4
D, H, TAIL, TAIL_MAX, N_UB, N_CTX = 256, 2, 256, 512, 64, 3000
LENGTHS = [100, 700, 1500, 2100, 1190]          # sequence lengths (positions stored)


@pytest.fixture(scope="module")
def L():
    import build
    build.build()
    import torch
    assert torch.cuda.is_available()
    return sjk.lib()


def _rows(rng, n):
    x = rng.standard_normal((n, H * D)).astype(np.float32)
    x[:, :D] *= 2.0
    return x


def _build(L, oracle_lib, bk, bv, body, seed):
    cfg = sjk.config(D, H, N_CTX, N_UB, bits_k=bk, bits_v=bv, body=body, tail=TAIL, tail_max=TAIL_MAX)
    pool = sjk.Pool()
    n_blocks = sum((n + 127) // 128 for n in LENGTHS) + 8
    sjk.check(L.sj_kvarn_pool_init(C.byref(pool), C.byref(cfg), 1, n_blocks), "pool_init")
    L.sj_kvarn_pool_alloc(C.byref(pool))                      # shift the block ids
    devs, oras = [], []
    for n in LENGTHS:
        devs.append(gu.DevSeq(cfg, 1, pool))
        oras.append(seqbuild.OracleSeq(bk, bv, 1 if body == 1 else 0, d=D, h=H, nl=1, tail=TAIL, tail_max=TAIL_MAX,
                                       n_ubatch=N_UB, n_ctx=N_CTX))
    rng = np.random.default_rng(seed)
    # grow the sequences interleaved, so their pool blocks interleave too
    pos = [0] * len(LENGTHS)
    while any(p < n for p, n in zip(pos, LENGTHS)):
        for i, n in enumerate(LENGTHS):
            if pos[i] >= n:
                continue
            m = min(1 + (pos[i] * 7 + i) % N_UB, n - pos[i])
            for s in (devs[i], oras[i]):
                assert s.begin_ubatch(pos[i], m) == 0
            k, v = _rows(rng, m), _rows(rng, m)
            for j in range(m):
                devs[i].store(pos[i] + j, k[j], v[j])
                oras[i].store(pos[i] + j, k[j], v[j])
            pos[i] += m
    gu.torch().cuda.synchronize()
    for d, o in zip(devs, oras):
        assert d.pol.B == o.pol.B
    return pool, devs, oras


def _attend_case(L, devs, oras, n_q, n_head, prefix_cut, seed):
    n_seq = len(devs)
    views = (sjk.View * n_seq)()
    Bs, Ns, Qs = (C.c_uint32 * n_seq)(), (C.c_uint32 * n_seq)(), (C.c_uint32 * n_seq)()
    for i, d in enumerate(devs):
        L.sjk_layer_view(C.byref(d.s.layers[0]), C.byref(views[i]))
        B, N = d.pol.B, d.n
        if prefix_cut and B > 128 + 200:
            N = B - 50                                        # a query over a prefix that ends inside a record
        Bs[i], Ns[i], Qs[i] = B, N, N - n_q
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n_seq, n_q, n_head, D)).astype(np.float32)
    dq, dout = gu.dev(q), gu.dev_zeros(q.nbytes)
    scale = np.float32(1.0 / 16.0)
    need = L.sjk_attend_batch_scratch_bytes(C.byref(views[0]), n_seq, n_q, n_head)
    scratch = gu.dev_zeros(need)
    sjk.check(L.sjk_attend_batch(views, Bs, Ns, Qs, n_seq, n_q, n_head, gu.ptr(dq), scale, gu.ptr(dout), gu.ptr(scratch),
                                 need, None), "attend_batch")
    out = gu.host(dout, np.float32, q.shape)
    # the same call twice gives the same bytes (no state carried between calls)
    sjk.check(L.sjk_attend_batch(views, Bs, Ns, Qs, n_seq, n_q, n_head, gu.ptr(dq), scale, gu.ptr(dout), gu.ptr(scratch),
                                 need, None), "attend_batch")
    assert np.array_equal(gu.host(dout, np.float32, q.shape), out)
    one_need = L.sjk_attend_scratch_bytes(C.byref(views[0]), 0, n_q, n_head)
    one_scratch = gu.dev_zeros(one_need)
    for i in range(n_seq):
        ref = oras[i].layers[0]
        ora = np.zeros((n_q, n_head, D), np.float32)
        import oracle
        oracle.lib().ora_attend(C.byref(ref), Bs[i], Ns[i], Qs[i], n_q, n_head, np.ascontiguousarray(q[i]).reshape(-1), scale,
                                ora.reshape(-1), 0)
        err = gu.rel_err_rows(out[i], ora)
        assert err <= ATTN_TOL_TIGHT, (i, Bs[i], Ns[i], n_q, n_head, err)
        dq1, do1 = gu.dev(q[i]), gu.dev_zeros(q[i].nbytes)
        sjk.check(L.sjk_attend(C.byref(views[i]), Bs[i], Ns[i], Qs[i], n_q, n_head, gu.ptr(dq1), scale, gu.ptr(do1),
                               gu.ptr(one_scratch), one_need, None), "attend")
        assert gu.rel_err_rows(out[i], gu.host(do1, np.float32, (n_q, n_head, D))) <= 1e-5, i
    assert L.sjk_device_status() == 0


@pytest.mark.parametrize("bk,bv,body", [(3, 3, 1), (3, 2, 1), (4, 4, 0)])
def test_attend_batch_pool(L, oracle_lib, bk, bv, body):
    pool, devs, oras = _build(L, oracle_lib, bk, bv, body, seed=31 + bk * 10 + bv)
    try:
        assert devs[0].n < 128 and devs[0].pol.B == 128      # a sequence inside its sink: no body records
        for n_q, n_head, cut, seed in [(1, 8, False, 1), (4, 8, False, 2), (4, 4, True, 3), (2, 2, False, 4)]:
            _attend_case(L, devs, oras, n_q, n_head, cut, seed)
    finally:
        for d in devs:
            d.close()
        for o in oras:
            o.close()
        L.sj_kvarn_pool_free(C.byref(pool))


def test_attend_batch_rejects_mixed_formats(L):
    """Views of different formats in one call are rejected before anything is launched."""
    a = sjk.config(D, H, 1024, 64, bits_k=3, bits_v=3, body=1, tail=TAIL, tail_max=TAIL_MAX)
    b = sjk.config(D, H, 1024, 64, bits_k=3, bits_v=2, body=1, tail=TAIL, tail_max=TAIL_MAX)
    la, lb = sjk.Layer(), sjk.Layer()
    sjk.check(L.sj_kvarn_layer_init(C.byref(la), C.byref(a)))
    sjk.check(L.sj_kvarn_layer_init(C.byref(lb), C.byref(b)))
    views = (sjk.View * 2)()
    L.sjk_layer_view(C.byref(la), C.byref(views[0]))
    L.sjk_layer_view(C.byref(lb), C.byref(views[1]))
    Bs, Ns, Qs = (C.c_uint32 * 2)(128, 128), (C.c_uint32 * 2)(200, 200), (C.c_uint32 * 2)(199, 199)
    q = gu.dev_zeros(2 * 8 * D * 4)
    out = gu.dev_zeros(2 * 8 * D * 4)
    need = L.sjk_attend_batch_scratch_bytes(C.byref(views[0]), 2, 1, 8)
    scratch = gu.dev_zeros(need)
    rc = L.sjk_attend_batch(views, Bs, Ns, Qs, 2, 1, 8, gu.ptr(q), 0.0625, gu.ptr(out), gu.ptr(scratch), need, None)
    assert rc == -100                                         # SJKVARN_ERR_ARG
    L.sj_kvarn_layer_free(C.byref(la))
    L.sj_kvarn_layer_free(C.byref(lb))


def test_store_batch_matches_store(L):
    """sjk_store_batch (one position in each of many caches, one launch) writes the same sink and ring bytes as one
    sjk_store call per item; positions in the sink, in the ring and past a ring wrap."""
    T = gu.torch()
    cfg = sjk.config(D, 4, 4096, 64, bits_k=3, bits_v=3, body=1, tail=TAIL, tail_max=TAIL_MAX)
    a = [sjk.Layer() for _ in range(3)]
    b = [sjk.Layer() for _ in range(3)]
    for lay in a + b:
        sjk.check(L.sj_kvarn_layer_init(C.byref(lay), C.byref(cfg)))
    va, vb = (sjk.View * 9)(), (sjk.View * 9)()
    pos = [0, 5, 127, 128, 300, 301, 127 + a[0].cap, 128 + 2 * a[0].cap + 7, 1000]
    layer_of = [0, 1, 2, 0, 1, 2, 0, 1, 2]
    for i, il in enumerate(layer_of):
        L.sjk_layer_view(C.byref(a[il]), C.byref(va[i]))
        L.sjk_layer_view(C.byref(b[il]), C.byref(vb[i]))
    rng = np.random.default_rng(7)
    k = rng.standard_normal((9, 4, D)).astype(np.float32) * 3
    v = rng.standard_normal((9, 4, D)).astype(np.float32)
    dk, dv = gu.dev(k), gu.dev(v)
    for rotate in (0, 1):
        for i in range(9):
            sjk.check(L.sjk_store(C.byref(va[i]), C.c_void_p(va[i].sink), C.c_void_p(va[i].ring), pos[i], 1,
                                  C.c_void_p(dk.data_ptr() + i * 4 * D * 4), C.c_void_p(dv.data_ptr() + i * 4 * D * 4), rotate,
                                  None))
        sjk.check(L.sjk_store_batch(vb, (C.c_uint32 * 9)(*pos), 9, gu.ptr(dk), gu.ptr(dv), rotate, None))
        T.cuda.synchronize()
        for il in range(3):
            for attr, n in (("ring", a[il].cap * 4 * 2 * a[il].stage_bytes), ("sink", 128 * 4 * D * 4)):
                assert np.array_equal(gu.d2h_ptr(getattr(a[il], attr), n), gu.d2h_ptr(getattr(b[il], attr), n)), (rotate, il, attr)
    for lay in a + b:
        L.sj_kvarn_layer_free(C.byref(lay))


def test_seq_store_prefill_matches_per_position(L):
    """sjk_seq_store (n positions of every layer per call) builds the same sequence state as sj_kvarn_seq_store
    per position, through the same policy decisions."""
    nl = 2
    cfg = sjk.config(D, H, 2048, 64, bits_k=3, bits_v=2, body=1, tail=TAIL, tail_max=TAIL_MAX)
    a, b = gu.DevSeq(cfg, nl), gu.DevSeq(cfg, nl)
    rng = np.random.default_rng(9)
    pos = 0
    T = gu.torch()
    while pos < 1300:
        m = min(64, 1300 - pos)
        k = rng.standard_normal((m, nl, H * D)).astype(np.float32)
        v = rng.standard_normal((m, nl, H * D)).astype(np.float32)
        assert a.begin_ubatch(pos, m) == 0 and b.begin_ubatch(pos, m) == 0
        for j in range(m):
            a.store(pos + j, k[j].reshape(-1), v[j].reshape(-1))
        kb = T.from_numpy(np.ascontiguousarray(k.transpose(1, 0, 2))).cuda()       # [n_layers][n_pos][H D]
        vb = T.from_numpy(np.ascontiguousarray(v.transpose(1, 0, 2))).cuda()
        sjk.check(L.sjk_seq_store(C.byref(b.s), pos, m, C.c_void_p(kb.data_ptr()), C.c_void_p(vb.data_ptr()), 0, 0, None))
        T.cuda.synchronize()
        pos += m
    assert a.n == b.n == 1300
    assert np.array_equal(a.state(), b.state())
    a.close()
    b.close()


@pytest.mark.parametrize("bk,bv,body", [(3, 3, 1), (4, 4, 0)])
def test_state_pool_interleaved(L, oracle_lib, bk, bv, body):
    """Sequences whose pool blocks interleave: their state streams (records gathered on the device, one copy per
    layer) equal the oracle's contiguous caches byte for byte; a truncation zeroes exactly the dropped blocks (one
    scrub launch through the block table, sj_kvarn.h:1581-1603); a stream restored into the scattered blocks the
    truncation freed (scatter on the device) writes back identically and attends like the original."""
    pool, devs, oras = _build(L, oracle_lib, bk, bv, body, seed=57 + bk)
    extra = []
    try:
        states = [d.state() for d in devs]
        for i, (st, o) in enumerate(zip(states, oras)):
            assert np.array_equal(st, o.state()), i
        # the long sequence's blocks are interleaved with the others': more than one run of consecutive ids
        d3 = devs[3]
        n_rec = (d3.pol.B - 128) // 128
        ids = [d3.s.blocks[g] for g in range(n_rec)]
        assert sum(ids[g] != ids[g - 1] + 1 for g in range(1, n_rec)) > 1
        grp = H * pool.lay.bytes
        layer0 = lambda: gu.d2h_ptr(pool.body, pool.n_blocks * grp).reshape(pool.n_blocks, grp)
        before = layer0()
        cut = 128 + 3 * 128 + 40
        r = d3.truncate(cut)
        assert r == 128 + 3 * 128
        dropped = ids[3:]
        after = layer0()
        assert not after[dropped].any()
        keep = [b for b in range(pool.n_blocks) if b not in dropped]
        assert np.array_equal(after[keep], before[keep])
        # restore sequence 2 into the freed blocks (popped in reverse: descending ids)
        r2 = gu.DevSeq(devs[2].cfg, 1, pool)
        extra.append(r2)
        assert r2.read_state(states[2]) == 0
        ids2 = [r2.s.blocks[g] for g in range((r2.pol.B - 128) // 128)]
        assert sum(ids2[g] != ids2[g - 1] + 1 for g in range(1, len(ids2))) > 1
        assert np.array_equal(r2.state(), states[2])
        _attend_case(L, [r2], [oras[2]], 2, 4, False, 9)
    finally:
        for d in devs + extra:
            d.close()
        for o in oras:
            o.close()
        L.sj_kvarn_pool_free(C.byref(pool))
