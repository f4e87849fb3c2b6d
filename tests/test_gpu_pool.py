"""The paged pool's bookkeeping on the device (sjk_pool_reserve_batch / sjk_pool_release_batch / sjk_truncate_batch)
against the host pool and the per-layer host truncation: the same block tables, the same free-id stack and the same
cache bytes, over seeded random batches (the reference's semantics: sj_kvarn.h:1716-1739 reserve / release,
1581-1603 truncate)."""
import ctypes as C

import numpy as np
import pytest

import gpu_util as gu
import sjk

pytestmark = pytest.mark.gpu

NO_BLOCK = 0xFFFFFFFF
POOL_FULL = -110


@pytest.fixture(scope="module")
def L():
    import build
    build.build()
    import torch
    assert torch.cuda.is_available()
    return sjk.lib()


def _host_reserve(L, pool, tbl, g0, g1):
    """sj_kvarn__seq_reserve on the host pool: NO_BLOCK entries of [g0, g1) take blocks in group order; a request
    that runs out releases what it took (in reverse order) and fails."""
    taken = []
    for g in range(g0, g1):
        if tbl[g] != NO_BLOCK:
            continue
        b = L.sj_kvarn_pool_alloc(C.byref(pool))
        if b == NO_BLOCK:
            for gg in reversed(taken):
                L.sj_kvarn_pool_release(C.byref(pool), int(tbl[gg]))
                tbl[gg] = NO_BLOCK
            return POOL_FULL
        tbl[g] = b
        taken.append(g)
    return 0


def _host_release(L, pool, tbl, g0, g1):
    for g in range(g0, g1):
        L.sj_kvarn_pool_release(C.byref(pool), int(tbl[g]))
        tbl[g] = NO_BLOCK


def _stack(pool):
    return [pool.free_ids[i] for i in range(pool.n_free)]


def test_reserve_release_batches_match_host_pool(L):
    T = gu.torch()
    cfg = sjk.config(n_ctx=8192)
    n_blocks, n_seq, n_grp = 48, 6, 24
    ref, mine = sjk.Pool(), sjk.Pool()                  # driven on the host / loaded into and back from the device
    sjk.check(L.sj_kvarn_pool_init(C.byref(ref), C.byref(cfg), 1, n_blocks))
    sjk.check(L.sj_kvarn_pool_init(C.byref(mine), C.byref(cfg), 1, n_blocks))
    try:
        dpool = T.zeros(int(L.sjk_pool_dev_bytes(n_blocks)), dtype=T.uint8, device="cuda")
        sjk.check(L.sjk_pool_dev_load(gu.ptr(dpool), C.byref(mine), None))
        tables = np.full((n_seq, n_grp), NO_BLOCK, np.uint32)
        dtab = T.from_numpy(tables.view(np.int32).copy()).cuda()
        status = T.zeros(sjk.POOL_MAX_REQ, dtype=T.int32, device="cuda")
        rng = np.random.default_rng(7)
        n_full = 0
        for step in range(40):
            n = int(rng.integers(1, 9))
            reqs = (sjk.BlockReq * n)()
            spans = []
            for i in range(n):
                s = int(rng.integers(0, n_seq))
                g0 = int(rng.integers(0, n_grp))
                g1 = int(rng.integers(g0, n_grp + 1))
                reqs[i].blocks = dtab.data_ptr() + s * n_grp * 4
                reqs[i].g0, reqs[i].g1 = g0, g1
                spans.append((s, g0, g1))
            if step % 3 == 2:                           # every third batch releases
                for s, g0, g1 in spans:
                    _host_release(L, ref, tables[s], g0, g1)
                sjk.check(L.sjk_pool_release_batch(gu.ptr(dpool), reqs, n, None))
            else:
                want = [_host_reserve(L, ref, tables[s], g0, g1) for s, g0, g1 in spans]
                n_full += sum(1 for w in want if w)
                sjk.check(L.sjk_pool_reserve_batch(gu.ptr(dpool), reqs, n, gu.ptr(status), None))
                assert gu.host(status, np.int32)[:n].tolist() == want, step
            got = gu.host(dtab, np.uint32).reshape(n_seq, n_grp)
            assert np.array_equal(got, tables), step
            sjk.check(L.sjk_pool_dev_store(gu.ptr(dpool), C.byref(mine), None))
            assert _stack(mine) == _stack(ref), step
        assert n_full > 0                               # the batches did run the pool dry at times
    finally:
        L.sj_kvarn_pool_free(C.byref(ref))
        L.sj_kvarn_pool_free(C.byref(mine))


def _fill(layer, seed):
    """Random bytes in a layer's sink, ring and (own) body, through the layer's device pointers."""
    T = gu.torch()
    rng = np.random.default_rng(seed)
    H, S, D = layer.cfg.n_head_kv, layer.cfg.sink, layer.cfg.head_dim
    sink_entry = D * 4 if layer.cfg.sink_type == 0 else 2 * layer.stage_bytes   # SJKVARN_SINK_F16 = 0
    sizes = {"sink": S * H * sink_entry, "ring": layer.cap * H * 2 * layer.stage_bytes,
             "body": layer.n_groups * H * layer.lay.bytes}
    bufs = {}
    for name, nbytes in sizes.items():
        a = rng.integers(0, 256, nbytes, dtype=np.uint8)
        bufs[name] = a
        t = T.from_numpy(a).cuda()
        assert gu.cudart().cudaMemcpy(C.c_void_p(getattr(layer, name)), C.c_void_p(t.data_ptr()), nbytes, 3) == 0
    return sizes, sink_entry


def _read(layer, sizes):
    return {name: gu.d2h_ptr(getattr(layer, name), n) for name, n in sizes.items()}


@pytest.mark.parametrize("sink_type", [0, 1])
def test_truncate_batch_matches_layer_truncate(L, sink_type):
    """Several layers truncated in one sjk_truncate_batch equal sj_kvarn_layer_truncate on copies of them, for cuts
    in the body (records dropped), in the ring and in the sink."""
    cfg = sjk.config(n_ctx=8192, sink_type=sink_type)
    cases = [  # (B_old, B_new, n_old, resume)
        (128 + 128 * 20, 128 + 128 * 7, 128 + 128 * 20 + 300, 128 + 128 * 7 + 40),
        (128 + 128 * 12, 128 + 128 * 12, 128 + 128 * 12 + 900, 128 + 128 * 12 + 17),
        (128 + 128 * 5, 128, 128 + 128 * 5 + 64, 60),
        (128 + 128 * 30, 128 + 128 * 29, 128 + 128 * 30 + 5000, 128 + 128 * 29 + 1),
    ]
    mine, ref = [], []
    try:
        for i in range(len(cases)):
            for group in (mine, ref):
                lay = sjk.Layer()
                sjk.check(L.sj_kvarn_layer_init(C.byref(lay), C.byref(cfg)))
                group.append(lay)
        reqs = (sjk.TruncReq * len(cases))()
        for i, (B_old, B_new, n_old, resume) in enumerate(cases):
            sizes, sink_entry = _fill(mine[i], 100 + i)
            _fill(ref[i], 100 + i)
            a = mine[i]
            r = reqs[i]
            r.body, r.sink, r.ring, r.blocks = a.body, a.sink, a.ring, None
            r.S, r.cap, r.n_head_kv, r.group = a.cfg.sink, a.cap, a.cfg.n_head_kv, a.cfg.group
            r.rec_bytes, r.sink_entry_bytes, r.stage_bytes = a.lay.bytes, sink_entry, a.stage_bytes
            r.B_old, r.B_new, r.n_old, r.resume, r.release = B_old, B_new, n_old, resume, 0
            L.sj_kvarn_layer_truncate(C.byref(ref[i]), B_old, B_new, n_old, resume)
        sjk.check(L.sjk_truncate_batch(reqs, len(cases), None, None))
        for i in range(len(cases)):
            got, want = _read(mine[i], sizes), _read(ref[i], sizes)
            for name in sizes:
                assert np.array_equal(got[name], want[name]), (i, name)
        assert L.sjk_device_status() == 0
    finally:
        for lay in mine + ref:
            L.sj_kvarn_layer_free(C.byref(lay))


def test_truncate_batch_pool_release(L):
    """Pool mode: the dropped groups' records are zeroed through the block table (NO_BLOCK entries skipped), the
    blocks go back to the device pool in request order, and the tables read NO_BLOCK - as the host pool's release."""
    T = gu.torch()
    cfg = sjk.config(n_ctx=8192)
    n_blocks, n_grp = 32, 12
    ref, mine = sjk.Pool(), sjk.Pool()
    sjk.check(L.sj_kvarn_pool_init(C.byref(ref), C.byref(cfg), 1, n_blocks))
    sjk.check(L.sj_kvarn_pool_init(C.byref(mine), C.byref(cfg), 1, n_blocks))
    try:
        tables = np.full((2, n_grp), NO_BLOCK, np.uint32)
        for s, g1 in ((0, 10), (1, 12)):
            assert _host_reserve(L, ref, tables[s], 0, g1) == 0
        L.sj_kvarn_pool_release(C.byref(ref), int(tables[1][4]))   # a hole the scrub must skip
        tables[1][4] = NO_BLOCK
        # device pool from the host pool's stack after those reservations
        mine.n_free = ref.n_free
        for i in range(ref.n_free):
            mine.free_ids[i] = ref.free_ids[i]
        dpool = T.zeros(int(L.sjk_pool_dev_bytes(n_blocks)), dtype=T.uint8, device="cuda")
        sjk.check(L.sjk_pool_dev_load(gu.ptr(dpool), C.byref(mine), None))
        dtab = T.from_numpy(tables.view(np.int32).copy()).cuda()
        grp = cfg.n_head_kv * ref.lay.bytes
        body = T.from_numpy(np.random.default_rng(3).integers(1, 256, n_blocks * grp, dtype=np.uint8)).cuda()
        want_body = gu.host(body).copy()
        sink_entry = cfg.head_dim * 4 if cfg.sink_type == 0 else 2 * 196
        sink = T.zeros(cfg.sink * cfg.n_head_kv * sink_entry, dtype=T.uint8, device="cuda")
        ring = T.zeros(8192 * cfg.n_head_kv * 2 * 196, dtype=T.uint8, device="cuda")
        cuts = [(0, 128 + 128 * 10, 128 + 128 * 3), (1, 128 + 128 * 12, 128 + 128 * 2)]
        reqs = (sjk.TruncReq * 2)()
        for i, (s, B_old, B_new) in enumerate(cuts):
            r = reqs[i]
            r.body, r.sink, r.ring, r.blocks = body.data_ptr(), sink.data_ptr(), ring.data_ptr(), dtab.data_ptr() + s * n_grp * 4
            r.S, r.cap, r.n_head_kv, r.group = cfg.sink, 8192, cfg.n_head_kv, cfg.group
            r.rec_bytes, r.sink_entry_bytes, r.stage_bytes = ref.lay.bytes, sink_entry, 196
            r.B_old, r.B_new, r.n_old, r.resume, r.release = B_old, B_new, B_old, B_new, 1
            g0, g1 = (B_new - cfg.sink) // cfg.group, (B_old - cfg.sink) // cfg.group
            for g in range(g0, g1):
                if tables[s][g] != NO_BLOCK:
                    want_body[int(tables[s][g]) * grp:(int(tables[s][g]) + 1) * grp] = 0
            _host_release(L, ref, tables[s], g0, g1)
        sjk.check(L.sjk_truncate_batch(reqs, 2, gu.ptr(dpool), None))
        assert np.array_equal(gu.host(body), want_body)
        assert np.array_equal(gu.host(dtab, np.uint32).reshape(2, n_grp), tables)
        sjk.check(L.sjk_pool_dev_store(gu.ptr(dpool), C.byref(mine), None))
        assert _stack(mine) == _stack(ref)
    finally:
        L.sj_kvarn_pool_free(C.byref(ref))
        L.sj_kvarn_pool_free(C.byref(mine))
