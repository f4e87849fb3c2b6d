"""Descriptor-driven calls (sjk_seal_dyn, sjk_store_dyn, sjk_attend_dyn) through the C-ABI: the reference's ggml op
boundary, whose seal and region-aware attention read an I32 descriptor at run time so one captured graph serves
every decode step (INTEGRATION_LLAMACPP.md:44-74 of the reference).

- sjk_attend_dyn plans on the device with the host path's own plan functions, so for the same (B, N, qpos0) its
  output equals sjk_attend's bit for bit, for every kernel family (trellis and 4-bit tensor-core bodies, the dense
  staged-row kernel, the CUDA-core kernel for D = 128 and for 4/2 bodies) and for prefix queries and sink-only caches.
- A decode loop replayed from ONE CUDA graph (seal, store and attention, only the descriptor and the step's rows
  changing) builds the same cache bytes and the same outputs as the host-planned sequence API, across seals.
- A descriptor that does not fit the cache makes every call write nothing (attention: zeros) and is reported
  through sjk_device_status()."""
import ctypes as C

import numpy as np
import pytest

import gpu_util as gu
import sjk

pytestmark = pytest.mark.gpu

H, TAIL, TAIL_MAX, N_UB = 2, 256, 512, 64


@pytest.fixture(scope="module")
def L():
    import build
    build.build()
    import torch
    assert torch.cuda.is_available()
    return sjk.lib()


def _grow(dseq, n, seed, D):
    rng = np.random.default_rng(seed)
    pos = 0
    while pos < n:
        m = min(1 + (pos * 5) % N_UB, n - pos)
        assert dseq.begin_ubatch(pos, m) == 0
        k = rng.standard_normal((m, H * D)).astype(np.float32)
        v = rng.standard_normal((m, H * D)).astype(np.float32)
        k[:, :D] *= 2.0
        for j in range(m):
            dseq.store(pos + j, k[j], v[j])
        pos += m
    gu.torch().cuda.synchronize()


def _attend_both(L, view, B, N, qpos0, n_q, n_head, D, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n_q, n_head, D)).astype(np.float32)
    dq = gu.dev(q)
    o1, o2 = gu.dev_zeros(q.nbytes), gu.dev_zeros(q.nbytes)
    need = L.sjk_attend_scratch_bytes(C.byref(view), N, n_q, n_head)
    s1 = gu.dev_zeros(need)
    scale = np.float32(1.0 / np.sqrt(D))
    sjk.check(L.sjk_attend(C.byref(view), B, N, qpos0, n_q, n_head, gu.ptr(dq), scale, gu.ptr(o1), gu.ptr(s1), need, None), "attend")
    need2 = L.sjk_attend_dyn_scratch_bytes(C.byref(view), n_q, n_head)
    s2 = gu.dev_zeros(need2)
    desc = gu.dev(sjk.desc_fill(view, B, B, N, qpos0))
    sjk.check(L.sjk_attend_dyn(C.byref(view), gu.ptr(desc), n_q, n_head, gu.ptr(dq), scale, gu.ptr(o2), gu.ptr(s2), need2, None),
              "attend_dyn")
    return gu.host(o1, np.float32, q.shape), gu.host(o2, np.float32, q.shape)


# (D, bits_k, bits_v, body, staging, sink_type): trellis / 4-bit tensor-core bodies with the dense kernel, fp16
# staging with an inherited sink, a 4/2 scalar body (CUDA-core body, dense staged rows), D = 128 (CUDA-core only)
FORMATS = [(256, 3, 3, 1, 0, 0), (256, 3, 2, 1, 0, 0), (256, 4, 4, 0, 0, 0), (256, 3, 3, 1, 1, 1), (256, 4, 2, 0, 0, 0),
           (128, 4, 4, 0, 0, 0)]


@pytest.mark.parametrize("D,bk,bv,body,staging,sink_type", FORMATS)
def test_attend_dyn_equals_attend(L, D, bk, bv, body, staging, sink_type):
    cfg = sjk.config(D, H, 4096, N_UB, bits_k=bk, bits_v=bv, body=body, staging=staging, sink_type=sink_type, tail=TAIL,
                     tail_max=TAIL_MAX)
    s = gu.DevSeq(cfg, 1)
    try:
        _grow(s, 1700, 5 + bk + 10 * bv + staging, D)
        view = sjk.View()
        L.sjk_layer_view(C.byref(s.s.layers[0]), C.byref(view))
        B, n = s.pol.B, s.n
        assert B > 128 + 4 * 128 and n > B
        cases = [(B, n, n - 1, 1, 8), (B, n, n - 4, 4, 4), (B, n, n - 2, 2, 2),
                 (B, B - 50, B - 52, 2, 8),          # a prefix that ends inside a record
                 (B, B - 128, B - 129, 1, 8),        # a prefix on a record boundary
                 (128, 100, 99, 1, 8),               # inside the sink only
                 (B, n, 0, 1, 2)]                    # one early query row: causal mask cuts most of the cache
        for i, (b, N, q0, n_q, n_head) in enumerate(cases):
            o1, o2 = _attend_both(L, view, b, N, q0, n_q, n_head, D, 100 + i)
            assert np.array_equal(o1, o2), (i, b, N, q0, n_q, n_head, float(np.abs(o1 - o2).max()))
            assert np.abs(o1).max() > 0
        assert L.sjk_device_status() == 0
    finally:
        s.close()


def test_graph_replay_decode(L):
    """One CUDA graph of a decode step (seal_dyn, store_dyn, attend_dyn), replayed for 1700 steps from position 0 with
    only the descriptor and the step's rows changing, against the host-planned sequence API on the same rows."""
    T = gu.torch()
    D, n_head, steps = 256, 8, 1700
    cfg = sjk.config(D, H, 2048, 1, bits_k=3, bits_v=3, body=1, tail=TAIL, tail_max=TAIL_MAX)
    a = gu.DevSeq(cfg, 1)                                      # reference: the sequence API, planned on the host
    g_layer = sjk.Layer()
    sjk.check(L.sj_kvarn_layer_init(C.byref(g_layer), C.byref(cfg)), "layer_init")
    pol = sjk.Policy()
    L.sj_kvarn_policy_init(C.byref(pol), cfg.sink, cfg.tail, cfg.tail_max, cfg.group, cfg.flush_chunk)
    try:
        vg, va = sjk.View(), sjk.View()
        L.sjk_layer_view(C.byref(g_layer), C.byref(vg))
        L.sjk_layer_view(C.byref(a.s.layers[0]), C.byref(va))
        st = T.cuda.Stream()
        desc = T.zeros(sjk.DESC_N_ENTRIES, dtype=T.int32, device="cuda")
        kb = T.zeros(H * D, dtype=T.float32, device="cuda")
        vb = T.zeros(H * D, dtype=T.float32, device="cuda")
        qb = T.zeros(n_head * D, dtype=T.float32, device="cuda")
        ob = T.zeros(n_head * D, dtype=T.float32, device="cuda")
        need = L.sjk_attend_dyn_scratch_bytes(C.byref(vg), 1, n_head)
        scratch = T.zeros(need, dtype=T.uint8, device="cuda")
        scale = np.float32(1.0 / 16.0)
        p = lambda t: C.c_void_p(t.data_ptr())

        def step_calls():
            sjk.check(L.sjk_seal_dyn(C.byref(vg), p(desc), 4, cfg.iters, C.c_void_p(st.cuda_stream)), "seal_dyn")
            sjk.check(L.sjk_store_dyn(C.byref(vg), p(desc), 1, p(kb), p(vb), 0, C.c_void_p(st.cuda_stream)), "store_dyn")
            sjk.check(L.sjk_attend_dyn(C.byref(vg), p(desc), 1, n_head, p(qb), scale, p(ob), p(scratch), need,
                                       C.c_void_p(st.cuda_stream)), "attend_dyn")

        rng = np.random.default_rng(77)
        graph = None
        seals = 0
        sa = gu.dev_zeros(L.sjk_attend_scratch_bytes(C.byref(va), steps, 1, n_head))
        oa = gu.dev_zeros(n_head * D * 4)
        for pos in range(steps):
            k = rng.standard_normal(H * D).astype(np.float32)
            v = rng.standard_normal(H * D).astype(np.float32)
            q = rng.standard_normal(n_head * D).astype(np.float32)
            # host-planned reference step
            assert a.begin_ubatch(pos, 1) == 0
            a.store(pos, k, v)
            dq = gu.dev(q)
            sjk.check(L.sjk_attend(C.byref(va), a.pol.B, pos + 1, pos, 1, n_head, gu.ptr(dq), scale, gu.ptr(oa), gu.ptr(sa),
                                   sa.numel(), None), "attend")
            # descriptor step: the host runs only the policy and writes the descriptor and the rows
            B_old = pol.B
            L.sj_kvarn_policy_begin_ubatch(C.byref(pol), pos, 1)
            seals += pol.B_pending > B_old
            d = sjk.desc_fill(vg, B_old, pol.B_pending, pos + 1, pos)
            with T.cuda.stream(st):
                desc.copy_(T.from_numpy(d))
                kb.copy_(T.from_numpy(k)); vb.copy_(T.from_numpy(v)); qb.copy_(T.from_numpy(q))
                if pos == 0:
                    step_calls()                               # first step eagerly (also warms the launches up)
                    graph = T.cuda.CUDAGraph()
                    with T.cuda.graph(graph, stream=st, capture_error_mode="relaxed"):
                        step_calls()
                else:
                    graph.replay()
            L.sj_kvarn_policy_commit(C.byref(pol))
            T.cuda.synchronize()
            assert pol.B == a.pol.B
            got, want = ob.cpu().numpy(), gu.host(oa, np.float32)
            assert np.array_equal(got, want), (pos, float(np.abs(got - want).max()))
        assert seals >= 3
        # the same cache bytes: records of [S, B) and the ring
        grp = H * vg.lay.bytes
        n_rec = (pol.B - cfg.sink) // 128
        assert np.array_equal(gu.d2h_ptr(vg.body, n_rec * grp), gu.d2h_ptr(va.body, n_rec * grp))
        ring_bytes = vg.cap * H * 2 * vg.stage_bytes
        assert np.array_equal(gu.d2h_ptr(vg.ring, ring_bytes), gu.d2h_ptr(va.ring, ring_bytes))
        sink_bytes = cfg.sink * H * 2 * D * 2
        assert np.array_equal(gu.d2h_ptr(vg.sink, sink_bytes), gu.d2h_ptr(va.sink, sink_bytes))
        del graph
        assert L.sjk_device_status() == 0
    finally:
        a.close()
        L.sj_kvarn_layer_free(C.byref(g_layer))


def test_bad_descriptor_writes_nothing(L):
    T = gu.torch()
    D, n_head = 256, 8
    cfg = sjk.config(D, H, 2048, N_UB, bits_k=3, bits_v=3, body=1, tail=TAIL, tail_max=TAIL_MAX)
    s = gu.DevSeq(cfg, 1)
    try:
        _grow(s, 900, 3, D)
        view = sjk.View()
        L.sjk_layer_view(C.byref(s.s.layers[0]), C.byref(view))
        assert L.sjk_device_status() == 0
        good = sjk.desc_fill(view, s.pol.B, s.pol.B, s.n, s.n - 1)
        ring_bytes = view.cap * H * 2 * view.stage_bytes
        ring0 = gu.d2h_ptr(view.ring, ring_bytes)
        body0 = gu.d2h_ptr(view.body, 2 * H * view.lay.bytes)
        for entry, value in [(sjk.DESC_S, 64), (sjk.DESC_HKV, 4), (sjk.DESC_B, s.pol.B + 5), (sjk.DESC_TYPE_K, 1),
                             (sjk.DESC_N, s.pol.B + view.cap + 1)]:
            d = good.copy()
            d[entry] = value
            dd = gu.dev(d)
            q = gu.dev(np.ones((n_head, D), np.float32))
            out = gu.dev(np.full((n_head, D), np.nan, np.float32))
            k = gu.dev(np.ones((H, D), np.float32))
            need = L.sjk_attend_dyn_scratch_bytes(C.byref(view), 1, n_head)
            scratch = gu.dev_zeros(need)
            sjk.check(L.sjk_store_dyn(C.byref(view), gu.ptr(dd), 1, gu.ptr(k), gu.ptr(k), 0, None))
            sjk.check(L.sjk_seal_dyn(C.byref(view), gu.ptr(dd), 4, cfg.iters, None))
            sjk.check(L.sjk_attend_dyn(C.byref(view), gu.ptr(dd), 1, n_head, gu.ptr(q), np.float32(0.0625), gu.ptr(out),
                                       gu.ptr(scratch), need, None))
            assert not gu.host(out, np.float32).any(), entry
            assert L.sjk_device_status() == sjk.DEVICE_DESC, entry
            assert np.array_equal(gu.d2h_ptr(view.ring, ring_bytes), ring0)
            assert np.array_equal(gu.d2h_ptr(view.body, 2 * H * view.lay.bytes), body0)
        T.cuda.synchronize()
    finally:
        s.close()


@pytest.mark.parametrize("bk,bv,body", [(3, 2, 1), (4, 4, 0)])
def test_dyn_calls_against_oracle(L, oracle_lib, bk, bv, body):
    """The descriptor-driven calls checked directly against the oracle (not only against the host-planned product
    path): a cache written by sjk_store_dyn and sealed by sjk_seal_dyn, one descriptor per ubatch, holds the oracle's
    sink, ring and record bytes, and sjk_attend_dyn matches the oracle's attention loop (sj_kvarn.h:1535-1564)."""
    import refcache
    D, n_ub, npos, n_q, n_head = 256, 64, 1700, 2, 8
    cfg = sjk.config(D, H, 2048, n_ub, bits_k=bk, bits_v=bv, body=body, tail=TAIL, tail_max=TAIL_MAX)
    layer = sjk.Layer()
    sjk.check(L.sj_kvarn_layer_init(C.byref(layer), C.byref(cfg)), "layer_init")
    trellis = L.sj_kvarn_body_resolve(body, bk, bv) == 1
    oc = oracle_lib.OracleCache(D, H, bk, bv, trellis, 16, 0, True, 128, TAIL, TAIL_MAX, n_ub, 2048)
    pol = sjk.Policy()
    L.sj_kvarn_policy_init(C.byref(pol), 128, TAIL, TAIL_MAX, 128, 0)
    view = sjk.View()
    L.sjk_layer_view(C.byref(layer), C.byref(view))
    O = oracle_lib.lib()
    scale_kv = refcache.synth_scales(21, 0, 1, H, D, lib=O)[0]
    try:
        for pos in range(0, npos, n_ub):
            n = min(n_ub, npos - pos)
            L.sj_kvarn_policy_begin_ubatch(C.byref(pol), pos, n)
            desc = gu.dev(sjk.desc_fill(view, pol.B, pol.B_pending, pos + n, pos))
            sjk.check(L.sjk_seal_dyn(C.byref(view), gu.ptr(desc), 16, 16, None), "seal_dyn")
            if pol.B_pending > pol.B:
                oc.seal(pol.B, pol.B_pending)
            L.sj_kvarn_policy_commit(C.byref(pol))
            k, v = refcache.synth_kv(21, 0, H, D, False, scale_kv, pos, n, lib=O)
            dk, dv = gu.dev(k), gu.dev(v)
            sjk.check(L.sjk_store_dyn(C.byref(view), gu.ptr(desc), n, gu.ptr(dk), gu.ptr(dv), 1, None), "store_dyn")
            kr, vr = oracle_lib.fwht_rows(k), oracle_lib.fwht_rows(v)
            for i in range(n):
                oc.store(pos + i, kr[i].ravel(), vr[i].ravel())
            gu.torch().cuda.synchronize()
        B = pol.B
        ng = (B - 128) // 128
        assert ng >= 8
        assert np.array_equal(gu.d2h_ptr(layer.body, ng * H * layer.lay.bytes), oc.body_bytes(ng)), "records"
        assert np.array_equal(gu.d2h_ptr(layer.ring, layer.cap * H * 2 * layer.stage_bytes), oc.ring_bytes()), "ring"
        q = oracle_lib.fwht_rows(np.random.default_rng(22).standard_normal((n_q, n_head, D)).astype(np.float32))
        dq = gu.dev(q)
        out = gu.dev_zeros(q.nbytes)
        need = L.sjk_attend_dyn_scratch_bytes(C.byref(view), n_q, n_head)
        scratch = gu.dev_zeros(need)
        desc = gu.dev(sjk.desc_fill(view, B, B, npos, npos - n_q))
        sjk.check(L.sjk_attend_dyn(C.byref(view), gu.ptr(desc), n_q, n_head, gu.ptr(dq), np.float32(1 / 16), gu.ptr(out),
                                   gu.ptr(scratch), need, None), "attend_dyn")
        ref = oc.attend(B, npos, npos - n_q, q, 1.0 / 16)
        err = gu.rel_err_rows(gu.host(out, np.float32, q.shape), ref)
        assert err <= 1e-4, err
        assert L.sjk_device_status() == 0
    finally:
        L.sj_kvarn_layer_free(C.byref(layer))
        oc.close()
