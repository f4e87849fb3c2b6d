"""sjk_attend_static - attention for callers that cannot allocate device memory (code running where
cudaMalloc is off limits: inside a stream capture, inside a custom allocator's callbacks, or in an engine
whose device memory is planned ahead). Its scratch is a fixed device array inside the library.

Checked through the C-ABI against sjk_attend with a caller-provided scratch buffer, on two calls in a row,
with the attention tolerance of the other GPU tests. Kept in its own file that pytest collects last."""
import ctypes as C

import numpy as np
import pytest

import gpu_util as gu
import sjk
import synth

pytestmark = pytest.mark.gpu
ATTN_TOL_TIGHT = 1e-4


def test_attend_static_matches_attend():
    import build
    import torch
    build.build()
    L = sjk.lib()
    D, H, npos, tail, tail_max, n_ub = 256, 4, 1536, 256, 512, 128
    cfg = sjk.config(D, H, 4096, n_ub, tail=tail, tail_max=tail_max)
    layer = sjk.Layer()
    sjk.check(L.sj_kvarn_layer_init(C.byref(layer), C.byref(cfg)), "layer_init")
    pol = sjk.Policy()
    L.sj_kvarn_policy_init(C.byref(pol), 128, tail, tail_max, 128, 0)
    st = synth.KVStream(3, 1, H, D)
    for pos in range(0, npos, n_ub):
        L.sj_kvarn_policy_begin_ubatch(C.byref(pol), pos, n_ub)
        if pol.B_pending > pol.B:
            sjk.check(L.sjk_layer_seal(C.byref(layer), pol.B, pol.B_pending, None), "seal")
        L.sj_kvarn_policy_commit(C.byref(pol))
        k, v = st.rows(pos, n_ub, layer=0)
        dk, dv = gu.dev(k), gu.dev(v)
        sjk.check(L.sjk_layer_store(C.byref(layer), pos, n_ub, gu.ptr(dk), gu.ptr(dv), 1, None), "store")
    torch.cuda.synchronize()
    view = sjk.view_of(layer)
    n_q, n_head = 4, 16
    q = torch.from_numpy(synth.queries(5, 1, n_q, n_head, D)[0]).cuda()
    sjk.check(L.sjk_hadamard(C.c_void_p(q.data_ptr()), n_q * n_head, D, None))
    nbytes = L.sjk_attend_scratch_bytes(C.byref(view), npos, n_q, n_head)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    ref = torch.empty_like(q)
    sjk.check(L.sjk_attend(C.byref(view), pol.B, npos, npos - n_q, n_q, n_head, C.c_void_p(q.data_ptr()), 1.0 / 16,
                           C.c_void_p(ref.data_ptr()), C.c_void_p(scratch.data_ptr()), nbytes, None), "attend")
    ref_h = ref.cpu().numpy()
    free_after = []
    outs = [torch.full_like(q, float("nan")) for _ in range(2)]
    for out in outs:
        rc = L.sjk_attend_static(C.byref(view), pol.B, npos, npos - n_q, n_q, n_head, C.c_void_p(q.data_ptr()), 1.0 / 16,
                                 C.c_void_p(out.data_ptr()), None)
        sjk.check(rc, "attend_static")
        torch.cuda.synchronize()
        free_after.append(torch.cuda.mem_get_info()[0])
        assert gu.rel_err_rows(out.cpu().numpy(), ref_h) <= ATTN_TOL_TIGHT
    assert free_after[0] == free_after[1]          # the second call took no device memory
    # a shape whose scratch bound exceeds the fixed array is refused with its own status
    big = L.sjk_attend_static(C.byref(view), pol.B, npos, npos - 64, 64, n_head, C.c_void_p(q.data_ptr()), 1.0 / 16,
                              C.c_void_p(ref.data_ptr()), None)
    assert big == -202
    assert b"no-allocation" in L.sj_kvarn_strerror(-202)
    assert L.sjk_device_status() == 0
    L.sj_kvarn_layer_free(C.byref(layer))
