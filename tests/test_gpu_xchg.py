"""The exchange of attention partials over peer memory (sjk_xchg_*, slices.PeerExchange): the merged output equals an
all-gather of the same triples followed by sjk_attend_merge, bit for bit, over consecutive layer calls (both slot
parities). One rank on one GPU always; two ranks as two processes on two GPUs when the machine has them (each rank
publishes into the other's buffer over NVLink; NVLS off; a short process-group timeout bounds every collective)."""
import ctypes as C
import os

import numpy as np
import pytest

import gpu_util as gu
import sjk

pytestmark = pytest.mark.gpu

ROWS, D = 64, 256


@pytest.fixture(scope="module")
def L():
    import build
    build.build()
    import torch
    assert torch.cuda.is_available()
    return sjk.lib()


def _parts(seed, n):
    """n partial sets [n][ROWS][D + 2] with the shapes of real ones: m finite or -inf, l > 0 (0 where m = -inf)."""
    rng = np.random.default_rng(seed)
    p = np.zeros((n, ROWS, D + 2), np.float32)
    p[:, :, 0] = rng.normal(3.0, 2.0, (n, ROWS))
    p[:, :, 1] = rng.uniform(0.5, 50.0, (n, ROWS))
    p[:, :, 2:] = rng.standard_normal((n, ROWS, D)) * p[:, :, 1:2]
    p[0, 5, 0], p[0, 5, 1], p[0, 5, 2:] = -np.inf, 0.0, 0.0          # a rank that saw no position of a row
    return p


def test_single_rank_exchange(L):
    import slices
    T = gu.torch()
    ex = slices.PeerExchange(None, 0, 1, ROWS, D)
    try:
        for call in range(3):
            part = T.from_numpy(_parts(call, 1)[0]).cuda()
            out = T.empty((ROWS, D), dtype=T.float32, device="cuda")
            ref = T.empty_like(out)
            ex.exchange(part, out, None)
            sjk.check(L.sjk_attend_merge(gu.ptr(part), 1, ROWS, D, gu.ptr(ref), None))
            assert np.array_equal(gu.host(out, np.uint32), gu.host(ref, np.uint32)), call
        assert L.sjk_device_status() == 0
    finally:
        ex.close()


def _two_rank_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        import slices
        L = sjk.lib()
        ex = slices.PeerExchange(dist, rank, world, ROWS, D)
        bad = []
        s = torch.cuda.Stream()
        for call in range(5):
            mine = torch.from_numpy(_parts(100 * call + rank, 1)[0]).cuda()
            out = torch.empty((ROWS, D), dtype=torch.float32, device="cuda")
            with torch.cuda.stream(s):
                ex.exchange(mine, out, C.c_void_p(s.cuda_stream))
            torch.cuda.synchronize()
            allp = torch.empty((world, ROWS, D + 2), dtype=torch.float32, device="cuda")
            dist.all_gather_into_tensor(allp, mine)
            ref = torch.empty_like(out)
            sjk.check(L.sjk_attend_merge(C.c_void_p(allp.data_ptr()), world, ROWS, D, C.c_void_p(ref.data_ptr()), None))
            torch.cuda.synchronize()
            if not torch.equal(out.view(torch.int32), ref.view(torch.int32)):
                bad.append(call)
        status = L.sjk_device_status()
        ex.close()
        dist.destroy_process_group()
        q.put((rank, bad, status))
    except Exception as e:          # reported to the parent, which fails the test
        q.put((rank, repr(e), -1))


def test_two_rank_exchange_matches_all_gather(L):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU: the two-rank exchange runs on machines with two or more")
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_two_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r, bad, status = q.get(timeout=180)
            res[r] = (bad, status)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert res == {0: ([], 0), 1: ([], 0)}, res


def test_single_rank_fused_partial_exchange(L):
    """sjk_attend_partial_xchg (the exchange folded into the call's merge kernel) equals sjk_attend_partial followed by
    sjk_attend_merge of the one partial, bit for bit, on a 4/4 cache (tensor-core body with the staged rows)."""
    import slices
    T = gu.torch()
    import configs
    sm = configs.SliceModel(0, 64, sink=True, tail=700, n_layers=1)
    sm.build()
    v = sjk.view_of(sm.layers[0])
    n_q, n_head = 4, 16
    syn = configs.DeviceSynth(4, 1)
    q = syn.queries(0, n_q)
    sjk.check(L.sjk_hadamard(gu.ptr(q), n_q * n_head, 256, None))
    need = L.sjk_attend_scratch_bytes(C.byref(v), sm.N, n_q, n_head)
    scratch = T.empty(int(need), dtype=T.uint8, device="cuda")
    part = T.empty((n_q * n_head, 258), dtype=T.float32, device="cuda")
    ref = T.empty((n_q * n_head, 256), dtype=T.float32, device="cuda")
    ex = slices.PeerExchange(None, 0, 1, n_q * n_head, 256)
    try:
        for call in range(3):
            qpos0 = sm.N - n_q - call
            sjk.check(L.sjk_attend_partial(C.byref(v), sm.B, sm.N, qpos0, n_q, n_head, 7, gu.ptr(q), np.float32(1 / 16),
                                           gu.ptr(part), gu.ptr(scratch), need, None))
            sjk.check(L.sjk_attend_merge(gu.ptr(part), 1, n_q * n_head, 256, gu.ptr(ref), None))
            out = T.empty_like(ref)
            ex.attend(v, sm.B, sm.N, qpos0, n_q, n_head, 7, gu.ptr(q), np.float32(1 / 16), scratch, need, gu.ptr(out), None)
            assert np.array_equal(gu.host(out, np.uint32), gu.host(ref, np.uint32)), call
        assert L.sjk_device_status() == 0
    finally:
        ex.close()
        sm.free()
