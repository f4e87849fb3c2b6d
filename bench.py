#!/usr/bin/env python
"""bench.py - B200 benchmark of the SJ-KVaRN hot path (one JSON line on rank 0).

Every cache is built on the GPU through the product API from the seeded generator of libsjk_b200.so (sjk_synth_*;
the host build of the same arithmetic draws identical bits, so the reference can rebuild any of these caches on the
host). The BASELINE configurations (sj-kvarn-codec_b200/configs.py):

  value     config 1 (headline): decode attention at 100K context over a 4/4 scalar body, 16 layers, 4 KV heads of
            D = 256, 16 query heads (GQA 4), decode width 4, batch 1; device time per layer call (us), inputs resident
            in HBM, CUDA events on the launching stream; a step = one attention call per layer (16 x 113 MB > L2)
  e2e       the same through the C-ABI with HOST buffers: per step the queries go host->device from pinned memory and
            the outputs come back, inside the timed region
  seal      config 0: the 4096-token commit (128 records, 4/4) out of an 8,320-position tq6_0 ring; Mtok/s, HBM and
            ALU-roofline fractions; plus the ring write of those 8,320 positions
  config2   3/2 trellis: per-layer seal of the same commit shape; attention at 32K (16 layers, per layer call); e2e
  config3   64-sequence paged pool, 3/3 trellis, decode width 1: tokens/s over a window of decode steps that holds
            policy-triggered seals; sequences split over the ranks by LPT (no collective)
  config4   one 1,048,576-token sequence sliced by context over the ranks: bulk seal (Mtok/s per GPU) and attention
            (partial per rank, the (m, l, o) triples exchanged over peer memory and merged), with per-phase times and
            the NCCL all-gather + merge path beside it
  parity    the GPU's config-0 records and config-1 / config-2 attention against the reference's, computed in the
            cpu_baseline leg from the same seeded rows (or against the committed golden hashes without that leg)
  cpu_baseline  the reference (oracle/_ref: sj_kvarn.h compiled from its own source) on the host cores: config-1
            attention on a sample of (row, head) pairs at the full context, config-0 seal (sj_kvarn_layer_seal on one
            thread, and the threaded harness on all cores), config-2 seal and attention, sampled configs 3 and 4

--impl reference times only the reference CPU path (rank 0; other ranks exit 0), on config 1's workload.
Multi-GPU (torchrun): config 1 runs one sequence replica per rank (weak scaling, no collective); config 3 splits the
pool's sequences; config 4 splits one sequence by context.
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "sj-kvarn-codec_b200")
for _p in (PKG, os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "decode-attn µs/call @100K ctx"
D, H, HQ, SINK, G = 256, 4, 16, 128, 128
SCALE = 1.0 / 16.0          # 1/sqrt(D)
REC = {(4, 4): 35072, (3, 3): 26880, (3, 2): 22784}
STAGE_ROW = 196             # bytes of one tq6_0 row (2 blocks of 98)


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {}


def hbm_peak():
    p = peaks().get("hbm_gbs")
    return (float(p), "measured") if p else (6650.0, "fallback")


def attn_bytes_per_call(B, N, nq=4, hq=HQ, rec_bytes=35072, sink=SINK):
    """Algorithmic bytes of one layer call: every record, staged row and sink row once, plus Q in and O out."""
    body = (B - sink) // G * H * rec_bytes
    tail = (N - B) * H * 2 * STAGE_ROW
    sk = sink * H * D * 4
    qo = 2 * nq * hq * D * 4
    return body + tail + sk + qo


def seal_bytes(records, rec_bytes):
    """per record: read 128 staged K and V rows (392 B per token and head), write the record"""
    return records * (G * 2 * STAGE_ROW + rec_bytes)


# Operation counts of one record's seal (the reference's algorithm, sj_kvarn.h:939-1012): the balancing rescales the
# 128 x 256 tile of each side with two fp32 divides per element, once before and twice per iteration (16 iterations);
# every iteration takes a column and a row standard deviation of each side in double (3 FP64 operations per element:
# the widening sum, the difference and the fused square-accumulate).
SEAL_DIVIDES = 2 * (2 * G * D * (2 * 16 + 1))          # 4.33 M fp32 divides per record
SEAL_FP64 = 2 * (2 * 3 * G * D * 16)                   # 6.29 M FP64 operations per record


def seal_alu_bound_s(records, sm_mhz, n_sm=148):
    """Lower bound on the seal time from the B200's per-SM pipe widths at the sampled SM clock: a correctly rounded
    fp32 divide takes at least 3 FP32-pipe operations (a multiply by the divisor's reciprocal and two fused residual
    corrections: the form the seal kernel uses), 128 FP32 lanes per SM; FP64 64 lanes per SM. The two pipes work
    concurrently, so the bound is the larger of the two."""
    clk = (sm_mhz or 1965.0) * 1e6
    fp32 = records * SEAL_DIVIDES * 3 / (128.0 * n_sm * clk)
    fp64 = records * SEAL_FP64 / (64.0 * n_sm * clk)
    return max(fp32, fp64)


def profile_traffic(name):
    """dram bytes per launch recorded by the committed ncu summary profiles/<name> (None if absent)."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        for ln in open(path):
            if ln.startswith("traffic_bytes_per_launch:"):
                return float(ln.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


def golden_config_hashes():
    """Committed reference hashes of the configurations' record bytes (tests/golden/config_hashes.txt)."""
    out = {}
    try:
        for ln in open(os.path.join(ROOT, "tests", "golden", "config_hashes.txt")):
            f = ln.split()
            if len(f) == 2 and not ln.startswith("#"):
                out[f[0]] = f[1]
    except OSError:
        pass
    return out


def digest(a):
    """SHA-256 (first 32 hex digits) of an array's bytes: the records' identity in the parity fields."""
    import hashlib
    return hashlib.sha256(a.tobytes()).hexdigest()[:32]


def dev_bytes(ptr, n):
    """n bytes at a raw device address, copied to a host numpy array"""
    import numpy as np
    out = np.empty(int(n), dtype=np.uint8)
    cudart = C.CDLL("libcudart.so.12")
    cudart.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    assert cudart.cudaDeviceSynchronize() == 0
    assert cudart.cudaMemcpy(out.ctypes.data, C.c_void_p(ptr), int(n), 2) == 0
    return out


class Clocks:
    """nvidia-smi sampling during the timed region (SM clock, throttle reasons)."""

    def __init__(self, gpu):
        self.gpu, self.p, self.out = gpu, None, None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p:
            time.sleep(0.25)
            self.p.terminate()
            try:
                self.out = self.p.communicate(timeout=5)[0]
            except Exception:
                self.out = None

    def summary(self):
        if not self.out:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.out.strip().splitlines():
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0])); mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def time_events(torch, stream_obj, fn, steps, warmup, sync=None):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if sync:
        sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream_obj)
    for _ in range(steps):
        fn()
    e1.record(stream_obj)
    torch.cuda.synchronize()
    if sync:
        sync()
    return e0.elapsed_time(e1) / steps          # ms per step


# ---------------------------------------------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------------------------------------------
class AttnStep:
    """One decode step over the layers of a PolicyModel: an sjk_layer_attend per layer (device buffers), and the
    end-to-end form with host queries in and host outputs out, layer by layer on two copy streams so that a layer's
    copies overlap the attention of its neighbours."""

    def __init__(self, torch, m, n_q, stream_obj, st):
        import sjk
        self.T, self.m, self.n_q, self.s, self.st, self.sjk = torch, m, n_q, stream_obj, st, sjk
        self.L = sjk.lib()
        nl = len(m.layers)
        self.q = torch.stack([m.syn.queries(il, n_q) for il in range(nl)]).contiguous()     # [nl][n_q][HQ][D]
        self.q_model = self.q.clone()                   # the model basis (sjk_layer_attend_model rotates inside)
        sjk.check(self.L.sjk_hadamard(C.c_void_p(self.q.data_ptr()), nl * n_q * HQ, D, None), "hadamard")
        self.out = torch.empty_like(self.q)
        self.out_model = torch.empty_like(self.q)
        torch.cuda.synchronize()
        self.per = n_q * HQ * D
        self.B, self.N = m.pol.B, m.n
        self.q_h = self.q.cpu().pin_memory()
        self.out_h = torch.empty(self.out.shape, dtype=self.out.dtype).pin_memory()
        self.cs_in, self.cs_out = torch.cuda.Stream(), torch.cuda.Stream()
        self.ev_in = [torch.cuda.Event() for _ in range(nl)]
        self.ev_out = [torch.cuda.Event() for _ in range(nl)]

    def attend(self, il):
        rc = self.L.sjk_layer_attend(C.byref(self.m.layers[il]), self.B, self.N, self.N - self.n_q, self.n_q, HQ,
                                     C.c_void_p(self.q.data_ptr() + il * self.per * 4), SCALE,
                                     C.c_void_p(self.out.data_ptr() + il * self.per * 4), self.st)
        if rc:
            raise self.sjk.SjkError(rc, "attend")

    def step(self):
        for il in range(len(self.m.layers)):
            self.attend(il)

    def step_model(self):
        """The same calls with the rotation folded in: model-basis queries in, model-basis outputs out."""
        for il in range(len(self.m.layers)):
            rc = self.L.sjk_layer_attend_model(C.byref(self.m.layers[il]), self.B, self.N, self.N - self.n_q, self.n_q, HQ,
                                               C.c_void_p(self.q_model.data_ptr() + il * self.per * 4), SCALE,
                                               C.c_void_p(self.out_model.data_ptr() + il * self.per * 4), self.st)
            if rc:
                raise self.sjk.SjkError(rc, "attend_model")

    def step_e2e(self):
        T, s = self.T, self.s
        self.cs_in.wait_stream(s)                                   # the previous step's reads of q are done
        for il in range(len(self.m.layers)):
            with T.cuda.stream(self.cs_in):
                self.q[il].copy_(self.q_h[il], non_blocking=True)
                self.ev_in[il].record(self.cs_in)
            s.wait_event(self.ev_in[il])
            self.attend(il)
            self.ev_out[il].record(s)
            self.cs_out.wait_event(self.ev_out[il])
            with T.cuda.stream(self.cs_out):
                self.out_h[il].copy_(self.out[il], non_blocking=True)
        s.wait_stream(self.cs_out)

    def bytes_h2d(self):
        return self.q.numel() * 4

    def bytes_d2h(self):
        return self.out.numel() * 4


def run_config1(args, torch, dist, local_rank):
    """Config 1 (headline). Every rank builds the same seeded sequence (seed 1) and serves it (weak scaling)."""
    import configs
    s = torch.cuda.Stream()
    st = C.c_void_p(s.cuda_stream)
    t0 = time.time()
    m = configs.build_config1(stream=st, layers=args.config1_layers)
    torch.cuda.synchronize()
    build_s = time.time() - t0
    a = AttnStep(torch, m, configs.CFG1["n_q"], s, st)
    barrier = (lambda: dist.barrier()) if dist else None
    with Clocks(local_rank) as clk:
        ms = time_events(torch, s, a.step, args.steps, args.warmup, barrier)
    ms_e2e = time_events(torch, s, a.step_e2e, args.steps, args.warmup, barrier)
    ms_model = time_events(torch, s, a.step_model, args.steps, args.warmup, barrier)
    a.step()
    torch.cuda.synchronize()
    out0 = a.out[0].cpu().numpy().copy()                            # layer 0's output, for the parity check
    if dist:
        t = torch.tensor([ms, ms_e2e, ms_model], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e, ms_model = float(t[0]), float(t[1]), float(t[2])
    res = dict(ms=ms, ms_e2e=ms_e2e, ms_model=ms_model, B=m.pol.B, N=m.n, build_s=build_s, clocks=clk.summary(), h2d=a.bytes_h2d(),
               d2h=a.bytes_d2h(), launches_per_step=2 * len(m.layers), out0=out0)
    m.free()
    return res


def run_seal0(args, torch, bits=(4, 4), heavy=False, seed=0):
    """Config 0 (or config 2's commit with bits (3, 2), heavy, seed 2): seal the 4096-token commit; the ring write of
    the 8,320 positions; the records' FNV-1a hash."""
    import configs
    import sjk
    L = sjk.lib()
    s = torch.cuda.Stream()
    st = C.c_void_p(s.cuda_stream)
    m, B0, B1 = configs.build_config0(stream=st, bits=bits, heavy=heavy, seed=seed)
    lay = m.layers[0]

    def seal():
        sjk.check(L.sjk_layer_seal(C.byref(lay), B0, B1, st), "seal")

    ms = time_events(torch, s, seal, max(3, args.steps), args.warmup)
    n_rec = (B1 - B0) // G * H
    rec_hash = digest(dev_bytes(lay.body, n_rec * lay.lay.bytes))
    k, v = m.syn.rows(0, 0, 8320)
    torch.cuda.synchronize()

    def store():
        sjk.check(L.sjk_layer_store(C.byref(lay), 0, 8320, C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()), 1, st),
                  "store")

    ms_store = time_events(torch, s, store, max(3, args.steps), args.warmup)
    m.free()
    return dict(ms=ms, ms_store=ms_store, records=n_rec, rec_bytes=REC[bits], rec_hash=rec_hash)


def run_config2(args, torch):
    """Config 2 (3/2 trellis, K Student-t(4) before the channel scales, seed 2): attention at 32K over 16 layers (per
    layer call) with its e2e form, and the seal of one 4096-token commit."""
    import configs
    s = torch.cuda.Stream()
    st = C.c_void_p(s.cuda_stream)
    t0 = time.time()
    m = configs.build_config2(stream=st, layers=args.config2_layers)
    torch.cuda.synchronize()
    build_s = time.time() - t0
    a = AttnStep(torch, m, configs.CFG2["n_q"], s, st)
    nl = len(m.layers)
    ms = time_events(torch, s, a.step, max(3, args.steps), args.warmup)
    ms_e2e = time_events(torch, s, a.step_e2e, max(3, args.steps), args.warmup)
    a.step()
    torch.cuda.synchronize()
    out0 = a.out[0].cpu().numpy().copy()
    B, N = m.pol.B, m.n
    m.free()
    sres = run_seal0(args, torch, bits=(3, 2), heavy=True, seed=2)
    return dict(ms=ms / nl, ms_e2e=ms_e2e / nl, B=B, N=N, layers=nl, build_s=build_s, out0=out0,
                bytes=attn_bytes_per_call(B, N, rec_bytes=22784), seal=sres, h2d=a.bytes_h2d() // nl,
                d2h=a.bytes_d2h() // nl)


def run_config4(args, torch, dist, rank, world):
    """Config 4: one 1,048,576-token sequence (8,192 groups per KV head and layer + 128 sink + 4,096 tail, seed 4)
    sliced by context: rank r holds a contiguous range of the 8,192 groups of every layer (rank 0 also the sink, the
    last rank the tail), balanced by attention cost (slices.group_range: a chunk of staged rows weighs 4.5 groups). Bulk seal: each layer's slice is staged into one staging buffer in the ring layout and
    sealed in one launch (timed: Mtok/s per GPU). Attention per layer call: sjk_attend_partial on every rank, then the
    (m, l, o) triples go to every rank over peer memory (slices.PeerExchange: NVLink stores, local merge in rank order);
    the NCCL all-gather + sjk_attend_merge path is timed beside it, and the phases separately. With
    several ranks, rank 0 also rebuilds layer 0 whole and checks the merged output against one call over it."""
    import configs
    import sjk
    import slices
    L = sjk.lib()
    c4 = configs.CFG4
    s = torch.cuda.Stream()
    st = C.c_void_p(s.cuda_stream)
    g0, g1 = slices.group_range(rank, world, c4["groups"], sink_chunks=(SINK + G - 1) // G, tail_chunks=c4["tail"] // G)
    t0 = time.time()
    sm = configs.SliceModel(g0, g1, sink=(rank == 0), tail=c4["tail"] if rank == world - 1 else 0,
                            n_layers=args.config4_layers, stream=st)
    nl = len(sm.layers)
    # every layer: its slice's rows staged (the staging buffer is shared by the layers), then its bulk seal; the seal
    # launches alone are timed with events (max over ranks)
    barrier = (lambda: dist.barrier()) if dist else None
    ms_seal = 0.0
    for il in range(nl):
        sm.write_layer(il)
        if barrier and il == 0:
            torch.cuda.synchronize()
            barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        sm.seal_layer(il)
        e1.record(s)
        torch.cuda.synchronize()
        ms_seal += e0.elapsed_time(e1)
    write_s = time.time() - t0
    tokens_sealed = sm.n_body * nl
    n_q, rows = c4["n_q"], c4["n_q"] * HQ
    q = torch.stack([sm.syn.queries(il, n_q) for il in range(nl)]).contiguous()
    sjk.check(L.sjk_hadamard(C.c_void_p(q.data_ptr()), nl * n_q * HQ, D, None), "hadamard")
    out = torch.empty_like(q)
    per = n_q * HQ * D
    views = [sjk.view_of(lay) for lay in sm.layers]
    need = L.sjk_attend_scratch_bytes(C.byref(views[0]), sm.N, n_q, HQ)
    scratch = torch.empty(int(need), dtype=torch.uint8, device="cuda")
    part = torch.empty((rows, D + 2), dtype=torch.float32, device="cuda")
    allp = torch.empty((world, rows, D + 2), dtype=torch.float32, device="cuda")
    reg = slices.regions(rank, world)
    qpos0 = sm.N - n_q if rank == world - 1 else sm.N
    torch.cuda.synchronize()

    def partial(il):
        rc = L.sjk_attend_partial(C.byref(views[il]), sm.B, sm.N, qpos0, n_q, HQ, reg,
                                  C.c_void_p(q.data_ptr() + il * per * 4), SCALE, C.c_void_p(part.data_ptr()),
                                  C.c_void_p(scratch.data_ptr()), need, st)
        if rc:
            raise sjk.SjkError(rc, "attend_partial")

    def exchange():
        if dist:
            dist.all_gather_into_tensor(allp, part)
        else:
            allp[0].copy_(part)

    def merge(il):
        rc = L.sjk_attend_merge(C.c_void_p(allp.data_ptr()), world, rows, D, C.c_void_p(out.data_ptr() + il * per * 4), st)
        if rc:
            raise sjk.SjkError(rc, "attend_merge")

    xch = slices.PeerExchange(dist, rank, world, rows, D)

    def p2p(il):
        xch.exchange(part, out[il], st)

    def fused(il):
        xch.attend(views[il], sm.B, sm.N, qpos0, n_q, HQ, reg, C.c_void_p(q.data_ptr() + il * per * 4), SCALE, scratch,
                   need, C.c_void_p(out.data_ptr() + il * per * 4), st)

    def step():                                                  # the product path: partial + exchange in one call
        with torch.cuda.stream(s):
            for il in range(nl):
                fused(il)

    def step_split():                                            # partial, then the stand-alone exchange
        with torch.cuda.stream(s):
            for il in range(nl):
                partial(il)
                p2p(il)

    def step_nccl():                                             # the same through NCCL all-gather + merge
        with torch.cuda.stream(s):
            for il in range(nl):
                partial(il)
                exchange()
                merge(il)

    ms = time_events(torch, s, step, max(3, args.steps), args.warmup, barrier)
    ms_split = time_events(torch, s, step_split, max(3, args.steps), args.warmup, barrier)
    ms_nccl = time_events(torch, s, step_nccl, max(3, args.steps), args.warmup, barrier)
    # per-phase device times over the same number of layer calls
    with torch.cuda.stream(s):
        ms_partial = time_events(torch, s, lambda: [partial(il) for il in range(nl)], max(3, args.steps), 1, barrier)
        ms_p2p = time_events(torch, s, lambda: [p2p(il) for il in range(nl)], max(3, args.steps), 1, barrier)
        ms_exchange = time_events(torch, s, lambda: [exchange() for _ in range(nl)], max(3, args.steps), 1, barrier)
        ms_merge = time_events(torch, s, lambda: [merge(il) for il in range(nl)], max(3, args.steps), 1, barrier)
    # the peer exchange's output against the NCCL path's (same triples, same merge order: identical bits)
    step()
    torch.cuda.synchronize()
    out_p2p = out.clone()
    step_nccl()
    torch.cuda.synchronize()
    p2p_equal = bool(torch.equal(out_p2p.view(torch.int32), out.view(torch.int32)))
    xch.close()
    check_err = None
    if world > 1 and rank == 0:
        whole = configs.SliceModel(0, c4["groups"], sink=True, tail=c4["tail"], n_layers=1, stream=st)
        whole.build()
        wout = torch.empty((n_q, HQ, D), dtype=torch.float32, device="cuda")
        sjk.check(L.sjk_layer_attend(C.byref(whole.layers[0]), whole.B, whole.N, whole.N - n_q, n_q, HQ,
                                     C.c_void_p(q.data_ptr()), SCALE, C.c_void_p(wout.data_ptr()), st), "attend whole")
        torch.cuda.synchronize()
        import numpy as np
        a, b = out[0].cpu().numpy().reshape(rows, D).astype(np.float64), wout.cpu().numpy().reshape(rows, D).astype(np.float64)
        check_err = float((np.linalg.norm(a - b, axis=1) / np.linalg.norm(b, axis=1)).max())
        whole.free()
    t = torch.tensor([ms, ms_partial, ms_exchange, ms_merge, ms_seal, ms_nccl, ms_p2p, 0.0 if p2p_equal else 1.0, ms_split],
                     device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_partial, ms_exchange, ms_merge, ms_seal, ms_nccl, ms_p2p, p2p_diff, ms_split = [float(x) for x in t]
    sm.free()
    B_global = SINK + c4["groups"] * G
    n_global = B_global + c4["tail"]
    return dict(ms=ms / nl, ms_partial=ms_partial / nl, ms_exchange=ms_exchange / nl, ms_merge=ms_merge / nl,
                ms_nccl=ms_nccl / nl, ms_p2p=ms_p2p / nl, p2p_equals_nccl=p2p_diff == 0.0, ms_split=ms_split / nl,
                bytes=attn_bytes_per_call(B_global, n_global), n_ctx=n_global, layers=nl, exchange=rows * (D + 2) * 4,
                groups_per_rank=g1 - g0, write_s=write_s, seal_ms=ms_seal, tokens_sealed=tokens_sealed,
                merged_vs_whole=check_err)


def run_config3(args, torch, dist, rank, world):
    """Config 3: a paged record pool of 64 sequences (contexts uniform in [8K, 64K], seed 3), 3/3 trellis body,
    adaptive tail 4096 -> 8192, fp16 sink 128, 16 layers, decode width 1 (16 query heads, GQA 4). Sequences go to the
    ranks by longest-processing-time on their contexts; every rank builds its own in one pool through the product's
    sequence API (sj_kvarn_seq_begin_ubatch: policy, block reservation and seals; sjk_seq_store: each 512-token
    ubatch's writes), with the seeded generator's rows of each sequence (generator seed 3000 + sequence index). One
    step appends one token to every sequence of every layer (sj_kvarn_seq_begin_ubatch, sealing where the policy
    says, then one sjk_store_batch launch) and runs one sjk_attend_batch call per layer. The timed window is placed so
    that the earliest policy-triggered seal of the pool falls in its middle, and it is long enough for the pool's
    natural seal rate (one 4096-token commit per sequence per 4,096 steps)."""
    import numpy as np
    import configs
    import sjk
    import slices
    L = sjk.lib()
    s = torch.cuda.Stream()
    st = C.c_void_p(s.cuda_stream)
    c3 = configs.CFG3
    NL, NQ = c3["layers"], c3["n_q"]
    ctx = np.random.default_rng(3).integers(c3["ctx_lo"], c3["ctx_hi"] + 1, size=c3["seqs"])[:args.config3_seqs]
    owner = slices.lpt_assign(ctx, world)
    mine = [i for i in range(len(ctx)) if owner[i] == rank]
    steps = max(args.steps, args.config3_steps)
    t0 = time.time()
    tail, tail_max = 4096, 8192
    # steps until each sequence's next commit after its build (the policy seals when pos0 - B >= tail_max)
    max_extra = steps + args.warmup + 2 * tail_max
    cfg = sjk.config(D, H, int(ctx.max()) + max_extra + 1024, 512, bits_k=3, bits_v=3, body=1, tail=tail, tail_max=tail_max)
    pool = sjk.Pool()
    n_blocks = sum((int(ctx[i]) + max_extra) // G + 2 for i in mine)
    sjk.check(L.sj_kvarn_pool_init(C.byref(pool), C.byref(cfg), NL, n_blocks), "pool_init")
    seqs = []
    for i in mine:
        sq = sjk.Seq()
        sjk.check(L.sj_kvarn_seq_init(C.byref(sq), C.byref(cfg), NL, C.byref(pool)), "seq_init")
        sq.stream = st.value
        seqs.append(sq)
    n_ub = 512
    kbuf = torch.empty((NL, n_ub, H, D), dtype=torch.float32, device="cuda")
    vbuf = torch.empty_like(kbuf)
    syns = {}
    for j, sq in enumerate(seqs):
        syn = syns[j] = configs.DeviceSynth(3000 + mine[j], NL, False, 0, st)
        target, pos = int(ctx[mine[j]]), 0
        while pos < target:
            n = min(n_ub, target - pos)
            sjk.check(L.sj_kvarn_seq_begin_ubatch(C.byref(sq), pos, n), "seq_begin_ubatch")
            for il in range(NL):
                syn.rows_into(il, pos, n, kbuf[il], vbuf[il])
            sjk.check(L.sjk_seq_store(C.byref(sq), pos, n, C.c_void_p(kbuf.data_ptr()), C.c_void_p(vbuf.data_ptr()),
                                      n_ub * H * D, 1, st), "seq_store")
            pos += n
    torch.cuda.synchronize()
    build_s = time.time() - t0
    n_seq = len(seqs)
    views = [(sjk.View * n_seq)() for _ in range(NL)]
    store_views = (sjk.View * (n_seq * NL))()
    for j, sq in enumerate(seqs):
        for il in range(NL):
            L.sjk_layer_view(C.byref(sq.layers[il]), C.byref(views[il][j]))
            L.sjk_layer_view(C.byref(sq.layers[il]), C.byref(store_views[j * NL + il]))
    # decode-step rows: per step, one new (K, V) row per (sequence, layer) from the sequence's generator
    k_step = torch.empty((n_seq * NL, H, D), dtype=torch.float32, device="cuda")
    v_step = torch.empty_like(k_step)
    q = torch.empty((NL, n_seq, NQ, HQ, D), dtype=torch.float32, device="cuda")
    for j in range(n_seq):
        for il in range(NL):
            q[il, j] = syns[j].queries(il, NQ)
    sjk.check(L.sjk_hadamard(C.c_void_p(q.data_ptr()), NL * n_seq * NQ * HQ, D, None), "hadamard")
    out = torch.empty_like(q)
    per_layer = n_seq * NQ * HQ * D * 4
    need = L.sjk_attend_batch_scratch_bytes(C.byref(views[0][0]), max(n_seq, 1), NQ, HQ)
    scratch = torch.empty(int(need), dtype=torch.uint8, device="cuda")
    Bs, Ns, Qs = (C.c_uint32 * n_seq)(), (C.c_uint32 * n_seq)(), (C.c_uint32 * n_seq)()
    pos_items = (C.c_uint32 * (n_seq * NL))()
    stats = dict(seal_steps=0, seal_records=0)
    torch.cuda.synchronize()

    def fill_rows():
        # the new rows of this step (position s.n of every sequence), drawn on the device
        for j, sq in enumerate(seqs):
            for il in range(NL):
                syns[j].rows_into(il, sq.n, 1, k_step[j * NL + il:j * NL + il + 1], v_step[j * NL + il:j * NL + il + 1])

    def step():
        sealed = 0
        for j, sq in enumerate(seqs):
            B_before = sq.pol.B
            sjk.check(L.sj_kvarn_seq_begin_ubatch(C.byref(sq), sq.n, 1), "seq_begin_ubatch")
            sealed += (sq.pol.B - B_before) // G * H * NL
            for il in range(NL):
                pos_items[j * NL + il] = sq.n
        sjk.check(L.sjk_store_batch(store_views, pos_items, n_seq * NL, C.c_void_p(k_step.data_ptr()),
                                    C.c_void_p(v_step.data_ptr()), 1, st), "store_batch")
        for j, sq in enumerate(seqs):
            sq.n = sq.n + 1
            Bs[j], Ns[j], Qs[j] = sq.pol.B, sq.n, sq.n - 1
        stats["seal_steps"] += int(sealed > 0)
        stats["seal_records"] += sealed
        for il in range(NL):
            rc = L.sjk_attend_batch(views[il], Bs, Ns, Qs, n_seq, NQ, HQ, C.c_void_p(q.data_ptr() + il * per_layer), SCALE,
                                    C.c_void_p(out.data_ptr() + il * per_layer), C.c_void_p(scratch.data_ptr()), need, st)
            if rc:
                raise sjk.SjkError(rc, "attend_batch")

    def steps_to_seal():
        # steps until the first sequence's begin_ubatch seals: due when pos0 - B >= tail_max
        return min((tail_max - (int(sq.n) - int(sq.pol.B)) for sq in seqs), default=0)

    def step_bytes():
        tot = 0
        for sq in seqs:
            B, N = sq.pol.B, sq.n
            tot += (B - G) // G * H * 26880 + (N - B) * H * 2 * STAGE_ROW + G * H * D * 4 + 2 * NQ * HQ * D * 4
        return tot * NL

    barrier = (lambda: dist.barrier()) if dist else None
    fill_rows()
    for _ in range(args.warmup):
        step()
    # place the first seal of the pool at the middle of the timed window (untimed steps before it); every rank agrees
    # on the same count (the max over ranks of what each would skip is not needed: each rank skips its own)
    skip = max(0, steps_to_seal() - steps // 2)
    t_skip = time.time()
    for _ in range(skip):
        step()
    torch.cuda.synchronize()
    skip_s = time.time() - t_skip
    if barrier:
        barrier()
    stats["seal_steps"] = 0
    stats["seal_records"] = 0
    b0 = step_bytes()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    evs[0].record(s)
    for i in range(steps):
        step()
        evs[i + 1].record(s)
    torch.cuda.synchronize()
    per_step = [evs[i].elapsed_time(evs[i + 1]) for i in range(steps)]
    ms = sum(per_step) / steps
    b1 = step_bytes()

    def attend_only():
        for il in range(NL):
            rc = L.sjk_attend_batch(views[il], Bs, Ns, Qs, n_seq, NQ, HQ, C.c_void_p(q.data_ptr() + il * per_layer), SCALE,
                                    C.c_void_p(out.data_ptr() + il * per_layer), C.c_void_p(scratch.data_ptr()), need, st)
            if rc:
                raise sjk.SjkError(rc, "attend_batch")

    ms_attn = time_events(torch, s, attend_only, min(steps, 20), 2, barrier)
    abytes = step_bytes()
    seal_steps, seal_records = stats["seal_steps"], stats["seal_records"]
    ms_max = max(per_step)
    t = torch.tensor([ms, ms_attn, ms_max], device="cuda")
    tb = torch.tensor([float(abytes), float((b0 + b1) / 2), float(seal_steps), float(seal_records)], device="cuda",
                      dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(tb, op=dist.ReduceOp.SUM)
    ms, ms_attn, ms_max = float(t[0]), float(t[1]), float(t[2])
    abytes, sbytes, seal_steps, seal_records = float(tb[0]), float(tb[1]), int(tb[2]), int(tb[3])
    status = L.sjk_device_status()
    for sq in seqs:
        L.sj_kvarn_seq_free(C.byref(sq))
    L.sj_kvarn_pool_free(C.byref(pool))
    return dict(ms=ms, ms_attn=ms_attn, ms_max_step=ms_max, attn_bytes=abytes, step_bytes=sbytes, seqs=n_seq,
                steps=steps, seal_steps=seal_steps, seal_records=seal_records, build_s=build_s, skip_steps=skip,
                skip_s=skip_s, ctx_total=int(ctx.sum()), device_status=status, n_total=len(ctx),
                launches_per_step=1 + 3 * NL + (2 * NL if seal_steps else 0))


# ---------------------------------------------------------------------------------------------------------------
# reference CPU path (oracle/_ref: the reference sj_kvarn.h compiled from its own source)
# ---------------------------------------------------------------------------------------------------------------
def ref_policy_layer(seed, bits, heavy, n_ctx, grow_to, idle_at=None, tail=4096, tail_max=8192, n_ub=512, threads=0):
    """One reference layer built through its own calls from the seeded rows (generator layer 0): the engine loop of
    begin_ubatch (seal what is due: threaded harness over the public per-record calls), commit, then
    sj_kvarn_hadamard + sj_kvarn_layer_store of the ubatch; optionally idled (keep 0) at idle_at."""
    import refcache
    rl = refcache.RefLayer(D, H, n_ctx, n_ub, bits_k=bits[0], bits_v=bits[1], tail=tail, tail_max=tail_max,
                           n_threads=threads)
    scale = refcache.synth_scales(seed, 0, 1, H, D, lib=rl.R)[0]
    pos = 0
    t_seal = 0.0
    while pos < grow_to:
        if idle_at is not None and pos == idle_at:
            t = time.perf_counter()
            rl.idle(0)
            t_seal += time.perf_counter() - t
        end = idle_at if idle_at is not None and pos < idle_at else grow_to
        n = min(n_ub, end - pos)
        t = time.perf_counter()
        rl.begin_ubatch(pos, n)
        t_seal += time.perf_counter() - t
        k, v = refcache.synth_kv(seed, 0, H, D, heavy, scale, pos, n, n_threads=threads, lib=rl.R)
        rl.store(pos, k, v)
        pos += n
    if idle_at is not None and idle_at == grow_to:
        t = time.perf_counter()
        rl.idle(0)
        t_seal += time.perf_counter() - t
    rl.seal_s = t_seal
    return rl


def ref_queries(rl, seed, n_q):
    import refcache
    return rl.rotate(refcache.synth_q(seed, 0, n_q, HQ, D, lib=rl.R))


def sample_pairs(n, n_q=4):
    """n (query row, query head) pairs spread over the pairs of a call and over all KV heads."""
    allp = [(iq, hq) for hq in range(HQ) for iq in range(n_q)]
    stride = max(1, len(allp) // n)
    return allp[::stride][:n]


def timed_pairs(rl, B, N, q, pairs, threads):
    t = time.perf_counter()
    outs = rl.attend_pairs(B, N, N - q.shape[0], q, pairs, SCALE, threads)
    return time.perf_counter() - t, outs


def rel_err(got, ref, pairs):
    import numpy as np
    a = np.stack([got[p] for p in pairs]).astype(np.float64)
    b = np.stack([ref[p] for p in pairs]).astype(np.float64)
    return float((np.linalg.norm(a - b, axis=1) / np.maximum(np.linalg.norm(b, axis=1), 1e-30)).max())


def cpu_config1(threads, gpu_out0=None):
    import configs
    c = configs.CFG1
    t0 = time.time()
    rl = ref_policy_layer(c["seed"], c["bits"], False, c["N"], c["N"], idle_at=c["idle_at"], threads=threads)
    build_s = time.time() - t0
    assert rl.pol.B == 93824, rl.pol.B
    q = ref_queries(rl, c["seed"], c["n_q"])
    pairs = sample_pairs(16)
    t, outs = timed_pairs(rl, rl.pol.B, c["N"], q, pairs, threads)
    res = dict(us_call=t * 1e6 * 64 / len(pairs), t=t, pairs=len(pairs), threads=rl.threads, build_s=build_s,
               seal_records=(rl.pol.B - SINK) // G * H, seal_s=rl.seal_s)
    if gpu_out0 is not None:
        res["parity_err"] = rel_err({p: gpu_out0[p] for p in pairs}, outs, pairs)
    rl.close()
    return res


def cpu_seal0(threads, bits=(4, 4), heavy=False, seed=0, single=True):
    """The config-0 schedule on the reference: 8,320 positions, then the 4096-token commit sealed by
    sj_kvarn_layer_seal on one thread (when `single`) and by the threaded harness on all cores; records hashed."""
    import configs
    c = configs.CFG0
    rl = ref_policy_layer(seed, bits, heavy, c["n_ctx"], c["npos"], threads=threads)
    R = rl.R
    R.sj_kvarn_policy_begin_ubatch(C.byref(rl.pol), c["npos"], c["n_ub"])
    B0, B1 = rl.pol.B, rl.pol.B_pending
    assert (B0, B1) == (128, 4224)
    res = {}
    if single:
        t = time.perf_counter()
        rl.seal(B0, B1, threaded=False)
        res["single_s"] = time.perf_counter() - t
    t = time.perf_counter()
    rl.seal(B0, B1, threaded=True)
    res["mt_s"] = time.perf_counter() - t
    ng = (B1 - B0) // G
    res["records"] = ng * H
    res["rec_hash"] = digest(rl.records(0, ng))
    res["threads"] = rl.threads
    rl.close()
    return res


def cpu_config2(threads, gpu_out0=None):
    import configs
    c = configs.CFG2
    t0 = time.time()
    rl = ref_policy_layer(c["seed"], c["bits"], True, c["N"] + 1024, c["N"], idle_at=c["N"], threads=threads)
    build_s = time.time() - t0
    assert rl.pol.B == 28672, rl.pol.B
    q = ref_queries(rl, c["seed"], c["n_q"])
    pairs = sample_pairs(16)
    t, outs = timed_pairs(rl, rl.pol.B, c["N"], q, pairs, threads)
    res = dict(us_call=t * 1e6 * 64 / len(pairs), pairs=len(pairs), build_s=build_s, threads=rl.threads,
               seal_records=(rl.pol.B - SINK) // G * H, seal_s=rl.seal_s)
    if gpu_out0 is not None:
        res["parity_err"] = rel_err({p: gpu_out0[p] for p in pairs}, outs, pairs)
    rl.close()
    return res


def cpu_config3(threads):
    """Sampled config 3: the pool's shortest sequence of at least 16K tokens (3/3 trellis), built through the policy
    on one layer (its seals timed as the seal sample), and its 16 (row, head) attention pairs at decode width 1;
    extrapolated to a decode step of the whole pool (attention cost in proportion to context, 16 layers) plus the seal
    work of a step at the pool's steady rate (64 sequences x 2,048 records per 4,096 steps)."""
    import numpy as np
    import configs
    c3 = configs.CFG3
    ctx = np.random.default_rng(3).integers(c3["ctx_lo"], c3["ctx_hi"] + 1, size=c3["seqs"])
    j = int(np.argmin(np.where(ctx >= 16384, ctx, 1 << 30)))
    n = int(ctx[j])
    t0 = time.time()
    rl = ref_policy_layer(3000 + j, (3, 3), False, n + 1024, n, threads=threads)
    build_s = time.time() - t0
    q = ref_queries(rl, 3000 + j, 1)
    pairs = [(0, hq) for hq in range(HQ)]
    t, _ = timed_pairs(rl, rl.pol.B, n, q, pairs, threads)
    recs = (rl.pol.B - SINK) // G * H
    per_rec_s = rl.seal_s / max(recs, 1)
    attn_step_s = t * float(ctx.sum()) / n * c3["layers"]
    seal_step_s = c3["seqs"] * (4096 // G) * H * c3["layers"] / 4096 * per_rec_s
    rl.close()
    return dict(ms_step=(attn_step_s + seal_step_s) * 1e3, tok_s=c3["seqs"] / (attn_step_s + seal_step_s),
                sample_ctx=n, sample_seq=j, attn_s=t, seal_records=recs, seal_s=rl.seal_s, build_s=build_s,
                threads=rl.threads)


def cpu_config4(threads):
    """Sampled config 4: one eighth of the sequence (groups [0, 1024) of layer 0 with the sink), built through the
    policy on one layer (its seals timed as the seal sample), 16 (row, head) pairs of attention over it; extrapolated
    to the whole 1,052,928-position call (x 8.2 by positions) and to the bulk seal of all 8,192 groups."""
    import configs
    c4 = configs.CFG4
    n = SINK + 1024 * G
    t0 = time.time()
    rl = ref_policy_layer(c4["seed"], (4, 4), False, n + 1024, n, idle_at=n, threads=threads)
    build_s = time.time() - t0
    q = ref_queries(rl, c4["seed"], c4["n_q"])
    pairs = sample_pairs(16)
    t, _ = timed_pairs(rl, rl.pol.B, n, q, pairs, threads)
    n_global = SINK + c4["groups"] * G + c4["tail"]
    recs = (rl.pol.B - SINK) // G * H
    us_call = t * 1e6 * 64 / len(pairs) * n_global / n
    rl.close()
    return dict(us_call=us_call, seal_mtoks=(recs // H * G) / rl.seal_s / 1e6, seal_records=recs, seal_s=rl.seal_s,
                sample_ctx=n, attn_s=t, build_s=build_s, threads=rl.threads)


def run_reference_arm(args):
    """--impl reference: the reference's own CPU attention (sj_kvarn_layer_attend_row) on config 1's cache (layer 0,
    seed 1, built with the reference's own calls from the same seeded rows as the GPU arm), a sample of (row, head)
    pairs per step on all host threads, scaled to a full layer call."""
    import configs
    c = configs.CFG1
    threads = args.cpu_threads
    t0 = time.time()
    rl = ref_policy_layer(c["seed"], c["bits"], False, c["N"], c["N"], idle_at=c["idle_at"], threads=threads)
    build_s = time.time() - t0
    q = ref_queries(rl, c["seed"], c["n_q"])
    pairs = sample_pairs(args.ref_pairs)
    for _ in range(min(args.warmup, 1)):
        timed_pairs(rl, rl.pol.B, c["N"], q, pairs[:rl.threads], threads)
    times = [timed_pairs(rl, rl.pol.B, c["N"], q, pairs, threads)[0] for _ in range(args.steps)]
    per_call_us = statistics.mean(times) * 1e6 * 64 / len(pairs)
    sample = (f"{len(pairs)} of the 64 (query row, query head) pairs of one layer call at N=100,000 "
              f"(B=93,824, 4/4 body, tq6_0 tail of 6,176), per step; scaled x{64 / len(pairs):g} to a full call; "
              f"cache built with the reference's own calls in {build_s:.1f} s")
    line = {"impl": "reference", "metric": METRIC, "value": per_call_us, "unit": "us/call", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.mean(times) * 1e3,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (the seeded generator of the GPU arm: same seed, same fp32 rows)",
            "config": {"workload": "config 1: decode attention, 100K ctx, 4/4 scalar body, 1 layer call (sampled)",
                       "n_ctx": c["N"], "B": rl.pol.B, "layers": 1, "kv_heads": H, "q_heads": HQ, "head_dim": D,
                       "decode_width": c["n_q"], "parallelism": "host threads"},
            "cpu_baseline": {"value": per_call_us, "unit": "us/call", "cores": rl.threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": per_call_us, "unit": "us/call", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    rl.close()
    print(json.dumps(line), flush=True)


def run_cpu_legs(args, gpu):
    """The cpu_baseline object (rank 0, N = 1): the reference on the host cores, with parity against the GPU."""
    import refcache
    if not refcache.available():
        return None
    threads = args.cpu_threads
    t_all = time.time()
    c1 = cpu_config1(threads, gpu.get("out0_c1"))
    s0 = cpu_seal0(threads)
    c2 = None if gpu.get("c2") is None else cpu_config2(threads, gpu.get("out0_c2"))
    s2 = None if gpu.get("c2") is None else cpu_seal0(threads, bits=(3, 2), heavy=True, seed=2, single=False)
    c3 = None if args.no_config3 else cpu_config3(threads)
    c4 = None if args.no_config4 else cpu_config4(threads)
    return dict(c1=c1, s0=s0, c2=c2, s2=s2, c3=c3, c4=c4, wall_s=time.time() - t_all)


# ---------------------------------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["sjk", "reference"], default="sjk")
    ap.add_argument("--cpu-threads", type=int, default=0, help="host threads for the CPU reference (0 = all)")
    ap.add_argument("--ref-pairs", type=int, default=16, help="(row, head) pairs per reference step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config2", action="store_true", help="skip the config-2 (3/2 trellis) measurement")
    ap.add_argument("--no-config4", action="store_true", help="skip the config-4 (1M context sliced over the ranks) measurement")
    ap.add_argument("--no-config3", action="store_true", help="skip the config-3 (64-sequence paged pool) measurement")
    ap.add_argument("--config3-seqs", type=int, default=64,
                    help="sequences of the config-3 pool (the first N of its 64; fewer only for small profiling runs)")
    ap.add_argument("--config3-steps", type=int, default=128, help="timed decode steps of config 3 (at least --steps)")
    ap.add_argument("--config4-layers", type=int, default=16, help="layers of the config-4 sequence")
    ap.add_argument("--config2-layers", type=int, default=16, help="layers of the config-2 model (fewer only for profiling)")
    ap.add_argument("--config1-layers", type=int, default=16, help="layers of the config-1 model (fewer only for profiling)")
    ap.add_argument("--only", choices=["seal", "seal2", "config1", "config2", "config3", "config4"], default=None,
                    help="run one section alone on one GPU and print its numbers (for profiling captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            run_reference_arm(args)
        return

    import torch
    import build as pkg_build
    import sjk
    if not os.path.exists(sjk.LIB_PATH):
        pkg_build.build()
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as td
        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
        dist = td
    if args.only:
        # one section alone (profiling): config 0's or config 2's seal, config 1's or config 2's attention, a
        # config-3 pool, or config 4 on one rank (the whole sequence)
        if args.only == "seal":
            r = run_seal0(args, torch)
        elif args.only == "seal2":
            r = run_seal0(args, torch, bits=(3, 2), heavy=True, seed=2)
        elif args.only == "config1":
            r = run_config1(args, torch, None, local_rank)
            r.pop("out0", None)
        elif args.only == "config2":
            r = run_config2(args, torch)
            r.pop("out0", None)
            r["seal"] = {k: r["seal"][k] for k in ("ms", "records")}
        elif args.only == "config3":
            r = run_config3(args, torch, None, 0, 1)
        else:
            r = run_config4(args, torch, None, 0, 1)
        print(json.dumps({"only": args.only, **{k: v for k, v in r.items() if not hasattr(v, "shape")}}), flush=True)
        return
    res = run_config1(args, torch, dist, local_rank)
    cfg4 = None if args.no_config4 else run_config4(args, torch, dist, rank, world)
    cfg3 = None if args.no_config3 else run_config3(args, torch, dist, rank, world)
    seal = run_seal0(args, torch) if rank == 0 else None
    cfg2 = run_config2(args, torch) if rank == 0 and not args.no_config2 else None
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    import numpy as np
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        gpu = {"out0_c1": res["out0"], "c2": cfg2, "out0_c2": cfg2["out0"] if cfg2 else None}
        cpu = run_cpu_legs(args, {k: v for k, v in gpu.items()})
    peak, peak_kind = hbm_peak()
    c1 = res
    per_call_ms = c1["ms"] / 16
    us_call = per_call_ms * 1e3
    us_call_e2e = c1["ms_e2e"] / 16 * 1e3
    abytes = attn_bytes_per_call(c1["B"], c1["N"])
    achieved = abytes / (per_call_ms * 1e-3) / 1e9
    traffic = profile_traffic("attend_config1_launches.md")
    sm_mhz = c1["clocks"].get("sm_mhz")

    def seal_obj(sr, what):
        mt = 4096 / (sr["ms"] * 1e-3) / 1e6
        gbs = seal_bytes(sr["records"], sr["rec_bytes"]) / (sr["ms"] * 1e-3) / 1e9
        bound = seal_alu_bound_s(sr["records"], sm_mhz)
        return {"metric": "seal Mtok/s (4096 commit)", "value": mt, "unit": "Mtok/s", "ms": sr["ms"], "workload": what,
                "records": sr["records"], "hbm_gbs": gbs, "hbm_frac": gbs / peak,
                "alu_bound_ms": bound * 1e3, "alu_frac": bound / (sr["ms"] * 1e-3),
                "alu_model": "per record 4.33 M fp32 divides (>= 3 FP32-pipe ops each, 128 lanes/SM) and 6.29 M FP64 "
                             "ops (64 lanes/SM) at the sampled SM clock, 148 SMs; the larger pipe time is the bound",
                "rec_hash": sr["rec_hash"]}

    # parity: live against the reference (cpu legs) or against the committed reference hashes
    gold = golden_config_hashes()
    parity = {"config0_records": {"gpu": seal["rec_hash"], "reference": (cpu or {}).get("s0", {}).get("rec_hash")
                                  or gold.get("config0_records"),
                                  "source": "live" if cpu else "tests/golden/config_hashes.txt"}}
    parity["config0_records"]["bit_exact"] = parity["config0_records"]["gpu"] == parity["config0_records"]["reference"]
    if cfg2:
        parity["config2_records"] = {"gpu": cfg2["seal"]["rec_hash"],
                                     "reference": (cpu or {}).get("s2", {}).get("rec_hash") if cpu and cpu.get("s2")
                                     else gold.get("config2_records")}
        parity["config2_records"]["bit_exact"] = parity["config2_records"]["gpu"] == parity["config2_records"]["reference"]
    if cpu:
        parity["config1_attention_max_rel_err"] = cpu["c1"].get("parity_err")
        if cpu.get("c2"):
            parity["config2_attention_max_rel_err"] = cpu["c2"].get("parity_err")
        parity["attention_pairs"] = "16 (row, head) pairs of layer 0 covering the 4 KV heads, vs sj_kvarn_layer_attend_row"
    if cfg4 and cfg4.get("merged_vs_whole") is not None:
        parity["config4_merged_vs_whole_max_rel_err"] = cfg4["merged_vs_whole"]

    line = {
        "metric": METRIC, "value": us_call, "unit": "us/call", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": c1["ms"], "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded SplitMix64 + Box-Muller generator (K = N(0,1) x LogNormal channel scales with 4 outlier "
                "channels x8 per head; V N(0,1); Q N(0,1) rounded to fp16), drawn on the device, bit-identical to its host build",
        "config": {"workload": "config 1: decode attention, 100K ctx, 4/4 scalar body, 16 layers", "n_ctx": c1["N"],
                   "B": c1["B"], "tail": c1["N"] - c1["B"], "sink": SINK, "layers": 16, "kv_heads": H,
                   "q_heads": HQ, "head_dim": D, "decode_width": 4, "batch": 1, "seed": 1,
                   "parallelism": f"sequence replicas x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (16 layers x 113 MB per step)"},
        "e2e": {"value": us_call_e2e, "unit": "us/call", "h2d_bytes_per_step": c1["h2d"], "d2h_bytes_per_step": c1["d2h"]},
        "model_basis": {"value": c1["ms_model"] / 16 * 1e3, "unit": "us/call",
                        "what": "sjk_layer_attend_model: model-basis queries in and outputs out, the rotations inside the "
                                "call (queries on chip in the body kernel, outputs in the merge kernel's clusters); the "
                                "headline takes rotated queries as sj_kvarn_layer_attend_row does"},
        "gpu_launches": c1["launches_per_step"] * args.steps,
        "clocks": c1["clocks"],
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "peak_kind": peak_kind, "frac_of_8tbs": achieved / 8000.0,
                     "kernel": "one sjk_attend call: attend_body_tc_kernel (sealed records + sink + staging ring) + attend_merge_kernel",
                     "algorithmic_bytes_per_launch": abytes},
        "parity": parity,
        "seal": dict(seal_obj(seal, "config 0: 1 layer, 4 KV heads, D=256, 4/4, 32 groups x 4 heads from an 8,320-row "
                                    "tq6_0 ring (seed 0)"),
                     ring_write_ms=seal["ms_store"],
                     ring_write_gbs=(8320 * (2 * H * D * 4) + SINK * H * 1024 + 8192 * H * 2 * STAGE_ROW)
                     / (seal["ms_store"] * 1e-3) / 1e9),
        "config2": None if cfg2 is None else {
            "workload": "config 2: 3/2 trellis body, K Student-t(4), seed 2; decode attention at 32K ctx (B = 28,672, tail "
                        "4,096), 16 layers, per layer call; seal of one 4096-token commit (128 records, 1 layer)",
            "attn_us_per_call": cfg2["ms"] * 1e3, "attn_bytes_per_call": cfg2["bytes"],
            "attn_gbs": cfg2["bytes"] / (cfg2["ms"] * 1e-3) / 1e9, "attn_frac": cfg2["bytes"] / (cfg2["ms"] * 1e-3) / 1e9 / peak,
            "e2e": {"value": cfg2["ms_e2e"] * 1e3, "unit": "us/call", "h2d_bytes_per_call": cfg2["h2d"],
                    "d2h_bytes_per_call": cfg2["d2h"]},
            "seal": seal_obj(cfg2["seal"], "config 2's commit: 32 groups x 4 heads, 3/2 trellis, from an 8,320-row ring"),
            "kernel": "attend_trellis_ws_kernel (sealed records) + attend_dense_tc_kernel (sink + staging ring) + attend_merge_kernel",
            "layers": cfg2["layers"], "build_s": cfg2["build_s"]},
        "config4": None if cfg4 is None else {
            "workload": f"config 4: one 1,048,576-token sequence (+ 128 sink, 4,096 tail), 4/4, seed 4, {cfg4['layers']} "
                        f"layers, split by context slice over {world} rank(s); bulk seal of each rank's slice; per layer "
                        "call: partial attention per rank + exchange of the (m, l, o) triples over peer memory + merge",
            "attn_us_per_call": cfg4["ms"] * 1e3, "attn_bytes_per_call": cfg4["bytes"], "n_ctx": cfg4["n_ctx"],
            "attn_gbs": cfg4["bytes"] / (cfg4["ms"] * 1e-3) / 1e9,
            "attn_frac_of_all_ranks": cfg4["bytes"] / (cfg4["ms"] * 1e-3) / 1e9 / (peak * world),
            "phases_us_per_call": {"partial": cfg4["ms_partial"] * 1e3, "peer_exchange": cfg4["ms_p2p"] * 1e3,
                                   "nccl_all_gather": cfg4["ms_exchange"] * 1e3, "nccl_merge": cfg4["ms_merge"] * 1e3},
            "nccl_path_us_per_call": cfg4["ms_nccl"] * 1e3, "split_exchange_path_us_per_call": cfg4["ms_split"] * 1e3,
            "peer_exchange_equals_nccl_path": cfg4["p2p_equals_nccl"],
            "exchange": "per layer call, one sjk_attend_partial_xchg: the partial attention, then one exchange launch "
                        "that stores the rank's (m, l, o) triples into every rank's exchange buffer over NVLink (CUDA "
                        "IPC mappings, 8-byte words tagged with the call's epoch), gathers the other ranks' and merges "
                        "all of them in rank order",
            "bulk_seal": {"mtoks_per_gpu": cfg4["tokens_sealed"] / (cfg4["seal_ms"] * 1e-3) / 1e6,
                          "mtoks_all_gpus": cfg4["tokens_sealed"] * world / (cfg4["seal_ms"] * 1e-3) / 1e6,
                          "ms": cfg4["seal_ms"], "tokens_per_gpu": cfg4["tokens_sealed"],
                          "what": "every layer's slice sealed from its staging buffer, one launch per layer; time = max over ranks"},
            "groups_per_rank": cfg4["groups_per_rank"], "exchange_bytes_per_rank": cfg4["exchange"],
            "merged_vs_whole_max_rel_err": cfg4["merged_vs_whole"],
            "scaling": "strong (fixed sequence)", "write_s": cfg4["write_s"]},
        "config3": None if cfg3 is None else {
            "workload": f"config 3: paged pool of {cfg3['n_total']} sequences (contexts U[8K, 64K], seed 3), 3/3 trellis, tail "
                        f"4096 -> 8192, sink 128, 16 layers, decode width 1; sequences split over {world} rank(s) by LPT on "
                        "context; one step = 1 appended token per sequence and layer (sealing as the policy says) + 1 "
                        "batched attention call per layer; the window holds the pool's first policy-triggered seals",
            "metric": f"decode tokens/s ({cfg3['n_total']} per step)", "value": cfg3["n_total"] / (cfg3["ms"] * 1e-3),
            "unit": "tok/s", "ms_per_step": cfg3["ms"], "ms_max_step": cfg3["ms_max_step"], "steps": cfg3["steps"],
            "steps_with_seal": cfg3["seal_steps"], "seal_records_in_window": cfg3["seal_records"],
            "untimed_steps_before_window": cfg3["skip_steps"],
            "attn_ms_per_step": cfg3["ms_attn"], "attn_bytes_per_step": cfg3["attn_bytes"],
            "attn_gbs": cfg3["attn_bytes"] / (cfg3["ms_attn"] * 1e-3) / 1e9,
            "attn_frac_of_all_ranks": cfg3["attn_bytes"] / (cfg3["ms_attn"] * 1e-3) / 1e9 / (peak * world),
            "step_gbs": cfg3["step_bytes"] / (cfg3["ms"] * 1e-3) / 1e9, "ctx_total": cfg3["ctx_total"],
            "seqs_rank0": cfg3["seqs"], "gpu_launches_per_step": cfg3["launches_per_step"],
            "kernel": "sjk_attend_batch: attend_trellis_ws_kernel (all records of all sequences) + attend_dense_tc_kernel "
                      "(sinks + staging rings) + attend_batch_merge_kernel; store_batch_kernel; seal_kernel on seal steps",
            "scaling": f"strong (fixed {cfg3['n_total']} sequences)", "device_status": cfg3["device_status"],
            "build_s": cfg3["build_s"]},
        "cpu_baseline": None,
        "build_s": c1["build_s"],
    }
    if cpu:
        c = cpu["c1"]
        cb = {"value": c["us_call"], "unit": "us/call", "cores": c["threads"], "kind": "reference",
              "sample": f"{c['pairs']} of the 64 (query row, query head) pairs of config 1's layer 0 at the full 100K context "
                        f"(sj_kvarn_layer_attend_row over a cache built with the reference's own calls from the same "
                        f"seeded rows), {c['t']:.2f} s on {c['threads']} threads, scaled x{64 / c['pairs']:g}",
              "wall_s": cpu["wall_s"]}
        s0 = cpu["s0"]
        cb["seal_config0"] = {"unit": "Mtok/s", "single_thread": 4096 / s0["single_s"] / 1e6,
                              "all_cores": 4096 / s0["mt_s"] / 1e6, "cores": s0["threads"],
                              "sample": "the whole 4096-token commit (128 records): sj_kvarn_layer_seal on one thread; "
                                        "the threaded harness over sj_kvarn_seal_group on all cores"}
        if cpu.get("c2"):
            cb["config2"] = {"attn_us_per_call": cpu["c2"]["us_call"], "cores": cpu["c2"]["threads"],
                             "seal_mtoks_all_cores": 4096 / cpu["s2"]["mt_s"] / 1e6,
                             "sample": "16 of 64 pairs at 32K (scaled x4); the whole 3/2t commit (128 records) on all cores"}
        if cpu.get("c3"):
            c = cpu["c3"]
            cb["config3"] = {"tok_s": c["tok_s"], "ms_step": c["ms_step"], "cores": c["threads"],
                             "sample": f"sequence {c['sample_seq']} of the pool ({c['sample_ctx']} tokens, 3/3t, 1 layer): "
                                       f"its {c['seal_records']} seals and 16 attention pairs; extrapolated to 64 sequences x "
                                       "16 layers by context, plus seals at the pool's steady rate"}
        if cpu.get("c4"):
            c = cpu["c4"]
            cb["config4"] = {"attn_us_per_call": c["us_call"], "seal_mtoks": c["seal_mtoks"], "cores": c["threads"],
                             "sample": f"groups [0, 1024) of layer 0 with the sink ({c['sample_ctx']} positions): its "
                                       f"{c['seal_records']} seals and 16 of 64 attention pairs, scaled x4 and by context x8.2"}
        line["cpu_baseline"] = cb
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
