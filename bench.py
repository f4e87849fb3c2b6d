#!/usr/bin/env python
"""bench.py - B200 benchmark of the SJ-KVaRN hot path (one JSON line on rank 0).

Headline workload: decode attention at 100K context over a 4/4 scalar body, 16 layers,
4 KV heads of D = 256, 16 query heads (GQA 4), decode width 4, batch 1. The cache is built on the GPU through
the adaptive-tail policy in 512-token ubatches (store = Hadamard + tq6_0 ring write, seal from the ring), then
idled at 97,920 (B = 93,824) and stored on to N = 100,000, so the tq6_0 tail holds 6,176 positions (the nearest
group-aligned tail to the config's 6,144). A step = one attention call per layer over all 16 layers.

  value    device time per layer call (us), inputs resident in HBM; CUDA events on the launching stream
  e2e      the same through the C-ABI with HOST buffers: per step the queries go host->device from pinned memory
           and the outputs come back, inside the timed region (layer by layer on two copy streams, overlapping the
           attention of the neighbouring layers)
  seal     BASELINE config 0: seal one 4096-token commit (32 groups x 4 heads = 128 records, 4/4) out of an
           8,320-position tq6_0 ring; Mtok/s = 4096 / time; plus the ring write of those 8,320 positions
  cpu_baseline  the reference's own CPU attention (oracle/_ref, sj_kvarn_layer_attend_row) on the host cores, on
           a sample of the (query row, query head) pairs of one layer call at the full 100K context

--impl reference times only the reference CPU path (rank 0; other ranks exit 0).
Multi-GPU (torchrun): every rank serves its own config-1 sequence (weak scaling, no collective on the data path);
value is the max over ranks.
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "sj-kvarn-codec_b200")
for _p in (PKG, os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "decode-attn µs/call @100K ctx"
CFG1 = dict(D=256, H=4, HQ=16, NQ=4, LAYERS=16, N=100000, IDLE_AT=97920, TAIL=4096, TAIL_MAX=8192, N_UB=512, SINK=128)
SCALE = 1.0 / 16.0          # 1/sqrt(D)


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        return {}


def hbm_peak():
    p = peaks().get("hbm_gbs")
    return (float(p), "measured") if p else (6650.0, "fallback")


def attn_bytes_per_call(B, N, D=256, H=4, nq=4, hq=16, rec_bytes=35072, sink=128, stage=196):
    body = (B - sink) // 128 * H * rec_bytes
    tail = (N - B) * H * 2 * stage
    sk = sink * H * D * 4
    qo = 2 * nq * hq * D * 4
    return body + tail + sk + qo


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


# ---------------------------------------------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------------------------------------------
class GpuModel:
    """16 device layer caches of one sequence + its policy, filled with seeded synthetic K/V on the GPU."""

    def __init__(self, torch, L, seed, stream, layers=CFG1["LAYERS"], n_ctx=CFG1["N"], bits=(4, 4), body=2, heavy=False):
        import sjk
        import synth
        self.T, self.L, self.sjk, self.st = torch, L, sjk, stream
        c = CFG1
        self.cfg = sjk.config(c["D"], c["H"], n_ctx, c["N_UB"], bits_k=bits[0], bits_v=bits[1], body=body,
                              tail=c["TAIL"], tail_max=c["TAIL_MAX"])
        self.layers = [sjk.Layer() for _ in range(layers)]
        for lay in self.layers:
            sjk.check(L.sj_kvarn_layer_init(C.byref(lay), C.byref(self.cfg)), "layer_init")
        self.pol = sjk.Policy()
        L.sj_kvarn_policy_init(C.byref(self.pol), c["SINK"], c["TAIL"], c["TAIL_MAX"], 128, 0)
        kv = synth.KVStream(seed, layers, c["H"], c["D"], heavy=heavy)
        self.scale = torch.from_numpy(kv.scale).cuda()
        self.gens = [torch.Generator(device="cuda").manual_seed(seed * 1009 + il) for il in range(layers)]
        self.heavy = heavy
        self.n = 0
        self.sealed_records = 0

    def _rows(self, il, n):
        T, c = self.T, CFG1
        g = self.gens[il]
        x = T.randn((n, c["H"], c["D"]), generator=g, device="cuda")
        if self.heavy:   # Student-t(4) = N / sqrt(chi2_4 / 4)
            chi = (T.randn((n, c["H"], c["D"], 4), generator=g, device="cuda") ** 2).sum(-1)
            x = x / T.sqrt(chi / 4)
        k = (x * self.scale[il][None]).contiguous()
        v = T.randn((n, c["H"], c["D"]), generator=g, device="cuda")
        return k, v

    def seal_pending(self):
        p = self.pol
        if p.B_pending > p.B:
            for lay in self.layers:
                self.sjk.check(self.L.sjk_layer_seal(C.byref(lay), p.B, p.B_pending, self.st), "seal")
            self.sealed_records += (p.B_pending - p.B) // 128 * CFG1["H"] * len(self.layers)
        self.L.sj_kvarn_policy_commit(C.byref(p))

    def store(self, pos0, n):
        with self.T.cuda.stream(self.T.cuda.ExternalStream(self.st.value) if self.st and self.st.value else self.T.cuda.current_stream()):
            for il, lay in enumerate(self.layers):
                k, v = self._rows(il, n)
                self.sjk.check(self.L.sjk_layer_store(C.byref(lay), pos0, n, C.c_void_p(k.data_ptr()),
                                                      C.c_void_p(v.data_ptr()), 1, self.st), "store")
        self.n = max(self.n, pos0 + n)

    def grow(self, to, n_ub=CFG1["N_UB"]):
        pos = self.n
        while pos < to:
            n = min(n_ub, to - pos)
            self.L.sj_kvarn_policy_begin_ubatch(C.byref(self.pol), pos, n)
            self.seal_pending()
            self.store(pos, n)
            pos += n

    def idle(self, keep=0):
        self.L.sj_kvarn_policy_idle(C.byref(self.pol), self.n, keep)
        self.seal_pending()

    def free(self):
        for lay in self.layers:
            self.L.sj_kvarn_layer_free(C.byref(lay))


def build_config1(torch, L, seed, stream):
    m = GpuModel(torch, L, seed, stream)
    m.grow(CFG1["IDLE_AT"])
    m.idle(0)
    m.grow(CFG1["N"])
    torch.cuda.synchronize()
    assert m.pol.B == 93824, m.pol.B
    return m


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


def run_gpu_arm(args, torch, dist, rank, world, local_rank):
    import sjk
    import synth
    L = sjk.lib()
    s = torch.cuda.Stream()
    st = C.c_void_p(s.cuda_stream)
    t_build = time.time()
    m = build_config1(torch, L, seed=1 + rank, stream=st)
    build_s = time.time() - t_build
    c = CFG1
    n_q, n_head, D, N = c["NQ"], c["HQ"], c["D"], c["N"]
    B = m.pol.B
    q = torch.from_numpy(synth.queries(1 + rank, c["LAYERS"], n_q, n_head, D)).cuda()
    sjk.check(L.sjk_hadamard(C.c_void_p(q.data_ptr()), c["LAYERS"] * n_q * n_head, D, None))
    out = torch.empty_like(q)
    torch.cuda.synchronize()
    per = n_q * n_head * D

    def step():
        for il, lay in enumerate(m.layers):
            rc = L.sjk_layer_attend(C.byref(lay), B, N, N - n_q, n_q, n_head, C.c_void_p(q.data_ptr() + il * per * 4),
                                    SCALE, C.c_void_p(out.data_ptr() + il * per * 4), st)
            if rc:
                raise sjk.SjkError(rc, "attend")

    barrier = (lambda: dist.barrier()) if dist else None
    with Clocks(local_rank) as clk:
        ms = time_events(torch, s, step, args.steps, args.warmup, barrier)
    # end to end: host queries in, host outputs back, every step
    q_h = q.cpu().pin_memory()
    out_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    # every step, the queries go host -> device and the outputs come back, layer by layer on two copy streams: layer
    # il's copy in overlaps the attention of the layers before it and its copy out the layers after it; the step ends
    # on `s` once the last output has landed in host memory
    cs_in, cs_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(c["LAYERS"])]
    ev_out = [torch.cuda.Event() for _ in range(c["LAYERS"])]

    def step_e2e():
        cs_in.wait_stream(s)                                   # the previous step's reads of q are done
        for il, lay in enumerate(m.layers):
            with torch.cuda.stream(cs_in):
                q[il].copy_(q_h[il], non_blocking=True)
                ev_in[il].record(cs_in)
            s.wait_event(ev_in[il])
            rc = L.sjk_layer_attend(C.byref(lay), B, N, N - n_q, n_q, n_head, C.c_void_p(q.data_ptr() + il * per * 4),
                                    SCALE, C.c_void_p(out.data_ptr() + il * per * 4), st)
            if rc:
                raise sjk.SjkError(rc, "attend")
            ev_out[il].record(s)
            cs_out.wait_event(ev_out[il])
            with torch.cuda.stream(cs_out):
                out_h[il].copy_(out[il], non_blocking=True)
        s.wait_stream(cs_out)

    ms_e2e = time_events(torch, s, step_e2e, args.steps, args.warmup, barrier)
    if dist:
        t = torch.tensor([ms, ms_e2e], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])
    res = dict(ms=ms, ms_e2e=ms_e2e, B=B, build_s=build_s, clocks=clk.summary(), h2d=q.numel() * 4, d2h=out.numel() * 4,
               launches_per_step=2 * c["LAYERS"], sealed_records=m.sealed_records)
    m.free()
    return res


def run_seal(args, torch, L, stream_obj):
    """1 layer, 8,320 positions through the tq6_0 ring, then one 4096-token commit (4/4)."""
    import sjk
    st = C.c_void_p(stream_obj.cuda_stream)
    m = GpuModel(torch, L, seed=0, stream=st, layers=1, n_ctx=16384)
    m.grow(8320)
    m.L.sj_kvarn_policy_begin_ubatch(C.byref(m.pol), 8320, 512)
    B0, B1 = m.pol.B, m.pol.B_pending
    assert (B0, B1) == (128, 4224), (B0, B1)
    lay = m.layers[0]

    def seal():
        rc = L.sjk_layer_seal(C.byref(lay), B0, B1, st)
        if rc:
            raise sjk.SjkError(rc, "seal")

    ms = time_events(torch, stream_obj, seal, max(3, args.steps), args.warmup)
    # ring write of the 8,320 positions (store kernel, Hadamard fused), inputs resident
    k, v = m._rows(0, 8320)
    torch.cuda.synchronize()

    def store():
        rc = L.sjk_layer_store(C.byref(lay), 0, 8320, C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()), 1, st)
        if rc:
            raise sjk.SjkError(rc, "store")

    ms_store = time_events(torch, stream_obj, store, max(3, args.steps), args.warmup)
    m.free()
    return dict(ms=ms, ms_store=ms_store, records=(B1 - B0) // 128 * 4)


CFG2 = dict(LAYERS=4, N=32768, TAIL=4096, TAIL_MAX=8192, N_UB=512)


def run_config2(args, torch, L, stream_obj):
    """BASELINE config 2 (3/2 trellis): the per-layer seal of one 4096-token commit, and decode attention at 32K
    context (B = 28,672 after idling at 32,768, tail 4,096). K is Student-t(4) before the channel scales. The
    attention metric is per layer call, so 4 layers stand in for the model's 16."""
    import sjk
    import synth
    st = C.c_void_p(stream_obj.cuda_stream)
    c, c2 = CFG1, CFG2
    t0 = time.time()
    m = GpuModel(torch, L, seed=2, stream=st, layers=c2["LAYERS"], n_ctx=c2["N"] + 1024, bits=(3, 2), body=2, heavy=True)
    m.grow(c2["N"])
    m.idle(0)
    torch.cuda.synchronize()
    B, N = m.pol.B, c2["N"]
    assert B == 28672, B
    build_s = time.time() - t0
    n_q, n_head, D = c["NQ"], c["HQ"], c["D"]
    q = torch.from_numpy(synth.queries(2, c2["LAYERS"], n_q, n_head, D)).cuda()
    out = torch.empty_like(q)
    per = n_q * n_head * D

    def step():
        for il, lay in enumerate(m.layers):
            rc = L.sjk_layer_attend(C.byref(lay), B, N, N - n_q, n_q, n_head, C.c_void_p(q.data_ptr() + il * per * 4),
                                    SCALE, C.c_void_p(out.data_ptr() + il * per * 4), st)
            if rc:
                raise sjk.SjkError(rc, "attend")

    ms = time_events(torch, stream_obj, step, max(3, args.steps), args.warmup)
    m.free()
    # the seal of one 4096-token commit (32 groups x 4 heads, 3/2 trellis) out of an 8,320-position ring
    ms_seal = None
    s = GpuModel(torch, L, seed=2, stream=st, layers=1, n_ctx=16384, bits=(3, 2), body=2, heavy=True)
    s.grow(8320)
    s.L.sj_kvarn_policy_begin_ubatch(C.byref(s.pol), 8320, 512)
    B0, B1 = s.pol.B, s.pol.B_pending
    lay = s.layers[0]

    def seal():
        rc = L.sjk_layer_seal(C.byref(lay), B0, B1, st)
        if rc:
            raise sjk.SjkError(rc, "seal")

    ms_seal = time_events(torch, stream_obj, seal, 3, 1)
    s.free()
    abytes = attn_bytes_per_call(B, N, rec_bytes=22784)
    return dict(ms=ms / c2["LAYERS"], B=B, N=N, bytes=abytes, ms_seal=ms_seal, records=(B1 - B0) // 128 * 4, build_s=build_s)


CFG4 = dict(LAYERS=2, GROUPS=8192, TAIL=4096)


def run_config4(args, torch, L, stream_obj, dist, rank, world):
    """one sequence of 1,048,576 sealed tokens (8,192 groups per KV head and layer) plus the
    128-token sink and a 4,096-token tail, split by context slice across the ranks. Rank r holds groups
    [8192 r / W, 8192 (r + 1) / W) of every layer; rank 0 also holds the sink, the last rank the tail. Per layer
    call every rank attends over its own regions (sjk_attend_partial), the (m, l, o) triples are all-gathered
    over NCCL and merged in rank order (sjk_attend_merge); every rank ends with the whole output. The metric is
    per layer call, so 2 layers stand in for 16. Each rank's slice holds its own seeded synthetic K/V."""
    import sjk
    import slices
    import synth
    st = C.c_void_p(stream_obj.cuda_stream)
    c, c4 = CFG1, CFG4
    g0, g1 = slices.group_range(rank, world, c4["GROUPS"])
    n_local = c["SINK"] + (g1 - g0) * 128 + c4["TAIL"]
    t0 = time.time()
    m = GpuModel(torch, L, seed=4000 + rank, stream=st, layers=c4["LAYERS"], n_ctx=n_local + 1024)
    m.grow(n_local)
    m.idle(c4["TAIL"])
    torch.cuda.synchronize()
    B = m.pol.B
    assert B == c["SINK"] + (g1 - g0) * 128, B
    build_s = time.time() - t0
    n_q, n_head, D = c["NQ"], c["HQ"], c["D"]
    n_global = c["SINK"] + c4["GROUPS"] * 128 + c4["TAIL"]
    qpos0 = n_global - n_q
    rows, per = n_q * n_head, n_q * n_head * D
    q = torch.from_numpy(synth.queries(4, c4["LAYERS"], n_q, n_head, D)).cuda()
    out = torch.empty_like(q)
    views = [sjk.view_of(lay) for lay in m.layers]
    need = L.sjk_attend_scratch_bytes(C.byref(views[0]), n_local, n_q, n_head)
    scratch = torch.empty(int(need), dtype=torch.uint8, device="cuda")
    part = torch.empty((rows, D + 2), dtype=torch.float32, device="cuda")
    reg = slices.regions(rank, world)

    def step():
        with torch.cuda.stream(stream_obj):
            for il in range(c4["LAYERS"]):
                rc = L.sjk_attend_partial(C.byref(views[il]), B, n_local, qpos0, n_q, n_head, reg,
                                          C.c_void_p(q.data_ptr() + il * per * 4), SCALE, C.c_void_p(part.data_ptr()),
                                          C.c_void_p(scratch.data_ptr()), need, st)
                if rc:
                    raise sjk.SjkError(rc, "attend_partial")
                allp = slices.gather(dist, part) if dist else part[None]
                rc = L.sjk_attend_merge(C.c_void_p(allp.data_ptr()), world, rows, D, C.c_void_p(out.data_ptr() + il * per * 4), st)
                if rc:
                    raise sjk.SjkError(rc, "attend_merge")

    barrier = (lambda: dist.barrier()) if dist else None
    ms = time_events(torch, stream_obj, step, max(3, args.steps), args.warmup, barrier)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    m.free()
    B_global = c["SINK"] + c4["GROUPS"] * 128
    return dict(ms=ms / c4["LAYERS"], bytes=attn_bytes_per_call(B_global, n_global), n_ctx=n_global, build_s=build_s,
                exchange=rows * (D + 2) * 4, groups_per_rank=g1 - g0)


CFG3 = dict(SEQS=64, CTX_LO=8192, CTX_HI=65536, LAYERS=16, NQ=1, ROWS=8192, MAX_STEPS=10)


def run_config3(args, torch, L, stream_obj, dist, rank, world):
    """a paged record pool of 64 sequences (contexts uniform in [8K, 64K], seed 3), 3/3 trellis
    body, adaptive tail 4096 -> 8192, fp16 sink 128, 16 layers, decode width 1 (16 query heads, GQA 4). The sequences
    are assigned to the ranks by longest-processing-time on their contexts (slices.lpt_assign) and every rank builds
    its own in one pool through the product's sequence API (sj_kvarn_seq_begin_ubatch: policy, block reservation and
    seals; sjk_seq_store: the ring / sink writes of each 512-token ubatch). One step appends one token to every
    sequence of every layer (sj_kvarn_seq_begin_ubatch, sealing where the policy says, then one sjk_store_batch
    launch for all (sequence, layer) pairs) and runs one sjk_attend_batch call per layer over all the rank's
    sequences. K/V rows come from 8,192 seeded rows per layer drawn from config 0's distribution, reused cyclically."""
    import numpy as np
    import sjk
    st = C.c_void_p(stream_obj.cuda_stream)
    c, c3 = CFG1, CFG3
    import slices
    H, D, HQ, NL, NQ, R = c["H"], c["D"], c["HQ"], c3["LAYERS"], c3["NQ"], c3["ROWS"]
    ctx = np.random.default_rng(3).integers(c3["CTX_LO"], c3["CTX_HI"] + 1, size=c3["SEQS"])[:args.config3_seqs]
    owner = slices.lpt_assign(ctx, world)
    mine = [i for i in range(len(ctx)) if owner[i] == rank]
    steps = min(max(3, args.steps), c3["MAX_STEPS"])
    extra = args.warmup + steps + 8
    t0 = time.time()
    cfg = sjk.config(D, H, int(ctx.max()) + extra + 1024, c["N_UB"], bits_k=3, bits_v=3, body=1, tail=c["TAIL"],
                     tail_max=c["TAIL_MAX"])
    pool = sjk.Pool()
    n_blocks = sum((int(ctx[i]) + extra) // 128 + 2 for i in mine)
    sjk.check(L.sj_kvarn_pool_init(C.byref(pool), C.byref(cfg), NL, n_blocks), "pool_init")
    seqs = []
    for i in mine:
        s = sjk.Seq()
        sjk.check(L.sj_kvarn_seq_init(C.byref(s), C.byref(cfg), NL, C.byref(pool)), "seq_init")
        s.stream = st.value
        seqs.append(s)
    # seeded rows of config 0's distribution, [NL][R][H][D]
    import synth
    kvs = synth.KVStream(3000 + rank, NL, H, D)
    gen = torch.Generator(device="cuda").manual_seed(3000 + rank)
    with torch.cuda.stream(stream_obj):
        scale = torch.from_numpy(kvs.scale).cuda()
        krows = (torch.randn((NL, R, H, D), generator=gen, device="cuda") * scale[:, None]).contiguous()
        vrows = torch.randn((NL, R, H, D), generator=gen, device="cuda")
    lstride = R * H * D
    n_ub = c["N_UB"]
    for j, s in enumerate(seqs):
        target, pos = int(ctx[mine[j]]), 0
        while pos < target:
            n = min(n_ub, target - pos)
            sjk.check(L.sj_kvarn_seq_begin_ubatch(C.byref(s), pos, n), "seq_begin_ubatch")
            o = (pos * 7 + 1031 * j) % (R - n_ub)
            sjk.check(L.sjk_seq_store(C.byref(s), pos, n, C.c_void_p(krows.data_ptr() + o * H * D * 4),
                                      C.c_void_p(vrows.data_ptr() + o * H * D * 4), lstride, 1, st), "seq_store")
            pos += n
    torch.cuda.synchronize()
    build_s = time.time() - t0
    n_seq = len(seqs)
    # static views: per layer over the rank's sequences; the store items are (sequence, layer) pairs
    views = [(sjk.View * n_seq)() for _ in range(NL)]
    store_views = (sjk.View * (n_seq * NL))()
    for j, s in enumerate(seqs):
        for il in range(NL):
            L.sjk_layer_view(C.byref(s.layers[il]), C.byref(views[il][j]))
            L.sjk_layer_view(C.byref(s.layers[il]), C.byref(store_views[j * NL + il]))
    idx = torch.arange(n_seq * NL, device="cuda")
    k_step = krows.view(NL, R, H, D)[idx % NL, (idx * 13) % R].contiguous()      # [items][H][D]
    v_step = vrows.view(NL, R, H, D)[idx % NL, (idx * 13) % R].contiguous()
    q = torch.randn((NL, n_seq, NQ, HQ, D), generator=gen, device="cuda")
    sjk.check(L.sjk_hadamard(C.c_void_p(q.data_ptr()), NL * n_seq * NQ * HQ, D, None))
    out = torch.empty_like(q)
    per_layer = n_seq * NQ * HQ * D * 4
    need = L.sjk_attend_batch_scratch_bytes(C.byref(views[0][0]), max(n_seq, 1), NQ, HQ)
    scratch = torch.empty(int(need), dtype=torch.uint8, device="cuda")
    Bs, Ns, Qs = (C.c_uint32 * n_seq)(), (C.c_uint32 * n_seq)(), (C.c_uint32 * n_seq)()
    pos_items = (C.c_uint32 * (n_seq * NL))()
    stats = dict(seal_steps=0, bytes=0)
    torch.cuda.synchronize()

    def step():
        sealed = False
        for j, s in enumerate(seqs):
            B_before = s.pol.B
            sjk.check(L.sj_kvarn_seq_begin_ubatch(C.byref(s), s.n, 1), "seq_begin_ubatch")
            sealed |= s.pol.B != B_before
            for il in range(NL):
                pos_items[j * NL + il] = s.n
        sjk.check(L.sjk_store_batch(store_views, pos_items, n_seq * NL, C.c_void_p(k_step.data_ptr()),
                                    C.c_void_p(v_step.data_ptr()), 1, st), "store_batch")
        for j, s in enumerate(seqs):
            s.n = s.n + 1
            Bs[j], Ns[j], Qs[j] = s.pol.B, s.n, s.n - 1
        stats["seal_steps"] += int(sealed)
        for il in range(NL):
            rc = L.sjk_attend_batch(views[il], Bs, Ns, Qs, n_seq, NQ, HQ, C.c_void_p(q.data_ptr() + il * per_layer), SCALE,
                                    C.c_void_p(out.data_ptr() + il * per_layer), C.c_void_p(scratch.data_ptr()), need, st)
            if rc:
                raise sjk.SjkError(rc, "attend_batch")

    def step_bytes():
        # algorithmic bytes of one step's attention: every record, staged row and sink row of every sequence and layer
        tot = 0
        for s in seqs:
            B, N = s.pol.B, s.n
            tot += (B - 128) // 128 * H * 26880 + (N - B) * H * 392 + 128 * H * 1024 + 2 * NQ * HQ * D * 4
        return tot * NL

    barrier = (lambda: dist.barrier()) if dist else None
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if barrier:
        barrier()
    stats["seal_steps"] = 0
    b0 = step_bytes()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream_obj)
    for _ in range(steps):
        step()
    e1.record(stream_obj)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    b1 = step_bytes()
    # attention alone (no appends), the same call shapes: bytes per step / time
    def attend_only():
        for il in range(NL):
            rc = L.sjk_attend_batch(views[il], Bs, Ns, Qs, n_seq, NQ, HQ, C.c_void_p(q.data_ptr() + il * per_layer), SCALE,
                                    C.c_void_p(out.data_ptr() + il * per_layer), C.c_void_p(scratch.data_ptr()), need, st)
            if rc:
                raise sjk.SjkError(rc, "attend_batch")

    ms_attn = time_events(torch, stream_obj, attend_only, steps, 2, barrier)
    abytes = step_bytes()
    if dist:
        t = torch.tensor([ms, ms_attn], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tb = torch.tensor([float(abytes), float((b0 + b1) / 2)], device="cuda", dtype=torch.float64)
        dist.all_reduce(tb, op=dist.ReduceOp.SUM)
        ms, ms_attn = float(t[0]), float(t[1])
        abytes, sbytes = float(tb[0]), float(tb[1])
    else:
        sbytes = (b0 + b1) / 2
    status = L.sjk_device_status()
    for s in seqs:
        L.sj_kvarn_seq_free(C.byref(s))
    L.sj_kvarn_pool_free(C.byref(pool))
    del krows, vrows, scratch
    return dict(ms=ms, ms_attn=ms_attn, attn_bytes=abytes, step_bytes=sbytes, seqs=n_seq, steps=steps,
                seal_steps=stats["seal_steps"], build_s=build_s, ctx_total=int(ctx.sum()), device_status=status, n_total=len(ctx),
                launches_per_step=1 + 3 * NL)


# ---------------------------------------------------------------------------------------------------------------
# reference CPU path (oracle/_ref: the reference sj_kvarn.h compiled from its own source)
# ---------------------------------------------------------------------------------------------------------------
class CpuReference:
    """One layer of the config-1 cache built on the host with the reference's public calls (rotation, store,
    seal of each record from its unstaged fp16 rows), spread over the host cores; then timed attention rows."""

    def __init__(self, n_threads=0, n_ctx=CFG1["N"], idle_at=CFG1["IDLE_AT"], seed=11):
        import numpy as np

        import oracle
        import sjk
        import synth
        self.np = np
        self.kind = "reference" if oracle.ref_available() else "port"
        c = CFG1
        self.cfg = sjk.config(c["D"], c["H"], n_ctx, c["N_UB"], tail=c["TAIL"], tail_max=c["TAIL_MAX"])
        if self.kind == "reference":
            R = oracle.ref()
            self.R = R
            R.sjref_layer_new.restype = C.c_void_p
            R.sjref_layer_new.argtypes = [C.c_void_p, C.POINTER(C.c_int)]
            R.sjref_layer_store_mt.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_int]
            R.sjref_rotate_mt.argtypes = [C.c_void_p, C.c_size_t, C.c_int, C.c_int]
            R.sjref_layer_seal_mt.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_int]
            R.sj_kvarn_layer_attend_row.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_int, C.c_uint32,
                                                    C.c_float, C.c_void_p]
            R.sjref_layer_delete.argtypes = [C.c_void_p]
            R.sj_kvarn_policy_init.argtypes = [C.c_void_p] + [C.c_uint32] * 5
            R.sj_kvarn_policy_begin_ubatch.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32]
            R.sj_kvarn_policy_commit.argtypes = [C.c_void_p]
            R.sj_kvarn_policy_idle.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32]
            self.threads = R.sjref_nthreads(n_threads)
            rc = C.c_int()
            self.layer = R.sjref_layer_new(C.byref(self.cfg), C.byref(rc))
            if not self.layer:
                raise RuntimeError(f"reference layer_init rc {rc.value}")
        else:
            self.threads = n_threads or os.cpu_count() or 1
            self.oc = oracle.OracleCache(c["D"], c["H"], 4, 4, False, 16, 0, True, c["SINK"], c["TAIL"], c["TAIL_MAX"],
                                         c["N_UB"], n_ctx)
        kv = synth.KVStream(seed, 1, c["H"], c["D"])
        pol = sjk.Policy()
        self.pol = pol
        if self.kind == "reference":
            self.R.sj_kvarn_policy_init(C.byref(pol), c["SINK"], c["TAIL"], c["TAIL_MAX"], 128, 0)
        else:
            sjk.lib().sj_kvarn_policy_init(C.byref(pol), c["SINK"], c["TAIL"], c["TAIL_MAX"], 128, 0)
        t0 = time.time()
        pos = 0
        while pos < n_ctx:
            if pos == idle_at:
                self._policy("idle", pos, 0)
            n = min(c["N_UB"], (idle_at if pos < idle_at else n_ctx) - pos)
            self._policy("begin", pos, n)          # seal what is due before this ubatch is stored
            k, v = kv.rows(pos, n, layer=0)
            self._store(pos, n, k, v)
            pos += n
        self.B, self.N = pol.B, n_ctx
        self.build_s = time.time() - t0

    def _policy(self, what, a, b):
        import sjk
        lib = self.R if self.kind == "reference" else sjk.lib()
        if what == "begin":
            lib.sj_kvarn_policy_begin_ubatch(C.byref(self.pol), a, b)
        else:
            lib.sj_kvarn_policy_idle(C.byref(self.pol), a, b)
        if self.pol.B_pending > self.pol.B:
            if self.kind == "reference":
                self.R.sjref_layer_seal_mt(self.layer, self.pol.B, self.pol.B_pending, self.threads)
            else:
                self.oc.seal(self.pol.B, self.pol.B_pending, self.threads)
        lib.sj_kvarn_policy_commit(C.byref(self.pol))

    def _store(self, pos, n, k, v):
        np = self.np
        k = np.ascontiguousarray(k); v = np.ascontiguousarray(v)
        if self.kind == "reference":
            self.R.sjref_rotate_mt(k.ctypes.data, k.size // CFG1["D"], CFG1["D"], self.threads)
            self.R.sjref_rotate_mt(v.ctypes.data, v.size // CFG1["D"], CFG1["D"], self.threads)
            self.R.sjref_layer_store_mt(self.layer, pos, n, k.ctypes.data, v.ctypes.data, self.threads)
        else:
            import oracle
            oracle.fwht_rows(k); oracle.fwht_rows(v)
            for i in range(n):
                self.oc.store(pos + i, k[i], v[i])

    def attend_pairs(self, pairs, q):
        """Attention of the given (row, query head) pairs, spread over the host threads; returns seconds."""
        from concurrent.futures import ThreadPoolExecutor
        np = self.np
        outs = {p: np.zeros(CFG1["D"], np.float32) for p in pairs}
        grp = CFG1["HQ"] // CFG1["H"]
        N = self.N

        def one(p):
            iq, hq = p
            qr = np.ascontiguousarray(q[iq, hq])
            if self.kind == "reference":
                self.R.sj_kvarn_layer_attend_row(self.layer, self.B, N, qr.ctypes.data, hq // grp, N - CFG1["NQ"] + iq,
                                                 SCALE, outs[p].ctypes.data)
            else:
                import oracle
                oracle.lib().ora_attend_row(C.byref(self.oc.c), self.B, N, qr, hq // grp, N - CFG1["NQ"] + iq,
                                            SCALE, outs[p])

        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=self.threads) as ex:
            list(ex.map(one, pairs))
        return time.perf_counter() - t0

    def close(self):
        if self.kind == "reference":
            self.R.sjref_layer_delete(self.layer)
        else:
            self.oc.close()


def sample_pairs(n):
    """n (query row, query head) pairs spread evenly over the 64 pairs of a call and over all KV heads."""
    allp = [(iq, hq) for hq in range(CFG1["HQ"]) for iq in range(CFG1["NQ"])]
    stride = max(1, len(allp) // n)
    return allp[::stride][:n]


def cpu_queries():
    import oracle
    import synth
    q = synth.queries(7, 1, CFG1["NQ"], CFG1["HQ"], CFG1["D"])[0]
    return oracle.fwht_rows(q.copy())


def run_reference_arm(args):
    ref = CpuReference(n_threads=args.cpu_threads)
    q = cpu_queries()
    pairs = sample_pairs(args.ref_pairs)
    for _ in range(min(args.warmup, 1)):
        ref.attend_pairs(pairs[:ref.threads], q)
    times = [ref.attend_pairs(pairs, q) for _ in range(args.steps)]
    per_call_us = statistics.mean(times) * 1e6 * (CFG1["NQ"] * CFG1["HQ"]) / len(pairs)
    sample = (f"{len(pairs)} of the 64 (query row, query head) pairs of one layer call at N=100,000 "
              f"(B=93,824, 4/4 body, tq6_0 tail of 6,176), per step; scaled x{64 / len(pairs):g} to a full call; "
              f"cache built with the reference's own calls in {ref.build_s:.1f} s")
    line = {"impl": "reference", "metric": METRIC, "value": per_call_us, "unit": "us/call", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.mean(times) * 1e3,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config 1: decode attention, 100K ctx, 4/4 scalar body, 1 layer call (sampled)",
                       "n_ctx": CFG1["N"], "B": ref.B, "layers": 1, "kv_heads": 4, "q_heads": 16, "head_dim": 256,
                       "decode_width": 4, "parallelism": "host threads"},
            "cpu_baseline": {"value": per_call_us, "unit": "us/call", "cores": ref.threads, "kind": ref.kind,
                             "sample": sample},
            "e2e": {"value": per_call_us, "unit": "us/call", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    ref.close()
    print(json.dumps(line), flush=True)


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
    ap.add_argument("--no-config2", action="store_true", help="skip the config-2 (3/2 trellis) side measurement")
    ap.add_argument("--no-config4", action="store_true", help="skip the config-4 (1M context sliced over the ranks) measurement")
    ap.add_argument("--no-config3", action="store_true", help="skip the config-3 (64-sequence paged pool) measurement")
    ap.add_argument("--config3-seqs", type=int, default=CFG3["SEQS"],
                    help="sequences of the config-3 pool (the first N of its 64; fewer only for small profiling runs)")
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
    res = run_gpu_arm(args, torch, dist, rank, world, local_rank)
    cfg4 = None if args.no_config4 else run_config4(args, torch, sjk.lib(), torch.cuda.Stream(), dist, rank, world)
    cfg3 = None if args.no_config3 else run_config3(args, torch, sjk.lib(), torch.cuda.Stream(), dist, rank, world)
    seal = run_seal(args, torch, sjk.lib(), torch.cuda.Stream()) if rank == 0 else None
    cfg2 = run_config2(args, torch, sjk.lib(), torch.cuda.Stream()) if rank == 0 and not args.no_config2 else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ref = CpuReference(n_threads=args.cpu_threads)
        pairs = sample_pairs(16)
        t = ref.attend_pairs(pairs, cpu_queries())
        v = t * 1e6 * 64 / len(pairs)
        cpu = {"value": v, "unit": "us/call", "cores": ref.threads, "kind": ref.kind,
               "sample": f"{len(pairs)} of the 64 (query row, query head) pairs of one config-1 layer call at the full "
                         f"100K context (reference sj_kvarn_layer_attend_row over a cache built with the reference's "
                         f"own calls), {t:.2f} s on {ref.threads} threads, scaled x{64 / len(pairs):g}"}
        ref.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    c = CFG1
    per_call_ms = res["ms"] / c["LAYERS"]
    us_call = per_call_ms * 1e3
    us_call_e2e = res["ms_e2e"] / c["LAYERS"] * 1e3
    abytes = attn_bytes_per_call(res["B"], c["N"])
    peak, peak_kind = hbm_peak()
    achieved = abytes / (per_call_ms * 1e-3) / 1e9
    traffic = profile_traffic("attend_config1_launches.md")
    seal_mtoks = 4096 / (seal["ms"] * 1e-3) / 1e6
    seal_bytes = seal["records"] * (128 * 392 + 35072)
    store_bytes = 8320 * (2 * 4 * 256 * 4) + 128 * 4 * 1024 + 8192 * 4 * 392
    line = {
        "metric": METRIC, "value": us_call, "unit": "us/call", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": res["ms"], "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) x LogNormal channel scales with outlier channels; V N(0,1); Q N(0,1) fp16)",
        "config": {"workload": "config 1: decode attention, 100K ctx, 4/4 scalar body, 16 layers", "n_ctx": c["N"],
                   "B": res["B"], "tail": c["N"] - res["B"], "sink": c["SINK"], "layers": c["LAYERS"], "kv_heads": c["H"],
                   "q_heads": c["HQ"], "head_dim": c["D"], "decode_width": c["NQ"], "batch": 1,
                   "parallelism": f"sequence replicas x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (16 layers x 113 MB per step)"},
        "e2e": {"value": us_call_e2e, "unit": "us/call", "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"]},
        "gpu_launches": res["launches_per_step"] * args.steps,
        "clocks": res["clocks"],
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "peak_kind": peak_kind, "frac_of_8tbs": achieved / 8000.0,
                     "kernel": "one sjk_attend call: attend_body_tc_kernel (sealed records + sink + staging ring) + attend_merge_kernel",
                     "algorithmic_bytes_per_launch": abytes},
        "seal": {"metric": "seal Mtok/s (4096 commit)", "value": seal_mtoks, "unit": "Mtok/s", "ms": seal["ms"],
                 "workload": "config 0: 1 layer, 4 KV heads, D=256, 4/4, 32 groups x 4 heads from an 8,320-row tq6_0 ring",
                 "hbm_gbs": seal_bytes / (seal["ms"] * 1e-3) / 1e9, "hbm_frac": seal_bytes / (seal["ms"] * 1e-3) / 1e9 / peak,
                 "ring_write_ms": seal["ms_store"],
                 "ring_write_gbs": store_bytes / (seal["ms_store"] * 1e-3) / 1e9},
        "config2": None if cfg2 is None else {
            "workload": "config 2: 3/2 trellis body, decode attention at 32K ctx (B = 28,672, tail 4,096), per layer call; "
                        "seal of one 4096-token commit (128 records, 1 layer)",
            "attn_us_per_call": cfg2["ms"] * 1e3, "attn_bytes_per_call": cfg2["bytes"],
            "attn_gbs": cfg2["bytes"] / (cfg2["ms"] * 1e-3) / 1e9, "attn_frac": cfg2["bytes"] / (cfg2["ms"] * 1e-3) / 1e9 / peak,
            "seal_mtoks": 4096 / (cfg2["ms_seal"] * 1e-3) / 1e6, "seal_ms": cfg2["ms_seal"],
            "seal_hbm_frac": cfg2["records"] * (128 * 392 + 22784) / (cfg2["ms_seal"] * 1e-3) / 1e9 / peak,
            "kernel": "attend_trellis_tc_kernel (sealed records) + attend_dense_tc_kernel (sink + staging ring) + attend_merge_kernel",
            "build_s": cfg2["build_s"]},
        "config4": None if cfg4 is None else {
            "workload": "config 4: one 1,048,576-token sequence (+ 128 sink, 4,096 tail), 4/4, split by context slice over "
                        f"{world} rank(s); per layer call: partial attention per rank + NCCL all-gather of (m, l, o) + merge",
            "attn_us_per_call": cfg4["ms"] * 1e3, "attn_bytes_per_call": cfg4["bytes"], "n_ctx": cfg4["n_ctx"],
            "attn_gbs": cfg4["bytes"] / (cfg4["ms"] * 1e-3) / 1e9,
            "attn_frac_of_all_ranks": cfg4["bytes"] / (cfg4["ms"] * 1e-3) / 1e9 / (peak * world),
            "groups_per_rank": cfg4["groups_per_rank"], "exchange_bytes_per_rank": cfg4["exchange"],
            "scaling": "strong (fixed sequence)", "build_s": cfg4["build_s"]},
        "config3": None if cfg3 is None else {
            "workload": f"config 3: paged pool of {cfg3['n_total']} sequences (contexts U[8K, 64K], seed 3), 3/3 trellis, tail 4096 -> 8192, "
                        f"sink 128, 16 layers, decode width 1; sequences split over {world} rank(s) by LPT on context; one step "
                        "= 1 appended token per sequence and layer (sealing as the policy says) + 1 batched attention call per layer",
            "metric": f"decode tokens/s ({cfg3['n_total']} per step)", "value": cfg3["n_total"] / (cfg3["ms"] * 1e-3), "unit": "tok/s",
            "ms_per_step": cfg3["ms"], "steps": cfg3["steps"], "steps_with_seal": cfg3["seal_steps"],
            "attn_ms_per_step": cfg3["ms_attn"], "attn_bytes_per_step": cfg3["attn_bytes"],
            "attn_gbs": cfg3["attn_bytes"] / (cfg3["ms_attn"] * 1e-3) / 1e9,
            "attn_frac_of_all_ranks": cfg3["attn_bytes"] / (cfg3["ms_attn"] * 1e-3) / 1e9 / (peak * world),
            "step_gbs": cfg3["step_bytes"] / (cfg3["ms"] * 1e-3) / 1e9, "ctx_total": cfg3["ctx_total"],
            "seqs_rank0": cfg3["seqs"], "gpu_launches_per_step": cfg3["launches_per_step"],
            "kernel": "sjk_attend_batch: attend_trellis_ws_kernel (all records of all sequences) + attend_dense_tc_kernel "
                      "(sinks + staging rings) + attend_batch_merge_kernel; store_batch_kernel",
            "scaling": f"strong (fixed {cfg3['n_total']} sequences)", "device_status": cfg3["device_status"], "build_s": cfg3["build_s"]},
        "cpu_baseline": cpu,
        "build_s": res["build_s"],
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
