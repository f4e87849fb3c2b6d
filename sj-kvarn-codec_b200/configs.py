"""The five benchmark configurations and their caches built on the device through the product API.

Every K/V/Q row comes from the seeded generator of libsjk_b200.so (sjk_synth_*; the host build of the same arithmetic
draws identical bits), so a cache built here can be rebuilt on the host through the reference's own calls and
compared byte for byte. Rows are drawn in the model basis and rotated inside the cache write (sjk_store, rotate = 1),
the reference's store path being sj_kvarn_hadamard + sj_kvarn_layer_store (sj_kvarn.h:735-752, 1475-1492).

  config 0  1 layer, H 4, D 256, 4/4 scalar, tail 4096 -> 8192, sink 128, ubatch 512, seed 0: 8,320 positions
            written through the policy (16 ubatches of 512 and one of 128), then the commit of 4,096 tokens that
            begin_ubatch(8320) asks for (B 128 -> 4,224: 32 groups x 4 heads = 128 records)
  config 1  16 layers, 4/4, 100,000 positions built in ubatches of 512 up to 97,920, idled there (B = 93,824),
            stored on to 100,000 (tail 6,176); decode width 4 x 16 query heads; seed 1
  config 2  3/2 trellis, K Student-t(4) before the channel scales; seal of the same 4096-token commit as config 0,
            attention at 32,768 (idle there: B = 28,672, tail 4,096); seed 2
  config 3  pool of 64 sequences, contexts U[8K, 64K] (seed 3), 3/3 trellis, decode width 1
  config 4  one sequence of 8,192 groups per KV head and layer (1,048,576 sealed tokens) + sink 128 + tail 4,096,
            4/4, bulk-sealed from a staging buffer in the ring layout; seed 4

Generator layers: layer il of a configuration draws from generator layer il (K/V, channel scales, queries).
"""
import ctypes as C

import sjk

D, H, HQ, SINK, G = 256, 4, 16, 128, 128
SCALE = 1.0 / 16.0          # 1 / sqrt(D)

CFG0 = dict(seed=0, bits=(4, 4), heavy=False, npos=8320, n_ub=512, tail=4096, tail_max=8192, n_ctx=16384)
CFG1 = dict(seed=1, bits=(4, 4), heavy=False, layers=16, N=100000, idle_at=97920, n_ub=512, tail=4096, tail_max=8192,
            n_q=4)
CFG2 = dict(seed=2, bits=(3, 2), heavy=True, N=32768, n_ub=512, tail=4096, tail_max=8192, n_q=4)
CFG3 = dict(seed=3, bits=(3, 3), heavy=False, seqs=64, ctx_lo=8192, ctx_hi=65536, layers=16, n_q=1, tail=4096,
            tail_max=8192)
CFG4 = dict(seed=4, bits=(4, 4), heavy=False, groups=8192, tail=4096, layers=16, n_q=4)


def _torch():
    import torch
    return torch


class DeviceSynth:
    """Device-side seeded rows of one configuration: per-layer channel scales resident on the GPU."""

    def __init__(self, seed, n_layers, heavy=False, layer0=0, stream=None):
        T = _torch()
        self.L = sjk.lib()
        self.seed, self.heavy, self.layer0, self.st = seed, heavy, layer0, stream
        self.scale = T.empty((n_layers, H, D), dtype=T.float32, device="cuda")
        sjk.check(self.L.sjk_synth_scales(seed, layer0, n_layers, H, D, C.c_void_p(self.scale.data_ptr()), stream),
                  "synth_scales")

    def rows_into(self, il, pos0, n, k, v):
        """Write layer il's model-basis rows of positions [pos0, pos0 + n) into device buffers k, v ([n][H][D])."""
        sjk.check(self.L.sjk_synth_kv(self.seed, self.layer0 + il, H, D, int(self.heavy),
                                      C.c_void_p(self.scale[il].data_ptr()), pos0, n, C.c_void_p(k.data_ptr()),
                                      C.c_void_p(v.data_ptr()), self.st), "synth_kv")

    def rows(self, il, pos0, n):
        T = _torch()
        k = T.empty((n, H, D), dtype=T.float32, device="cuda")
        v = T.empty_like(k)
        self.rows_into(il, pos0, n, k, v)
        return k, v

    def queries(self, il, n_q, n_head=HQ):
        """Layer il's query rows [n_q][n_head][D] (fp16-rounded, model basis)."""
        T = _torch()
        q = T.empty((n_q, n_head, D), dtype=T.float32, device="cuda")
        sjk.check(self.L.sjk_synth_q(self.seed, self.layer0 + il, n_q * n_head, D, C.c_void_p(q.data_ptr()), self.st),
                  "synth_q")
        return q


class PolicyModel:
    """n_layers device layer caches of one sequence with the reference's adaptive-tail policy (the engine loop:
    begin_ubatch, seal what is due, commit, store the ubatch), filled from the seeded generator."""

    def __init__(self, seed, n_layers, n_ctx, bits=(4, 4), heavy=False, body=2, n_ub=512, tail=4096, tail_max=8192,
                 stream=None, layer0=0):
        T = _torch()
        self.T, self.L, self.st = T, sjk.lib(), stream
        self.cfg = sjk.config(D, H, n_ctx, n_ub, bits_k=bits[0], bits_v=bits[1], body=body, tail=tail, tail_max=tail_max)
        self.layers = [sjk.Layer() for _ in range(n_layers)]
        for lay in self.layers:
            sjk.check(self.L.sj_kvarn_layer_init(C.byref(lay), C.byref(self.cfg)), "layer_init")
        self.pol = sjk.Policy()
        self.L.sj_kvarn_policy_init(C.byref(self.pol), SINK, tail, tail_max, G, 0)
        self.syn = DeviceSynth(seed, n_layers, heavy, layer0, stream)
        self.n_ub = n_ub
        self.n = 0
        self.sealed_records = 0
        self._k = T.empty((n_ub, H, D), dtype=T.float32, device="cuda")
        self._v = T.empty_like(self._k)

    def seal_pending(self):
        p = self.pol
        if p.B_pending > p.B:
            for lay in self.layers:
                sjk.check(self.L.sjk_layer_seal(C.byref(lay), p.B, p.B_pending, self.st), "seal")
            self.sealed_records += (p.B_pending - p.B) // G * H * len(self.layers)
        self.L.sj_kvarn_policy_commit(C.byref(p))

    def store(self, pos0, n):
        for il, lay in enumerate(self.layers):
            self.syn.rows_into(il, pos0, n, self._k, self._v)
            sjk.check(self.L.sjk_layer_store(C.byref(lay), pos0, n, C.c_void_p(self._k.data_ptr()),
                                             C.c_void_p(self._v.data_ptr()), 1, self.st), "store")
        self.n = max(self.n, pos0 + n)

    def begin(self, pos0, n):
        self.L.sj_kvarn_policy_begin_ubatch(C.byref(self.pol), pos0, n)
        self.seal_pending()

    def grow(self, to):
        pos = self.n
        while pos < to:
            n = min(self.n_ub, to - pos)
            self.begin(pos, n)
            self.store(pos, n)
            pos += n

    def idle(self, keep=0):
        self.L.sj_kvarn_policy_idle(C.byref(self.pol), self.n, keep)
        self.seal_pending()

    def free(self):
        for lay in self.layers:
            self.L.sj_kvarn_layer_free(C.byref(lay))
        self.layers = []


def build_config0(stream=None, bits=CFG0["bits"], heavy=CFG0["heavy"], seed=CFG0["seed"]):
    """Config 0 (or config 2's seal commit with bits=(3, 2), heavy=True, seed=2): 8,320 positions through the
    policy; returns (model, B_from, B_to) of the pending 4096-token commit, not yet sealed."""
    c = CFG0
    m = PolicyModel(seed, 1, c["n_ctx"], bits=bits, heavy=heavy, n_ub=c["n_ub"], tail=c["tail"], tail_max=c["tail_max"],
                    stream=stream)
    m.grow(c["npos"])
    m.L.sj_kvarn_policy_begin_ubatch(C.byref(m.pol), c["npos"], c["n_ub"])
    B0, B1 = m.pol.B, m.pol.B_pending
    assert (B0, B1) == (128, 4224), (B0, B1)
    return m, B0, B1


def build_config1(stream=None, layers=CFG1["layers"]):
    c = CFG1
    m = PolicyModel(c["seed"], layers, c["N"], bits=c["bits"], n_ub=c["n_ub"], tail=c["tail"], tail_max=c["tail_max"],
                    stream=stream)
    m.grow(c["idle_at"])
    m.idle(0)
    m.grow(c["N"])
    assert m.pol.B == 93824, m.pol.B
    return m


def build_config2(stream=None, layers=1):
    c = CFG2
    m = PolicyModel(c["seed"], layers, c["N"] + 1024, bits=c["bits"], heavy=True, n_ub=c["n_ub"], tail=c["tail"],
                    tail_max=c["tail_max"], stream=stream)
    m.grow(c["N"])
    m.idle(0)
    assert m.pol.B == 28672, m.pol.B
    return m


class SliceModel:
    """Config 4's context slice on one rank: groups [g0, g1) of every layer of the one seeded sequence, plus the sink
    (when `sink`) and the ring tail (when `tail` > 0, the newest positions). The slice's own positions are local:
    local S + 128 (g - g0) + t holds global position S + 128 g + t, so local record g - g0 is global record g, and the
    tail's local positions follow the slice's body. The body is bulk-sealed: the slice's rows are staged into one
    staging buffer in the ring layout (a view whose ring holds every body position), then each layer's records are
    sealed from it in one launch (sjk_seal_ring), which reads the same staged rows as sj_kvarn_layer_seal would."""

    def __init__(self, g0, g1, sink, tail, n_layers=CFG4["layers"], stream=None, seed=CFG4["seed"], chunk=16384):
        T = _torch()
        self.T, self.L, self.st = T, sjk.lib(), stream
        self.g0, self.g1, self.has_sink, self.tail = g0, g1, sink, tail
        self.n_body = (g1 - g0) * G
        self.B = SINK + self.n_body
        self.N = self.B + tail
        self.cfg = sjk.config(D, H, self.N + 1024, 512, bits_k=4, bits_v=4, body=2, tail=4096, tail_max=8192)
        self.layers = [sjk.Layer() for _ in range(n_layers)]
        for lay in self.layers:
            sjk.check(self.L.sj_kvarn_layer_init(C.byref(lay), C.byref(self.cfg)), "layer_init")
        self.syn = DeviceSynth(seed, n_layers, False, 0, stream)
        self.chunk = chunk
        # staging buffer of the whole body slice in the ring layout: slot (pos - S) % cap with cap = n_body
        v0 = sjk.view_of(self.layers[0])
        self.stage_row = 2 * int(v0.stage_bytes) * H
        self.staging = T.empty(max(self.n_body, 1) * self.stage_row, dtype=T.uint8, device="cuda")
        self.global_B = SINK + CFG4["groups"] * G

    def stage_view(self, il):
        v = sjk.view_of(self.layers[il])
        v.ring = self.staging.data_ptr()
        v.cap = max(self.n_body, 1)
        return v

    def write_layer(self, il):
        """Sink, staged body rows and tail of layer il (the seal is separate: seal_layer)."""
        T, L = self.T, self.L
        lay = self.layers[il]
        k = T.empty((self.chunk, H, D), dtype=T.float32, device="cuda")
        v = T.empty_like(k)
        if self.has_sink:
            self.syn.rows_into(il, 0, SINK, k, v)
            sjk.check(L.sjk_layer_store(C.byref(lay), 0, SINK, C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()), 1,
                                        self.st), "store sink")
        sv = self.stage_view(il)
        for off in range(0, self.n_body, self.chunk):
            n = min(self.chunk, self.n_body - off)
            self.syn.rows_into(il, SINK + self.g0 * G + off, n, k, v)
            sjk.check(L.sjk_store(C.byref(sv), C.c_void_p(lay.sink), C.c_void_p(self.staging.data_ptr()), SINK + off, n,
                                  C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()), 1, self.st), "store staging")
        if self.tail:
            for off in range(0, self.tail, self.chunk):
                n = min(self.chunk, self.tail - off)
                self.syn.rows_into(il, self.global_B + off, n, k, v)
                sjk.check(L.sjk_layer_store(C.byref(lay), self.B + off, n, C.c_void_p(k.data_ptr()),
                                            C.c_void_p(v.data_ptr()), 1, self.st), "store tail")

    def seal_layer(self, il):
        """Seal layer il's body from the staging buffer; call it after write_layer(il) and before the next layer's
        write_layer, which reuses the buffer."""
        lay = self.layers[il]
        sv = self.stage_view(il)
        sjk.check(self.L.sjk_seal_ring(C.byref(sv), C.c_void_p(lay.body), SINK, self.B, lay.cfg.iters, self.st),
                  "bulk seal")

    def build(self):
        for il in range(len(self.layers)):
            self.write_layer(il)
            self.seal_layer(il)

    def free(self):
        for lay in self.layers:
            self.L.sj_kvarn_layer_free(C.byref(lay))
        self.layers = []
        self.staging = None
