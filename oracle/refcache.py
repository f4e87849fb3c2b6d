"""The compiled reference (oracle/_ref/libsjref.so, sj_kvarn.h built from its own source) driven through its own
public API, plus the host side of the seeded input generator. TEST INFRASTRUCTURE ONLY: the configuration parity
tests and bench.py's CPU legs (the reference arm and cpu_baseline) use it; the product never imports it.

RefLayer builds one layer's cache exactly as an engine on the reference would: K/V rows in the model basis are
rotated with sj_kvarn_hadamard, stored with sj_kvarn_layer_store (spread over host threads; distinct positions write
distinct ring rows), sealed with sj_kvarn_layer_seal (or the threaded harness over the same public per-record calls),
and read with sj_kvarn_layer_attend_row / sj_kvarn_layer_kv_row / sj_kvarn_decode_*_row.
"""
import ctypes as C
import os

import numpy as np

import oracle

vp, u32, f32p = C.c_void_p, C.c_uint32, C.c_void_p


class RefConfig(C.Structure):
    """sj_kvarn_config (sj_kvarn.h:279-290)"""
    _fields_ = [(n, C.c_int) for n in ("head_dim", "n_head_kv", "group", "bits_k", "bits_v", "body", "iters", "staging",
                                       "sink_type")] + \
               [(n, u32) for n in ("sink", "tail", "tail_max", "flush_chunk", "n_ubatch", "n_ctx")]


_bound = set()


def _bind_synth(L):
    if id(L) in _bound:
        return L
    L.sjk_synth_scales_host.argtypes = [C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_int, vp]
    L.sjk_synth_kv_host.argtypes = [C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_int, vp, u32, u32, vp, vp, C.c_int]
    L.sjk_synth_q_host.argtypes = [C.c_uint64, C.c_int, u32, C.c_int, vp]
    L.sjk_synth_ln.argtypes = [C.c_double]; L.sjk_synth_ln.restype = C.c_double
    L.sjk_synth_exp.argtypes = [C.c_double]; L.sjk_synth_exp.restype = C.c_double
    L.sjk_synth_cossin.argtypes = [C.c_double, C.POINTER(C.c_double), C.POINTER(C.c_double)]
    L.sjk_synth_f16.argtypes = [C.c_float]; L.sjk_synth_f16.restype = C.c_uint16
    _bound.add(id(L))
    return L


def ref():
    """The compiled reference library with its argument types set."""
    R = oracle.ref()
    if id(R) in _bound:
        return R
    R.sj_kvarn_config_default.argtypes = [C.c_int, C.c_int, u32, u32]
    R.sj_kvarn_config_default.restype = RefConfig
    R.sjref_layer_new.argtypes = [C.POINTER(RefConfig), C.POINTER(C.c_int)]; R.sjref_layer_new.restype = vp
    R.sjref_layer_delete.argtypes = [vp]
    R.sjref_layer_store_mt.argtypes = [vp, u32, u32, vp, vp, C.c_int]
    R.sjref_rotate_mt.argtypes = [vp, C.c_size_t, C.c_int, C.c_int]
    R.sjref_layer_seal_mt.argtypes = [vp, u32, u32, C.c_int]
    R.sj_kvarn_layer_seal.argtypes = [vp, u32, u32]
    R.sj_kvarn_layer_attend_row.argtypes = [vp, u32, u32, vp, C.c_int, u32, C.c_float, vp]
    R.sj_kvarn_layer_kv_row.argtypes = [vp, u32, u32, C.c_int, vp, vp]
    R.sj_kvarn_layer_record.argtypes = [vp, u32, C.c_int]; R.sj_kvarn_layer_record.restype = vp
    R.sjref_attend.argtypes = [vp, u32, u32, u32, C.c_int, C.c_int, vp, C.c_float, vp, C.c_int]
    R.sjref_layer_ring.argtypes = [vp, C.POINTER(C.c_size_t)]; R.sjref_layer_ring.restype = vp
    R.sjref_layer_sink.argtypes = [vp, C.POINTER(C.c_size_t)]; R.sjref_layer_sink.restype = vp
    R.sjref_layer_cap.argtypes = [vp]; R.sjref_layer_cap.restype = u32
    R.sjref_layer_record_bytes.argtypes = [vp]; R.sjref_layer_record_bytes.restype = u32
    R.sjref_layer_layout.argtypes = [vp]; R.sjref_layer_layout.restype = vp
    R.sj_kvarn_decode_k_row.argtypes = [vp, vp, C.c_int, vp]
    R.sj_kvarn_decode_v_row.argtypes = [vp, vp, C.c_int, vp]
    R.sjref_seal_batch.argtypes = [vp, vp, vp, C.c_size_t, C.c_int, C.c_int, C.c_int, vp, C.c_int]
    R.sj_kvarn_seal_group.argtypes = [vp, vp, vp, C.c_size_t, C.c_int, vp, vp]
    R.sj_kvarn_seal_workspace_bytes.argtypes = [vp]; R.sj_kvarn_seal_workspace_bytes.restype = C.c_size_t
    R.sj_kvarn_policy_init.argtypes = [vp] + [u32] * 5
    R.sj_kvarn_policy_begin_ubatch.argtypes = [vp, u32, u32]; R.sj_kvarn_policy_begin_ubatch.restype = u32
    R.sj_kvarn_policy_commit.argtypes = [vp]
    R.sj_kvarn_policy_idle.argtypes = [vp, u32, u32]; R.sj_kvarn_policy_idle.restype = u32
    R.sj_kvarn_hadamard.argtypes = [vp, C.c_int]
    R.sjref_nthreads.argtypes = [C.c_int]
    _bind_synth(R)
    _bound.add(id(R))
    return R


def available():
    return oracle.ref_available()


# ---- the seeded input generator (host side of sjk_synth.h), from the oracle or the reference library ----

def _gen(lib):
    return _bind_synth(lib if lib is not None else oracle.lib())


def synth_scales(seed, layer0, n_layers, H, D, lib=None):
    out = np.zeros((n_layers, H, D), np.float32)
    _gen(lib).sjk_synth_scales_host(seed, layer0, n_layers, H, D, out.ctypes.data)
    return out


def synth_kv(seed, layer, H, D, heavy, scale, pos0, n, n_threads=0, lib=None):
    """(K, V) float32 [n][H][D] of positions pos0 .. pos0 + n - 1 in the model basis; scale: [H][D] of the layer."""
    k = np.empty((n, H, D), np.float32)
    v = np.empty((n, H, D), np.float32)
    sc = np.ascontiguousarray(scale, np.float32)
    _gen(lib).sjk_synth_kv_host(seed, layer, H, D, int(heavy), sc.ctypes.data, pos0, n, k.ctypes.data, v.ctypes.data,
                                n_threads)
    return k, v


def synth_q(seed, layer, n_q, n_head, D, lib=None):
    q = np.empty((n_q, n_head, D), np.float32)
    _gen(lib).sjk_synth_q_host(seed, layer, n_q * n_head, D, q.ctypes.data)
    return q


# ---- one layer of the reference cache ----

class RefLayer:
    """One sj_kvarn_layer of the compiled reference (host memory), with its own adaptive-tail policy."""

    def __init__(self, D, H, n_ctx, n_ubatch, bits_k=4, bits_v=4, body=2, tail=4096, tail_max=8192, sink=128, iters=16,
                 staging=0, sink_type=0, n_threads=0):
        R = self.R = ref()
        cfg = R.sj_kvarn_config_default(D, H, n_ctx, n_ubatch)
        cfg.bits_k, cfg.bits_v, cfg.body, cfg.tail, cfg.tail_max, cfg.sink = bits_k, bits_v, body, tail, tail_max, sink
        cfg.iters, cfg.staging, cfg.sink_type = iters, staging, sink_type
        self.cfg = cfg
        rc = C.c_int()
        self.L = R.sjref_layer_new(C.byref(cfg), C.byref(rc))
        if not self.L:
            raise RuntimeError(f"reference sj_kvarn_layer_init rc {rc.value}")
        self.D, self.H, self.S = D, H, sink
        self.threads = R.sjref_nthreads(n_threads)
        self.pol = oracle.Policy()
        R.sj_kvarn_policy_init(C.byref(self.pol), sink, tail, tail_max, 128, 0)
        self.rec_bytes = R.sjref_layer_record_bytes(self.L)
        self.n = 0

    def close(self):
        if self.L:
            self.R.sjref_layer_delete(self.L)
            self.L = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # writes
    def store(self, pos0, k, v):
        """Store model-basis rows [n][H][D] at positions pos0 ..: sj_kvarn_hadamard per head, sj_kvarn_layer_store."""
        k = np.array(k, np.float32, copy=True, order="C")
        v = np.array(v, np.float32, copy=True, order="C")
        n = k.shape[0]
        self.R.sjref_rotate_mt(k.ctypes.data, k.size // self.D, self.D, self.threads)
        self.R.sjref_rotate_mt(v.ctypes.data, v.size // self.D, self.D, self.threads)
        self.R.sjref_layer_store_mt(self.L, pos0, n, k.ctypes.data, v.ctypes.data, self.threads)
        self.n = max(self.n, pos0 + n)

    def seal(self, B_from, B_to, threaded=True):
        """Seal [B_from, B_to): sj_kvarn_layer_seal itself (threaded=False) or the threaded harness over the same
        public per-record calls (unstage, fp16 rounding, sj_kvarn_seal_group)."""
        if B_to <= B_from:
            return
        if threaded:
            self.R.sjref_layer_seal_mt(self.L, B_from, B_to, self.threads)
        else:
            self.R.sj_kvarn_layer_seal(self.L, B_from, B_to)

    def begin_ubatch(self, pos0, n, threaded=True):
        """sj_kvarn_policy_begin_ubatch, the seal it asks for, then commit (the engine loop's order)."""
        R = self.R
        R.sj_kvarn_policy_begin_ubatch(C.byref(self.pol), pos0, n)
        self.seal(self.pol.B, self.pol.B_pending, threaded)
        R.sj_kvarn_policy_commit(C.byref(self.pol))

    def idle(self, keep=0, threaded=True):
        R = self.R
        R.sj_kvarn_policy_idle(C.byref(self.pol), self.n, keep)
        self.seal(self.pol.B, self.pol.B_pending, threaded)
        R.sj_kvarn_policy_commit(C.byref(self.pol))

    # reads
    def record(self, g, h):
        p = self.R.sj_kvarn_layer_record(self.L, g, h)
        return np.ctypeslib.as_array((C.c_uint8 * self.rec_bytes).from_address(p)).copy()

    def records(self, g0, g1):
        """records of groups [g0, g1), all heads, in body order: [g1 - g0][H][record]"""
        p = self.R.sj_kvarn_layer_record(self.L, g0, 0)
        n = (g1 - g0) * self.H * self.rec_bytes
        return np.ctypeslib.as_array((C.c_uint8 * n).from_address(p)).copy()

    def ring_bytes(self):
        n = C.c_size_t()
        p = self.R.sjref_layer_ring(self.L, C.byref(n))
        return np.ctypeslib.as_array((C.c_uint8 * n.value).from_address(p)).copy()

    def sink_bytes(self):
        n = C.c_size_t()
        p = self.R.sjref_layer_sink(self.L, C.byref(n))
        return np.ctypeslib.as_array((C.c_uint8 * n.value).from_address(p)).copy()

    def decode(self, g, h):
        """all G rows of record (g, h) through sj_kvarn_decode_k_row / _v_row: (K, V) float32 [G][D]"""
        R = self.R
        lay = R.sjref_layer_layout(self.L)
        rec = R.sj_kvarn_layer_record(self.L, g, h)
        k = np.zeros((128, self.D), np.float32)
        v = np.zeros((128, self.D), np.float32)
        for t in range(128):
            R.sj_kvarn_decode_k_row(lay, rec, t, k[t].ctypes.data)
            R.sj_kvarn_decode_v_row(lay, rec, t, v[t].ctypes.data)
        return k, v

    def attend_row(self, B, N, q_rot, h, qpos, scale):
        out = np.zeros(self.D, np.float32)
        q = np.ascontiguousarray(q_rot, np.float32)
        self.R.sj_kvarn_layer_attend_row(self.L, B, N, q.ctypes.data, h, qpos, scale, out.ctypes.data)
        return out

    def attend_pairs(self, B, N, qpos0, q_rot, pairs, scale, n_threads=0):
        """sj_kvarn_layer_attend_row for the given (query row, query head) pairs, spread over host threads;
        q_rot: [n_q][n_head][D]. Returns {pair: out[D]}."""
        from concurrent.futures import ThreadPoolExecutor
        n_head = q_rot.shape[1]
        grp = n_head // self.H
        q = np.ascontiguousarray(q_rot, np.float32)

        def one(p):
            iq, hq = p
            return p, self.attend_row(B, N, q[iq, hq], hq // grp, qpos0 + iq, scale)

        with ThreadPoolExecutor(max_workers=n_threads or self.threads) as ex:
            return dict(ex.map(one, pairs))

    def rotate(self, x):
        """sj_kvarn_hadamard over the last axis of a copy of x"""
        x = np.array(x, np.float32, copy=True, order="C")
        self.R.sjref_rotate_mt(x.ctypes.data, x.size // x.shape[-1], x.shape[-1], self.threads)
        return x
