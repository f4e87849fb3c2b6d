"""ctypes binding of the CPU oracle (liboracle.so) and of the compiled reference
(_ref/libsjref.so). TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg use it as the checker; the product never imports it.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libsjref.so")

u8p = np.ctypeslib.ndpointer(np.uint8, flags="C")
u16p = np.ctypeslib.ndpointer(np.uint16, flags="C")
f32p = np.ctypeslib.ndpointer(np.float32, flags="C")


class Layout(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("D", "G", "bits_k", "bits_v", "trellis")] + \
               [(n, C.c_uint32) for n in ("kp", "vp", "ks", "kz", "kt", "vc", "vs", "vz", "bytes")]


class Policy(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("sink", "tail", "tail_max", "group", "flush_chunk", "B", "B_prev",
                                          "B_pending")] + [("draining", C.c_int)]


class Cache(C.Structure):
    _fields_ = [("lay", Layout), ("H", C.c_int), ("staging", C.c_int), ("sink_f16", C.c_int), ("iters", C.c_int),
                ("S", C.c_uint32), ("cap", C.c_uint32), ("n_groups", C.c_uint32), ("stage_bytes", C.c_size_t),
                ("sink", C.c_void_p), ("ring", C.c_void_p), ("body", C.c_void_p), ("blocks", C.c_void_p)]


def reference_dir():
    """The reference checkout: SJK_REF_DIR, else a `reference` directory beside this repository (None if absent)."""
    for d in (os.environ.get("SJK_REF_DIR"), os.path.join(HERE, "..", "..", "reference")):
        if d and os.path.isfile(os.path.join(d, "sj_kvarn.h")):
            return os.path.abspath(d)
    return None


def build():
    """Compile liboracle.so (and _ref/libsjref.so when the reference sources exist)."""
    import subprocess
    ref_dir = reference_dir()
    subprocess.run(["make", "-s", "-C", HERE] + ([f"SJK_REF_DIR={ref_dir}"] if ref_dir else []), check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        L.ora_layout_init.argtypes = [C.POINTER(Layout), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
        L.ora_f2h.argtypes = [C.c_float]; L.ora_f2h.restype = C.c_uint16
        L.ora_h2f.argtypes = [C.c_uint16]; L.ora_h2f.restype = C.c_float
        L.ora_fwht.argtypes = [f32p, C.c_int]
        L.ora_code_bit.argtypes = [C.POINTER(Layout), C.c_int, C.c_int, C.c_int]; L.ora_code_bit.restype = C.c_uint32
        L.ora_k_ch.argtypes = [C.POINTER(Layout), C.c_int]
        L.ora_v_ch.argtypes = [C.POINTER(Layout), C.c_int]
        L.ora_tq6_encode.argtypes = [f32p, u8p, C.c_int]
        L.ora_tq6_decode.argtypes = [u8p, f32p, C.c_int]
        L.ora_stage_row.argtypes = [C.c_int, f32p, u8p, C.c_int]
        L.ora_unstage_row.argtypes = [C.c_int, u8p, f32p, C.c_int]
        L.ora_seal.argtypes = [C.POINTER(Layout), u16p, u16p, C.c_size_t, C.c_int, u8p]
        L.ora_seal_batch.argtypes = [C.POINTER(Layout), u16p, u16p, C.c_size_t, C.c_int, C.c_int, C.c_int, u8p, C.c_int]
        L.ora_decode_k.argtypes = [C.POINTER(Layout), u8p, C.c_int, f32p]
        L.ora_decode_v.argtypes = [C.POINTER(Layout), u8p, C.c_int, f32p]
        L.ora_policy_init.argtypes = [C.POINTER(Policy)] + [C.c_uint32] * 5
        L.ora_policy_begin.argtypes = [C.POINTER(Policy), C.c_uint32, C.c_uint32]; L.ora_policy_begin.restype = C.c_uint32
        L.ora_policy_commit.argtypes = [C.POINTER(Policy)]
        L.ora_policy_idle.argtypes = [C.POINTER(Policy), C.c_uint32, C.c_uint32]; L.ora_policy_idle.restype = C.c_uint32
        L.ora_policy_truncate.argtypes = [C.POINTER(Policy), C.c_uint32, C.POINTER(C.c_uint32)]
        L.ora_policy_truncate.restype = C.c_uint32
        L.ora_ring_capacity.argtypes = [C.c_uint32] * 4; L.ora_ring_capacity.restype = C.c_uint32
        L.ora_cache_init.argtypes = [C.POINTER(Cache)] + [C.c_int] * 8 + [C.c_uint32] * 5
        L.ora_cache_free.argtypes = [C.POINTER(Cache)]
        L.ora_store.argtypes = [C.POINTER(Cache), C.c_uint32, f32p, f32p]
        L.ora_seal_range.argtypes = [C.POINTER(Cache), C.c_uint32, C.c_uint32, C.c_int]
        L.ora_record.argtypes = [C.POINTER(Cache), C.c_uint32, C.c_int]; L.ora_record.restype = C.c_void_p
        L.ora_kv_row.argtypes = [C.POINTER(Cache), C.c_uint32, C.c_uint32, C.c_int, f32p, f32p]
        L.ora_attend_row.argtypes = [C.POINTER(Cache), C.c_uint32, C.c_uint32, f32p, C.c_int, C.c_uint32, C.c_float, f32p]
        L.ora_attend.argtypes = [C.POINTER(Cache), C.c_uint32, C.c_uint32, C.c_uint32, C.c_int, C.c_int, f32p, C.c_float,
                                 f32p, C.c_int]
        L.ora_state_write.argtypes = [C.POINTER(Cache), C.c_int, C.POINTER(Policy), C.c_uint32] + [C.c_int] * 6 + \
                                     [C.c_uint32] * 3 + [C.c_void_p]
        L.ora_state_write.restype = C.c_size_t
        L.ora_fnv.argtypes = [C.c_void_p, C.c_size_t, C.c_uint64]; L.ora_fnv.restype = C.c_uint64
        L.ora_trace_balance.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t]
        L.ora_balance_step.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]
        L.ora_trace_counts.argtypes = [C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]
        L.ora_libm_log_exp.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]
        _lib = L
    return _lib


def layout(D, bits_k, bits_v, trellis, G=128):
    l = Layout()
    rc = lib().ora_layout_init(C.byref(l), D, G, bits_k, bits_v, int(trellis))
    if rc:
        raise ValueError(f"layout rc {rc}")
    return l


def fnv(a, h=1469598103934665603):
    a = np.ascontiguousarray(a)
    return lib().ora_fnv(a.ctypes.data, a.nbytes, h)


def f2h(x):
    x = np.asarray(x, dtype=np.float32).ravel()
    return np.array([lib().ora_f2h(float(v)) for v in x], dtype=np.uint16)


def fwht_rows(x):
    """Rotate every row of x (float32 [..., n]) in place with the orthonormal FWHT."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    flat = x.reshape(-1, n)
    for i in range(flat.shape[0]):
        row = np.ascontiguousarray(flat[i])
        lib().ora_fwht(row, n)
        flat[i] = row
    return x


def tq6_encode(x):
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.zeros(x.size // 128 * 98, dtype=np.uint8)
    lib().ora_tq6_encode(x, out, x.size)
    return out


def tq6_decode(blocks, n):
    out = np.zeros(n, dtype=np.float32)
    lib().ora_tq6_decode(np.ascontiguousarray(blocks, dtype=np.uint8), out, n)
    return out


def seal(l, K, V, iters=16, row_stride=None):
    rec = np.zeros(l.bytes, dtype=np.uint8)
    lib().ora_seal(C.byref(l), np.ascontiguousarray(K, dtype=np.uint16), np.ascontiguousarray(V, dtype=np.uint16),
                   row_stride or l.D, iters, rec)
    return rec


def seal_batch(l, k, v, row_stride, H, n_rec, iters=16, n_threads=0):
    body = np.zeros(n_rec * l.bytes, dtype=np.uint8)
    lib().ora_seal_batch(C.byref(l), np.ascontiguousarray(k, dtype=np.uint16), np.ascontiguousarray(v, dtype=np.uint16),
                         row_stride, H, n_rec, iters, body, n_threads)
    return body


def decode(l, rec):
    """Decode all G rows of one record: (K [G][D], V [G][D]) float32."""
    rec = np.ascontiguousarray(rec, dtype=np.uint8)
    k = np.zeros((l.G, l.D), np.float32)
    v = np.zeros((l.G, l.D), np.float32)
    row = np.zeros(l.D, np.float32)
    for t in range(l.G):
        lib().ora_decode_k(C.byref(l), rec, t, row); k[t] = row
        lib().ora_decode_v(C.byref(l), rec, t, row); v[t] = row
    return k, v


class OracleCache:
    """Host cache with the reference memory layout, built and read through the oracle."""

    def __init__(self, D, H, bits_k=4, bits_v=4, trellis=False, iters=16, staging=0, sink_f16=True, S=128,
                 tail=4096, tail_max=8192, n_ubatch=512, n_ctx=16384):
        self.c = Cache()
        rc = lib().ora_cache_init(C.byref(self.c), D, H, bits_k, bits_v, int(trellis), iters, staging, int(sink_f16),
                                  S, tail, tail_max, n_ubatch, n_ctx)
        if rc:
            raise ValueError("oracle cache init failed")
        self.D, self.H = D, H

    def close(self):
        if self.c.ring:
            lib().ora_cache_free(C.byref(self.c))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def store(self, pos, k_rot, v_rot):
        lib().ora_store(C.byref(self.c), pos, np.ascontiguousarray(k_rot, np.float32).ravel(),
                        np.ascontiguousarray(v_rot, np.float32).ravel())

    def seal(self, B_from, B_to, n_threads=0):
        lib().ora_seal_range(C.byref(self.c), B_from, B_to, n_threads)

    def ring_bytes(self):
        n = self.c.cap * self.H * 2 * self.c.stage_bytes
        return np.ctypeslib.as_array((C.c_uint8 * n).from_address(self.c.ring)).copy()

    def sink_bytes(self):
        per = self.D * 4 if self.c.sink_f16 else 2 * self.c.stage_bytes
        n = self.c.S * self.H * per
        return np.ctypeslib.as_array((C.c_uint8 * n).from_address(self.c.sink)).copy()

    def record(self, g, h):
        p = lib().ora_record(C.byref(self.c), g, h)
        return np.ctypeslib.as_array((C.c_uint8 * self.c.lay.bytes).from_address(p)).copy()

    def body_bytes(self, n_groups):
        n = n_groups * self.H * self.c.lay.bytes
        return np.ctypeslib.as_array((C.c_uint8 * n).from_address(self.c.body)).copy()

    def kv_row(self, B, pos, h):
        k = np.zeros(self.D, np.float32); v = np.zeros(self.D, np.float32)
        lib().ora_kv_row(C.byref(self.c), B, pos, h, k, v)
        return k, v

    def attend(self, B, N, qpos0, q, scale, n_threads=0):
        """q: [n_q][n_head][D] float32 -> out of the same shape."""
        q = np.ascontiguousarray(q, np.float32)
        n_q, n_head = q.shape[0], q.shape[1]
        out = np.zeros_like(q)
        lib().ora_attend(C.byref(self.c), B, N, qpos0, n_q, n_head, q.reshape(-1), scale, out.reshape(-1), n_threads)
        return out


# ---- the compiled reference (oracle/_ref) -------------------------------------------------------------

_ref = None


def ref_available():
    return os.path.exists(REF_PATH)


def ref():
    global _ref
    if _ref is None:
        _ref = C.CDLL(REF_PATH)
    return _ref
