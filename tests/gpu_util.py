"""Device-memory helpers for the GPU tests (torch is only the allocator and copier here)."""
import ctypes as C

import numpy as np


def torch():
    import torch as T
    return T


def dev(a):
    """numpy array -> contiguous CUDA tensor (same dtype bytes)."""
    T = torch()
    a = np.ascontiguousarray(a)
    t = T.from_numpy(a.view(np.uint8).reshape(-1).copy()).cuda()
    return t


def dev_zeros(nbytes):
    T = torch()
    return T.zeros(int(nbytes), dtype=T.uint8, device="cuda")


def host(t, dtype=np.uint8, shape=None):
    T = torch()
    T.cuda.synchronize()
    a = t.detach().cpu().numpy().view(dtype)
    return a.reshape(shape) if shape is not None else a


def ptr(t):
    return C.c_void_p(t.data_ptr())


def rel_err_rows(out, ref):
    """max over rows of ||out - ref|| / ||ref|| (the reference's device test metric, tests/test_cuda.cu:126-133)."""
    o = out.reshape(-1, out.shape[-1]).astype(np.float64)
    r = ref.reshape(-1, ref.shape[-1]).astype(np.float64)
    num = np.sqrt(((o - r) ** 2).sum(-1))
    den = np.sqrt((r ** 2).sum(-1))
    den[den == 0] = 1.0
    return float((num / den).max())


_cudart = None


def cudart():
    global _cudart
    if _cudart is None:
        import sjk
        sjk.lib()                                    # loads the runtime the library links
        _cudart = C.CDLL("libcudart.so.12")
        _cudart.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
        _cudart.cudaDeviceSynchronize.argtypes = []
    return _cudart


def d2h_ptr(p, nbytes):
    """Copy nbytes at device address p to a new numpy uint8 array."""
    out = np.zeros(int(nbytes), dtype=np.uint8)
    if nbytes:
        assert cudart().cudaDeviceSynchronize() == 0
        assert cudart().cudaMemcpy(out.ctypes.data, C.c_void_p(p), int(nbytes), 2) == 0
    return out


class DevSeq:
    """A product sequence (libsjk_b200 sj_kvarn_seq) driven through the sj_kvarn.h-style API."""

    def __init__(self, cfg, n_layers, pool=None):
        import sjk
        self.L = sjk.lib()
        self.s = sjk.Seq()
        self.cfg = cfg
        self.nl = n_layers
        self.pool = pool
        rc = self.L.sj_kvarn_seq_init(C.byref(self.s), C.byref(cfg), n_layers, C.byref(pool) if pool else None)
        sjk.check(rc, "seq_init")
        self.T = torch()

    @property
    def n(self):
        return self.s.n

    @property
    def pol(self):
        return self.s.pol

    def close(self):
        self.L.sj_kvarn_seq_free(C.byref(self.s))

    def begin_ubatch(self, pos0, n_tokens):
        return self.L.sj_kvarn_seq_begin_ubatch(C.byref(self.s), pos0, n_tokens)

    def idle(self, keep):
        return self.L.sj_kvarn_seq_idle(C.byref(self.s), keep)

    def truncate(self, pos):
        return self.L.sj_kvarn_seq_truncate(C.byref(self.s), pos)

    def store(self, pos, k, v):
        kt = self.T.from_numpy(np.ascontiguousarray(k, np.float32)).cuda()
        vt = self.T.from_numpy(np.ascontiguousarray(v, np.float32)).cuda()
        self.L.sj_kvarn_seq_store(C.byref(self.s), pos, C.c_void_p(kt.data_ptr()), C.c_void_p(vt.data_ptr()))
        import sjk
        sjk.check_sticky("seq_store")
        self._keep = (kt, vt)                        # keep alive until the stream has consumed them

    def state(self):
        import sjk
        n = self.L.sj_kvarn_seq_state_size(C.byref(self.s))
        buf = np.zeros(n, dtype=np.uint8)
        w = C.c_size_t()
        sjk.check(self.L.sj_kvarn_seq_state_write(C.byref(self.s), buf.ctypes.data, n, C.byref(w)), "state_write")
        assert w.value == n
        return buf

    def read_state(self, st):
        return self.L.sj_kvarn_seq_state_read(C.byref(self.s), st.ctypes.data, st.size)
