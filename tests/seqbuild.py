"""Sequence builds through the policy, restated from the reference's state test
(tests/test_state.c:18-70 of the reference: D=128, H=2, 2 layers, sink 128, tail 256,
tail_max 512, n_ctx 2304, n_ubatch 64, and its `grow` ubatch-size pattern)."""
import numpy as np

import inputs

D, H, NL, SINK, G, TAIL, TAILMAX, NCTX = 128, 2, 2, 128, 128, 256, 512, 2304
ROW = NL * H * D
NO_POS = 0xFFFFFFFF

# (name, bits_k, bits_v, trellis, staging, sink_f16, flush_chunk) of the five golden streams
GOLDEN_CFGS = [
    ("4/4", 4, 4, 0, 0, 1, 0),
    ("3/3", 3, 3, 0, 0, 1, 0),
    ("3/3t", 3, 3, 1, 0, 1, 1),
    ("3/2t", 3, 2, 1, 0, 1, 0),
    ("4/4f", 4, 4, 0, 1, 0, 1),
]


def row_of(seed, edit_from, edit_variant, pos):
    var = edit_variant if pos >= edit_from else 0
    return inputs.seq_row(seed, var, pos, ROW, 0), inputs.seq_row(seed, var, pos, ROW, 1)


def ubatch_sizes(frm, to, pattern):
    pos, step = frm, 0
    while pos < to:
        if pattern == 0:
            n = 1
        elif step % 5 == 4:
            n = 1 + (pattern * 7 + step * 13) % 64
        else:
            n = 1 + (step + pattern) % 4
        n = min(n, to - pos)
        yield pos, n
        pos += n
        step += 1


def grow(seq, seed, frm, to, pattern, edit_from=NO_POS, edit_variant=0):
    """Drive any sequence object with begin_ubatch(pos0, n) -> rc and store(pos, k, v)."""
    for pos, n in ubatch_sizes(frm, to, pattern):
        rc = seq.begin_ubatch(pos, n)
        if rc:
            return rc
        for i in range(n):
            k, v = row_of(seed, edit_from, edit_variant, pos + i)
            seq.store(pos + i, k, v)
    return 0


class OracleSeq:
    """A sequence of NL oracle caches sharing one oracle policy (contiguous bodies)."""

    def __init__(self, bits_k, bits_v, trellis, staging=0, sink_f16=1, flush_chunk=0, iters=16,
                 d=D, h=H, nl=NL, sink=SINK, tail=TAIL, tail_max=TAILMAX, n_ubatch=64, n_ctx=NCTX):
        import ctypes as C
        import oracle
        self.o = oracle
        self.C = C
        self.cfg = dict(bits_k=bits_k, bits_v=bits_v, trellis=trellis, staging=staging, sink_f16=sink_f16,
                        flush_chunk=flush_chunk, iters=iters, tail=tail, tail_max=tail_max)
        self.D, self.H, self.nl = d, h, nl
        self.layers = (oracle.Cache * nl)()
        for il in range(nl):
            rc = oracle.lib().ora_cache_init(C.byref(self.layers[il]), d, h, bits_k, bits_v, trellis, iters, staging,
                                             sink_f16, sink, tail, tail_max, n_ubatch, n_ctx)
            assert rc == 0
        self.pol = oracle.Policy()
        oracle.lib().ora_policy_init(C.byref(self.pol), sink, tail, tail_max, 128, flush_chunk)
        self.n = 0

    def close(self):
        for il in range(self.nl):
            self.o.lib().ora_cache_free(self.C.byref(self.layers[il]))

    def begin_ubatch(self, pos0, n_tokens):
        if pos0 > self.n:
            return -100
        L = self.o.lib()
        L.ora_policy_begin(self.C.byref(self.pol), pos0, n_tokens)
        if self.pol.B_pending > self.pol.B:
            for il in range(self.nl):
                L.ora_seal_range(self.C.byref(self.layers[il]), self.pol.B, self.pol.B_pending, 0)
        L.ora_policy_commit(self.C.byref(self.pol))
        return 0

    def idle(self, keep_recent):
        L = self.o.lib()
        L.ora_policy_idle(self.C.byref(self.pol), self.n, keep_recent)
        if self.pol.B_pending > self.pol.B:
            for il in range(self.nl):
                L.ora_seal_range(self.C.byref(self.layers[il]), self.pol.B, self.pol.B_pending, 0)
        L.ora_policy_commit(self.C.byref(self.pol))
        return 0

    def store(self, pos, k, v):
        per = self.H * self.D
        for il in range(self.nl):
            self.o.lib().ora_store(self.C.byref(self.layers[il]), pos, np.ascontiguousarray(k[il * per:(il + 1) * per]),
                                   np.ascontiguousarray(v[il * per:(il + 1) * per]))
        self.n = max(self.n, pos + 1)

    def state(self):
        c = self.cfg
        args = (self.layers, self.nl, self.C.byref(self.pol), self.n, c["bits_k"], c["bits_v"], c["trellis"],
                c["iters"], c["staging"], c["sink_f16"], c["tail"], c["tail_max"], c["flush_chunk"])
        size = self.o.lib().ora_state_write(*args, None)
        buf = np.zeros(size, dtype=np.uint8)
        self.o.lib().ora_state_write(*args, buf.ctypes.data)
        return buf
