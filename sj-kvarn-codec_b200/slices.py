"""Work partitions across GPUs: context slices of one long sequence and whole sequences of a
paged pool.

Pool (config 3): sequences are independent, so each rank owns whole sequences, assigned by longest-processing-time
on their context lengths (largest first, each to the least-loaded rank); no collective touches the data path.

Context slices (config 4):

Every rank holds a contiguous range of the sealed groups of each layer. Rank 0 also holds the sink, and the last
rank holds the staging ring (the newest positions). Each rank attends over its own regions with
sjk_attend_partial, getting one (m, l, o[D]) triple per (query row, query head). The triples are all-gathered over
the process group (NCCL over NVLink on the GPU box) and merged in rank order with sjk_attend_merge. Every rank
therefore ends with the same output, equal to attention over the whole context (sj_kvarn.h:1535-1564) up to fp32
rounding. The only exchange per layer call is the all-gather of n_q * n_head * (D + 2) floats per rank.
"""
import numpy as np

SJK_REGION_SINK, SJK_REGION_BODY, SJK_REGION_RING = 1, 2, 4


# attention time of one 128-position chunk of staged rows (sink or staging ring) in units of one sealed record of
# the same KV head: the tensor-core body kernel decodes a tq6_0 chunk in about 4.5 record times
CHUNK_WEIGHT = 4.5


def group_range(rank, world, n_groups, sink_chunks=0, tail_chunks=0, chunk_weight=CHUNK_WEIGHT):
    """Contiguous range [g0, g1) of the sealed groups owned by `rank`, balanced by attention cost: rank 0 also
    attends over `sink_chunks` chunks of sink rows and the last rank over `tail_chunks` chunks of the staging ring,
    each costing `chunk_weight` groups, so those ranks get correspondingly fewer groups (with no sink or tail:
    n_groups / world each, to within one group)."""
    total = n_groups + chunk_weight * (sink_chunks + tail_chunks)

    def bound(r):                                   # first group of rank r
        if r <= 0:
            return 0
        if r >= world:
            return n_groups
        b = int(np.floor(total * r / world - chunk_weight * sink_chunks + 0.5)) if (sink_chunks or tail_chunks) \
            else n_groups * r // world
        return min(max(b, 0), n_groups)

    return bound(rank), bound(rank + 1)


def regions(rank, world):
    """The cache regions `rank` attends over: its body slice, plus the sink on rank 0 and the ring on the last rank."""
    r = SJK_REGION_BODY
    if rank == 0:
        r |= SJK_REGION_SINK
    if rank == world - 1:
        r |= SJK_REGION_RING
    return r


def gather(dist, part):
    """All-gather the partial triples of every rank, in rank order: [world, rows, D + 2] (one NCCL all-gather into
    a single buffer on the GPU box; a list all-gather on backends without it)."""
    import torch
    world = dist.get_world_size()
    out = torch.empty((world,) + tuple(part.shape), dtype=part.dtype, device=part.device)
    if dist.get_backend() == "nccl":
        dist.all_gather_into_tensor(out, part.contiguous())
    else:
        dist.all_gather(list(out.unbind(0)), part.contiguous())
    return out


def merge_partials_np(parts):
    """Combine partial triples [P, rows, D + 2] in index order into [rows, D] (the merge kernel's arithmetic in
    numpy, for host-side checks): out = sum_i o_i e^(m_i - m) / sum_i l_i e^(m_i - m), m = max_i m_i."""
    parts = np.asarray(parts, np.float64)
    m, l, o = parts[:, :, 0], parts[:, :, 1], parts[:, :, 2:]
    mx = m.max(axis=0)
    w = np.where(np.isneginf(m), 0.0, np.exp(m - np.where(np.isneginf(mx), 0.0, mx)))
    den = (l * w).sum(axis=0)
    num = (o * w[:, :, None]).sum(axis=0)
    return np.where(den[:, None] > 0, num / np.where(den == 0, 1.0, den)[:, None], 0.0)


def partial_np(q, k, v, scale):
    """Reference partial triple over one slice of positions: q [rows, D], k, v [n, D] -> [rows, D + 2]."""
    s = (q.astype(np.float64) @ k.astype(np.float64).T) * scale
    if s.shape[1] == 0:
        out = np.zeros((q.shape[0], q.shape[1] + 2))
        out[:, 0] = -np.inf
        return out
    m = s.max(axis=1)
    p = np.exp(s - m[:, None])
    return np.concatenate([m[:, None], p.sum(axis=1)[:, None], p @ v.astype(np.float64)], axis=1)


def lpt_assign(costs, world):
    """Owner rank of every item: items in decreasing cost order (ties by index) go to the least-loaded rank (ties by
    rank index). Deterministic, so every rank computes the same assignment."""
    order = sorted(range(len(costs)), key=lambda i: (-float(costs[i]), i))
    load = [0.0] * world
    owner = [0] * len(costs)
    for i in order:
        r = min(range(world), key=lambda j: (load[j], j))
        owner[i] = r
        load[r] += float(costs[i])
    return owner


class PeerExchange:
    """The per-layer exchange of config 4's partial triples over peer memory (sjk_xchg_*): every rank allocates one
    exchange buffer, the ranks swap its CUDA IPC handle once through the process group, and each layer call stores the
    rank's triples into every rank's buffer with NVLink stores and merges all ranks' triples locally in rank order.
    The output equals an all-gather + sjk_attend_merge of the same triples bit for bit."""

    def __init__(self, dist, rank, world, n_rows, D):
        import ctypes as C

        import sjk
        self.C, self.sjk, self.L = C, sjk, sjk.lib()
        self.rank, self.world, self.n_rows, self.D = rank, world, n_rows, D
        nbytes = self.L.sjk_xchg_bytes(world, n_rows, D)
        if nbytes == 0:
            raise ValueError("exchange shape out of range")
        self.buf = C.c_void_p()
        handle = (C.c_uint8 * 64)()
        sjk.check(self.L.sjk_xchg_alloc(nbytes, C.byref(self.buf), handle), "xchg_alloc")
        handles = [bytes(handle)] * world
        if dist is not None and world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle))
        self.peers = sjk.XchgPeers()
        self.peers.world, self.peers.rank = world, rank
        self.opened = []
        for r in range(world):
            if r == rank:
                self.peers.buf[r] = self.buf.value
            else:
                p = C.c_void_p()
                hb = (C.c_uint8 * 64).from_buffer_copy(handles[r])
                sjk.check(self.L.sjk_xchg_open(hb, C.byref(p)), "xchg_open")
                self.peers.buf[r] = p.value
                self.opened.append(p)
        self.dist = dist
        self.epoch = 0

    def exchange(self, part, out, stream):
        """part: this rank's [n_rows][D + 2] triples (device); out: [n_rows][D] merged output (device)."""
        C = self.C
        self.epoch += 1
        self.sjk.check(self.L.sjk_xchg_exchange(C.byref(self.peers), C.c_void_p(part.data_ptr()), self.n_rows, self.D,
                                                self.epoch, C.c_void_p(out.data_ptr()), stream), "xchg_exchange")

    def attend(self, view, B, N, qpos0, n_q, n_head, regions, q_ptr, scale, scratch, need, out_ptr, stream):
        """sjk_attend_partial_xchg: this rank's partial attention with the exchange and merge in its last kernel."""
        C = self.C
        self.epoch += 1
        self.sjk.check(self.L.sjk_attend_partial_xchg(C.byref(view), B, N, qpos0, n_q, n_head, regions, q_ptr, scale,
                                                      C.c_void_p(scratch.data_ptr()), need, C.byref(self.peers), self.epoch,
                                                      out_ptr, stream), "attend_partial_xchg")

    def close(self):
        """Collective: every rank calls it once all its exchanges have completed on the device."""
        import torch
        torch.cuda.synchronize()
        if self.dist is not None and self.world > 1:
            self.dist.barrier()
        for p in self.opened:
            self.L.sjk_xchg_close(p)
        self.opened = []
        if self.buf:
            self.L.sjk_xchg_free(self.buf)
            self.buf = self.C.c_void_p()
