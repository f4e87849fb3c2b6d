"""ctypes binding of libsjk_b200.so (include/sjk.h): the sj_kvarn.h API surface over device buffers
plus the device layer (sjk_*). Device pointers are plain integers (e.g. torch tensor .data_ptr()).

Loading fails loudly when the library has not been built: there is no CPU fallback.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsjk_b200.so")

u32 = C.c_uint32
vp = C.c_void_p


class Layout(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("D", "G", "bits_k", "bits_v", "body")] + \
               [(n, u32) for n in ("k_payload", "v_payload", "k_scale", "k_zero", "k_tok", "v_ch", "v_scale", "v_zero",
                                   "bytes")]


class Config(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("head_dim", "n_head_kv", "group", "bits_k", "bits_v", "body", "iters", "staging",
                                       "sink_type")] + \
               [(n, u32) for n in ("sink", "tail", "tail_max", "flush_chunk", "n_ubatch", "n_ctx")]


class Policy(C.Structure):
    _fields_ = [(n, u32) for n in ("sink", "tail", "tail_max", "group", "flush_chunk", "B", "B_prev", "B_pending")] + \
               [("draining", C.c_int)]


class Layer(C.Structure):
    _fields_ = [("cfg", Config), ("lay", Layout), ("cap", u32), ("n_groups", u32), ("stage_bytes", C.c_size_t),
                ("ring", vp), ("sink", vp), ("body", vp), ("blocks", vp), ("d_blocks", vp), ("owns_body", C.c_int),
                ("work", vp), ("work_bytes", C.c_size_t), ("stream", vp)]


class Pool(C.Structure):
    _fields_ = [("cfg", Config), ("lay", Layout), ("n_layers", C.c_int), ("n_blocks", u32), ("body", vp),
                ("free_ids", C.POINTER(u32)), ("n_free", u32)]


class Seq(C.Structure):
    _fields_ = [("cfg", Config), ("n_layers", C.c_int), ("layers", C.POINTER(Layer)), ("pol", Policy), ("n", u32),
                ("pool", C.POINTER(Pool)), ("blocks", C.POINTER(u32)), ("d_blocks", vp), ("stream", vp)]


class View(C.Structure):
    _fields_ = [("lay", Layout), ("n_head_kv", C.c_int), ("staging", C.c_int), ("sink_type", C.c_int), ("S", u32),
                ("cap", u32), ("stage_bytes", C.c_size_t), ("sink", vp), ("ring", vp), ("body", vp), ("blocks", vp)]


XCHG_MAX_WORLD = 16


class XchgPeers(C.Structure):
    _fields_ = [("buf", vp * XCHG_MAX_WORLD), ("world", C.c_int), ("rank", C.c_int)]


POOL_MAX_REQ, TRUNC_MAX_REQ = 128, 256


class BlockReq(C.Structure):
    """sjk_block_req: groups [g0, g1) of one sequence's DEVICE block table."""
    _fields_ = [("blocks", vp), ("g0", u32), ("g1", u32)]


class TruncReq(C.Structure):
    """sjk_trunc_req: one (sequence, layer) cache to scrub after a truncation (DEVICE pointers)."""
    _fields_ = [("body", vp), ("sink", vp), ("ring", vp), ("blocks", vp), ("S", u32), ("cap", u32), ("n_head_kv", u32),
                ("group", u32), ("rec_bytes", u32), ("sink_entry_bytes", u32), ("stage_bytes", u32), ("B_old", u32),
                ("B_new", u32), ("n_old", u32), ("resume", u32), ("release", C.c_int)]


class StateInfo(C.Structure):
    _fields_ = [("state_version", u32), ("format_version", u32), ("cfg", Config), ("rotation", u32),
                ("rotation_n", u32), ("codebook_id", C.c_uint64), ("n_layers", C.c_int), ("n", u32), ("B", u32),
                ("B_prev", u32), ("draining", u32), ("total_bytes", C.c_size_t)]


P = C.POINTER
SIGNATURES = {
    # host helpers
    "sj_kvarn_f32_to_f16": (C.c_uint16, [C.c_float]),
    "sj_kvarn_f16_to_f32": (C.c_float, [C.c_uint16]),
    "sj_kvarn_body_resolve": (C.c_int, [C.c_int, C.c_int, C.c_int]),
    "sj_kvarn_layout_init": (C.c_int, [P(Layout), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    "sj_kvarn_record_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int]),
    "sj_kvarn_body_bits_per_element": (C.c_double, [P(Layout)]),
    "sj_kvarn_code_bit": (u32, [P(Layout), C.c_int, C.c_int, C.c_int]),
    "sj_kvarn_k_ch_idx": (C.c_int, [P(Layout), C.c_int]),
    "sj_kvarn_v_ch_idx": (C.c_int, [P(Layout), C.c_int]),
    "sj_kvarn_seal_workspace_bytes": (C.c_size_t, [P(Layout)]),
    "sj_kvarn_stage_row_bytes": (C.c_size_t, [C.c_int, C.c_int]),
    # codec on device pointers
    "sj_kvarn_hadamard": (None, [vp, C.c_int]),
    "sj_kvarn_rotate_heads": (None, [vp, C.c_int, C.c_int]),
    "sj_kvarn_seal_group": (None, [P(Layout), vp, vp, C.c_size_t, C.c_int, vp, vp]),
    "sj_kvarn_decode_k_row": (None, [P(Layout), vp, C.c_int, vp]),
    "sj_kvarn_decode_v_row": (None, [P(Layout), vp, C.c_int, vp]),
    "sj_kvarn_record_scores": (None, [P(Layout), vp, vp, C.c_int, vp]),
    "sj_kvarn_record_accum_v": (None, [P(Layout), vp, vp, C.c_int, vp]),
    "sj_kvarn_tq6_quantize_row": (None, [vp, vp, C.c_int]),
    "sj_kvarn_tq6_dequantize_row": (None, [vp, vp, C.c_int]),
    "sj_kvarn_stage_row": (None, [C.c_int, vp, vp, C.c_int]),
    "sj_kvarn_unstage_row": (None, [C.c_int, vp, vp, C.c_int]),
    # policy
    "sj_kvarn_policy_init": (None, [P(Policy), u32, u32, u32, u32, u32]),
    "sj_kvarn_policy_reset": (None, [P(Policy)]),
    "sj_kvarn_policy_begin_ubatch": (u32, [P(Policy), u32, u32]),
    "sj_kvarn_policy_commit": (None, [P(Policy)]),
    "sj_kvarn_policy_idle": (u32, [P(Policy), u32, u32]),
    "sj_kvarn_group_floor": (u32, [u32, u32, u32]),
    "sj_kvarn_policy_trunc_floor": (u32, [P(Policy), u32]),
    "sj_kvarn_policy_truncate": (u32, [P(Policy), u32, P(u32)]),
    "sj_kvarn_ring_capacity": (u32, [u32, u32, u32, u32]),
    "sj_kvarn_ring_slot": (u32, [u32, u32, u32]),
    # layer
    "sj_kvarn_config_default": (Config, [C.c_int, C.c_int, u32, u32]),
    "sj_kvarn_layer_init": (C.c_int, [P(Layer), P(Config)]),
    "sj_kvarn_layer_free": (None, [P(Layer)]),
    "sj_kvarn_layer_store": (None, [P(Layer), u32, vp, vp]),
    "sj_kvarn_layer_seal": (None, [P(Layer), u32, u32]),
    "sj_kvarn_layer_kv_row": (None, [P(Layer), u32, u32, C.c_int, vp, vp]),
    "sj_kvarn_layer_attend_row": (None, [P(Layer), u32, u32, vp, C.c_int, u32, C.c_float, vp]),
    "sj_kvarn_layer_record": (vp, [P(Layer), u32, C.c_int]),
    "sj_kvarn_layer_truncate": (None, [P(Layer), u32, u32, u32, u32]),
    "sj_kvarn_strerror": (C.c_char_p, [C.c_int]),
    # pool / sequence / state
    "sj_kvarn_pool_init": (C.c_int, [P(Pool), P(Config), C.c_int, u32]),
    "sj_kvarn_pool_free": (None, [P(Pool)]),
    "sj_kvarn_pool_alloc": (u32, [P(Pool)]),
    "sj_kvarn_pool_release": (None, [P(Pool), u32]),
    "sj_kvarn_seq_init": (C.c_int, [P(Seq), P(Config), C.c_int, P(Pool)]),
    "sj_kvarn_seq_free": (None, [P(Seq)]),
    "sj_kvarn_seq_reset": (None, [P(Seq)]),
    "sj_kvarn_seq_begin_ubatch": (C.c_int, [P(Seq), u32, u32]),
    "sj_kvarn_seq_store": (None, [P(Seq), u32, vp, vp]),
    "sj_kvarn_seq_idle": (C.c_int, [P(Seq), u32]),
    "sj_kvarn_seq_truncate": (u32, [P(Seq), u32]),
    "sj_kvarn_seq_attend_row": (None, [P(Seq), C.c_int, vp, C.c_int, u32, C.c_float, vp]),
    "sj_kvarn_seq_state_size": (C.c_size_t, [P(Seq)]),
    "sj_kvarn_state_size_max": (C.c_size_t, [P(Config), C.c_int]),
    "sj_kvarn_seq_state_write": (C.c_int, [P(Seq), vp, C.c_size_t, P(C.c_size_t)]),
    "sj_kvarn_state_peek": (C.c_int, [vp, C.c_size_t, P(StateInfo)]),
    "sj_kvarn_seq_state_read": (C.c_int, [P(Seq), vp, C.c_size_t]),
    # device layer
    "sjk_last_error": (C.c_int, []),
    "sjk_last_cuda_error": (C.c_int, []),
    "sjk_device_status": (C.c_int, []),
    "sjk_version": (C.c_char_p, []),
    "sjk_hadamard": (C.c_int, [vp, C.c_int, C.c_int, vp]),
    "sjk_stage_rows": (C.c_int, [C.c_int, vp, vp, C.c_size_t, C.c_int, C.c_int, vp]),
    "sjk_unstage_rows": (C.c_int, [C.c_int, vp, C.c_size_t, vp, C.c_int, C.c_int, vp]),
    "sjk_store": (C.c_int, [P(View), vp, vp, u32, u32, vp, vp, C.c_int, vp]),
    "sjk_seal": (C.c_int, [P(Layout), vp, vp, C.c_size_t, C.c_int, C.c_int, C.c_int, vp, vp, vp]),
    "sjk_seal_ring": (C.c_int, [P(View), vp, u32, u32, C.c_int, vp]),
    "sjk_decode": (C.c_int, [P(Layout), vp, C.c_int, vp, vp, vp]),
    "sjk_attend_scratch_bytes": (C.c_size_t, [P(View), u32, C.c_int, C.c_int]),
    "sjk_attend": (C.c_int, [P(View), u32, u32, u32, C.c_int, C.c_int, vp, C.c_float, vp, vp, C.c_size_t, vp]),
    "sjk_attend_model": (C.c_int, [P(View), u32, u32, u32, C.c_int, C.c_int, vp, C.c_float, vp, vp, C.c_size_t, vp]),
    "sjk_layer_attend_model": (C.c_int, [P(Layer), u32, u32, u32, C.c_int, C.c_int, vp, C.c_float, vp, vp]),
    "sjk_attend_static": (C.c_int, [P(View), u32, u32, u32, C.c_int, C.c_int, vp, C.c_float, vp, vp]),
    "sjk_attend_partial": (C.c_int, [P(View), u32, u32, u32, C.c_int, C.c_int, C.c_uint, vp, C.c_float, vp, vp, C.c_size_t, vp]),
    "sjk_attend_merge": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, vp, vp]),
    "sjk_store_batch": (C.c_int, [P(View), P(u32), C.c_int, vp, vp, C.c_int, vp]),
    "sjk_seq_store": (C.c_int, [P(Seq), u32, u32, vp, vp, C.c_size_t, C.c_int, vp]),
    "sjk_attend_batch_scratch_bytes": (C.c_size_t, [P(View), C.c_int, C.c_int, C.c_int]),
    "sjk_attend_batch": (C.c_int, [P(View), P(u32), P(u32), P(u32), C.c_int, C.c_int, C.c_int, vp, C.c_float, vp, vp,
                                   C.c_size_t, vp]),
    "sjk_desc_fill": (C.c_int, [P(View), u32, u32, u32, u32, P(C.c_int32)]),
    "sjk_seal_dyn": (C.c_int, [P(View), vp, u32, C.c_int, vp]),
    "sjk_store_dyn": (C.c_int, [P(View), vp, u32, vp, vp, C.c_int, vp]),
    "sjk_attend_dyn_scratch_bytes": (C.c_size_t, [P(View), C.c_int, C.c_int]),
    "sjk_attend_dyn": (C.c_int, [P(View), vp, C.c_int, C.c_int, vp, C.c_float, vp, vp, C.c_size_t, vp]),
    "sjk_layer_store": (C.c_int, [P(Layer), u32, u32, vp, vp, C.c_int, vp]),
    "sjk_layer_seal": (C.c_int, [P(Layer), u32, u32, vp]),
    "sjk_layer_attend": (C.c_int, [P(Layer), u32, u32, u32, C.c_int, C.c_int, vp, C.c_float, vp, vp]),
    "sjk_layer_view": (None, [P(Layer), P(View)]),
    "sjk_layer_record_copy": (C.c_int, [P(Layer), u32, C.c_int, vp]),
    # exchange of partials over peer memory
    "sjk_pool_dev_bytes": (C.c_size_t, [u32]),
    "sjk_pool_dev_load": (C.c_int, [vp, P(Pool), vp]),
    "sjk_pool_dev_store": (C.c_int, [vp, P(Pool), vp]),
    "sjk_pool_reserve_batch": (C.c_int, [vp, P(BlockReq), C.c_int, vp, vp]),
    "sjk_pool_release_batch": (C.c_int, [vp, P(BlockReq), C.c_int, vp]),
    "sjk_truncate_batch": (C.c_int, [P(TruncReq), C.c_int, vp, vp]),
    "sjk_xchg_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int]),
    "sjk_xchg_alloc": (C.c_int, [C.c_size_t, P(vp), vp]),
    "sjk_xchg_free": (C.c_int, [vp]),
    "sjk_xchg_open": (C.c_int, [vp, P(vp)]),
    "sjk_xchg_close": (C.c_int, [vp]),
    "sjk_xchg_exchange": (C.c_int, [P(XchgPeers), vp, C.c_int, C.c_int, u32, vp, vp]),
    "sjk_attend_partial_xchg": (C.c_int, [P(View), u32, u32, u32, C.c_int, C.c_int, C.c_uint, vp, C.c_float, vp, C.c_size_t,
                                          P(XchgPeers), u32, vp, vp]),
    # seeded synthetic inputs
    "sjk_synth_scales": (C.c_int, [C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_int, vp, vp]),
    "sjk_synth_kv": (C.c_int, [C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_int, vp, u32, u32, vp, vp, vp]),
    "sjk_synth_q": (C.c_int, [C.c_uint64, C.c_int, u32, C.c_int, vp, vp]),
    "sjk_seal_libm_probe": (C.c_int, [vp, C.c_size_t, vp, vp, vp]),
}

_lib = None


def lib():
    """Load libsjk_b200.so (build it first with build.py / __graft_entry__.build())."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built: run `python build.py` in {HERE} (no CPU fallback exists)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


class SjkError(RuntimeError):
    def __init__(self, rc, what=""):
        self.rc = rc
        msg = lib().sj_kvarn_strerror(rc).decode()
        if rc == -200:
            msg += f" (cudaError {lib().sjk_last_cuda_error()})"
        super().__init__(f"{what}: {rc} {msg}" if what else f"{rc} {msg}")


def check(rc, what=""):
    if rc != 0:
        raise SjkError(rc, what)
    return rc


def check_sticky(what=""):
    rc = lib().sjk_last_error()
    if rc:
        raise SjkError(rc, what)


def layout(D, bits_k, bits_v, body, G=128):
    lay = Layout()
    check(lib().sj_kvarn_layout_init(C.byref(lay), D, G, bits_k, bits_v, body), "layout")
    return lay


def config(head_dim=256, n_head_kv=4, n_ctx=16384, n_ubatch=512, **kw):
    c = lib().sj_kvarn_config_default(head_dim, n_head_kv, n_ctx, n_ubatch)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


# descriptor entries of the descriptor-driven calls (include/sjk.h, the reference's ggml_sjkvarn_desc order)
(DESC_S, DESC_CAP, DESC_B, DESC_N, DESC_QPOS0, DESC_G, DESC_D, DESC_RECBYTES, DESC_HKV, DESC_B_OLD, DESC_TYPE_K,
 DESC_TYPE_V, DESC_BODY_TYPE, DESC_SINK_TYPE) = range(14)
DESC_N_ENTRIES = 16
DEVICE_TIMEOUT, DEVICE_DESC = 1, 2


def desc_fill(view, B_old, B, N, qpos0):
    """Host descriptor (numpy int32[16]) for view; raises SjkError when the kernels would reject the values."""
    import numpy as np
    d = np.zeros(DESC_N_ENTRIES, np.int32)
    check(lib().sjk_desc_fill(C.byref(view), B_old, B, N, qpos0, d.ctypes.data_as(C.POINTER(C.c_int32))), "desc_fill")
    return d


# region mask of sjk_attend_partial (include/sjk.h)
REGION_SINK, REGION_BODY, REGION_RING, REGION_ALL = 1, 2, 4, 7


def view_of(layer):
    v = View()
    lib().sjk_layer_view(C.byref(layer), C.byref(v))
    return v


def exported_symbols_in_header():
    """Names of every function declared in include/sjk.h."""
    import re
    hdr = open(os.path.join(HERE, "..", "include", "sjk.h")).read()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    names = set(re.findall(r"\b((?:sj_kvarn|sjk)_[a-z0-9_]+)\s*\(", hdr))
    return sorted(names)
