// sjk_host.cpp - the sj_kvarn.h API surface over device buffers: status codes, fp16 and layout helpers,
// the adaptive-tail policy, the per-layer cache, the paged record pool, sequences and the versioned
// sequence-state stream. Host control code; every byte of cache data lives in device memory and moves
// through the kernels of the device layer (sjk_*) or through plain cudaMemcpy for state save/restore.
#include <cuda_runtime.h>

#include <stdlib.h>
#include <string.h>

#include <cmath>

#include "../../include/sjk.h"
#include "sjk_internal.h"
#include "sjk_tables.h"

// ---- status plumbing --------------------------------------------------------------------------------------
static thread_local int g_sticky = 0;
static thread_local int g_cuda_err = 0;

void sjk_set_cuda_error(cudaError_t e) { g_cuda_err = (int) e; }
void sjk_set_sticky(int status) { if (status && !g_sticky) g_sticky = status; }

extern "C" int sjk_last_error(void) { const int s = g_sticky; g_sticky = 0; return s; }
extern "C" int sjk_last_cuda_error(void) { return g_cuda_err; }
extern "C" const char * sjk_version(void) { return "sjk-b200 2.0 (format 1, state 1)"; }

static int ck(cudaError_t e) {
    if (e != cudaSuccess) { g_cuda_err = (int) e; return SJK_ERR_DEVICE; }
    return 0;
}

// ---- fp16 (host) ----------------------------------------------------------------------------------------------
static inline uint16_t host_f2h(float f) {
    uint32_t w; memcpy(&w, &f, 4);
    const uint32_t sign = (w >> 16) & 0x8000u, a = w & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return (uint16_t) (sign | 0x7E00u);
    if (a >= 0x477FF000u) return (uint16_t) (sign | 0x7C00u);
    if (a < 0x38800000u) {
        if (a < 0x33000000u) return (uint16_t) sign;
        const int sh = 126 - (int) (a >> 23);
        const uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
        uint32_t q = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t) (sign | q);
    }
    uint32_t q = (a - 0x38000000u) >> 13;
    const uint32_t rem = a & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t) (sign | q);
}

static inline float host_h2f(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 31u;
    uint32_t m = h & 0x3FFu, w;
    if (e == 31u) w = sign | 0x7F800000u | (m << 13);
    else if (e) w = sign | ((e + 112u) << 23) | (m << 13);
    else if (!m) w = sign;
    else {
        const int lz = __builtin_clz(m) - 21;
        m <<= lz;
        w = sign | ((uint32_t) (113 - lz) << 23) | ((m & 0x3FFu) << 13);
    }
    float f; memcpy(&f, &w, 4);
    return f;
}

extern "C" uint16_t sj_kvarn_f32_to_f16(float f) { return host_f2h(f); }
extern "C" float sj_kvarn_f16_to_f32(uint16_t h) { return host_h2f(h); }

// ---- layout (sj_kvarn.h:763-849) -------------------------------------------------------------------------------
extern "C" int sj_kvarn_body_resolve(int body, int bits_k, int bits_v) {
    if (body != SJKVARN_BODY_AUTO) return body;
    const bool lk = bits_k == 2 || bits_k == 3, lv = bits_v == 2 || bits_v == 3;
    return lk && lv && bits_v <= bits_k ? SJKVARN_BODY_TRELLIS : SJKVARN_BODY_SCALAR;
}

extern "C" int sj_kvarn_layout_init(sj_kvarn_layout * l, int D, int G, int bits_k, int bits_v, int body) {
    if (D < 32 || (D & (D - 1)) || G <= 0 || G % 16) return -1;
    if (bits_k < 2 || bits_k > 4 || bits_v < 2 || bits_v > 4) return -2;
    if (body != SJKVARN_BODY_SCALAR && body != SJKVARN_BODY_TRELLIS) return -3;
    if (body == SJKVARN_BODY_TRELLIS && (bits_k == 4 || bits_v == 4 || bits_v > bits_k || G != 128 || D % 128)) return -4;
    l->D = D; l->G = G; l->bits_k = bits_k; l->bits_v = bits_v; l->body = body;
    l->k_payload = 0;
    l->v_payload = (uint32_t) (D * bits_k / 8) * (uint32_t) G;
    l->k_scale = l->v_payload + (uint32_t) (D * bits_v / 8) * (uint32_t) G;
    l->k_zero = l->k_scale + 2u * (uint32_t) D;
    l->k_tok = l->k_zero + 2u * (uint32_t) D;
    l->v_ch = l->k_tok + 2u * (uint32_t) G;
    l->v_scale = l->v_ch + 2u * (uint32_t) D;
    l->v_zero = l->v_scale + 2u * (uint32_t) G;
    l->bytes = l->v_zero + 2u * (uint32_t) G;
    return 0;
}

extern "C" size_t sj_kvarn_record_bytes(int D, int G, int bits_k, int bits_v) {
    return (size_t) G * D * bits_k / 8 + (size_t) G * D * bits_v / 8 + 2 * (3 * (size_t) D + 3 * (size_t) G);
}

extern "C" double sj_kvarn_body_bits_per_element(const sj_kvarn_layout * l) {
    return 8.0 * (double) l->bytes / (2.0 * (double) l->D * (double) l->G);
}

static bool frag_side(const sj_kvarn_layout * l, int bits) {
    return l->body == SJKVARN_BODY_SCALAR && bits == 4 && l->D % 16 == 0 && l->G % 16 == 0;
}

extern "C" uint32_t sj_kvarn_code_bit(const sj_kvarn_layout * l, int t, int d, int is_v) {
    const int bits = is_v ? l->bits_v : l->bits_k;
    if (l->body == SJKVARN_BODY_TRELLIS) return ((uint32_t) d * (uint32_t) l->G + (uint32_t) t) * (uint32_t) bits;
    if (!frag_side(l, bits)) return ((uint32_t) t * (uint32_t) l->D + (uint32_t) d) * (uint32_t) bits;
    const int row = is_v ? (d & 15) : (t & 15), col = is_v ? (t & 15) : (d & 15);
    const uint32_t tile = (uint32_t) ((t >> 4) * (l->D >> 4) + (d >> 4));
    const uint32_t lane = (uint32_t) (4 * (row & 7) + ((col >> 1) & 3));
    const uint32_t nib = (uint32_t) ((row >> 3) + 2 * (col >> 3) + 4 * (col & 1));
    return (tile * 32u + lane) * 32u + nib * 4u;
}

extern "C" int sj_kvarn_k_ch_idx(const sj_kvarn_layout * l, int d) {
    if (!frag_side(l, l->bits_k)) return d;
    const int dd = d & 15, pair = dd >> 1;
    return (pair & 3) * (l->D / 4) + (d >> 4) * 4 + (pair >> 2) * 2 + (dd & 1);
}

extern "C" int sj_kvarn_v_ch_idx(const sj_kvarn_layout * l, int d) {
    if (!frag_side(l, l->bits_v)) return d;
    const int dd = d & 15;
    return (dd & 7) * (l->D / 8) + (d >> 4) * 2 + (dd >> 3);
}

extern "C" size_t sj_kvarn_seal_workspace_bytes(const sj_kvarn_layout * l) { (void) l; return 0; }

extern "C" size_t sj_kvarn_stage_row_bytes(int staging, int D) {
    return staging == SJKVARN_STAGING_F16 ? (size_t) D * 2 : (size_t) (D / SJKVARN_TQ6_QK) * SJKVARN_TQ6_BLOCK_BYTES;
}

// ---- policy (sj_kvarn.h:1315-1407) -------------------------------------------------------------------------------
extern "C" void sj_kvarn_policy_reset(sj_kvarn_policy * p) {
    p->B = p->B_prev = p->B_pending = p->sink;
    p->draining = 0;
}

extern "C" void sj_kvarn_policy_init(sj_kvarn_policy * p, uint32_t sink, uint32_t tail, uint32_t tail_max, uint32_t group,
                                     uint32_t flush_chunk) {
    p->sink = sink; p->tail = tail; p->tail_max = tail_max; p->group = group; p->flush_chunk = flush_chunk;
    sj_kvarn_policy_reset(p);
}

extern "C" uint32_t sj_kvarn_group_floor(uint32_t sink, uint32_t group, uint32_t pos) {
    return pos <= sink ? pos : sink + group * ((pos - sink) / group);
}

// A commit is due when the unsealed span [B, pos0) reaches tail_max (or always with a fixed tail, or while
// a chunked drain is unfinished); it seals whole groups down to `tail` exact positions behind pos0.
extern "C" uint32_t sj_kvarn_policy_begin_ubatch(sj_kvarn_policy * p, uint32_t pos0, uint32_t n_tokens) {
    const bool due = p->tail_max == 0 || p->draining || (pos0 > p->B && pos0 - p->B >= p->tail_max);
    p->B_pending = p->B;
    p->draining = 0;
    if (due && pos0 > p->sink + p->tail) {
        uint32_t target = sj_kvarn_group_floor(p->sink, p->group, pos0 - p->tail);
        if (target < p->B) target = p->B;
        if (p->tail_max > 0 && p->flush_chunk > 0 && n_tokens < p->group) {
            const uint32_t cap = p->B + p->group * p->flush_chunk;
            if (target > cap) { target = cap; p->draining = 1; }
        }
        p->B_pending = target;
    }
    return p->B_pending;
}

extern "C" void sj_kvarn_policy_commit(sj_kvarn_policy * p) {
    p->B_prev = p->B;
    p->B = p->B_pending;
}

extern "C" uint32_t sj_kvarn_policy_idle(sj_kvarn_policy * p, uint32_t end, uint32_t keep_recent) {
    p->B_pending = p->B;
    if (p->tail_max == 0 || end <= p->sink + p->tail) return p->B;
    uint32_t target = sj_kvarn_group_floor(p->sink, p->group, end - p->tail);
    bool clamped = false;
    if (keep_recent > p->tail) {
        const uint32_t keep_from = end > keep_recent ? end - keep_recent : 0;
        const uint32_t lim = keep_from <= p->sink ? p->sink : sj_kvarn_group_floor(p->sink, p->group, keep_from);
        if (lim < target) { target = lim; clamped = true; }
    }
    if (!clamped) p->draining = 0;
    if (target <= p->B) return p->B;
    p->B_pending = target;
    return target;
}

extern "C" uint32_t sj_kvarn_policy_trunc_floor(const sj_kvarn_policy * p, uint32_t pos) {
    if (pos >= p->B || pos <= p->sink) return pos;
    return sj_kvarn_group_floor(p->sink, p->group, pos);
}

extern "C" uint32_t sj_kvarn_policy_truncate(sj_kvarn_policy * p, uint32_t pos, uint32_t * n_dropped) {
    if (n_dropped) *n_dropped = 0;
    if (p->B_pending != p->B) return SJKVARN_NO_POS;
    const uint32_t r = sj_kvarn_policy_trunc_floor(p, pos);
    if (r < p->B) {
        const uint32_t nb = r > p->sink ? r : p->sink;
        if (n_dropped) *n_dropped = (p->B - nb) / p->group;
        p->B = p->B_prev = p->B_pending = nb;
        p->draining = 0;
    }
    return r;
}

extern "C" uint32_t sj_kvarn_ring_capacity(uint32_t tail, uint32_t tail_max, uint32_t group, uint32_t n_ubatch) {
    const uint32_t need = (tail > tail_max ? tail : tail_max) + group + 2u * n_ubatch;
    return (need + 127u) / 128u * 128u;
}

extern "C" uint32_t sj_kvarn_ring_slot(uint32_t sink, uint32_t cap, uint32_t pos) { return (pos - sink) % cap; }

extern "C" const char * sj_kvarn_strerror(int code) {
    switch (code) {
        case SJKVARN_OK: return "ok";
        case -1: return "layout: head_dim must be a power of two >= 32 and group a multiple of 16";
        case -2: return "layout: bits_k and bits_v must be 2, 3 or 4";
        case -3: return "layout: unknown body type";
        case -4: return "layout: trellis bodies need 3/3, 3/2 or 2/2 bits, group 128 and head_dim a multiple of 128";
        case -10: return "config: head_dim % 128, group % 16, sink (non-zero, % 64), tail % group or tail_max invalid";
        case -11: return "out of memory";
        case SJKVARN_ERR_ARG: return "invalid argument";
        case SJKVARN_ERR_NOMEM: return "out of memory";
        case SJKVARN_ERR_BUFFER: return "destination buffer too small for the sequence state";
        case SJKVARN_ERR_TRUNCATED: return "state stream is shorter than its header says";
        case SJKVARN_ERR_MAGIC: return "not an SJ-KVaRN sequence state (bad magic)";
        case SJKVARN_ERR_VERSION: return "unsupported SJ-KVaRN state version";
        case SJKVARN_ERR_FORMAT: return "state was written with a different record/staging byte format";
        case SJKVARN_ERR_CORRUPT: return "state checksum or consistency check failed";
        case SJKVARN_ERR_PENDING: return "a seal is pending (call commit first)";
        case SJKVARN_ERR_CAPACITY: return "state does not fit this cache (context, ring or group capacity)";
        case SJKVARN_ERR_POOL_FULL: return "record pool has no free block";
        case SJKVARN_ERR_HEAD_DIM: return "config mismatch: head_dim";
        case SJKVARN_ERR_N_HEAD_KV: return "config mismatch: n_head_kv";
        case SJKVARN_ERR_GROUP: return "config mismatch: group size";
        case SJKVARN_ERR_SINK: return "config mismatch: sink length or sink type";
        case SJKVARN_ERR_BITS: return "config mismatch: bits_k/bits_v";
        case SJKVARN_ERR_BODY: return "config mismatch: body type (scalar/trellis)";
        case SJKVARN_ERR_ITERS: return "config mismatch: variance-balancing iterations";
        case SJKVARN_ERR_STAGING: return "config mismatch: staging type";
        case SJKVARN_ERR_TAIL: return "config mismatch: tail, tail_max or flush_chunk";
        case SJKVARN_ERR_ROTATION: return "config mismatch: rotation";
        case SJKVARN_ERR_CODEBOOK: return "config mismatch: trellis codebook";
        case SJKVARN_ERR_N_LAYERS: return "config mismatch: number of layers";
        case SJK_ERR_DEVICE: return "CUDA error (see sjk_last_cuda_error)";
        case SJK_ERR_UNSUPPORTED: return "shape not implemented by the B200 kernels";
        case SJK_ERR_SCRATCH_LIMIT: return "shape needs more scratch than the fixed no-allocation buffer holds (16 MiB)";
        default: return "unknown SJ-KVaRN status code";
    }
}

// ---- single-object codec calls on device pointers (sj_kvarn.h:197-216) -------------------------------------
static void sticky(int rc) { if (rc) sjk_set_sticky(rc); }

extern "C" void sj_kvarn_hadamard(float * x, int n) { sticky(sjk_hadamard(x, 1, n, 0)); }
extern "C" void sj_kvarn_rotate_heads(float * x, int n_heads, int head_dim) { sticky(sjk_hadamard(x, n_heads, head_dim, 0)); }

extern "C" void sj_kvarn_seal_group(const sj_kvarn_layout * l, const uint16_t * K, const uint16_t * V, size_t row_stride,
                                    int iters, uint8_t * rec, void * work) {
    sticky(sjk_seal(l, K, V, row_stride, 1, 1, iters, rec, work, 0));
}
extern "C" void sj_kvarn_decode_k_row(const sj_kvarn_layout * l, const uint8_t * rec, int t, float * out) {
    sticky(sjk_decode_row(l, rec, t, 0, out, 0));
}
extern "C" void sj_kvarn_decode_v_row(const sj_kvarn_layout * l, const uint8_t * rec, int t, float * out) {
    sticky(sjk_decode_row(l, rec, t, 1, out, 0));
}
extern "C" void sj_kvarn_record_scores(const sj_kvarn_layout * l, const uint8_t * rec, const float * q, int n, float * scores) {
    sticky(sjk_record_scores(l, rec, q, n, scores, 0));
}
extern "C" void sj_kvarn_record_accum_v(const sj_kvarn_layout * l, const uint8_t * rec, const float * w, int n, float * acc) {
    sticky(sjk_record_accum_v(l, rec, w, n, acc, 0));
}
extern "C" void sj_kvarn_tq6_quantize_row(const float * x, sj_kvarn_tq6_block * y, int n) {
    sticky(sjk_stage_rows(SJKVARN_STAGING_TQ6_0, x, (uint8_t *) y, (size_t) n / 128 * SJKVARN_TQ6_BLOCK_BYTES, n, 1, 0));
}
extern "C" void sj_kvarn_tq6_dequantize_row(const sj_kvarn_tq6_block * y, float * x, int n) {
    sticky(sjk_unstage_rows(SJKVARN_STAGING_TQ6_0, (const uint8_t *) y, (size_t) n / 128 * SJKVARN_TQ6_BLOCK_BYTES, x, n, 1, 0));
}
extern "C" void sj_kvarn_stage_row(int staging, const float * x_rot, void * dst, int D) {
    sticky(sjk_stage_rows(staging, x_rot, (uint8_t *) dst, sj_kvarn_stage_row_bytes(staging, D), D, 1, 0));
}
extern "C" void sj_kvarn_unstage_row(int staging, const void * src, float * x_rot, int D) {
    sticky(sjk_unstage_rows(staging, (const uint8_t *) src, sj_kvarn_stage_row_bytes(staging, D), x_rot, D, 1, 0));
}

// ---- per-layer cache (sj_kvarn.h:1409-1603) ---------------------------------------------------------------------
extern "C" sj_kvarn_config sj_kvarn_config_default(int head_dim, int n_head_kv, uint32_t n_ctx, uint32_t n_ubatch) {
    sj_kvarn_config c;
    memset(&c, 0, sizeof c);
    c.head_dim = head_dim; c.n_head_kv = n_head_kv;
    c.group = SJKVARN_GROUP_DEFAULT;
    c.bits_k = 4; c.bits_v = 4;
    c.body = SJKVARN_BODY_AUTO;
    c.iters = SJKVARN_ITERS_DEFAULT;
    c.staging = SJKVARN_STAGING_TQ6_0;
    c.sink_type = SJKVARN_SINK_F16;
    c.sink = SJKVARN_SINK_DEFAULT;
    c.tail = SJKVARN_TAIL_DEFAULT;
    c.tail_max = SJKVARN_TAIL_MAX_DEFAULT;
    c.flush_chunk = 0;
    c.n_ubatch = n_ubatch;
    c.n_ctx = n_ctx;
    return c;
}

extern "C" void sjk_layer_view(const sj_kvarn_layer * L, sjk_view * v) {
    v->lay = L->lay;
    v->n_head_kv = L->cfg.n_head_kv;
    v->staging = L->cfg.staging;
    v->sink_type = L->cfg.sink_type;
    v->S = L->cfg.sink;
    v->cap = L->cap;
    v->stage_bytes = L->stage_bytes;
    v->sink = L->sink;
    v->ring = L->ring;
    v->body = L->body;
    v->blocks = L->blocks ? L->d_blocks : NULL;
}

static size_t sink_entry_bytes(const sj_kvarn_layer * L) {
    return L->cfg.sink_type == SJKVARN_SINK_F16 ? (size_t) L->cfg.head_dim * 4 : 2 * L->stage_bytes;
}

static int layer_init_impl(sj_kvarn_layer * L, const sj_kvarn_config * cfg, int own_body) {
    const int D = cfg->head_dim, H = cfg->n_head_kv;
    memset(L, 0, sizeof(*L));
    L->cfg = *cfg;
    const int body = sj_kvarn_body_resolve(cfg->body, cfg->bits_k, cfg->bits_v);
    L->cfg.body = body;
    if (D % SJKVARN_TQ6_QK != 0 || cfg->group % 16 != 0 || cfg->sink == 0 || cfg->sink % 64 != 0 ||
        cfg->tail % (uint32_t) cfg->group != 0 || (cfg->tail_max != 0 && (cfg->tail_max < cfg->tail || cfg->tail_max % 128 != 0)))
        return -10;
    const int rc = sj_kvarn_layout_init(&L->lay, D, cfg->group, cfg->bits_k, cfg->bits_v, body);
    if (rc) return rc;
    if (H <= 0) return SJKVARN_ERR_ARG;
    L->cap = sj_kvarn_ring_capacity(cfg->tail, cfg->tail_max, (uint32_t) cfg->group, cfg->n_ubatch);
    L->n_groups = cfg->n_ctx > cfg->sink ? (cfg->n_ctx - cfg->sink + (uint32_t) cfg->group - 1) / (uint32_t) cfg->group : 1;
    L->stage_bytes = sj_kvarn_stage_row_bytes(cfg->staging, D);
    L->owns_body = own_body;
    const size_t ring_b = (size_t) L->cap * H * 2 * L->stage_bytes;
    const size_t sink_b = (size_t) cfg->sink * H * sink_entry_bytes(L);
    const size_t body_b = own_body ? (size_t) L->n_groups * H * L->lay.bytes : 0;
    sjk_view v;
    sjk_layer_view(L, &v);
    L->work_bytes = sjk_attend_heads_scratch_bytes(&v, 1, 1, 1);
    bool ok = cudaMalloc((void **) &L->ring, ring_b) == cudaSuccess && cudaMalloc((void **) &L->sink, sink_b) == cudaSuccess &&
              cudaMalloc(&L->work, L->work_bytes) == cudaSuccess;
    if (ok && own_body) ok = cudaMalloc((void **) &L->body, body_b) == cudaSuccess;
    if (ok) ok = cudaMemset(L->ring, 0, ring_b) == cudaSuccess && cudaMemset(L->sink, 0, sink_b) == cudaSuccess &&
                 (!own_body || cudaMemset(L->body, 0, body_b) == cudaSuccess);
    if (!ok) {
        cudaGetLastError();
        sj_kvarn_layer_free(L);
        return -11;
    }
    return 0;
}

extern "C" int sj_kvarn_layer_init(sj_kvarn_layer * L, const sj_kvarn_config * cfg) { return layer_init_impl(L, cfg, 1); }

extern "C" void sj_kvarn_layer_free(sj_kvarn_layer * L) {
    if (L->ring) cudaFree(L->ring);
    if (L->sink) cudaFree(L->sink);
    if (L->owns_body && L->body) cudaFree(L->body);
    if (L->work) cudaFree(L->work);
    L->ring = L->sink = L->body = NULL;
    L->work = NULL;
    L->blocks = NULL; L->d_blocks = NULL;
    L->owns_body = 0;
}

extern "C" int sjk_layer_store(sj_kvarn_layer * L, uint32_t pos0, uint32_t n_pos, const float * k, const float * v,
                               int rotate, sjk_stream st) {
    sjk_view vw;
    sjk_layer_view(L, &vw);
    return sjk_store(&vw, L->sink, L->ring, pos0, n_pos, k, v, rotate, st);
}

extern "C" int sjk_layer_seal(sj_kvarn_layer * L, uint32_t B_from, uint32_t B_to, sjk_stream st) {
    sjk_view vw;
    sjk_layer_view(L, &vw);
    return sjk_seal_ring(&vw, L->body, B_from, B_to, L->cfg.iters, st);
}

// the layer's attention scratch, grown to `need` (outside any stream capture; the old buffer is released after the
// stream drains)
static int layer_work(const sj_kvarn_layer * L, size_t need, sjk_stream st) {
    if (need <= L->work_bytes) return 0;
    void * w = NULL;
    if (ck(cudaStreamSynchronize(st))) return SJK_ERR_DEVICE;
    if (ck(cudaMalloc(&w, need))) return SJK_ERR_DEVICE;
    sj_kvarn_layer * Lm = (sj_kvarn_layer *) L;
    cudaFree(Lm->work);
    Lm->work = w; Lm->work_bytes = need;
    return 0;
}

extern "C" int sjk_layer_attend(const sj_kvarn_layer * L, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head,
                                const float * q, float scale, float * out, sjk_stream st) {
    sjk_view vw;
    sjk_layer_view(L, &vw);
    const int rc = layer_work(L, sjk_attend_scratch_bytes(&vw, N, n_q, n_head), st);
    if (rc) return rc;
    return sjk_attend(&vw, B, N, qpos0, n_q, n_head, q, scale, out, L->work, L->work_bytes, st);
}

extern "C" int sjk_layer_attend_model(const sj_kvarn_layer * L, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head,
                                      const float * q, float scale, float * out, sjk_stream st) {
    sjk_view vw;
    sjk_layer_view(L, &vw);
    const int rc = layer_work(L, sjk_attend_scratch_bytes(&vw, N, n_q, n_head), st);
    if (rc) return rc;
    return sjk_attend_model(&vw, B, N, qpos0, n_q, n_head, q, scale, out, L->work, L->work_bytes, st);
}

extern "C" void sj_kvarn_layer_store(sj_kvarn_layer * L, uint32_t pos, const float * k_rot, const float * v_rot) {
    sticky(sjk_layer_store(L, pos, 1, k_rot, v_rot, 0, L->stream));
}

extern "C" void sj_kvarn_layer_seal(sj_kvarn_layer * L, uint32_t B_from, uint32_t B_to) {
    sticky(sjk_layer_seal(L, B_from, B_to, L->stream));
}

extern "C" void sj_kvarn_layer_kv_row(const sj_kvarn_layer * L, uint32_t B, uint32_t pos, int h, float * k, float * v) {
    sjk_view vw;
    sjk_layer_view(L, &vw);
    sticky(sjk_kv_row(&vw, B, pos, h, k, v, L->stream));
}

extern "C" void sj_kvarn_layer_attend_row(const sj_kvarn_layer * L, uint32_t B, uint32_t N, const float * q_rot, int h,
                                          uint32_t qpos, float scale, float * out_rot) {
    sjk_view vw;
    sjk_layer_view(L, &vw);
    sticky(sjk_attend_heads(&vw, B, N, qpos, 1, 1, h, 1, q_rot, scale, out_rot, L->work, L->work_bytes, L->stream,
                            SJK_REGION_ALL, nullptr));
}

extern "C" uint8_t * sj_kvarn_layer_record(const sj_kvarn_layer * L, uint32_t g, int h) {
    const uint32_t blk = L->blocks ? L->blocks[g] : g;
    return L->body + ((size_t) blk * (size_t) L->cfg.n_head_kv + (size_t) h) * L->lay.bytes;
}

extern "C" int sjk_layer_record_copy(const sj_kvarn_layer * L, uint32_t g, int h, void * host_dst) {
    if (ck(cudaStreamSynchronize(L->stream))) return SJK_ERR_DEVICE;
    return ck(cudaMemcpy(host_dst, sj_kvarn_layer_record(L, g, h), L->lay.bytes, cudaMemcpyDeviceToHost));
}

static uint8_t * sink_row(const sj_kvarn_layer * L, uint32_t pos, int h) {
    return L->sink + ((size_t) pos * (size_t) L->cfg.n_head_kv + (size_t) h) * sink_entry_bytes(L);
}

static uint8_t * ring_row(const sj_kvarn_layer * L, uint32_t pos, int h) {
    return L->ring + ((size_t) sj_kvarn_ring_slot(L->cfg.sink, L->cap, pos) * (size_t) L->cfg.n_head_kv + (size_t) h) * 2 *
                         L->stage_bytes;
}

// Scrub after a truncation (sj_kvarn.h:1581-1603): zero dropped records and the sink/ring rows of
// positions [resume, n_old). Runs as stream-ordered memsets on whole contiguous spans.
extern "C" void sj_kvarn_layer_truncate(sj_kvarn_layer * L, uint32_t B_old, uint32_t B_new, uint32_t n_old, uint32_t resume) {
    const uint32_t S = L->cfg.sink, G = (uint32_t) L->cfg.group;
    const int H = L->cfg.n_head_kv;
    int rc = 0;
    if (B_new < B_old) {
        // the dropped groups: one memset over a contiguous body, one scrub launch through a pool's block table
        const uint32_t g0 = (B_new - S) / G, g1 = (B_old - S) / G;
        const size_t grp = (size_t) H * L->lay.bytes;
        if (!L->blocks) rc = ck(cudaMemsetAsync(L->body + (size_t) g0 * grp, 0, (size_t) (g1 - g0) * grp, L->stream));
        else if (L->d_blocks) rc = sjk_group_move(L->body, L->d_blocks, g0, g1 - g0, grp, NULL, 2, L->stream);
        else
            for (uint32_t g = g0; g < g1 && !rc; ++g)
                if (L->blocks[g] != SJKVARN_NO_BLOCK) rc = ck(cudaMemsetAsync(L->body + (size_t) L->blocks[g] * grp, 0, grp, L->stream));
    }
    if (resume < n_old && resume < S && !rc) {
        const uint32_t end = n_old < S ? n_old : S;
        rc = ck(cudaMemsetAsync(sink_row(L, resume, 0), 0, (size_t) (end - resume) * H * sink_entry_bytes(L), L->stream));
    }
    uint32_t from = resume > S ? resume : S;
    if (n_old > from && n_old - from > L->cap) from = n_old - L->cap;
    // ring rows of [from, n_old): contiguous slot runs (at most two, the ring wraps once)
    while (from < n_old && !rc) {
        const uint32_t slot = sj_kvarn_ring_slot(S, L->cap, from);
        uint32_t run = L->cap - slot;
        if (run > n_old - from) run = n_old - from;
        rc = ck(cudaMemsetAsync(ring_row(L, from, 0), 0, (size_t) run * H * 2 * L->stage_bytes, L->stream));
        from += run;
    }
    sticky(rc);
}

// ---- paged record pool (sj_kvarn.h:1643-1675) ---------------------------------------------------------------------
extern "C" int sj_kvarn_pool_init(sj_kvarn_pool * pool, const sj_kvarn_config * cfg, int n_layers, uint32_t n_blocks) {
    memset(pool, 0, sizeof(*pool));
    if (n_layers <= 0 || n_blocks == 0 || cfg->n_head_kv <= 0) return SJKVARN_ERR_ARG;
    pool->cfg = *cfg;
    pool->cfg.body = sj_kvarn_body_resolve(cfg->body, cfg->bits_k, cfg->bits_v);
    const int rc = sj_kvarn_layout_init(&pool->lay, cfg->head_dim, cfg->group, cfg->bits_k, cfg->bits_v, pool->cfg.body);
    if (rc) return rc;
    pool->n_layers = n_layers;
    pool->n_blocks = n_blocks;
    const size_t bytes = (size_t) n_layers * n_blocks * (size_t) cfg->n_head_kv * pool->lay.bytes;
    pool->free_ids = (uint32_t *) malloc((size_t) n_blocks * sizeof(uint32_t));
    if (!pool->free_ids || cudaMalloc((void **) &pool->body, bytes) != cudaSuccess || cudaMemset(pool->body, 0, bytes) != cudaSuccess) {
        cudaGetLastError();
        sj_kvarn_pool_free(pool);
        return SJKVARN_ERR_NOMEM;
    }
    for (uint32_t i = 0; i < n_blocks; ++i) pool->free_ids[i] = n_blocks - 1u - i;   // block 0 is handed out first
    pool->n_free = n_blocks;
    return SJKVARN_OK;
}

extern "C" void sj_kvarn_pool_free(sj_kvarn_pool * pool) {
    if (pool->body) cudaFree(pool->body);
    free(pool->free_ids);
    pool->body = NULL; pool->free_ids = NULL; pool->n_free = 0;
}

extern "C" uint32_t sj_kvarn_pool_alloc(sj_kvarn_pool * pool) {
    return pool->n_free ? pool->free_ids[--pool->n_free] : SJKVARN_NO_BLOCK;
}

extern "C" void sj_kvarn_pool_release(sj_kvarn_pool * pool, uint32_t id) {
    if (id != SJKVARN_NO_BLOCK && pool->n_free < pool->n_blocks) pool->free_ids[pool->n_free++] = id;
}

// ---- sequence (sj_kvarn.h:1677-1809) -------------------------------------------------------------------------------
static int push_blocks(sj_kvarn_seq * s, uint32_t g0, uint32_t g1) {
    if (!s->pool || !s->d_blocks || g1 <= g0) return 0;
    return ck(cudaMemcpyAsync(s->d_blocks + g0, s->blocks + g0, (size_t) (g1 - g0) * sizeof(uint32_t),
                              cudaMemcpyHostToDevice, s->stream));
}

extern "C" int sj_kvarn_seq_init(sj_kvarn_seq * s, const sj_kvarn_config * cfg, int n_layers, sj_kvarn_pool * pool) {
    memset(s, 0, sizeof(*s));
    if (n_layers <= 0) return SJKVARN_ERR_ARG;
    s->cfg = *cfg;
    s->cfg.body = sj_kvarn_body_resolve(cfg->body, cfg->bits_k, cfg->bits_v);
    if (pool) {
        const sj_kvarn_config * pc = &pool->cfg;
        if (pool->n_layers != n_layers || pc->head_dim != cfg->head_dim || pc->n_head_kv != cfg->n_head_kv ||
            pc->group != cfg->group || pc->bits_k != cfg->bits_k || pc->bits_v != cfg->bits_v || pc->body != s->cfg.body)
            return SJKVARN_ERR_ARG;
    }
    s->n_layers = n_layers;
    s->pool = pool;
    s->layers = (sj_kvarn_layer *) calloc((size_t) n_layers, sizeof(sj_kvarn_layer));
    if (!s->layers) return SJKVARN_ERR_NOMEM;
    for (int il = 0; il < n_layers; ++il) {
        const int rc = layer_init_impl(&s->layers[il], cfg, pool == NULL);
        if (rc) { s->n_layers = il; sj_kvarn_seq_free(s); return rc; }
    }
    if (pool) {
        const uint32_t ng = s->layers[0].n_groups;
        s->blocks = (uint32_t *) malloc((size_t) ng * sizeof(uint32_t));
        if (!s->blocks || cudaMalloc((void **) &s->d_blocks, (size_t) ng * sizeof(uint32_t)) != cudaSuccess) {
            cudaGetLastError();
            sj_kvarn_seq_free(s);
            return SJKVARN_ERR_NOMEM;
        }
        for (uint32_t g = 0; g < ng; ++g) s->blocks[g] = SJKVARN_NO_BLOCK;
        if (push_blocks(s, 0, ng)) { sj_kvarn_seq_free(s); return SJKVARN_ERR_NOMEM; }
        for (int il = 0; il < n_layers; ++il) {
            s->layers[il].body = pool->body + (size_t) il * pool->n_blocks * (size_t) cfg->n_head_kv * pool->lay.bytes;
            s->layers[il].blocks = s->blocks;
            s->layers[il].d_blocks = s->d_blocks;
        }
    }
    sj_kvarn_policy_init(&s->pol, cfg->sink, cfg->tail, cfg->tail_max, (uint32_t) cfg->group, cfg->flush_chunk);
    s->n = 0;
    return SJKVARN_OK;
}

// pool mode: return the blocks of groups [g0, g1) to the pool
static void seq_release(sj_kvarn_seq * s, uint32_t g0, uint32_t g1) {
    if (!s->pool || !s->blocks) return;
    const uint32_t ng = s->layers[0].n_groups;
    if (g1 > ng) g1 = ng;
    for (uint32_t g = g0; g < g1; ++g) {
        sj_kvarn_pool_release(s->pool, s->blocks[g]);
        s->blocks[g] = SJKVARN_NO_BLOCK;
    }
    sticky(push_blocks(s, g0, g1));
}

// pool mode: give groups [g0, g1) blocks; on failure release what this call took
static int seq_reserve(sj_kvarn_seq * s, uint32_t g0, uint32_t g1) {
    if (!s->pool) return SJKVARN_OK;
    if (g1 > s->layers[0].n_groups) return SJKVARN_ERR_CAPACITY;
    for (uint32_t g = g0; g < g1; ++g) {
        if (s->blocks[g] != SJKVARN_NO_BLOCK) continue;
        s->blocks[g] = sj_kvarn_pool_alloc(s->pool);
        if (s->blocks[g] == SJKVARN_NO_BLOCK) {
            while (g-- > g0) { sj_kvarn_pool_release(s->pool, s->blocks[g]); s->blocks[g] = SJKVARN_NO_BLOCK; }
            return SJKVARN_ERR_POOL_FULL;
        }
    }
    return push_blocks(s, g0, g1);
}

extern "C" void sj_kvarn_seq_free(sj_kvarn_seq * s) {
    if (s->layers) {
        if (s->pool && s->blocks) seq_release(s, 0, s->layers[0].n_groups);
        for (int il = 0; il < s->n_layers; ++il) sj_kvarn_layer_free(&s->layers[il]);
    }
    free(s->layers);
    free(s->blocks);
    if (s->d_blocks) cudaFree(s->d_blocks);
    s->layers = NULL; s->blocks = NULL; s->d_blocks = NULL; s->n_layers = 0; s->n = 0;
}

extern "C" void sj_kvarn_seq_reset(sj_kvarn_seq * s) {
    for (int il = 0; il < s->n_layers; ++il) sj_kvarn_layer_truncate(&s->layers[il], s->pol.B, s->cfg.sink, s->n, 0);
    seq_release(s, 0, s->layers[0].n_groups);
    sj_kvarn_policy_reset(&s->pol);
    s->n = 0;
}

static void set_layer_streams(sj_kvarn_seq * s) {
    for (int il = 0; il < s->n_layers; ++il) s->layers[il].stream = s->stream;
}

// seal [B, B_pending) in every layer and commit, or undo the policy step
static int seq_seal_commit(sj_kvarn_seq * s, const sj_kvarn_policy * before) {
    const uint32_t S = s->cfg.sink, G = (uint32_t) s->cfg.group;
    set_layer_streams(s);
    if (s->pol.B_pending > s->pol.B) {
        const int rc = seq_reserve(s, (s->pol.B - S) / G, (s->pol.B_pending - S) / G);
        if (rc != SJKVARN_OK) { s->pol = *before; return rc; }
        for (int il = 0; il < s->n_layers; ++il) {
            const int r2 = sjk_layer_seal(&s->layers[il], s->pol.B, s->pol.B_pending, s->stream);
            if (r2) { s->pol = *before; return r2; }
        }
    }
    sj_kvarn_policy_commit(&s->pol);
    return SJKVARN_OK;
}

extern "C" int sj_kvarn_seq_begin_ubatch(sj_kvarn_seq * s, uint32_t pos0, uint32_t n_tokens) {
    const sj_kvarn_policy before = s->pol;
    if (pos0 > s->n) return SJKVARN_ERR_ARG;
    sj_kvarn_policy_begin_ubatch(&s->pol, pos0, n_tokens);
    return seq_seal_commit(s, &before);
}

extern "C" void sj_kvarn_seq_store(sj_kvarn_seq * s, uint32_t pos, const float * k_rot, const float * v_rot) {
    const size_t stride = (size_t) s->cfg.n_head_kv * (size_t) s->cfg.head_dim;
    for (int il = 0; il < s->n_layers; ++il)
        sticky(sjk_layer_store(&s->layers[il], pos, 1, k_rot + (size_t) il * stride, v_rot + (size_t) il * stride, 0, s->stream));
    if (pos + 1u > s->n) s->n = pos + 1u;
}

// Prefill form of sj_kvarn_seq_store: n_pos consecutive positions of every layer in one call per layer. Layer il's rows
// are DEVICE [n_pos][n_head_kv][D] floats at k + il layer_stride (0: n_pos n_head_kv D), rotated (rotate = 0) or in
// the model basis (rotate = 1).
extern "C" int sjk_seq_store(sj_kvarn_seq * s, uint32_t pos0, uint32_t n_pos, const float * k, const float * v,
                             size_t layer_stride, int rotate, sjk_stream st) {
    if (!s || !k || !v || pos0 > s->n) return SJKVARN_ERR_ARG;
    if (n_pos == 0) return 0;
    const size_t stride = layer_stride ? layer_stride : (size_t) n_pos * (size_t) s->cfg.n_head_kv * (size_t) s->cfg.head_dim;
    for (int il = 0; il < s->n_layers; ++il) {
        const int rc = sjk_layer_store(&s->layers[il], pos0, n_pos, k + (size_t) il * stride, v + (size_t) il * stride, rotate, st);
        if (rc) return rc;
    }
    if (pos0 + n_pos > s->n) s->n = pos0 + n_pos;
    return 0;
}

extern "C" int sj_kvarn_seq_idle(sj_kvarn_seq * s, uint32_t keep_recent) {
    const sj_kvarn_policy before = s->pol;
    sj_kvarn_policy_idle(&s->pol, s->n, keep_recent);
    return seq_seal_commit(s, &before);
}

extern "C" uint32_t sj_kvarn_seq_truncate(sj_kvarn_seq * s, uint32_t pos) {
    const uint32_t S = s->cfg.sink, G = (uint32_t) s->cfg.group, B_old = s->pol.B, n_old = s->n;
    const uint32_t r = sj_kvarn_policy_truncate(&s->pol, pos, NULL);
    if (r == SJKVARN_NO_POS) return r;
    set_layer_streams(s);
    for (int il = 0; il < s->n_layers; ++il) sj_kvarn_layer_truncate(&s->layers[il], B_old, s->pol.B, n_old, r);
    if (s->pol.B < B_old) seq_release(s, (s->pol.B - S) / G, (B_old - S) / G);
    if (r < s->n) s->n = r;
    return r;
}

extern "C" void sj_kvarn_seq_attend_row(const sj_kvarn_seq * s, int il, const float * q_rot, int h, uint32_t qpos, float scale,
                                        float * out_rot) {
    sj_kvarn_layer * L = &s->layers[il];
    L->stream = s->stream;
    sj_kvarn_layer_attend_row(L, s->pol.B, s->n, q_rot, h, qpos, scale, out_rot);
}

// ---- sequence state (sj_kvarn.h:417-453, 1811-2034) ----------------------------------------------------------------
// Stream: 128-byte little-endian header, then per layer the sink rows of [0, min(sink, n)), the records
// of groups [0, (B-sink)/G) in [group][head] order and the staging rows of [B, n) in position order, then
// an FNV-1a 64 checksum of everything before it. Payload bytes are copied straight from device memory.
static const uint8_t k_magic[8] = {'S', 'J', 'K', 'V', 'S', 'E', 'Q', 0};
static const uint64_t k_fnv0 = 1469598103934665603ULL;

static uint64_t fnv1a(const uint8_t * p, size_t n, uint64_t h) {
    for (size_t i = 0; i < n; ++i) { h ^= p[i]; h *= 1099511628211ULL; }
    return h;
}
static void wr32(uint8_t * p, uint32_t v) { for (int i = 0; i < 4; ++i) p[i] = (uint8_t) (v >> (8 * i)); }
static void wr64(uint8_t * p, uint64_t v) { wr32(p, (uint32_t) v); wr32(p + 4, (uint32_t) (v >> 32)); }
static uint32_t rd32(const uint8_t * p) { return (uint32_t) p[0] | (uint32_t) p[1] << 8 | (uint32_t) p[2] << 16 | (uint32_t) p[3] << 24; }
static uint64_t rd64(const uint8_t * p) { return (uint64_t) rd32(p) | (uint64_t) rd32(p + 4) << 32; }

// FNV-1a 64 of the K then V codebook tables of a trellis body (0 for scalar bodies)
static uint64_t codebook_id(int body, int bits_k, int bits_v) {
    if (body != SJKVARN_BODY_TRELLIS) return 0;
    static const uint16_t cb3k[512] = SJK_CB3_K_INIT, cb3v[512] = SJK_CB3_V_INIT;
    static const uint16_t cb2k[256] = SJK_CB2_K_INIT, cb2v[256] = SJK_CB2_V_INIT;
    const uint16_t * k = bits_k == 3 ? cb3k : cb2k;
    const uint16_t * v = bits_v == 3 ? cb3v : cb2v;
    uint8_t buf[1024];
    uint64_t h = k_fnv0;
    const int nk = bits_k == 3 ? 512 : 256, nv = bits_v == 3 ? 512 : 256;
    for (int i = 0; i < nk; ++i) { buf[2 * i] = (uint8_t) k[i]; buf[2 * i + 1] = (uint8_t) (k[i] >> 8); }
    h = fnv1a(buf, (size_t) nk * 2, h);
    for (int i = 0; i < nv; ++i) { buf[2 * i] = (uint8_t) v[i]; buf[2 * i + 1] = (uint8_t) (v[i] >> 8); }
    return fnv1a(buf, (size_t) nv * 2, h);
}

static size_t layer_payload(const sj_kvarn_config * c, const sj_kvarn_layout * lay, uint32_t n, uint32_t B) {
    const size_t H = (size_t) c->n_head_kv;
    const size_t srow = c->sink_type == SJKVARN_SINK_F16 ? (size_t) c->head_dim * 4 : 2 * sj_kvarn_stage_row_bytes(c->staging, c->head_dim);
    const size_t rrow = 2 * sj_kvarn_stage_row_bytes(c->staging, c->head_dim);
    const uint32_t n_sink = n < c->sink ? n : c->sink;
    const uint32_t n_rec = (B - c->sink) / (uint32_t) c->group;
    const uint32_t n_tail = n > B ? n - B : 0;
    return (size_t) n_sink * H * srow + (size_t) n_rec * H * lay->bytes + (size_t) n_tail * H * rrow;
}

extern "C" size_t sj_kvarn_seq_state_size(const sj_kvarn_seq * s) {
    return SJKVARN_STATE_HEADER_BYTES + (size_t) s->n_layers * layer_payload(&s->cfg, &s->layers[0].lay, s->n, s->pol.B) + 8;
}

extern "C" size_t sj_kvarn_state_size_max(const sj_kvarn_config * cfg, int n_layers) {
    sj_kvarn_config c = *cfg;
    sj_kvarn_layout lay;
    c.body = sj_kvarn_body_resolve(cfg->body, cfg->bits_k, cfg->bits_v);
    if (n_layers <= 0 || sj_kvarn_layout_init(&lay, c.head_dim, c.group, c.bits_k, c.bits_v, c.body) != 0) return 0;
    const uint32_t G = (uint32_t) c.group;
    const uint32_t B_all = c.n_ctx > c.sink ? c.sink + G * ((c.n_ctx - c.sink + G - 1u) / G) : c.sink;
    const size_t a = layer_payload(&c, &lay, c.n_ctx, c.sink), b = layer_payload(&c, &lay, c.n_ctx, B_all);
    return SJKVARN_STATE_HEADER_BYTES + (size_t) n_layers * (a > b ? a : b) + 8;
}

// Copy [pos_from, pos_to) ring rows of L between device and host, in position order (slot runs).
static int ring_span(const sj_kvarn_layer * L, uint32_t pos_from, uint32_t pos_to, uint8_t * host, int to_host, sjk_stream st) {
    const size_t row = (size_t) L->cfg.n_head_kv * 2 * L->stage_bytes;
    while (pos_from < pos_to) {
        const uint32_t slot = sj_kvarn_ring_slot(L->cfg.sink, L->cap, pos_from);
        uint32_t run = L->cap - slot;
        if (run > pos_to - pos_from) run = pos_to - pos_from;
        uint8_t * dev = L->ring + (size_t) slot * row;
        const int rc = to_host ? ck(cudaMemcpyAsync(host, dev, run * row, cudaMemcpyDeviceToHost, st))
                               : ck(cudaMemcpyAsync(dev, host, run * row, cudaMemcpyHostToDevice, st));
        if (rc) return rc;
        host += run * row;
        pos_from += run;
    }
    return 0;
}

// Copy records of groups [0, n_rec) between device and host. A contiguous body moves in one copy; a pool's
// scattered blocks are gathered into (or scattered from) a stream-ordered device staging buffer by one kernel, so
// the host sees one copy per layer instead of one per run of consecutive blocks.
static int record_span(const sj_kvarn_layer * L, uint32_t n_rec, uint8_t * host, int to_host, sjk_stream st) {
    const size_t grp = (size_t) L->cfg.n_head_kv * L->lay.bytes;
    if (n_rec == 0) return 0;
    uint32_t runs = 1;
    for (uint32_t g = 1; g < n_rec && L->blocks; ++g) runs += L->blocks[g] != L->blocks[g - 1] + 1u;
    if (L->blocks && L->d_blocks && runs > 1) {
        uint8_t * stage = NULL;
        const size_t bytes = (size_t) n_rec * grp;
        int rc = ck(cudaMallocAsync((void **) &stage, bytes, st));
        if (rc) return rc;
        if (to_host) {
            rc = sjk_group_move(L->body, L->d_blocks, 0, n_rec, grp, stage, 0, st);
            if (!rc) rc = ck(cudaMemcpyAsync(host, stage, bytes, cudaMemcpyDeviceToHost, st));
        } else {
            rc = ck(cudaMemcpyAsync(stage, host, bytes, cudaMemcpyHostToDevice, st));
            if (!rc) rc = sjk_group_move(L->body, L->d_blocks, 0, n_rec, grp, stage, 1, st);
        }
        const int rf = ck(cudaFreeAsync(stage, st));
        return rc ? rc : rf;
    }
    uint32_t g = 0;
    while (g < n_rec) {
        const uint32_t b0 = L->blocks ? L->blocks[g] : g;
        uint32_t run = 1;
        while (g + run < n_rec && (L->blocks ? L->blocks[g + run] : g + run) == b0 + run) ++run;
        uint8_t * dev = L->body + (size_t) b0 * grp;
        const int rc = to_host ? ck(cudaMemcpyAsync(host, dev, run * grp, cudaMemcpyDeviceToHost, st))
                               : ck(cudaMemcpyAsync(dev, host, run * grp, cudaMemcpyHostToDevice, st));
        if (rc) return rc;
        host += run * grp;
        g += run;
    }
    return 0;
}

extern "C" int sj_kvarn_seq_state_write(const sj_kvarn_seq * s, void * dst, size_t dst_size, size_t * written) {
    if (written) *written = 0;
    if (!s->layers || (!dst && dst_size)) return SJKVARN_ERR_ARG;
    if (s->pol.B_pending != s->pol.B) return SJKVARN_ERR_PENDING;
    const size_t total = sj_kvarn_seq_state_size(s);
    if (dst_size < total) return SJKVARN_ERR_BUFFER;
    const sj_kvarn_config * c = &s->cfg;
    const uint32_t S = c->sink, G = (uint32_t) c->group, B = s->pol.B, n = s->n;
    const int H = c->n_head_kv;
    uint8_t * o = (uint8_t *) dst;
    memset(o, 0, SJKVARN_STATE_HEADER_BYTES);
    memcpy(o, k_magic, 8);
    wr32(o + 8, SJKVARN_STATE_VERSION); wr32(o + 12, SJKVARN_FORMAT_VERSION); wr32(o + 16, SJKVARN_STATE_HEADER_BYTES);
    wr32(o + 20, (uint32_t) c->head_dim); wr32(o + 24, (uint32_t) c->n_head_kv); wr32(o + 28, (uint32_t) c->group);
    wr32(o + 32, c->sink); wr32(o + 36, (uint32_t) c->sink_type); wr32(o + 40, (uint32_t) c->bits_k);
    wr32(o + 44, (uint32_t) c->bits_v); wr32(o + 48, (uint32_t) c->body); wr32(o + 52, (uint32_t) c->iters);
    wr32(o + 56, (uint32_t) c->staging); wr32(o + 60, c->tail); wr32(o + 64, c->tail_max); wr32(o + 68, c->flush_chunk);
    wr32(o + 72, SJKVARN_ROTATION_HADAMARD); wr32(o + 76, (uint32_t) c->head_dim);
    wr64(o + 80, codebook_id(c->body, c->bits_k, c->bits_v));
    wr32(o + 88, (uint32_t) s->n_layers); wr32(o + 92, n); wr32(o + 96, B); wr32(o + 100, s->pol.B_prev);
    wr32(o + 104, (uint32_t) s->pol.draining); wr64(o + 108, (uint64_t) (total - SJKVARN_STATE_HEADER_BYTES - 8));
    uint8_t * w = o + SJKVARN_STATE_HEADER_BYTES;
    const uint32_t n_sink = n < S ? n : S, n_rec = (B - S) / G;
    int rc = 0;
    for (int il = 0; il < s->n_layers && !rc; ++il) {
        const sj_kvarn_layer * L = &s->layers[il];
        const size_t sb = (size_t) n_sink * H * sink_entry_bytes(L);
        if (sb) rc = ck(cudaMemcpyAsync(w, L->sink, sb, cudaMemcpyDeviceToHost, s->stream));
        w += sb;
        if (!rc) rc = record_span(L, n_rec, w, 1, s->stream);
        w += (size_t) n_rec * H * L->lay.bytes;
        if (!rc) rc = ring_span(L, B, n > B ? n : B, w, 1, s->stream);
        w += (size_t) (n > B ? n - B : 0) * H * 2 * L->stage_bytes;
    }
    if (!rc) rc = ck(cudaStreamSynchronize(s->stream));
    if (rc) return rc;
    wr64(w, fnv1a(o, (size_t) (w - o), k_fnv0));
    if (written) *written = total;
    return SJKVARN_OK;
}

extern "C" int sj_kvarn_state_peek(const void * src, size_t size, sj_kvarn_state_info * info) {
    const uint8_t * p = (const uint8_t *) src;
    if (!src || !info) return SJKVARN_ERR_ARG;
    sj_kvarn_state_info t;
    memset(&t, 0, sizeof t);
    if (size < 8) return SJKVARN_ERR_TRUNCATED;
    if (memcmp(p, k_magic, 8) != 0) return SJKVARN_ERR_MAGIC;
    if (size < 16) return SJKVARN_ERR_TRUNCATED;
    t.state_version = rd32(p + 8);
    t.format_version = rd32(p + 12);
    if (t.state_version != SJKVARN_STATE_VERSION) return SJKVARN_ERR_VERSION;
    if (size < SJKVARN_STATE_HEADER_BYTES + 8) return SJKVARN_ERR_TRUNCATED;
    if (rd32(p + 16) != SJKVARN_STATE_HEADER_BYTES) return SJKVARN_ERR_CORRUPT;
    const uint64_t payload = rd64(p + 108);
    if (payload > (uint64_t) (size - SJKVARN_STATE_HEADER_BYTES - 8)) return SJKVARN_ERR_TRUNCATED;
    t.total_bytes = SJKVARN_STATE_HEADER_BYTES + (size_t) payload + 8;
    if (fnv1a(p, t.total_bytes - 8, k_fnv0) != rd64(p + t.total_bytes - 8)) return SJKVARN_ERR_CORRUPT;
    if (t.format_version != SJKVARN_FORMAT_VERSION) return SJKVARN_ERR_FORMAT;
    t.cfg.head_dim = (int) rd32(p + 20); t.cfg.n_head_kv = (int) rd32(p + 24); t.cfg.group = (int) rd32(p + 28);
    t.cfg.sink = rd32(p + 32); t.cfg.sink_type = (int) rd32(p + 36); t.cfg.bits_k = (int) rd32(p + 40);
    t.cfg.bits_v = (int) rd32(p + 44); t.cfg.body = (int) rd32(p + 48); t.cfg.iters = (int) rd32(p + 52);
    t.cfg.staging = (int) rd32(p + 56); t.cfg.tail = rd32(p + 60); t.cfg.tail_max = rd32(p + 64);
    t.cfg.flush_chunk = rd32(p + 68);
    t.rotation = rd32(p + 72); t.rotation_n = rd32(p + 76); t.codebook_id = rd64(p + 80);
    t.n_layers = (int) rd32(p + 88); t.n = rd32(p + 92); t.B = rd32(p + 96); t.B_prev = rd32(p + 100);
    t.draining = rd32(p + 104);
    *info = t;
    return SJKVARN_OK;
}

extern "C" int sj_kvarn_seq_state_read(sj_kvarn_seq * s, const void * src, size_t size) {
    if (!s->layers) return SJKVARN_ERR_ARG;
    sj_kvarn_state_info t;
    int rc = sj_kvarn_state_peek(src, size, &t);
    if (rc != SJKVARN_OK) return rc;
    const sj_kvarn_config * c = &s->cfg;
    // everything that changes stored bytes or the policy must match
    if (t.cfg.head_dim != c->head_dim) return SJKVARN_ERR_HEAD_DIM;
    if (t.cfg.n_head_kv != c->n_head_kv) return SJKVARN_ERR_N_HEAD_KV;
    if (t.cfg.group != c->group) return SJKVARN_ERR_GROUP;
    if (t.cfg.sink != c->sink || t.cfg.sink_type != c->sink_type) return SJKVARN_ERR_SINK;
    if (t.cfg.bits_k != c->bits_k || t.cfg.bits_v != c->bits_v) return SJKVARN_ERR_BITS;
    if (t.cfg.body != c->body) return SJKVARN_ERR_BODY;
    if (t.cfg.iters != c->iters) return SJKVARN_ERR_ITERS;
    if (t.cfg.staging != c->staging) return SJKVARN_ERR_STAGING;
    if (t.cfg.tail != c->tail || t.cfg.tail_max != c->tail_max || t.cfg.flush_chunk != c->flush_chunk) return SJKVARN_ERR_TAIL;
    if (t.rotation != SJKVARN_ROTATION_HADAMARD || t.rotation_n != (uint32_t) c->head_dim) return SJKVARN_ERR_ROTATION;
    if (t.codebook_id != codebook_id(c->body, c->bits_k, c->bits_v)) return SJKVARN_ERR_CODEBOOK;
    if (t.n_layers != s->n_layers) return SJKVARN_ERR_N_LAYERS;
    const uint32_t S = c->sink, G = (uint32_t) c->group;
    if (t.B < S || (t.B - S) % G != 0 || t.B_prev < S || t.B_prev > t.B || (t.B_prev - S) % G != 0 || t.draining > 1 ||
        (t.B > S && t.B > t.n))
        return SJKVARN_ERR_CORRUPT;
    if (t.total_bytes != SJKVARN_STATE_HEADER_BYTES + (size_t) s->n_layers * layer_payload(c, &s->layers[0].lay, t.n, t.B) + 8)
        return SJKVARN_ERR_CORRUPT;
    const uint32_t n_rec = (t.B - S) / G;
    if (t.n > c->n_ctx || n_rec > s->layers[0].n_groups || (t.n > t.B && t.n - t.B > s->layers[0].cap)) return SJKVARN_ERR_CAPACITY;
    if (s->pool) {
        uint32_t held = 0;
        for (uint32_t g = 0; g < s->layers[0].n_groups; ++g) held += s->blocks[g] != SJKVARN_NO_BLOCK;
        if (s->pool->n_free + held < n_rec) return SJKVARN_ERR_POOL_FULL;
    }
    // accepted: replace the sequence
    sj_kvarn_seq_reset(s);
    if (seq_reserve(s, 0, n_rec) != SJKVARN_OK) return SJKVARN_ERR_POOL_FULL;
    const uint8_t * r = (const uint8_t *) src + SJKVARN_STATE_HEADER_BYTES;
    const uint32_t n_sink = t.n < S ? t.n : S;
    const int H = c->n_head_kv;
    rc = 0;
    for (int il = 0; il < s->n_layers && !rc; ++il) {
        sj_kvarn_layer * L = &s->layers[il];
        const size_t sb = (size_t) n_sink * H * sink_entry_bytes(L);
        if (sb) rc = ck(cudaMemcpyAsync(L->sink, r, sb, cudaMemcpyHostToDevice, s->stream));
        r += sb;
        if (!rc) rc = record_span(L, n_rec, (uint8_t *) r, 0, s->stream);
        r += (size_t) n_rec * H * L->lay.bytes;
        if (!rc) rc = ring_span(L, t.B, t.n > t.B ? t.n : t.B, (uint8_t *) r, 0, s->stream);
        r += (size_t) (t.n > t.B ? t.n - t.B : 0) * H * 2 * L->stage_bytes;
    }
    if (!rc) rc = ck(cudaStreamSynchronize(s->stream));
    if (rc) return rc;
    s->pol.B = s->pol.B_pending = t.B;
    s->pol.B_prev = t.B_prev;
    s->pol.draining = (int) t.draining;
    s->n = t.n;
    return SJKVARN_OK;
}
