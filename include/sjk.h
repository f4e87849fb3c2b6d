/*
 * sjk.h - B200 (sm_100a) implementation of the SJ-KVaRN hot path behind the sj_kvarn.h C API.
 *
 * Link libsjk_b200.so and include this header instead of the reference's single-header
 * library (JakeATX/sj-kvarn-codec, sj_kvarn.h). Names, argument meaning, status codes and
 * stored bytes are those of sj_kvarn.h; the difference is where the data lives:
 *
 *   - every cache buffer (sink, staging ring, sealed body, pool slab) is DEVICE memory;
 *   - row arguments of the codec and cache calls (k_rot, v_rot, q_rot, out_rot, records,
 *     staging rows, seal inputs) are DEVICE pointers;
 *   - state save/restore streams (sj_kvarn_seq_state_write/_read/_peek) are HOST buffers;
 *   - the policy, layout, pool bookkeeping and status calls are host code, unchanged.
 *
 * Cache calls run on the object's stream (sj_kvarn_layer.stream / sj_kvarn_seq.stream,
 * 0 = the legacy default stream) and are asynchronous like any CUDA launch; calls that
 * return data to the host (state write, sj_kvarn_layer_record_copy) synchronise it.
 * Functions that return void in sj_kvarn.h record a sticky error instead (sjk_last_error).
 *
 * A second, thinner layer (sjk_*) exposes the device kernels with explicit streams and
 * batched shapes; it mirrors the reference's CUDA entry points (sj_kvarn_cuda.cuh) and is
 * what an engine's own graph calls.
 */
#ifndef SJK_H
#define SJK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st * sjk_stream;   /* same type as cudaStream_t */

/* ---- versions and format constants (sj_kvarn.h:85-128) ---- */
#define SJKVARN_VERSION_MAJOR 2
#define SJKVARN_VERSION_MINOR 0
#define SJKVARN_FORMAT_VERSION 1
#define SJKVARN_STATE_VERSION  1

#define SJKVARN_GROUP_DEFAULT     128
#define SJKVARN_SINK_DEFAULT      128
#define SJKVARN_TAIL_DEFAULT      4096
#define SJKVARN_TAIL_MAX_DEFAULT  8192
#define SJKVARN_ITERS_DEFAULT     16
#define SJKVARN_RED_LANES         8
#define SJKVARN_TQ6_QK            128
#define SJKVARN_TQ6_BLOCK_BYTES   98
#define SJKVARN_TRELLIS_SEQ       128
#define SJKVARN_TRELLIS_HIST_BITS 6
#define SJKVARN_TRELLIS_NSTATE    64

typedef enum sj_kvarn_body {
    SJKVARN_BODY_SCALAR  = 0,
    SJKVARN_BODY_TRELLIS = 1,
    SJKVARN_BODY_AUTO    = 2
} sj_kvarn_body;

typedef enum sj_kvarn_staging {
    SJKVARN_STAGING_TQ6_0 = 0,
    SJKVARN_STAGING_F16   = 1
} sj_kvarn_staging;

typedef enum sj_kvarn_sink_type {
    SJKVARN_SINK_F16     = 0,
    SJKVARN_SINK_INHERIT = 1
} sj_kvarn_sink_type;

/* staging block, 98 bytes (sj_kvarn.h:146-154) */
typedef struct sj_kvarn_tq6_block {
    uint16_t norm;
    uint8_t  qs[64];
    uint8_t  qh[32];
} sj_kvarn_tq6_block;

/* record layout (sj_kvarn.h:156-175) */
typedef struct sj_kvarn_layout {
    int D, G, bits_k, bits_v, body;
    uint32_t k_payload, v_payload;
    uint32_t k_scale, k_zero, k_tok, v_ch, v_scale, v_zero;
    uint32_t bytes;
} sj_kvarn_layout;

/* ---- fp16 (host; sj_kvarn.h:178-179) ---- */
uint16_t sj_kvarn_f32_to_f16(float f);
float    sj_kvarn_f16_to_f32(uint16_t h);

/* ---- rotation (sj_kvarn.h:182-185). x: DEVICE [n] / [n_heads][head_dim] floats, in place. ---- */
void sj_kvarn_hadamard(float * x, int n);
void sj_kvarn_rotate_heads(float * x, int n_heads, int head_dim);

/* ---- record layout (host; sj_kvarn.h:187-195) ---- */
int      sj_kvarn_body_resolve(int body, int bits_k, int bits_v);
int      sj_kvarn_layout_init(sj_kvarn_layout * l, int D, int G, int bits_k, int bits_v, int body);
size_t   sj_kvarn_record_bytes(int D, int G, int bits_k, int bits_v);
double   sj_kvarn_body_bits_per_element(const sj_kvarn_layout * l);
uint32_t sj_kvarn_code_bit(const sj_kvarn_layout * l, int t, int d, int is_v);
int      sj_kvarn_k_ch_idx(const sj_kvarn_layout * l, int d);
int      sj_kvarn_v_ch_idx(const sj_kvarn_layout * l, int d);

/* ---- seal / decode / staging of single objects (sj_kvarn.h:197-216); DEVICE pointers ---- */
/* The B200 sealer keeps its scratch on chip; `work` is accepted and ignored (may be NULL). */
size_t sj_kvarn_seal_workspace_bytes(const sj_kvarn_layout * l);
void   sj_kvarn_seal_group(const sj_kvarn_layout * l, const uint16_t * K, const uint16_t * V,
                           size_t row_stride, int iters, uint8_t * rec, void * work);
void   sj_kvarn_decode_k_row(const sj_kvarn_layout * l, const uint8_t * rec, int t, float * out);
void   sj_kvarn_decode_v_row(const sj_kvarn_layout * l, const uint8_t * rec, int t, float * out);
void   sj_kvarn_tq6_quantize_row(const float * x, sj_kvarn_tq6_block * y, int n);
void   sj_kvarn_tq6_dequantize_row(const sj_kvarn_tq6_block * y, float * x, int n);
size_t sj_kvarn_stage_row_bytes(int staging, int D);
void   sj_kvarn_stage_row(int staging, const float * x_rot, void * dst, int D);
void   sj_kvarn_unstage_row(int staging, const void * src, float * x_rot, int D);

/* ---- reference attention helpers (rotated basis; sj_kvarn.h:218-222, 1288-1311); DEVICE pointers ---- */
/* scores[t] = dot(q, K[t]) for the first n tokens of a record: each a sequential fp32 sum over the channels */
void   sj_kvarn_record_scores(const sj_kvarn_layout * l, const uint8_t * rec, const float * q, int n, float * scores);
/* acc[d] += sum_t w[t] * V[t, d] for the first n tokens of a record, added in token order */
void   sj_kvarn_record_accum_v(const sj_kvarn_layout * l, const uint8_t * rec, const float * w, int n, float * acc);

/* ---- adaptive tail / journal policy (host; sj_kvarn.h:224-274) ---- */
typedef struct sj_kvarn_policy {
    uint32_t sink, tail, tail_max, group, flush_chunk;
    uint32_t B;
    uint32_t B_prev;
    uint32_t B_pending;
    int      draining;
} sj_kvarn_policy;

void     sj_kvarn_policy_init(sj_kvarn_policy * p, uint32_t sink, uint32_t tail, uint32_t tail_max,
                              uint32_t group, uint32_t flush_chunk);
void     sj_kvarn_policy_reset(sj_kvarn_policy * p);
uint32_t sj_kvarn_policy_begin_ubatch(sj_kvarn_policy * p, uint32_t pos0, uint32_t n_tokens);
void     sj_kvarn_policy_commit(sj_kvarn_policy * p);
uint32_t sj_kvarn_policy_idle(sj_kvarn_policy * p, uint32_t end, uint32_t keep_recent);

#define SJKVARN_NO_POS UINT32_MAX
uint32_t sj_kvarn_group_floor(uint32_t sink, uint32_t group, uint32_t pos);
uint32_t sj_kvarn_policy_trunc_floor(const sj_kvarn_policy * p, uint32_t pos);
uint32_t sj_kvarn_policy_truncate(sj_kvarn_policy * p, uint32_t pos, uint32_t * n_dropped);
uint32_t sj_kvarn_ring_capacity(uint32_t tail, uint32_t tail_max, uint32_t group, uint32_t n_ubatch);
uint32_t sj_kvarn_ring_slot(uint32_t sink, uint32_t cap, uint32_t pos);

/* ---- per-layer cache (sj_kvarn.h:276-330); buffers in DEVICE memory ---- */
typedef struct sj_kvarn_config {
    int      head_dim;
    int      n_head_kv;
    int      group;
    int      bits_k, bits_v;
    int      body;
    int      iters;
    int      staging;
    int      sink_type;
    uint32_t sink, tail, tail_max, flush_chunk;
    uint32_t n_ubatch;
    uint32_t n_ctx;
} sj_kvarn_config;

typedef struct sj_kvarn_layer {
    sj_kvarn_config cfg;
    sj_kvarn_layout lay;
    uint32_t cap;
    uint32_t n_groups;
    size_t   stage_bytes;
    uint8_t * ring;            /* device [cap][n_head_kv][K row | V row] */
    uint8_t * sink;            /* device, f16: [sink][n_head_kv][K D | V D]; inherit: staging rows */
    uint8_t * body;            /* device [n_groups][n_head_kv][record] or a pool slab */
    const uint32_t * blocks;   /* host block table (pool mode), NULL = contiguous body */
    const uint32_t * d_blocks; /* device copy of the block table (pool mode) */
    int       owns_body;
    void    * work;            /* device attention scratch (split partials) */
    size_t    work_bytes;
    sjk_stream stream;         /* stream of the layer's calls (0 = legacy default stream) */
} sj_kvarn_layer;

sj_kvarn_config sj_kvarn_config_default(int head_dim, int n_head_kv, uint32_t n_ctx, uint32_t n_ubatch);
int      sj_kvarn_layer_init(sj_kvarn_layer * L, const sj_kvarn_config * cfg);
void     sj_kvarn_layer_free(sj_kvarn_layer * L);
/* k_rot / v_rot: DEVICE [n_head_kv][D] rotated floats of position pos */
void     sj_kvarn_layer_store(sj_kvarn_layer * L, uint32_t pos, const float * k_rot, const float * v_rot);
void     sj_kvarn_layer_seal(sj_kvarn_layer * L, uint32_t B_from, uint32_t B_to);
/* k, v: DEVICE [D] outputs */
void     sj_kvarn_layer_kv_row(const sj_kvarn_layer * L, uint32_t B, uint32_t pos, int h, float * k, float * v);
/* q_rot, out_rot: DEVICE [D] */
void     sj_kvarn_layer_attend_row(const sj_kvarn_layer * L, uint32_t B, uint32_t N, const float * q_rot,
                                   int h, uint32_t qpos, float scale, float * out_rot);
/* DEVICE address of record (g, h) */
uint8_t * sj_kvarn_layer_record(const sj_kvarn_layer * L, uint32_t g, int h);
void     sj_kvarn_layer_truncate(sj_kvarn_layer * L, uint32_t B_old, uint32_t B_new, uint32_t n_old, uint32_t resume);

/* ---- status codes (sj_kvarn.h:332-361) ---- */
enum {
    SJKVARN_OK                = 0,
    SJKVARN_ERR_ARG           = -100,
    SJKVARN_ERR_NOMEM         = -101,
    SJKVARN_ERR_BUFFER        = -102,
    SJKVARN_ERR_TRUNCATED     = -103,
    SJKVARN_ERR_MAGIC         = -104,
    SJKVARN_ERR_VERSION       = -105,
    SJKVARN_ERR_FORMAT        = -106,
    SJKVARN_ERR_CORRUPT       = -107,
    SJKVARN_ERR_PENDING       = -108,
    SJKVARN_ERR_CAPACITY      = -109,
    SJKVARN_ERR_POOL_FULL     = -110,
    SJKVARN_ERR_HEAD_DIM      = -120,
    SJKVARN_ERR_N_HEAD_KV     = -121,
    SJKVARN_ERR_GROUP         = -122,
    SJKVARN_ERR_SINK          = -123,
    SJKVARN_ERR_BITS          = -124,
    SJKVARN_ERR_BODY          = -125,
    SJKVARN_ERR_ITERS         = -126,
    SJKVARN_ERR_STAGING       = -127,
    SJKVARN_ERR_TAIL          = -128,
    SJKVARN_ERR_ROTATION      = -129,
    SJKVARN_ERR_CODEBOOK      = -130,
    SJKVARN_ERR_N_LAYERS      = -131,
    /* B200 build only: a CUDA call failed (the CUDA error is in sjk_last_cuda_error()) */
    SJK_ERR_DEVICE            = -200,
    /* B200 build only: a shape the device kernels do not implement (e.g. head_dim > 256) */
    SJK_ERR_UNSUPPORTED       = -201,
    /* B200 build only: the shape needs more scratch than sjk_attend_static's fixed buffer holds */
    SJK_ERR_SCRATCH_LIMIT     = -202
};
const char * sj_kvarn_strerror(int code);

/* ---- paged record pool (sj_kvarn.h:363-381); slab in DEVICE memory ---- */
#define SJKVARN_NO_BLOCK UINT32_MAX
typedef struct sj_kvarn_pool {
    sj_kvarn_config cfg;
    sj_kvarn_layout lay;
    int       n_layers;
    uint32_t  n_blocks;
    uint8_t * body;            /* device [n_layers][n_blocks][n_head_kv][lay.bytes] */
    uint32_t * free_ids;       /* host stack of free block ids */
    uint32_t  n_free;
} sj_kvarn_pool;

int      sj_kvarn_pool_init(sj_kvarn_pool * pool, const sj_kvarn_config * cfg, int n_layers, uint32_t n_blocks);
void     sj_kvarn_pool_free(sj_kvarn_pool * pool);
uint32_t sj_kvarn_pool_alloc(sj_kvarn_pool * pool);
void     sj_kvarn_pool_release(sj_kvarn_pool * pool, uint32_t id);

/* ---- sequence (sj_kvarn.h:383-415) ---- */
typedef struct sj_kvarn_seq {
    sj_kvarn_config  cfg;
    int              n_layers;
    sj_kvarn_layer * layers;
    sj_kvarn_policy  pol;
    uint32_t         n;
    sj_kvarn_pool  * pool;
    uint32_t       * blocks;   /* host block table (pool mode) */
    uint32_t       * d_blocks; /* device mirror of blocks */
    sjk_stream       stream;
} sj_kvarn_seq;

int      sj_kvarn_seq_init(sj_kvarn_seq * s, const sj_kvarn_config * cfg, int n_layers, sj_kvarn_pool * pool);
void     sj_kvarn_seq_free(sj_kvarn_seq * s);
void     sj_kvarn_seq_reset(sj_kvarn_seq * s);
int      sj_kvarn_seq_begin_ubatch(sj_kvarn_seq * s, uint32_t pos0, uint32_t n_tokens);
/* k_rot / v_rot: DEVICE [n_layers][n_head_kv][D] rotated floats */
void     sj_kvarn_seq_store(sj_kvarn_seq * s, uint32_t pos, const float * k_rot, const float * v_rot);
int      sj_kvarn_seq_idle(sj_kvarn_seq * s, uint32_t keep_recent);
uint32_t sj_kvarn_seq_truncate(sj_kvarn_seq * s, uint32_t pos);
void     sj_kvarn_seq_attend_row(const sj_kvarn_seq * s, int il, const float * q_rot, int h, uint32_t qpos,
                                 float scale, float * out_rot);

/* ---- sequence state (sj_kvarn.h:417-453); streams are HOST buffers ---- */
#define SJKVARN_STATE_HEADER_BYTES 128
#define SJKVARN_ROTATION_HADAMARD  1

typedef struct sj_kvarn_state_info {
    uint32_t state_version, format_version;
    sj_kvarn_config cfg;
    uint32_t rotation, rotation_n;
    uint64_t codebook_id;
    int      n_layers;
    uint32_t n, B, B_prev, draining;
    size_t   total_bytes;
} sj_kvarn_state_info;

size_t sj_kvarn_seq_state_size(const sj_kvarn_seq * s);
size_t sj_kvarn_state_size_max(const sj_kvarn_config * cfg, int n_layers);
int    sj_kvarn_seq_state_write(const sj_kvarn_seq * s, void * dst, size_t dst_size, size_t * written);
int    sj_kvarn_state_peek(const void * src, size_t size, sj_kvarn_state_info * info);
int    sj_kvarn_seq_state_read(sj_kvarn_seq * s, const void * src, size_t size);

/* =====================================================================================
 * Device layer (sjk_*): explicit streams, batched shapes, DEVICE pointers. Every call
 * returns 0 or a negative status (SJK_ERR_DEVICE with the CUDA error in
 * sjk_last_cuda_error(), SJKVARN_ERR_ARG, SJK_ERR_UNSUPPORTED).
 * ===================================================================================== */

/* Device view of one layer's cache (sj_kvarn_cuda.cuh:27-42), plus an optional device
 * block table: record (g, h) is at body + ((blocks ? blocks[g] : g)*n_head_kv + h)*lay.bytes. */
typedef struct sjk_view {
    sj_kvarn_layout lay;
    int      n_head_kv;
    int      staging;
    int      sink_type;
    uint32_t S, cap;
    size_t   stage_bytes;
    const uint8_t * sink;
    const uint8_t * ring;
    const uint8_t * body;
    const uint32_t * blocks;
} sjk_view;

int          sjk_last_error(void);          /* sticky status of the void-returning calls; clears it */
/* Device status word of the kernels (synchronizes the device): 0 = fine, bit 1 (SJK_DEVICE_TIMEOUT) = a bounded
 * in-kernel wait ran out (the kernel skipped its remaining work and released its resources), bit 2
 * (SJK_DEVICE_DESC) = a descriptor-driven call met a descriptor that does not fit its cache. Reading clears it. */
int          sjk_device_status(void);
int          sjk_last_cuda_error(void);     /* cudaError_t of the last failed CUDA call */
const char * sjk_version(void);

/* In-place orthonormal FWHT of n_rows rows of n floats (n a power of two, 32..1024). */
int sjk_hadamard(float * x, int n_rows, int n, sjk_stream st);

/* Stage n_rows rotated rows of D floats (sj_kvarn_cuda.cuh:68-74). */
int sjk_stage_rows(int staging, const float * x_rot, uint8_t * dst, size_t dst_row_bytes, int D, int n_rows, sjk_stream st);
/* Widen n_rows staged rows back to floats (sj_kvarn_cuda.cuh:76-80). */
int sjk_unstage_rows(int staging, const uint8_t * src, size_t src_row_bytes, float * x, int D, int n_rows, sjk_stream st);

/* Store n_pos consecutive positions pos0.. of one layer: k, v are [n_pos][n_head_kv][D]
 * floats, rotated (rotate = 0) or in the model basis (rotate = 1: the per-head Hadamard
 * runs inside the kernel). Positions below the sink go to the sink (fp16 or staging rows),
 * the rest to ring slot (pos - S) % cap as tq6_0 / fp16 rows (sj_kvarn.h:1475-1492). */
int sjk_store(const sjk_view * v, uint8_t * sink, uint8_t * ring, uint32_t pos0, uint32_t n_pos,
              const float * k, const float * vv, int rotate, sjk_stream st);

/* One position in each of n_items layer caches in one launch - the decode step's cache write across the layers and
 * sequences of a batch (sj_kvarn.h:1475-1492 per item): item i stores the rows k + i*n_head_kv*D, vv + i*n_head_kv*D
 * (rotated, or model basis with rotate = 1) at position pos[i] (host array) of views[i]'s sink or staging ring. All
 * views share the layout, formats, sink length and ring capacity. No counterpart in the reference. */
int sjk_store_batch(const sjk_view * views, const uint32_t * pos, int n_items, const float * k, const float * vv,
                    int rotate, sjk_stream st);

/* Seal n_groups x n_head_kv records from fp16 rows (sj_kvarn_cuda.cuh:136-152): record
 * r = g*n_head_kv + h reads rows k + g*G*row_stride + h*D. work is ignored (may be NULL). */
int sjk_seal(const sj_kvarn_layout * lay, const uint16_t * k, const uint16_t * v, size_t row_stride,
             int n_head_kv, int n_groups, int iters, uint8_t * body, void * work, sjk_stream st);

/* Seal positions [B_from, B_to) of a layer straight out of its staging ring: each row is
 * widened, rounded to fp16 and sealed in one kernel (sj_kvarn.h:1494-1514). Record
 * addresses follow v->blocks. iters: balancing iterations. */
int sjk_seal_ring(const sjk_view * v, uint8_t * body, uint32_t B_from, uint32_t B_to, int iters, sjk_stream st);

/* Decode n_rec records to [n_rec][G][D] floats (sj_kvarn_cuda.cuh:57-66). */
int sjk_decode(const sj_kvarn_layout * lay, const uint8_t * body, int n_rec, float * out_k, float * out_v, sjk_stream st);

/* Causal attention of n_q query rows (positions qpos0..) x n_head query heads over [0, N)
 * of one layer (sj_kvarn_cuda.cuh:103-134; GQA head hq reads KV head hq/(n_head/n_head_kv)).
 * q, out: [n_q][n_head][D] rotated floats. scratch: sjk_attend_scratch_bytes() bytes. */
size_t sjk_attend_scratch_bytes(const sjk_view * v, uint32_t N, int n_q, int n_head);
int sjk_attend(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, const float * q,
               float scale, float * out, void * scratch, size_t scratch_bytes, sjk_stream st);

/* Attention split by context (a single long sequence sliced across GPUs, sj_kvarn.h:1535-1564 computed piecewise):
 * sjk_attend_partial attends over the regions selected by `regions` and returns one partial per
 * (query row, query head): part_out[n_q * n_head][D + 2] = (m, l, o[D]), with m the running max of the scaled
 * scores (natural log), l the sum of exp(score - m) and o the V rows weighted by exp(score - m), not normalized.
 * sjk_attend_merge combines n_parts such partial sets, parts[n_parts][n_rows][D + 2], in index order into
 * out[n_rows][D]; partials of disjoint position sets combine to the attention over their union. No
 * counterpart in the reference, whose attention runs over one cache on one device. */
enum { SJK_REGION_SINK = 1, SJK_REGION_BODY = 2, SJK_REGION_RING = 4, SJK_REGION_ALL = 7 };
int sjk_attend_partial(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, unsigned regions,
                       const float * q, float scale, float * part_out, void * scratch, size_t scratch_bytes, sjk_stream st);
int sjk_attend_merge(const float * parts, int n_parts, int n_rows, int D, float * out, sjk_stream st);

/* Attention of a batch of sequences of one layer in one call: the decode step of a paged record pool, where
 * sequence s (views[s]: its sink, staging ring, pool slab and device block table; every view has the same layout,
 * formats, sink length and ring capacity) attends with query rows q + s*n_q*n_head*D at positions qpos0[s].. over
 * [0, N[s]) with [S, B[s]) sealed, and writes out + s*n_q*n_head*D. Equivalent to n_seq sjk_attend calls
 * (sj_kvarn.h:1535-1564 per sequence and head; the pool resolution of sj_kvarn.h:1429-1432, 1706-1739); trellis
 * layers take three launches for the whole batch. B, N, qpos0 are host arrays; scratch: at least
 * sjk_attend_batch_scratch_bytes() bytes. No counterpart in the reference, whose attention is per sequence. */
size_t sjk_attend_batch_scratch_bytes(const sjk_view * v, int n_seq, int n_q, int n_head);
int sjk_attend_batch(const sjk_view * views, const uint32_t * B, const uint32_t * N, const uint32_t * qpos0, int n_seq,
                     int n_q, int n_head, const float * q, float scale, float * out, void * scratch, size_t scratch_bytes,
                     sjk_stream st);

/* sjk_attend / sjk_layer_attend with the rotation folded in: q ([n_q][n_head][D], DEVICE) in the model basis and out
 * in the model basis, where sjk_attend takes and returns rotated rows (the reference's attend_row contract, whose
 * caller rotates: README.md:44-54). The 4-bit body kernel rotates its queries on chip and the merge kernel rotates
 * the outputs (the D / 64 tile CTAs of a row as one cluster); calls that read q in other kernels rotate it once into
 * the scratch first. Outputs equal sjk_hadamard(q) -> sjk_attend -> sjk_hadamard(out) bit for bit. D = 128, 256 or
 * 512; scratch: sjk_attend_scratch_bytes() bytes. */
int sjk_attend_model(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, const float * q,
                     float scale, float * out, void * scratch, size_t scratch_bytes, sjk_stream st);
int sjk_layer_attend_model(const sj_kvarn_layer * L, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head,
                           const float * q, float scale, float * out, sjk_stream st);

/* sjk_attend for callers that cannot allocate device memory - code that runs where cudaMalloc is off
 * limits, such as inside a stream capture, a custom allocator's own callbacks or an engine whose memory
 * is planned ahead. No counterpart in the reference. The scratch for the split partials is a fixed 16 MiB
 * device array inside the library (held by every GPU that loads it, until exit) instead of a caller
 * buffer; shapes whose split partials need more than 16 MiB return SJK_ERR_SCRATCH_LIMIT.
 * The array's address is looked up on the first call on each device, so make that first call outside any
 * stream capture. All calls share the array: calls that overlap on the GPU race. Allocates nothing. */
int sjk_attend_static(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, const float * q,
                      float scale, float * out, sjk_stream st);

/* ---- descriptor-driven calls: the reference's ggml op boundary (INTEGRATION_LLAMACPP.md:44-74) ----
 * A descriptor is SJK_DESC_N_ENTRIES int32 values in DEVICE memory describing one sequence's cache for one
 * ubatch, in the reference's entry order (ggml_sjkvarn_desc). The calls below read it when their kernels run,
 * not when they are issued: their launch shapes depend only on the cache and on fixed maxima, so a CUDA graph
 * captured once (seal, store and attention of every layer) replays for every decode step with only the
 * descriptor's contents changing (INTEGRATION_LLAMACPP.md:72-74). TYPE_K / TYPE_V hold the cache's
 * SJKVARN_STAGING_* value, BODY_TYPE its SJKVARN_BODY_*, SINK_TYPE its SJKVARN_SINK_*; entries 14 and 15 are
 * reserved (0). Every kernel checks the static entries (S, CAP, G, D, RECBYTES, HKV, the types) against the view
 * it was launched on, B and B_OLD for group boundaries at or past the sink with B_OLD <= B, and that the staged
 * positions [max(B, S), N) fit the ring; a descriptor that fails makes the call write nothing (sjk_attend_dyn: a
 * zero output) and sets bit SJK_DEVICE_DESC in sjk_device_status(). */
enum {
    SJK_DESC_S = 0, SJK_DESC_CAP, SJK_DESC_B, SJK_DESC_N, SJK_DESC_QPOS0, SJK_DESC_G, SJK_DESC_D, SJK_DESC_RECBYTES,
    SJK_DESC_HKV, SJK_DESC_B_OLD, SJK_DESC_TYPE_K, SJK_DESC_TYPE_V, SJK_DESC_BODY_TYPE, SJK_DESC_SINK_TYPE,
    SJK_DESC_N_ENTRIES = 16
};
enum { SJK_DEVICE_TIMEOUT = 1, SJK_DEVICE_DESC = 2 };
/* Fill a host descriptor for view v: seal [B_old, B) this ubatch, positions [0, N) visible, first query row at
 * qpos0. Returns SJKVARN_ERR_ARG for values that the kernels would reject. */
int sjk_desc_fill(const sjk_view * v, uint32_t B_old, uint32_t B, uint32_t N, uint32_t qpos0, int32_t * desc);
/* ggml_sjkvarn_seal_dyn (INTEGRATION_LLAMACPP.md:49): seal the groups covering [B_OLD, B) out of the staging ring
 * into v->body (records at v->blocks), as sjk_seal_ring. The launch covers n_groups_max groups; a descriptor asking
 * for more is rejected. */
int sjk_seal_dyn(const sjk_view * v, const int32_t * desc, uint32_t n_groups_max, int iters, sjk_stream st);
/* ggml_set_rows_stage (INTEGRATION_LLAMACPP.md:48): store n_pos positions QPOS0 .. QPOS0 + n_pos - 1 as sjk_store
 * (k, vv: [n_pos][n_head_kv][D] device floats; rotate as sjk_store). */
int sjk_store_dyn(const sjk_view * v, const int32_t * desc, uint32_t n_pos, const float * k, const float * vv, int rotate,
                  sjk_stream st);
/* The region-aware flash attention (INTEGRATION_LLAMACPP.md:50): sjk_attend with B, N and qpos0 taken from the
 * descriptor. Same kernels and the same work split as sjk_attend for the same values, so the output is identical.
 * scratch: at least sjk_attend_dyn_scratch_bytes() bytes (the launch plans and the split partials); allocates
 * nothing. */
size_t sjk_attend_dyn_scratch_bytes(const sjk_view * v, int n_q, int n_head);
int sjk_attend_dyn(const sjk_view * v, const int32_t * desc, int n_q, int n_head, const float * q, float scale, float * out,
                   void * scratch, size_t scratch_bytes, sjk_stream st);

/* Whole-layer helpers over a device-backed sj_kvarn_layer (its stream is ignored; st used). */
int sjk_layer_store(sj_kvarn_layer * L, uint32_t pos0, uint32_t n_pos, const float * k, const float * v, int rotate,
                    sjk_stream st);
int sjk_layer_seal(sj_kvarn_layer * L, uint32_t B_from, uint32_t B_to, sjk_stream st);
int sjk_layer_attend(const sj_kvarn_layer * L, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head,
                     const float * q, float scale, float * out, sjk_stream st);
void sjk_layer_view(const sj_kvarn_layer * L, sjk_view * v);
/* Prefill form of sj_kvarn_seq_store (sj_kvarn.h:1645-1700): positions pos0 .. pos0 + n_pos - 1 of every layer;
 * layer il's rows are DEVICE [n_pos][n_head_kv][D] floats at k + il*layer_stride, v + il*layer_stride (layer_stride
 * in floats; 0 means n_pos*n_head_kv*D), rotate as sjk_store. Raises the sequence's length to pos0 + n_pos. Call
 * sj_kvarn_seq_begin_ubatch(s, pos0, n_pos) first, as for sj_kvarn_seq_store. */
int sjk_seq_store(sj_kvarn_seq * s, uint32_t pos0, uint32_t n_pos, const float * k, const float * v, size_t layer_stride,
                  int rotate, sjk_stream st);
/* copy record (g, h) to host memory (synchronous) */
int sjk_layer_record_copy(const sj_kvarn_layer * L, uint32_t g, int h, void * host_dst);

/* ---- exchange of attention partials between GPUs over peer memory ----
 * For a sequence split by context slice over `world` GPUs (one process per GPU), every rank attends over its own
 * slice (one (m, l, o[D]) triple per (query row, query head)) and needs the merge of all ranks' triples. These calls
 * replace an all-gather + sjk_attend_merge by NVLink stores into the other ranks' exchange buffers and a local merge,
 * with the same arithmetic in the same rank order, so the output is the same bit for bit. No counterpart in the
 * reference, whose attention runs on one device.
 * Set-up: each rank allocates one exchange buffer of sjk_xchg_bytes(world, n_rows, D) bytes (sjk_xchg_alloc, zeroed),
 * sends its CUDA IPC handle (SJK_XCHG_HANDLE_BYTES) to the other ranks and maps theirs (sjk_xchg_open); the
 * sjk_xchg_peers it passes holds every rank's buffer as this process sees it (buf[rank] = its own). Every call carries
 * an epoch that all ranks count up alike from 1, one per exchange; consecutive epochs use alternate slot sets, so a
 * rank may publish epoch e + 1 while others still merge epoch e. Every 8-byte word of a slot carries the epoch that
 * wrote it, so a reader knows a value is current without a flag or a fence. A rank's wait for the others is bounded (about 1 s):
 * a rank that never publishes makes the others write zeros and raise SJK_DEVICE_TIMEOUT in sjk_device_status().
 * Plain stores and loads only: no TMA, no multicast. Buffers are freed (sjk_xchg_close, sjk_xchg_free) only after
 * every rank's last exchange completed. */
#define SJK_XCHG_MAX_WORLD   16
#define SJK_XCHG_HANDLE_BYTES 64
typedef struct sjk_xchg_peers {
    void * buf[SJK_XCHG_MAX_WORLD];
    int    world, rank;
} sjk_xchg_peers;
size_t sjk_xchg_bytes(int world, int n_rows, int D);
int    sjk_xchg_alloc(size_t bytes, void ** buf, void * ipc_handle);
int    sjk_xchg_free(void * buf);
int    sjk_xchg_open(const void * ipc_handle, void ** peer_buf);
int    sjk_xchg_close(void * peer_buf);
/* This rank's triples part[n_rows][D + 2] (DEVICE, e.g. from sjk_attend_partial) go to every rank; out[n_rows][D]
 * (DEVICE) gets the merge of all ranks' triples in rank order. One launch. */
int    sjk_xchg_exchange(const sjk_xchg_peers * x, const float * part, int n_rows, int D, uint32_t epoch, float * out,
                         sjk_stream st);
/* sjk_attend_partial followed by the exchange, in one call: this rank's triples are formed at the end of the scratch
 * (sjk_attend_scratch_bytes() leaves room for them) and one exchange launch stores them into every rank's buffer,
 * gathers the others' and writes the merged output out[n_q * n_head][D] (the exchange shape: n_rows = n_q * n_head,
 * D = head_dim). */
int    sjk_attend_partial_xchg(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, unsigned regions,
                               const float * q, float scale, void * scratch, size_t scratch_bytes, const sjk_xchg_peers * x,
                               uint32_t epoch, float * out, sjk_stream st);

/* ---- the paged pool's bookkeeping on the device: batched reservation, release and truncation ----
 * Replaces, for many sequences at once, the host loops over sj_kvarn_pool_alloc / sj_kvarn_pool_release that a
 * sequence's commit and truncation run (sj_kvarn.h:1716-1739 reserve / release, 1581-1603 truncate). The device pool is
 * the host pool's free-id stack in device memory (sjk_pool_dev_bytes(n_blocks) bytes): sjk_pool_dev_load copies a
 * host pool's stack in, sjk_pool_dev_store copies it back (both synchronous). Requests are served in order with the
 * host's semantics, so a batch leaves the same block tables and the same stack as the same calls on the host pool.
 * Block tables are DEVICE arrays of uint32 block ids (SJKVARN_NO_BLOCK = none), e.g. sj_kvarn_seq.d_blocks. */
#define SJK_POOL_MAX_REQ  128
#define SJK_TRUNC_MAX_REQ 256
typedef struct sjk_block_req {
    uint32_t * blocks;         /* DEVICE block table of one sequence */
    uint32_t   g0, g1;         /* groups [g0, g1) */
} sjk_block_req;
size_t sjk_pool_dev_bytes(uint32_t n_blocks);
int    sjk_pool_dev_load(void * dev_pool, const sj_kvarn_pool * pool, sjk_stream st);
int    sjk_pool_dev_store(const void * dev_pool, sj_kvarn_pool * pool, sjk_stream st);
/* every NO_BLOCK entry of [g0, g1) takes the id on top of the stack, in group order; a request that needs more
 * blocks than are free takes none: status[i] (DEVICE int per request) = 0 or SJKVARN_ERR_POOL_FULL. One launch. */
int    sjk_pool_reserve_batch(void * dev_pool, const sjk_block_req * reqs, int n, int * status, sjk_stream st);
/* every entry of [g0, g1) that holds a block pushes it (in group order) and becomes SJKVARN_NO_BLOCK. One launch. */
int    sjk_pool_release_batch(void * dev_pool, const sjk_block_req * reqs, int n, sjk_stream st);
/* sj_kvarn_layer_truncate for a batch of (sequence, layer) caches: each request zeroes the records of the dropped
 * groups (through its block table when blocks != NULL, skipping NO_BLOCK), the sink rows of [resume, min(n_old, S))
 * and the resident ring rows of [max(resume, S), n_old), all requests in one launch; requests with release != 0
 * (one per sequence: the layers share its blocks) then return the dropped groups' blocks to the device pool in
 * request order (one more launch). body / sink / ring / blocks are DEVICE pointers (sj_kvarn_layer fields). */
typedef struct sjk_trunc_req {
    uint8_t  * body, * sink, * ring;
    uint32_t * blocks;
    uint32_t   S, cap, n_head_kv, group;
    uint32_t   rec_bytes, sink_entry_bytes, stage_bytes;
    uint32_t   B_old, B_new, n_old, resume;
    int        release;
} sjk_trunc_req;
int    sjk_truncate_batch(const sjk_trunc_req * reqs, int n, void * dev_pool, sjk_stream st);

/* ---- seeded synthetic inputs of the benchmark configurations (DEVICE outputs) ----
 * Input generation for benchmarks and parity tests; no counterpart in the reference. K = X * s with X ~ N(0, 1)
 * (Student-t(4) when heavy) and s ~ LogNormal(0, 1) channel scales with 4 outlier channels x 8 per (layer, head);
 * V ~ N(0, 1); Q ~ N(0, 1) rounded to fp16. SplitMix64 draws and Box-Muller normals computed with correctly rounded
 * double operations only, so a host build of the same arithmetic (csrc/sjk_synth.h) produces identical bits; every
 * value is a function of (seed, layer, position, head, channel), so any position range can be generated alone. */
/* scale: DEVICE [n_layers][H][D] channel scales of layers layer0 .. layer0 + n_layers - 1 */
int sjk_synth_scales(uint64_t seed, int layer0, int n_layers, int H, int D, float * scale, sjk_stream st);
/* k, v: DEVICE [n][H][D] model-basis rows of positions pos0 .. pos0 + n - 1 of one layer; scale: DEVICE [H][D] of that
 * layer (sjk_synth_scales); H * D even, k and v 8-byte aligned */
int sjk_synth_kv(uint64_t seed, int layer, int H, int D, int heavy, const float * scale, uint32_t pos0, uint32_t n,
                 float * k, float * v, sjk_stream st);
/* q: DEVICE [n_rows][D] query rows of one layer (row = query row * n_head + query head), fp16-rounded floats */
int sjk_synth_q(uint64_t seed, int layer, uint32_t n_rows, int D, float * q, sjk_stream st);

/* Self-check of the seal's math library: lg[i] = log(x[i]) and ex[i] = exp(x[i]) with the device's double log and
 * exp, the two calls the balancing makes per scale update (sj_kvarn.h:1001-1008). Record bytes equal the
 * reference's only where these equal the host libm's results on the arguments the balancing reaches. x, lg, ex:
 * DEVICE arrays of n doubles. No counterpart in the reference. */
int sjk_seal_libm_probe(const double * x, size_t n, double * lg, double * ex, sjk_stream st);

#ifdef __cplusplus
}
#endif
#endif /* SJK_H */
