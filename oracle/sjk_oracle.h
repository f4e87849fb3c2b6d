/*
 * sjk_oracle.h - CPU oracle for the SJ-KVaRN hot path (TEST INFRASTRUCTURE ONLY).
 *
 * A plain-C restatement of the reference codec in sj_kvarn.h (JakeATX/sj-kvarn-codec):
 * fp16 conversion, Hadamard rotation, record layout, tq6_0 staging, seal (variance
 * balancing + RTN / trellis), decode, the adaptive-tail policy, a host per-layer cache
 * (store / seal / attention loop) and the sequence-state stream. Each function cites the
 * reference lines it follows.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this
 * library, and only as the checker. The product (libsjk_b200.so) never links it.
 *
 * Parity pins: the record/decode/tq6_0 results are checked against the reference's 21
 * golden FNV-1a hashes (tests/golden/expected_vectors.txt), the fp16 conversion
 * exhaustively against the reference's round-to-nearest-even rule, and the state stream
 * against the reference's 5 golden stream hashes (tests/golden/expected_state.txt).
 *
 * Build: -O2 -ffp-contract=off, no -ffast-math (every float op rounds once; fma() only
 * where the reference calls fma). Links libm for double log/exp/sqrt, as the reference.
 */
#ifndef SJK_ORACLE_H
#define SJK_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* record layout, sj_kvarn.h:156-175, 771-790 */
typedef struct ora_layout {
    int D, G, bits_k, bits_v, trellis;
    uint32_t kp, vp, ks, kz, kt, vc, vs, vz, bytes;
} ora_layout;

int      ora_layout_init(ora_layout * l, int D, int G, int bits_k, int bits_v, int trellis);
uint16_t ora_f2h(float f);
float    ora_h2f(uint16_t h);
void     ora_fwht(float * x, int n);
uint32_t ora_code_bit(const ora_layout * l, int t, int d, int is_v);
int      ora_k_ch(const ora_layout * l, int d);
int      ora_v_ch(const ora_layout * l, int d);

/* tq6_0 staging: n % 128 == 0, 98-byte blocks (sj_kvarn.h:146-154, 1211-1284) */
void ora_tq6_encode(const float * x, uint8_t * blocks, int n);
void ora_tq6_decode(const uint8_t * blocks, float * x, int n);
void ora_stage_row(int staging, const float * x, uint8_t * dst, int D);
void ora_unstage_row(int staging, const uint8_t * src, float * x, int D);
size_t ora_stage_bytes(int staging, int D);

/* seal one (group, head) from G fp16 rows (row t at K + t*row_stride); sj_kvarn.h:1149-1174 */
void ora_seal(const ora_layout * l, const uint16_t * K, const uint16_t * V, size_t row_stride, int iters, uint8_t * rec);
/* seal n_rec records: record r = g*H + h from rows k + g*G*row_stride + h*D (sj_kvarn_cuda.cuh:48-55),
 * spread over n_threads host threads (0 = all cores) */
void ora_seal_batch(const ora_layout * l, const uint16_t * k, const uint16_t * v, size_t row_stride, int H,
                    int n_rec, int iters, uint8_t * body, int n_threads);
void ora_decode_k(const ora_layout * l, const uint8_t * rec, int t, float * out);
void ora_decode_v(const ora_layout * l, const uint8_t * rec, int t, float * out);

/* adaptive-tail policy, sj_kvarn.h:228-234, 1315-1407 */
typedef struct ora_policy {
    uint32_t sink, tail, tail_max, group, flush_chunk;
    uint32_t B, B_prev, B_pending;
    int draining;
} ora_policy;
void     ora_policy_init(ora_policy * p, uint32_t sink, uint32_t tail, uint32_t tail_max, uint32_t group, uint32_t flush_chunk);
uint32_t ora_policy_begin(ora_policy * p, uint32_t pos0, uint32_t n_tokens);
void     ora_policy_commit(ora_policy * p);
uint32_t ora_policy_idle(ora_policy * p, uint32_t end, uint32_t keep_recent);
uint32_t ora_policy_truncate(ora_policy * p, uint32_t pos, uint32_t * n_dropped);
uint32_t ora_group_floor(uint32_t sink, uint32_t group, uint32_t pos);
uint32_t ora_ring_capacity(uint32_t tail, uint32_t tail_max, uint32_t group, uint32_t n_ubatch);

/* host per-layer cache with the reference memory layout (sj_kvarn.h:293-309) */
typedef struct ora_cache {
    ora_layout lay;
    int H, staging, sink_f16, iters;
    uint32_t S, cap, n_groups;
    size_t stage_bytes;
    uint8_t * sink;            /* f16: [S][H][K D | V D] fp16; inherit: [S][H][2*stage_bytes] */
    uint8_t * ring;            /* [cap][H][K row | V row] */
    uint8_t * body;            /* [n_groups][H][record] (or a pool slab when blocks != NULL) */
    const uint32_t * blocks;   /* group -> block, NULL = contiguous */
} ora_cache;
/* allocates sink/ring/body (calloc); returns 0 or -1 */
int  ora_cache_init(ora_cache * c, int D, int H, int bits_k, int bits_v, int trellis, int iters, int staging,
                    int sink_f16, uint32_t S, uint32_t tail, uint32_t tail_max, uint32_t n_ubatch, uint32_t n_ctx);
void ora_cache_free(ora_cache * c);
void ora_store(ora_cache * c, uint32_t pos, const float * k_rot, const float * v_rot);
void ora_seal_range(ora_cache * c, uint32_t B_from, uint32_t B_to, int n_threads);
uint8_t * ora_record(const ora_cache * c, uint32_t g, int h);
void ora_kv_row(const ora_cache * c, uint32_t B, uint32_t pos, int h, float * k, float * v);
void ora_attend_row(const ora_cache * c, uint32_t B, uint32_t N, const float * q, int h, uint32_t qpos, float scale, float * out);
/* n_q rows x n_head query heads, [n_q][n_head][D] in and out, over n_threads threads (0 = all cores) */
void ora_attend(const ora_cache * c, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, const float * q,
                float scale, float * out, int n_threads);

/* sequence-state stream of nl caches that share one policy (sj_kvarn.h:417-431, 1873-1929).
 * Returns the stream size; writes it when dst != NULL. */
size_t ora_state_write(const ora_cache * layers, int nl, const ora_policy * p, uint32_t n, int bits_k, int bits_v,
                       int trellis, int iters, int staging, int sink_f16, uint32_t tail, uint32_t tail_max,
                       uint32_t flush_chunk, uint8_t * dst);

/* trace every log()/exp() argument of the balancing (and the running log-scale each log result is added to) into
 * the given arrays (NULL stops tracing); counts of the arguments seen since (only the first cap are kept) */
void ora_trace_balance(double * log_args, double * log_prev, double * exp_args, size_t cap);
/* out[i] = clamp(prev[i] + lg[i], -0.3, 10): the balancing's update of a running log-scale */
void ora_balance_step(const double * prev, const double * lg, size_t n, double * out);
void ora_trace_counts(size_t * n_log, size_t * n_exp);
/* this host's libm log and exp of n doubles */
void ora_libm_log_exp(const double * x, size_t n, double * lg, double * ex);

uint64_t ora_fnv(const void * p, size_t n, uint64_t h);
#define ORA_FNV0 1469598103934665603ULL

#ifdef __cplusplus
}
#endif
#endif
