// sjk_internal.h - entry points shared between the library's translation units (not exported API).
#pragma once
#include <cuda_runtime.h>

#include "../../include/sjk.h"

void sjk_set_cuda_error(cudaError_t e);
void sjk_set_sticky(int status);

// attention over KV heads [kv_head0, kv_head0 + n_kv) only (query heads kv*grp.. of those)
// regions: SJK_REGION_* mask of the positions attended to; part_out: when not null, the combined partial
// (m, l, o[D]) per (query row, query head) instead of the normalized output
int sjk_attend_heads(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, int kv_head0,
                     int n_kv, const float * q, float scale, float * out, void * scratch, size_t scratch_bytes,
                     sjk_stream st, unsigned regions, float * part_out);
size_t sjk_attend_heads_scratch_bytes(const sjk_view * v, int n_q, int n_head, int n_kv);
// decode the K and V rows of position pos, KV head h, to k[D], v[D] (device)
int sjk_kv_row(const sjk_view * v, uint32_t B, uint32_t pos, int h, float * k, float * vo, sjk_stream st);
// decode row t of one record (is_v selects V) to out[D] (device)
int sjk_decode_row(const sj_kvarn_layout * lay, const uint8_t * rec, int t, int is_v, float * out, sjk_stream st);
// the reference's record attention helpers on device pointers (sjk_decode.cu)
int sjk_record_scores(const sj_kvarn_layout * lay, const uint8_t * rec, const float * q, int n, float * scores, sjk_stream st);
int sjk_record_accum_v(const sj_kvarn_layout * lay, const uint8_t * rec, const float * w, int n, float * acc, sjk_stream st);

// tensor-core attention over the sealed body of a 4-bit scalar layer (sjk_attend_tc.cu); dense_regions: the same
// CTAs also take the staged rows (bit 0 the sink, bit 1 the staging ring; formats of sjk_tc_dense_supported). *splits_out gets the
// number of partial slots per query row the launch writes (from split0).
int sjk_tc_body_supported(const sjk_view * v, int n_q, int grp);
int sjk_tc_body_max_splits(int n_kv);
// max_ctas: SMs the kernel may take (fewer than 148 when the dense kernel runs beside it); q_model: q holds model-basis
// queries, which the kernel rotates on chip
int sjk_tc_body_launch(const sjk_view * v, uint32_t B, uint32_t N, uint32_t n_rec, int dense_regions, uint32_t qpos0, int n_q,
                       int n_head, int kv0, int n_kv, const float * q, float scale, float * part, int split0, int max_ctas,
                       bool q_model, int * splits_out, sjk_stream st);

// tensor-core attention over the sealed body of a trellis layer (2- and 3-bit codes, sjk_attend_trellis.cu)
int sjk_tc_trellis_supported(const sjk_view * v, int n_q, int grp);
int sjk_tc_trellis_max_splits(int n_kv);
// splits: per KV head, from the call's plan (sjk_plan_counts)
int sjk_tc_trellis_launch(const sjk_view * v, uint32_t B, uint32_t N, uint32_t n_rec, uint32_t qpos0, int n_q, int n_head,
                          int kv0, int n_kv, const float * q, float scale, float * part, int split0, int splits,
                          int * splits_out, sjk_stream st);

// tensor-core attention over the staged rows: the sink [0, S) and the staging ring [B, N) (sjk_attend_dense.cu)
int sjk_tc_dense_supported(const sjk_view * v, int n_q, int grp);
int sjk_tc_dense_splits(uint32_t n_chunks, int n_kv, int * chunks_per_split);
// beside_tc: launched right after the same call's trellis kernel, as its programmatic dependent (side by side on the
// SMs it leaves free; the kernel's completion still follows the trellis kernel's)
int sjk_tc_dense_launch(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, int kv0, int n_kv,
                        const float * q, float scale, float * part, int split0, int splits, uint32_t n_sink_chunks,
                        uint32_t n_chunks, int chunks_per_split, bool beside_tc, sjk_stream st);

// device status words of the tensor-core translation units (read and cleared; -1 on a CUDA error)
int sjk_tc_body_status_take(void);
int sjk_tc_dense_status_take(void);
int sjk_tc_trellis_status_take(void);
int sjk_xchg_status_take(void);

// Move the record groups [g0, g0 + n) of one layer (group_bytes = n_head_kv x record bytes) through
// an optional device block table: op 0 gathers them into buf (group order), op 1 scatters buf into them, op 2
// zeroes them. Groups with no block are skipped (op 0 writes zeros for them). One launch (sjk_decode.cu).
int sjk_group_move(uint8_t * body, const uint32_t * blocks, uint32_t g0, uint32_t n, size_t group_bytes, uint8_t * buf, int op,
                   sjk_stream st);

// ---- descriptor-driven attention (sjk_attend_dyn): the counts are planned on the device into a sjk_dyn_state
// (sjk_plan.cuh); each kernel family's planner kernel writes its launch plan into `params` (device memory of the
// family's *_params_bytes()) and its kernel reads it there
struct sjk_dyn_state;
size_t sjk_tc_body_params_bytes(void);
size_t sjk_tc_trellis_params_bytes(void);
size_t sjk_tc_dense_params_bytes(void);
int sjk_tc_body_dyn_launch(const sjk_view * v, int n_q, int n_head, int kv0, int n_kv, const float * q, float scale,
                           float * part, const sjk_dyn_state * ds, void * params, sjk_stream st);
int sjk_tc_trellis_dyn_launch(const sjk_view * v, int n_q, int n_head, int kv0, int n_kv, const float * q, float scale,
                              float * part, const sjk_dyn_state * ds, void * params, sjk_stream st);
int sjk_tc_dense_dyn_launch(const sjk_view * v, int n_q, int n_head, int kv0, int n_kv, const float * q, float scale,
                            float * part, const sjk_dyn_state * ds, void * params, int max_items, sjk_stream st);
// descriptor faults of the seal and store kernels (SJK_DEVICE_DESC; read and cleared)
int sjk_seal_desc_status_take(void);
int sjk_stage_desc_status_take(void);
