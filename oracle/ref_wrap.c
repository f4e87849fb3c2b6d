/* Compiles the unmodified reference header (sj_kvarn.h, found through -I$SJK_REF_DIR)
 * into oracle/_ref/libsjref.so: the reference's own CPU codec, used only as a checker
 * for the oracle and as the timed CPU baseline. Nothing of the reference is copied here.
 * Adds two threaded harnesses over the reference's public, re-entrant calls
 * (sj_kvarn_seal_group with a per-thread workspace; sj_kvarn_layer_attend_row), which
 * the CPU baseline uses to occupy every host core. */
#define _GNU_SOURCE
#define SJ_KVARN_IMPLEMENTATION
#include "sj_kvarn.h"

#include <pthread.h>
#include <stdlib.h>
#include <unistd.h>

typedef struct ref_job {
    const sj_kvarn_layout * l;
    const uint16_t * k, * v;
    size_t row_stride;
    int H, n_rec, iters, nt, tid;
    uint8_t * body;
    const sj_kvarn_layer * L;
    uint32_t B, N, qpos0;
    int n_q, n_head;
    const float * q;
    float scale;
    float * out;
} ref_job;

static int ref_threads(int n) {
    if (n > 0) return n > 256 ? 256 : n;
    n = (int) sysconf(_SC_NPROCESSORS_ONLN);
    return n < 1 ? 1 : (n > 256 ? 256 : n);
}

static void * ref_seal_worker(void * a) {
    ref_job * j = (ref_job *) a;
    void * work = malloc(sj_kvarn_seal_workspace_bytes(j->l));
    int r;
    for (r = j->tid; work && r < j->n_rec; r += j->nt) {
        const int g = r / j->H, h = r % j->H;
        const size_t off = (size_t) g * j->l->G * j->row_stride + (size_t) h * j->l->D;
        sj_kvarn_seal_group(j->l, j->k + off, j->v + off, j->row_stride, j->iters, j->body + (size_t) r * j->l->bytes, work);
    }
    free(work);
    return NULL;
}

void sjref_seal_batch(const sj_kvarn_layout * l, const uint16_t * k, const uint16_t * v, size_t row_stride, int H,
                      int n_rec, int iters, uint8_t * body, int n_threads) {
    pthread_t th[256];
    ref_job jb[256];
    int i, nt = ref_threads(n_threads);
    for (i = 0; i < nt; ++i) {
        jb[i].l = l; jb[i].k = k; jb[i].v = v; jb[i].row_stride = row_stride; jb[i].H = H; jb[i].n_rec = n_rec;
        jb[i].iters = iters; jb[i].nt = nt; jb[i].tid = i; jb[i].body = body;
        pthread_create(&th[i], NULL, ref_seal_worker, &jb[i]);
    }
    for (i = 0; i < nt; ++i) pthread_join(th[i], NULL);
}

static void * ref_attend_worker(void * a) {
    ref_job * j = (ref_job *) a;
    const int D = j->L->cfg.head_dim, grp = j->n_head / j->L->cfg.n_head_kv;
    int i;
    for (i = j->tid; i < j->n_q * j->n_head; i += j->nt) {
        const int iq = i / j->n_head, hq = i % j->n_head;
        sj_kvarn_layer_attend_row(j->L, j->B, j->N, j->q + (size_t) i * D, hq / grp, j->qpos0 + (uint32_t) iq, j->scale,
                                  j->out + (size_t) i * D);
    }
    return NULL;
}

void sjref_attend(const sj_kvarn_layer * L, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, const float * q,
                  float scale, float * out, int n_threads) {
    pthread_t th[256];
    ref_job jb[256];
    int i, nt = ref_threads(n_threads);
    for (i = 0; i < nt; ++i) {
        jb[i].L = L; jb[i].B = B; jb[i].N = N; jb[i].qpos0 = qpos0; jb[i].n_q = n_q; jb[i].n_head = n_head; jb[i].q = q;
        jb[i].scale = scale; jb[i].out = out; jb[i].nt = nt; jb[i].tid = i;
        pthread_create(&th[i], NULL, ref_attend_worker, &jb[i]);
    }
    for (i = 0; i < nt; ++i) pthread_join(th[i], NULL);
}

size_t sjref_sizeof_layer(void) { return sizeof(sj_kvarn_layer); }
size_t sjref_sizeof_seq(void) { return sizeof(sj_kvarn_seq); }
size_t sjref_sizeof_pool(void) { return sizeof(sj_kvarn_pool); }

/* ---- threaded cache building over the reference's public per-position / per-record calls ---- */
sj_kvarn_layer * sjref_layer_new(const sj_kvarn_config * cfg, int * rc) {
    sj_kvarn_layer * L = (sj_kvarn_layer *) calloc(1, sizeof(sj_kvarn_layer));
    *rc = L ? sj_kvarn_layer_init(L, cfg) : -11;
    if (*rc) { free(L); return NULL; }
    return L;
}

void sjref_layer_delete(sj_kvarn_layer * L) {
    if (L) { sj_kvarn_layer_free(L); free(L); }
}

typedef struct ref_store_job {
    sj_kvarn_layer * L;
    uint32_t pos0, n;
    const float * k, * v;
    float * x;
    size_t rows;
    int D, nt, tid;
    uint32_t B_from, ng;
} ref_store_job;

static void * ref_store_worker(void * a) {
    ref_store_job * j = (ref_store_job *) a;
    const size_t row = (size_t) j->L->cfg.n_head_kv * j->L->cfg.head_dim;
    uint32_t i;
    for (i = (uint32_t) j->tid; i < j->n; i += (uint32_t) j->nt)   /* distinct positions -> distinct ring rows */
        sj_kvarn_layer_store(j->L, j->pos0 + i, j->k + (size_t) i * row, j->v + (size_t) i * row);
    return NULL;
}

/* store positions [pos0, pos0+n): k, v are [n][n_head_kv][head_dim] rotated floats */
void sjref_layer_store_mt(sj_kvarn_layer * L, uint32_t pos0, uint32_t n, const float * k, const float * v, int n_threads) {
    pthread_t th[256];
    ref_store_job jb[256];
    int i, nt = ref_threads(n_threads);
    for (i = 0; i < nt; ++i) {
        jb[i].L = L; jb[i].pos0 = pos0; jb[i].n = n; jb[i].k = k; jb[i].v = v; jb[i].nt = nt; jb[i].tid = i;
        pthread_create(&th[i], NULL, ref_store_worker, &jb[i]);
    }
    for (i = 0; i < nt; ++i) pthread_join(th[i], NULL);
}

static void * ref_rotate_worker(void * a) {
    ref_store_job * j = (ref_store_job *) a;
    size_t r;
    for (r = (size_t) j->tid; r < j->rows; r += (size_t) j->nt) sj_kvarn_hadamard(j->x + r * (size_t) j->D, j->D);
    return NULL;
}

void sjref_rotate_mt(float * x, size_t rows, int D, int n_threads) {
    pthread_t th[256];
    ref_store_job jb[256];
    int i, nt = ref_threads(n_threads);
    for (i = 0; i < nt; ++i) {
        jb[i].x = x; jb[i].rows = rows; jb[i].D = D; jb[i].nt = nt; jb[i].tid = i;
        pthread_create(&th[i], NULL, ref_rotate_worker, &jb[i]);
    }
    for (i = 0; i < nt; ++i) pthread_join(th[i], NULL);
}

/* The reference's layer_seal (sj_kvarn.h:1494-1514) spread over threads: every (group, head) record is
 * sealed from its unstaged, fp16-rounded ring rows with a per-thread workspace, as layer_seal does. */
static void * ref_seal_ring_worker(void * a) {
    ref_store_job * j = (ref_store_job *) a;
    sj_kvarn_layer * L = j->L;
    const int D = L->cfg.head_dim, H = L->cfg.n_head_kv, G = L->cfg.group;
    uint16_t * ks = (uint16_t *) malloc((size_t) G * D * 2), * vs = (uint16_t *) malloc((size_t) G * D * 2);
    float * row = (float *) malloc((size_t) D * 4);
    void * work = malloc(sj_kvarn_seal_workspace_bytes(&L->lay));
    uint32_t r;
    for (r = (uint32_t) j->tid; ks && vs && row && work && r < j->ng * (uint32_t) H; r += (uint32_t) j->nt) {
        const uint32_t gi = r / (uint32_t) H, p0 = j->B_from + gi * (uint32_t) G;
        const int h = (int) (r % (uint32_t) H);
        int t, i;
        for (t = 0; t < G; ++t) {
            const uint8_t * src = L->ring + ((size_t) sj_kvarn_ring_slot(L->cfg.sink, L->cap, p0 + (uint32_t) t) * H + h) * 2 * L->stage_bytes;
            sj_kvarn_unstage_row(L->cfg.staging, src, row, D);
            for (i = 0; i < D; ++i) ks[(size_t) t * D + i] = sj_kvarn_f32_to_f16(row[i]);
            sj_kvarn_unstage_row(L->cfg.staging, src + L->stage_bytes, row, D);
            for (i = 0; i < D; ++i) vs[(size_t) t * D + i] = sj_kvarn_f32_to_f16(row[i]);
        }
        sj_kvarn_seal_group(&L->lay, ks, vs, (size_t) D, L->cfg.iters,
                            sj_kvarn_layer_record(L, (p0 - L->cfg.sink) / (uint32_t) G, h), work);
    }
    free(ks); free(vs); free(row); free(work);
    return NULL;
}

void sjref_layer_seal_mt(sj_kvarn_layer * L, uint32_t B_from, uint32_t B_to, int n_threads) {
    pthread_t th[256];
    ref_store_job jb[256];
    int i, nt = ref_threads(n_threads);
    if (B_to <= B_from) return;
    for (i = 0; i < nt; ++i) {
        jb[i].L = L; jb[i].B_from = B_from; jb[i].ng = (B_to - B_from) / (uint32_t) L->cfg.group; jb[i].nt = nt; jb[i].tid = i;
        pthread_create(&th[i], NULL, ref_seal_ring_worker, &jb[i]);
    }
    for (i = 0; i < nt; ++i) pthread_join(th[i], NULL);
}

int sjref_nthreads(int n) { return ref_threads(n); }

/* ---- buffers of a reference layer, for byte comparisons with the device caches ---- */
const uint8_t * sjref_layer_ring(const sj_kvarn_layer * L, size_t * bytes) {
    *bytes = (size_t) L->cap * (size_t) L->cfg.n_head_kv * 2 * L->stage_bytes;
    return L->ring;
}

const uint8_t * sjref_layer_sink(const sj_kvarn_layer * L, size_t * bytes) {
    const size_t per = L->cfg.sink_type == SJKVARN_SINK_F16 ? (size_t) L->cfg.head_dim * 4 : 2 * L->stage_bytes;
    *bytes = (size_t) L->cfg.sink * (size_t) L->cfg.n_head_kv * per;
    return L->sink;
}

uint32_t sjref_layer_cap(const sj_kvarn_layer * L) { return L->cap; }
uint32_t sjref_layer_record_bytes(const sj_kvarn_layer * L) { return L->lay.bytes; }
const sj_kvarn_layout * sjref_layer_layout(const sj_kvarn_layer * L) { return &L->lay; }
