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
