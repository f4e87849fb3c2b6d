/* Host side of the seeded synthetic input generator (sj-kvarn-codec_b200/csrc/sjk_synth.h), compiled into the
 * CPU checkers (liboracle.so) and the reference build (_ref/libsjref.so) so that the oracle, the compiled reference
 * and the device kernels (sjk_synth_* in libsjk_b200.so) all see the same fp32 bytes. Input generation only.
 * Build with -ffp-contract=off (every double operation rounds once, as on the device). */
#define _GNU_SOURCE
#include "../sj-kvarn-codec_b200/csrc/sjk_synth.h"

#include <pthread.h>
#include <stdlib.h>
#include <unistd.h>

/* scale: [n_layers][H][D] channel scales of layers layer0 .. layer0 + n_layers - 1 */
void sjk_synth_scales_host(uint64_t seed, int layer0, int n_layers, int H, int D, float * scale) {
    int il, h;
    for (il = 0; il < n_layers; ++il)
        for (h = 0; h < H; ++h)
            sjk_syn_scales_head(seed, (uint32_t) (layer0 + il), h, D, scale + ((size_t) il * H + h) * D);
}

typedef struct syn_job {
    uint64_t kk, vk, ck, qk;
    int heavy, H, D, nt, tid;
    const float * scale;
    uint64_t j0, n_pairs;
    float * k, * v, * q;
} syn_job;

static void * syn_kv_worker(void * a) {
    syn_job * j = (syn_job *) a;
    const uint64_t hd = (uint64_t) j->H * (uint64_t) j->D;
    uint64_t p;
    for (p = (uint64_t) j->tid; p < j->n_pairs; p += (uint64_t) j->nt) {
        const uint64_t e = j->j0 + 2 * p;                 /* global element index (even) */
        const uint64_t c = e % hd;                        /* h * D + d of element e; e + 1 is the next channel */
        sjk_syn_kv_pair(j->kk, j->vk, j->ck, j->heavy, e >> 1, j->scale[c], j->scale[c + 1], j->k + 2 * p,
                        j->k + 2 * p + 1, j->v + 2 * p, j->v + 2 * p + 1);
    }
    return NULL;
}

static int syn_threads(int n) {
    if (n > 0) return n > 256 ? 256 : n;
    n = (int) sysconf(_SC_NPROCESSORS_ONLN);
    return n < 1 ? 1 : (n > 256 ? 256 : n);
}

/* K and V rows of positions [pos0, pos0 + n) of one layer: k, v are [n][H][D] floats (model basis);
 * scale: that layer's [H][D] channel scales (sjk_synth_scales_host). H * D must be even. */
void sjk_synth_kv_host(uint64_t seed, int layer, int H, int D, int heavy, const float * scale, uint32_t pos0, uint32_t n,
                       float * k, float * v, int n_threads) {
    pthread_t th[256];
    syn_job jb[256];
    int i, nt = syn_threads(n_threads);
    const uint64_t hd = (uint64_t) H * (uint64_t) D;
    if (n_threads == 1 || (uint64_t) n * hd < 65536) nt = 1;
    for (i = 0; i < nt; ++i) {
        jb[i].kk = sjk_syn_key(seed, (uint32_t) layer, SJK_SYN_K);
        jb[i].vk = sjk_syn_key(seed, (uint32_t) layer, SJK_SYN_V);
        jb[i].ck = sjk_syn_key(seed, (uint32_t) layer, SJK_SYN_CHI);
        jb[i].heavy = heavy; jb[i].H = H; jb[i].D = D; jb[i].nt = nt; jb[i].tid = i; jb[i].scale = scale;
        jb[i].j0 = (uint64_t) pos0 * hd; jb[i].n_pairs = (uint64_t) n * hd / 2; jb[i].k = k; jb[i].v = v;
    }
    if (nt == 1) {
        syn_kv_worker(&jb[0]);
        return;
    }
    for (i = 0; i < nt; ++i) pthread_create(&th[i], NULL, syn_kv_worker, &jb[i]);
    for (i = 0; i < nt; ++i) pthread_join(th[i], NULL);
}

/* n_rows query rows of D values (fp16-rounded floats) of one layer: q is [n_rows][D], row r = iq * n_head + hq */
void sjk_synth_q_host(uint64_t seed, int layer, uint32_t n_rows, int D, float * q) {
    const uint64_t key = sjk_syn_key(seed, (uint32_t) layer, SJK_SYN_Q);
    uint64_t p;
    for (p = 0; p < (uint64_t) n_rows * (uint64_t) D / 2; ++p) sjk_syn_q_pair(key, p, q + 2 * p, q + 2 * p + 1);
}

/* the portable ln / exp / cos-sin of the generator, exposed for their accuracy test */
double sjk_synth_ln(double x) { return sjk_syn_ln(x); }
double sjk_synth_exp(double x) { return sjk_syn_exp(x); }
void sjk_synth_cossin(double v, double * c, double * s) { sjk_syn_cossin_turns(v, c, s); }
uint16_t sjk_synth_f16(float f) { return sjk_syn_f16(f); }
