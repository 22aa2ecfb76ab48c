/* ref_mux.c — one kernel table over all the per-block reference builds. TEST INFRASTRUCTURE ONLY.
 *
 * The reference fixes its activation block at compile time (E2_I8_BLOCK, src/int8.h:68) and runs its
 * per-row mode as a build with E2_I8_BLOCK = K, so a layer whose GEMMs have different K (768 for
 * q|k|v and gate|up, 1152 for down, 3072 for the head) needs one build per K. This library loads
 * oracle/_ref/libe2ref_b<B>.so for every B present (RTLD_LOCAL, so their identical symbol names stay
 * apart) and routes each quantise / GEMM / weight-quantise call to the build whose block matches:
 * B = K in per-row mode, B = 128 in block mode. The fp32 vtable and the thread pool come from the
 * 128 build only, so exactly one pool runs and every per-K kernel executes inside its workers
 * (the reference kernels are reentrant, src/text.c:301-318).
 */
#include <dlfcn.h>
#include <stdio.h>
#include <string.h>

#include "e2_oracle.h"

#define MAXB 16
static int g_nb;
static int g_block[MAXB];
static const e2o_kernels *g_tab[MAXB];
static const e2o_kernels *g_base; /* the 128 build */
static int g_mode_ablk;           /* 0: per-row, else 128 */
static char g_err[256];

const char *e2refmux_error(void) { return g_err; }

static const e2o_kernels *for_k(int K) {
    const int want = g_mode_ablk ? g_mode_ablk : K;
    for (int i = 0; i < g_nb; i++)
        if (g_block[i] == want) return g_tab[i];
    fprintf(stderr, "ref_mux: no reference build with E2_I8_BLOCK=%d\n", want);
    return NULL;
}

static void mux_quantize(int8_t *out, float *scales, const float *x, int M, int K, float lo, float hi) {
    const e2o_kernels *k = for_k(K);
    if (k) k->quantize(out, scales, x, M, K, lo, hi);
}
static void mux_gemm(float *y, const int8_t *qa, const float *as, const e2o_q8w *w, int M, int N, int n0, int n1) {
    const e2o_kernels *k = for_k(w->K);
    if (k) k->gemm(y, qa, as, w, M, N, n0, n1);
}
static int mux_q8w(e2o_q8w *q, const float *w, int N, int K) {
    const e2o_kernels *k = for_k(K);
    return k ? k->q8w_from_f32(q, w, N, K) : -1;
}

/* Load every build found in `dir`; start the pool of the 128 build with `nthreads` workers (0: the
 * reference's default). Returns the worker count, or -1. */
int e2refmux_init(const char *dir, int nthreads) {
    static const int blocks[] = { 128, 256, 512, 768, 1024, 1152, 2048, 3072, 8192 };
    if (g_nb) return g_base ? g_base->nthreads : -1;
    for (size_t i = 0; i < sizeof blocks / sizeof blocks[0] && g_nb < MAXB; i++) {
        char path[1024];
        snprintf(path, sizeof path, "%s/libe2ref_b%d.so", dir, blocks[i]);
        void *h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
        if (!h) continue;
        int (*init)(int) = (int (*)(int))dlsym(h, "e2ref_init");
        void (*init_cpu)(void) = (void (*)(void))dlsym(h, "e2ref_init_cpu");
        const e2o_kernels *(*tab)(void) = (const e2o_kernels *(*)(void))dlsym(h, "e2ref_kernels");
        if (!init || !init_cpu || !tab) continue;
        if (blocks[i] == 128) {
            if (init(nthreads) <= 0) {
                snprintf(g_err, sizeof g_err, "pool init failed");
                return -1;
            }
        } else {
            init_cpu();
        }
        g_block[g_nb] = blocks[i];
        g_tab[g_nb] = tab();
        if (blocks[i] == 128) g_base = g_tab[g_nb];
        g_nb++;
    }
    if (!g_base) {
        snprintf(g_err, sizeof g_err, "no libe2ref_b128.so in %s", dir);
        return -1;
    }
    return g_base->nthreads;
}

/* The table for block mode `ablk` (128) or per-row mode (0). */
const e2o_kernels *e2refmux_kernels(int ablk) {
    static e2o_kernels k;
    if (!g_base) return NULL;
    k = *g_base;
    k.name = "reference";
    g_mode_ablk = ablk;
    k.ablk = ablk;
    k.quantize = mux_quantize;
    k.gemm = mux_gemm;
    k.q8w_from_f32 = mux_q8w;
    return &k;
}
