/* ref_glue.c — binds the reference's own compiled kernels into the oracle's kernel table.
 * TEST INFRASTRUCTURE ONLY: linked with the reference sources (compiled where they lie, by
 * oracle/Makefile, one library per activation block E2_I8_BLOCK) into oracle/_ref/libe2ref_b<B>.so.
 *
 * What runs through this table is the reference implementation itself: e2_cpu_init()'s best int8
 * backend (AVX512-VNNI here, src/kernels.c:506-527), its fp32 vtable (src/kernels_avx512.c), its
 * blocked fp32 GEMM and its thread pool (src/threads.c). Only the composition (encoder.c) is ours.
 */
#include <stddef.h>

#include "e2_oracle.h"
#include "int8.h"
#include "kernels.h"
#include "threads.h"

/* e2o_q8w mirrors e2_q8w byte for byte so one pointer serves both */
_Static_assert(sizeof(e2o_q8w) == sizeof(e2_q8w), "e2o_q8w layout");
_Static_assert(offsetof(e2o_q8w, w) == offsetof(e2_q8w, w), "w");
_Static_assert(offsetof(e2o_q8w, bsq) == offsetof(e2_q8w, bsq), "bsq");
_Static_assert(offsetof(e2o_q8w, scale) == offsetof(e2_q8w, scale), "scale");
_Static_assert(offsetof(e2o_q8w, Npad) == offsetof(e2_q8w, Npad), "Npad");
_Static_assert(offsetof(e2o_q8w, out_min) == offsetof(e2_q8w, out_min), "out_min");
_Static_assert(offsetof(e2o_q8w, borrowed) == offsetof(e2_q8w, borrowed), "borrowed");

int e2ref_block(void) { return E2_I8_BLOCK; }

/* Selects the CPU backends and starts the reference pool with `nthreads` workers (0 = the pool's own
 * default: physical cores, capped at 64, src/threads.c:184-272). Returns the worker count. */
int e2ref_init(int nthreads) {
    e2_cpu_init();
    static int pool_up;
    if (!pool_up) {
        if (e2_pool_global_init(nthreads) <= 0) return -1; /* returns the worker count */
        pool_up = 1;
    }
    return e2_nthreads();
}

/* Backend selection only, no pool: for a library whose kernels run inside another library's pool
 * workers (ref_mux.c). */
void e2ref_init_cpu(void) { e2_cpu_init(); }

const char *e2ref_backend(void) { return e2_cpu_name(); }

static void ref_quantize(int8_t *out, float *scales, const float *x, int M, int K, float lo, float hi) {
    e2_i8_quantize(out, scales, x, M, K, lo, hi);
}
static void ref_gemm(float *y, const int8_t *qa, const float *as, const e2o_q8w *w, int M, int N,
                     int n0, int n1) {
    e2_i8_gemm(y, qa, as, (const e2_q8w *)w, M, N, n0, n1);
}
static int ref_q8w(e2o_q8w *q, const float *w, int N, int K) {
    return e2_q8w_from_f32((e2_q8w *)q, w, N, K);
}
static void ref_q8w_free(e2o_q8w *q) { e2_q8w_free((e2_q8w *)q); }
static void ref_rmsnorm(float *x, int M, int D, const float *g, float eps) {
    e2_k()->rmsnorm(x, M, D, g, eps);
}
static void ref_norm_split(float *x, float *res, int rows, int D, const float *g, float eps) {
    e2_k()->norm_split(x, res, rows, D, g, eps);
}
static void ref_norm_add(float *out, const float *src, const float *res, int rows, int D,
                         const float *g, float eps) {
    e2_k()->norm_add(out, src, res, rows, D, g, eps);
}
static void ref_gelu(float *x, size_t n) { e2_k()->gelu_tanh(x, n); }
static void ref_mul(float *a, const float *b, size_t n) { e2_k()->mul(a, b, n); }
static void ref_softmax(float *x, int n) { e2_k()->softmax(x, n); }
static void ref_rope(float *x, int r0, int r1, int ng, int hd, int blk, const float *cs, const float *sn) {
    e2_k()->rope_rows(x, r0, r1, ng, hd, blk, cs, sn);
}
static void ref_sgemm(float *C, int ldc, const float *A, int lda, const float *B, int ldb, int M, int N,
                      int K, int m0, int m1) {
    e2_sgemm_nn_range(C, ldc, A, lda, B, ldb, M, N, K, m0, m1);
}
static void ref_parallel(e2o_task_fn fn, void *arg) { e2_parallel((e2_task_fn)fn, arg); }

const e2o_kernels *e2ref_kernels(void) {
    static e2o_kernels k;
    k.name = "reference";
    k.ablk = E2_I8_BLOCK;
    k.quantize = ref_quantize;
    k.gemm = ref_gemm;
    k.q8w_from_f32 = ref_q8w;
    k.q8w_free = ref_q8w_free;
    k.rmsnorm = ref_rmsnorm;
    k.norm_split = ref_norm_split;
    k.norm_add = ref_norm_add;
    k.gelu_tanh = ref_gelu;
    k.mul = ref_mul;
    k.softmax = ref_softmax;
    k.rope_rows = ref_rope;
    k.sgemm_nn = ref_sgemm;
    k.meanpool = e2_meanpool_f32;
    k.l2norm = e2_l2norm_f32;
    k.parallel = ref_parallel;
    k.nthreads = e2_nthreads();
    return &k;
}

/* The reference's quantise + N-split GEMM region over the pool (src/text.c:367-411), for timing a
 * single quantised linear layer: y = int8 GEMM(quant(x)). */
struct lin_task {
    const float *x;
    int8_t *qa;
    float *as;
    const e2_q8w *w;
    float *y;
    int M, K, N, nb, tile;
    _Atomic int qnext, qdone, next;
};

static void lin_worker(void *arg, int tid, int nthreads) {
    struct lin_task *t = arg;
    (void)tid;
    for (;;) {
        const int m0 = __atomic_fetch_add(&t->qnext, 16, __ATOMIC_RELAXED);
        if (m0 >= t->M) break;
        const int n = t->M - m0 < 16 ? t->M - m0 : 16;
        e2_i8_quantize(t->qa + (size_t)m0 * t->K, t->as + (size_t)m0 * t->nb, t->x + (size_t)m0 * t->K,
                       n, t->K, -__builtin_inff(), __builtin_inff());
    }
    __atomic_fetch_add(&t->qdone, 1, __ATOMIC_RELEASE);
    while (__atomic_load_n(&t->qdone, __ATOMIC_ACQUIRE) < nthreads) e2_pause();
    for (;;) {
        const int a = __atomic_fetch_add(&t->next, t->tile, __ATOMIC_RELAXED);
        if (a >= t->N) break;
        const int b = a + t->tile < t->N ? a + t->tile : t->N;
        e2_i8_gemm(t->y, t->qa, t->as, t->w, t->M, t->N, a, b);
    }
}

int e2ref_linear(const float *x, int M, int K, const e2o_q8w *w, int8_t *qa_scratch,
                 float *as_scratch, float *y) {
    struct lin_task t;
    t.x = x;
    t.qa = qa_scratch;
    t.as = as_scratch;
    t.w = (const e2_q8w *)w;
    t.y = y;
    t.M = M;
    t.K = K;
    t.N = w->N;
    t.nb = (K + E2_I8_BLOCK - 1) / E2_I8_BLOCK;
    int tile = t.N / (4 * e2_nthreads());
    if (tile > 64) tile = 64;
    tile = (tile + 15) & ~15;
    t.tile = tile < 16 ? 16 : tile;
    t.qnext = t.qdone = t.next = 0;
    e2_parallel(lin_worker, &t);
    return 0;
}
