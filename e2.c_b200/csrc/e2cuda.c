/* e2cuda.c — the e2cuda C ABI (include/e2cuda.h): library state, weight upload, the op API, the
 * fused FFN block and the host-buffer drop-ins. C11 host code over the CUDA runtime; every kernel
 * is reached through the launchers of launch.h. */
#include "e2cuda.h"

#include <cuda_runtime.h>
#include <math.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "internal.h"
#include "launch.h"

/* ------------------------------------------------------------------ errors */
static _Thread_local char g_err[512];

const char *e2cuda_last_error(void) { return g_err; }

void e2cu_err(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

int e2cu_cuda(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return 0;
    e2cu_err("%s: %s", what, cudaGetErrorString(e));
    return -1;
}

int e2cu_launch(int rc, const char *what) {
    if (rc == 0) return 0;
    e2cu_err("%s: %s", what, e2c_msg());
    return -1;
}

/* ------------------------------------------------------------------ per-device status word */
#define E2CU_MAX_DEV 64
static int *g_status[E2CU_MAX_DEV];

int *e2cu_status(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= E2CU_MAX_DEV) return NULL;
    if (!g_status[dev]) {
        int *p = NULL;
        if (cudaMalloc((void **)&p, sizeof(int)) != cudaSuccess) return NULL;
        if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) {
            cudaFree(p);
            return NULL;
        }
        g_status[dev] = p;
    }
    return g_status[dev];
}

static const char *status_name(int s) {
    switch (s) {
    case 0x101: return "TMA producer timed out waiting for a free stage";
    case 0x102: return "MMA issuer timed out waiting for operands";
    case 0x103: return "epilogue timed out waiting for an accumulator";
    case 0x104: return "attention softmax timed out";
    case 0x105: return "drain of in-flight copies timed out";
    case 0x106: return "token id outside the embedding table";
    case 0x107: return "dynamic shared memory not 1024-byte aligned (kernel skipped)";
    default: return "unknown device failure";
    }
}

/* ------------------------------------------------------------------ workspace generations */
/* The weight-streaming GEMM leaves its workspace zero after every launch that completes; one that
 * failed may leave partial sums behind. Every reported device failure bumps this count, and a
 * workspace cleared at an older count is cleared again before its next use. */
static int g_fail_gen;

void e2cu_note_failure(void) { __atomic_add_fetch(&g_fail_gen, 1, __ATOMIC_RELEASE); }

int e2cu_ws_refresh(int *ws, size_t bytes, int *gen, cudaStream_t st) {
    const int now = __atomic_load_n(&g_fail_gen, __ATOMIC_ACQUIRE);
    if (*gen == now) return 0;
    if (e2cu_cuda(cudaMemsetAsync(ws, 0, bytes, st), "workspace clear")) return -1;
    *gen = now;
    return 0;
}

int e2cuda_check(void *stream) {
    if (e2cu_cuda(cudaStreamSynchronize((cudaStream_t)stream), "synchronize")) return -1;
    int *st = e2cu_status();
    if (!st) {
        e2cu_err("no CUDA device");
        return -1;
    }
    int h = 0;
    if (e2cu_cuda(cudaMemcpy(&h, st, sizeof h, cudaMemcpyDeviceToHost), "status read")) return -1;
    if (h) {
        cudaMemset(st, 0, sizeof(int));
        e2cu_note_failure();
        e2cu_err("device kernel failure 0x%x: %s", h, status_name(h));
        return -1;
    }
    return 0;
}

const char *e2cuda_device(void) {
    static _Thread_local char name[256];
    int dev = 0;
    struct cudaDeviceProp prop;
    name[0] = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaGetDeviceProperties(&prop, dev) == cudaSuccess)
        snprintf(name, sizeof name, "%s", prop.name);
    return name;
}

/* ------------------------------------------------------------------ weights */
static int round_up(int x, int m) { return (x + m - 1) / m * m; }

int e2cu_w8_alloc(e2cuda_w8 *out, int N, int K) {
    memset(out, 0, sizeof *out);
    out->N = N;
    out->K = K;
    out->rows = round_up(N, 16);
    out->ld = round_up(K, 16);
    out->out_min = -1e31f;
    out->out_max = 1e31f;
    if (e2cu_cuda(cudaMalloc((void **)&out->w, (size_t)out->rows * out->ld), "weight alloc") ||
        e2cu_cuda(cudaMalloc((void **)&out->scale, sizeof(float) * (size_t)out->rows), "scale alloc")) {
        e2cuda_w8_free(out);
        return -1;
    }
    return 0;
}

/* quad-interleaved [Npad/8][K/4][8][4] (e2.c src/int8.h:14-18) -> row-major rows [n][ld] */
void e2cu_unpack_q8w(const e2cuda_q8w *q, int8_t *dst, int ld) {
    const int N = q->N, K = q->K, kq = (K + 3) / 4;
    for (int n = 0; n < N; n++) {
        const int8_t *src = q->w + (size_t)(n >> 3) * kq * 32 + (n & 7) * 4;
        int8_t *row = dst + (size_t)n * ld;
        for (int k4 = 0; k4 < kq; k4++) {
            const int8_t *quad = src + (size_t)k4 * 32;
            for (int j = 0; j < 4 && 4 * k4 + j < K; j++) row[4 * k4 + j] = quad[j];
        }
    }
}

int e2cuda_w8_from_int8(const int8_t *w, const float *scale, int N, int K, e2cuda_w8 *out) {
    if (!w || !scale || !out || N <= 0 || K <= 0) {
        e2cu_err("w8_from_int8: bad arguments");
        return -1;
    }
    if (e2cu_w8_alloc(out, N, K)) return -1;
    int8_t *h = calloc((size_t)out->rows, (size_t)out->ld);
    float *s = calloc((size_t)out->rows, sizeof(float));
    if (!h || !s) {
        free(h);
        free(s);
        e2cuda_w8_free(out);
        e2cu_err("w8_from_int8: out of host memory");
        return -1;
    }
    for (int n = 0; n < N; n++) memcpy(h + (size_t)n * out->ld, w + (size_t)n * K, (size_t)K);
    memcpy(s, scale, sizeof(float) * (size_t)N);
    int rc = e2cu_cuda(cudaMemcpy(out->w, h, (size_t)out->rows * out->ld, cudaMemcpyHostToDevice), "weight upload") ||
             e2cu_cuda(cudaMemcpy(out->scale, s, sizeof(float) * out->rows, cudaMemcpyHostToDevice), "scale upload");
    free(h);
    free(s);
    if (rc) e2cuda_w8_free(out);
    return rc ? -1 : 0;
}

int e2cuda_w8_from_q8w(const e2cuda_q8w *q, e2cuda_w8 *out) {
    if (!q || !q->w || !q->scale || !out || q->N <= 0 || q->K <= 0) {
        e2cu_err("w8_from_q8w: bad arguments");
        return -1;
    }
    int8_t *plain = calloc((size_t)q->N, (size_t)q->K);
    if (!plain) {
        e2cu_err("w8_from_q8w: out of host memory");
        return -1;
    }
    e2cu_unpack_q8w(q, plain, q->K);
    const int rc = e2cuda_w8_from_int8(plain, q->scale, q->N, q->K, out);
    free(plain);
    if (!rc) {
        out->out_min = q->out_min;
        out->out_max = q->out_max;
    }
    return rc;
}

void e2cuda_w8_free(e2cuda_w8 *w) {
    if (!w) return;
    if (w->w) cudaFree(w->w);
    if (w->scale) cudaFree(w->scale);
    memset(w, 0, sizeof *w);
}

/* ------------------------------------------------------------------ op API */
int e2cuda_quantize_rows(const float *x, int8_t *q, float *scales, int M, int K, int ablk, float lo, float hi,
                         void *stream) {
    if (M < 0 || (M > 0 && (!x || !q || !scales))) {
        e2cu_err("quantize_rows: bad arguments");
        return -1;
    }
    return e2cu_launch(e2c_quantize(x, K, q, K, scales, M, K, ablk, lo, hi, 0, stream), "quantize_rows");
}

void e2cu_gemm_args(e2c_gemm_args *a, const e2cuda_w8 *w, const int8_t *qa, const float *as, int M, int ablk) {
    memset(a, 0, sizeof *a);
    a->a = qa;
    a->lda = w->ld;
    a->a_scale = as;
    a->w = w->w;
    a->ldw = w->ld;
    a->wrows = w->rows;
    a->w_scale = w->scale;
    a->M = M;
    a->K = w->ld;
    a->ablk = ablk == w->K ? w->ld : ablk;
    a->n0 = 0;
    a->n1 = w->N;
    a->out_min = w->out_min;
    a->out_max = w->out_max;
    a->status = e2cu_status();
}

/* ------------------------------------------------------------------ per-stream GEMM workspace */
/* The op API's GEMM keeps one weight-streaming workspace per (device, stream), grown on demand: a
 * workspace serves one stream at a time, and calls on one stream are ordered. A stream that is
 * being captured never allocates (it uses what it has, or the other GEMM kernels). */
#define E2CU_WS_SLOTS 32
static pthread_mutex_t g_ws_mu = PTHREAD_MUTEX_INITIALIZER;
static struct {
    int used, dev, gen;
    cudaStream_t st;
    int *p;
    size_t n;
} g_ws[E2CU_WS_SLOTS];

/* a ready (zeroed, stream-ordered) workspace of at least `need` bytes for `st`, or NULL */
static int *stream_ws(cudaStream_t st, size_t need, size_t *got) {
    int dev = 0;
    if (!need || cudaGetDevice(&dev) != cudaSuccess) return NULL;
    enum cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) {
        cudaGetLastError();
        return NULL;
    }
    int *out = NULL;
    pthread_mutex_lock(&g_ws_mu);
    int slot = -1, free_slot = -1;
    for (int i = 0; i < E2CU_WS_SLOTS; i++) {
        if (g_ws[i].used && g_ws[i].dev == dev && g_ws[i].st == st) slot = i;
        if (!g_ws[i].used && free_slot < 0) free_slot = i;
    }
    if (slot < 0 && free_slot >= 0 && cap == cudaStreamCaptureStatusNone) {
        slot = free_slot;
        g_ws[slot].used = 1;
        g_ws[slot].dev = dev;
        g_ws[slot].st = st;
        g_ws[slot].p = NULL;
        g_ws[slot].n = 0;
    }
    if (slot >= 0) {
        if (g_ws[slot].n < need && cap == cudaStreamCaptureStatusNone) {
            /* grow: the old buffer may still be in use by queued work on this stream */
            if (g_ws[slot].p) {
                cudaStreamSynchronize(st);
                cudaFree(g_ws[slot].p);
            }
            g_ws[slot].p = NULL;
            g_ws[slot].n = 0;
            int *p = NULL;
            if (cudaMalloc((void **)&p, need) == cudaSuccess) {
                g_ws[slot].p = p;
                g_ws[slot].n = need;
                g_ws[slot].gen = __atomic_load_n(&g_fail_gen, __ATOMIC_ACQUIRE) - 1; /* cleared below */
            } else {
                cudaGetLastError();
            }
        }
        if (g_ws[slot].p && g_ws[slot].n >= need &&
            e2cu_ws_refresh(g_ws[slot].p, g_ws[slot].n, &g_ws[slot].gen, st) == 0) {
            out = g_ws[slot].p;
            *got = g_ws[slot].n;
        }
    }
    pthread_mutex_unlock(&g_ws_mu);
    return out;
}

int e2cuda_i8_gemm(const e2cuda_w8 *w, const int8_t *qa, const float *a_scales, int M, int ablk, int n0, int n1,
                   const e2cuda_epilogue *ep, float *y, int ldy, void *stream) {
    if (!w || !w->w || M < 0 || (M > 0 && (!qa || !a_scales)) || n0 < 0 || n1 > w->N || n0 > n1) {
        e2cu_err("i8_gemm: bad arguments");
        return -1;
    }
    if (w->ld != w->K && ablk != w->K) {
        e2cu_err("i8_gemm: per-block scales need K (%d) to be a multiple of 16", w->K);
        return -1;
    }
    e2c_gemm_args a;
    e2cu_gemm_args(&a, w, qa, a_scales, M, ablk);
    a.n0 = n0;
    a.n1 = n1;
    a.y = y;
    a.ldy = ldy;
    a.epi = E2C_EPI_F32;
    if (ep && ep->dots) {
        a.epi = E2C_EPI_I32;
        a.dots = ep->dots;
        a.ldd = w->N;
    } else if (ep && ep->residual) {
        a.epi = E2C_EPI_RESID;
        a.resid = ep->residual;
        a.ldr = ep->ld_residual;
    }
    if (a.epi != E2C_EPI_I32 && !y) {
        e2cu_err("i8_gemm: no output");
        return -1;
    }
    if (a.epi != E2C_EPI_I32 && ablk == w->K) {
        const size_t need = e2c_gemm_ws_bytes(M);
        if (need) a.ws = stream_ws((cudaStream_t)stream, need, &a.ws_bytes);
    }
    return e2cu_launch(e2c_gemm(&a, stream), "i8_gemm");
}

int e2cuda_attention(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid, float *ctx, int B,
                     int S, int H, float scale, void *stream) {
    if (!q || !k || !vt || !ctx) {
        e2cu_err("attention: bad arguments");
        return -1;
    }
    return e2cu_launch(e2c_attention(q, k, vt, ldvt, valid, ctx, B, S, H, scale, e2cu_status(), stream), "attention");
}

int e2cuda_attention_gqa(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid, float *ctx,
                         int B, int S, int H, int KV, int D, float scale, void *stream) {
    if (!q || !k || !vt || !ctx) {
        e2cu_err("attention_gqa: bad arguments");
        return -1;
    }
    return e2cu_launch(e2c_attention_gqa(q, k, vt, ldvt, valid, ctx, B, S, H, KV, D, scale, e2cu_status(), stream),
                       "attention_gqa");
}

int e2cuda_attention_window(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid, float *ctx,
                            int B, int S, int H, int KV, int D, float scale, int window, void *stream) {
    if (!q || !k || !vt || !ctx) {
        e2cu_err("attention_window: bad arguments");
        return -1;
    }
    return e2cu_launch(e2c_attention_win(q, k, vt, ldvt, valid, ctx, B, S, H, KV, D, scale, window, e2cu_status(), stream),
                       "attention_window");
}

/* ------------------------------------------------------------------ fused FFN (config 1) */
struct e2cuda_ffn {
    int D, I, max_tokens;
    int fused; /* gate|up + GELU + h's quantiser in one kernel (E2C_EPI_GELUQ), h never stored */
    float eps;
    e2cuda_w8 wgu, wd; /* gate|up interleaved per 128 rows */
    float *gamma;
    int8_t *qa, *qh;   /* quantised normed x [M][D]; quantised h [M][I] */
    float *qs, *qhs, *h;
};

/* gate|up interleaved per 128 rows: [g0..127 | u0..127 | g128..255 | u128..255 | ...] so one
 * 256-column GEMM tile holds matching gate and up columns (the GELU-gate epilogue) */
int e2cu_upload_gate_up(const e2cuda_q8w *g, const e2cuda_q8w *u, e2cuda_w8 *out) {
    const int I = g->N, D = g->K;
    if (u->N != I || u->K != D || I % 128) {
        e2cu_err("gate/up: shapes differ or I=%d is not a multiple of 128", I);
        return -1;
    }
    int8_t *gp = malloc((size_t)I * D), *up = malloc((size_t)I * D), *w = malloc((size_t)2 * I * D);
    float *s = malloc(sizeof(float) * 2 * (size_t)I);
    int rc = -1;
    if (!gp || !up || !w || !s) {
        e2cu_err("gate/up: out of host memory");
        goto done;
    }
    e2cu_unpack_q8w(g, gp, D);
    e2cu_unpack_q8w(u, up, D);
    for (int t = 0; t < I / 128; t++)
        for (int i = 0; i < 128; i++) {
            const int n = t * 128 + i;
            memcpy(w + ((size_t)t * 256 + i) * D, gp + (size_t)n * D, (size_t)D);
            memcpy(w + ((size_t)t * 256 + 128 + i) * D, up + (size_t)n * D, (size_t)D);
            s[t * 256 + i] = g->scale[n];
            s[t * 256 + 128 + i] = u->scale[n];
        }
    rc = e2cuda_w8_from_int8(w, s, 2 * I, D, out);
done:
    free(gp);
    free(up);
    free(w);
    free(s);
    return rc;
}

e2cuda_ffn *e2cuda_ffn_create(const e2cuda_q8w *gate, const e2cuda_q8w *up, const e2cuda_q8w *down,
                              const float *gamma, float eps, int max_tokens) {
    if (!gate || !up || !down || !gamma || max_tokens <= 0 || down->K != gate->N || down->N != gate->K ||
        gate->K % 128 || gate->K > 1024) {
        e2cu_err("ffn_create: bad shapes (need gate/up [I][D], down [D][I], D a multiple of 128 up to 1024)");
        return NULL;
    }
    e2cuda_ffn *f = calloc(1, sizeof *f);
    if (!f) {
        e2cu_err("ffn_create: out of host memory");
        return NULL;
    }
    f->D = gate->K;
    f->I = gate->N;
    f->eps = eps;
    f->max_tokens = max_tokens;
    const size_t M = (size_t)max_tokens;
    const char *env = getenv("E2C_FUSED_GELU");
    f->fused = f->I % 128 == 0 && f->I / 128 <= 16 && !(env && env[0] == '0') &&
               e2c_gemm_gelu_quant_supported(f->I / 128);
    if (e2cu_upload_gate_up(gate, up, &f->wgu) || e2cuda_w8_from_q8w(down, &f->wd) ||
        e2cu_cuda(cudaMalloc((void **)&f->gamma, sizeof(float) * f->D), "ffn alloc") ||
        e2cu_cuda(cudaMalloc((void **)&f->qa, M * (size_t)(f->I > f->D ? f->I : f->D)), "ffn alloc") ||
        e2cu_cuda(cudaMalloc((void **)&f->qs, M * sizeof(float)), "ffn alloc") ||
        (f->fused ? (e2cu_cuda(cudaMalloc((void **)&f->qh, M * (size_t)f->I), "ffn alloc") ||
                     e2cu_cuda(cudaMalloc((void **)&f->qhs, M * sizeof(float)), "ffn alloc"))
                  : e2cu_cuda(cudaMalloc((void **)&f->h, M * (size_t)f->I * sizeof(float)), "ffn alloc")) ||
        e2cu_cuda(cudaMemcpy(f->gamma, gamma, sizeof(float) * f->D, cudaMemcpyHostToDevice), "ffn upload")) {
        e2cuda_ffn_destroy(f);
        return NULL;
    }
    return f;
}

void e2cuda_ffn_destroy(e2cuda_ffn *f) {
    if (!f) return;
    e2cuda_w8_free(&f->wgu);
    e2cuda_w8_free(&f->wd);
    cudaFree(f->gamma);
    cudaFree(f->qa);
    cudaFree(f->qs);
    cudaFree(f->qh);
    cudaFree(f->qhs);
    cudaFree(f->h);
    free(f);
}

int e2cuda_ffn_forward(e2cuda_ffn *f, const float *x, int M, float *y, void *stream) {
    if (!f || !x || !y || M < 0 || M > f->max_tokens) {
        e2cu_err("ffn_forward: bad arguments (M=%d, max %d)", M, f ? f->max_tokens : 0);
        return -1;
    }
    if (M == 0) return 0;
    if (e2cu_launch(e2c_norm_quant(x, f->gamma, f->eps, f->qa, f->qs, M, f->D, f->D, stream), "ffn norm_quant"))
        return -1;
    e2c_gemm_args a;
    e2cu_gemm_args(&a, &f->wgu, f->qa, f->qs, M, f->D);
    if (f->fused) {
        /* gate_quant (src/text.c:424-468) in the gate|up GEMM's epilogue: bit-identical to the
         * GELU epilogue followed by the quantiser */
        a.epi = E2C_EPI_GELUQ;
        a.q8 = f->qh;
        a.ldq = f->I;
        a.q8_scale = f->qhs;
        if (e2cu_launch(e2c_gemm(&a, stream), "ffn gate|up + quantise")) return -1;
        e2cu_gemm_args(&a, &f->wd, f->qh, f->qhs, M, f->I);
    } else {
        a.epi = E2C_EPI_GELU;
        a.y = f->h;
        a.ldy = f->I;
        if (e2cu_launch(e2c_gemm(&a, stream), "ffn gate|up")) return -1;
        if (e2cu_launch(e2c_quantize(f->h, f->I, f->qa, f->I, f->qs, M, f->I, f->I, -INFINITY, INFINITY, 0, stream),
                        "ffn quantize"))
            return -1;
        e2cu_gemm_args(&a, &f->wd, f->qa, f->qs, M, f->I);
    }
    a.epi = E2C_EPI_RESID;
    a.y = y;
    a.ldy = f->D;
    a.resid = x;
    a.ldr = f->D;
    return e2cu_launch(e2c_gemm(&a, stream), "ffn down");
}

/* ------------------------------------------------------------------ host drop-ins */
/* The drop-ins share one weight cache and three scratch buffers. e2.c calls its GEMM from every
 * pool worker at once, each on its own column range (src/text.c:301-318), so every drop-in call
 * holds this lock: concurrent calls are safe and run one after another on the device. */
static pthread_mutex_t g_host_mu = PTHREAD_MUTEX_INITIALIZER;
static int g_act_block = 128;

void e2cuda_set_act_block(int ablk) { g_act_block = ablk > 0 ? ablk : 128; }

typedef struct {
    const int8_t *key;
    int N, K, dev;
    e2cuda_w8 w;
} cache_entry;
#define E2CU_CACHE 64
static cache_entry g_cache[E2CU_CACHE];
static int g_cache_next;

/* scratch for the host drop-ins, grown on demand */
static struct {
    void *p;
    size_t n;
    int dev;
} g_scratch[3];

static void *scratch(int i, size_t n) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (g_scratch[i].n < n || g_scratch[i].dev != dev) {
        if (g_scratch[i].p && g_scratch[i].dev == dev) cudaFree(g_scratch[i].p);
        g_scratch[i].p = NULL;
        g_scratch[i].n = 0;
        if (cudaMalloc(&g_scratch[i].p, n) != cudaSuccess) return NULL;
        g_scratch[i].n = n;
        g_scratch[i].dev = dev;
    }
    return g_scratch[i].p;
}

static const e2cuda_w8 *cached_weight(const e2cuda_q8w *q) {
    int dev = 0;
    cudaGetDevice(&dev);
    for (int i = 0; i < E2CU_CACHE; i++)
        if (g_cache[i].key == q->w && g_cache[i].N == q->N && g_cache[i].K == q->K && g_cache[i].dev == dev)
            return &g_cache[i].w;
    cache_entry *e = &g_cache[g_cache_next];
    g_cache_next = (g_cache_next + 1) % E2CU_CACHE;
    if (e->key) e2cuda_w8_free(&e->w);
    e->key = NULL;
    if (e2cuda_w8_from_q8w(q, &e->w)) return NULL;
    e->key = q->w;
    e->N = q->N;
    e->K = q->K;
    e->dev = dev;
    return &e->w;
}

void e2cuda_host_cache_clear(void) {
    pthread_mutex_lock(&g_host_mu);
    for (int i = 0; i < E2CU_CACHE; i++)
        if (g_cache[i].key) {
            e2cuda_w8_free(&g_cache[i].w);
            g_cache[i].key = NULL;
        }
    pthread_mutex_unlock(&g_host_mu);
}

static void quantize_host_locked(int8_t *out, float *scales, const float *x, int M, int K, float lo, float hi) {
    const int ablk = g_act_block < K ? g_act_block : K;
    if (!out || !scales || !x || M <= 0 || K % ablk || K % 16) {
        e2cu_err("i8_quantize_host: bad arguments (M=%d K=%d block %d)", M, K, ablk);
        return;
    }
    const int nb = K / ablk;
    float *dx = scratch(0, sizeof(float) * (size_t)M * K);
    int8_t *dq = scratch(1, (size_t)M * K);
    float *ds = scratch(2, sizeof(float) * (size_t)M * nb);
    if (!dx || !dq || !ds) {
        e2cu_err("i8_quantize_host: device allocation failed");
        return;
    }
    if (e2cu_cuda(cudaMemcpy(dx, x, sizeof(float) * (size_t)M * K, cudaMemcpyHostToDevice), "upload") ||
        e2cu_launch(e2c_quantize(dx, K, dq, K, ds, M, K, ablk, lo, hi, 1, NULL), "i8_quantize_host") ||
        e2cuda_check(NULL) ||
        e2cu_cuda(cudaMemcpy(out, dq, (size_t)M * K, cudaMemcpyDeviceToHost), "download") ||
        e2cu_cuda(cudaMemcpy(scales, ds, sizeof(float) * (size_t)M * nb, cudaMemcpyDeviceToHost), "download"))
        return;
    g_err[0] = 0;
}

void e2cuda_i8_quantize_host(int8_t *out, float *scales, const float *x, int M, int K, float lo, float hi) {
    pthread_mutex_lock(&g_host_mu);
    quantize_host_locked(out, scales, x, M, K, lo, hi);
    pthread_mutex_unlock(&g_host_mu);
}

static void gemm_host_locked(float *y, const int8_t *qa, const float *a_scales, const e2cuda_q8w *w, int M, int N,
                             int n0, int n1) {
    if (!y || !qa || !a_scales || !w || M <= 0 || n0 < 0 || n1 > w->N || n0 >= n1 || w->K % 16 || w->nblocks <= 0 ||
        w->K % w->nblocks) {
        e2cu_err("i8_gemm_host: bad arguments");
        return;
    }
    const int K = w->K, nb = w->nblocks, ablk = K / nb;
    const e2cuda_w8 *dw = cached_weight(w);
    if (!dw) return;
    int8_t *dq = scratch(1, (size_t)M * K);
    float *ds = scratch(2, sizeof(float) * (size_t)M * nb);
    float *dy = scratch(0, sizeof(float) * (size_t)M * (n1 - n0));
    if (!dq || !ds || !dy) {
        e2cu_err("i8_gemm_host: device allocation failed");
        return;
    }
    if (e2cu_cuda(cudaMemcpy(dq, qa, (size_t)M * K, cudaMemcpyHostToDevice), "upload") ||
        e2cu_launch(e2c_flip_bias(dq, (size_t)M * K, NULL), "bias flip") ||
        e2cu_cuda(cudaMemcpy(ds, a_scales, sizeof(float) * (size_t)M * nb, cudaMemcpyHostToDevice), "upload"))
        return;
    /* compute columns [n0, n1) into a dense [M][n1-n0] block, then scatter into y's row stride N */
    e2c_gemm_args a;
    e2cu_gemm_args(&a, dw, dq, ds, M, ablk);
    a.n0 = n0;
    a.n1 = n1;
    a.y = dy - n0; /* column n lands at dy[m * (n1-n0) + n - n0] */
    a.ldy = n1 - n0;
    a.epi = E2C_EPI_F32;
    if (ablk == K) {
        const size_t need = e2c_gemm_ws_bytes(M);
        if (need) a.ws = stream_ws(NULL, need, &a.ws_bytes);
    }
    if (e2cu_launch(e2c_gemm(&a, NULL), "i8_gemm_host") || e2cuda_check(NULL) ||
        e2cu_cuda(cudaMemcpy2D(y + n0, sizeof(float) * (size_t)N, dy, sizeof(float) * (size_t)(n1 - n0),
                               sizeof(float) * (size_t)(n1 - n0), (size_t)M, cudaMemcpyDeviceToHost),
                  "download"))
        return;
    g_err[0] = 0;
}

void e2cuda_i8_gemm_host(float *y, const int8_t *qa, const float *a_scales, const e2cuda_q8w *w, int M, int N,
                         int n0, int n1) {
    pthread_mutex_lock(&g_host_mu);
    gemm_host_locked(y, qa, a_scales, w, M, N, n0, n1);
    pthread_mutex_unlock(&g_host_mu);
}
