/* text_tower.c — e2.c's own EmbeddingGemma-2 text tower over the e2cuda kernels: weights uploaded
 * once, one device pass per chunk of whole sequences, replayed from a CUDA graph per shape.
 *
 * The pass, following src/text.c:924-984 (activations quantised per 128-element block, as e2.c's
 * default build does; every GEMM writes fp32):
 *
 *   gather: x = bf16 table[id] * embed_scale; quantise(x); quantise(rmsnorm(x) * input_ln[0])
 *   PLE:    ple = GEMM(x) [M][L * P] (its scale and per-slice RMSNorm with ple_proj_norm are applied
 *           where layer l's PLE gate reads slice l)
 *   per layer l:
 *     GEMM q|k|v -> per-head RMSNorm + RoPE -> bf16 Q, K, V^T
 *     attention (sliding window or full, head dim 256 or 512) -> ctx; quantise(ctx)
 *     GEMM o_proj -> x = rmsnorm(.) * post_attn_ln + x; quantise(rmsnorm(x) * pre_ffn_ln)
 *     GEMM gate|up -> quantise(gelu_tanh(gate) * up)
 *     GEMM down -> x = rmsnorm(.) * post_ffn_ln + x; quantise(x)
 *     GEMM ple_gate -> quantise(gelu_tanh(.) * rmsnorm(ple[:, l P .. +P] * ple_scale) * ple_proj_norm)
 *     GEMM ple_proj -> x = (rmsnorm(.) * ple_norm + x) * layer_scalar;
 *                      quantise(rmsnorm(x) * input_ln[l + 1]), after the last layer final_norm
 *   GEMM embed_proj -> masked mean pool -> L2
 *
 * 14 kernels per layer, 5 around them; one fewer each where gate|up applies GELU-gate and h's
 * per-block quantiser in its epilogue, where the q|k|v GEMM finishes its heads of 256 in its
 * epilogue, and for each of o_proj, down and the PLE projection with the residual norms in its
 * epilogue (per-block mode: 9 on layers with heads of 256, 10 on the others). int8 activations alternate between qa (inputs of the
 * hidden-wide GEMMs) and qb (ctx, h and the PLE gate's output), so a row kernel never writes the
 * buffer the GEMM before it still reads.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "internal.h"

#define TT_MAX_GRAPHS 128
#define TT_MAX_LAYERS 64

typedef struct {
    int B, S, has_valid;
    cudaGraphExec_t exec;
    int kernels;
} tt_graph;

typedef struct {
    e2cuda_w8 qkv, o, gu, d, pg, pp;
    int hd, kv, qdim, window, rope; /* rope: index of the layer's RoPE table */
    float ls;
    float *norms; /* device: input, post_attn, pre_ffn, post_ffn, ple_norm [D] + q_norm, k_norm [hd] */
} tt_layer;

struct e2cuda_text {
    int L, D, I, P, H, V, DO, max_seq, ablk, max_tokens;
    int fused_gelu; /* per-block gate|up GEMM with GELU-gate + quantiser epilogue (E2C_FUSED_GELU=0: off) */
    int fused_qkv;  /* per-block q|k|v GEMM with the finish in its epilogue, heads of 256 (E2C_FUSED_QKV=0: off) */
    int fused_norm; /* per-block o_proj / down / PLE projection with the residual norms in the epilogue
                       (E2C_FUSED_NORM=0: off) */
    float eps, embed_scale, ple_scale;
    tt_layer layer[TT_MAX_LAYERS];
    e2cuda_w8 ple_model, embed_proj;
    uint16_t *table;
    float *ple_norm, *final_norm;
    int nrope, rope_hd[2];
    float rope_theta[2];
    float *rope_cos[2], *rope_sin[2];
    /* workspace */
    int32_t *ids;
    uint8_t *valid;
    float *res, *tmp, *yf, *ctx, *ple, *pooled;
    int8_t *qa, *qb, *qp;
    float *qas, *qbs, *qps;
    void *Q, *K, *Vt;
    size_t vt_bytes;
    int *status;
    cudaStream_t stream;
    tt_graph graphs[TT_MAX_GRAPHS];
    int ngraphs;
    long calls, kernels_last;
    double last_ms;
};

static float *lnorm(const e2cuda_text *t, int l, int which) {
    const tt_layer *y = &t->layer[l];
    return which < 5 ? y->norms + (size_t)which * t->D : y->norms + 5 * (size_t)t->D + (size_t)(which - 5) * y->hd;
}

void e2cuda_text_destroy(e2cuda_text *t) {
    if (!t) return;
    for (int i = 0; i < t->ngraphs; i++) cudaGraphExecDestroy(t->graphs[i].exec);
    for (int l = 0; l < t->L; l++) {
        tt_layer *y = &t->layer[l];
        e2cuda_w8_free(&y->qkv);
        e2cuda_w8_free(&y->o);
        e2cuda_w8_free(&y->gu);
        e2cuda_w8_free(&y->d);
        e2cuda_w8_free(&y->pg);
        e2cuda_w8_free(&y->pp);
        if (y->norms) cudaFree(y->norms);
    }
    e2cuda_w8_free(&t->ple_model);
    e2cuda_w8_free(&t->embed_proj);
    void *dev[] = { t->table, t->ple_norm, t->final_norm, t->rope_cos[0], t->rope_sin[0], t->rope_cos[1], t->rope_sin[1],
                    t->ids, t->valid, t->res, t->tmp, t->yf, t->ctx, t->ple, t->pooled, t->qa, t->qb, t->qp, t->qas,
                    t->qbs, t->qps, t->Q, t->K, t->Vt };
    for (size_t i = 0; i < sizeof dev / sizeof dev[0]; i++)
        if (dev[i]) cudaFree(dev[i]);
    if (t->stream) cudaStreamDestroy(t->stream);
    free(t);
}

#define DALLOC(ptr, bytes) e2cu_cuda(cudaMalloc((void **)&(ptr), (bytes)), "text tower alloc " #ptr)

static int upload_floats(float **dst, const float *src, size_t n, const char *what) {
    return e2cu_cuda(cudaMalloc((void **)dst, sizeof(float) * n), what) ||
           e2cu_cuda(cudaMemcpy(*dst, src, sizeof(float) * n, cudaMemcpyHostToDevice), what);
}

/* rows of several e2_q8w stacked into one device weight (q|k|v) */
static int upload_stack(const e2cuda_q8w *const *parts, int nparts, e2cuda_w8 *out) {
    int N = 0;
    const int K = parts[0]->K;
    for (int i = 0; i < nparts; i++) {
        if (parts[i]->K != K) {
            e2cu_err("text tower: projections to stack differ in K");
            return -1;
        }
        N += parts[i]->N;
    }
    int8_t *w = malloc((size_t)N * K);
    float *s = malloc(sizeof(float) * (size_t)N);
    int rc = -1;
    if (w && s) {
        int off = 0;
        for (int i = 0; i < nparts; i++) {
            e2cu_unpack_q8w(parts[i], w + (size_t)off * K, K);
            memcpy(s + off, parts[i]->scale, sizeof(float) * parts[i]->N);
            off += parts[i]->N;
        }
        rc = e2cuda_w8_from_int8(w, s, N, K, out);
    } else {
        e2cu_err("text tower: out of host memory");
    }
    free(w);
    free(s);
    return rc;
}

/* e2.c src/text.c:483-506: inv = 1 / theta^(2i / hd), angle = pos * inv; e2.c duplicates the halves,
 * here they are stored once, position-major ([max_seq][hd/2]) for the q|k|v finish's warp per position */
static int rope_table(e2cuda_text *t, int slot, int hd, float theta) {
    const int half = hd / 2;
    const size_t n = (size_t)t->max_seq * half;
    float *c = malloc(sizeof(float) * n), *s = malloc(sizeof(float) * n);
    if (!c || !s) {
        free(c);
        free(s);
        e2cu_err("text tower: out of host memory");
        return -1;
    }
    for (int p = 0; p < t->max_seq; p++)
        for (int i = 0; i < half; i++) {
            const float inv = 1.0f / powf(theta, (float)(2 * i) / (float)hd);
            const float f = (float)p * inv;
            c[(size_t)p * half + i] = cosf(f);
            s[(size_t)p * half + i] = sinf(f);
        }
    const int rc = upload_floats(&t->rope_cos[slot], c, n, "rope upload") || upload_floats(&t->rope_sin[slot], s, n, "rope upload");
    free(c);
    free(s);
    t->rope_hd[slot] = hd;
    t->rope_theta[slot] = theta;
    return rc;
}

static int q8w_is(const e2cuda_q8w *q, int N, int K) { return q && q->w && q->scale && q->N == N && q->K == K; }

e2cuda_text *e2cuda_text_create(const e2cuda_text_desc *d, int max_tokens) {
    if (!d || d->n_layers <= 0 || d->n_layers > TT_MAX_LAYERS || d->hidden % 128 || d->hidden > 1024 || d->intermediate % 128 ||
        d->intermediate > 2048 || d->ple_dim % 128 || d->ple_dim > 1024 || d->n_heads <= 0 || d->vocab <= 0 ||
        d->out_dim <= 0 || d->out_dim % 4 || d->max_seq <= 0 || max_tokens <= 0 || !d->embed_tokens || !d->layers ||
        !d->ple_proj_norm || !d->final_norm) {
        e2cu_err("text_create: unsupported geometry (hidden and ple_dim multiples of 128 up to 1024, intermediate a "
                 "multiple of 128 up to 2048, at most %d layers)", TT_MAX_LAYERS);
        return NULL;
    }
    /* per-token scales (ablk = hidden) quantise every activation row as one block */
    const int ablk = d->ablk ? d->ablk : 128;
    if (ablk != 128 && ablk != d->hidden) {
        e2cu_err("text_create: ablk must be 128 or hidden");
        return NULL;
    }
    e2cuda_text *t = calloc(1, sizeof *t);
    if (!t) {
        e2cu_err("text_create: out of host memory");
        return NULL;
    }
    t->L = d->n_layers;
    t->D = d->hidden;
    t->I = d->intermediate;
    t->P = d->ple_dim;
    t->H = d->n_heads;
    t->V = d->vocab;
    t->DO = d->out_dim;
    t->max_seq = d->max_seq;
    t->ablk = ablk;
    {
        const char *fg = getenv("E2C_FUSED_GELU"), *fq = getenv("E2C_FUSED_QKV"), *fz = getenv("E2C_FUSED_NORM");
        t->fused_gelu = ablk == 128 && !(fg && fg[0] == '0');
        t->fused_qkv = ablk == 128 && !(fq && fq[0] == '0');
        t->fused_norm = ablk == 128 && d->hidden / 128 <= 8 && !(fz && fz[0] == '0');
    }
    t->max_tokens = max_tokens;
    t->eps = d->eps;
    t->embed_scale = d->embed_scale;
    t->ple_scale = d->ple_scale;
    const int L = t->L, D = t->D, I = t->I, P = t->P;
    int qdim_max = 0, yw = 2 * I > P ? 2 * I : P;
    /* the whole description is checked before any device work */
    for (int l = 0; l < L; l++) {
        const e2cuda_text_layer *x = &d->layers[l];
        const int hd = x->head_dim, kv = x->n_kv_heads, qd = t->H * hd;
        if ((hd != 256 && hd != 512) || kv <= 0 || t->H % kv || kv * hd > 512 || !q8w_is(x->q, qd, D) ||
            !q8w_is(x->k, kv * hd, D) || !q8w_is(x->v, kv * hd, D) || !q8w_is(x->o, D, qd) || !q8w_is(x->gate, I, D) ||
            !q8w_is(x->up, I, D) || !q8w_is(x->down, D, I) || !q8w_is(x->ple_gate, P, D) || !q8w_is(x->ple_proj, D, P) ||
            !x->input_ln || !x->post_attn_ln || !x->pre_ffn_ln || !x->post_ffn_ln || !x->ple_norm || !x->q_norm ||
            !x->k_norm) {
            e2cu_err("text_create: layer %d: shapes do not match (head_dim 256 or 512, KV heads dividing %d heads, "
                     "KV heads x head_dim <= 512)", l, t->H);
            goto fail;
        }
    }
    if (!q8w_is(d->ple_model_proj, L * P, D) || !q8w_is(d->embed_proj, t->DO, D)) {
        e2cu_err("text_create: PLE projection or embed_proj shapes do not match");
        goto fail;
    }
    for (int l = 0; l < L; l++) {
        const e2cuda_text_layer *x = &d->layers[l];
        tt_layer *y = &t->layer[l];
        const int hd = x->head_dim, kv = x->n_kv_heads, qd = t->H * hd;
        y->hd = hd;
        y->kv = kv;
        y->qdim = qd;
        y->window = x->window;
        y->ls = x->layer_scalar;
        if (qd > qdim_max) qdim_max = qd;
        if (qd + 2 * kv * hd > yw) yw = qd + 2 * kv * hd;
        /* the layer's RoPE table: one per distinct (head dim, theta) */
        y->rope = -1;
        for (int r = 0; r < t->nrope; r++)
            if (t->rope_hd[r] == hd && t->rope_theta[r] == x->rope_theta) y->rope = r;
        if (y->rope < 0) {
            if (t->nrope == 2) {
                e2cu_err("text_create: more than two (head_dim, rope_theta) layer types");
                goto fail;
            }
            if (rope_table(t, t->nrope, hd, x->rope_theta)) goto fail;
            y->rope = t->nrope++;
        }
        const e2cuda_q8w *qkv[3] = { x->q, x->k, x->v };
        if (upload_stack(qkv, 3, &y->qkv) || e2cuda_w8_from_q8w(x->o, &y->o) || e2cu_upload_gate_up(x->gate, x->up, &y->gu) ||
            e2cuda_w8_from_q8w(x->down, &y->d) || e2cuda_w8_from_q8w(x->ple_gate, &y->pg) ||
            e2cuda_w8_from_q8w(x->ple_proj, &y->pp))
            goto fail;
        const size_t nn = 5 * (size_t)D + 2 * (size_t)hd;
        float *hn = malloc(sizeof(float) * nn);
        if (!hn) {
            e2cu_err("text_create: out of host memory");
            goto fail;
        }
        const float *src[5] = { x->input_ln, x->post_attn_ln, x->pre_ffn_ln, x->post_ffn_ln, x->ple_norm };
        for (int i = 0; i < 5; i++) memcpy(hn + (size_t)i * D, src[i], sizeof(float) * D);
        memcpy(hn + 5 * (size_t)D, x->q_norm, sizeof(float) * hd);
        memcpy(hn + 5 * (size_t)D + hd, x->k_norm, sizeof(float) * hd);
        const int rc = upload_floats(&y->norms, hn, nn, "norm upload");
        free(hn);
        if (rc) goto fail;
    }
    if (e2cuda_w8_from_q8w(d->ple_model_proj, &t->ple_model) || e2cuda_w8_from_q8w(d->embed_proj, &t->embed_proj) ||
        upload_floats(&t->ple_norm, d->ple_proj_norm, (size_t)P, "norm upload") ||
        upload_floats(&t->final_norm, d->final_norm, (size_t)D, "norm upload") || DALLOC(t->table, (size_t)t->V * D * 2) ||
        e2cu_cuda(cudaMemcpy(t->table, d->embed_tokens, (size_t)t->V * D * 2, cudaMemcpyHostToDevice), "table upload"))
        goto fail;
    {
        const size_t M = (size_t)max_tokens;
        int KQ = D > qdim_max ? D : qdim_max;
        if (I > KQ) KQ = I;
        if (P > KQ) KQ = P;
        if (t->DO > yw) yw = t->DO;
        if (DALLOC(t->ids, sizeof(int32_t) * M) || DALLOC(t->valid, M) || DALLOC(t->res, sizeof(float) * M * D) ||
            DALLOC(t->tmp, sizeof(float) * M * D) || DALLOC(t->yf, sizeof(float) * M * (size_t)yw) ||
            DALLOC(t->ctx, sizeof(float) * M * (size_t)qdim_max) || DALLOC(t->ple, sizeof(float) * M * (size_t)L * P) ||
            DALLOC(t->pooled, sizeof(float) * M * (size_t)t->DO) || DALLOC(t->qa, M * (size_t)KQ) ||
            DALLOC(t->qb, M * (size_t)KQ) || DALLOC(t->qp, M * (size_t)D) ||
            DALLOC(t->qas, sizeof(float) * M * (size_t)(KQ / 128 + 1)) ||
            DALLOC(t->qbs, sizeof(float) * M * (size_t)(KQ / 128 + 1)) ||
            DALLOC(t->qps, sizeof(float) * M * (size_t)(D / 128 + 1)) || DALLOC(t->Q, 2 * M * (size_t)qdim_max) ||
            DALLOC(t->K, 2 * M * (size_t)qdim_max))
            goto fail;
    }
    t->status = e2cu_status();
    if (!t->status || e2cu_cuda(cudaStreamCreateWithFlags(&t->stream, cudaStreamNonBlocking), "stream")) goto fail;
    return t;
fail:
    e2cuda_text_destroy(t);
    return NULL;
}

static int round8(int x) { return (x + 7) & ~7; }

/* the launcher's return code (0, or negative with its message in e2c_msg) */
static int gemm_f32(const e2cuda_w8 *w, const int8_t *qa, const float *qs, int M, int ablk, float *y, int ldy,
                    cudaStream_t st) {
    e2c_gemm_args a;
    e2cu_gemm_args(&a, w, qa, qs, M, ablk);
    a.epi = E2C_EPI_F32;
    a.y = y;
    a.ldy = ldy;
    return e2c_gemm(&a, st);
}

/* the GEMM with the residual norms in its epilogue: x = (rmsnorm(y) g1 + res) ls -> res, then the
 * int8 rows of rmsnorm(x) g2 (or of x itself, g2 NULL) into qa / qas */
static int gemm_norm(const e2cuda_text *t, const e2cuda_w8 *w, const int8_t *qin, const float *qsin, int M, int ablk,
                     const float *g1, float ls, const float *g2, cudaStream_t st) {
    e2c_gemm_args a;
    e2cu_gemm_args(&a, w, qin, qsin, M, ablk);
    a.epi = E2C_EPI_NORMADD;
    a.res = t->res;
    a.ldres = t->D;
    a.norm_g1 = g1;
    a.norm_g2 = g2;
    a.norm_ls = ls;
    a.q8 = t->qa;
    a.ldq = t->D;
    a.q8_scale = t->qas;
    a.eps = t->eps;
    return e2c_gemm(&a, st);
}

/* queue one pass over B sequences of S tokens already in t->ids / t->valid; returns kernels queued */
static int forward(e2cuda_text *t, int B, int S, int has_valid, cudaStream_t st) {
    const int M = B * S, D = t->D, I = t->I, P = t->P, L = t->L, H = t->H;
    const int ab = t->ablk;
    const int ab_i = ab == 128 ? 128 : I, ab_p = ab == 128 ? 128 : P;
    const int ldvt = round8(S);
    const uint8_t *valid = has_valid ? t->valid : NULL;
    int n = 0;
#define Q(call, what)                          \
    do {                                       \
        if (e2cu_launch((call), what)) return -1; \
        n++;                                   \
    } while (0)
    Q(e2c_tt_embed(t->ids, t->table, t->embed_scale, lnorm(t, 0, 0), t->eps, t->res, t->qp, t->qps, t->qa, t->qas, M, D, ab,
                   t->V, t->status, st),
      "text embed");
    Q(gemm_f32(&t->ple_model, t->qp, t->qps, M, ab, t->ple, L * P, st), "text PLE projection");
    for (int l = 0; l < L; l++) {
        const tt_layer *y = &t->layer[l];
        const int hd = y->hd, kv = y->kv, qd = y->qdim, ab_q = ab == 128 ? 128 : qd;
        const int ldy = qd + 2 * kv * hd;
        if (t->fused_qkv && hd == 256) {
            e2c_gemm_args a;
            e2cu_gemm_args(&a, &y->qkv, t->qa, t->qas, M, ab);
            a.epi = E2C_EPI_QKVPB;
            a.nq = H;
            a.q_out = t->Q;
            a.k_out = t->K;
            a.vt_out = t->Vt;
            a.ldvt = ldvt;
            a.seq_len = S;
            a.q_gamma = lnorm(t, l, 5);
            a.k_gamma = lnorm(t, l, 6);
            a.rope_cos = t->rope_cos[y->rope];
            a.rope_sin = t->rope_sin[y->rope];
            a.ldrope = hd / 2;
            a.eps = t->eps;
            Q(e2c_gemm(&a, st), "text qkv + finish");
        } else {
            Q(gemm_f32(&y->qkv, t->qa, t->qas, M, ab, t->yf, ldy, st), "text qkv");
            Q(e2c_tt_qkv_post(t->yf, ldy, H, kv, hd, lnorm(t, l, 5), lnorm(t, l, 6), t->eps, t->rope_cos[y->rope],
                              t->rope_sin[y->rope], hd / 2, 1, S, t->Q, t->K, t->Vt, ldvt, M, st),
              "text qkv post");
        }
        Q(e2c_attention_win(t->Q, t->K, t->Vt, ldvt, valid, t->ctx, B, S, H, kv, hd, 1.0f, y->window, t->status, st),
          "text attention");
        Q(e2c_quantize(t->ctx, qd, t->qb, qd, t->qbs, M, qd, ab_q, -INFINITY, INFINITY, 0, st), "text ctx quant");
        if (t->fused_norm) {
            Q(gemm_norm(t, &y->o, t->qb, t->qbs, M, ab_q, lnorm(t, l, 1), 1.0f, lnorm(t, l, 2), st),
              "text o_proj + post-attention norms");
        } else {
            Q(gemm_f32(&y->o, t->qb, t->qbs, M, ab_q, t->tmp, D, st), "text o_proj");
            Q(e2c_tt_norm_add(t->tmp, t->res, lnorm(t, l, 1), 1.0f, lnorm(t, l, 2), t->eps, t->qa, t->qas, M, D, ab, st),
              "text post-attention norms");
        }
        if (t->fused_gelu) {
            e2c_gemm_args a;
            e2cu_gemm_args(&a, &y->gu, t->qa, t->qas, M, ab);
            a.epi = E2C_EPI_GELUQ;
            a.q8 = t->qb;
            a.ldq = I;
            a.q8_scale = t->qbs;
            Q(e2c_gemm(&a, st), "text gate|up + h quant");
        } else {
            Q(gemm_f32(&y->gu, t->qa, t->qas, M, ab, t->yf, 2 * I, st), "text gate|up");
            Q(e2c_gelu_mul_quant(t->yf, 2 * I, I, t->qb, t->qbs, M, ab_i, st), "text gelu quant");
        }
        if (t->fused_norm) {
            Q(gemm_norm(t, &y->d, t->qb, t->qbs, M, ab_i, lnorm(t, l, 3), 1.0f, NULL, st), "text down + post-ffn norm");
        } else {
            Q(gemm_f32(&y->d, t->qb, t->qbs, M, ab_i, t->tmp, D, st), "text down");
            Q(e2c_tt_norm_add(t->tmp, t->res, lnorm(t, l, 3), 1.0f, NULL, t->eps, t->qa, t->qas, M, D, ab, st),
              "text post-ffn norm");
        }
        Q(gemm_f32(&y->pg, t->qa, t->qas, M, ab, t->yf, P, st), "text PLE gate");
        Q(e2c_tt_gate_quant(t->yf, P, t->ple + (size_t)l * P, L * P, t->ple_scale, t->ple_norm, t->eps, P, t->qb, t->qbs, M,
                            ab_p, st),
          "text PLE gate quant");
        const float *gnext = l + 1 < L ? lnorm(t, l + 1, 0) : t->final_norm;
        if (t->fused_norm) {
            Q(gemm_norm(t, &y->pp, t->qb, t->qbs, M, ab_p, lnorm(t, l, 4), y->ls, gnext, st), "text PLE projection + norms");
        } else {
            Q(gemm_f32(&y->pp, t->qb, t->qbs, M, ab_p, t->tmp, D, st), "text PLE projection");
            Q(e2c_tt_norm_add(t->tmp, t->res, lnorm(t, l, 4), y->ls, gnext, t->eps, t->qa, t->qas, M, D, ab, st),
              "text PLE norms");
        }
    }
    Q(gemm_f32(&t->embed_proj, t->qa, t->qas, M, ab, t->yf, t->DO, st), "text embed_proj");
    Q(e2c_meanpool(t->yf, valid, t->pooled, B, S, t->DO, st), "text pool");
    Q(e2c_l2norm_rows(t->pooled, valid, B, S, t->DO, st), "text l2");
#undef Q
    return n;
}

static int ensure_vt(e2cuda_text *t, int B, int S) {
    int kvd = 0;
    for (int l = 0; l < t->L; l++)
        if (t->layer[l].kv * t->layer[l].hd > kvd) kvd = t->layer[l].kv * t->layer[l].hd;
    const size_t need = (size_t)B * kvd * round8(S) * 2;
    if (need <= t->vt_bytes) return 0;
    for (int i = 0; i < t->ngraphs; i++) cudaGraphExecDestroy(t->graphs[i].exec);
    t->ngraphs = 0;
    if (t->Vt) cudaFree(t->Vt);
    t->Vt = NULL;
    t->vt_bytes = 0;
    if (e2cu_cuda(cudaMalloc(&t->Vt, need), "text V^T alloc")) return -1;
    t->vt_bytes = need;
    return 0;
}

static int pass(e2cuda_text *t, int B, int S, int has_valid, cudaStream_t st) {
    if (ensure_vt(t, B, S)) return -1;
    tt_graph *g = NULL;
    for (int i = 0; i < t->ngraphs; i++)
        if (t->graphs[i].B == B && t->graphs[i].S == S && t->graphs[i].has_valid == has_valid) g = &t->graphs[i];
    if (g) {
        t->kernels_last = g->kernels;
        return e2cu_cuda(cudaGraphLaunch(g->exec, st), "text graph launch");
    }
    const int n = forward(t, B, S, has_valid, st);
    if (n < 0) return -1;
    t->kernels_last = n;
    if (st && t->ngraphs < TT_MAX_GRAPHS) {
        cudaGraph_t graph = NULL;
        if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const int n2 = forward(t, B, S, has_valid, st);
            const cudaError_t ce = cudaStreamEndCapture(st, &graph);
            cudaGraphExec_t exec = NULL;
            if (n2 >= 0 && ce == cudaSuccess && graph && cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess) {
                tt_graph *s = &t->graphs[t->ngraphs++];
                s->B = B;
                s->S = S;
                s->has_valid = has_valid;
                s->exec = exec;
                s->kernels = n2;
            }
            if (graph) cudaGraphDestroy(graph);
        }
        cudaGetLastError(); /* a failed capture only means no graph for this shape */
    }
    return 0;
}

int e2cuda_text_embed_batch_device(e2cuda_text *t, const int32_t *d_ids, const uint8_t *d_valid, int batch, int seq_len,
                                   float *d_out, void *stream) {
    if (!t || !d_ids || !d_out || batch <= 0 || seq_len <= 0 || seq_len > t->max_seq) {
        e2cu_err("text_embed_batch_device: bad arguments (seq_len %d, max %d)", seq_len, t ? t->max_seq : 0);
        return -1;
    }
    cudaStream_t st = (cudaStream_t)stream;
    const int per = t->max_tokens / seq_len;
    if (per <= 0) {
        e2cu_err("text_embed_batch_device: seq_len %d exceeds max_tokens %d", seq_len, t->max_tokens);
        return -1;
    }
    for (int b0 = 0; b0 < batch; b0 += per) {
        const int B = batch - b0 < per ? batch - b0 : per;
        const size_t rows = (size_t)B * seq_len, off = (size_t)b0 * seq_len;
        if (e2cu_cuda(cudaMemcpyAsync(t->ids, d_ids + off, sizeof(int32_t) * rows, cudaMemcpyDeviceToDevice, st), "ids") ||
            (d_valid && e2cu_cuda(cudaMemcpyAsync(t->valid, d_valid + off, rows, cudaMemcpyDeviceToDevice, st), "valid")) ||
            pass(t, B, seq_len, d_valid != NULL, st) ||
            e2cu_cuda(cudaMemcpyAsync(d_out + (size_t)b0 * t->DO, t->pooled, sizeof(float) * (size_t)B * t->DO,
                                      cudaMemcpyDeviceToDevice, st),
                      "out"))
            return -1;
    }
    t->calls++;
    return 0;
}

static double now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec / 1e6;
}

int e2cuda_text_embed_batch(e2cuda_text *t, const int32_t *ids, const uint8_t *valid, int batch, int seq_len, float *out) {
    const double t0 = now_ms();
    if (!t || !ids || !out || batch <= 0 || seq_len <= 0 || seq_len > t->max_seq) {
        e2cu_err("text_embed_batch: bad batch geometry");
        return -1;
    }
    /* validate the whole request before touching the output (src/text.c:1005-1011) */
    const size_t total = (size_t)batch * seq_len;
    for (size_t i = 0; i < total; i++)
        if (ids[i] < 0 || ids[i] >= t->V) {
            e2cu_err("token id %d out of range", ids[i]);
            return -1;
        }
    const int per = t->max_tokens / seq_len;
    if (per <= 0) {
        e2cu_err("text_embed_batch: seq_len %d exceeds max_tokens %d", seq_len, t->max_tokens);
        return -1;
    }
    cudaStream_t st = t->stream;
    for (int b0 = 0; b0 < batch; b0 += per) {
        const int B = batch - b0 < per ? batch - b0 : per;
        const size_t rows = (size_t)B * seq_len, off = (size_t)b0 * seq_len;
        if (e2cu_cuda(cudaMemcpyAsync(t->ids, ids + off, sizeof(int32_t) * rows, cudaMemcpyHostToDevice, st), "ids") ||
            (valid && e2cu_cuda(cudaMemcpyAsync(t->valid, valid + off, rows, cudaMemcpyHostToDevice, st), "valid")) ||
            pass(t, B, seq_len, valid != NULL, st) ||
            e2cu_cuda(cudaMemcpyAsync(out + (size_t)b0 * t->DO, t->pooled, sizeof(float) * (size_t)B * t->DO,
                                      cudaMemcpyDeviceToHost, st),
                      "out") ||
            e2cuda_check(st))
            return -1;
    }
    t->calls++;
    t->last_ms = now_ms() - t0;
    return 0;
}

int e2cuda_text_embed(e2cuda_text *t, const int32_t *ids, int n_ids, float *out) {
    return e2cuda_text_embed_batch(t, ids, NULL, 1, n_ids, out);
}

int e2cuda_text_stats(e2cuda_text *t, long *calls, long *kernels_last, double *last_ms) {
    if (!t) {
        e2cu_err("text_stats: null text tower");
        return -1;
    }
    if (calls) *calls = t->calls;
    if (kernels_last) *kernels_last = t->kernels_last;
    if (last_ms) *last_ms = t->last_ms;
    return 0;
}

/* sizes of the description structures, for binding layers that mirror them (not part of the ABI) */
void e2c_text_struct_sizes(int *desc, int *layer) {
    *desc = (int)sizeof(e2cuda_text_desc);
    *layer = (int)sizeof(e2cuda_text_layer);
}
