/* encoder.c — the config-1 FFN block and the config-2 synthetic encoder, composed from a kernel
 * table. TEST INFRASTRUCTURE ONLY (parity oracle and timed CPU baseline).
 *
 * The layer recipe is the reference text tower's, src/text.c:939-961, minus the PLE block and the
 * layer scalar (the synthetic model has neither), with the config-2 head (mean pool, dense
 * hidden->dense_hidden->out_dim, L2) in place of the reference's final projection + pool:
 *
 *   norm_split(x, res, input_ln)                  text.c:944
 *   q|k|v = int8 GEMM(quant(x))                   text.c:827-833 (gemm_segs: one quantisation)
 *   rmsnorm q (q_norm), k (k_norm), v (no scale)  text.c:836-838
 *   rope q, k; attention per sequence             text.c:842-886
 *   tmp = int8 GEMM(quant(ctx)) (o_proj)          text.c:890
 *   norm_add(x, tmp, res, post_attn_ln)           text.c:947
 *   norm_split(x, res, pre_ffn_ln)                text.c:950
 *   g|u = int8 GEMM(quant(x)); quant(gelu(g)*u)   text.c:893-903, gate_quant :424-468
 *   tmp = int8 GEMM (down); norm_add(post_ffn_ln) text.c:954
 *
 * Work is split like the reference's pool regions: GEMMs by 16-aligned column claims
 * (src/text.c:277-411), attention by (sequence, head, 32-query block), row ops by row chunks.
 */
#include "e2_oracle.h"

#include <math.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ parallel helpers */
typedef void (*item_fn)(void *ctx, int i0, int i1);

struct claim_task {
    item_fn fn;
    void *ctx;
    int n, grain;
    _Atomic int next;
};

static void claim_worker(void *arg, int tid, int nthreads) {
    struct claim_task *t = arg;
    (void)tid;
    (void)nthreads;
    for (;;) {
        const int i0 = atomic_fetch_add_explicit(&t->next, t->grain, memory_order_relaxed);
        if (i0 >= t->n) break;
        const int i1 = i0 + t->grain < t->n ? i0 + t->grain : t->n;
        t->fn(t->ctx, i0, i1);
    }
}

static void par_for(const e2o_kernels *k, int n, int grain, item_fn fn, void *ctx) {
    if (n <= 0) return;
    if (grain < 1) grain = 1;
    struct claim_task t;
    t.fn = fn;
    t.ctx = ctx;
    t.n = n;
    t.grain = grain;
    atomic_init(&t.next, 0);
    if (k->parallel && k->nthreads > 1 && n > grain) k->parallel(claim_worker, &t);
    else claim_worker(&t, 0, 1);
}

static int rows_grain(const e2o_kernels *k, int rows) {
    int g = rows / (4 * (k->nthreads > 0 ? k->nthreads : 1));
    if (g < 1) g = 1;
    if (g > 64) g = 64;
    return g;
}

/* activation scale blocks per row of width K (ablk 0: per-row) */
static int nblk(const e2o_kernels *k, int K) { return k->ablk ? (K + k->ablk - 1) / k->ablk : 1; }
static int ablk_ok(const e2o_kernels *k, int K) { return k->ablk == 0 || K % k->ablk == 0; }

/* quantise rows [i0,i1) of x */
struct quant_ctx {
    const e2o_kernels *k;
    int8_t *q;
    float *s;
    const float *x;
    int K, nb;
};
static void quant_items(void *c, int i0, int i1) {
    struct quant_ctx *q = c;
    q->k->quantize(q->q + (size_t)i0 * q->K, q->s + (size_t)i0 * q->nb, q->x + (size_t)i0 * q->K,
                   i1 - i0, q->K, -INFINITY, INFINITY);
}
static void par_quantize(const e2o_kernels *k, int8_t *q, float *s, const float *x, int M, int K) {
    struct quant_ctx c = { k, q, s, x, K, nblk(k, K) };
    par_for(k, M, rows_grain(k, M) < 16 ? rows_grain(k, M) : 16, quant_items, &c);
}

/* column claims of one or more GEMMs that share their quantised input */
struct gemm_ctx {
    const e2o_kernels *k;
    const int8_t *qa;
    const float *as;
    int M, nseg;
    float *y[4];
    const e2o_q8w *w[4];
};
static void gemm_items(void *c, int a, int b) {
    struct gemm_ctx *g = c;
    int off = 0;
    for (int s = 0; s < g->nseg && off < b; s++) {
        const int n = g->w[s]->N;
        const int n0 = a > off ? a - off : 0;
        const int n1 = b - off < n ? b - off : n;
        if (n1 > n0) g->k->gemm(g->y[s], g->qa, g->as, g->w[s], g->M, n, n0, n1);
        off += n;
    }
}
static void par_gemm(const e2o_kernels *k, const int8_t *qa, const float *as, int M, int nseg,
                     float *const *y, const e2o_q8w *const *w) {
    struct gemm_ctx g;
    memset(&g, 0, sizeof g);
    g.k = k;
    g.qa = qa;
    g.as = as;
    g.M = M;
    g.nseg = nseg;
    int total = 0;
    for (int s = 0; s < nseg; s++) {
        g.y[s] = y[s];
        g.w[s] = w[s];
        total += w[s]->N;
    }
    /* src/text.c:393-405: tiles of 16..64 columns, 16-aligned */
    int tile = total / (4 * (k->nthreads > 0 ? k->nthreads : 1));
    if (tile > 64) tile = 64;
    tile = (tile + 15) & ~15;
    if (tile < 16) tile = 16;
    par_for(k, total, tile, gemm_items, &g);
}

enum { OP_RMS, OP_SPLIT, OP_ADD, OP_GELU_MUL };
struct row_ctx {
    const e2o_kernels *k;
    int op, D, stride;
    float *a;
    float *b;
    const float *c, *gamma;
    float eps;
};
static void row_items(void *cv, int i0, int i1) {
    struct row_ctx *r = cv;
    const size_t o = (size_t)i0 * r->D;
    switch (r->op) {
    case OP_RMS: r->k->rmsnorm(r->a + o, i1 - i0, r->D, r->gamma, r->eps); break;
    case OP_SPLIT: r->k->norm_split(r->a + o, r->b + o, i1 - i0, r->D, r->gamma, r->eps); break;
    case OP_ADD: r->k->norm_add(r->a + o, r->c + o, r->b + o, i1 - i0, r->D, r->gamma, r->eps); break;
    case OP_GELU_MUL:
        /* src/text.c:424-447: gelu over the rows, times up (row stride `stride`) */
        r->k->gelu_tanh(r->a + o, (size_t)(i1 - i0) * r->D);
        for (int i = i0; i < i1; i++)
            r->k->mul(r->a + (size_t)i * r->D, r->c + (size_t)i * r->stride, (size_t)r->D);
        break;
    }
}
static void par_rows(const e2o_kernels *k, int op, int rows, int D, float *a, float *b, const float *c,
                     const float *gamma, float eps, int stride) {
    struct row_ctx r = { k, op, D, stride, a, b, c, gamma, eps };
    par_for(k, rows, rows_grain(k, rows), row_items, &r);
}

/* ------------------------------------------------------------------ FFN block (config 1) */
int e2o_ffn_block(const e2o_kernels *k, const float *x, int M, int D, int I, const float *gamma,
                  float eps, const e2o_q8w *wg, const e2o_q8w *wu, const e2o_q8w *wd, float *y,
                  int8_t *xq, float *xs, int8_t *hq, float *hs, float *gu) {
    if (M <= 0 || !ablk_ok(k, D) || !ablk_ok(k, I)) return -1;
    const int nbD = nblk(k, D), nbI = nblk(k, I);
    float *xn = malloc(sizeof(float) * (size_t)M * D);
    float *res = malloc(sizeof(float) * (size_t)M * D);
    float *g = malloc(sizeof(float) * (size_t)M * I);
    float *u = malloc(sizeof(float) * (size_t)M * I);
    int8_t *qa = malloc((size_t)M * (D > I ? D : I));
    float *as = malloc(sizeof(float) * (size_t)M * (nbD > nbI ? nbD : nbI));
    if (!xn || !res || !g || !u || !qa || !as) {
        free(xn); free(res); free(g); free(u); free(qa); free(as);
        return -1;
    }
    memcpy(xn, x, sizeof(float) * (size_t)M * D);
    par_rows(k, OP_SPLIT, M, D, xn, res, NULL, gamma, eps, 0);
    par_quantize(k, qa, as, xn, M, D);
    if (xq) memcpy(xq, qa, (size_t)M * D);
    if (xs) memcpy(xs, as, sizeof(float) * (size_t)M * nbD);
    {
        float *ys[2] = { g, u };
        const e2o_q8w *ws[2] = { wg, wu };
        par_gemm(k, qa, as, M, 2, ys, ws);
    }
    if (gu)
        for (int m = 0; m < M; m++) {
            memcpy(gu + (size_t)m * 2 * I, g + (size_t)m * I, sizeof(float) * I);
            memcpy(gu + (size_t)m * 2 * I + I, u + (size_t)m * I, sizeof(float) * I);
        }
    par_rows(k, OP_GELU_MUL, M, I, g, NULL, u, NULL, 0.f, I);
    par_quantize(k, qa, as, g, M, I);
    if (hq) memcpy(hq, qa, (size_t)M * I);
    if (hs) memcpy(hs, as, sizeof(float) * (size_t)M * nbI);
    {
        float *ys[1] = { y };
        const e2o_q8w *ws[1] = { wd };
        par_gemm(k, qa, as, M, 1, ys, ws);
    }
    /* config 1: plain residual add (the encoder uses norm_add instead) */
    for (size_t i = 0; i < (size_t)M * D; i++) y[i] += res[i];
    free(xn); free(res); free(g); free(u); free(qa); free(as);
    return 0;
}

/* ------------------------------------------------------------------ attention */
struct attn_ctx {
    const e2o_kernels *k;
    const float *q, *kk, *v;
    float *ctx;
    const uint8_t *valid;
    int S, H, KV, D, nblk;
    float scale;
    float *scratch; /* per-thread: [32][S] logits + [D][S] K^T share per call (allocated by caller) */
    float *kt;      /* [KV][D][S] transposed keys, valid keys compacted */
    float *vc;      /* [KV][S][D] values, valid keys compacted */
    int nvalid;
    _Atomic int slot;
};

#define ATT_BQ 32 /* src/model.h:62 E2_ATT_BQ */

static void attn_items(void *cv, int i0, int i1) {
    struct attn_ctx *a = cv;
    const int S = a->S, D = a->D, GD = a->H * D, KVD = a->KV * D, nv = a->nvalid;
    const int slot = atomic_fetch_add_explicit(&a->slot, 1, memory_order_relaxed);
    float *sc = a->scratch + (size_t)slot * (ATT_BQ * (size_t)S + (size_t)ATT_BQ * D);
    float *qs = sc + (size_t)ATT_BQ * S;
    for (int it = i0; it < i1; it++) {
        const int h = it / a->nblk, blk = it - h * a->nblk;
        const int m0 = blk * ATT_BQ;
        const int rows = S - m0 < ATT_BQ ? S - m0 : ATT_BQ;
        const int kvh = h / (a->H / a->KV);
        /* scaled queries of this block: logits = (scale q) . k */
        for (int i = 0; i < rows; i++)
            for (int d = 0; d < D; d++)
                qs[(size_t)i * D + d] = a->q[(size_t)(m0 + i) * GD + (size_t)h * D + d] * a->scale;
        if (nv > 0)
            a->k->sgemm_nn(sc, nv, qs, D, a->kt + (size_t)kvh * D * S, S, rows, nv, D, 0, rows);
        for (int i = 0; i < rows; i++) {
            float *o = a->ctx + (size_t)(m0 + i) * GD + (size_t)h * D;
            if ((a->valid && !a->valid[m0 + i]) || nv == 0) {
                memset(o, 0, sizeof(float) * D);
                continue;
            }
            a->k->softmax(sc + (size_t)i * nv, nv);
            a->k->sgemm_nn(o, GD, sc + (size_t)i * nv, nv, a->vc + (size_t)kvh * S * D, D, 1, D, nv,
                           0, 1);
        }
        (void)KVD;
    }
}

void e2o_attention_f32(const e2o_kernels *k, const float *q, const float *kk, const float *v,
                       float *ctx, const uint8_t *valid, int S, int H, int KV, int D, float scale) {
    struct attn_ctx a;
    memset(&a, 0, sizeof a);
    a.k = k;
    a.q = q;
    a.kk = kk;
    a.v = v;
    a.ctx = ctx;
    a.valid = valid;
    a.S = S;
    a.H = H;
    a.KV = KV;
    a.D = D;
    a.scale = scale;
    a.nblk = (S + ATT_BQ - 1) / ATT_BQ;
    const int KVD = KV * D;
    const int nt = k->nthreads > 0 ? k->nthreads : 1;
    a.kt = malloc(sizeof(float) * (size_t)KV * D * S);
    a.vc = malloc(sizeof(float) * (size_t)KV * S * D);
    /* every claim takes a fresh slot; claims <= items */
    const int items = H * a.nblk;
    a.scratch = malloc(sizeof(float) * (size_t)(items + nt) * (ATT_BQ * (size_t)S + ATT_BQ * (size_t)D));
    if (!a.kt || !a.vc || !a.scratch) {
        free(a.kt); free(a.vc); free(a.scratch);
        return;
    }
    int nv = 0;
    for (int j = 0; j < S; j++) {
        if (valid && !valid[j]) continue;
        for (int h = 0; h < KV; h++)
            for (int d = 0; d < D; d++) {
                a.kt[((size_t)h * D + d) * S + nv] = kk[(size_t)j * KVD + (size_t)h * D + d];
                a.vc[((size_t)h * S + nv) * D + d] = v[(size_t)j * KVD + (size_t)h * D + d];
            }
        nv++;
    }
    a.nvalid = nv;
    atomic_init(&a.slot, 0);
    par_for(k, items, 1, attn_items, &a);
    free(a.kt);
    free(a.vc);
    free(a.scratch);
}

/* ------------------------------------------------------------------ encoder (config 2) */
int e2o_encoder_forward(const e2o_kernels *k, const e2o_encoder *e, const int32_t *ids,
                        const uint8_t *valid, int B, int S, float *out, float *last_hidden,
                        float *layer0) {
    const int D = e->hidden, H = e->n_heads, KV = e->n_kv_heads, Dh = e->head_dim, I = e->ffn;
    const int GD = H * Dh, KVD = KV * Dh, M = B * S;
    if (B <= 0 || S <= 0 || !ablk_ok(k, D) || !ablk_ok(k, I) || !ablk_ok(k, GD) ||
        !ablk_ok(k, e->dense_hidden) || H % KV)
        return -1;
    for (size_t i = 0; i < (size_t)M; i++)
        if (ids[i] < 0 || ids[i] >= e->vocab) return -1;
    const int KQ = D > I ? (D > GD ? D : GD) : (I > GD ? I : GD);
    float *x = malloc(sizeof(float) * (size_t)M * D);
    float *res = malloc(sizeof(float) * (size_t)M * D);
    float *tmp = malloc(sizeof(float) * (size_t)M * D);
    float *q = malloc(sizeof(float) * (size_t)M * GD);
    float *kk = malloc(sizeof(float) * (size_t)M * KVD);
    float *v = malloc(sizeof(float) * (size_t)M * KVD);
    float *ctx = malloc(sizeof(float) * (size_t)M * GD);
    float *g = malloc(sizeof(float) * (size_t)M * I);
    float *u = malloc(sizeof(float) * (size_t)M * I);
    int8_t *qa = malloc((size_t)M * KQ);
    float *as = malloc(sizeof(float) * (size_t)M * (KQ / 16));
    float *cs = malloc(sizeof(float) * (size_t)S * Dh);
    float *sn = malloc(sizeof(float) * (size_t)S * Dh);
    int rc = -1;
    if (!x || !res || !tmp || !q || !kk || !v || !ctx || !g || !u || !qa || !as || !cs || !sn)
        goto done;
    e2o_rope_tables(cs, sn, S, Dh, e->rope_theta);

    /* token gather: int8 row x row scale x embed_scale (F7) */
    for (int i = 0; i < M; i++) {
        const int8_t *tr = e->table + (size_t)ids[i] * D;
        const float ts = e->table_scale[ids[i]];
        for (int d = 0; d < D; d++) x[(size_t)i * D + d] = ((float)tr[d] * ts) * e->embed_scale;
    }

    for (int l = 0; l < e->n_layers; l++) {
        par_rows(k, OP_SPLIT, M, D, x, res, NULL, e->input_ln[l], e->eps, 0);
        par_quantize(k, qa, as, x, M, D);
        {
            float *ys[3] = { q, kk, v };
            const e2o_q8w *ws[3] = { &e->wq[l], &e->wk[l], &e->wv[l] };
            par_gemm(k, qa, as, M, 3, ys, ws);
        }
        par_rows(k, OP_RMS, M * H, Dh, q, NULL, NULL, e->q_norm[l], e->eps, 0);
        par_rows(k, OP_RMS, M * KV, Dh, kk, NULL, NULL, e->k_norm[l], e->eps, 0);
        par_rows(k, OP_RMS, M * KV, Dh, v, NULL, NULL, NULL, e->eps, 0);
        for (int b = 0; b < B; b++) {
            float *qb = q + (size_t)b * S * GD, *kb = kk + (size_t)b * S * KVD;
            k->rope_rows(qb, 0, S * H, H, Dh, Dh, cs, sn);
            k->rope_rows(kb, 0, S * KV, KV, Dh, Dh, cs, sn);
            e2o_attention_f32(k, qb, kb, v + (size_t)b * S * KVD, ctx + (size_t)b * S * GD,
                              valid ? valid + (size_t)b * S : NULL, S, H, KV, Dh, e->attn_scale);
        }
        par_quantize(k, qa, as, ctx, M, GD);
        {
            float *ys[1] = { tmp };
            const e2o_q8w *ws[1] = { &e->wo[l] };
            par_gemm(k, qa, as, M, 1, ys, ws);
        }
        par_rows(k, OP_ADD, M, D, x, res, tmp, e->post_attn_ln[l], e->eps, 0);
        par_rows(k, OP_SPLIT, M, D, x, res, NULL, e->pre_ffn_ln[l], e->eps, 0);
        par_quantize(k, qa, as, x, M, D);
        {
            float *ys[2] = { g, u };
            const e2o_q8w *ws[2] = { &e->wg[l], &e->wu[l] };
            par_gemm(k, qa, as, M, 2, ys, ws);
        }
        par_rows(k, OP_GELU_MUL, M, I, g, NULL, u, NULL, 0.f, I);
        par_quantize(k, qa, as, g, M, I);
        {
            float *ys[1] = { tmp };
            const e2o_q8w *ws[1] = { &e->wd[l] };
            par_gemm(k, qa, as, M, 1, ys, ws);
        }
        par_rows(k, OP_ADD, M, D, x, res, tmp, e->post_ffn_ln[l], e->eps, 0);
        if (l == 0 && layer0) memcpy(layer0, x, sizeof(float) * (size_t)M * D);
    }
    par_rows(k, OP_RMS, M, D, x, NULL, NULL, e->final_norm, e->eps, 0);
    if (last_hidden) memcpy(last_hidden, x, sizeof(float) * (size_t)M * D);

    /* head: masked mean pool -> dense -> dense -> L2 (all-invalid sequence -> exact zero) */
    {
        const int DH = e->dense_hidden, DO = e->out_dim;
        float *pooled = malloc(sizeof(float) * (size_t)B * D);
        float *h1 = malloc(sizeof(float) * (size_t)B * DH);
        int8_t *pq = malloc((size_t)B * (DH > D ? DH : D));
        float *ps = malloc(sizeof(float) * (size_t)B * ((DH > D ? DH : D) / 16));
        if (!pooled || !h1 || !pq || !ps) {
            free(pooled); free(h1); free(pq); free(ps);
            goto done;
        }
        for (int b = 0; b < B; b++)
            k->meanpool(pooled + (size_t)b * D, x + (size_t)b * S * D, S, D,
                        valid ? valid + (size_t)b * S : NULL);
        k->quantize(pq, ps, pooled, B, D, -INFINITY, INFINITY);
        k->gemm(h1, pq, ps, e->dense1, B, DH, 0, DH);
        k->quantize(pq, ps, h1, B, DH, -INFINITY, INFINITY);
        k->gemm(out, pq, ps, e->dense2, B, DO, 0, DO);
        for (int b = 0; b < B; b++) {
            int any = 1;
            if (valid) {
                any = 0;
                for (int i = 0; i < S; i++) any |= valid[(size_t)b * S + i];
            }
            if (any) k->l2norm(out + (size_t)b * DO, DO);
            else memset(out + (size_t)b * DO, 0, sizeof(float) * DO);
        }
        free(pooled); free(h1); free(pq); free(ps);
    }
    rc = 0;
done:
    free(x); free(res); free(tmp); free(q); free(kk); free(v); free(ctx); free(g); free(u);
    free(qa); free(as); free(cs); free(sn);
    return rc;
}
