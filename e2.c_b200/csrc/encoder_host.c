/* encoder_host.c — the synthetic encoder (config 2) over the e2cuda kernels: weights uploaded once,
 * one device pass per chunk of whole sequences, replayed from a CUDA graph per shape.
 *
 * Layer recipe: e2.c src/text.c:939-961 without the PLE block; head: masked mean pool -> dense ->
 * dense -> L2 (the config-2 head). Per layer:
 *
 *   [prev tail] norm_add + norm_split + quant      (layer 0: embed gather + norm + quant)
 *   GEMM q|k|v  -> per-head RMSNorm + RoPE -> bf16 Q, K, V^T     (epilogue, gemm_i8.cu)
 *   attention   -> ctx fp32                                       (attention.cu)
 *   quant ctx ; GEMM o_proj + norm_add(post_attn) + norm_split(pre_ffn) + quant
 *   GEMM gate|up -> GELU(g)*u (epilogue) ; quant h
 *   GEMM down + norm_add(post_ffn) + norm_split(next input_ln) + quant   (last layer: final norm)
 *
 * With per-token scales and a hidden size of 128 x (1..8) the residual norms run in the o_proj and
 * down GEMMs' epilogue (whole rows per cluster of CTAs), and with an FFN width of 128 x (1..16) h's
 * quantiser runs in the gate|up GEMM's epilogue (6 kernels per layer). With per-128-block scales
 * the same six: the q|k|v finish, the residual norms and h's quantiser run in the GEMMs'
 * epilogues with the per-block fold, the int8 outputs quantised per 128-column block.
 *
 * int8 activations alternate between two buffers: the layer's input (and the fused tails' output)
 * in qb, the quantised ctx and h in qa. A fused tail writes int8 rows of its output while other CTAs
 * still read the GEMM's input rows, so the two must never be the same buffer.
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "internal.h"

#define MAX_GRAPHS 128

typedef struct {
    int B, S, has_valid;
    cudaGraphExec_t exec;
    int kernels;
} graph_slot;

struct e2cuda_encoder {
    int L, D, H, Dh, I, V, DH, DO, max_seq, ablk, max_tokens;
    float eps, attn_scale, embed_scale;
    e2cuda_w8 *wqkv, *wo, *wgu, *wd;
    e2cuda_w8 dense1, dense2;
    int8_t *table;
    float *table_scale;
    float *norms; /* per layer: input, post_attn, pre_ffn, post_ffn [D] + q_norm, k_norm [Dh]; then final [D] */
    float *rope_cos, *rope_sin;
    float *rope_cos_pm, *rope_sin_pm; /* per-128-block mode: the same tables position-major [max_seq][Dh/2] */
    /* workspace */
    int32_t *ids;
    uint8_t *valid;
    float *out, *res, *tmp, *ctx, *h, *pooled, *h1;
    float *qkvf, *guf; /* per-128-block mode only: the q|k|v and gate|up GEMMs' fp32 outputs */
    int8_t *qa, *qb, *pq;
    float *qs, *qsb, *ps;
    int fused_norm, fused_gelu, fused_qkv;
    void *Q, *K, *Vt;
    size_t vt_bytes;
    int *status;
    int *gws;          /* workspace of the weight-streaming GEMM (the head's short GEMMs) */
    size_t gws_bytes;
    int gws_rows, gws_gen;
    cudaStream_t stream;
    float *host_out;
    graph_slot graphs[MAX_GRAPHS];
    int ngraphs;
    long calls, kernels_last;
    double last_ms;
};

static size_t norm_stride(const e2cuda_encoder *e) { return (size_t)4 * e->D + 2 * (size_t)e->Dh; }
static float *nrm(const e2cuda_encoder *e, int l, int which) {
    float *b = e->norms + (size_t)l * norm_stride(e);
    return which < 4 ? b + (size_t)which * e->D : b + 4 * (size_t)e->D + (size_t)(which - 4) * e->Dh;
}
static float *final_norm(const e2cuda_encoder *e) { return e->norms + (size_t)e->L * norm_stride(e); }

/* concatenate projections (rows) into one device weight */
static int upload_concat(const e2cuda_q8w *const *parts, int nparts, e2cuda_w8 *out) {
    int N = 0;
    const int K = parts[0]->K;
    for (int i = 0; i < nparts; i++) {
        if (parts[i]->K != K) {
            e2cu_err("encoder: projections to concatenate differ in K");
            return -1;
        }
        N += parts[i]->N;
    }
    int8_t *w = malloc((size_t)N * K);
    float *s = malloc(sizeof(float) * (size_t)N);
    if (!w || !s) {
        free(w);
        free(s);
        e2cu_err("encoder: out of host memory");
        return -1;
    }
    int off = 0;
    for (int i = 0; i < nparts; i++) {
        e2cu_unpack_q8w(parts[i], w + (size_t)off * K, K);
        memcpy(s + off, parts[i]->scale, sizeof(float) * parts[i]->N);
        off += parts[i]->N;
    }
    const int rc = e2cuda_w8_from_int8(w, s, N, K, out);
    free(w);
    free(s);
    return rc;
}

void e2cuda_encoder_destroy(e2cuda_encoder *e) {
    if (!e) return;
    for (int i = 0; i < e->ngraphs; i++) cudaGraphExecDestroy(e->graphs[i].exec);
    for (int l = 0; l < e->L; l++) {
        if (e->wqkv) e2cuda_w8_free(&e->wqkv[l]);
        if (e->wo) e2cuda_w8_free(&e->wo[l]);
        if (e->wgu) e2cuda_w8_free(&e->wgu[l]);
        if (e->wd) e2cuda_w8_free(&e->wd[l]);
    }
    free(e->wqkv);
    free(e->wo);
    free(e->wgu);
    free(e->wd);
    e2cuda_w8_free(&e->dense1);
    e2cuda_w8_free(&e->dense2);
    void *dev[] = { e->table, e->table_scale, e->norms, e->rope_cos, e->rope_sin, e->ids, e->valid, e->out, e->res,
                    e->tmp, e->ctx, e->h, e->pooled, e->h1, e->qa, e->qb, e->pq, e->qs, e->qsb, e->ps, e->Q, e->K,
                    e->Vt, e->gws, e->qkvf, e->guf, e->rope_cos_pm, e->rope_sin_pm };
    for (size_t i = 0; i < sizeof dev / sizeof dev[0]; i++)
        if (dev[i]) cudaFree(dev[i]);
    if (e->host_out) cudaFreeHost(e->host_out);
    if (e->stream) cudaStreamDestroy(e->stream);
    free(e);
}

#define DALLOC(ptr, bytes) e2cu_cuda(cudaMalloc((void **)&(ptr), (bytes)), "encoder alloc " #ptr)

e2cuda_encoder *e2cuda_encoder_create(const e2cuda_encoder_desc *d, int max_tokens) {
    if (!d || d->n_layers <= 0 || d->head_dim != 256 || d->n_kv_heads != 1 || d->hidden % 128 || d->hidden > 1024 ||
        d->n_heads <= 0 || d->ffn % 128 || d->vocab <= 0 || d->max_seq <= 0 || max_tokens <= 0 || !d->table ||
        !d->table_scale || d->dense_hidden % 128 || d->out_dim <= 0) {
        e2cu_err("encoder_create: unsupported geometry (needs head_dim 256, one KV head, hidden and ffn multiples "
                 "of 128, hidden <= 1024)");
        return NULL;
    }
    const int ablk = d->ablk ? d->ablk : d->hidden;
    if (ablk != d->hidden && ablk != 128) {
        e2cu_err("encoder_create: ablk must be hidden (per token) or 128");
        return NULL;
    }
    e2cuda_encoder *e = calloc(1, sizeof *e);
    if (!e) {
        e2cu_err("encoder_create: out of host memory");
        return NULL;
    }
    e->L = d->n_layers;
    e->D = d->hidden;
    e->H = d->n_heads;
    e->Dh = d->head_dim;
    e->I = d->ffn;
    e->V = d->vocab;
    e->DH = d->dense_hidden;
    e->DO = d->out_dim;
    e->max_seq = d->max_seq;
    e->ablk = ablk;
    e->max_tokens = max_tokens;
    e->eps = d->eps;
    e->attn_scale = d->attn_scale;
    e->embed_scale = d->embed_scale;
    const int L = e->L, D = e->D, GD = e->H * e->Dh;
    const size_t M = (size_t)max_tokens;

    e->wqkv = calloc((size_t)L, sizeof(e2cuda_w8));
    e->wo = calloc((size_t)L, sizeof(e2cuda_w8));
    e->wgu = calloc((size_t)L, sizeof(e2cuda_w8));
    e->wd = calloc((size_t)L, sizeof(e2cuda_w8));
    if (!e->wqkv || !e->wo || !e->wgu || !e->wd) {
        e2cu_err("encoder_create: out of host memory");
        goto fail;
    }
    for (int l = 0; l < L; l++) {
        const e2cuda_q8w *parts[3] = { &d->wq[l], &d->wk[l], &d->wv[l] };
        if (d->wq[l].N != GD || d->wk[l].N != e->Dh || d->wv[l].N != e->Dh || d->wq[l].K != D || d->wo[l].N != D ||
            d->wo[l].K != GD || d->wg[l].N != e->I || d->wd[l].K != e->I || d->wd[l].N != D) {
            e2cu_err("encoder_create: layer %d projection shapes do not match the geometry", l);
            goto fail;
        }
        if (upload_concat(parts, 3, &e->wqkv[l]) || e2cuda_w8_from_q8w(&d->wo[l], &e->wo[l]) ||
            e2cu_upload_gate_up(&d->wg[l], &d->wu[l], &e->wgu[l]) || e2cuda_w8_from_q8w(&d->wd[l], &e->wd[l]))
            goto fail;
    }
    if (d->dense1->K != D || d->dense1->N != e->DH || d->dense2->K != e->DH || d->dense2->N != e->DO) {
        e2cu_err("encoder_create: head shapes do not match");
        goto fail;
    }
    if (e2cuda_w8_from_q8w(d->dense1, &e->dense1) || e2cuda_w8_from_q8w(d->dense2, &e->dense2)) goto fail;

    /* token table, norms, RoPE tables */
    if (DALLOC(e->table, (size_t)e->V * D) || DALLOC(e->table_scale, sizeof(float) * (size_t)e->V) ||
        e2cu_cuda(cudaMemcpy(e->table, d->table, (size_t)e->V * D, cudaMemcpyHostToDevice), "table upload") ||
        e2cu_cuda(cudaMemcpy(e->table_scale, d->table_scale, sizeof(float) * e->V, cudaMemcpyHostToDevice),
                  "table upload"))
        goto fail;
    {
        const size_t nn = (size_t)L * norm_stride(e) + D;
        float *hn = malloc(sizeof(float) * nn);
        if (!hn) {
            e2cu_err("encoder_create: out of host memory");
            goto fail;
        }
        for (int l = 0; l < L; l++) {
            float *b = hn + (size_t)l * norm_stride(e);
            memcpy(b, d->input_ln[l], sizeof(float) * D);
            memcpy(b + D, d->post_attn_ln[l], sizeof(float) * D);
            memcpy(b + 2 * D, d->pre_ffn_ln[l], sizeof(float) * D);
            memcpy(b + 3 * D, d->post_ffn_ln[l], sizeof(float) * D);
            memcpy(b + 4 * D, d->q_norm[l], sizeof(float) * e->Dh);
            memcpy(b + 4 * D + e->Dh, d->k_norm[l], sizeof(float) * e->Dh);
        }
        memcpy(hn + (size_t)L * norm_stride(e), d->final_norm, sizeof(float) * D);
        const int rc = DALLOC(e->norms, sizeof(float) * nn) ||
                       e2cu_cuda(cudaMemcpy(e->norms, hn, sizeof(float) * nn, cudaMemcpyHostToDevice), "norm upload");
        free(hn);
        if (rc) goto fail;
    }
    {
        /* e2.c src/text.c:483-506: inv = 1/theta^(2i/D), angle = pos * inv; halves duplicated there,
         * stored once here, pair-major ([Dh/2][max_seq]) so the QKV epilogue reads a warp's 32
         * positions of one pair in one line */
        const int half = e->Dh / 2;
        float *c = malloc(sizeof(float) * (size_t)e->max_seq * half), *s = malloc(sizeof(float) * (size_t)e->max_seq * half);
        if (!c || !s) {
            free(c);
            free(s);
            e2cu_err("encoder_create: out of host memory");
            goto fail;
        }
        for (int p = 0; p < e->max_seq; p++)
            for (int i = 0; i < half; i++) {
                const float inv = 1.0f / powf(d->rope_theta, (float)(2 * i) / (float)e->Dh);
                const float f = (float)p * inv;
                c[(size_t)i * e->max_seq + p] = cosf(f);
                s[(size_t)i * e->max_seq + p] = sinf(f);
            }
        const size_t nb = sizeof(float) * (size_t)e->max_seq * half;
        int rc = DALLOC(e->rope_cos, nb) || DALLOC(e->rope_sin, nb) ||
                 e2cu_cuda(cudaMemcpy(e->rope_cos, c, nb, cudaMemcpyHostToDevice), "rope upload") ||
                 e2cu_cuda(cudaMemcpy(e->rope_sin, s, nb, cudaMemcpyHostToDevice), "rope upload");
        if (!rc && e->ablk != D) {
            /* per-block mode's q|k|v epilogue reads a lane's (one position's) pairs in 16-byte runs */
            float *ct = malloc(nb), *st = malloc(nb);
            if (!ct || !st) {
                e2cu_err("encoder_create: out of host memory");
                rc = 1;
            } else {
                for (int p = 0; p < e->max_seq; p++)
                    for (int i = 0; i < half; i++) {
                        ct[(size_t)p * half + i] = c[(size_t)i * e->max_seq + p];
                        st[(size_t)p * half + i] = s[(size_t)i * e->max_seq + p];
                    }
                rc = DALLOC(e->rope_cos_pm, nb) || DALLOC(e->rope_sin_pm, nb) ||
                     e2cu_cuda(cudaMemcpy(e->rope_cos_pm, ct, nb, cudaMemcpyHostToDevice), "rope upload") ||
                     e2cu_cuda(cudaMemcpy(e->rope_sin_pm, st, nb, cudaMemcpyHostToDevice), "rope upload");
            }
            free(ct);
            free(st);
        }
        free(c);
        free(s);
        if (rc) goto fail;
    }
    /* workspace; the widest activation row is max(D, GD, I) */
    {
        int KQ = D > GD ? D : GD;
        if (e->I > KQ) KQ = e->I;
        const size_t MB = M; /* at most one sequence per token */
        if (DALLOC(e->ids, sizeof(int32_t) * M) || DALLOC(e->valid, M) || DALLOC(e->res, sizeof(float) * M * D) ||
            DALLOC(e->tmp, sizeof(float) * M * D) || DALLOC(e->ctx, sizeof(float) * M * GD) ||
            DALLOC(e->h, sizeof(float) * M * e->I) || DALLOC(e->qa, M * (size_t)KQ) ||
            DALLOC(e->qs, sizeof(float) * M * (size_t)(KQ / 128 + 1)) || DALLOC(e->qb, M * (size_t)D) ||
            DALLOC(e->qsb, sizeof(float) * M * (size_t)(D / 128 + 1)) || DALLOC(e->Q, 2 * M * GD) ||
            DALLOC(e->K, 2 * M * e->Dh) || DALLOC(e->out, sizeof(float) * MB * e->DO) ||
            DALLOC(e->pooled, sizeof(float) * MB * D) || DALLOC(e->h1, sizeof(float) * MB * e->DH) ||
            DALLOC(e->pq, MB * (size_t)(e->DH > D ? e->DH : D)) ||
            DALLOC(e->ps, sizeof(float) * MB * (size_t)((e->DH > D ? e->DH : D) / 128 + 1)))
            goto fail;
        /* per-128-block activation scales: the QKV epilogue needs whole-row (per-token) scales, so
         * that GEMM writes fp32 and a row kernel finishes it; the gate|up fp32 buffer serves the
         * two-kernel path (E2C_FUSED_GELU=0) */
        if (e->ablk != D && (DALLOC(e->qkvf, sizeof(float) * M * (size_t)(GD + 2 * e->Dh)) ||
                             DALLOC(e->guf, sizeof(float) * M * (size_t)(2 * e->I))))
            goto fail;
    }
    /* o_proj / down run with the residual norms in their epilogue (one launch instead of two, the
     * GEMM output never written; per-128-block scales: the per-block fold and a per-block quantiser)
     * where the shape allows; E2C_FUSED_NORM=0 selects the GEMM + row
     * kernel pair instead. */
    {
        const char *fz = getenv("E2C_FUSED_NORM");
        e->fused_norm = !(fz && fz[0] == '0') && D % 128 == 0 && D / 128 <= 8;
        /* gate|up runs with GELU-gate and h's quantiser in its epilogue (h never stored): per token
         * where the device holds a cluster of I / 128 CTAs, per 128-block in the per-block GEMM;
         * E2C_FUSED_GELU=0 selects the two-kernel paths instead */
        const char *fg = getenv("E2C_FUSED_GELU");
        e->fused_gelu = !(fg && fg[0] == '0') && e->I % 128 == 0 &&
                        (e->ablk == D ? e->I / 128 <= 16 && e2c_gemm_gelu_quant_supported(e->I / 128)
                                      : e->ablk == 128);
        /* per-block mode: q|k|v with the head finish in its epilogue (heads of 256);
         * E2C_FUSED_QKV=0 selects the GEMM + row kernel pair */
        const char *fq = getenv("E2C_FUSED_QKV");
        e->fused_qkv = !(fq && fq[0] == '0') && e->ablk != D && e->Dh == 256;
    }
    /* the head's GEMMs have one row per sequence: up to 256 of them run on the weight-streaming
     * kernel, whose workspace starts zeroed and is left zeroed by every launch that completes */
    e->gws_rows = M < 256 ? (int)M : 256;
    e->gws_bytes = e2c_gemm_ws_bytes(e->gws_rows);
    if (e->gws_bytes && (DALLOC(e->gws, e->gws_bytes) || e2cu_cuda(cudaMemset(e->gws, 0, e->gws_bytes), "workspace clear")))
        goto fail;
    if (!e->gws_bytes) e->gws_rows = 0;
    e->status = e2cu_status();
    if (!e->status || e2cu_cuda(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking), "stream")) goto fail;
    return e;
fail:
    e2cuda_encoder_destroy(e);
    return NULL;
}

static int round8(int x) { return (x + 7) & ~7; }

/* o_proj / down and the residual norms after them: res = rmsnorm(gemm) * g1 + res, then qb / qsb =
 * quantise(rmsnorm(res) * g2), or (g2 NULL, after the last layer) res = rmsnorm(res) * gf. Adds the
 * kernels queued to *n. */
static int gemm_norms(e2cuda_encoder *e, const e2cuda_w8 *w, int M, int ablk, const float *g1, const float *g2,
                      const float *gf, int *n, cudaStream_t st, const char *what) {
    const int D = e->D;
    e2c_gemm_args a;
    e2cu_gemm_args(&a, w, e->qa, e->qs, M, ablk);
    if (e->fused_norm) {
        a.epi = E2C_EPI_NORMADD;
        a.res = e->res;
        a.ldres = D;
        a.norm_g1 = g1;
        a.norm_g2 = g2;
        a.norm_gf = gf;
        a.q8 = g2 ? e->qb : NULL;
        a.ldq = D;
        a.q8_scale = g2 ? e->qsb : NULL;
        a.eps = e->eps;
        *n += 1;
        return e2cu_launch(e2c_gemm(&a, st), what);
    }
    a.epi = E2C_EPI_F32;
    a.y = e->tmp;
    a.ldy = D;
    *n += 2;
    return e2cu_launch(e2c_gemm(&a, st), what) ||
           e2cu_launch(e2c_norm_add_norm_quant(e->tmp, e->res, g1, g2, gf, e->eps, e->qb, e->qsb, M, D,
                                               e->ablk == D ? D : 128, st),
                       what);
}

/* queue one pass over B sequences of S tokens already in e->ids / e->valid; returns kernels queued */
static int encode(e2cuda_encoder *e, int B, int S, int has_valid, cudaStream_t st) {
    const int M = B * S, D = e->D, GD = e->H * e->Dh, I = e->I, L = e->L;
    const int ab_d = e->ablk == D ? D : 128, ab_gd = e->ablk == D ? GD : 128, ab_i = e->ablk == D ? I : 128;
    const int ldvt = round8(S);
    const uint8_t *valid = has_valid ? e->valid : NULL;
    int n = 0;
    if (e2cu_launch(e2c_embed_norm_quant(e->ids, e->table, e->table_scale, e->embed_scale, nrm(e, 0, 0), e->eps, e->res,
                                         e->qb, e->qsb, M, D, ab_d, e->V, e->status, st),
                    "encoder embed"))
        return -1;
    n++;
    e2c_gemm_args a;
    for (int l = 0; l < L; l++) {
        /* q|k|v with per-head RMSNorm + RoPE */
        e2cu_gemm_args(&a, &e->wqkv[l], e->qb, e->qsb, M, ab_d);
        if (e->fused_qkv) {
            a.epi = E2C_EPI_QKVPB;
            a.nq = e->H;
            a.q_out = e->Q;
            a.k_out = e->K;
            a.vt_out = e->Vt;
            a.ldvt = ldvt;
            a.seq_len = S;
            a.q_gamma = nrm(e, l, 4);
            a.k_gamma = nrm(e, l, 5);
            a.rope_cos = e->rope_cos_pm;
            a.rope_sin = e->rope_sin_pm;
            a.ldrope = e->Dh / 2;
            a.eps = e->eps;
            if (e2cu_launch(e2c_gemm(&a, st), "encoder qkv + finish")) return -1;
        } else if (e->ablk != D) {
            /* per-block scales: the GEMM folds block by block into fp32, a row kernel does the rest */
            a.epi = E2C_EPI_F32;
            a.y = e->qkvf;
            a.ldy = GD + 2 * e->Dh;
            if (e2cu_launch(e2c_gemm(&a, st), "encoder qkv") ||
                e2cu_launch(e2c_qkv_post(e->qkvf, GD + 2 * e->Dh, e->H, nrm(e, l, 4), nrm(e, l, 5), e->eps, e->rope_cos,
                                         e->rope_sin, e->max_seq, S, e->Q, e->K, e->Vt, ldvt, M, st),
                            "encoder qkv post"))
                return -1;
            n += 1;
        } else {
        a.epi = E2C_EPI_QKV;
        a.nq = e->H;
        a.q_out = e->Q;
        a.k_out = e->K;
        a.vt_out = e->Vt;
        a.ldvt = ldvt;
        a.seq_len = S;
        a.q_gamma = nrm(e, l, 4);
        a.k_gamma = nrm(e, l, 5);
        a.rope_cos = e->rope_cos;
        a.rope_sin = e->rope_sin;
        a.ldrope = e->max_seq;
        a.eps = e->eps;
        if (e2cu_launch(e2c_gemm(&a, st), "encoder qkv")) return -1;
        }
        if (e2cu_launch(e2c_attention(e->Q, e->K, e->Vt, ldvt, valid, e->ctx, B, S, e->H, e->attn_scale, e->status, st),
                        "encoder attention"))
            return -1;
        if (e2cu_launch(e2c_quantize(e->ctx, GD, e->qa, GD, e->qs, M, GD, ab_gd, -INFINITY, INFINITY, 0, st),
                        "encoder ctx quant"))
            return -1;
        if (gemm_norms(e, &e->wo[l], M, ab_gd, nrm(e, l, 1), nrm(e, l, 2), NULL, &n, st, "encoder o_proj + norms")) return -1;
        e2cu_gemm_args(&a, &e->wgu[l], e->qb, e->qsb, M, ab_d);
        if (e->fused_gelu) {
            a.epi = E2C_EPI_GELUQ;
            a.q8 = e->qa;
            a.ldq = I;
            a.q8_scale = e->qs;
            if (e2cu_launch(e2c_gemm(&a, st), "encoder gate|up + h quant")) return -1;
        } else if (e->ablk != D) {
            a.epi = E2C_EPI_F32;
            a.y = e->guf;
            a.ldy = 2 * I;
            if (e2cu_launch(e2c_gemm(&a, st), "encoder gate|up") ||
                e2cu_launch(e2c_gelu_mul_quant(e->guf, 2 * I, I, e->qa, e->qs, M, ab_i, st), "encoder gelu quant"))
                return -1;
            n += 1;
        } else {
            a.epi = E2C_EPI_GELU;
            a.y = e->h;
            a.ldy = I;
            if (e2cu_launch(e2c_gemm(&a, st), "encoder gate|up")) return -1;
            if (e2cu_launch(e2c_quantize(e->h, I, e->qa, I, e->qs, M, I, ab_i, -INFINITY, INFINITY, 0, st),
                            "encoder h quant"))
                return -1;
            n += 1;
        }
        const int last = l + 1 == L;
        if (gemm_norms(e, &e->wd[l], M, ab_i, nrm(e, l, 3), last ? NULL : nrm(e, l + 1, 0), last ? final_norm(e) : NULL,
                       &n, st, "encoder down + norms"))
            return -1;
        n += 4;
    }
    /* head */
    const int ab_dh = e->ablk == D ? e->DH : 128;
    if (e2cu_launch(e2c_meanpool(e->res, valid, e->pooled, B, S, D, st), "encoder pool") ||
        e2cu_launch(e2c_quantize(e->pooled, D, e->pq, D, e->ps, B, D, ab_d, -INFINITY, INFINITY, 0, st), "encoder head quant"))
        return -1;
    e2cu_gemm_args(&a, &e->dense1, e->pq, e->ps, B, ab_d);
    a.y = e->h1;
    a.ldy = e->DH;
    if (B <= e->gws_rows) {
        a.ws = e->gws;
        a.ws_bytes = e->gws_bytes;
    }
    if (e2cu_launch(e2c_gemm(&a, st), "encoder dense1") ||
        e2cu_launch(e2c_quantize(e->h1, e->DH, e->pq, e->DH, e->ps, B, e->DH, ab_dh, -INFINITY, INFINITY, 0, st),
                    "encoder head quant"))
        return -1;
    e2cu_gemm_args(&a, &e->dense2, e->pq, e->ps, B, ab_dh);
    a.y = e->out;
    a.ldy = e->DO;
    if (B <= e->gws_rows) {
        a.ws = e->gws;
        a.ws_bytes = e->gws_bytes;
    }
    if (e2cu_launch(e2c_gemm(&a, st), "encoder dense2") ||
        e2cu_launch(e2c_l2norm_rows(e->out, valid, B, S, e->DO, st), "encoder l2"))
        return -1;
    return n + 6;
}

static int ensure_vt(e2cuda_encoder *e, int B, int S) {
    const size_t need = (size_t)B * 256 * round8(S) * 2;
    if (need <= e->vt_bytes) return 0;
    /* captured graphs hold the old buffer */
    for (int i = 0; i < e->ngraphs; i++) cudaGraphExecDestroy(e->graphs[i].exec);
    e->ngraphs = 0;
    if (e->Vt) cudaFree(e->Vt);
    e->Vt = NULL;
    e->vt_bytes = 0;
    if (e2cu_cuda(cudaMalloc(&e->Vt, need), "encoder V^T alloc")) return -1;
    e->vt_bytes = need;
    return 0;
}

/* one pass, inputs already in e->ids / e->valid, result in e->out */
static int pass(e2cuda_encoder *e, int B, int S, int has_valid, cudaStream_t st) {
    if (ensure_vt(e, B, S)) return -1;
    if (e->gws && e2cu_ws_refresh(e->gws, e->gws_bytes, &e->gws_gen, st)) return -1;
    graph_slot *g = NULL;
    for (int i = 0; i < e->ngraphs; i++)
        if (e->graphs[i].B == B && e->graphs[i].S == S && e->graphs[i].has_valid == has_valid) g = &e->graphs[i];
    if (g) {
        e->kernels_last = g->kernels;
        return e2cu_cuda(cudaGraphLaunch(g->exec, st), "encoder graph launch");
    }
    const int n = encode(e, B, S, has_valid, st);
    if (n < 0) return -1;
    e->kernels_last = n;
    /* record the same sequence for the next call of this shape (not on the legacy stream) */
    if (st && e->ngraphs < MAX_GRAPHS) {
        cudaGraph_t graph = NULL;
        if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const int n2 = encode(e, B, S, has_valid, st);
            const cudaError_t ce = cudaStreamEndCapture(st, &graph);
            cudaGraphExec_t exec = NULL;
            if (n2 >= 0 && ce == cudaSuccess && graph && cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess) {
                graph_slot *s = &e->graphs[e->ngraphs++];
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

int e2cuda_encoder_embed_batch_device(e2cuda_encoder *e, const int32_t *d_ids, const uint8_t *d_valid, int batch,
                                      int seq_len, float *d_out, void *stream) {
    if (!e || !d_ids || !d_out || batch <= 0 || seq_len <= 0 || seq_len > e->max_seq) {
        e2cu_err("encoder_embed_batch_device: bad arguments (seq_len %d, max %d)", seq_len, e ? e->max_seq : 0);
        return -1;
    }
    cudaStream_t st = (cudaStream_t)stream;
    const int per = e->max_tokens / seq_len;
    if (per <= 0) {
        e2cu_err("encoder_embed_batch_device: seq_len %d exceeds max_tokens %d", seq_len, e->max_tokens);
        return -1;
    }
    for (int b0 = 0; b0 < batch; b0 += per) {
        const int B = batch - b0 < per ? batch - b0 : per;
        const size_t rows = (size_t)B * seq_len, off = (size_t)b0 * seq_len;
        if (e2cu_cuda(cudaMemcpyAsync(e->ids, d_ids + off, sizeof(int32_t) * rows, cudaMemcpyDeviceToDevice, st), "ids") ||
            (d_valid && e2cu_cuda(cudaMemcpyAsync(e->valid, d_valid + off, rows, cudaMemcpyDeviceToDevice, st), "valid")))
            return -1;
        if (pass(e, B, seq_len, d_valid != NULL, st)) return -1;
        if (e2cu_cuda(cudaMemcpyAsync(d_out + (size_t)b0 * e->DO, e->out, sizeof(float) * (size_t)B * e->DO,
                                      cudaMemcpyDeviceToDevice, st),
                      "out"))
            return -1;
    }
    e->calls++;
    return 0;
}

static double now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec / 1e6;
}

int e2cuda_encoder_embed_batch(e2cuda_encoder *e, const int32_t *ids, const uint8_t *valid, int batch, int seq_len,
                               float *out) {
    const double t0 = now_ms();
    if (!e || !ids || !out || batch <= 0 || seq_len <= 0 || seq_len > e->max_seq) {
        e2cu_err("encoder_embed_batch: bad batch geometry");
        return -1;
    }
    /* validate the whole request before touching the output (e2.c src/text.c:1005-1011) */
    const size_t total = (size_t)batch * seq_len;
    for (size_t i = 0; i < total; i++)
        if (ids[i] < 0 || ids[i] >= e->V) {
            e2cu_err("token id %d out of range", ids[i]);
            return -1;
        }
    const int per = e->max_tokens / seq_len;
    if (per <= 0) {
        e2cu_err("encoder_embed_batch: seq_len %d exceeds max_tokens %d", seq_len, e->max_tokens);
        return -1;
    }
    cudaStream_t st = e->stream;
    for (int b0 = 0; b0 < batch; b0 += per) {
        const int B = batch - b0 < per ? batch - b0 : per;
        const size_t rows = (size_t)B * seq_len, off = (size_t)b0 * seq_len;
        if (e2cu_cuda(cudaMemcpyAsync(e->ids, ids + off, sizeof(int32_t) * rows, cudaMemcpyHostToDevice, st), "ids") ||
            (valid && e2cu_cuda(cudaMemcpyAsync(e->valid, valid + off, rows, cudaMemcpyHostToDevice, st), "valid")))
            return -1;
        if (pass(e, B, seq_len, valid != NULL, st)) return -1;
        if (e2cu_cuda(cudaMemcpyAsync(out + (size_t)b0 * e->DO, e->out, sizeof(float) * (size_t)B * e->DO,
                                      cudaMemcpyDeviceToHost, st),
                      "out") ||
            e2cuda_check(st))
            return -1;
    }
    e->calls++;
    e->last_ms = now_ms() - t0;
    return 0;
}

int e2cuda_encoder_stats(e2cuda_encoder *e, long *calls, long *kernels_last, double *last_ms) {
    if (!e) {
        e2cu_err("encoder_stats: null encoder");
        return -1;
    }
    if (calls) *calls = e->calls;
    if (kernels_last) *kernels_last = e->kernels_last;
    if (last_ms) *last_ms = e->last_ms;
    return 0;
}
