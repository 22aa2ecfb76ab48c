/* ref_text.c — TEST INFRASTRUCTURE ONLY. e2.c's own engine (compiled from its sources into
 * oracle/_ref/libe2ref_text.so) as the checker of the device text tower, and the binding e2.c would
 * carry for it (the shape of src/gpu/hip/hip.c's e2_hip_create, include/e2hip.h:32-64).
 *
 * The checker: ref_text_load runs e2.c's own loader (src/e2.c:253-420) on a model directory. The
 * loader builds every tower unless it is writing a packed cache restricted to the text tower
 * (E2_Q8_WRITE + E2_Q8_TOWERS=text, src/e2.c:243-252,285,413-415), which is how a text-only
 * checkpoint loads; the cache it writes goes to `cache_path` and is not used here. ref_text_embed_batch
 * is e2_text_embed_batch itself (src/text.c:991-1023). ref_text_attention forces the text
 * attention's precision (e2_attn_override, src/dispatch.h:79): E2_ATTN_F32 (0) is the blocked fp32
 * path, E2_ATTN_I8 (2) the int8 one e2.c picks from 128 keys, -1 the dispatch table.
 *
 * The binding: e2_cuda_create fills an e2cuda_text_desc from the e2_model's fields (the e2_q8w
 * weights the loader built, passed by pointer: e2cuda_q8w has e2_q8w's layout) and uploads it.
 */
#include <stdlib.h>
#include <string.h>

#include "dispatch.h"
#include "e2cuda.h"
#include "model.h"

static e2_model *g_model;

int ref_text_load(const char *model_dir, const char *cache_path) {
    if (g_model) return 0;
    setenv("E2_Q8_WRITE", cache_path, 1);
    setenv("E2_Q8_TOWERS", "text", 1);
    g_model = e2_load(model_dir);
    unsetenv("E2_Q8_WRITE");
    unsetenv("E2_Q8_TOWERS");
    return g_model ? 0 : -1;
}

const char *ref_text_error(void) { return e2_last_error(); }

int ref_text_embed_batch(const int32_t *ids, const uint8_t *valid, int batch, int seq_len, float *out) {
    return g_model ? e2_text_embed_batch(g_model, ids, valid, batch, seq_len, out) : -1;
}

void ref_text_attention(int kind) { e2_attn_override(E2_TOWER_TEXT, kind); }

int ref_text_threads(void) { return e2_nthreads(); }

void ref_text_free(void) {
    if (g_model) e2_free(g_model);
    g_model = NULL;
}

/* ------------------------------------------------------------------ the binding */
/* e2cuda_text_desc over a loaded e2_model; `layers` has room for E2_MAX_LAYERS entries */
int e2_cuda_describe(e2_model *m, e2cuda_text_desc *d, e2cuda_text_layer *layers) {
    if (!m || !m->use_int8) return -1;
    memset(d, 0, sizeof *d);
    d->n_layers = m->n_layers;
    d->hidden = m->hidden;
    d->intermediate = m->intermediate;
    d->ple_dim = m->ple_dim;
    d->n_heads = E2_NUM_HEADS;
    d->vocab = E2_VOCAB;
    d->out_dim = E2_EMBED_DIM;
    d->max_seq = E2_MAX_SEQ;
    d->ablk = E2_I8_BLOCK;
    d->eps = m->rms_eps;
    d->embed_scale = m->embed_scale;
    d->ple_scale = m->ple_scale;
    d->embed_tokens = m->embed_tokens;
    d->ple_model_proj = (const e2cuda_q8w *)&m->q8_ple_model;
    d->embed_proj = (const e2cuda_q8w *)&m->q8_embed_proj;
    d->ple_proj_norm = m->ple_proj_norm;
    d->final_norm = m->final_norm;
    for (int l = 0; l < m->n_layers; l++) {
        const e2_layer *L = &m->layers[l];
        e2cuda_text_layer *y = &layers[l];
        y->q = (const e2cuda_q8w *)&L->q8_q;
        y->k = (const e2cuda_q8w *)&L->q8_k;
        y->v = (const e2cuda_q8w *)&L->q8_v;
        y->o = (const e2cuda_q8w *)&L->q8_o;
        y->gate = (const e2cuda_q8w *)&L->q8_gate;
        y->up = (const e2cuda_q8w *)&L->q8_up;
        y->down = (const e2cuda_q8w *)&L->q8_down;
        y->ple_gate = (const e2cuda_q8w *)&L->q8_ple_gate;
        y->ple_proj = (const e2cuda_q8w *)&L->q8_ple_proj;
        y->input_ln = L->input_ln;
        y->post_attn_ln = L->post_attn_ln;
        y->pre_ffn_ln = L->pre_ffn_ln;
        y->post_ffn_ln = L->post_ffn_ln;
        y->ple_norm = L->ple_norm;
        y->q_norm = L->q_norm;
        y->k_norm = L->k_norm;
        y->layer_scalar = L->layer_scalar;
        y->head_dim = L->head_dim;
        y->n_kv_heads = L->n_kv_heads;
        y->window = L->sliding ? L->window : -1;
        y->rope_theta = L->sliding ? m->rope_theta_sliding : m->rope_theta_full;
    }
    d->layers = layers;
    return 0;
}

typedef struct e2_cuda {
    e2cuda_text *t;
} e2_cuda;

/* e2_hip_create's counterpart: the model is read once; `m` may be freed afterwards */
e2_cuda *e2_cuda_create(e2_model *m) {
    e2cuda_text_desc d;
    e2cuda_text_layer layers[E2_MAX_LAYERS];
    if (e2_cuda_describe(m, &d, layers)) return NULL;
    e2_cuda *g = calloc(1, sizeof *g);
    if (!g) return NULL;
    g->t = e2cuda_text_create(&d, E2_MAX_SEQ * 16);
    if (!g->t) {
        free(g);
        return NULL;
    }
    return g;
}

void e2_cuda_destroy(e2_cuda *g) {
    if (!g) return;
    e2cuda_text_destroy(g->t);
    free(g);
}

int e2_cuda_text_embed_batch(e2_cuda *g, const int32_t *ids, const uint8_t *valid, int batch, int seq_len, float *out) {
    return g ? e2cuda_text_embed_batch(g->t, ids, valid, batch, seq_len, out) : -1;
}

int e2_cuda_text_embed(e2_cuda *g, const int32_t *ids, int n_ids, float *out768) {
    return g ? e2cuda_text_embed(g->t, ids, n_ids, out768) : -1;
}

/* for the tests: the binding over the model ref_text_load holds */
e2_cuda *ref_text_cuda_create(void) { return e2_cuda_create(g_model); }
int ref_text_describe(e2cuda_text_desc *d, e2cuda_text_layer *layers) { return e2_cuda_describe(g_model, d, layers); }
