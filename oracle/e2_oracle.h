/* e2_oracle.h — CPU checker for the e2cuda int8 hot path. TEST INFRASTRUCTURE ONLY.
 *
 * Nothing in the product (the e2cuda library, its Python mirror) links, loads or calls this. Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm use it, and only as
 * the checker or the timed CPU baseline.
 *
 * Two halves:
 *   1. A plain-C restatement ("port") of the reference e2.c kernels on the path: the activation
 *      quantiser, the per-row weight quantiser and its quad-interleaved pack, the int8 GEMM fold,
 *      RMSNorm / norm_split / norm_add, GELU-tanh with the AVX-512 polynomial exp, softmax, RoPE,
 *      the fp32 NN GEMM, mean pool and L2 norm. Each function cites the reference file:line it
 *      restates (paths are relative to the e2.c project root).
 *   2. Compositions over a kernel table (e2o_kernels): the config-1 FFN block and the config-2
 *      synthetic encoder, in the layer order of src/text.c:939-961 minus the PLE block. The table
 *      is filled either from the port (liboracle.so) or from the reference's own kernels compiled
 *      from its sources (oracle/_ref/libe2ref_b<ABLK>.so, see ref_glue.c), so one composition
 *      serves as the parity oracle and as the timed CPU baseline.
 *
 * Pinning: the port is checked against the reference build (oracle/_ref) and against the fixtures
 * under tests/golden/ that tests/golden/make_golden.py generated from it.
 */
#ifndef E2_ORACLE_H
#define E2_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same memory layout as the reference's e2_q8w (src/int8.h:79-92), so a pointer to one can be
 * handed to the reference kernels unchanged (ref_glue.c asserts the offsets). */
typedef struct {
    int8_t *w;      /* [Npad/8][K/4][8][4] quad-interleaved */
    int32_t *bsq;   /* [nblocks][Npad] per-block weight sums */
    float *scale;   /* [Npad] per-row weight scale */
    int N, K, nblocks, Npad;
    float out_min, out_max;
    int borrowed;
} e2o_q8w;

typedef void (*e2o_task_fn)(void *arg, int tid, int nthreads);

/* The kernels a composition runs on. `ablk` is the activation block the quantiser and GEMM use
 * (E2_I8_BLOCK in the reference, one build per block size); 0 means per-row scales, i.e. the block
 * is the K of each call (the reference's per-row mode, -DE2_I8_BLOCK=K, one build per K). */
typedef struct {
    const char *name;
    int ablk;
    void (*quantize)(int8_t *out, float *scales, const float *x, int M, int K, float lo, float hi);
    void (*gemm)(float *y, const int8_t *qa, const float *as, const e2o_q8w *w, int M, int N, int n0,
                 int n1);
    int (*q8w_from_f32)(e2o_q8w *q, const float *w, int N, int K);
    void (*q8w_free)(e2o_q8w *q);
    void (*rmsnorm)(float *x, int M, int D, const float *gamma, float eps);
    void (*norm_split)(float *x, float *res, int rows, int D, const float *gamma, float eps);
    void (*norm_add)(float *out, const float *src, const float *res, int rows, int D,
                     const float *gamma, float eps);
    void (*gelu_tanh)(float *x, size_t n);
    void (*mul)(float *a, const float *b, size_t n);
    void (*softmax)(float *x, int n);
    void (*rope_rows)(float *x, int r0, int r1, int ngroups, int head_dim, int block, const float *cs,
                      const float *sn);
    void (*sgemm_nn)(float *C, int ldc, const float *A, int lda, const float *B, int ldb, int M, int N,
                     int K, int m0, int m1);
    void (*meanpool)(float *out, const float *x, int M, int D, const uint8_t *valid);
    void (*l2norm)(float *x, int n);
    /* fn(arg, tid, nthreads) once per worker; NULL runs fn(arg, 0, 1) inline */
    void (*parallel)(e2o_task_fn fn, void *arg);
    int nthreads;
} e2o_kernels;

/* ------------------------------------------------------------------ the port (e2_oracle.c) */
/* The kernel table over the port, for activation block `ablk` (a block dividing every K the caller
 * uses, or 0 for per-row scales). Serial. */
const e2o_kernels *e2o_port_kernels(int ablk);

/* src/int8.c:178-209 with the scale/reciprocal forms the reference's -ffast-math AVX-512 build
 * produces (see the definition). Stores q+128 like the reference. */
void e2o_quantize_blocks(int8_t *out, float *scales, const float *x, int M, int K, int ablk, float lo,
                         float hi);
/* The same quantiser storing signed q (the e2cuda convention): out[i] = q, not q+128. */
void e2o_quantize_rows_signed(int8_t *out, float *scales, const float *x, int M, int K, int ablk);
/* src/int8.c:19-66 (per-row weight quantiser + quad-interleaved pack + block sums). */
int e2o_q8w_from_f32(e2o_q8w *q, const float *w, int N, int K, int ablk);
void e2o_q8w_free(e2o_q8w *q);
/* Unpack a quad-interleaved weight to plain row-major [N][K] int8 (the inverse of the pack). */
void e2o_q8w_unpack(const e2o_q8w *q, int8_t *wk);
/* src/kernels_i8_avx512_vnni.c:276-307: per (row, col, block) int32 dot, then
 * f = fma(float(dot), as*ws, f) over blocks in order, clamp at the store. Biased activations. */
void e2o_i8_gemm(float *y, const int8_t *qa, const float *as, const e2o_q8w *w, int M, int N, int n0,
                 int n1, int ablk);
/* The same fold from plain operands: signed qa [M][K], row-major int8 w [N][K], ws [N]. Optionally
 * also returns the raw int32 per-block dots dots[M][N][K/ablk] (NULL to skip). */
void e2o_i8_gemm_plain(float *y, int32_t *dots, const int8_t *qa, const float *as, const int8_t *w,
                       const float *ws, int M, int N, int K, int ablk, float out_min, float out_max);

void e2o_rmsnorm(float *x, int M, int D, const float *gamma, float eps);
void e2o_norm_split(float *x, float *res, int rows, int D, const float *gamma, float eps);
void e2o_norm_add(float *out, const float *src, const float *res, int rows, int D, const float *gamma,
                  float eps);
void e2o_gelu_tanh(float *x, size_t n);
void e2o_softmax(float *x, int n);
void e2o_rope_rows(float *x, int r0, int r1, int ngroups, int head_dim, int block, const float *cs,
                   const float *sn);
void e2o_sgemm_nn(float *C, int ldc, const float *A, int lda, const float *B, int ldb, int M, int N,
                  int K, int m0, int m1);
void e2o_meanpool(float *out, const float *x, int M, int D, const uint8_t *valid);
void e2o_l2norm(float *x, int n);
/* src/text.c:483-506 RoPE tables: cos/sin [npos][head_dim], halves duplicated. */
void e2o_rope_tables(float *cs, float *sn, int npos, int head_dim, float theta);

/* splitmix64 stream + Box-Muller: the seeded synthetic data of every config. */
uint64_t e2o_splitmix64(uint64_t *state);
void e2o_fill_normal(float *dst, size_t n, uint64_t seed, float mean, float std);

/* ------------------------------------------------------------------ compositions (encoder.c) */
/* Config-1 gated FFN block on fp32 hidden [M][D] (src/text.c:947-954 + mlp :893-903):
 *   res = x; xn = rmsnorm(x)*gamma; g|u = int8 GEMM(quant(xn)); h = gelu(g)*u;
 *   y = int8 GEMM(quant(h)) + res            (plain residual add, config 1)
 * Writes y [M][D]. Optional stage dumps (NULL to skip): xq/xs the quantised normed input,
 * hq/hs the quantised h (biased bytes, reference convention), gu [M][2I] (gate | up). */
int e2o_ffn_block(const e2o_kernels *k, const float *x, int M, int D, int I, const float *gamma,
                  float eps, const e2o_q8w *wg, const e2o_q8w *wu, const e2o_q8w *wd, float *y,
                  int8_t *xq, float *xs, int8_t *hq, float *hs, float *gu);

/* The synthetic encoder of config 2. Weights are the reference's packed e2o_q8w per projection. */
typedef struct {
    int n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab;
    int dense_hidden, out_dim; /* head: hidden -> dense_hidden -> out_dim, then L2 */
    float rope_theta, eps, attn_scale, embed_scale;
    /* token table: int8 [vocab][hidden] + per-row scale (F7: int8 table with row scale) */
    const int8_t *table;
    const float *table_scale;
    /* per layer (arrays of n_layers) */
    const e2o_q8w *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    const float *const *input_ln, *const *post_attn_ln, *const *pre_ffn_ln, *const *post_ffn_ln;
    const float *const *q_norm, *const *k_norm;
    const float *final_norm;
    const e2o_q8w *dense1, *dense2;
} e2o_encoder;

/* ids [B][S], valid [B][S] or NULL; out [B][out_dim]. Full (bidirectional) attention over the valid
 * keys of each sequence, fp32 (the reference's blocked fp32 path, src/text.c:702-741), scaled by
 * attn_scale. Returns 0, or -1 on a bad argument. If last_hidden is not NULL it receives the final
 * normed hidden state [B*S][hidden]; if layer0 is not NULL it receives x after layer 0. */
int e2o_encoder_forward(const e2o_kernels *k, const e2o_encoder *e, const int32_t *ids,
                        const uint8_t *valid, int B, int S, float *out, float *last_hidden,
                        float *layer0);

/* fp32 attention of one sequence with GQA, used by the encoder and by the attention parity tests:
 * q [S][H*D], k/v [S][KV*D], ctx [S][H*D]; rows with valid[i]==0 get ctx 0 and are skipped as keys. */
void e2o_attention_f32(const e2o_kernels *k, const float *q, const float *kk, const float *v,
                       float *ctx, const uint8_t *valid, int S, int H, int KV, int D, float scale);

#ifdef __cplusplus
}
#endif
#endif
