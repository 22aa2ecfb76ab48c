/* launch.h — the C-callable kernel launchers behind the e2cuda C ABI.
 *
 * The host side of e2cuda (e2cuda.c, encoder.c) is C11; every function here is implemented in a
 * .cu file and exported with C linkage. All pointers are device pointers unless named otherwise;
 * `stream` is a cudaStream_t. Launchers check arguments they can check cheaply and return 0, or a
 * negative code with a message in e2c_msg.
 */
#ifndef E2C_LAUNCH_H
#define E2C_LAUNCH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* last launcher error message (thread-local) */
const char *e2c_msg(void);
void e2c_set_msg(const char *fmt, ...);

/* Activation quantiser (src/int8.c:178-209 semantics in the forms the -ffast-math build computes): x fp32 [M][K] (row stride
 * ldx floats) -> q int8 [M][K] (row stride ldq bytes), scales [M][K/ablk]. biased != 0 stores q+128
 * (the reference's byte convention), else signed q. ablk = K for per-row, else a divisor of K that
 * is a multiple of 16. */
int e2c_quantize(const float *x, int ldx, int8_t *q, int ldq, float *scales, int M, int K, int ablk,
                 float lo, float hi, int biased, void *stream);

/* bytes ^= 0x80: converts between the reference's biased q+128 and signed q, in place */
int e2c_flip_bias(int8_t *q, size_t n, void *stream);

/* int8 GEMM epilogues */
enum {
    E2C_EPI_F32 = 0,   /* y = dequant (clamped)                                            */
    E2C_EPI_RESID = 1, /* y = dequant (clamped) + resid                                    */
    E2C_EPI_I32 = 2,   /* dots[m][n][b] = raw int32 block dots (debug; bit-exact check)      */
    E2C_EPI_GELU = 3,  /* weight rows interleaved per 128: h = gelu(g) * u, fp32 [M][N/2]  */
    E2C_EPI_QKV = 4,   /* per-head RMSNorm (+gamma) + RoPE -> bf16 Q, K, V^T               */
    E2C_EPI_NORMADD = 5 /* y = gemm (never stored); x = rmsnorm(y) * g1 + res; res = x;
                          q = quantise(rmsnorm(x) * g2) per token (g2 NULL: res = rmsnorm(x) * gf).
                          Whole rows per cluster of CTAs (N = 768: 6 x 128 columns). With 128-wide
                          activation blocks: the per-block fold, and q per 128-column block with
                          q8_scale [M][N/128] */,
    E2C_EPI_GELUQ = 6, /* GELU-gate as E2C_EPI_GELU, then the per-token quantiser of h over its
                          N/2 columns: int8 q8 [M][ldq] and q8_scale [M] (h itself is not stored).
                          Whole rows per cluster of N/256 CTAs (N = 2304: 9). With per-128-block
                          activation scales: h's per-block quantiser, q8_scale [M][N/256] */
    E2C_EPI_QKVPB = 7  /* per-128-block activation scales: the q|k|v finish of heads of 256.
                          Columns [0, 256 nq) are q heads, then nkv k heads, then nkv v heads
                          (nkv = (N/256 - nq) / 2): per-head RMSNorm (q_gamma, k_gamma; v without a
                          gain), RoPE on q and k from position-major tables (cos of pair i at
                          position p: rope_cos[p * ldrope + i]), bf16 Q [M][256 nq], K [M][256 nkv]
                          and V^T [B][256 nkv][ldvt] */
};

typedef struct {
    /* operands */
    const int8_t *a;       /* [M][K] signed, row stride lda bytes (multiple of 16)          */
    int lda;
    const float *a_scale;  /* [M][K/ablk]                                                  */
    const int8_t *w;       /* [wrows][K] K-major, row stride ldw bytes (multiple of 16)     */
    int ldw, wrows;
    const float *w_scale;  /* [wrows]                                                      */
    int M, K, ablk;
    int n0, n1;            /* columns (= weight rows) to compute                            */
    int epi;
    /* outputs */
    float *y;              /* F32 / RESID / GELU output, row stride ldy floats              */
    int ldy;
    const float *resid;    /* RESID: row stride ldr floats                                  */
    int ldr;
    int32_t *dots;         /* I32: [M][ldd][K/ablk]                                         */
    int ldd;
    float out_min, out_max;
    /* QKV epilogue: columns [0, 256*nq) are q heads, then one k head, then one v head */
    int nq;
    void *q_out, *k_out, *vt_out; /* bf16: Q [M][256*nq], K [M][256], V^T [B][256][ldvt]  */
    int ldvt, seq_len;     /* position of row m = m % seq_len; V^T row block = m / seq_len  */
    const float *q_gamma, *k_gamma; /* [256] */
    const float *rope_cos, *rope_sin; /* pair-major [128][ldrope]: (i, pos) at i * ldrope + pos */
    int ldrope;            /* >= seq_len                                                    */
    float eps;
    /* NORMADD epilogue: the residual stream res [M][ldres] (read and written), the two norm gains,
     * the final norm's gain (used when norm_g2 is NULL), the quantised rows q8 [M][ldq] and their
     * per-token scales q8_scale [M] */
    float *res;
    int ldres;
    const float *norm_g1, *norm_g2, *norm_gf;
    int8_t *q8;
    int ldq;
    float *q8_scale;
    int *status;
    /* Optional workspace of the weight-streaming kernel (short activation matrices): zero before
     * its first use, used by one stream at a time, 128-byte aligned; NULL: that kernel is not used.
     * Every launch that completes leaves it zero. */
    int *ws;
    size_t ws_bytes;
    /* NORMADD: x is multiplied by norm_ls after the residual add (0: no scaling); with q8 given but
     * neither norm_g2 nor norm_gf, x itself is quantised (g2 = 1, no second norm) */
    float norm_ls;
} e2c_gemm_args;

int e2c_gemm(const e2c_gemm_args *a, void *stream);
/* The same GEMM with K split over a cluster of S CTAs per 128 x bn output tile (S a power of two,
 * 2..16; bn 128 or 256), partial sums reduced in distributed shared memory: the launcher e2c_gemm
 * picks it for short activation matrices (few output tiles). Per-row scales, F32 or residual
 * epilogue only. */
int e2c_gemm_splitk(const e2c_gemm_args *a, int bn, int S, void *stream);
/* Its co-resident variant for 1..32 rows (BN 128, at most one CTA per SM, the weight's first stages
 * requested before griddepcontrol.wait); -1 without launching where it does not apply */
int e2c_gemm_splitk_co(const e2c_gemm_args *a, void *stream);
/* The weight-streaming GEMM for 1..256 rows (gemm_i8_stream.cu): the weight in the MMA's 128-row
 * slot, stream-K over every SM, split weight tiles reduced through the workspace a->ws. Per-row
 * scales, F32 or residual epilogue. e2c_gemm picks it when a workspace is given and the activation
 * matrix is short. */
int e2c_gemm_stream(const e2c_gemm_args *a, void *stream);
/* bytes of workspace a launch over M rows needs on a device with num_sms SMs */
size_t e2c_gemm_stream_ws_bytes(int M, int num_sms);
int e2c_gemm_stream_ctas(const e2c_gemm_args *a, int num_sms);
/* bytes of workspace e2c_gemm's weight-streaming path needs for M rows on the current device (0
 * without a device, or for M outside 1..256) */
size_t e2c_gemm_ws_bytes(int M);
/* the kernel family e2c_gemm last launched on this thread: "stream", "splitk", "persistent",
 * "persistent_pair" (the fused epilogues: "persistent"), or under programmatic dependent launch
 * "stream_coresident" / "splitk_coresident" */
const char *e2c_gemm_last_kernel(void);
/* E2C_EPI_NORMADD (gemm_i8_norm.cu): rows of 128 x (1..8) columns over a cluster of CTAs, the
 * residual norms in the epilogue; called by e2c_gemm after its checks */
int e2c_gemm_norm(const e2c_gemm_args *a, void *stream);
/* E2C_EPI_GELUQ (gemm_i8_gelu.cu), called by e2c_gemm after its checks; _supported(ncl) is 1 when
 * the device holds clusters of ncl such CTAs */
int e2c_gemm_gelu_quant(const e2c_gemm_args *a, void *stream);
int e2c_gemm_gelu_quant_supported(int ncl);
/* the split that puts most CTAs to work with every cluster resident at once: returns the CTA count
 * (0 when the split kernel does not apply) and sets *bn, *S */
int e2c_gemm_splitk_plan(const e2c_gemm_args *a, int num_sms, int *bn, int *S);
/* the tile the GEMM picks for these arguments, for traffic accounting: *bm x *bn */
void e2c_gemm_tile(const e2c_gemm_args *a, int *bm, int *bn);

/* ---- row kernels of the encoder (one warp per token row, D = hidden, a multiple of 128;
 * ablk is 128 or D) */
/* x = table[id] * table_scale[id] * embed_scale; res = x; quantise(rmsnorm(x) * gamma) per row.
 * An id outside [0, vocab) reads row 0 and records status 0x106. */
int e2c_embed_norm_quant(const int32_t *ids, const int8_t *table, const float *table_scale,
                         float embed_scale, const float *gamma, float eps, float *res, int8_t *q,
                         float *qs, int M, int D, int ablk, int vocab, int *status, void *stream);
/* x = rmsnorm(t) * g1 + res; then res = x and quantise(rmsnorm(x) * g2) per row. With g2 NULL:
 * out = rmsnorm(x) * gfinal written to `res` instead (the last layer's final norm), no quantise. */
int e2c_norm_add_norm_quant(const float *t, float *res, const float *g1, const float *g2,
                            const float *gfinal, float eps, int8_t *q, float *qs, int M, int D,
                            int ablk, void *stream);
/* quantise(rmsnorm(x) * gamma) per row (config-1 FFN prologue; the residual is x itself) */
int e2c_norm_quant(const float *x, const float *gamma, float eps, int8_t *q, float *qs, int M, int D,
                   int ablk, void *stream);
/* Per-128-block activation mode (the reference's default recipe), where the fused epilogues that
 * need per-token scales cannot run. q|k|v fp32 y [M][ldy] (heads of 256: nq q heads, then k, then v)
 * -> per-head RMSNorm (q_gamma, k_gamma; v without) -> RoPE on q and k -> bf16 Q [M][256 nq],
 * K [M][256], V^T [M / seq_len][256][ldvt]; the same arithmetic as the QKV epilogue. */
int e2c_qkv_post(const float *y, int ldy, int nq, const float *q_gamma, const float *k_gamma, float eps,
                 const float *rope_cos, const float *rope_sin, int ldrope, int seq_len, void *q_out, void *k_out,
                 void *vt_out, int ldvt, int M, void *stream);
/* gate|up fp32 y [M][ldy], columns interleaved per 128 -> h = gelu_tanh(gate) * up -> q [M][I] int8
 * and scales [M][I / ablk] (ablk 128 or I) */
int e2c_gelu_mul_quant(const float *y, int ldy, int I, int8_t *q, float *qs, int M, int ablk, void *stream);
/* pooled[b][d] = mean over valid rows of x[b*S + s][d] (all-invalid -> 0) */
int e2c_meanpool(const float *x, const uint8_t *valid, float *pooled, int B, int S, int D, void *stream);
/* rows of y [B][D] L2-normalised in place; rows whose sequence has no valid token become 0 */
int e2c_l2norm_rows(float *y, const uint8_t *valid, int B, int S, int D, void *stream);

/* ---- row kernels of e2.c's own text tower (text_rows.cu); D, P, I multiples of 128, ablk 128 or
 * the row width */
/* x = bf16 table[id] * embed_scale -> res; quantise(x) -> qx, qxs; quantise(rmsnorm(x) * gamma) -> qn,
 * qns. An id outside [0, vocab) reads row 0 and records status 0x106. */
int e2c_tt_embed(const int32_t *ids, const uint16_t *table, float embed_scale, const float *gamma, float eps,
                 float *res, int8_t *qx, float *qxs, int8_t *qn, float *qns, int M, int D, int ablk, int vocab,
                 int *status, void *stream);
/* q|k|v fp32 y [M][ldy] as [H q heads | KV k heads | KV v heads] of D (256 or 512, KV D <= 512) -> per-head
 * RMSNorm (q_gamma, k_gamma [D]; v without) -> RoPE on q and k -> bf16 Q [M][H D], K [M][KV D],
 * V^T [M / seq_len][KV D][ldvt]. RoPE tables position-major ([pos][ldrope], rope_pos_major != 0) or
 * pair-major ([D/2][ldrope]). */
int e2c_tt_qkv_post(const float *y, int ldy, int H, int KV, int D, const float *q_gamma, const float *k_gamma,
                    float eps, const float *rope_cos, const float *rope_sin, int ldrope, int rope_pos_major,
                    int seq_len, void *q_out, void *k_out, void *vt_out, int ldvt, int M, void *stream);
/* x = (rmsnorm(t) * g1 + res) * layer_scalar -> res; quantise(rmsnorm(x) * g2) -> q, qs, or
 * quantise(x) when g2 is NULL */
int e2c_tt_norm_add(const float *t, float *res, const float *g1, float layer_scalar, const float *g2, float eps,
                    int8_t *q, float *qs, int M, int D, int ablk, void *stream);
/* h = gelu_tanh(g) * u over I columns (g rows ldg floats apart, u rows ldu apart) -> quantise -> q, qs.
 * ugamma given: u is first rmsnorm(u * uscale) * ugamma over its I values (the PLE slice's norm). */
int e2c_tt_gate_quant(const float *g, int ldg, const float *u, int ldu, float uscale, const float *ugamma, float eps,
                      int I, int8_t *q, float *qs, int M, int ablk, void *stream);

/* ---- attention: bf16 Q [B*S][H*256], K [B*S][256], V^T [B][256][ldvt] -> ctx fp32 [B*S][H*256] */
int e2c_attention(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid,
                  float *ctx, int B, int S, int H, float scale, int *status, void *stream);
/* the same for head dim D (64 or 256) and KV key/value heads (KV divides H; query head h reads KV
 * head h / (H / KV)): Q [B*S][H*D], K [B*S][KV*D], V^T [B][KV*D][ldvt] -> ctx [B*S][H*D] */
int e2c_attention_gqa(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid, float *ctx,
                      int B, int S, int H, int KV, int D, float scale, int *status, void *stream);
/* the same with a sliding window: query i attends to keys j with |i - j| <= window (window < 0: all
 * keys), e2.c src/text.c:656-661; D 64, 256 or 512 (512: attention_wide.cu) */
int e2c_attention_win(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid, float *ctx,
                      int B, int S, int H, int KV, int D, float scale, int window, int *status, void *stream);
/* head dim 512 (attention_wide.cu), called by e2c_attention_win after its checks */
int e2c_attention_wide(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid, float *ctx,
                       int B, int S, int H, int KV, float scale, int window, int *status, void *stream);

/* ---- self-test of the bounded wait (selftest.cu): one warp waits on an mbarrier that receives
 * its arrival first (arrive != 0) or never (arrive == 0). *completed is 1 if the wait completed, 0
 * if it gave up after its bound (~2 s) and recorded `code` (0x101..0x105) in *status. */
int e2c_wait_selftest(int *status, int code, int arrive, int *completed, void *stream);

#ifdef __cplusplus
}
#endif
#endif
