/* e2cuda.h — e2.c's int8 hot path on an NVIDIA B200 (sm_100a), as a C ABI.
 *
 * The CUDA sibling of the engine's GPU backends (include/e2gpu.h, include/e2hip.h in e2.c): the same
 * W8A8 recipe — int8 weights with one fp32 scale per output row (the q8cache's e2_q8w), activations
 * quantised dynamically per token (or per 128-element block) — on the Blackwell tensor cores:
 *
 *   - activation quantiser          replaces e2_i8_quantize      (e2.c src/kernels.h:72)
 *   - W8A8 GEMM + fused epilogues   replaces e2_i8_gemm          (e2.c src/int8.h:96-97)
 *   - bf16 flash attention          replaces attention_blocked   (e2.c src/text.c:780-815)
 *   - the synthetic encoder         the text tower's layer recipe (e2.c src/text.c:924-984) over
 *                                   the kernels above, batch API shaped like e2_hip_text_embed_batch
 *                                   (e2.c include/e2hip.h:44-50)
 *
 * Conventions (those of e2gpu.h/e2hip.h): calls return 0 on success and -1 on failure, with the
 * reason in e2cuda_last_error() (thread-local). Input validation failures leave outputs untouched.
 * Functions taking a `stream` (a cudaStream_t, passed as void*) work on DEVICE pointers and are
 * stream-ordered: they return once the work is queued. A kernel that stops making progress records
 * a status code instead of hanging (every wait in the kernels is bounded to ~2 s); e2cuda_check()
 * synchronises a stream and reports such a failure. Host-buffer entry points (`_host`, the encoder's
 * embed_batch) synchronise and check before returning.
 *
 * Signed int8 activations: the device path stores q, not the reference's q+128 (V_DOT4-style, like
 * e2hip.h), so the +128 zero-point correction (e2_q8w.bsq) never exists on the device. Bytes are
 * the reference's with the top bit flipped; the `_host` entry points convert at the boundary.
 *
 * No TMA multicast and no peer-memory access anywhere: each GPU reads only its own memory.
 */
#ifndef E2CUDA_H
#define E2CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define E2CUDA_ABI_VERSION 1

/* Byte-for-byte the reference's e2_q8w (e2.c src/int8.h:79-92): quad-interleaved int8 weights
 * [Npad/8][K/4][8][4], per-block sums [nblocks][Npad], per-row scales [Npad], optional output clamp.
 * e2.c passes its `const e2_q8w *` cast to this type. */
typedef struct e2cuda_q8w {
    int8_t *w;
    int32_t *bsq;
    float *scale;
    int N, K, nblocks, Npad;
    float out_min, out_max;
    int borrowed;
} e2cuda_q8w;

/* A device-resident int8 weight in the layout the TMA engine streams: row-major [rows][ld] (K
 * contiguous, ld = K rounded up to 16 bytes, rows = N rounded up to 16), fp32 scale per row. */
typedef struct e2cuda_w8 {
    int8_t *w;
    float *scale;
    int N, K, rows, ld;
    float out_min, out_max; /* the e2_q8w clamp, applied at the GEMM's store */
} e2cuda_w8;

/* ------------------------------------------------------------------ library */
const char *e2cuda_last_error(void);
/* Name of the current CUDA device ("" if none); e2_hip_device's counterpart (e2hip.h:41). */
const char *e2cuda_device(void);
/* Synchronise `stream` and report (then clear) a device-side failure recorded by any e2cuda kernel
 * on the current device since the last check. 0 = clean. */
int e2cuda_check(void *stream);

/* ------------------------------------------------------------------ weights (A2, A11) */
/* Repack a reference e2_q8w (quad-interleaved, host) into a device e2cuda_w8. The int8 values and
 * scales are copied, never re-quantised, so device weights are bit-identical to the q8cache's.
 * Replaces the HIP backend's upload (e2.c src/gpu/hip/forward.c:28-64). */
int e2cuda_w8_from_q8w(const e2cuda_q8w *q, e2cuda_w8 *out);
/* The same from a plain row-major int8 [N][K] host matrix and its N row scales. */
int e2cuda_w8_from_int8(const int8_t *w, const float *scale, int N, int K, e2cuda_w8 *out);
void e2cuda_w8_free(e2cuda_w8 *w);

/* ---- q8cache (.e8cq) model-cache files (A11). The reference's format (e2.c src/q8cache.c:1-12) is
 * read and written byte-compatibly for kinds 1-3 (bf16, f32, e2_q8w). Kind 4 is an int8 weight in the
 * e2cuda_w8 device layout (int8 [rows][ld], then fp32 scale [rows]; dims N, K, rows, ld), loaded with
 * one host-to-device copy and no repack. A file holding a kind-4 entry is version 2; one without is
 * version 1, which the reference's reader accepts. Calls return 0 / -1 (NULL) with e2cuda_last_error(). */
enum { E2CUDA_Q8C_BF16 = 1, E2CUDA_Q8C_F32 = 2, E2CUDA_Q8C_Q8W = 3, E2CUDA_Q8C_W8 = 4 };
typedef struct e2cuda_q8c e2cuda_q8c;
typedef struct e2cuda_q8c_writer e2cuda_q8c_writer;
/* Map a cache and check every index entry before any is used (q8c_read_open, src/q8cache.c:242-317). */
e2cuda_q8c *e2cuda_q8c_open(const char *path);
void e2cuda_q8c_close(e2cuda_q8c *c); /* q8c_read_close, src/q8cache.c:319 */
int e2cuda_q8c_version(const e2cuda_q8c *c);
int e2cuda_q8c_count(const e2cuda_q8c *c);
/* entry i's name (valid until close), kind, rank, dims (zero past the rank) and blob size */
int e2cuda_q8c_entry(const e2cuda_q8c *c, int i, const char **name, int *kind, int *ndim, int64_t dims[4],
                     uint64_t *nbytes);
/* the blob stored under `name` as `kind`, pointing into the mapping (q8c_get, src/q8cache.c:329-349) */
const void *e2cuda_q8c_get(const e2cuda_q8c *c, const char *name, int kind, size_t *nbytes);
/* a kind-3 entry as a borrowed e2_q8w pointing into the mapping, unclamped (q8c_get_q8w,
 * src/q8cache.c:357-385) */
int e2cuda_q8c_get_q8w(const e2cuda_q8c *c, const char *name, e2cuda_q8w *q);
/* a kind-4 entry copied to the device as is; a kind-3 entry repacked as e2cuda_w8_from_q8w does */
int e2cuda_q8c_upload_w8(const e2cuda_q8c *c, const char *name, e2cuda_w8 *out);
/* Writer: blobs stream to a temporary file beside `path`; the commit appends the index, rewrites the
 * header and renames the file into place; abort (or a failed commit) leaves an existing file
 * untouched (q8c_write_open / q8c_write_close / q8c_write_abort, src/q8cache.c:61-80,183-221). */
e2cuda_q8c_writer *e2cuda_q8c_create(const char *path);
/* a dense kind-1/2 tensor; nbytes must be its element count times 2 or 4 */
int e2cuda_q8c_put(e2cuda_q8c_writer *w, const char *name, int kind, int ndim, const int64_t *dims, const void *p,
                   size_t nbytes);
int e2cuda_q8c_put_q8w(e2cuda_q8c_writer *w, const char *name, const e2cuda_q8w *q); /* kind 3, q8c_put_q8w :163-181 */
int e2cuda_q8c_put_w8(e2cuda_q8c_writer *w, const char *name, const e2cuda_q8w *q);  /* kind 4, repacked on the host */
int e2cuda_q8c_commit(e2cuda_q8c_writer *w); /* frees the writer */
void e2cuda_q8c_abort(e2cuda_q8c_writer *w); /* frees the writer */
/* Copy a cache with every kind-3 weight rewritten as kind 4 and every other entry byte for byte:
 * the step an exporter (e2.c tools/export_cache.c) adds to write a cache that loads without repack. */
int e2cuda_q8c_convert(const char *in, const char *out);

/* ------------------------------------------------------------------ op API (device pointers) */
/* Activation quantiser (A1), e2.c src/int8.c:178-209 / src/kernels_i8_avx512_vnni.c:312-366:
 * per block of `ablk` elements (ablk = K: per-token scales), amax of the input clamped to [lo, hi]
 * (-INFINITY/INFINITY: no clamp), scale = amax/127 (1 for an all-zero block), q = round(x*127/amax).
 * x [M][K] fp32 -> q [M][K] signed int8, scales [M][K/ablk]. K and ablk multiples of 16. */
int e2cuda_quantize_rows(const float *x, int8_t *q, float *scales, int M, int K, int ablk, float lo,
                         float hi, void *stream);

/* Optional epilogue of e2cuda_i8_gemm. */
typedef struct e2cuda_epilogue {
    const float *residual; /* y = gemm + residual[m * ld_residual + n] (NULL: none)              */
    int ld_residual;
    int32_t *dots;         /* debug: raw int32 block dots [M][N][K/ablk] instead of y (NULL: off) */
} e2cuda_epilogue;

/* W8A8 GEMM (A3), e2.c src/kernels_i8_avx512_vnni.c:276-307: for n in [n0, n1),
 *   y[m * ldy + n] = clamp(sum_b fma-fold float(dot_b(qa[m], w[n])) * (a_scales[m][b] * w.scale[n]))
 * bit-identical to the reference kernel. ablk = K (per-token scales, the fast path) or a multiple of
 * 128 dividing K. For short activation matrices (M <= 256) against long weights the call may use a
 * weight-streaming kernel that keeps a small zeroed device workspace per (device, stream): it is
 * allocated by the first such call on a stream that is not being captured (make one before
 * capturing a graph on that stream) and held until the process exits. With M <= 32 and a short
 * weight the call launches with programmatic dependent launch (E2C_PDL_SMALL=0: off) and requests
 * the weight's first tiles before waiting for the stream's previous kernel: a weight must not be
 * written by a kernel on the stream that signals its dependents early. */
int e2cuda_i8_gemm(const e2cuda_w8 *w, const int8_t *qa, const float *a_scales, int M, int ablk,
                   int n0, int n1, const e2cuda_epilogue *ep, float *y, int ldy, void *stream);

/* Quantise-then-GEMM with no allocation. This entry point has no counterpart in the reference. e2.c
 * quantises into its model workspace (ws.qa) and then runs the GEMM tiles over it (gemm_segs /
 * gemm_quant_phase, e2.c src/text.c:321-411). This call does the same two steps without any
 * buffer from the caller or the library, for callers that cannot let a library allocate device
 * memory. Typical reasons:
 *   - a serving process's own allocator already holds the device memory it budgeted;
 *   - cudaMalloc/cudaFree may block the calling thread and synchronise the device;
 *   - the host wants a fixed, known device footprint.
 *
 * What it computes: y[m * ldy + n] for n in [0, w->N) — e2cuda_quantize_rows(x, ablk, no clamp)
 * followed by e2cuda_i8_gemm with the F32 epilogue, i.e. the same result.
 *   - x is device fp32 [M][w->K]; w->K must be a multiple of 16.
 *   - ablk is w->K (per-token scales) or a multiple of 128 dividing w->K.
 *
 * Scratch. The quantised activations and this call's status word live in one fixed array of
 * E2CUDA_NOALLOC_SCRATCH_BYTES (8 MiB). Each GPU reserves it when it loads this library's device
 * code and keeps it until the process exits.
 *   - The call needs 256 + M*K bytes (rounded up to 256) + 4*M*K/ablk bytes. A larger M is rejected
 *     with an error: split the rows into smaller calls.
 *   - Every call on a device shares the array, and it keeps the last call's contents. The status
 *     word is cleared at the start of each call; everything else is rewritten before it is read.
 *     Calls that overlap on the GPU (other streams, other host threads) race on it: serialise them.
 *   - The first call on each device looks up the array's device address, with that device current.
 *     Make that first call before any stream capture.
 *
 * The call is queued on `stream`, then synchronises `stream` to read its device status; it returns
 * once y is written. A stream that is being captured is refused with an error before anything is
 * queued, since the synchronisation would invalidate the capture. Calls no cudaMalloc, cudaFree or
 * allocating library routine. */
#define E2CUDA_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)
int e2cuda_i8_linear_noalloc(const e2cuda_w8 *w, const float *x, int M, int ablk, float *y, int ldy,
                             void *stream);

/* bf16 attention (A8), full bidirectional over the valid keys of each sequence, GQA with one KV
 * head: q [B*S][H*256], k [B*S][256], vt [B][256][ldvt] (V transposed, ldvt >= S, multiple of 8),
 * valid [B*S] or NULL -> ctx fp32 [B*S][H*256]. scale multiplies the logits. */
int e2cuda_attention(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid,
                     float *ctx, int B, int S, int H, float scale, void *stream);
/* The same for head dim D = 64 or 256 and KV key/value heads (KV divides H; query head h attends with
 * KV head h / (H / KV)): q [B*S][H*D], k [B*S][KV*D], vt [B][KV*D][ldvt] -> ctx fp32 [B*S][H*D]. D = 64
 * with KV = H is the vision tower's attention (e2.c src/vision.c:540-571: 12 heads of 64, scale 1,
 * up to 2520 patches); D = 256 with KV = 1 is e2cuda_attention. */
int e2cuda_attention_gqa(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid,
                         float *ctx, int B, int S, int H, int KV, int D, float scale, void *stream);
/* The same with a sliding window (e2.c's attention_blocked / attn_rows with L->sliding, src/text.c:
 * 656-661,723-729): query i attends to keys j with |i - j| <= window; window < 0 attends to every key.
 * D is 64, 256 or 512 (512: e2.c's full-attention layers; each 128-query tile runs as two halves of
 * the value dimensions). */
int e2cuda_attention_window(const void *q, const void *k, const void *vt, int ldvt, const uint8_t *valid,
                            float *ctx, int B, int S, int H, int KV, int D, float scale, int window, void *stream);

/* ------------------------------------------------------------------ fused FFN block (config 1) */
typedef struct e2cuda_ffn e2cuda_ffn;
/* y = down(quant(GELU_tanh(gate(q)) * up(q))) + x with q = quant(rmsnorm(x) * gamma), e2.c
 * src/text.c:893-903 + gate_quant :424-468, per-token activation scales. gate/up [I][D], down
 * [D][I] host e2_q8w; gamma [D] host. */
e2cuda_ffn *e2cuda_ffn_create(const e2cuda_q8w *gate, const e2cuda_q8w *up, const e2cuda_q8w *down,
                              const float *gamma, float eps, int max_tokens);
void e2cuda_ffn_destroy(e2cuda_ffn *f);
/* x, y device fp32 [M][D] (M <= max_tokens). */
int e2cuda_ffn_forward(e2cuda_ffn *f, const float *x, int M, float *y, void *stream);

/* ------------------------------------------------------------------ drop-ins on host buffers */
/* Exactly the reference's op signatures (e2_i8_gemm_fn, e2_i8_quantize), biased q+128 bytes, so
 * e2.c can install them in its kernel registry (e2.c src/kernels.c:438-459). Each call copies its
 * operands to the device and its result back; weights are uploaded once per distinct e2_q8w and
 * cached. ablk for the quantiser is e2cuda_set_act_block's (default 128, like E2_I8_BLOCK); the
 * GEMM infers it from w->K / w->nblocks. Failures are reported through e2cuda_last_error(). */
void e2cuda_set_act_block(int ablk);
void e2cuda_i8_quantize_host(int8_t *out, float *scales, const float *x, int M, int K, float lo,
                             float hi);
void e2cuda_i8_gemm_host(float *y, const int8_t *qa, const float *a_scales, const e2cuda_q8w *w,
                         int M, int N, int n0, int n1);
/* Drop every cached weight upload (call before freeing the e2_q8w arrays they mirror). */
void e2cuda_host_cache_clear(void);

/* ------------------------------------------------------------------ the synthetic encoder (config 2) */
typedef struct e2cuda_encoder e2cuda_encoder;

typedef struct e2cuda_encoder_desc {
    int n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab, dense_hidden, out_dim;
    int max_seq;        /* longest sequence a call may pass (RoPE table size)                        */
    int ablk;           /* activation block: hidden (per token, default when 0) or 128                */
    float rope_theta, eps, attn_scale, embed_scale;
    /* host arrays, copied at create time */
    const int8_t *table;          /* [vocab][hidden] int8 token table (F7)                           */
    const float *table_scale;     /* [vocab]                                                          */
    const e2cuda_q8w *wq, *wk, *wv, *wo, *wg, *wu, *wd; /* [n_layers] each                           */
    const float *const *input_ln, *const *post_attn_ln, *const *pre_ffn_ln, *const *post_ffn_ln;
    const float *const *q_norm, *const *k_norm;         /* [n_layers] pointers to [head_dim]          */
    const float *final_norm;
    const e2cuda_q8w *dense1, *dense2;                  /* hidden -> dense_hidden -> out_dim           */
} e2cuda_encoder_desc;

/* Uploads everything once. max_tokens bounds batch * seq_len of one device pass (larger batches
 * are chunked by whole sequences). Returns NULL on failure. Restrictions of this build: head_dim
 * 256, one KV head, hidden a multiple of 128 up to 1024. */
e2cuda_encoder *e2cuda_encoder_create(const e2cuda_encoder_desc *d, int max_tokens);
void e2cuda_encoder_destroy(e2cuda_encoder *e);
/* Host buffers, e2_hip_text_embed_batch's contract (e2.c include/e2hip.h:44-50): ids [batch][seq_len],
 * valid NULL or [batch][seq_len] (nonzero keeps a token), out [batch][out_dim] unit vectors; a
 * sequence with no valid token yields exact zeros. Positions restart per sequence. */
int e2cuda_encoder_embed_batch(e2cuda_encoder *e, const int32_t *ids, const uint8_t *valid,
                               int batch, int seq_len, float *out);
/* The same on device buffers, stream-ordered (call e2cuda_check before reading d_out). The first
 * call for a (batch, seq_len) shape runs eagerly; later calls replay a captured CUDA graph. */
int e2cuda_encoder_embed_batch_device(e2cuda_encoder *e, const int32_t *d_ids, const uint8_t *d_valid,
                                      int batch, int seq_len, float *d_out, void *stream);
/* Calls served, kernels in the last pass, wall time of the last host call (e2hip.h:62-64). */
int e2cuda_encoder_stats(e2cuda_encoder *e, long *calls, long *kernels_last, double *last_ms);

/* ------------------------------------------------------------------ e2.c's own text tower */
/* EmbeddingGemma-2's text tower as e2.c runs it (src/text.c:924-984): per layer RMSNorm ->
 * attention (q/k/v projections, q/k/v RMSNorm, RoPE, 4 query heads, head dim 256 with 2 KV heads and
 * a 512-key sliding window, or head dim 512 with 1 KV head and full attention; scale 1.0) ->
 * residual norms -> gated GELU-tanh MLP -> residual norms -> per-layer-embedding (PLE) block ->
 * layer scalar; PLE projection of the input embeddings; final norm, embed_proj to out_dim, masked
 * mean pool, L2. This is the device half of the backend e2hip.h gives AMD GPUs (e2hip.h:32-64):
 * e2.c's loader fills the description from its e2_model (the e2_q8w weights it built, the bf16 token
 * table it mapped, the fp32 norm vectors), the library uploads it once. */
typedef struct e2cuda_text e2cuda_text;

typedef struct e2cuda_text_layer {
    const e2cuda_q8w *q, *k, *v, *o, *gate, *up, *down, *ple_gate, *ple_proj; /* e2_layer.q8_*      */
    const float *input_ln, *post_attn_ln, *pre_ffn_ln, *post_ffn_ln, *ple_norm; /* [hidden]        */
    const float *q_norm, *k_norm;                                               /* [head_dim]      */
    float layer_scalar;
    int head_dim, n_kv_heads; /* 256 / 2 (sliding) or 512 / 1 (full) in EmbeddingGemma-2        */
    int window;               /* keys with |i - j| <= window attend; < 0: full attention          */
    float rope_theta;
} e2cuda_text_layer;

typedef struct e2cuda_text_desc {
    int n_layers, hidden, intermediate, ple_dim, n_heads, vocab, out_dim;
    int max_seq;  /* longest sequence a call may pass (RoPE table size; e2.c: 2048)               */
    int ablk;     /* activation block: 128 (e2.c's E2_I8_BLOCK; the default when 0) or hidden    */
    float eps, embed_scale, ple_scale;
    const uint16_t *embed_tokens;     /* bf16 [vocab][hidden], copied at create time              */
    const e2cuda_q8w *ple_model_proj; /* [n_layers * ple_dim][hidden]                             */
    const e2cuda_q8w *embed_proj;     /* [out_dim][hidden]                                        */
    const float *ple_proj_norm;       /* [ple_dim]                                                */
    const float *final_norm;          /* [hidden]                                                 */
    const e2cuda_text_layer *layers;  /* [n_layers]                                               */
} e2cuda_text_desc;

/* Uploads everything once (e2_hip_create, e2hip.h:32). max_tokens bounds batch * seq_len of one
 * device pass (larger batches are chunked by whole sequences). NULL on failure. */
e2cuda_text *e2cuda_text_create(const e2cuda_text_desc *d, int max_tokens);
void e2cuda_text_destroy(e2cuda_text *t);
/* One sequence of n_ids tokens -> one out_dim unit vector (e2_hip_text_embed, e2hip.h:39). */
int e2cuda_text_embed(e2cuda_text *t, const int32_t *ids, int n_ids, float *out);
/* batch x seq_len tokens, valid NULL or nonzero-keeps, positions restart per sequence; all-invalid
 * sequences give zeros (e2_hip_text_embed_batch, e2hip.h:44-50). Host buffers. */
int e2cuda_text_embed_batch(e2cuda_text *t, const int32_t *ids, const uint8_t *valid, int batch, int seq_len,
                            float *out);
/* The same on device buffers, stream-ordered (e2cuda_check before reading d_out). */
int e2cuda_text_embed_batch_device(e2cuda_text *t, const int32_t *d_ids, const uint8_t *d_valid, int batch,
                                   int seq_len, float *d_out, void *stream);
/* Calls served, kernels in the last pass, wall time of the last host call (e2_hip_stats, e2hip.h:62). */
int e2cuda_text_stats(e2cuda_text *t, long *calls, long *kernels_last, double *last_ms);

#ifdef __cplusplus
}
#endif
#endif
