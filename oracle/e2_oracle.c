/* e2_oracle.c — plain-C restatement of the reference e2.c kernels on the int8 hot path.
 * TEST INFRASTRUCTURE ONLY: the checker for the e2cuda kernels, never part of the product.
 *
 * Built with -O3 -fno-fast-math -ffp-contract=off so every fp32 operation rounds exactly where the
 * source says it does; fused multiply-adds are spelled fmaf() where the reference's AVX-512 kernels
 * issue one. File:line citations are into the reference project (Damix48/e2.c).
 */
#include "e2_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ quantiser forms
 * The reference builds libe2 with -ffast-math (CMakeLists.txt:110). In the compiled activation
 * quantiser (src/kernels_i8_avx512_vnni.c:312-366) that turns `sc = amax / 127.0f` into a multiply
 * by the rounded reciprocal of 127, and `1.0f / sc` into `127.0f / amax`. The weight quantiser
 * (src/int8.c:19-66) gets the same scale form. tests/test_oracle.py pins both against the
 * reference build, element for element. */
static const float k_inv127 = 1.0f / 127.0f; /* fl(1/127) = 0x1.020408p-7 */

static inline float q_scale(float amax) { return amax > 0.f ? amax * k_inv127 : 1.0f; }
static inline float q_inv(float amax) { return amax > 0.f ? 127.0f / amax : 1.0f; }
static inline int q_round(float v) {
    int r = (int)lrintf(v); /* round to nearest even, as cvtps2dq under the default MXCSR */
    if (r > 127) r = 127;
    if (r < -127) r = -127;
    return r;
}

/* src/int8.c:178-209 / src/kernels_i8_avx512_vnni.c:312-366. */
void e2o_quantize_blocks(int8_t *out, float *scales, const float *x, int M, int K, int ablk, float lo,
                         float hi) {
    const int nb = (K + ablk - 1) / ablk;
    const int clamp = lo > -INFINITY || hi < INFINITY;
    for (int m = 0; m < M; m++) {
        const float *xr = x + (size_t)m * K;
        int8_t *orow = out + (size_t)m * K;
        for (int b = 0; b < nb; b++) {
            const int k0 = b * ablk;
            const int k1 = k0 + ablk < K ? k0 + ablk : K;
            float amax = 0.f;
            for (int k = k0; k < k1; k++) {
                float v = xr[k];
                if (clamp) v = v < lo ? lo : (v > hi ? hi : v);
                const float a = fabsf(v);
                if (a > amax) amax = a;
            }
            const float inv = q_inv(amax);
            for (int k = k0; k < k1; k++) {
                float v = xr[k];
                if (clamp) v = v < lo ? lo : (v > hi ? hi : v);
                orow[k] = (int8_t)(q_round(v * inv) + 128);
            }
            scales[(size_t)m * nb + b] = q_scale(amax);
        }
    }
}

void e2o_quantize_rows_signed(int8_t *out, float *scales, const float *x, int M, int K, int ablk) {
    e2o_quantize_blocks(out, scales, x, M, K, ablk, -INFINITY, INFINITY);
    for (size_t i = 0; i < (size_t)M * K; i++) out[i] = (int8_t)((uint8_t)out[i] ^ 0x80u);
}

/* ------------------------------------------------------------------ weights
 * src/int8.c:19-66: per-row scale, round to nearest, saturate to +-127, pack quad-interleaved
 * [N/8][K/4][8][4] with Npad = N rounded up to 8, and per-block sums bsq[b][Npad]. */
int e2o_q8w_from_f32(e2o_q8w *q, const float *w, int N, int K, int ablk) {
    memset(q, 0, sizeof *q);
    q->N = N;
    q->K = K;
    const int nblocks = (K + ablk - 1) / ablk;
    const int kq = (K + 3) / 4;
    const int Npad = (N + 7) & ~7;
    q->nblocks = nblocks;
    q->Npad = Npad;
    q->out_min = -1e31f;
    q->out_max = 1e31f;
    q->w = calloc((size_t)(Npad / 8) * kq * 32, 1);
    q->scale = calloc((size_t)Npad, sizeof(float));
    q->bsq = calloc((size_t)nblocks * Npad, sizeof(int32_t));
    if (!q->w || !q->scale || !q->bsq) {
        e2o_q8w_free(q);
        return -1;
    }
    for (int n = 0; n < N; n++) {
        const float *wr = w + (size_t)n * K;
        float amax = 0.f;
        for (int k = 0; k < K; k++) {
            const float a = fabsf(wr[k]);
            if (a > amax) amax = a;
        }
        const float inv = q_inv(amax);
        for (int b = 0; b < nblocks; b++) {
            int32_t sum = 0;
            const int k0 = b * ablk, k1 = k0 + ablk < K ? k0 + ablk : K;
            for (int k = k0; k < k1; k++) {
                const int r = q_round(wr[k] * inv);
                q->w[(size_t)(n >> 3) * kq * 32 + (size_t)(k >> 2) * 32 + (n & 7) * 4 + (k & 3)] =
                    (int8_t)r;
                sum += r;
            }
            q->bsq[(size_t)b * Npad + n] = sum;
        }
        q->scale[n] = q_scale(amax);
    }
    return 0;
}

void e2o_q8w_free(e2o_q8w *q) {
    if (!q->borrowed) {
        free(q->w);
        free(q->scale);
        free(q->bsq);
    }
    memset(q, 0, sizeof *q);
}

void e2o_q8w_unpack(const e2o_q8w *q, int8_t *wk) {
    const int N = q->N, K = q->K, kq = (K + 3) / 4;
    for (int n = 0; n < N; n++)
        for (int k = 0; k < K; k++)
            wk[(size_t)n * K + k] =
                q->w[(size_t)(n >> 3) * kq * 32 + (size_t)(k >> 2) * 32 + (n & 7) * 4 + (k & 3)];
}

/* ------------------------------------------------------------------ int8 GEMM
 * src/kernels_i8_avx512_vnni.c:84-125,276-307 (and the scalar definition src/int8.c:114-171): the
 * per-block dot sum_k (a-128)*w is exact int32 (acc - 128*bsq in the kernel); it is converted to
 * float and folded with one FMA per block, f = fma(float(dot), as*ws, f), blocks in order; the store
 * clamps to [out_min, out_max]. */
void e2o_i8_gemm(float *y, const int8_t *qa, const float *as, const e2o_q8w *w, int M, int N, int n0,
                 int n1, int ablk) {
    const int K = w->K, nb = w->nblocks, kq = (K + 3) / 4;
    int8_t *wr = malloc((size_t)K);
    if (!wr) return;
    for (int n = n0; n < n1; n++) {
        /* this row's weights, un-interleaved once (the arithmetic does not depend on the layout) */
        const int8_t *wb = w->w + (size_t)(n >> 3) * kq * 32 + (n & 7) * 4;
        for (int k = 0; k < K; k++) wr[k] = wb[(size_t)(k >> 2) * 32 + (k & 3)];
        const float ws = w->scale[n];
        for (int m = 0; m < M; m++) {
            const uint8_t *ar = (const uint8_t *)qa + (size_t)m * K;
            float f = 0.f;
            for (int b = 0; b < nb; b++) {
                const int k0 = b * ablk, k1 = k0 + ablk < K ? k0 + ablk : K;
                int32_t d = 0;
                for (int k = k0; k < k1; k++) d += ((int)ar[k] - 128) * (int)wr[k];
                f = fmaf((float)d, as[(size_t)m * nb + b] * ws, f);
            }
            if (f < w->out_min) f = w->out_min;
            if (f > w->out_max) f = w->out_max;
            y[(size_t)m * N + n] = f;
        }
    }
    free(wr);
}

void e2o_i8_gemm_plain(float *y, int32_t *dots, const int8_t *qa, const float *as, const int8_t *w,
                       const float *ws, int M, int N, int K, int ablk, float out_min, float out_max) {
    const int nb = (K + ablk - 1) / ablk;
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) {
            const int8_t *ar = qa + (size_t)m * K, *wr = w + (size_t)n * K;
            float f = 0.f;
            for (int b = 0; b < nb; b++) {
                const int k0 = b * ablk, k1 = k0 + ablk < K ? k0 + ablk : K;
                int32_t d = 0;
                for (int k = k0; k < k1; k++) d += (int)ar[k] * (int)wr[k];
                if (dots) dots[((size_t)m * N + n) * nb + b] = d;
                f = fmaf((float)d, as[(size_t)m * nb + b] * ws[n], f);
            }
            if (f < out_min) f = out_min;
            if (f > out_max) f = out_max;
            if (y) y[(size_t)m * N + n] = f;
        }
}

/* ------------------------------------------------------------------ fp32 row ops
 * src/kernels.c:76-87 (rmsnorm), :144-171 (norm_split / norm_add): inv = 1/sqrt(mean(x^2) + eps),
 * x*inv*gamma. The reference's -ffast-math AVX-512 build sums in 16 lanes and may use an
 * rsqrt+Newton step: these agree with it to a few ulp, and tests gate them by tolerance. */
static float row_inv(const float *x, int D, float eps) {
    float ss = 0.f;
    for (int d = 0; d < D; d++) ss += x[d] * x[d];
    return 1.0f / sqrtf(ss / (float)D + eps);
}

void e2o_rmsnorm(float *x, int M, int D, const float *gamma, float eps) {
    for (int m = 0; m < M; m++) {
        float *row = x + (size_t)m * D;
        const float inv = row_inv(row, D, eps);
        for (int d = 0; d < D; d++) row[d] = gamma ? row[d] * inv * gamma[d] : row[d] * inv;
    }
}

void e2o_norm_split(float *x, float *res, int rows, int D, const float *gamma, float eps) {
    for (int r = 0; r < rows; r++) {
        float *xr = x + (size_t)r * D, *rr = res + (size_t)r * D;
        const float inv = row_inv(xr, D, eps);
        for (int d = 0; d < D; d++) {
            const float v = xr[d];
            rr[d] = v;
            xr[d] = v * inv * (gamma ? gamma[d] : 1.0f);
        }
    }
}

void e2o_norm_add(float *out, const float *src, const float *res, int rows, int D, const float *gamma,
                  float eps) {
    for (int r = 0; r < rows; r++) {
        const float *sr = src + (size_t)r * D, *rr = res + (size_t)r * D;
        float *orow = out + (size_t)r * D;
        const float inv = row_inv(sr, D, eps);
        for (int d = 0; d < D; d++) orow[d] = sr[d] * inv * (gamma ? gamma[d] : 1.0f) + rr[d];
    }
}

/* src/kernels_avx512.c:19-44: exp by range reduction to r = x - n ln2 (two-constant Cody-Waite)
 * and a degree-5 polynomial, 2^n by exponent-field construction. */
static float exp_poly(float x) {
    if (x < -87.0f) x = -87.0f;
    if (x > 88.0f) x = 88.0f;
    const float t = x * 1.4426950408889634f;
    const float n = rintf(t);
    float r = fmaf(-n, 0.6931471805599453f, x);
    r = fmaf(-n, -1.904654299957768e-9f, r);
    float p = 1.9875691500e-4f;
    p = fmaf(p, r, 1.3981999507e-3f);
    p = fmaf(p, r, 8.3334519073e-3f);
    p = fmaf(p, r, 4.1665795894e-2f);
    p = fmaf(p, r, 1.6666665459e-1f);
    p = fmaf(p, r, 5.0000001201e-1f);
    p = fmaf(p, r * r, r);
    p = p + 1.0f;
    const int ni = (int)lrintf(n);
    const uint32_t bits = (uint32_t)(ni + 127) << 23;
    float sc;
    memcpy(&sc, &bits, 4);
    return p * sc;
}

/* src/kernels_avx512.c:46-55: tanh(z) = sign(z) (1 - 2/(exp(2|z|)+1)), 1 beyond |z| > 15. */
static float tanh_poly(float z) {
    const float a = fabsf(z);
    const float e = exp_poly(a + a);
    float r = 1.0f - 2.0f / (e + 1.0f);
    if (a > 15.0f) r = 1.0f;
    return z < 0.f ? -r : r; /* xor of the sign bit; tanh(-0) = -0 */
}

/* src/kernels_avx512.c:186-203: 0.5 v (1 + tanh(c (v + 0.044715 v^3))), v^3 = (v v) v, the inner
 * sum as one FMA. */
void e2o_gelu_tanh(float *x, size_t n) {
    for (size_t i = 0; i < n; i++) {
        const float v = x[i];
        const float v3 = (v * v) * v;
        const float inner = 0.7978845608028654f * fmaf(0.044715f, v3, v);
        const float t = tanh_poly(inner);
        x[i] = (0.5f * v) * (1.0f + t);
    }
}

/* src/kernels_avx512.c:205-230 (exp as above; the sum order differs, gated by tolerance). */
void e2o_softmax(float *x, int n) {
    if (n <= 0) return;
    float m = x[0];
    for (int i = 1; i < n; i++)
        if (x[i] > m) m = x[i];
    float s = 0.f;
    for (int i = 0; i < n; i++) {
        x[i] = exp_poly(x[i] - m);
        s += x[i];
    }
    const float inv = 1.0f / s;
    for (int i = 0; i < n; i++) x[i] *= inv;
}

/* src/kernels.c:112-126 (rotate-half over `block`, position = row / ngroups). */
void e2o_rope_rows(float *x, int r0, int r1, int ngroups, int head_dim, int block, const float *cs,
                   const float *sn) {
    const int half = block / 2;
    for (int r = r0; r < r1; r++) {
        float *v = x + (size_t)r * head_dim;
        const float *c = cs + (size_t)(r / ngroups) * head_dim;
        const float *s = sn + (size_t)(r / ngroups) * head_dim;
        for (int b = 0; b < head_dim; b += block)
            for (int i = 0; i < half; i++) {
                /* the AVX-512 form (src/kernels_avx512.c:246-250): fmsub / fmadd */
                const float a = v[b + i], y = v[b + half + i];
                v[b + i] = fmaf(a, c[b + i], -(y * s[b + i]));
                v[b + half + i] = fmaf(a, s[b + i], y * c[b + i]);
            }
    }
}

/* src/text.c:483-506. */
void e2o_rope_tables(float *cs, float *sn, int npos, int head_dim, float theta) {
    for (int p = 0; p < npos; p++) {
        float *c = cs + (size_t)p * head_dim, *s = sn + (size_t)p * head_dim;
        for (int i = 0; i < head_dim / 2; i++) {
            const float inv = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
            const float f = (float)p * inv;
            c[i] = c[i + head_dim / 2] = cosf(f);
            s[i] = s[i + head_dim / 2] = sinf(f);
        }
    }
}

/* src/kernels.c:210-243: C = A B, rows [m0, m1), every element accumulated over k in order. */
void e2o_sgemm_nn(float *C, int ldc, const float *A, int lda, const float *B, int ldb, int M, int N,
                  int K, int m0, int m1) {
    (void)M;
    for (int m = m0; m < m1; m++) {
        float *crow = C + (size_t)m * ldc;
        for (int n = 0; n < N; n++) crow[n] = 0.f;
        for (int k = 0; k < K; k++) {
            const float av = A[(size_t)m * lda + k];
            const float *b = B + (size_t)k * ldb;
            for (int n = 0; n < N; n++) crow[n] += av * b[n];
        }
    }
}

/* src/kernels.c:29-39. */
void e2o_meanpool(float *out, const float *x, int M, int D, const uint8_t *valid) {
    memset(out, 0, sizeof(float) * (size_t)D);
    int cnt = 0;
    for (int m = 0; m < M; m++) {
        if (valid && !valid[m]) continue;
        for (int d = 0; d < D; d++) out[d] += x[(size_t)m * D + d];
        cnt++;
    }
    if (cnt > 0)
        for (int d = 0; d < D; d++) out[d] /= (float)cnt;
}

/* src/kernels.c:22-27. */
void e2o_l2norm(float *x, int n) {
    float s = 0.f;
    for (int i = 0; i < n; i++) s += x[i] * x[i];
    const float inv = 1.f / sqrtf(s);
    for (int i = 0; i < n; i++) x[i] *= inv;
}

static void e2o_mul(float *a, const float *b, size_t n) {
    for (size_t i = 0; i < n; i++) a[i] *= b[i];
}

/* ------------------------------------------------------------------ synthetic data */
uint64_t e2o_splitmix64(uint64_t *state) {
    uint64_t z = (*state += 0x9e3779b97f4a7c15ull);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

void e2o_fill_normal(float *dst, size_t n, uint64_t seed, float mean, float std) {
    uint64_t st = seed;
    for (size_t i = 0; i < n; i += 2) {
        /* u1 in (0, 1], u2 in [0, 1): 53-bit uniforms */
        const double u1 = ((double)(e2o_splitmix64(&st) >> 11) + 1.0) * 0x1.0p-53;
        const double u2 = (double)(e2o_splitmix64(&st) >> 11) * 0x1.0p-53;
        const double r = sqrt(-2.0 * log(u1));
        dst[i] = (float)(mean + std * r * cos(6.283185307179586 * u2));
        if (i + 1 < n) dst[i + 1] = (float)(mean + std * r * sin(6.283185307179586 * u2));
    }
}

/* ------------------------------------------------------------------ the port's kernel table */
static int g_port_ablk = 128; /* 0: per-row (block = K of each call) */

static void port_quantize(int8_t *out, float *scales, const float *x, int M, int K, float lo, float hi) {
    e2o_quantize_blocks(out, scales, x, M, K, g_port_ablk ? g_port_ablk : K, lo, hi);
}
static void port_gemm(float *y, const int8_t *qa, const float *as, const e2o_q8w *w, int M, int N,
                      int n0, int n1) {
    e2o_i8_gemm(y, qa, as, w, M, N, n0, n1, g_port_ablk ? g_port_ablk : w->K);
}
static int port_q8w(e2o_q8w *q, const float *w, int N, int K) {
    return e2o_q8w_from_f32(q, w, N, K, g_port_ablk ? g_port_ablk : K);
}

const e2o_kernels *e2o_port_kernels(int ablk) {
    static e2o_kernels k;
    g_port_ablk = ablk;
    k.name = "port";
    k.ablk = ablk;
    k.quantize = port_quantize;
    k.gemm = port_gemm;
    k.q8w_from_f32 = port_q8w;
    k.q8w_free = e2o_q8w_free;
    k.rmsnorm = e2o_rmsnorm;
    k.norm_split = e2o_norm_split;
    k.norm_add = e2o_norm_add;
    k.gelu_tanh = e2o_gelu_tanh;
    k.mul = e2o_mul;
    k.softmax = e2o_softmax;
    k.rope_rows = e2o_rope_rows;
    k.sgemm_nn = e2o_sgemm_nn;
    k.meanpool = e2o_meanpool;
    k.l2norm = e2o_l2norm;
    k.parallel = NULL;
    k.nthreads = 1;
    return &k;
}
