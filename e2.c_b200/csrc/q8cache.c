/* q8cache.c — .e8cq model-cache files (A11): the reference's format for kinds 1-3, read and written
 * byte-compatibly (e2.c src/q8cache.c:1-12 layout, :163-206 writer, :242-280 reader checks), plus
 * kind 4, an int8 weight stored in this library's device layout so that loading it is one copy to
 * the GPU with no repack.
 *
 *   offset 0    u32 magic "E8CQ", u32 version, u32 n_entries, u32 index_offset
 *   offset 16   the blobs, each padded with zeros to a multiple of 16 bytes
 *   index       n_entries x { char name[96]; u32 kind; u32 ndim; i64 dims[4]; u64 nbytes; u64 off }
 *
 *   kind 1 (bf16), 2 (f32)  the tensor's elements; dims = its shape (rank 0 = one element)
 *   kind 3 (an e2_q8w)      quad-interleaved int8 [Npad/8][ceil(K/4)][8][4], fp32 scale [Npad],
 *                           int32 bsq [nblocks][Npad]; dims = N, K, nblocks, Npad (= N rounded up
 *                           to 8)
 *   kind 4 (device layout)  int8 [rows][ld], K contiguous, zero padded, then fp32 scale [rows];
 *                           dims = N, K, rows (= N rounded up to 16), ld (= K rounded up to 16)
 *
 * A file holding a kind-4 entry carries version 2, which the reference's reader refuses (it
 * accepts version 1 only). A file without one is version 1 and reads back in the reference. The
 * header's 32-bit index offset limits both versions to 4 GiB, as in the reference.
 */
#include <fcntl.h>
#include <limits.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "internal.h"

#define Q8C_MAGIC 0x51433845u /* "E8CQ", little-endian */
#define Q8C_DATA_OFF 16u

enum { NAMELEN = 96, MAXDIM = 4 };

typedef struct {
    char name[NAMELEN];
    uint32_t kind, ndim;
    int64_t dims[MAXDIM];
    uint64_t nbytes, off;
} q8c_entry;
_Static_assert(sizeof(q8c_entry) == 152, "index entry layout of the .e8cq format");

struct e2cuda_q8c {
    int fd;
    const uint8_t *base;
    size_t size;
    const q8c_entry *idx;
    uint32_t n, version;
};

struct e2cuda_q8c_writer {
    FILE *f;
    char *path, *tmp;
    uint64_t off;
    q8c_entry *idx;
    size_t n, cap;
    int version;
};

static int64_t round_to(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

/* ------------------------------------------------------------------ sizes of the payloads */
/* bytes of a kind-3 payload, or 0 when the dims do not describe one */
static uint64_t q8w_bytes(const int64_t *d) {
    const int64_t N = d[0], K = d[1], nb = d[2], Npad = d[3];
    if (N <= 0 || K <= 0 || N > INT_MAX || K > INT_MAX || Npad != round_to(N, 8) || nb < 1 || nb > K) return 0;
    return (uint64_t)Npad * (uint64_t)((K + 3) / 4) * 4 + (uint64_t)Npad * 4 + (uint64_t)nb * (uint64_t)Npad * 4;
}
/* bytes of a kind-4 payload, or 0 */
static uint64_t w8_bytes(const int64_t *d) {
    const int64_t N = d[0], K = d[1], rows = d[2], ld = d[3];
    if (N <= 0 || K <= 0 || N > INT_MAX || K > INT_MAX || rows != round_to(N, 16) || ld != round_to(K, 16)) return 0;
    return (uint64_t)rows * (uint64_t)ld + (uint64_t)rows * 4;
}
/* bytes of a kind-1/2 tensor; -1 on overflow */
static int dense_bytes(int kind, uint32_t ndim, const int64_t *d, uint64_t *out) {
    uint64_t n = kind == E2CUDA_Q8C_BF16 ? 2 : 4;
    for (uint32_t i = 0; i < ndim; i++) {
        if (d[i] == 0) {
            n = 0;
            continue;
        }
        if (n && (uint64_t)d[i] > UINT64_MAX / n) return -1;
        n *= (uint64_t)d[i];
    }
    *out = n;
    return 0;
}

/* ------------------------------------------------------------------ reader */
static int entry_ok(const e2cuda_q8c *c, const q8c_entry *e, uint64_t idx_off, const char *path) {
    if (!memchr(e->name, 0, sizeof e->name) || !e->name[0]) {
        e2cu_err("%s: an index entry has an empty or unterminated name", path);
        return -1;
    }
    const uint32_t k = e->kind;
    if (k < E2CUDA_Q8C_BF16 || k > E2CUDA_Q8C_W8 || (k == E2CUDA_Q8C_W8 && c->version < 2)) {
        e2cu_err("%s: %s: unknown kind %u for version %u", path, e->name, k, c->version);
        return -1;
    }
    if (e->ndim > MAXDIM || ((k == E2CUDA_Q8C_Q8W || k == E2CUDA_Q8C_W8) && e->ndim != 4)) {
        e2cu_err("%s: %s: bad rank %u", path, e->name, e->ndim);
        return -1;
    }
    for (uint32_t i = 0; i < e->ndim; i++)
        if (e->dims[i] < 0) {
            e2cu_err("%s: %s: negative dimension", path, e->name);
            return -1;
        }
    if (e->off < Q8C_DATA_OFF || (e->off & 15) || e->off > idx_off || e->nbytes > idx_off - e->off) {
        e2cu_err("%s: %s: blob outside the data area", path, e->name);
        return -1;
    }
    uint64_t want = 0;
    if (k == E2CUDA_Q8C_Q8W) want = q8w_bytes(e->dims);
    else if (k == E2CUDA_Q8C_W8) want = w8_bytes(e->dims);
    else if (dense_bytes((int)k, e->ndim, e->dims, &want)) {
        e2cu_err("%s: %s: element count overflows", path, e->name);
        return -1;
    }
    if ((k == E2CUDA_Q8C_Q8W || k == E2CUDA_Q8C_W8) && !want) {
        e2cu_err("%s: %s: dims do not describe a packed weight", path, e->name);
        return -1;
    }
    if (e->nbytes != want) {
        e2cu_err("%s: %s: blob of %llu bytes, its dims need %llu", path, e->name, (unsigned long long)e->nbytes,
                 (unsigned long long)want);
        return -1;
    }
    return 0;
}

e2cuda_q8c *e2cuda_q8c_open(const char *path) {
    if (!path) {
        e2cu_err("q8c_open: no path");
        return NULL;
    }
    e2cuda_q8c *c = calloc(1, sizeof *c);
    if (!c) {
        e2cu_err("q8c_open: out of host memory");
        return NULL;
    }
    c->fd = open(path, O_RDONLY | O_CLOEXEC);
    struct stat st;
    if (c->fd < 0 || fstat(c->fd, &st) || st.st_size < (off_t)Q8C_DATA_OFF) {
        e2cu_err("%s: cannot open, or shorter than the header", path);
        goto fail;
    }
    c->size = (size_t)st.st_size;
    void *m = mmap(NULL, c->size, PROT_READ, MAP_PRIVATE, c->fd, 0);
    if (m == MAP_FAILED) {
        e2cu_err("%s: mmap failed", path);
        goto fail;
    }
    c->base = m;
    uint32_t hdr[4];
    memcpy(hdr, c->base, sizeof hdr);
    if (hdr[0] != Q8C_MAGIC || hdr[1] < 1 || hdr[1] > 2) {
        e2cu_err("%s: not an .e8cq file of version 1 or 2", path);
        goto fail;
    }
    c->version = hdr[1];
    c->n = hdr[2];
    const uint64_t idx = hdr[3];
    if (idx < Q8C_DATA_OFF || (idx & 15) || idx > c->size || (uint64_t)c->n > (c->size - idx) / sizeof(q8c_entry)) {
        e2cu_err("%s: truncated or misaligned index", path);
        goto fail;
    }
    c->idx = (const q8c_entry *)(c->base + idx);
    for (uint32_t i = 0; i < c->n; i++)
        if (entry_ok(c, &c->idx[i], idx, path)) goto fail;
    return c;
fail:
    e2cuda_q8c_close(c);
    return NULL;
}

void e2cuda_q8c_close(e2cuda_q8c *c) {
    if (!c) return;
    if (c->base) munmap((void *)c->base, c->size);
    if (c->fd >= 0) close(c->fd);
    free(c);
}

int e2cuda_q8c_version(const e2cuda_q8c *c) { return c ? (int)c->version : -1; }
int e2cuda_q8c_count(const e2cuda_q8c *c) { return c ? (int)c->n : -1; }

int e2cuda_q8c_entry(const e2cuda_q8c *c, int i, const char **name, int *kind, int *ndim, int64_t dims[4],
                     uint64_t *nbytes) {
    if (!c || i < 0 || (uint32_t)i >= c->n) {
        e2cu_err("q8c_entry: no entry %d", i);
        return -1;
    }
    const q8c_entry *e = &c->idx[i];
    if (name) *name = e->name;
    if (kind) *kind = (int)e->kind;
    if (ndim) *ndim = (int)e->ndim;
    if (dims)
        for (int d = 0; d < MAXDIM; d++) dims[d] = d < (int)e->ndim ? e->dims[d] : 0;
    if (nbytes) *nbytes = e->nbytes;
    return 0;
}

static const q8c_entry *find(const e2cuda_q8c *c, const char *name) {
    for (uint32_t i = 0; i < c->n; i++)
        if (!strcmp(c->idx[i].name, name)) return &c->idx[i];
    return NULL;
}

const void *e2cuda_q8c_get(const e2cuda_q8c *c, const char *name, int kind, size_t *nbytes) {
    const q8c_entry *e = c && name ? find(c, name) : NULL;
    if (!e) {
        e2cu_err("q8c_get: %s: not in the cache", name ? name : "(null)");
        return NULL;
    }
    if ((int)e->kind != kind) {
        e2cu_err("q8c_get: %s: stored as kind %u, asked for %d", name, e->kind, kind);
        return NULL;
    }
    if (nbytes) *nbytes = (size_t)e->nbytes;
    return c->base + e->off; /* inside the mapping: e2cuda_q8c_open checked every entry */
}

int e2cuda_q8c_get_q8w(const e2cuda_q8c *c, const char *name, e2cuda_q8w *q) {
    if (!q || !e2cuda_q8c_get(c, name, E2CUDA_Q8C_Q8W, NULL)) {
        if (!q) e2cu_err("q8c_get_q8w: no output");
        return -1;
    }
    const q8c_entry *e = find(c, name);
    const uint8_t *p = c->base + e->off;
    memset(q, 0, sizeof *q);
    q->N = (int)e->dims[0];
    q->K = (int)e->dims[1];
    q->nblocks = (int)e->dims[2];
    q->Npad = (int)e->dims[3];
    const size_t nw = (size_t)q->Npad * (size_t)((q->K + 3) / 4) * 4, ns = (size_t)q->Npad * 4;
    q->w = (int8_t *)(uintptr_t)p;
    q->scale = (float *)(uintptr_t)(p + nw);
    q->bsq = (int32_t *)(uintptr_t)(p + nw + ns);
    /* the cache holds no clamp bounds (the reference's loader sets them from the checkpoint) */
    q->out_min = -1e31f;
    q->out_max = 1e31f;
    q->borrowed = 1;
    return 0;
}

int e2cuda_q8c_upload_w8(const e2cuda_q8c *c, const char *name, e2cuda_w8 *out) {
    const q8c_entry *e = c && name ? find(c, name) : NULL;
    if (!e || !out || (e->kind != E2CUDA_Q8C_W8 && e->kind != E2CUDA_Q8C_Q8W)) {
        e2cu_err("q8c_upload_w8: %s: no packed weight of that name", name ? name : "(null)");
        return -1;
    }
    if (e->kind == E2CUDA_Q8C_Q8W) { /* a version-1 entry: repacked on the way */
        e2cuda_q8w q;
        return e2cuda_q8c_get_q8w(c, name, &q) || e2cuda_w8_from_q8w(&q, out) ? -1 : 0;
    }
    const int N = (int)e->dims[0], K = (int)e->dims[1], rows = (int)e->dims[2], ld = (int)e->dims[3];
    const uint8_t *p = c->base + e->off;
    if (e2cu_w8_alloc(out, N, K)) return -1;
    if (out->rows != rows || out->ld != ld) { /* w8_bytes pinned both to the allocator's rounding */
        e2cuda_w8_free(out);
        e2cu_err("q8c_upload_w8: %s: layout %d x %d, the device wants %d x %d", name, rows, ld, out->rows, out->ld);
        return -1;
    }
    if (e2cu_cuda(cudaMemcpy(out->w, p, (size_t)rows * ld, cudaMemcpyHostToDevice), "q8c weight upload") ||
        e2cu_cuda(cudaMemcpy(out->scale, p + (size_t)rows * ld, sizeof(float) * (size_t)rows, cudaMemcpyHostToDevice),
                  "q8c scale upload")) {
        e2cuda_w8_free(out);
        return -1;
    }
    return 0;
}

/* ------------------------------------------------------------------ writer */
e2cuda_q8c_writer *e2cuda_q8c_create(const char *path) {
    if (!path || !path[0]) {
        e2cu_err("q8c_create: no path");
        return NULL;
    }
    e2cuda_q8c_writer *w = calloc(1, sizeof *w);
    const size_t n = strlen(path);
    if (w) {
        w->path = strdup(path);
        w->tmp = malloc(n + 16);
    }
    if (!w || !w->path || !w->tmp) {
        e2cu_err("q8c_create: out of host memory");
        if (w) {
            free(w->path);
            free(w->tmp);
            free(w);
        }
        return NULL;
    }
    w->version = 1;
    snprintf(w->tmp, n + 16, "%s.tmp.XXXXXX", path);
    const int fd = mkstemp(w->tmp);
    if (fd < 0 || !(w->f = fdopen(fd, "wb"))) {
        if (fd >= 0) close(fd);
        e2cu_err("q8c_create: cannot write next to %s", path);
        if (fd < 0) w->tmp[0] = 0;
        e2cuda_q8c_abort(w);
        return NULL;
    }
    const uint32_t hdr[4] = {Q8C_MAGIC, 1u, 0u, 0u}; /* rewritten by the commit */
    if (fwrite(hdr, sizeof hdr, 1, w->f) != 1) {
        e2cu_err("q8c_create: short write");
        e2cuda_q8c_abort(w);
        return NULL;
    }
    w->off = Q8C_DATA_OFF;
    return w;
}

/* open an index entry for a blob about to be written at the current offset */
static q8c_entry *begin(e2cuda_q8c_writer *w, const char *name, int kind, int ndim, const int64_t *dims) {
    if (!w || !w->f || !name) {
        e2cu_err("q8c_put: writer closed or no name");
        return NULL;
    }
    if (!name[0] || strlen(name) >= NAMELEN) {
        e2cu_err("q8c_put: name empty or longer than %d bytes: %s", NAMELEN - 1, name);
        return NULL;
    }
    for (size_t i = 0; i < w->n; i++)
        if (!strcmp(w->idx[i].name, name)) {
            e2cu_err("q8c_put: %s is already in the cache", name);
            return NULL;
        }
    if (w->n == w->cap) {
        const size_t cap = w->cap ? 2 * w->cap : 256;
        q8c_entry *p = realloc(w->idx, cap * sizeof *p);
        if (!p) {
            e2cu_err("q8c_put: out of host memory");
            return NULL;
        }
        w->idx = p;
        w->cap = cap;
    }
    q8c_entry *e = &w->idx[w->n];
    memset(e, 0, sizeof *e);
    memcpy(e->name, name, strlen(name));
    e->kind = (uint32_t)kind;
    e->ndim = (uint32_t)ndim;
    for (int d = 0; d < ndim; d++) e->dims[d] = dims[d];
    e->off = w->off;
    return e;
}
static int put_bytes(e2cuda_q8c_writer *w, q8c_entry *e, const void *p, size_t n) {
    if (n && fwrite(p, 1, n, w->f) != n) {
        e2cu_err("q8c_put: short write");
        return -1;
    }
    e->nbytes += n;
    w->off += n;
    return 0;
}
/* close the entry: pad the blob to 16 bytes */
static int finish(e2cuda_q8c_writer *w) {
    static const uint8_t zeros[16] = {0};
    const size_t pad = (size_t)((16 - (w->off & 15)) & 15);
    if (pad && fwrite(zeros, 1, pad, w->f) != pad) {
        e2cu_err("q8c_put: short write");
        return -1;
    }
    w->off += pad;
    w->n++;
    return 0;
}

int e2cuda_q8c_put(e2cuda_q8c_writer *w, const char *name, int kind, int ndim, const int64_t *dims, const void *p,
                   size_t nbytes) {
    uint64_t want = 0;
    if ((kind != E2CUDA_Q8C_BF16 && kind != E2CUDA_Q8C_F32) || ndim < 0 || ndim > MAXDIM || (ndim && !dims)) {
        e2cu_err("q8c_put: %s: kind %d rank %d (dense bf16/f32 tensors of rank <= 4 only)", name ? name : "", kind, ndim);
        return -1;
    }
    for (int d = 0; d < ndim; d++)
        if (dims[d] < 0) {
            e2cu_err("q8c_put: %s: negative dimension", name ? name : "");
            return -1;
        }
    if (dense_bytes(kind, (uint32_t)ndim, dims, &want) || want != nbytes || (nbytes && !p)) {
        e2cu_err("q8c_put: %s: %zu bytes given for dims needing %llu", name ? name : "", nbytes, (unsigned long long)want);
        return -1;
    }
    q8c_entry *e = begin(w, name, kind, ndim, dims);
    return e && !put_bytes(w, e, p, nbytes) ? finish(w) : -1;
}

int e2cuda_q8c_put_q8w(e2cuda_q8c_writer *w, const char *name, const e2cuda_q8w *q) {
    if (!q || !q->w || !q->scale || !q->bsq) {
        e2cu_err("q8c_put_q8w: %s: incomplete e2_q8w", name ? name : "");
        return -1;
    }
    const int64_t dims[4] = {q->N, q->K, q->nblocks, q->Npad};
    if (!q8w_bytes(dims)) {
        e2cu_err("q8c_put_q8w: %s: N %d K %d nblocks %d Npad %d is not a packed e2_q8w", name ? name : "", q->N, q->K,
                 q->nblocks, q->Npad);
        return -1;
    }
    const size_t nw = (size_t)q->Npad * (size_t)((q->K + 3) / 4) * 4, ns = (size_t)q->Npad * 4,
                 nb = (size_t)q->nblocks * (size_t)q->Npad * 4;
    q8c_entry *e = begin(w, name, E2CUDA_Q8C_Q8W, 4, dims);
    return e && !put_bytes(w, e, q->w, nw) && !put_bytes(w, e, q->scale, ns) && !put_bytes(w, e, q->bsq, nb) ? finish(w)
                                                                                                           : -1;
}

int e2cuda_q8c_put_w8(e2cuda_q8c_writer *w, const char *name, const e2cuda_q8w *q) {
    if (!q || !q->w || !q->scale || q->N <= 0 || q->K <= 0) {
        e2cu_err("q8c_put_w8: %s: incomplete e2_q8w", name ? name : "");
        return -1;
    }
    const int rows = (int)round_to(q->N, 16), ld = (int)round_to(q->K, 16);
    int8_t *t = calloc((size_t)rows, (size_t)ld);
    float *s = calloc((size_t)rows, sizeof(float));
    if (!t || !s) {
        free(t);
        free(s);
        e2cu_err("q8c_put_w8: out of host memory");
        return -1;
    }
    e2cu_unpack_q8w(q, t, ld);
    memcpy(s, q->scale, sizeof(float) * (size_t)q->N);
    const int64_t dims[4] = {q->N, q->K, rows, ld};
    q8c_entry *e = begin(w, name, E2CUDA_Q8C_W8, 4, dims);
    const int rc = e && !put_bytes(w, e, t, (size_t)rows * ld) && !put_bytes(w, e, s, sizeof(float) * rows) ? finish(w)
                                                                                                           : -1;
    free(t);
    free(s);
    if (!rc) w->version = 2;
    return rc;
}

int e2cuda_q8c_commit(e2cuda_q8c_writer *w) {
    if (!w || !w->f) {
        e2cu_err("q8c_commit: writer closed");
        e2cuda_q8c_abort(w);
        return -1;
    }
    int rc = 0;
    if (w->off > UINT32_MAX || w->n > UINT32_MAX) {
        e2cu_err("q8c_commit: the cache exceeds the format's 32-bit index offset");
        rc = -1;
    }
    if (!rc) {
        const uint32_t hdr[4] = {Q8C_MAGIC, (uint32_t)w->version, (uint32_t)w->n, (uint32_t)w->off};
        if ((w->n && fwrite(w->idx, sizeof *w->idx, w->n, w->f) != w->n) || fseek(w->f, 0, SEEK_SET) ||
            fwrite(hdr, sizeof hdr, 1, w->f) != 1 || fflush(w->f) || fsync(fileno(w->f))) {
            e2cu_err("q8c_commit: write failed");
            rc = -1;
        }
    }
    if (fclose(w->f) && !rc) {
        e2cu_err("q8c_commit: close failed");
        rc = -1;
    }
    w->f = NULL;
    if (!rc && rename(w->tmp, w->path)) {
        e2cu_err("q8c_commit: cannot rename onto %s", w->path);
        rc = -1;
    }
    if (!rc) w->tmp[0] = 0; /* committed: nothing left to unlink */
    e2cuda_q8c_abort(w);
    return rc;
}

void e2cuda_q8c_abort(e2cuda_q8c_writer *w) {
    if (!w) return;
    if (w->f) fclose(w->f);
    if (w->tmp && w->tmp[0]) unlink(w->tmp);
    free(w->tmp);
    free(w->path);
    free(w->idx);
    free(w);
}

/* ------------------------------------------------------------------ conversion */
int e2cuda_q8c_convert(const char *in, const char *out) {
    e2cuda_q8c *c = e2cuda_q8c_open(in);
    if (!c) return -1;
    e2cuda_q8c_writer *w = e2cuda_q8c_create(out);
    if (!w) {
        e2cuda_q8c_close(c);
        return -1;
    }
    int rc = 0;
    for (uint32_t i = 0; i < c->n && !rc; i++) {
        const q8c_entry *e = &c->idx[i];
        const void *p = c->base + e->off;
        if (e->kind == E2CUDA_Q8C_Q8W) {
            e2cuda_q8w q;
            rc = e2cuda_q8c_get_q8w(c, e->name, &q) || e2cuda_q8c_put_w8(w, e->name, &q);
        } else if (e->kind == E2CUDA_Q8C_W8) {
            q8c_entry *o = begin(w, e->name, E2CUDA_Q8C_W8, 4, e->dims);
            rc = !o || put_bytes(w, o, p, (size_t)e->nbytes) || finish(w);
            if (!rc) w->version = 2;
        } else {
            rc = e2cuda_q8c_put(w, e->name, (int)e->kind, (int)e->ndim, e->dims, p, (size_t)e->nbytes);
        }
    }
    e2cuda_q8c_close(c);
    if (rc) {
        e2cuda_q8c_abort(w);
        return -1;
    }
    return e2cuda_q8c_commit(w);
}
