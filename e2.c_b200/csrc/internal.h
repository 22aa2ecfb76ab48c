/* internal.h — helpers shared by the C host files of e2cuda (not part of the ABI). */
#ifndef E2CU_INTERNAL_H
#define E2CU_INTERNAL_H

#include <cuda_runtime.h>

#include "e2cuda.h"
#include "launch.h"

/* record a message for e2cuda_last_error() */
void e2cu_err(const char *fmt, ...);
/* 0 on cudaSuccess, else -1 with "<what>: <cuda error>" recorded */
int e2cu_cuda(cudaError_t e, const char *what);
/* 0 if a launcher returned 0, else -1 with "<what>: <launcher message>" recorded */
int e2cu_launch(int rc, const char *what);
/* the current device's status word (allocated on first use), NULL without a device */
int *e2cu_status(void);
/* a device failure was reported: every weight-streaming workspace is cleared before its next use */
void e2cu_note_failure(void);
/* clear `ws` (bytes) on `st` if a failure was reported since it was last cleared (*gen) */
int e2cu_ws_refresh(int *ws, size_t bytes, int *gen, cudaStream_t st);

int e2cu_w8_alloc(e2cuda_w8 *out, int N, int K);
/* quad-interleaved e2_q8w -> row-major int8 rows of stride ld */
void e2cu_unpack_q8w(const e2cuda_q8w *q, int8_t *dst, int ld);
int e2cu_upload_gate_up(const e2cuda_q8w *g, const e2cuda_q8w *u, e2cuda_w8 *out);
/* GEMM arguments for weight w over activations qa/as (row stride w->ld), all columns */
void e2cu_gemm_args(e2c_gemm_args *a, const e2cuda_w8 *w, const int8_t *qa, const float *as, int M, int ablk);

#endif
