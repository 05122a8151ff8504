/*
 * theria_ln.h -- C ABI of the task-batched LayerNorm used by the full-MAML
 * model (libtheria_sm100.so), with its first and second derivatives.
 *
 * x, y, gy, gx, u, dx, dgy are [nt, R, D] float32, contiguous; w, b are
 * [nt, D] float32 with row stride ldw (elements; 0 = one row shared by
 * all tasks); a, c have row strides lda, ldc the same way; gw, gb, dw are
 * [nt, D] contiguous.  eps is added to the variance (as torch layer_norm).
 *   forward      y  = (x - mean) * rstd * w + b
 *   backward     gx = rstd * P(gy * w), gw = sum_rows gy * xhat, gb = sum_rows gy
 *   backward of the backward, for cotangents (u, a, c) of (gx, gw, gb):
 *                dx, dw, dgy   (u, a, c may be NULL: zero)
 * where P(v) = v - mean(v) - xhat * mean(v * xhat).  The row sums go through
 * a caller-owned workspace of theria_ln_workspace_bytes(nt, R, D) bytes and a
 * second deterministic kernel.  Stream-ordered, no allocation, no host
 * synchronisation; each call returns a THERIA_* status (theria_sdpa.h).
 *
 * The reference library has no LayerNorm of its own: its MAML loops
 * (theria/maml/loops.py:42-123) run user models through torch autograd.
 * These entry points serve this build's benchmark model, whose LayerNorm
 * double backward would otherwise be dozens of small torch kernels.
 */
#ifndef THERIA_LN_H
#define THERIA_LN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* largest normalised dimension the kernels accept */
#define THERIA_LN_MAX_D 256

int64_t theria_ln_workspace_bytes(int64_t nt, int64_t R, int64_t D);

int theria_ln_fwd(const float* x, const float* w, const float* b, int64_t ldw, float* y,
                  int64_t nt, int64_t R, int64_t D, float eps, void* stream);

int theria_ln_bwd(const float* x, const float* w, int64_t ldw, const float* gy, float* gx,
                  float* gw, float* gb, void* workspace, int64_t workspace_bytes,
                  int64_t nt, int64_t R, int64_t D, float eps, void* stream);

/* a, c: rows at strides lda, ldc (like ldw) */
int theria_ln_bwd2(const float* x, const float* w, int64_t ldw, const float* gy,
                   const float* u, const float* a, int64_t lda, const float* c, int64_t ldc,
                   float* dx, float* dw, float* dgy, void* workspace, int64_t workspace_bytes,
                   int64_t nt, int64_t R, int64_t D, float eps, void* stream);

/* out[t][c] = sum_r x[t][r][c] for x [nt, R, C] float32 contiguous (the
 * bias gradient of the model's task-batched linears), C <= 1024, through a
 * workspace of theria_rowsum_workspace_bytes(nt, R, C) bytes; deterministic. */
int64_t theria_rowsum_workspace_bytes(int64_t nt, int64_t R, int64_t C);
int theria_rowsum(const float* x, float* out, void* workspace, int64_t workspace_bytes,
                  int64_t nt, int64_t R, int64_t C, void* stream);

/* out = x + b (broadcast over rows) [+ res]: x, res, out [nt, R, C] float32
 * contiguous, b rows at stride ldb (0: shared); res may be NULL. */
int theria_add_bias(const float* x, const float* b, int64_t ldb, const float* res, float* out,
                    int64_t nt, int64_t R, int64_t C, void* stream);

/* out[t][e] = sum_c x[t][c][e] for x [nt, S, W] float32 contiguous (the
 * partial products of the model's split long-row matmuls); deterministic. */
int theria_chunk_sum(const float* x, float* out, int64_t nt, int64_t S, int64_t W,
                     void* stream);

/* Second derivative of the exact GELU through its backward gx = gy *
 * gelu'(x): for a cotangent u of gx, dgy = u * gelu'(x) and
 * dx = u * gy * gelu''(x); x, gy, u, dx, dgy hold n float32 each. */
int theria_gelu_bwd2(const float* x, const float* gy, const float* u, float* dx, float* dgy,
                     int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* THERIA_LN_H */
