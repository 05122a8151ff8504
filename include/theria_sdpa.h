/*
 * theria_sdpa.h -- C ABI of the B200 (sm_100a) higher-order SDPA library
 * (libtheria_sm100.so).
 *
 * Every entry point takes raw device pointers to contiguous row-major
 * tensors, plain sizes, and a cudaStream_t passed as void*.  Layouts:
 *   q, tq, dout, w, o, o_tan, dq, hq       [B, H, T, D]
 *   k, v, tk, tv, dk, dv, hk, hv           [B, H, M, D]
 *   lse                                    [B, H, T]  float32
 * D == Dv.  All input tensors of one call share `dtype`.  Nothing here
 * allocates device memory: outputs and the workspace are the caller's.
 * Calls are stream-ordered and asynchronous (no host synchronisation).
 * The library's mutable state is limited to a per-device error word
 * (theria_get_device_error), a process-wide launch counter, and the
 * fixed scratch array of theria_sdpa_bwd_noalloc; no call keeps data
 * between calls otherwise.  Each returns a THERIA_* status.
 *
 * Causal masking is top-left aligned: query row i attends to keys j <= i.
 *
 * The reference library (alexgabel/theria) has no native layer; the entry
 * points replace its Python/Triton operator functions, cited per function
 * (paths inside the theria project).
 */
#ifndef THERIA_SDPA_H
#define THERIA_SDPA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define THERIA_OK 0
#define THERIA_ERR_INVALID_ARG 1  /* null pointer, bad size, bad dtype   */
#define THERIA_ERR_UNSUPPORTED 2  /* head_dim or shape out of range      */
#define THERIA_ERR_LAUNCH 3       /* a CUDA launch returned an error     */
#define THERIA_ERR_WORKSPACE 4    /* workspace missing or too small      */
#define THERIA_ERR_DEVICE_TIMEOUT 5 /* a device-side wait gave up        */
#define THERIA_ERR_SCRATCH_LIMIT 6 /* problem exceeds the fixed scratch of
                                      theria_sdpa_bwd_noalloc            */

/* element types.  THERIA_F64 (double precision throughout, for
 * gradcheck-style verification) runs only in the whole-head kernels: the
 * forward, backward, JVP and HVP accept it for T, M <= 64 and D <= 64 where
 * the head fits in shared memory as doubles, and return
 * THERIA_ERR_UNSUPPORTED otherwise; lse stays float32.  The dense score and
 * probability entry points do not take it. */
#define THERIA_F32 0
#define THERIA_F16 1
#define THERIA_BF16 2
#define THERIA_F64 3

/* largest head dimension any entry point accepts */
#define THERIA_MAX_HEAD_DIM 128

/* Human-readable text for a status code (static string, never NULL). */
const char* theria_status_string(int status);

/* Library version, e.g. "theria-sm100 0.1.0". */
const char* theria_version(void);

/*
 * Forward: o = softmax(scale * q k^T [+ causal mask]) v, and the row
 * logsumexp lse = m + log(l) of the scaled scores.
 * `o_dtype` is THERIA_F32 or `dtype` (the reference's fused forward returns
 * float32; its public sdpa_custom returns q.dtype).  `lse` may be NULL.
 * Replaces triton_sdpa_fused / _fused_sdpa_kernel
 * (theria/attention/triton_qk.py:242-369).
 */
int theria_sdpa_fwd(const void* q, const void* k, const void* v,
                    void* o, int o_dtype, float* lse,
                    int64_t B, int64_t H, int64_t T, int64_t M, int64_t D,
                    int dtype, float scale, int causal, void* stream);

/* Bytes of workspace theria_sdpa_bwd / theria_sdpa_hvp need. */
int64_t theria_sdpa_bwd_workspace_bytes(int64_t B, int64_t H, int64_t T,
                                        int64_t M, int64_t D);
int64_t theria_sdpa_hvp_workspace_bytes(int64_t B, int64_t H, int64_t T,
                                        int64_t M, int64_t D);

/*
 * Backward: dq, dk, dv of <o, dout> from the saved lse.
 * `o` (the forward output, dtype `o_dtype`) may be NULL, in which case the
 * row term z = rowsum(dout * o) is rebuilt from lse.  Any of dq/dk/dv may be
 * NULL to skip storing it.  Outputs have `dtype`.
 * Replaces sdpa_bwd_dq / sdpa_bwd_dk / sdpa_bwd_dv
 * (theria/attention/triton_sdpa_backward.py:505-696, :269-462, :106-266)
 * and the backward of TritonFusedSDPAFunction (triton_qk.py:379-387).
 */
int theria_sdpa_bwd(const void* q, const void* k, const void* v,
                    const void* o, int o_dtype, const void* dout,
                    const float* lse, void* dq, void* dk, void* dv,
                    void* workspace, int64_t workspace_bytes,
                    int64_t B, int64_t H, int64_t T, int64_t M, int64_t D,
                    int dtype, float scale, int causal, void* stream);

/*
 * Frozen-stats JVP: o_tan = Pdot v + P tv with P rebuilt from lse and
 * Pdot = P * (Sdot - rowsum(P * Sdot)), Sdot = scale (tq k^T + q tk^T).
 * At the saved point this is the exact tangent of o.
 * Replaces sdpa_jvp (theria/attention/triton_sdpa_backward.py:465-503).
 */
int theria_sdpa_jvp(const void* q, const void* k, const void* v,
                    const void* tq, const void* tk, const void* tv,
                    const float* lse, void* o_tan,
                    int64_t B, int64_t H, int64_t T, int64_t M, int64_t D,
                    int dtype, float scale, int causal, void* stream);

/*
 * Hessian-vector product of L = <o, w> along u = (tq, tk, tv):
 *   hq, hk, hv = d/de grad_{q,k,v} L(q + e tq, k + e tk, v + e tv) at e = 0
 * and o_tan = J u (the derivative of <grad L, u> with respect to w).
 * This is the double-backward of the attention backward.  Any output may
 * be NULL to skip storing it.
 * Replaces hvp_fd_vjp (theria/attention/hvp_utils.py:30-49), sdpa_hvp
 * (theria/attention/reference_hvp_sdpa.py:46-97) and the
 * create_graph=True backward of SDPACustom
 * (theria/autograd/sdpa_custom_function.py:31-53).
 */
int theria_sdpa_hvp(const void* q, const void* k, const void* v,
                    const void* w, const float* lse,
                    const void* tq, const void* tk, const void* tv,
                    void* hq, void* hk, void* hv, void* o_tan,
                    void* workspace, int64_t workspace_bytes,
                    int64_t B, int64_t H, int64_t T, int64_t M, int64_t D,
                    int dtype, float scale, int causal, void* stream);

/*
 * Allocation-free backward.  No counterpart in the reference library.
 *
 * Same arguments, outputs and results as theria_sdpa_bwd, minus the
 * workspace: the scratch it needs (one float per query row) lives in a
 * fixed array inside the library, THERIA_NOALLOC_SCRATCH_BYTES per GPU,
 * held by every GPU that loads the library until the process exits.  It is
 * for callers that cannot allocate device memory at call time -- code
 * running under a foreign allocator or memory pool that forbids
 * cudaMalloc, or a host that has no allocator handle at all (a plain C
 * caller holding only raw pointers).  This entry point performs no device
 * allocation of any kind.
 *
 * Limits: B*H*T*4 bytes must fit in THERIA_NOALLOC_SCRATCH_BYTES, else it
 * returns THERIA_ERR_SCRATCH_LIMIT without launching anything.  Which
 * kernels run depends on the size as well: the 16-bit tensor-core backward
 * also keeps an fp32 dQ accumulator in the scratch, so it is used only when
 * B*H*T*(D+1)*4 bytes (each part rounded up to 256) fit; larger accepted
 * problems run the CUDA-core backward kernels -- same results within the
 * usual tolerance, but far slower.  theria_sdpa_bwd_noalloc_uses_tc reports
 * which path a shape takes.  All calls
 * on a GPU share the one array, so calls that overlap on the GPU (two
 * streams, or two host threads on different streams) race and corrupt each
 * other's results; serialise them.  The first call on each device looks up
 * the array's device address with that device current (one-time set-up)
 * and caches it for the life of the process; make that first call before
 * any stream capture.  The cache does not survive cudaDeviceReset or the
 * destruction of the device's primary context: do not call this entry
 * point after either.  The array keeps the last
 * call's contents; nothing in it needs to start at zero (every element a
 * call reads was written earlier in that same call).
 */
#define THERIA_NOALLOC_SCRATCH_BYTES (4 * 1024 * 1024)
int theria_sdpa_bwd_noalloc(const void* q, const void* k, const void* v,
                            const void* o, int o_dtype, const void* dout,
                            const float* lse, void* dq, void* dk, void* dv,
                            int64_t B, int64_t H, int64_t T, int64_t M, int64_t D,
                            int dtype, float scale, int causal, void* stream);
/* 1 if theria_sdpa_bwd_noalloc runs the tensor-core backward for this
 * shape and dtype, 0 if it runs the CUDA-core kernels, or a negative
 * THERIA_* status (negated) if it would refuse the problem.  Looks only at
 * sizes (pointer alignment is assumed to be 16 bytes). */
int theria_sdpa_bwd_noalloc_uses_tc(int64_t B, int64_t H, int64_t T, int64_t M, int64_t D,
                                    int dtype);

/*
 * Dense attention scores: out[b,h,t,m] = scale * sum_d q[b,h,t,d] k[b,h,m,d],
 * out [B,H,T,M] row-major in out_dtype (THERIA_F32, or the input dtype).
 * Replaces the reference's QK^T kernels theria/attention/triton_qk.py:16-70
 * (_qk_kernel, fp32 out; callers pass scale 1) and triton_qk.py:394-455
 * (_qk_kernel_fast, input-dtype out).  Accumulates in fp32.
 */
int theria_sdpa_scores(const void* q, const void* k, void* out, int out_dtype,
                       int64_t B, int64_t H, int64_t T, int64_t M, int64_t D,
                       int dtype, float scale, void* stream);

/*
 * Dense attention probabilities: out[b,h,t,m] = exp(scale * q_t . k_m -
 * lse[b,h,t]) as fp32 [B,H,T,M] (zero for m > t when causal), where lse is
 * the row log-sum-exp theria_sdpa_fwd wrote for the same q, k, scale.
 * Replaces the fused QK^T + softmax kernel theria/attention/triton_qk.py:
 * 130-240 (_qk_softmax_kernel, triton_qk_softmax).
 */
int theria_sdpa_probs(const void* q, const void* k, const float* lse, float* out,
                      int64_t B, int64_t H, int64_t T, int64_t M, int64_t D,
                      int dtype, float scale, int causal, void* stream);

/* Packed self-attention (T == M) for short sequences (T <= 64, D <= 64,
 * the whole-head kernels; otherwise THERIA_ERR_UNSUPPORTED): q, k, v are
 * read in place from a fused projection qkv [B, T, 3, H, D] (q at offset 0,
 * k at H*D, v at 2*H*D of each token row), O-shaped tensors (o, dout / w,
 * o_tan) are [B, T, H, D], and gradients (dqkv, hqkv) come back packed like
 * qkv.  Same arithmetic as theria_sdpa_fwd / _bwd / _hvp; the layout saves
 * the copies between a [B, T, 3, H, D] projection and [B, H, T, D] heads.
 * fwd writes o in the input dtype.  hvp: hqkv or o_tan may be NULL.
 * Replaces no reference entry point: the reference's attention callers
 * (examples/minimal_decoder_transformer.py:82-263) split heads with
 * reshape/transpose before calling the attention op. */
int theria_sdpa_qkv_fwd(const void* qkv, void* o, float* lse, int64_t B, int64_t H,
                        int64_t T, int64_t D, int dtype, float scale, int causal,
                        void* stream);
int theria_sdpa_qkv_bwd(const void* qkv, const void* dout, const float* lse, void* dqkv,
                        int64_t B, int64_t H, int64_t T, int64_t D, int dtype, float scale,
                        int causal, void* stream);
int theria_sdpa_qkv_hvp(const void* qkv, const void* w, const float* lse, const void* tqkv,
                        void* hqkv, void* o_tan, int64_t B, int64_t H, int64_t T, int64_t D,
                        int dtype, float scale, int causal, void* stream);

/* Number of kernels this library has launched in this process (all devices,
 * all threads); for accounting in benchmarks and tests. */
int64_t theria_launch_count(void);

/*
 * Device-side error word of the current device: non-zero once a kernel's
 * bounded wait gave up (THERIA_ERR_DEVICE_TIMEOUT).  Reading it synchronises
 * `stream`.  theria_clear_device_error resets it (stream-ordered).
 */
int theria_get_device_error(int* out_flag, void* stream);
int theria_clear_device_error(void* stream);

/*
 * Diagnostic of the bounded device-side waits (no counterpart in the
 * reference).  Launches one CTA whose first warp waits, with a limit of
 * `max_polls` polls (1 .. 2^20), on an mbarrier phase that nothing
 * completes, and whose second warp waits on the same phase with the
 * library's normal limit.  The first warp must give up, set the device
 * error word to THERIA_ERR_DEVICE_TIMEOUT and raise the CTA's abort flag;
 * the second must then unwind.  `out` is 2 device ints: out[0] = 1 if the
 * first wait gave up, out[1] = 1 if the second unwound.  No wait in it is
 * unbounded, and the kernel leaves the GPU context usable.
 */
int theria_diag_bounded_wait(int max_polls, int* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* THERIA_SDPA_H */
