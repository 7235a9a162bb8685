/*
 * nnb.h -- C ABI of the B200 (sm_100a) build of nn-cpp's dense-contraction path.
 *
 * Every entry point takes device pointers, plain sizes and a cudaStream_t passed as void*
 * (NULL = the legacy default stream), returns an nnb_status, never allocates visible device
 * memory for the caller, and enqueues its work asynchronously on the stream. Argument checks
 * happen on the host before anything is enqueued; a rejected call enqueues nothing.
 *
 * Each declaration names the reference interface it replaces (file:line within nn-cpp v2.0.0).
 */
#ifndef NNB_H
#define NNB_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NNB_API __attribute__((visibility("default")))
#else
#define NNB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum nnb_status {
	NNB_OK = 0,
	NNB_ERR_INVALID = 1,     /* bad argument: null pointer with a nonzero size, ld too small, ... */
	NNB_ERR_CUDA = 2,        /* a CUDA runtime call failed; nnb_last_error() has the text */
	NNB_ERR_UNSUPPORTED = 3, /* no sm_100a device, or a shape outside the documented limits */
	NNB_ERR_DEVICE = 4,      /* a kernel reported a bounded wait that ran out (nnb_device_error) */
	NNB_ERR_SHAPE = 5        /* tensor shapes do not agree (the reference throws TensorShapeError) */
} nnb_status;

/* Arithmetic of the fp32 GEMM: 3xTF32 split (fp32-grade accuracy) or plain TF32 (fast). */
typedef enum nnb_math_mode {
	NNB_MATH_FP32X3 = 0,
	NNB_MATH_TF32 = 1
} nnb_math_mode;

/* ---- runtime ------------------------------------------------------------------------------ */

/* Library version, "major.minor.patch". */
NNB_API const char* nnb_version(void);

/* Text of the last error reported by any nnb_* call on this host thread ("" if none). */
NNB_API const char* nnb_last_error(void);

/* Process-wide default math mode used by nnb_sgemm (initially NNB_MATH_FP32X3; the environment
 * variable NNB_MATH=tf32|fp32x3 overrides the initial value). */
NNB_API nnb_status nnb_set_math_mode(int mode);
NNB_API int nnb_get_math_mode(void);

/* Waits for `stream`, then returns and clears the device error word of the current device
 * (0 = no kernel reported a timed-out wait). */
NNB_API int nnb_device_error(void* stream);

/* ---- tracing (the counterpart of the reference bench's per-op timing, apps/bench/runner.cpp:29-96) */

/* Kernel kinds for nnb_trace_query. */
typedef enum nnb_trace_kind {
	NNB_TRACE_GEMM = 0,      /* tcgen05 GEMM main kernel */
	NNB_TRACE_PACK = 1,      /* operand pack / TF32 split */
	NNB_TRACE_AUX = 2,       /* fills and small helpers */
	NNB_TRACE_ROWWISE = 3,   /* layernorm / batchnorm / softmax / elementwise */
	NNB_TRACE_ATTENTION = 4, /* fused attention */
	NNB_TRACE_CONV = 5       /* convolution gathers */
} nnb_trace_kind;

/* With tracing on, CUDA events are recorded on the launching stream around every kernel this
 * library launches. */
NNB_API void nnb_trace_enable(int on);
/* Drops recorded events and zeroes the totals and the launch counter. */
NNB_API void nnb_trace_reset(void);
/* Total device milliseconds and launches of one kernel kind since the last reset (waits for the
 * recorded events). */
NNB_API nnb_status nnb_trace_query(int kind, double* total_ms, long long* launches);
/* Kernels launched by this library since the last reset (counted whether tracing is on or not). */
NNB_API long long nnb_launch_count(void);

/* ---- GEMM (replaces nn::kernels::sgemm, include/nn/kernels/gemm.hpp:57-59) ----------------- */

/*
 * Row-major C = op(A)·op(B), or C += op(A)·op(B) when accumulate != 0, in the process default
 * math mode. trans_a: A is stored k x m; trans_b: B is stored n x k. Only the m x n region of C
 * is written; C must not alias A or B. m == 0 or n == 0 does nothing; k == 0 stores +0 (or
 * leaves C) as the reference does (src/kernels/gemm.cpp:345-350).
 */
NNB_API nnb_status nnb_sgemm(void* stream, int trans_a, int trans_b, size_t m, size_t n, size_t k,
		const float* a, size_t lda, const float* b, size_t ldb, float* c, size_t ldc,
		int accumulate);

/* nnb_sgemm with an explicit math mode (nnb_math_mode). */
NNB_API nnb_status nnb_sgemm_ex(void* stream, int trans_a, int trans_b, size_t m, size_t n, size_t k,
		const float* a, size_t lda, const float* b, size_t ldb, float* c, size_t ldc,
		int accumulate, int math_mode);

/*
 * `batch` independent products C_i = op(A_i)·op(B_i) (+= when accumulating) with
 * A_i = a + i*stride_a, B_i = b + i*stride_b, C_i = c + i*stride_c (strides in floats; a stride
 * of 0 broadcasts that operand). The per-matrix loop of nn::matmul's batched path
 * (src/tensor.cpp:597-640) and the per-(n,h) products of attention (src/autograd/ops.cpp:1256)
 * map onto one launch of this.
 */
NNB_API nnb_status nnb_sgemm_strided_batched(void* stream, int trans_a, int trans_b, size_t m, size_t n,
		size_t k, const float* a, size_t lda, size_t stride_a, const float* b, size_t ldb,
		size_t stride_b, float* c, size_t ldc, size_t stride_c, size_t batch, int accumulate,
		int math_mode);

/*
 * nnb_sgemm_ex for callers that cannot allocate device memory. This entry point has no
 * counterpart in the reference (nn-cpp has no GPU and no allocator boundary); it exists for hosts
 * that must not enter the CUDA allocator on the call path: an application that has already handed
 * all device memory to its own arena, a latency-critical loop where cudaMalloc's device-wide
 * synchronisation (or a memory-pool growth) is not acceptable, or an embedding whose allocator is
 * not ours to call. The caller still passes A, B and C; the packed operands and flags go into a
 * fixed 32 MiB device array that every GPU loading this library holds until the process exits.
 *
 * - Limit: (roundup(m,128) + roundup(n,256)) * roundup(k,16) * S * 4 bytes of packed operands plus
 *   a few KB of flags must fit in 32 MiB (S = 2 in NNB_MATH_FP32X3, 1 in NNB_MATH_TF32); e.g.
 *   1024 x 1024 x 1024 in 3xTF32 uses 16 MiB. Larger calls return NNB_ERR_UNSUPPORTED and
 *   enqueue nothing.
 * - The first call on a device (with that device current) looks up the array's device address and
 *   sets kernel attributes; make that first call before any stream capture.
 * - All calls share the array, which keeps the last call's contents; the flags that must start at
 *   zero are cleared on the stream by every call. Calls that overlap on the GPU race on the array:
 *   order them (one stream, or events) yourself.
 * - No cudaMalloc/cudaFree or other allocating routine is called. A bounded wait that expires in this
 *   entry point's kernels is recorded in a device word of its own, not in nnb_device_error.
 */
NNB_API nnb_status nnb_sgemm_noalloc(void* stream, int trans_a, int trans_b, size_t m, size_t n,
		size_t k, const float* a, size_t lda, const float* b, size_t ldb, float* c, size_t ldc,
		int accumulate, int math_mode);

#ifdef __cplusplus
}
#endif

#endif /* NNB_H */
