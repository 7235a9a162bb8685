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

/* Peer memory between the processes of one node (one process per GPU): export a device pointer
 * as a CUDA IPC handle (64 bytes) plus its offset inside its allocation; open another process's
 * handle as a pointer this GPU can load from and store to over NVLink; close it again (before the
 * owner frees the memory). Used by the sharded GEMM, whose epilogue stores each rank's tiles of C
 * straight into the gathering GPU's C. */
NNB_API nnb_status nnb_ipc_export(const void* ptr, unsigned char* handle, size_t* offset);
NNB_API nnb_status nnb_ipc_open(const unsigned char* handle, size_t offset, void** ptr);
NNB_API nnb_status nnb_ipc_close(void* ptr, size_t offset);
/* bytes from src to dst on `stream` by the copy engines (device, peer-mapped or host memory). */
NNB_API nnb_status nnb_copy_async(void* stream, void* dst, const void* src, size_t bytes);

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

/* nn::kernels::sgemm on HOST buffers (include/nn/kernels/gemm.hpp:57-59, the reference's own calling
 * convention: row-major, host pointers, returns with C written): the drop-in for the reference's
 * kernel. B is copied to the device and packed once, then op(A) in row bands whose GEMMs run while
 * the next bands are copied in and finished bands of C are copied back (a copy stream, two compute
 * streams, a copy-back stream). Bitwise equal to nnb_sgemm on device copies of the same operands.
 * Page-locked host buffers give full copy speed. The device buffers it grows are kept per device
 * for the next call until nnb_sgemm_host_release. */
NNB_API nnb_status nnb_sgemm_host(int trans_a, int trans_b, size_t m, size_t n, size_t k, const float* a,
		size_t lda, const float* b, size_t ldb, float* c, size_t ldc, int accumulate);
/* The same, stream-ordered and not blocking: it starts once `stream` reaches it and `stream` waits for
 * the last copy-back, so the host buffers must stay valid until then (events on `stream` time it). */
NNB_API nnb_status nnb_sgemm_host_async(void* stream, int trans_a, int trans_b, size_t m, size_t n, size_t k,
		const float* a, size_t lda, const float* b, size_t ldb, float* c, size_t ldc, int accumulate, int math_mode);
/* Waits for every device's host-buffer GEMM work and frees the device buffers it keeps between calls
 * (about 5 x the operands' bytes after an 8192^3 call); the next call grows them again. No reference
 * counterpart: the reference's kernel keeps only host-side thread-local packing buffers. */
NNB_API nnb_status nnb_sgemm_host_release(void);

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

/* ---- batched Tensor matmul (replaces nn::matmul, include/nn/tensor.hpp:475,491; src/tensor.cpp:571-641) */

/*
 * a (a_ndim axes, a_shape) times b (b_ndim axes), both dense row-major on the device, with the
 * reference's rules: a batched a (not transposed) times a 2-D b is folded into one product over all
 * of a's rows; otherwise the batch axes broadcast numpy-style and each output matrix is one product.
 * out_shape (room for 16 axes) and out_ndim receive the result shape; with c == NULL only the shape
 * is computed. Mismatched inner sizes or batch axes return NNB_ERR_SHAPE (TensorShapeError).
 */
NNB_API nnb_status nnb_matmul(void* stream, const float* a, const int64_t* a_shape, int a_ndim, const float* b,
		const int64_t* b_shape, int b_ndim, int trans_a, int trans_b, float* c, int64_t* out_shape, int* out_ndim);

/* ---- linear (replaces Value linear, include/nn/autograd/ops.hpp:304; src/autograd/ops.cpp:714-745)
 *
 * "first" flags follow Value::grad_accum (src/autograd/value.cpp:60-64): 1 stores the value (+0),
 * 0 adds it to what the buffer holds. A NULL gradient output is skipped.
 */

/* y[M, n] = x[M, K] · w[n, K]^T + bias[n] (bias added in the GEMM epilogue). */
NNB_API nnb_status nnb_linear_fwd(void* stream, size_t M, size_t K, size_t n, const float* x, const float* w,
		const float* bias, float* y);
/* linear of one input under `count` weights (the q, k and v projections of a self-attention,
 * src/nn/attention.cpp:34, `q_.forward(query), k_.forward(context), v_.forward(context)` with
 * query == context): y_i = x · w_i^T + b_i with w_i = w + i·w_stride, b_i = bias + i·bias_stride and
 * y_i = y + i·y_stride (floats), i < count. x is packed once and the products run as one launch;
 * every y_i has the bits of nnb_linear_fwd(x, w_i, b_i). Strides that make consecutive weights,
 * biases or outputs overlap are rejected (NNB_ERR_INVALID). */
NNB_API nnb_status nnb_linear_multi_fwd(void* stream, size_t count, size_t M, size_t K, size_t n, const float* x,
		const float* w, size_t w_stride, const float* bias, size_t bias_stride, float* y, size_t y_stride);
/* gelu(linear(x, w, bias)) as one GEMM with the GELU in its epilogue (the transformer's fc1 followed
 * by gelu, ops.cpp:451-466): y = gelu(pre), pre = x·w^T + bias is kept for the backward pass
 * (nnb_gelu_bwd with tanh_saved = NULL recomputes the tanh from pre, bit for bit). */
NNB_API nnb_status nnb_linear_gelu_fwd(void* stream, size_t M, size_t K, size_t n, const float* x, const float* w,
		const float* bias, float* y, float* pre);
/* dx (+)= g·w, dw (+)= g^T·x, db (+)= column sums of g (fixed chunked order: serial within 256-row
 * chunks, then over chunks; the reference's serial order whenever M <= 256). When both dx and dw are
 * asked for, g is packed once: the dx product's packed copy (M x n x 8 bytes in 3xTF32, scratch from
 * the memory pool, freed in stream order) is read again by the dw product. */
NNB_API nnb_status nnb_linear_bwd(void* stream, size_t M, size_t K, size_t n, const float* g, const float* x,
		const float* w, float* dx, int dx_first, float* dw, int dw_first, float* db, int db_first);
/* nnb_linear_bwd whose weight and bias gradients are kept per group: the M rows are `groups`
 * consecutive groups, and group z's dW (n x K) and db (n) are computed from its rows only (one
 * batched launch) into dw + z*dw_stride and db + z*db_stride (a stride of 0 packs the groups
 * back to back). dx covers all rows. The data-parallel step uses one group per virtual shard so
 * that the shard sum can be taken in a fixed order. No reference counterpart: the reference has no
 * distributed training. */
NNB_API nnb_status nnb_linear_bwd_grouped(void* stream, size_t M, size_t K, size_t n, size_t groups, const float* g,
		const float* x, const float* w, float* dx, int dx_first, float* dw, size_t dw_stride, int dw_first, float* db,
		size_t db_stride, int db_first);
/* The linear forward and backward with the input's packed operand kept between them (no reference
 * counterpart: the reference packs inside each sgemm call, src/kernels/gemm.cpp:372-378, and keeps
 * nothing). Both linear GEMMs of the backward read the input X and the output gradient G, the
 * forward GEMM reads X: packing X once in the forward and G once in the backward, and letting the
 * weight gradient G^T X read both packs as they are, saves two of the four operand passes of a
 * linear layer's training step. Results are bitwise those of nnb_linear_fwd / nnb_linear_multi_fwd /
 * nnb_linear_gelu_fwd and nnb_linear_bwd_grouped.
 * nnb_linear_pack_bytes: bytes of the kept pack of an M x K input in the given math mode.
 * nnb_linear_fwd_ex: count (>= 1) products y_i = x w_i^T + b_i as nnb_linear_multi_fwd (strides
 *   as there; ignored when count == 1); with pre non-null (count 1 only) the GELU form of
 *   nnb_linear_gelu_fwd. x_pack (nullable) receives x's pack in the current math mode.
 * nnb_linear_bwd_ex: nnb_linear_bwd_grouped (groups 1: nnb_linear_bwd) whose weight gradient
 *   reads x_pack (nullable) when it holds x's pack written in math mode x_pack_mode by
 *   nnb_linear_fwd_ex with this same x; a pack of another mode, or a group shape the tensor core
 *   cannot read from a pack (groups not whole 16-row blocks), is ignored and X is packed as usual. */
NNB_API size_t nnb_linear_pack_bytes(size_t M, size_t K, int math_mode);
NNB_API nnb_status nnb_linear_fwd_ex(void* stream, size_t count, size_t M, size_t K, size_t n, const float* x,
		const float* w, size_t w_stride, const float* bias, size_t bias_stride, float* y, size_t y_stride, float* pre,
		void* x_pack);
NNB_API nnb_status nnb_linear_bwd_ex(void* stream, size_t M, size_t K, size_t n, size_t groups, const float* g,
		const float* x, const void* x_pack, int x_pack_mode, const float* w, float* dx, int dx_first, float* dw,
		size_t dw_stride, int dw_first, float* db, size_t db_stride, int db_first);
/* out[j] (+)= sum_r g[r][j] in the order above (Tensor::sum(0), src/tensor.cpp:422-455). */
NNB_API nnb_status nnb_column_sum(void* stream, size_t rows, size_t cols, const float* g, float* out, int first);

/* ---- normalisation ------------------------------------------------------------------------ */

/* layernorm over the last axis (ops.hpp:130; ops.cpp:1003-1032): x is R rows of D; mean and
 * inv_std (R each) are saved for the backward pass. */
NNB_API nnb_status nnb_layernorm_fwd(void* stream, size_t R, size_t D, const float* x, const float* gamma,
		const float* beta, float eps, float* y, float* mean, float* inv_std);
/* layernorm backward (ops.cpp:1033-1076). */
NNB_API nnb_status nnb_layernorm_bwd(void* stream, size_t R, size_t D, const float* g, const float* x,
		const float* gamma, const float* mean, const float* inv_std, float* dx, int dx_first, float* dgamma,
		int dgamma_first, float* dbeta, int dbeta_first);
/* layernorm backward with dgamma/dbeta kept per group of R/groups consecutive rows, group z at
 * dgamma + z*dgamma_stride (0: back to back); see nnb_linear_bwd_grouped. */
NNB_API nnb_status nnb_layernorm_bwd_grouped(void* stream, size_t R, size_t D, size_t groups, const float* g,
		const float* x, const float* gamma, const float* mean, const float* inv_std, float* dx, int dx_first,
		float* dgamma, size_t dgamma_stride, int dgamma_first, float* dbeta, size_t dbeta_stride, int dbeta_first);
/* Training-mode batchnorm over [N, C, S] (ops.hpp:114; ops.cpp:900-961): per-channel statistics with
 * the reference's fp64 sums of 8-lane partials; fuse_relu folds a ReLU and writes its 1-byte alive
 * mask; mean, var (biased) and inv_std (C each) are written. */
NNB_API nnb_status nnb_batchnorm_fwd(void* stream, size_t N, size_t C, size_t S, const float* x,
		const float* weight, const float* bias, float eps, int fuse_relu, float* y, unsigned char* alive,
		float* mean, float* var, float* inv_std);
/* batchnorm backward (ops.cpp:963-1000); alive = the forward's mask when the ReLU was folded, else NULL. */
NNB_API nnb_status nnb_batchnorm_bwd(void* stream, size_t N, size_t C, size_t S, const float* g, const float* x,
		const float* weight, const float* mean, const float* inv_std, const unsigned char* alive, float* dx,
		int dx_first, float* dweight, int dweight_first, float* dbias, int dbias_first);

/* BatchNorm1d / BatchNorm2d module pieces (src/nn/batchnorm.cpp): after a training-mode forward,
 * running_mean = (1 - momentum) running_mean + momentum mean and, when count > 1, running_var =
 * (1 - momentum) running_var + momentum var count / (count - 1) (batchnorm.cpp:38-47; count = N*S). */
NNB_API nnb_status nnb_batchnorm_running_update(void* stream, size_t C, size_t count, const float* mean,
		const float* var, float momentum, float* running_mean, float* running_var);
/* Evaluation mode (batchnorm.cpp:51-55): y = ((x - running_mean) / sqrt(running_var + eps)) w + b,
 * optionally followed by ReLU with its alive mask; the backward gives dx, dweight and dbias. x is
 * [N, C, H, W] (S = H * W in the forward; a 3-D input is [N, C, L, 1], a 2-D one [N, C, 1, 1]); the
 * parameter gradients are summed over N, then H, then W, as the reference's sum_to_shape does. */
NNB_API nnb_status nnb_batchnorm_eval_fwd(void* stream, size_t N, size_t C, size_t S, const float* x,
		const float* running_mean, const float* running_var, float eps, const float* weight, const float* bias,
		int fuse_relu, float* y, unsigned char* alive);
NNB_API nnb_status nnb_batchnorm_eval_bwd(void* stream, size_t N, size_t C, size_t H, size_t W, const float* g,
		const float* x, const float* running_mean, const float* running_var, float eps, const float* weight,
		const unsigned char* alive, float* dx, int dx_first, float* dweight, int dweight_first, float* dbias,
		int dbias_first);

/* ---- attention (replaces Value attention, ops.hpp:324; ops.cpp:1183-1296) ------------------ */

/* q [N, Tq, D], k/v [N, Tk, D], heads | D; key_padding_mask [N, Tk] (0 = padded) or NULL;
 * causal needs Tq == Tk. out [N, Tq, D]; probs [N, heads, Tq, Tk] is kept for the backward pass. */
NNB_API nnb_status nnb_attention_fwd(void* stream, size_t N, size_t Tq, size_t Tk, size_t D, size_t heads,
		const float* q, const float* k, const float* v, const float* key_padding_mask, int causal, float* out,
		float* probs);
NNB_API nnb_status nnb_attention_bwd(void* stream, size_t N, size_t Tq, size_t Tk, size_t D, size_t heads,
		const float* g, const float* q, const float* k, const float* v, const float* probs,
		const float* key_padding_mask, int causal, float* dq, int dq_first, float* dk, int dk_first, float* dv,
		int dv_first);
/* Fused attention for head size 64 (D / heads == 64): the same op and masks as nnb_attention_*,
 * without the [N, heads, Tq, Tk] probabilities. The forward writes out and stats [N, heads, Tq, 2]
 * (per query row: the max m of the masked scaled scores and the sum l of exp(score - m), from
 * which the backward recomputes the probabilities); the backward takes the forward's out and stats. Results agree with nnb_attention_* to fp32 rounding
 * (the softmax is computed online over 64-key tiles); each output element is written by one CTA
 * in a fixed order, so they are bitwise reproducible. Other head sizes: NNB_ERR_UNSUPPORTED.
 * Replaces the same reference interface as nnb_attention_fwd / _bwd (ops.cpp:1226-1296). */
NNB_API int nnb_flash_attention_supported(size_t D, size_t heads);
NNB_API nnb_status nnb_flash_attention_fwd(void* stream, size_t N, size_t Tq, size_t Tk, size_t D, size_t heads,
		const float* q, const float* k, const float* v, const float* key_padding_mask, int causal, float* out,
		float* lse);
NNB_API nnb_status nnb_flash_attention_bwd(void* stream, size_t N, size_t Tq, size_t Tk, size_t D, size_t heads,
		const float* g, const float* q, const float* k, const float* v, const float* out, const float* lse,
		const float* key_padding_mask, int causal, float* dq, int dq_first, float* dk, int dk_first, float* dv,
		int dv_first);
/* attention with dropout on the weights: MultiHeadAttention's composed path when its Dropout is
 * active (src/nn/attention.cpp:36-47: matmul_bt, scaled_masked_softmax ops.cpp:1298-1343,
 * Dropout::forward src/nn/dropout.cpp:20-31, matmul). keep = the dropout mask of the N*H*Tq*Tk
 * weights from nnb_dropout_mask (bit e % 32 of word e / 32 = element e kept); probs and weights
 * ([N, heads, Tq, Tk], the softmax and the dropped weights) are kept for the backward. */
NNB_API nnb_status nnb_attention_dropout_fwd(void* stream, size_t N, size_t Tq, size_t Tk, size_t D, size_t heads,
		const float* q, const float* k, const float* v, const float* key_padding_mask, int causal, float p,
		const uint32_t* keep, float* out, float* probs, float* weights);
NNB_API nnb_status nnb_attention_dropout_bwd(void* stream, size_t N, size_t Tq, size_t Tk, size_t D, size_t heads,
		const float* g, const float* q, const float* k, const float* v, const float* probs, const float* weights,
		float p, const uint32_t* keep, const float* key_padding_mask, int causal, float* dq, int dq_first, float* dk,
		int dk_first, float* dv, int dv_first);
/* masked_softmax_row over [N, H, Tq, Tk] scores in place (ops.cpp:1183-1204), and its backward
 * turning dL/dP into dL/dS in place (ops.cpp:1216-1224). */
NNB_API nnb_status nnb_masked_softmax_fwd(void* stream, size_t N, size_t H, size_t Tq, size_t Tk, float* scores,
		const float* key_padding_mask, int causal, float scale);
NNB_API nnb_status nnb_masked_softmax_bwd(void* stream, size_t N, size_t H, size_t Tq, size_t Tk,
		const float* probs, float* grad, const float* key_padding_mask, int causal, float scale);
/* scaled_masked_softmax (ops.hpp scaled_masked_softmax; ops.cpp:1298-1343): y = the masked softmax of
 * x [N, H, Tq, Tk] (x is not modified; causal rows need not be square). The backward writes
 * dL/dx into dx under the grad_accum rule: dx_first stores (0 at masked positions), otherwise it
 * adds and leaves masked positions as they are. */
NNB_API nnb_status nnb_scaled_masked_softmax_fwd(void* stream, size_t N, size_t H, size_t Tq, size_t Tk,
		const float* x, float* y, const float* key_padding_mask, int causal, float scale);
NNB_API nnb_status nnb_scaled_masked_softmax_bwd(void* stream, size_t N, size_t H, size_t Tq, size_t Tk,
		const float* y, const float* g, float* dx, int dx_first, const float* key_padding_mask, int causal,
		float scale);

/* ---- convolution (replaces conv2d / conv2d_relu, ops.hpp:402; ops.cpp:1345-1472) ------------ */

/* x [N, Cin, H, W], weight [Cout, Cin, kh, kw], bias [Cout] -> y [N, Cout, ho, wo];
 * fuse_relu = conv2d_relu with its 1-byte alive mask (same layout as y). */
NNB_API nnb_status nnb_conv2d_fwd(void* stream, size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh,
		size_t kw, int stride, int padding, const float* x, const float* weight, const float* bias, int fuse_relu,
		float* y, unsigned char* alive);
NNB_API nnb_status nnb_conv2d_bwd(void* stream, size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh,
		size_t kw, int stride, int padding, const float* grad, const float* x, const float* weight,
		const unsigned char* alive, float* dx, int dx_first, float* dweight, int dweight_first, float* dbias,
		int dbias_first);

/* conv2d with dilation and groups (replaces the general conv2d, ops.hpp:421; ops.cpp:1525-1607):
 * weight [Cout, Cin/groups, kh, kw]; per sample and group an im2col + GEMM, the bias added after
 * the product; the backward's bias gradient sums samples then positions serially, the weight
 * gradient sums per-sample products in sample order, as the reference. */
NNB_API nnb_status nnb_conv2d_ex_fwd(void* stream, size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh,
		size_t kw, int stride, int padding, int dilation, int groups, const float* x, const float* weight,
		const float* bias, float* y);
NNB_API nnb_status nnb_conv2d_ex_bwd(void* stream, size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh,
		size_t kw, int stride, int padding, int dilation, int groups, const float* grad, const float* x,
		const float* weight, float* dx, int dx_first, float* dweight, int dweight_first, float* dbias,
		int dbias_first);

/* ---- support ops on the configs' paths ----------------------------------------------------- */

/* relu (ops.cpp:775-793) */
NNB_API nnb_status nnb_relu_fwd(void* stream, size_t n, const float* x, float* y);
NNB_API nnb_status nnb_relu_bwd(void* stream, size_t n, const float* x, const float* g, float* dx, int dx_first);
/* tanh-GELU (ops.cpp:451-481, kernels::tanh_inplace src/kernels/vmath.cpp:117): tanh_saved gets the
 * tanh for the backward pass; the backward recomputes it when tanh_saved is NULL. */
NNB_API nnb_status nnb_gelu_fwd(void* stream, size_t n, const float* x, float* y, float* tanh_saved);
NNB_API nnb_status nnb_gelu_bwd(void* stream, size_t n, const float* x, const float* tanh_saved, const float* g,
		float* dx, int dx_first);
/* y[0..n) = value (Tensor(shape, fill) / Tensor::zeros, include/nn/tensor.hpp:147,354). */
NNB_API nnb_status nnb_fill(void* stream, size_t n, float value, float* y);
/* y = alpha * x (Tensor scale, src/tensor.cpp:558-566). */
NNB_API nnb_status nnb_scale(void* stream, size_t n, float alpha, const float* x, float* y);
/* y = a + b, b repeated every b_period elements (add with a broadcast leading axis, ops.cpp:331). */
NNB_API nnb_status nnb_add_fwd(void* stream, size_t n, const float* a, const float* b, size_t b_period, float* y);
/* dst (+)= src or (-)= src with the grad_accum convention (ops.cpp:77-92, add_to_grad). */
NNB_API nnb_status nnb_accumulate(void* stream, size_t n, const float* src, float* dst, int first, int negate);
/* maxpool2d (ops.cpp:1609-1705): argmax = offset inside the plane, first maximum wins. */
NNB_API nnb_status nnb_maxpool2d_fwd(void* stream, size_t N, size_t C, size_t H, size_t W, size_t kernel,
		size_t stride, const float* x, float* y, uint32_t* argmax);
NNB_API nnb_status nnb_maxpool2d_bwd(void* stream, size_t N, size_t C, size_t H, size_t W, size_t kernel,
		size_t stride, const float* g, const uint32_t* argmax, float* dx, int dx_first);
/* avgpool2d (ops.cpp:1707-1772): window sums in (row, column) order times 1/kernel^2. */
NNB_API nnb_status nnb_avgpool2d_fwd(void* stream, size_t N, size_t C, size_t H, size_t W, size_t kernel,
		size_t stride, const float* x, float* y);
NNB_API nnb_status nnb_avgpool2d_bwd(void* stream, size_t N, size_t C, size_t H, size_t W, size_t kernel,
		size_t stride, const float* g, float* dx, int dx_first);
/* sum / mean over one axis of x viewed as [outer, n, inner] (Value sum / mean, ops.hpp:86-88;
 * reduce_axis ops.cpp:284-376): a serial sum from +0, times 1/n for the mean. */
NNB_API nnb_status nnb_reduce_axis_fwd(void* stream, size_t outer, size_t n, size_t inner, const float* x, int average,
		float* y);
NNB_API nnb_status nnb_reduce_axis_bwd(void* stream, size_t outer, size_t n, size_t inner, const float* g, int average,
		float* dx, int dx_first);
/* cross_entropy_loss (ops.cpp:1774-1840) over logits [N, C], targets (device int64) [N]; loss and
 * norm are device scalars (norm = N, the divisor of the backward scale). An out-of-range target
 * makes the loss NaN and sets the device error word (the reference throws TensorIndexError). */
NNB_API nnb_status nnb_cross_entropy_fwd(void* stream, size_t N, size_t C, const float* logits,
		const int64_t* targets, float* softmax, float* loss, float* norm);
NNB_API nnb_status nnb_cross_entropy_bwd(void* stream, size_t N, size_t C, const float* softmax,
		const int64_t* targets, const float* grad_loss, const float* norm, float* dlogits, int first);
/* sequence_cross_entropy (ops.cpp:1908-1979) over P positions of V logits with ignore_index and
 * label smoothing; norm = 1/count of non-ignored positions (device scalar). */
NNB_API nnb_status nnb_sequence_ce_fwd(void* stream, size_t P, size_t V, const float* logits,
		const int64_t* targets, int64_t ignore_index, float label_smoothing, float* softmax, float* loss,
		float* norm);
NNB_API nnb_status nnb_sequence_ce_bwd(void* stream, size_t P, size_t V, const float* softmax,
		const int64_t* targets, int64_t ignore_index, float label_smoothing, const float* grad_loss,
		const float* norm, float* dlogits, int first);
/* embedding (ops.cpp:1991-2015): out[i] = weight[ids[i]]; the backward adds g rows into dweight in
 * token order per row (deterministic, no float atomics), starting from 0 when first != 0 and from
 * dweight's contents otherwise; V <= 40000 for the backward. */
NNB_API nnb_status nnb_embedding_fwd(void* stream, size_t V, size_t D, const float* weight, const int64_t* ids,
		size_t count, float* out);
NNB_API nnb_status nnb_embedding_bwd(void* stream, size_t V, size_t D, const int64_t* ids, size_t count,
		const float* g, float* dweight, int first);
/* embedding backward per group of count/groups consecutive ids, group z into
 * dweight + z*dweight_stride (0: V*D). */
NNB_API nnb_status nnb_embedding_bwd_grouped(void* stream, size_t V, size_t D, size_t groups, const int64_t* ids,
		size_t count, const float* g, float* dweight, size_t dweight_stride, int first);
/* One AdamW step on one parameter (src/optim/adamw.cpp:15-24 then src/optim/adam.cpp:24-43);
 * step counts from 1 (the value of Adam::t_ after its increment). */
NNB_API nnb_status nnb_adamw_step(void* stream, size_t n, float* w, const float* g, float* m, float* v, float lr,
		float beta1, float beta2, float eps, float weight_decay, long long step);
/* Adam's bias corrections (adam.cpp:25-27) for t = 1..len as out[2(t-1)] = 1 - beta1^t and
 * out[2(t-1)+1] = 1 - beta2^t, computed on the host exactly as the reference computes them; the
 * table ends at the first t where both are exactly 1.0f (every later t has the same values) or at
 * max_len (at most 2^24). Returns len. Host only. */
NNB_API size_t nnb_adam_bias_table(float beta1, float beta2, float* out, size_t max_len);
/* *step += 1 on the device (a step counter that CUDA-graph replays advance). */
NNB_API nnb_status nnb_step_advance(void* stream, int64_t* step);
/* nnb_adamw_step with its scalars in device memory, for CUDA-graph replay: hyper = {1 - lr * wd, lr,
 * beta1, beta2, eps}, the corrections table[min(*step, table_len) - 1] from nnb_adam_bias_table.
 * Same arithmetic, same bits. */
NNB_API nnb_status nnb_adamw_step_device(void* stream, size_t n, float* w, const float* g, float* m, float* v,
		const float* hyper, const float* bias_table, size_t table_len, const int64_t* step);

/*
 * nnb_sgemm_ex for callers that cannot allocate device memory. This entry point has no
 * counterpart in the reference (nn-cpp has no GPU and no allocator boundary); it exists for hosts
 * that must not enter the CUDA allocator on the call path: an application that has already handed
 * all device memory to its own arena, a latency-critical loop where cudaMalloc's device-wide
 * synchronisation (or a memory-pool growth) is not acceptable, or an embedding whose allocator is
 * not ours to call. The caller still passes A, B and C; the packed operands and flags go into a
 * fixed 32 MiB device array that every GPU loading this library holds until the process exits.
 *
 * - Limit: (roundup(m,128) * roundup(k,32) + roundup(n,256) * roundup(k,16)) * S * 4 bytes of
 *   packed operands plus a few KB of flags must fit in 32 MiB (S = 2 in NNB_MATH_FP32X3, 1 in
 *   NNB_MATH_TF32); e.g. 1024 x 1024 x 1024 in 3xTF32 uses 16 MiB. Larger calls return NNB_ERR_UNSUPPORTED and
 *   enqueue nothing.
 * - The first call on a device (with that device current) looks up the array's device address and
 *   sets kernel attributes; make that first call before any stream capture.
 * - All calls share the array, which keeps the last call's contents; the flags that must start at
 *   zero are cleared on the stream by every call. Calls that overlap on the GPU race on the array:
 *   order them (one stream, or events) yourself.
 * - No cudaMalloc/cudaFree or other allocating routine is called. A bounded wait that expires in this
 *   entry point's kernels is recorded in a device word of its own, not in nnb_device_error: read it
 *   with nnb_sgemm_noalloc_error after the calls whose results matter.
 * - The tile is always 256 columns wide and the product is never cut along its depth. nnb_sgemm_ex
 *   cuts a long-depth product (k >= 2 * max(1024, n)) into consecutive depth pieces summed in order
 *   (its counterpart of the reference's depth cut, gemm.cpp:453-485), so for such shapes the two
 *   entry points give different bits (both within the fp32 bound) and this one keeps fewer SMs busy
 *   when the output is small. For every other shape they give the same bits.
 */
NNB_API nnb_status nnb_sgemm_noalloc(void* stream, int trans_a, int trans_b, size_t m, size_t n,
		size_t k, const float* a, size_t lda, const float* b, size_t ldb, float* c, size_t ldc,
		int accumulate, int math_mode);
/* The error word of nnb_sgemm_noalloc's kernels on the current device (no counterpart in the
 * reference): *out = 0 if no bounded wait in them has expired since the word was last cleared,
 * otherwise the code of the first wait that gave up (1-6, the same codes nnb_device_error reports);
 * the C of that call is then incomplete. Waits for `stream` to reach this point and clears the word
 * when `clear` is set. Allocates nothing (plain copies from and to the device symbol). */
NNB_API nnb_status nnb_sgemm_noalloc_error(void* stream, int* out, int clear);

/* ---- random streams and dropout (src/random.cpp, src/nn/dropout.cpp) ------------------------ */

/* manual_seed / is_seeded / seed_epoch (include/nn/random.hpp:25-47); host only. */
NNB_API void nnb_manual_seed(uint64_t seed);
NNB_API int nnb_is_seeded(void);
NNB_API uint64_t nnb_seed_epoch(void);
/* derive_generator(stream) (random.hpp:58, random.cpp:67-79) as an mt19937 state in HOST memory:
 * state[0..623] the untempered words, state[624] the index of the next word (624 after seeding).
 * Copy it to the device for nnb_dropout_mask. Host only. */
NNB_API nnb_status nnb_derive_generator(const char* stream_name, uint32_t* state);
/* std::mt19937 seeded from std::seed_seq{seeds[0..count)}, in the same 625-word form; host only. */
NNB_API nnb_status nnb_mt19937_seed_seq(const uint32_t* seeds, size_t count, uint32_t* state);
/* Dropout::forward's draws (dropout.cpp:20-31): n outputs from the DEVICE state (advanced in place)
 * into the keep mask keep[(n + 31) / 32] (bit e % 32 of word e / 32 = element e kept, i.e.
 * u = float(x >> 8) * 2^-24 >= p). p == 0 keeps and p == 1 drops everything without drawing. */
NNB_API nnb_status nnb_dropout_mask(void* stream, uint32_t* state, size_t n, float p, uint32_t* keep);
/* The same draw of `total` outputs (the state ends where nnb_dropout_mask(total) leaves it) keeping
 * only the decisions of outputs [offset, offset + count) in keep[(count + 31) / 32] (bit e of the
 * slice = output offset + e; offset a multiple of 32): one data-parallel rank's rows of a layer's
 * mask, bit for bit the rows of the whole batch's mask (dropout.cpp:20-31 draws the batch row-major
 * from one generator). The serial generator still runs through every output. */
NNB_API nnb_status nnb_dropout_mask_slice(void* stream, uint32_t* state, size_t total, size_t offset, size_t count,
		float p, uint32_t* keep);
/* y = x * m, m = kept ? 1 / (1 - p) : 0 (mul with the mask, ops.cpp:347). */
NNB_API nnb_status nnb_dropout_apply(void* stream, size_t n, float p, const float* x, const uint32_t* keep, float* y);
/* dx (+)= g * m with the grad_accum convention. */
NNB_API nnb_status nnb_dropout_bwd(void* stream, size_t n, float p, const float* g, const uint32_t* keep, float* dx,
		int dx_first);

/* Host-side draws of the reference's data pipeline (all host only, no device work):
 * std::mt19937(seed) linear seeding (random_split, src/data/subset.cpp:63) in the 625-word form;
 * n raw outputs of a host state; the FNV-1a / splitmix64 functions of derive_generator
 * (random.hpp detail::); the portable Fisher-Yates shuffle (src/data/shuffle.hpp:45-49, rejection
 * draws from raw outputs); the weighted draws of a weighted DataLoader epoch
 * (dataloader.cpp:58-69: 53-bit uniform from two outputs, first running sum above u * total). */
NNB_API nnb_status nnb_mt19937_seed(uint32_t seed, uint32_t* state);
NNB_API nnb_status nnb_mt19937_next(uint32_t* state, size_t n, uint32_t* out);
NNB_API uint64_t nnb_fnv1a64(const char* s);
NNB_API uint64_t nnb_splitmix64(uint64_t x);
NNB_API nnb_status nnb_portable_shuffle(uint32_t* state, uint64_t* v, size_t n);
NNB_API nnb_status nnb_weighted_draws(uint32_t* state, const double* cumulative, size_t count, size_t num_samples,
		uint64_t* out);

/* ---- batch assembly from HBM-resident datasets (DataLoader::get_batch, dataloader.cpp:76-96) --- */

/* dst[r] = src[index[r]] for r < count, rows of row_bytes bytes (TensorDataset rows). An index
 * outside [0, rows) writes a zero row and sets the device error word. */
NNB_API nnb_status nnb_gather_rows(void* stream, const void* src, size_t row_bytes, size_t rows, const int64_t* index,
		size_t count, void* dst);
/* SequenceDataset windows (src/data/text.cpp:60-70): x[b][t] = tokens[start[b] + t],
 * y[b][t] = tokens[start[b] + 1 + t], t < block, as int64 ids; start[b] < n_tokens - block. */
NNB_API nnb_status nnb_gather_windows(void* stream, const int32_t* tokens, size_t n_tokens, const int64_t* start,
		size_t count, size_t block, int64_t* x, int64_t* y);

#ifdef __cplusplus
}
#endif

#endif /* NNB_H */
