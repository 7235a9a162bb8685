// ops_linear.cu -- `linear` (src/autograd/ops.cpp:714-745) and the column reduction its bias
// gradient needs.
//
// Forward: one GEMM Y = X W^T with the bias added in the epilogue (acc + 0, then + b[j]: the
// reference's sgemm store followed by `out += b[j]`, ops.cpp:725-730).
// Backward: dX (+)= G W and dW (+)= G^T X are GEMMs with accumulate = !first (ops.cpp:737,741);
// db (+)= the column sums of G.
//
// Column sums: the reference reduces the rows of G one after another per column
// (Tensor::sum(0), src/tensor.cpp:422-455). A strictly serial column sum would leave a GPU with
// one thread per column, so it is split into chunks of kColChunk rows, each summed serially from
// +0 in row order, and the chunk partials are then summed serially in chunk order. The order
// depends only on the number of rows, never on the launch, and with at most kColChunk rows it is
// the reference's order exactly.
#include "nnb_gemm.h"
#include "nnb_internal.h"
#include "nnb_math.cuh"
#include "nnb_ops.h"
#include "nnb_trace.h"

namespace nnb {

namespace {

constexpr int kColChunk = 256;

// y = gelu(pre) with the tanh of the reference's Cephes method (ops.cpp:451-466), four elements per
// thread when aligned
__global__ void gelu_apply_vec_kernel(long long n4, const float* __restrict__ pre, float* __restrict__ y) {
	for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
		const float4 v = __ldg(reinterpret_cast<const float4*>(pre) + i);
		reinterpret_cast<float4*>(y)[i] = make_float4(gelu_fwd(v.x, tanh_one(gelu_tanh_arg(v.x))),
			gelu_fwd(v.y, tanh_one(gelu_tanh_arg(v.y))), gelu_fwd(v.z, tanh_one(gelu_tanh_arg(v.z))),
			gelu_fwd(v.w, tanh_one(gelu_tanh_arg(v.w))));
	}
}
__global__ void gelu_apply_kernel(long long n, const float* __restrict__ pre, float* __restrict__ y) {
	for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
		const float v = pre[i];
		y[i] = gelu_fwd(v, tanh_one(gelu_tanh_arg(v)));
	}
}

// partial[z][c][j] = sum over rows [c*kColChunk, ...) of group z of g[r][j], serial from +0.
__global__ void colsum_partial_kernel(const float* __restrict__ g, long long rows, long long cols,
		float* __restrict__ partial) {
	const long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x;
	const long long c = blockIdx.y, chunks = gridDim.y, z = blockIdx.z;
	if (j >= cols) return;
	const float* gz = g + z * rows * cols + j;
	const long long r0 = c * kColChunk, r1 = min(rows, r0 + kColChunk);
	// serial in row order; 32 loads are issued ahead of their adds so that each thread keeps enough
	// bytes in flight for the column walk to run at HBM speed
	float s = 0.0f;
	long long r = r0;
	for (; r + 32 <= r1; r += 32) {
		float v[32];
#pragma unroll
		for (int u = 0; u < 32; ++u) v[u] = __ldg(gz + (r + u) * cols);
#pragma unroll
		for (int u = 0; u < 32; ++u) s += v[u];
	}
	for (; r < r1; ++r) s += __ldg(gz + r * cols);
	partial[(z * chunks + c) * cols + j] = s;
}

// The same partials for tall, narrow sums (one shard's bias gradient: 4096 rows x 512 columns): a
// block of 256 threads stages its chunk's rows x 32 columns in shared memory with every load in
// flight, then warp 0 sums each column serially in row order from +0 -- the same additions in the
// same order as colsum_partial_kernel, without its per-thread latency chain.
__global__ void __launch_bounds__(256) colsum_partial_staged_kernel(const float* __restrict__ g, long long rows,
		long long cols, float* __restrict__ partial) {
	__shared__ __align__(16) float tile[kColChunk][32];
	const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
	const long long j = blockIdx.x * 32LL + lane;
	const long long c = blockIdx.y, chunks = gridDim.y, z = blockIdx.z;
	const long long r0 = c * kColChunk, n = min(rows - r0, (long long)kColChunk);
	const float* gz = g + z * rows * cols;
	const long long j0 = blockIdx.x * 32LL;
	if (n == kColChunk && j0 + 32 <= cols && cols % 4 == 0 && (reinterpret_cast<uintptr_t>(g) & 15) == 0) {
		// a whole chunk of 32 full columns: eight 16-byte loads per thread, all issued before any store
		const int c4 = (threadIdx.x & 7) * 4, rq = threadIdx.x >> 3;
		float4 v[kColChunk / 32];
#pragma unroll
		for (int u = 0; u < kColChunk / 32; ++u)
			v[u] = __ldg(reinterpret_cast<const float4*>(gz + (r0 + rq + 32 * u) * cols + j0 + c4));
#pragma unroll
		for (int u = 0; u < kColChunk / 32; ++u) *reinterpret_cast<float4*>(&tile[rq + 32 * u][c4]) = v[u];
	} else {
		for (int rr = warp; rr < n; rr += 8) tile[rr][lane] = j < cols ? __ldg(gz + (r0 + rr) * cols + j) : 0.0f;
	}
	__syncthreads();
	if (warp != 0 || j >= cols) return;
	float s = 0.0f;
	for (int rr = 0; rr < n; ++rr) s += tile[rr][lane];
	partial[(z * chunks + c) * cols + j] = s;
}

// out[z*out_stride + j] = (first ? 0 : out[..]) + sum_c partial[z][c][j] (serial from +0 in chunk order).
__global__ void colsum_final_kernel(const float* __restrict__ partial, long long chunks, long long cols,
		float* __restrict__ out, long long out_stride, int first) {
	const long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x;
	const long long z = blockIdx.y;
	if (j >= cols) return;
	const float* pz = partial + z * chunks * cols;
	float s = 0.0f;
	for (long long c = 0; c < chunks; ++c) s += pz[c * cols + j];
	float* o = out + z * out_stride + j;
	*o = first ? s + 0.0f : *o + s;
}

}  // namespace

// The two GEMMs of a linear backward that read the output gradient G [rows x n]: dX = G W packs G as
// its A operand (once, even when dX is cut along its depth); when both run that pack is kept in a scratch
// buffer and the weight gradient dW = G^T X reads it MN-major instead of packing G^T again -- one
// pass over G instead of two, with the same bits. Likewise X: when the forward kept its pack
// (x_pack, written in math mode x_pack_mode by nnb_linear_fwd_ex), dW reads X from it instead of
// packing X^T. `groups` consecutive row blocks of G and X give one weight gradient each (dw_stride
// apart).
nnb_status linear_bwd_gemms(cudaStream_t s, long long rows, long long K, long long n, long long groups, const float* g,
		const float* x, const void* x_pack, int x_pack_mode, const float* w, float* dx, int dx_first, float* dw,
		long long dw_stride, int dw_first) {
	const int mode = math_mode();
	const long long rg = rows / groups;
	GemmDesc dxd;                 // dX = G W: [rows, n] x [n, K]
	dxd.m = rows; dxd.n = K; dxd.k = n;
	dxd.a = g; dxd.lda = n; dxd.b = w; dxd.ldb = K; dxd.c = dx; dxd.ldc = K;
	dxd.accumulate = !dx_first; dxd.mode = mode;
	GemmDesc dwd;                 // dW_z = G_z^T X_z: [n, rg] x [rg, K] per group z, one batched launch
	dwd.ta = 1;
	dwd.m = n; dwd.n = K; dwd.k = rg;
	dwd.a = g; dwd.lda = n; dwd.b = x; dwd.ldb = K; dwd.c = dw; dwd.ldc = K;
	dwd.batch_outer = groups;
	if (groups > 1) {
		dwd.sa_outer = rg * n; dwd.sb_outer = rg * K;
		dwd.sc_outer = dw_stride ? dw_stride : n * K;
	}
	dwd.accumulate = !dw_first; dwd.mode = mode;
	void* kept = nullptr;
	// the weight gradient can read the pack only when every group is whole 16-row blocks
	if (dx && dw && rows > 0 && n > 0 && K > 0 && rg % 16 == 0) {
		NNB_TRY(scratch_alloc(&kept, gemm_row_pack_bytes(rows, n, mode), s));
		dxd.keep_a = kept;
		dwd.mn_a.buf = kept; dwd.mn_a.base = g; dwd.mn_a.ld = n; dwd.mn_a.rows = rows; dwd.mn_a.cols = n;
		dwd.mn_a.mode = mode;
	}
	if (x_pack) {
		dwd.mn_b.buf = x_pack; dwd.mn_b.base = x; dwd.mn_b.ld = K; dwd.mn_b.rows = rows; dwd.mn_b.cols = K;
		dwd.mn_b.mode = x_pack_mode;
	}
	nnb_status st = NNB_OK;
	if (dx) st = gemm_run(s, dxd);
	if (st == NNB_OK && dw) st = gemm_run(s, dwd);
	nnb_status st2 = scratch_free(kept, s);
	return st != NNB_OK ? st : st2;
}

nnb_status colsum(cudaStream_t s, const float* g, long long rows, long long cols, float* out, int first) {
	return colsum_grouped(s, g, rows, cols, 1, out, cols, first);
}

nnb_status colsum_grouped(cudaStream_t s, const float* g, long long rows, long long cols, long long groups, float* out,
		long long out_stride, int first) {
	if (cols == 0 || groups == 0) return NNB_OK;
	if (rows % groups != 0) return fail(NNB_ERR_SHAPE, "column sum: %lld rows do not split into %lld groups", rows, groups);
	rows /= groups;                                   // rows per group
	if (rows == 0) {
		if (first)
			for (long long z = 0; z < groups; ++z) NNB_CUDA_TRY(cudaMemsetAsync(out + z * out_stride, 0, cols * sizeof(float), s));
		return NNB_OK;
	}
	const long long chunks = (rows + kColChunk - 1) / kColChunk;
	if (chunks > 65535 || groups > 65535) return fail(NNB_ERR_UNSUPPORTED, "column sum too large for one launch");
	void* ws = nullptr;
	NNB_TRY(scratch_alloc(&ws, groups * chunks * cols * sizeof(float), s));
	float* partial = static_cast<float*>(ws);
	// The chunk partition (the summation order) is fixed by the row count; the block width only sets how
	// many blocks share the SMs: 32 columns per block when the columns alone would not fill them (one
	// shard's 512 columns x 16 chunks become 256 blocks), 128 for wide sums (the shard-gradient sum)
	const unsigned tpb = cols * chunks * groups >= 148LL * 1024 ? 128u : 32u;
	const unsigned bx = (unsigned)((cols + tpb - 1) / tpb);
	{
		TraceScope ts(s, kTraceRowwise);
		if (rows >= 64)          // tall sums: staged through shared memory (same order, loads in flight)
			colsum_partial_staged_kernel<<<dim3((unsigned)((cols + 31) / 32), (unsigned)chunks, (unsigned)groups), 256, 0,
				s>>>(g, rows, cols, partial);
		else
			colsum_partial_kernel<<<dim3(bx, (unsigned)chunks, (unsigned)groups), tpb, 0, s>>>(g, rows, cols, partial);
	}
	{
		TraceScope ts(s, kTraceRowwise);
		colsum_final_kernel<<<dim3(bx, (unsigned)groups), tpb, 0, s>>>(partial, chunks, cols, out, out_stride, first);
	}
	nnb_status st = cuda_status(cudaGetLastError(), "column sum launch");
	nnb_status st2 = scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

}  // namespace nnb

extern "C" {

nnb_status nnb_linear_fwd(void* stream, size_t M, size_t K, size_t n, const float* x, const float* w,
		const float* bias, float* y) {
	if (M == 0 || n == 0) return NNB_OK;
	if (!x || !w || !bias || !y) return nnb::fail(NNB_ERR_INVALID, "linear_fwd: null pointer");
	if (K == 0) return nnb::fail(NNB_ERR_SHAPE, "linear_fwd: zero input features");
	nnb::GemmDesc d;
	d.ta = 0; d.tb = 1;
	d.m = (long long)M; d.n = (long long)n; d.k = (long long)K;
	d.a = x; d.lda = (long long)K; d.b = w; d.ldb = (long long)K; d.c = y; d.ldc = (long long)n;
	d.mode = nnb::math_mode();
	d.epi.bias = bias; d.epi.bias_mode = nnb::kBiasCol;
	return nnb::gemm_run(static_cast<cudaStream_t>(stream), d);
}

nnb_status nnb_linear_multi_fwd(void* stream, size_t count, size_t M, size_t K, size_t n, const float* x, const float* w,
		size_t w_stride, const float* bias, size_t bias_stride, float* y, size_t y_stride) {
	if (count == 0 || M == 0 || n == 0) return NNB_OK;
	if (!x || !w || !bias || !y) return nnb::fail(NNB_ERR_INVALID, "linear_multi_fwd: null pointer");
	if (K == 0) return nnb::fail(NNB_ERR_SHAPE, "linear_multi_fwd: zero input features");
	if (count > 1 && (w_stride < n * K || bias_stride < n || y_stride < M * n))
		return nnb::fail(NNB_ERR_INVALID, "linear_multi_fwd: strides overlap consecutive weights, biases or outputs");
	if (count > 65535) return nnb::fail(NNB_ERR_UNSUPPORTED, "linear_multi_fwd: more than 65535 weights");
	// one batched GEMM whose A (x) is shared by every entry, so x is packed once; entry i is the product
	// nnb_linear_fwd would compute for (x, w_i, b_i), with the same operations for every element
	nnb::GemmDesc d;
	d.ta = 0; d.tb = 1;
	d.m = (long long)M; d.n = (long long)n; d.k = (long long)K;
	d.a = x; d.lda = (long long)K; d.b = w; d.ldb = (long long)K; d.c = y; d.ldc = (long long)n;
	d.batch_outer = (long long)count;
	d.sa_outer = 0; d.sb_outer = (long long)w_stride; d.sc_outer = (long long)y_stride;
	d.mode = nnb::math_mode();
	d.epi.bias = bias; d.epi.bias_mode = nnb::kBiasCol; d.epi.s_bias_outer = (long long)bias_stride;
	return nnb::gemm_run(static_cast<cudaStream_t>(stream), d);
}

nnb_status nnb_linear_gelu_fwd(void* stream, size_t M, size_t K, size_t n, const float* x, const float* w,
		const float* bias, float* y, float* pre) {
	if (M == 0 || n == 0) return NNB_OK;
	if (!x || !w || !bias || !y || !pre) return nnb::fail(NNB_ERR_INVALID, "linear_gelu_fwd: null pointer");
	if (K == 0) return nnb::fail(NNB_ERR_SHAPE, "linear_gelu_fwd: zero input features");
	// The GEMM stores pre = x w^T + b (bias in its epilogue); the GELU then runs as its own HBM-bound
	// pass. Computing the Cephes tanh inside the GEMM epilogue (4 warps per SM) left the tensor cores
	// waiting on it; the separate pass gives the same bits (the same function of the same pre).
	nnb::GemmDesc d;
	d.ta = 0; d.tb = 1;
	d.m = (long long)M; d.n = (long long)n; d.k = (long long)K;
	d.a = x; d.lda = (long long)K; d.b = w; d.ldb = (long long)K; d.c = pre; d.ldc = (long long)n;
	d.mode = nnb::math_mode();
	d.epi.bias = bias; d.epi.bias_mode = nnb::kBiasCol;
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	NNB_TRY(nnb::gemm_run(s, d));
	const long long total = (long long)M * (long long)n;
	nnb::TraceScope ts(s, nnb::kTraceRowwise);
	if (total % 4 == 0 && ((reinterpret_cast<uintptr_t>(pre) | reinterpret_cast<uintptr_t>(y)) & 15) == 0)
		nnb::gelu_apply_vec_kernel<<<nnb::grid_for(total / 4, 256), 256, 0, s>>>(total / 4, pre, y);
	else
		nnb::gelu_apply_kernel<<<nnb::grid_for(total, 256), 256, 0, s>>>(total, pre, y);
	return nnb::cuda_status(cudaGetLastError(), "linear_gelu_fwd gelu launch");
}

nnb_status nnb_linear_bwd(void* stream, size_t M, size_t K, size_t n, const float* g, const float* x,
		const float* w, float* dx, int dx_first, float* dw, int dw_first, float* db, int db_first) {
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	if (!g || !x || !w) return nnb::fail(NNB_ERR_INVALID, "linear_bwd: null input");
	// dX = G W: [M, n] x [n, K]; dW = G^T X: [n, M] x [M, K]
	NNB_TRY(nnb::linear_bwd_gemms(s, (long long)M, (long long)K, (long long)n, 1, g, x, nullptr, 0, w, dx, dx_first, dw,
		0, dw_first));
	if (db) NNB_TRY(nnb::colsum(s, g, (long long)M, (long long)n, db, db_first));
	return NNB_OK;
}

nnb_status nnb_linear_bwd_grouped(void* stream, size_t M, size_t K, size_t n, size_t groups, const float* g,
		const float* x, const float* w, float* dx, int dx_first, float* dw, size_t dw_stride, int dw_first, float* db,
		size_t db_stride, int db_first) {
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	if (!g || !x || !w) return nnb::fail(NNB_ERR_INVALID, "linear_bwd_grouped: null input");
	if (groups == 0 || M % groups != 0) return nnb::fail(NNB_ERR_SHAPE, "linear_bwd_grouped: %zu rows in %zu groups", M, groups);
	// dX = G W over all rows; dW_z = G_z^T X_z per group z, one batched launch (depth-cut per group)
	NNB_TRY(nnb::linear_bwd_gemms(s, (long long)M, (long long)K, (long long)n, (long long)groups, g, x, nullptr, 0, w,
		dx, dx_first, dw, (long long)dw_stride, dw_first));
	if (db)
		NNB_TRY(nnb::colsum_grouped(s, g, (long long)M, (long long)n, (long long)groups, db,
			db_stride ? (long long)db_stride : (long long)n, db_first));
	return NNB_OK;
}

size_t nnb_linear_pack_bytes(size_t M, size_t K, int math_mode) {
	if (math_mode != NNB_MATH_FP32X3 && math_mode != NNB_MATH_TF32) return 0;
	return nnb::gemm_row_pack_bytes((long long)M, (long long)K, math_mode);
}

nnb_status nnb_linear_fwd_ex(void* stream, size_t count, size_t M, size_t K, size_t n, const float* x, const float* w,
		size_t w_stride, const float* bias, size_t bias_stride, float* y, size_t y_stride, float* pre, void* x_pack) {
	if (count == 0 || M == 0 || n == 0) return NNB_OK;
	if (!x || !w || !bias || !y) return nnb::fail(NNB_ERR_INVALID, "linear_fwd_ex: null pointer");
	if (K == 0) return nnb::fail(NNB_ERR_SHAPE, "linear_fwd_ex: zero input features");
	if (pre && count != 1) return nnb::fail(NNB_ERR_INVALID, "linear_fwd_ex: the GELU form takes one weight");
	if (count > 1 && (w_stride < n * K || bias_stride < n || y_stride < M * n))
		return nnb::fail(NNB_ERR_INVALID, "linear_fwd_ex: strides overlap consecutive weights, biases or outputs");
	if (count > 65535) return nnb::fail(NNB_ERR_UNSUPPORTED, "linear_fwd_ex: more than 65535 weights");
	// the products of nnb_linear_fwd / nnb_linear_multi_fwd / nnb_linear_gelu_fwd (same bits); x's pack
	// (the A operand every entry shares) is written into x_pack and left there for the backward
	nnb::GemmDesc d;
	d.ta = 0; d.tb = 1;
	d.m = (long long)M; d.n = (long long)n; d.k = (long long)K;
	d.a = x; d.lda = (long long)K; d.b = w; d.ldb = (long long)K; d.c = pre ? pre : y; d.ldc = (long long)n;
	if (count > 1) {
		d.batch_outer = (long long)count;
		d.sb_outer = (long long)w_stride; d.sc_outer = (long long)y_stride;
		d.epi.s_bias_outer = (long long)bias_stride;
	}
	d.mode = nnb::math_mode();
	d.epi.bias = bias; d.epi.bias_mode = nnb::kBiasCol;
	d.keep_a = x_pack;
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	NNB_TRY(nnb::gemm_run(s, d));
	if (!pre) return NNB_OK;
	const long long total = (long long)M * (long long)n;
	nnb::TraceScope ts(s, nnb::kTraceRowwise);
	if (total % 4 == 0 && ((reinterpret_cast<uintptr_t>(pre) | reinterpret_cast<uintptr_t>(y)) & 15) == 0)
		nnb::gelu_apply_vec_kernel<<<nnb::grid_for(total / 4, 256), 256, 0, s>>>(total / 4, pre, y);
	else
		nnb::gelu_apply_kernel<<<nnb::grid_for(total, 256), 256, 0, s>>>(total, pre, y);
	return nnb::cuda_status(cudaGetLastError(), "linear_fwd_ex gelu launch");
}

nnb_status nnb_linear_bwd_ex(void* stream, size_t M, size_t K, size_t n, size_t groups, const float* g, const float* x,
		const void* x_pack, int x_pack_mode, const float* w, float* dx, int dx_first, float* dw, size_t dw_stride,
		int dw_first, float* db, size_t db_stride, int db_first) {
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	if (!g || !x || !w) return nnb::fail(NNB_ERR_INVALID, "linear_bwd_ex: null input");
	if (groups == 0 || M % groups != 0) return nnb::fail(NNB_ERR_SHAPE, "linear_bwd_ex: %zu rows in %zu groups", M, groups);
	NNB_TRY(nnb::linear_bwd_gemms(s, (long long)M, (long long)K, (long long)n, (long long)groups, g, x, x_pack,
		x_pack_mode, w, dx, dx_first, dw, groups > 1 ? (long long)dw_stride : 0, dw_first));
	if (db) {
		if (groups > 1)
			NNB_TRY(nnb::colsum_grouped(s, g, (long long)M, (long long)n, (long long)groups, db,
				db_stride ? (long long)db_stride : (long long)n, db_first));
		else
			NNB_TRY(nnb::colsum(s, g, (long long)M, (long long)n, db, db_first));
	}
	return NNB_OK;
}

nnb_status nnb_column_sum(void* stream, size_t rows, size_t cols, const float* g, float* out, int first) {
	if (cols && (!g || !out)) return nnb::fail(NNB_ERR_INVALID, "column_sum: null pointer");
	return nnb::colsum(static_cast<cudaStream_t>(stream), g, (long long)rows, (long long)cols, out, first);
}

}  // extern "C"
