// ops_attention.cu -- multi-head `attention` (src/autograd/ops.cpp:1226-1296) with the masked
// softmax of ops.cpp:1183-1224.
//
// The reference loops over (sample n, head h) and runs two sgemm calls per pair with heads read in
// place (row stride D, column offset h*Dh). Here each of those products is ONE launch of the
// tensor-core GEMM over all N*H pairs (a two-level batch: outer stride over samples, inner
// stride over heads), so the N*H small products fill the machine together. The probabilities P
// {N, H, Tq, Tk} are kept for the backward pass, as the reference keeps them.
//
// Softmax rows (one warp per row): scale, key-padding mask -> -1e9, causal j > i -> -2e9, max,
// exp of the live prefix (causally hidden keys are exactly 0), normalise. Backward: dot = g.y,
// g = masked ? 0 : scale*(y*(g - dot)) + 0.
#include <cmath>

#include "nnb_gemm.h"
#include "nnb_internal.h"
#include "nnb_ops.h"
#include "nnb_trace.h"

namespace nnb {

namespace {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
	for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
	return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
	for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
	return v;
}

__device__ __forceinline__ float keep_factor(const uint32_t* keep, long long i, float keep_scale) {
	return ((keep[i >> 5] >> (i & 31)) & 1u) ? keep_scale : 0.0f;
}

// rows = N*H*Tq rows of Tk scores, in place. Row r: n = r / (H*Tq), i = r % Tq. With a keep mask
// (dropout on the weights, attention.cpp:43-45) the dropped weights P * m also go to `weights`,
// m = kept ? keep_scale : 0 (bit e of keep[e / 32] for element e = r * Tk + j).
__global__ void masked_softmax_fwd_kernel(float* __restrict__ p, long long rows, int H, int Tq, int Tk,
		const float* __restrict__ pad, int causal, float scale, const uint32_t* __restrict__ keep = nullptr,
		float keep_scale = 0.0f, float* __restrict__ weights = nullptr) {
	const int lane = threadIdx.x & 31;
	const long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
	if (r >= rows) return;
	const long long n = r / ((long long)H * Tq);
	const int i = (int)(r % Tq);
	const float* ph = pad ? pad + n * Tk : nullptr;
	float* row = p + r * Tk;
	float m = -INFINITY;
	for (int j = lane; j < Tk; j += 32) {
		float v = row[j] * scale;
		if (ph && ph[j] == 0.0f) v = -1e9f;
		if (causal && j > i) v = -2e9f;
		row[j] = v;
		m = fmaxf(m, v);
	}
	m = warp_max(m);
	const int live = causal ? min(Tk, i + 1) : Tk;
	float s = 0.0f;
	for (int j = lane; j < Tk; j += 32) {
		if (j < live) {
			const float e = expf(row[j] - m);
			row[j] = e;
			s += e;
		} else {
			row[j] = 0.0f;
		}
	}
	s = warp_sum(s);
	if (keep) {
		float* wrow = weights + r * Tk;
		for (int j = lane; j < Tk; j += 32) {
			const float y = row[j] / s;
			row[j] = y;
			wrow[j] = y * keep_factor(keep, r * Tk + j, keep_scale);
		}
	} else {
		for (int j = lane; j < Tk; j += 32) row[j] = row[j] / s;
	}
}

// g holds dL/dP on entry and dL/dS on exit; y = P. With a keep mask g holds dL/d(P*m) on entry and
// dL/dP = g * m + 0 (mul's backward into a fresh gradient, ops.cpp:347-356, 67-73) is used.
__global__ void masked_softmax_bwd_kernel(const float* __restrict__ y, float* __restrict__ g, long long rows, int H,
		int Tq, int Tk, const float* __restrict__ pad, int causal, float scale, const uint32_t* __restrict__ keep = nullptr,
		float keep_scale = 0.0f) {
	const int lane = threadIdx.x & 31;
	const long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
	if (r >= rows) return;
	const long long n = r / ((long long)H * Tq);
	const int i = (int)(r % Tq);
	const float* ph = pad ? pad + n * Tk : nullptr;
	const float* yr = y + r * Tk;
	float* gr = g + r * Tk;
	float dot = 0.0f;
	if (keep) {
		for (int j = lane; j < Tk; j += 32) {
			const float gj = gr[j] * keep_factor(keep, r * Tk + j, keep_scale) + 0.0f;
			gr[j] = gj;
			dot += gj * yr[j];
		}
	} else {
		for (int j = lane; j < Tk; j += 32) dot += gr[j] * yr[j];
	}
	dot = warp_sum(dot);
	for (int j = lane; j < Tk; j += 32) {
		const bool masked = (ph && ph[j] == 0.0f) || (causal && j > i);
		gr[j] = masked ? 0.0f : scale * (yr[j] * (gr[j] - dot)) + 0.0f;
	}
}

// scaled_masked_softmax (ops.cpp:1298-1343) out of place: y = softmax rows of x, the same row
// arithmetic as masked_softmax_fwd_kernel. Causal rows need not be square here (row i keeps keys
// 0..i of however many there are), as in the reference.
__global__ void softmax_rows_fwd_kernel(const float* __restrict__ x, float* __restrict__ y, long long rows, int H,
		int Tq, int Tk, const float* __restrict__ pad, int causal, float scale) {
	const int lane = threadIdx.x & 31;
	const long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
	if (r >= rows) return;
	const long long n = r / ((long long)H * Tq);
	const int i = (int)(r % Tq);
	const float* ph = pad ? pad + n * Tk : nullptr;
	const float* xr = x + r * Tk;
	float* row = y + r * Tk;
	float m = -INFINITY;
	for (int j = lane; j < Tk; j += 32) {
		float v = xr[j] * scale;
		if (ph && ph[j] == 0.0f) v = -1e9f;
		if (causal && j > i) v = -2e9f;
		row[j] = v;
		m = fmaxf(m, v);
	}
	m = warp_max(m);
	const int live = causal ? min(Tk, i + 1) : Tk;
	float s = 0.0f;
	for (int j = lane; j < Tk; j += 32) {
		if (j < live) {
			const float e = expf(row[j] - m);
			row[j] = e;
			s += e;
		} else {
			row[j] = 0.0f;
		}
	}
	s = warp_sum(s);
	for (int j = lane; j < Tk; j += 32) row[j] = row[j] / s;
}

// Its backward into a gradient buffer under the grad_accum rule: first stores term + 0 (0 at masked
// positions), otherwise adds term and leaves masked positions untouched (ops.cpp:1331-1338).
__global__ void softmax_rows_bwd_kernel(const float* __restrict__ y, const float* __restrict__ g,
		float* __restrict__ dx, int first, long long rows, int H, int Tq, int Tk, const float* __restrict__ pad,
		int causal, float scale) {
	const int lane = threadIdx.x & 31;
	const long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
	if (r >= rows) return;
	const long long n = r / ((long long)H * Tq);
	const int i = (int)(r % Tq);
	const float* ph = pad ? pad + n * Tk : nullptr;
	const float* yr = y + r * Tk;
	const float* gr = g + r * Tk;
	float* dr = dx + r * Tk;
	float dot = 0.0f;
	for (int j = lane; j < Tk; j += 32) dot += gr[j] * yr[j];
	dot = warp_sum(dot);
	for (int j = lane; j < Tk; j += 32) {
		const bool masked = (ph && ph[j] == 0.0f) || (causal && j > i);
		const float term = scale * (yr[j] * (gr[j] - dot));
		if (first) dr[j] = masked ? 0.0f : term + 0.0f;
		else if (!masked) dr[j] += term;
	}
}

}  // namespace

// Head-batched GEMM over all (n, h): X_(n,h) = x + n * sx_n + h * sx_h
static GemmDesc head_gemm(int ta, int tb, long long m, long long n, long long k, const float* a, long long lda,
		long long sa_n, long long sa_h, const float* b, long long ldb, long long sb_n, long long sb_h, float* c,
		long long ldc, long long sc_n, long long sc_h, long long N, long long H, int accumulate) {
	GemmDesc d;
	d.ta = ta; d.tb = tb; d.m = m; d.n = n; d.k = k;
	d.a = a; d.lda = lda; d.b = b; d.ldb = ldb; d.c = c; d.ldc = ldc;
	d.batch_outer = N; d.batch_inner = H;
	d.sa_outer = sa_n; d.sa_inner = sa_h; d.sb_outer = sb_n; d.sb_inner = sb_h; d.sc_outer = sc_n; d.sc_inner = sc_h;
	d.accumulate = accumulate;
	d.mode = math_mode();
	return d;
}

static nnb_status check_shapes(size_t N, size_t Tq, size_t Tk, size_t D, size_t heads, int causal) {
	if (heads == 0 || D % heads != 0 || Tq == 0 || Tk == 0 || (causal && Tq != Tk))
		return fail(NNB_ERR_SHAPE, "attention: bad shapes (N %zu, Tq %zu, Tk %zu, D %zu, heads %zu, causal %d)", N, Tq,
			Tk, D, heads, causal);
	return NNB_OK;
}

}  // namespace nnb

extern "C" {

nnb_status nnb_attention_fwd(void* stream, size_t N, size_t Tq, size_t Tk, size_t D, size_t heads, const float* q,
		const float* k, const float* v, const float* key_padding_mask, int causal, float* out, float* probs) {
	NNB_TRY(nnb::check_shapes(N, Tq, Tk, D, heads, causal));
	if (N == 0) return NNB_OK;
	if (!q || !k || !v || !out || !probs) return nnb::fail(NNB_ERR_INVALID, "attention_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long H = (long long)heads, Dh = (long long)(D / heads);
	const long long qs = (long long)Tq * D, ks = (long long)Tk * D, ps = (long long)Tq * Tk;
	const float scale = 1.0f / std::sqrt(static_cast<float>(Dh));     // ops.cpp:1236
	// S = Q_h K_h^T into P  (ops.cpp:1256)
	NNB_TRY(nnb::gemm_run(s, nnb::head_gemm(0, 1, Tq, Tk, Dh, q, D, qs, Dh, k, D, ks, Dh, probs, Tk, H * ps, ps,
		N, H, 0)));
	const long long rows = (long long)N * H * Tq;
	{
		nnb::TraceScope ts(s, nnb::kTraceAttention);
		nnb::masked_softmax_fwd_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(probs, rows, (int)H, (int)Tq,
			(int)Tk, key_padding_mask, causal, scale);
	}
	NNB_CUDA_TRY(cudaGetLastError());
	// O_h = P V_h  (ops.cpp:1259)
	return nnb::gemm_run(s, nnb::head_gemm(0, 0, Tq, Dh, Tk, probs, Tk, H * ps, ps, v, D, ks, Dh, out, D, qs, Dh, N, H,
		0));
}

nnb_status nnb_attention_bwd(void* stream, size_t N, size_t Tq, size_t Tk, size_t D, size_t heads, const float* g,
		const float* q, const float* k, const float* v, const float* probs, const float* key_padding_mask, int causal,
		float* dq, int dq_first, float* dk, int dk_first, float* dv, int dv_first) {
	NNB_TRY(nnb::check_shapes(N, Tq, Tk, D, heads, causal));
	if (N == 0) return NNB_OK;
	if (!g || !q || !k || !v || !probs) return nnb::fail(NNB_ERR_INVALID, "attention_bwd: null input");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long H = (long long)heads, Dh = (long long)(D / heads);
	const long long qs = (long long)Tq * D, ks = (long long)Tk * D, ps = (long long)Tq * Tk;
	const float scale = 1.0f / std::sqrt(static_cast<float>(Dh));
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, (size_t)N * H * ps * sizeof(float), s));
	float* ds = static_cast<float*>(ws);
	nnb_status st = NNB_OK;
	do {
		// dP = G V_h^T  (ops.cpp:1286)
		if ((st = nnb::gemm_run(s, nnb::head_gemm(0, 1, Tq, Tk, Dh, g, D, qs, Dh, v, D, ks, Dh, ds, Tk, H * ps, ps, N, H,
				0))) != NNB_OK) break;
		// dV (+)= P^T G  (ops.cpp:1287)
		if (dv && (st = nnb::gemm_run(s, nnb::head_gemm(1, 0, Tk, Dh, Tq, probs, Tk, H * ps, ps, g, D, qs, Dh, dv, D, ks,
				Dh, N, H, !dv_first))) != NNB_OK) break;
		if (!dq && !dk) break;
		const long long rows = (long long)N * H * Tq;
		{
			nnb::TraceScope ts(s, nnb::kTraceAttention);
			nnb::masked_softmax_bwd_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(probs, ds, rows, (int)H,
				(int)Tq, (int)Tk, key_padding_mask, causal, scale);
		}
		if ((st = nnb::cuda_status(cudaGetLastError(), "softmax backward launch")) != NNB_OK) break;
		// dQ (+)= dS K_h  (ops.cpp:1290)
		if (dq && (st = nnb::gemm_run(s, nnb::head_gemm(0, 0, Tq, Dh, Tk, ds, Tk, H * ps, ps, k, D, ks, Dh, dq, D, qs, Dh,
				N, H, !dq_first))) != NNB_OK) break;
		// dK (+)= dS^T Q_h  (ops.cpp:1291)
		if (dk && (st = nnb::gemm_run(s, nnb::head_gemm(1, 0, Tk, Dh, Tq, ds, Tk, H * ps, ps, q, D, qs, Dh, dk, D, ks, Dh,
				N, H, !dk_first))) != NNB_OK) break;
	} while (0);
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

// Dropout on the attention weights (attention.cpp:36-47): the same head-batched products around
// the masked softmax, with W = P * m between them; m comes from a keep mask drawn beforehand
// (nnb_dropout_mask over the N*H*Tq*Tk weights in row-major order, as Dropout::forward draws).
nnb_status nnb_attention_dropout_fwd(void* stream, size_t N, size_t Tq, size_t Tk, size_t D, size_t heads,
		const float* q, const float* k, const float* v, const float* key_padding_mask, int causal, float p,
		const uint32_t* keep, float* out, float* probs, float* weights) {
	NNB_TRY(nnb::check_shapes(N, Tq, Tk, D, heads, causal));
	if (!(p >= 0.0f && p <= 1.0f)) return nnb::fail(NNB_ERR_INVALID, "attention_dropout_fwd: p must be in [0, 1]");
	if (N == 0) return NNB_OK;
	if (!q || !k || !v || !keep || !out || !probs || !weights)
		return nnb::fail(NNB_ERR_INVALID, "attention_dropout_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long H = (long long)heads, Dh = (long long)(D / heads);
	const long long qs = (long long)Tq * D, ks = (long long)Tk * D, ps = (long long)Tq * Tk;
	const float scale = 1.0f / std::sqrt(static_cast<float>(Dh));     // attention.cpp:44
	// scores = q k^T  (matmul_bt, attention.cpp:43)
	NNB_TRY(nnb::gemm_run(s, nnb::head_gemm(0, 1, Tq, Tk, Dh, q, D, qs, Dh, k, D, ks, Dh, probs, Tk, H * ps, ps,
		N, H, 0)));
	const long long rows = (long long)N * H * Tq;
	{
		nnb::TraceScope ts(s, nnb::kTraceAttention);
		nnb::masked_softmax_fwd_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(probs, rows, (int)H, (int)Tq,
			(int)Tk, key_padding_mask, causal, scale, keep, nnb::dropout_keep_scale(p), weights);
	}
	NNB_CUDA_TRY(cudaGetLastError());
	// merged = W v  (matmul, attention.cpp:46), written in place of the head transpose
	return nnb::gemm_run(s, nnb::head_gemm(0, 0, Tq, Dh, Tk, weights, Tk, H * ps, ps, v, D, ks, Dh, out, D, qs, Dh, N,
		H, 0));
}

nnb_status nnb_attention_dropout_bwd(void* stream, size_t N, size_t Tq, size_t Tk, size_t D, size_t heads,
		const float* g, const float* q, const float* k, const float* v, const float* probs, const float* weights,
		float p, const uint32_t* keep, const float* key_padding_mask, int causal, float* dq, int dq_first, float* dk,
		int dk_first, float* dv, int dv_first) {
	NNB_TRY(nnb::check_shapes(N, Tq, Tk, D, heads, causal));
	if (!(p >= 0.0f && p <= 1.0f)) return nnb::fail(NNB_ERR_INVALID, "attention_dropout_bwd: p must be in [0, 1]");
	if (N == 0) return NNB_OK;
	if (!g || !q || !k || !v || !probs || !weights || !keep)
		return nnb::fail(NNB_ERR_INVALID, "attention_dropout_bwd: null input");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long H = (long long)heads, Dh = (long long)(D / heads);
	const long long qs = (long long)Tq * D, ks = (long long)Tk * D, ps = (long long)Tq * Tk;
	const float scale = 1.0f / std::sqrt(static_cast<float>(Dh));
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, (size_t)N * H * ps * sizeof(float), s));
	float* ds = static_cast<float*>(ws);
	nnb_status st = NNB_OK;
	do {
		// dW = G v^T, dv (+)= W^T G  (matmul's backward)
		if ((st = nnb::gemm_run(s, nnb::head_gemm(0, 1, Tq, Tk, Dh, g, D, qs, Dh, v, D, ks, Dh, ds, Tk, H * ps, ps, N, H,
				0))) != NNB_OK) break;
		if (dv && (st = nnb::gemm_run(s, nnb::head_gemm(1, 0, Tk, Dh, Tq, weights, Tk, H * ps, ps, g, D, qs, Dh, dv, D,
				ks, Dh, N, H, !dv_first))) != NNB_OK) break;
		if (!dq && !dk) break;
		// dP = dW * m, then the masked softmax's backward, in one pass per row
		const long long rows = (long long)N * H * Tq;
		{
			nnb::TraceScope ts(s, nnb::kTraceAttention);
			nnb::masked_softmax_bwd_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(probs, ds, rows, (int)H,
				(int)Tq, (int)Tk, key_padding_mask, causal, scale, keep, nnb::dropout_keep_scale(p));
		}
		if ((st = nnb::cuda_status(cudaGetLastError(), "softmax backward launch")) != NNB_OK) break;
		// dq (+)= dS k, dk (+)= dS^T q  (matmul_bt's backward)
		if (dq && (st = nnb::gemm_run(s, nnb::head_gemm(0, 0, Tq, Dh, Tk, ds, Tk, H * ps, ps, k, D, ks, Dh, dq, D, qs, Dh,
				N, H, !dq_first))) != NNB_OK) break;
		if (dk && (st = nnb::gemm_run(s, nnb::head_gemm(1, 0, Tk, Dh, Tq, ds, Tk, H * ps, ps, q, D, qs, Dh, dk, D, ks, Dh,
				N, H, !dk_first))) != NNB_OK) break;
	} while (0);
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

nnb_status nnb_masked_softmax_fwd(void* stream, size_t N, size_t H, size_t Tq, size_t Tk, float* scores,
		const float* key_padding_mask, int causal, float scale) {
	if (Tk == 0) return nnb::fail(NNB_ERR_SHAPE, "masked_softmax: empty rows");
	if (causal && Tq != Tk) return nnb::fail(NNB_ERR_SHAPE, "masked_softmax: causal needs Tq == Tk");
	const long long rows = (long long)N * H * Tq;
	if (rows == 0) return NNB_OK;
	if (!scores) return nnb::fail(NNB_ERR_INVALID, "masked_softmax_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	nnb::TraceScope ts(s, nnb::kTraceAttention);
	nnb::masked_softmax_fwd_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(scores, rows, (int)H, (int)Tq,
		(int)Tk, key_padding_mask, causal, scale);
	return nnb::cuda_status(cudaGetLastError(), "masked_softmax_fwd launch");
}

nnb_status nnb_masked_softmax_bwd(void* stream, size_t N, size_t H, size_t Tq, size_t Tk, const float* probs,
		float* grad, const float* key_padding_mask, int causal, float scale) {
	if (Tk == 0) return nnb::fail(NNB_ERR_SHAPE, "masked_softmax: empty rows");
	const long long rows = (long long)N * H * Tq;
	if (rows == 0) return NNB_OK;
	if (!probs || !grad) return nnb::fail(NNB_ERR_INVALID, "masked_softmax_bwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	nnb::TraceScope ts(s, nnb::kTraceAttention);
	nnb::masked_softmax_bwd_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(probs, grad, rows, (int)H, (int)Tq,
		(int)Tk, key_padding_mask, causal, scale);
	return nnb::cuda_status(cudaGetLastError(), "masked_softmax_bwd launch");
}

nnb_status nnb_scaled_masked_softmax_fwd(void* stream, size_t N, size_t H, size_t Tq, size_t Tk, const float* x,
		float* y, const float* key_padding_mask, int causal, float scale) {
	if (Tk == 0) return nnb::fail(NNB_ERR_SHAPE, "scaled_masked_softmax: empty rows");
	const long long rows = (long long)N * H * Tq;
	if (rows == 0) return NNB_OK;
	if (!x || !y) return nnb::fail(NNB_ERR_INVALID, "scaled_masked_softmax_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	nnb::TraceScope ts(s, nnb::kTraceAttention);
	nnb::softmax_rows_fwd_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(x, y, rows, (int)H, (int)Tq,
		(int)Tk, key_padding_mask, causal, scale);
	return nnb::cuda_status(cudaGetLastError(), "scaled_masked_softmax_fwd launch");
}

nnb_status nnb_scaled_masked_softmax_bwd(void* stream, size_t N, size_t H, size_t Tq, size_t Tk, const float* y,
		const float* g, float* dx, int dx_first, const float* key_padding_mask, int causal, float scale) {
	if (Tk == 0) return nnb::fail(NNB_ERR_SHAPE, "scaled_masked_softmax: empty rows");
	const long long rows = (long long)N * H * Tq;
	if (rows == 0) return NNB_OK;
	if (!y || !g || !dx) return nnb::fail(NNB_ERR_INVALID, "scaled_masked_softmax_bwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	nnb::TraceScope ts(s, nnb::kTraceAttention);
	nnb::softmax_rows_bwd_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, s>>>(y, g, dx, dx_first, rows, (int)H,
		(int)Tq, (int)Tk, key_padding_mask, causal, scale);
	return nnb::cuda_status(cudaGetLastError(), "scaled_masked_softmax_bwd launch");
}

}  // extern "C"
