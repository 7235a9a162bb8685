// matmul.cu -- nn::matmul(a, b, trans_a, trans_b) (src/tensor.cpp:571-641) on dense row-major
// device tensors.
//
// The reference's two paths are kept: a batched left operand times a plain matrix is folded into
// ONE GEMM over all its rows (tensor.cpp:589-596); otherwise the batch axes broadcast
// numpy-style (tensor.cpp:121-136) and every output matrix is one product. Where the reference
// spreads those products over its thread pool, here the last two batch axes become the
// two-level batch of a single tensor-core launch (a broadcast axis has stride 0); only batch
// ranks above two loop on the host over the leading axes.
#include <vector>

#include "nnb_gemm.h"
#include "nnb_internal.h"

namespace nnb {
namespace {

constexpr int kMaxRank = 16;

nnb_status broadcast_batch(const std::vector<long long>& a, const std::vector<long long>& b, std::vector<long long>& out) {
	const size_t rank = std::max(a.size(), b.size());
	out.assign(rank, 1);
	for (size_t i = 0; i < rank; ++i) {
		const long long ad = i < rank - a.size() ? 1 : a[i - (rank - a.size())];
		const long long bd = i < rank - b.size() ? 1 : b[i - (rank - b.size())];
		if (ad == bd || bd == 1) out[i] = ad;
		else if (ad == 1) out[i] = bd;
		else return fail(NNB_ERR_SHAPE, "matmul: batch axes %lld and %lld do not broadcast", ad, bd);
	}
	return NNB_OK;
}

// Element stride of each batch axis of `shape` aligned to the broadcast rank (0 where broadcast).
std::vector<long long> batch_strides(const std::vector<long long>& shape, size_t rank, long long matrix) {
	std::vector<long long> st(rank, 0);
	long long s = matrix;
	for (size_t i = 0; i < shape.size(); ++i) {
		const size_t d = shape.size() - 1 - i;      // from the innermost batch axis outwards
		const size_t o = rank - 1 - i;
		st[o] = shape[d] == 1 ? 0 : s;
		s *= shape[d];
	}
	return st;
}

}  // namespace
}  // namespace nnb

extern "C" nnb_status nnb_matmul(void* stream, const float* a, const int64_t* a_shape, int a_ndim, const float* b,
		const int64_t* b_shape, int b_ndim, int trans_a, int trans_b, float* c, int64_t* out_shape, int* out_ndim) {
	using namespace nnb;
	if (a_ndim < 2 || b_ndim < 2) return fail(NNB_ERR_SHAPE, "matmul: operands need two or more axes");
	if (a_ndim > kMaxRank || b_ndim > kMaxRank) return fail(NNB_ERR_UNSUPPORTED, "matmul: rank above %d", kMaxRank);
	if (!a_shape || !b_shape || !out_ndim) return fail(NNB_ERR_INVALID, "matmul: null shape pointer");
	const long long a_rows = a_shape[a_ndim - 2], a_cols = a_shape[a_ndim - 1];
	const long long b_rows = b_shape[b_ndim - 2], b_cols = b_shape[b_ndim - 1];
	const long long m = trans_a ? a_cols : a_rows, k = trans_a ? a_rows : a_cols;
	const long long k2 = trans_b ? b_cols : b_rows, n = trans_b ? b_rows : b_cols;
	if (k != k2) return fail(NNB_ERR_SHAPE, "matmul: inner sizes %lld and %lld differ", k, k2);
	cudaStream_t s = static_cast<cudaStream_t>(stream);

	GemmDesc d;
	d.ta = trans_a != 0; d.tb = trans_b != 0;
	d.k = k; d.n = n;
	d.lda = a_cols; d.ldb = b_cols; d.ldc = n;
	d.a = a; d.b = b; d.c = c;
	d.mode = math_mode();

	// fold: batched a (not transposed) times a 2-D b (tensor.cpp:589-596)
	if (b_ndim == 2 && !trans_a && a_ndim > 2) {
		long long rows = 1;
		for (int i = 0; i < a_ndim - 1; ++i) rows *= a_shape[i];
		*out_ndim = a_ndim;
		if (out_shape) {
			for (int i = 0; i < a_ndim - 1; ++i) out_shape[i] = a_shape[i];
			out_shape[a_ndim - 1] = n;
		}
		if (!c) return NNB_OK;
		d.m = rows;
		return gemm_run(s, d);
	}

	std::vector<long long> ab(a_shape, a_shape + a_ndim - 2), bb(b_shape, b_shape + b_ndim - 2), batch;
	NNB_TRY(broadcast_batch(ab, bb, batch));
	const size_t R = batch.size();
	*out_ndim = (int)R + 2;
	if (out_shape) {
		for (size_t i = 0; i < R; ++i) out_shape[i] = batch[i];
		out_shape[R] = m;
		out_shape[R + 1] = n;
	}
	if (!c) return NNB_OK;
	d.m = m;
	if (R == 0) return gemm_run(s, d);
	const std::vector<long long> sa = batch_strides(ab, R, a_rows * a_cols);
	const std::vector<long long> sb = batch_strides(bb, R, b_rows * b_cols);
	std::vector<long long> sc(R);
	long long acc = m * n;
	for (size_t i = R; i-- > 0;) {
		sc[i] = acc;
		acc *= batch[i];
	}
	// the last batch axis is the inner level, the one before it the outer level
	d.batch_inner = batch[R - 1];
	d.sa_inner = sa[R - 1]; d.sb_inner = sb[R - 1]; d.sc_inner = sc[R - 1];
	if (R >= 2) {
		d.batch_outer = batch[R - 2];
		d.sa_outer = sa[R - 2]; d.sb_outer = sb[R - 2]; d.sc_outer = sc[R - 2];
	}
	long long lead = 1;
	for (size_t i = 0; i + 2 < R; ++i) lead *= batch[i];
	for (long long li = 0; li < lead; ++li) {
		long long rem = li, oa = 0, ob = 0, oc = 0;
		for (size_t i = R >= 2 ? R - 2 : 0; i-- > 0;) {     // the axes before the outer level
			const long long idx = rem % batch[i];
			rem /= batch[i];
			oa += idx * sa[i];
			ob += idx * sb[i];
			oc += idx * sc[i];
		}
		GemmDesc e = d;
		e.a = a + oa; e.b = b + ob; e.c = c + oc;
		NNB_TRY(gemm_run(s, e));
	}
	return NNB_OK;
}
