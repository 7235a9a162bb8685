// host_gemm.cu -- nn::kernels::sgemm (include/nn/kernels/gemm.hpp:57-59) on HOST buffers: the literal
// drop-in for the reference's kernel, which takes host pointers and returns with C written.
//
// The product is pipelined over three streams so the PCIe copies overlap the tensor cores:
//   copy stream    B (all of it: every band needs it), then A in row bands of op(A) (and, when
//                  accumulating, the matching bands of C);
//   compute stream waits for B and for band i, runs the device GEMM on band i;
//   out stream     waits for band i's GEMM and copies band i of C back to the host.
// Bands are whole 128-row tiles of C, so each band's tile sequence and k order are those of the full
// product: the result is bitwise the one nnb_sgemm gives on device copies of the same operands (and,
// as there, independent of the band count). Strided host layouts are moved with 2-D copies. The host
// buffers should be page-locked for full copy speed; pageable memory works, at the copy engine's
// pageable rate. Device buffers and streams are kept per device and grown on demand; consecutive
// calls are chained, so a call never overwrites buffers the previous one still reads. The stream-
// ordered form starts after the caller's stream reaches it and makes that stream wait for the last
// copy-back, so CUDA events on the caller's stream time the whole call.
#include <mutex>
#include <vector>

#include "nnb_gemm.h"
#include "nnb_internal.h"

namespace nnb {

namespace {

struct HostGemmCtx {
	bool ready = false;
	cudaStream_t copy = nullptr, compute = nullptr, out = nullptr;
	cudaEvent_t b_done = nullptr, start = nullptr, done = nullptr;
	bool has_prev = false;                       // `done` marks the previous call's last copy-back
	std::vector<cudaEvent_t> a_done, c_done;
	float *da = nullptr, *db = nullptr, *dc = nullptr;
	size_t cap_a = 0, cap_b = 0, cap_c = 0;
};

constexpr int kMaxDev = 64;
HostGemmCtx g_ctx[kMaxDev];
std::mutex g_mu[kMaxDev];
constexpr int kMaxBands = 16;

nnb_status grow(float** p, size_t* cap, size_t floats) {
	if (floats <= *cap) return NNB_OK;
	if (*p) NNB_CUDA_TRY(cudaFree(*p));
	*p = nullptr;
	*cap = 0;
	NNB_CUDA_TRY(cudaMalloc(p, floats * sizeof(float)));
	*cap = floats;
	return NNB_OK;
}

nnb_status ctx_setup(HostGemmCtx& c) {
	if (c.ready) return NNB_OK;
	NNB_CUDA_TRY(cudaStreamCreateWithFlags(&c.copy, cudaStreamNonBlocking));
	NNB_CUDA_TRY(cudaStreamCreateWithFlags(&c.compute, cudaStreamNonBlocking));
	NNB_CUDA_TRY(cudaStreamCreateWithFlags(&c.out, cudaStreamNonBlocking));
	NNB_CUDA_TRY(cudaEventCreateWithFlags(&c.b_done, cudaEventDisableTiming));
	NNB_CUDA_TRY(cudaEventCreateWithFlags(&c.start, cudaEventDisableTiming));
	NNB_CUDA_TRY(cudaEventCreateWithFlags(&c.done, cudaEventDisableTiming));
	c.a_done.resize(kMaxBands);
	c.c_done.resize(kMaxBands);
	for (int i = 0; i < kMaxBands; ++i) {
		NNB_CUDA_TRY(cudaEventCreateWithFlags(&c.a_done[i], cudaEventDisableTiming));
		NNB_CUDA_TRY(cudaEventCreateWithFlags(&c.c_done[i], cudaEventDisableTiming));
	}
	c.ready = true;
	return NNB_OK;
}

// rows x cols floats with host leading dimension ld <-> a dense device block (row pitch cols)
nnb_status h2d(float* dst, const float* src, size_t rows, size_t cols, size_t ld, cudaStream_t s) {
	if (rows == 0 || cols == 0) return NNB_OK;
	NNB_CUDA_TRY(cudaMemcpy2DAsync(dst, cols * sizeof(float), src, ld * sizeof(float), cols * sizeof(float), rows,
		cudaMemcpyHostToDevice, s));
	return NNB_OK;
}

nnb_status d2h(float* dst, size_t ld, const float* src, size_t rows, size_t cols, cudaStream_t s) {
	if (rows == 0 || cols == 0) return NNB_OK;
	NNB_CUDA_TRY(cudaMemcpy2DAsync(dst, ld * sizeof(float), src, cols * sizeof(float), cols * sizeof(float), rows,
		cudaMemcpyDeviceToHost, s));
	return NNB_OK;
}

}  // namespace

nnb_status sgemm_host(cudaStream_t caller, bool blocking, int ta, int tb, size_t m, size_t n, size_t k, const float* a,
		size_t lda, const float* b, size_t ldb, float* c, size_t ldc, int accumulate, int mode) {
	if (m == 0 || n == 0) return NNB_OK;
	if (!c || (k > 0 && (!a || !b))) return fail(NNB_ERR_INVALID, "sgemm_host: null pointer");
	if (ldc < n || (k > 0 && (lda < (ta ? m : k) || ldb < (tb ? k : n))))
		return fail(NNB_ERR_INVALID, "sgemm_host: leading dimension too small");
	DeviceState* dev = nullptr;
	NNB_TRY(device_state(&dev));
	const int di = dev->device & (kMaxDev - 1);
	std::lock_guard<std::mutex> lock(g_mu[di]);
	HostGemmCtx& x = g_ctx[di];
	NNB_TRY(ctx_setup(x));
	// ordered after the caller's stream and after the previous call (whose buffers are reused)
	NNB_CUDA_TRY(cudaEventRecord(x.start, caller));
	for (cudaStream_t st : {x.copy, x.compute, x.out}) {
		NNB_CUDA_TRY(cudaStreamWaitEvent(st, x.start, 0));
		if (x.has_prev) NNB_CUDA_TRY(cudaStreamWaitEvent(st, x.done, 0));
	}
	// op(A) band r0..r1 on the device: rows of A (ta = 0, dense band x k) or columns of A (ta = 1,
	// dense k x band); B dense as stored (k x n or n x k); C dense m x n
	NNB_TRY(grow(&x.da, &x.cap_a, m * k));
	NNB_TRY(grow(&x.db, &x.cap_b, k * n));
	NNB_TRY(grow(&x.dc, &x.cap_c, m * n));
	// band height: about two waves of 128 x 256 tiles on the SMs (an 8192-wide C: 9 row tiles, 288
	// tiles, 97 % of two waves), at most kMaxBands bands
	const size_t tiles = (m + 127) / 128, tiles_n = (n + 255) / 256;
	size_t per_tiles = std::max<size_t>(1, (size_t)(2 * dev->sm_count) / tiles_n);
	per_tiles = std::max(per_tiles, (tiles + kMaxBands - 1) / kMaxBands);
	const size_t per = per_tiles * 128;                                         // rows per band, whole tiles
	if (k > 0) {
		if (tb) NNB_TRY(h2d(x.db, b, n, k, ldb, x.copy));
		else NNB_TRY(h2d(x.db, b, k, n, ldb, x.copy));
	}
	NNB_CUDA_TRY(cudaEventRecord(x.b_done, x.copy));
	NNB_CUDA_TRY(cudaStreamWaitEvent(x.compute, x.b_done, 0));
	size_t band = 0;
	for (size_t r0 = 0; r0 < m; r0 += per, ++band) {
		const size_t rows = std::min(per, m - r0);
		float* da = x.da + r0 * k;                                            // band blocks, one after another
		float* dc = x.dc + r0 * n;
		if (k > 0) {
			if (ta) NNB_TRY(h2d(da, a + r0, k, rows, lda, x.copy));            // k x rows slice of the k x m storage
			else NNB_TRY(h2d(da, a + r0 * lda, rows, k, lda, x.copy));
		}
		if (accumulate) NNB_TRY(h2d(dc, c + r0 * ldc, rows, n, ldc, x.copy));
		NNB_CUDA_TRY(cudaEventRecord(x.a_done[band], x.copy));
		NNB_CUDA_TRY(cudaStreamWaitEvent(x.compute, x.a_done[band], 0));
		GemmDesc d;
		d.ta = ta; d.tb = tb; d.m = (long long)rows; d.n = (long long)n; d.k = (long long)k;
		d.a = da; d.lda = ta ? (long long)rows : (long long)k;
		d.b = x.db; d.ldb = tb ? (long long)k : (long long)n;
		d.c = dc; d.ldc = (long long)n; d.accumulate = accumulate != 0; d.mode = mode;
		NNB_TRY(gemm_run(x.compute, d));
		NNB_CUDA_TRY(cudaEventRecord(x.c_done[band], x.compute));
		NNB_CUDA_TRY(cudaStreamWaitEvent(x.out, x.c_done[band], 0));
		NNB_TRY(d2h(c + r0 * ldc, ldc, dc, rows, n, x.out));
	}
	// the out stream has waited for every GEMM, and every GEMM for its copies: its end is the call's end
	NNB_CUDA_TRY(cudaEventRecord(x.done, x.out));
	x.has_prev = true;
	NNB_CUDA_TRY(cudaStreamWaitEvent(caller, x.done, 0));
	if (blocking) NNB_CUDA_TRY(cudaStreamSynchronize(caller));
	return NNB_OK;
}

}  // namespace nnb

extern "C" {

nnb_status nnb_sgemm_host(int trans_a, int trans_b, size_t m, size_t n, size_t k, const float* a, size_t lda,
		const float* b, size_t ldb, float* c, size_t ldc, int accumulate) {
	return nnb::sgemm_host(nullptr, true, trans_a != 0, trans_b != 0, m, n, k, a, lda, b, ldb, c, ldc, accumulate,
		nnb::math_mode());
}

nnb_status nnb_sgemm_host_async(void* stream, int trans_a, int trans_b, size_t m, size_t n, size_t k, const float* a,
		size_t lda, const float* b, size_t ldb, float* c, size_t ldc, int accumulate, int math_mode) {
	if (math_mode != NNB_MATH_FP32X3 && math_mode != NNB_MATH_TF32)
		return nnb::fail(NNB_ERR_INVALID, "sgemm_host: unknown math mode %d", math_mode);
	return nnb::sgemm_host(static_cast<cudaStream_t>(stream), false, trans_a != 0, trans_b != 0, m, n, k, a, lda, b, ldb,
		c, ldc, accumulate, math_mode);
}

}  // extern "C"
