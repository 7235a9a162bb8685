// host_gemm.cu -- nn::kernels::sgemm (include/nn/kernels/gemm.hpp:57-59) on HOST buffers: the literal
// drop-in for the reference's kernel, which takes host pointers and returns with C written.
//
// The product is pipelined over four streams so the PCIe copies overlap the tensor cores:
//   copy stream      B (all of it: every band needs it), then A in row bands of op(A) (and, when
//                    accumulating, the matching bands of C);
//   compute streams  B packed once into the GEMM's panel layout as soon as it has arrived, then the
//                    device GEMM of band i on stream i % 2 once band i has arrived: a band's kernel
//                    starts on the SMs the previous band's last wave leaves idle;
//   out stream       waits for band i's GEMM and copies band i of C back to the host.
// Bands are about one wave of tiles high, and the last wave's worth is cut into halves, quarters, ...
// down to one row of tiles, with the narrower tile width when the packed B allows it: the last band
// -- computed and copied back after the last byte of A has arrived -- is short. Bands are whole
// 128-row tiles of C and each element is one k-ordered chain, so the result is bitwise the one
// nnb_sgemm gives on device copies of the same operands (and, as there, independent of the band
// count and tile width). When the product's depth is cut into pieces (a deep k next to a narrow n),
// every band packs its own B as nnb_sgemm does. Strided host layouts are moved with 2-D copies.
// The host buffers should be page-locked for full copy speed; pageable memory works, at the copy
// engine's pageable rate. Device buffers and streams are kept per device and grown on demand
// (nnb_sgemm_host_release frees the buffers); consecutive calls are chained, so a call never
// overwrites buffers the previous one still reads. The stream-ordered form starts after the
// caller's stream reaches it and makes that stream wait for the last copy-back, so CUDA events on the
// caller's stream time the whole call.
#include <mutex>
#include <vector>

#include "nnb_gemm.h"
#include "nnb_internal.h"

namespace nnb {

namespace {

struct HostGemmCtx {
	bool ready = false;
	int device = -1;
	cudaStream_t copy = nullptr, compute[2] = {nullptr, nullptr}, out = nullptr;
	cudaEvent_t b_done = nullptr, b_packed = nullptr, start = nullptr, done = nullptr;
	bool has_prev = false;                       // `done` marks the previous call's last copy-back
	std::vector<cudaEvent_t> a_done, c_done;
	float *da = nullptr, *db = nullptr, *dc = nullptr, *pb = nullptr;
	size_t cap_a = 0, cap_b = 0, cap_c = 0, cap_pb = 0;
};

constexpr int kMaxDev = 64;
HostGemmCtx g_ctx[kMaxDev];
std::mutex g_mu[kMaxDev];
constexpr size_t kMaxBands = 32;                 // full-height bands; the halved tail adds a few

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
	NNB_CUDA_TRY(cudaStreamCreateWithFlags(&c.compute[0], cudaStreamNonBlocking));
	NNB_CUDA_TRY(cudaStreamCreateWithFlags(&c.compute[1], cudaStreamNonBlocking));
	NNB_CUDA_TRY(cudaStreamCreateWithFlags(&c.out, cudaStreamNonBlocking));
	NNB_CUDA_TRY(cudaEventCreateWithFlags(&c.b_done, cudaEventDisableTiming));
	NNB_CUDA_TRY(cudaEventCreateWithFlags(&c.b_packed, cudaEventDisableTiming));
	NNB_CUDA_TRY(cudaEventCreateWithFlags(&c.start, cudaEventDisableTiming));
	NNB_CUDA_TRY(cudaEventCreateWithFlags(&c.done, cudaEventDisableTiming));
	c.ready = true;
	return NNB_OK;
}

// Waits for the context's streams and frees its device buffers (streams and events are kept).
nnb_status release_buffers(HostGemmCtx& c) {
	if (!c.ready) return NNB_OK;
	int prev = 0;
	NNB_CUDA_TRY(cudaGetDevice(&prev));
	NNB_CUDA_TRY(cudaSetDevice(c.device));
	nnb_status st = NNB_OK;
	for (cudaStream_t s : {c.copy, c.compute[0], c.compute[1], c.out})
		if (st == NNB_OK) st = cuda_status(cudaStreamSynchronize(s), "sgemm_host_release");
	for (float** p : {&c.da, &c.db, &c.dc, &c.pb}) {
		if (*p && st == NNB_OK) st = cuda_status(cudaFree(*p), "sgemm_host_release");
		if (st == NNB_OK) *p = nullptr;
	}
	if (st == NNB_OK) c.cap_a = c.cap_b = c.cap_c = c.cap_pb = 0;
	const nnb_status st2 = cuda_status(cudaSetDevice(prev), "sgemm_host_release");
	return st != NNB_OK ? st : st2;
}

nnb_status ensure_events(HostGemmCtx& c, size_t count) {
	while (c.a_done.size() < count) {
		cudaEvent_t ea = nullptr, ec = nullptr;
		NNB_CUDA_TRY(cudaEventCreateWithFlags(&ea, cudaEventDisableTiming));
		c.a_done.push_back(ea);
		NNB_CUDA_TRY(cudaEventCreateWithFlags(&ec, cudaEventDisableTiming));
		c.c_done.push_back(ec);
	}
	return NNB_OK;
}

// Row tiles per band: `per` while more than `per` remain, then halves of what is left down to 1
// (per 4: ..., 4, 4, 2, 1, 1).
std::vector<size_t> band_tiles(size_t tiles, size_t per) {
	std::vector<size_t> out;
	size_t left = tiles;
	while (left > per) { out.push_back(per); left -= per; }
	while (left > 1) { const size_t t = (left + 1) / 2; out.push_back(t); left -= t; }
	if (left) out.push_back(left);
	return out;
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

// The enqueued part of one call: copies, packs and band GEMMs over the context's streams.
nnb_status enqueue(HostGemmCtx& x, const DeviceState* dev, int ta, int tb, size_t m, size_t n, size_t k,
		const float* a, size_t lda, const float* b, size_t ldb, float* c, size_t ldc, int accumulate, int mode) {
	// op(A) band r0..r1 on the device: rows of A (ta = 0, dense band x k) or columns of A (ta = 1,
	// dense k x band); B dense as stored (k x n or n x k); C dense m x n
	NNB_TRY(grow(&x.da, &x.cap_a, m * k));
	NNB_TRY(grow(&x.db, &x.cap_b, k * n));
	NNB_TRY(grow(&x.dc, &x.cap_c, m * n));
	// band height: about one wave of 128 x 256 tiles on the SMs (an 8192-wide C: 4 row tiles, 128
	// tiles), at most kMaxBands full-height bands
	const size_t tiles = (m + 127) / 128, tiles_n = (n + 255) / 256;
	size_t per_tiles = std::max<size_t>(1, (size_t)dev->sm_count / tiles_n);
	per_tiles = std::max(per_tiles, (tiles + kMaxBands - 1) / kMaxBands);
	const size_t per = per_tiles * 128;                                         // rows per band, whole tiles
	const std::vector<size_t> plan = band_tiles(tiles, per_tiles);
	NNB_TRY(ensure_events(x, plan.size()));
	GemmDesc whole;                                                               // the band-independent part
	whole.ta = ta; whole.tb = tb; whole.n = (long long)n; whole.k = (long long)k;
	whole.b = x.db; whole.ldb = tb ? (long long)k : (long long)n;
	whole.ldc = (long long)n; whole.accumulate = accumulate != 0; whole.mode = mode;
	if (k > 0) {
		if (tb) NNB_TRY(h2d(x.db, b, n, k, ldb, x.copy));
		else NNB_TRY(h2d(x.db, b, k, n, ldb, x.copy));
	}
	NNB_CUDA_TRY(cudaEventRecord(x.b_done, x.copy));
	NNB_CUDA_TRY(cudaStreamWaitEvent(x.compute[0], x.b_done, 0));
	// B packed once for every band, unless the depth cut packs per piece
	GemmDesc shape = whole;
	shape.m = (long long)std::min(per, m);
	shape.a = x.da; shape.lda = ta ? shape.m : (long long)k; shape.c = x.dc;
	const bool pre = k > 0 && gemm_depth_pieces(whole) == 1;
	const int bn = pre ? gemm_tile_width(shape, dev->sm_count) : 0;
	if (pre) {
		const size_t bytes = gemm_packed_b_bytes(shape, bn);
		if (bytes == 0) return fail(NNB_ERR_UNSUPPORTED, "sgemm_host: B too large to pack");
		NNB_TRY(grow(&x.pb, &x.cap_pb, (bytes + sizeof(float) - 1) / sizeof(float)));
		NNB_TRY(gemm_pack_b(x.compute[0], shape, bn, x.pb));
		NNB_CUDA_TRY(cudaEventRecord(x.b_packed, x.compute[0]));
		NNB_CUDA_TRY(cudaStreamWaitEvent(x.compute[1], x.b_packed, 0));
	} else {
		NNB_CUDA_TRY(cudaStreamWaitEvent(x.compute[1], x.b_done, 0));
	}
	size_t r0 = 0;
	for (size_t band = 0; band < plan.size(); r0 += plan[band] * 128, ++band) {
		const size_t rows = std::min(plan[band] * 128, m - r0);
		float* da = x.da + r0 * k;                                            // band blocks, one after another
		float* dc = x.dc + r0 * n;
		if (k > 0) {
			if (ta) NNB_TRY(h2d(da, a + r0, k, rows, lda, x.copy));            // k x rows slice of the k x m storage
			else NNB_TRY(h2d(da, a + r0 * lda, rows, k, lda, x.copy));
		}
		if (accumulate) NNB_TRY(h2d(dc, c + r0 * ldc, rows, n, ldc, x.copy));
		NNB_CUDA_TRY(cudaEventRecord(x.a_done[band], x.copy));
		cudaStream_t cs = x.compute[band & 1];
		NNB_CUDA_TRY(cudaStreamWaitEvent(cs, x.a_done[band], 0));
		GemmDesc d = whole;
		d.m = (long long)rows;
		d.a = da; d.lda = ta ? (long long)rows : (long long)k;
		d.c = dc;
		if (pre) {
			// a short band may go from 256 to 128, which reads the same 128-row panels of B over the
			// same padded width; every other band keeps the width B was packed for
			int w = gemm_tile_width(d, dev->sm_count);
			if (!(bn == 256 && w < bn && (n + 127) / 128 * 128 == (n + 255) / 256 * 256)) w = bn;
			else w = 128;
			d.packed_b = x.pb;
			d.bn = w;
		}
		NNB_TRY(gemm_run(cs, d));
		NNB_CUDA_TRY(cudaEventRecord(x.c_done[band], cs));
		NNB_CUDA_TRY(cudaStreamWaitEvent(x.out, x.c_done[band], 0));
		NNB_TRY(d2h(c + r0 * ldc, ldc, dc, rows, n, x.out));
	}
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
	x.device = dev->device;
	// ordered after the caller's stream and after the previous call (whose buffers are reused)
	NNB_CUDA_TRY(cudaEventRecord(x.start, caller));
	for (cudaStream_t st : {x.copy, x.compute[0], x.compute[1], x.out}) {
		NNB_CUDA_TRY(cudaStreamWaitEvent(st, x.start, 0));
		if (x.has_prev) NNB_CUDA_TRY(cudaStreamWaitEvent(st, x.done, 0));
	}
	const nnb_status st = enqueue(x, dev, ta, tb, m, n, k, a, lda, b, ldb, c, ldc, accumulate, mode);
	// the call ends when all four streams have: joined on the out stream even when enqueueing failed
	// part-way, so the next call never reuses buffers that work enqueued here still reads or writes
	for (cudaStream_t s : {x.copy, x.compute[0], x.compute[1]}) {
		NNB_CUDA_TRY(cudaEventRecord(x.start, s));
		NNB_CUDA_TRY(cudaStreamWaitEvent(x.out, x.start, 0));
	}
	NNB_CUDA_TRY(cudaEventRecord(x.done, x.out));
	x.has_prev = true;
	NNB_CUDA_TRY(cudaStreamWaitEvent(caller, x.done, 0));
	if (st != NNB_OK) return st;
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

nnb_status nnb_sgemm_host_release(void) {
	for (int i = 0; i < nnb::kMaxDev; ++i) {
		std::lock_guard<std::mutex> lock(nnb::g_mu[i]);
		NNB_TRY(nnb::release_buffers(nnb::g_ctx[i]));
	}
	return NNB_OK;
}

nnb_status nnb_sgemm_host_async(void* stream, int trans_a, int trans_b, size_t m, size_t n, size_t k, const float* a,
		size_t lda, const float* b, size_t ldb, float* c, size_t ldc, int accumulate, int math_mode) {
	if (math_mode != NNB_MATH_FP32X3 && math_mode != NNB_MATH_TF32)
		return nnb::fail(NNB_ERR_INVALID, "sgemm_host: unknown math mode %d", math_mode);
	return nnb::sgemm_host(static_cast<cudaStream_t>(stream), false, trans_a != 0, trans_b != 0, m, n, k, a, lda, b, ldb,
		c, ldc, accumulate, math_mode);
}

}  // extern "C"
