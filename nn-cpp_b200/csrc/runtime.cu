// runtime.cu -- library-wide state behind the C ABI: error text, math mode, per-device state,
// tensor-map encoding and stream-ordered scratch.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "nnb_internal.h"

namespace nnb {

namespace {

thread_local char g_last_error[512] = "";

std::atomic<int> g_math_mode{-1};

constexpr int kMaxDevices = 64;
DeviceState g_devices[kMaxDevices];
std::mutex g_device_mutex;

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

PFN_cuMemGetAddressRange_v3020 g_range = nullptr;
std::once_flag g_range_once;

}  // namespace

nnb_status fail(nnb_status st, const char* fmt, ...) {
	va_list ap;
	va_start(ap, fmt);
	vsnprintf(g_last_error, sizeof g_last_error, fmt, ap);
	va_end(ap);
	return st;
}

nnb_status cuda_status(cudaError_t e, const char* what) {
	if (e == cudaSuccess) return NNB_OK;
	return fail(NNB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int math_mode() {
	int m = g_math_mode.load(std::memory_order_relaxed);
	if (m >= 0) return m;
	m = NNB_MATH_FP32X3;
	if (const char* env = std::getenv("NNB_MATH")) {
		if (std::strcmp(env, "tf32") == 0) m = NNB_MATH_TF32;
	}
	int expected = -1;
	g_math_mode.compare_exchange_strong(expected, m);
	return g_math_mode.load();
}

nnb_status device_state(DeviceState** out) {
	int dev = 0;
	NNB_CUDA_TRY(cudaGetDevice(&dev));
	if (dev < 0 || dev >= kMaxDevices) return fail(NNB_ERR_UNSUPPORTED, "device index %d out of range", dev);
	DeviceState& st = g_devices[dev];
	if (st.ready) {
		*out = &st;
		return NNB_OK;
	}
	std::lock_guard<std::mutex> lock(g_device_mutex);
	if (!st.ready) {
		cudaDeviceProp prop;
		NNB_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
		if (prop.major != 10)
			return fail(NNB_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
				dev, prop.major, prop.minor);
		st.device = dev;
		st.sm_count = prop.multiProcessorCount;
		NNB_CUDA_TRY(cudaMalloc(&st.error_word, sizeof(int)));
		NNB_CUDA_TRY(cudaMemset(st.error_word, 0, sizeof(int)));
		// Keep freed scratch cached in the default pool instead of returning it to the driver
		cudaMemPool_t pool;
		NNB_CUDA_TRY(cudaDeviceGetDefaultMemPool(&pool, dev));
		uint64_t threshold = UINT64_MAX;
		NNB_CUDA_TRY(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold));
		st.ready = true;
	}
	*out = &st;
	return NNB_OK;
}

static nnb_status load_encode() {
	std::call_once(g_encode_once, [] {
		void* fn = nullptr;
		cudaDriverEntryPointQueryResult q;
		if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess
				&& q == cudaDriverEntryPointSuccess)
			g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
	});
	if (!g_encode) return fail(NNB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
	return NNB_OK;
}

nnb_status encode_tiled_nd(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
		const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle) {
	NNB_TRY(load_encode());
	if (rank < 2 || rank > 5) return fail(NNB_ERR_INVALID, "tensor map rank %d", rank);
	cuuint64_t d[5], st[4];
	cuuint32_t b[5], e[5];
	for (int i = 0; i < rank; ++i) {
		d[i] = dims[i];
		b[i] = box[i];
		e[i] = 1;
		if (i + 1 < rank) st[i] = strides[i];
	}
	CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<void*>(base), d, st, b, e,
		CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
	if (r != CUDA_SUCCESS)
		return fail(NNB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): rank %d, dims %llu x %llu", (int)r, rank,
			(unsigned long long)dims[0], (unsigned long long)dims[1]);
	return NNB_OK;
}

nnb_status encode_tiled_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
		uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
		CUtensorMapSwizzle swizzle) {
	NNB_TRY(load_encode());
	const cuuint64_t dims[2] = {inner, outer};
	const cuuint64_t strides[1] = {row_stride_bytes};
	const cuuint32_t box[2] = {box_inner, box_outer};
	const cuuint32_t estr[2] = {1, 1};
	CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims,
		strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
		CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
	if (r != CUDA_SUCCESS)
		return fail(NNB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): inner %llu outer %llu stride %llu",
			(int)r, (unsigned long long)inner, (unsigned long long)outer,
			(unsigned long long)row_stride_bytes);
	return NNB_OK;
}

nnb_status scratch_alloc(void** p, size_t bytes, cudaStream_t s) {
	*p = nullptr;
	if (bytes == 0) return NNB_OK;
	NNB_CUDA_TRY(cudaMallocAsync(p, bytes, s));
	return NNB_OK;
}

nnb_status scratch_free(void* p, cudaStream_t s) {
	if (!p) return NNB_OK;
	NNB_CUDA_TRY(cudaFreeAsync(p, s));
	return NNB_OK;
}

}  // namespace nnb

extern "C" {

const char* nnb_version(void) { return "0.1.0"; }

const char* nnb_last_error(void) { return nnb::g_last_error; }

nnb_status nnb_set_math_mode(int mode) {
	if (mode != NNB_MATH_FP32X3 && mode != NNB_MATH_TF32)
		return nnb::fail(NNB_ERR_INVALID, "unknown math mode %d", mode);
	nnb::g_math_mode.store(mode);
	return NNB_OK;
}

int nnb_get_math_mode(void) { return nnb::math_mode(); }

nnb_status nnb_ipc_export(const void* ptr, unsigned char* handle, size_t* offset) {
	if (!ptr || !handle || !offset) return nnb::fail(NNB_ERR_INVALID, "ipc_export: null pointer");
	std::call_once(nnb::g_range_once, [] {
		void* fn = nullptr;
		cudaDriverEntryPointQueryResult q;
		if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess
				&& q == cudaDriverEntryPointSuccess)
			nnb::g_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
	});
	if (!nnb::g_range) return nnb::fail(NNB_ERR_CUDA, "cuMemGetAddressRange is not available from the driver");
	CUdeviceptr base = 0;
	size_t size = 0;
	if (nnb::g_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
		return nnb::fail(NNB_ERR_INVALID, "ipc_export: not a device allocation");
	cudaIpcMemHandle_t h;
	NNB_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
	std::memcpy(handle, &h, sizeof h);
	*offset = static_cast<size_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
	return NNB_OK;
}

nnb_status nnb_ipc_open(const unsigned char* handle, size_t offset, void** ptr) {
	if (!handle || !ptr) return nnb::fail(NNB_ERR_INVALID, "ipc_open: null pointer");
	cudaIpcMemHandle_t h;
	std::memcpy(&h, handle, sizeof h);
	void* base = nullptr;
	NNB_CUDA_TRY(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
	*ptr = static_cast<char*>(base) + offset;
	return NNB_OK;
}

nnb_status nnb_copy_async(void* stream, void* dst, const void* src, size_t bytes) {
	if (bytes == 0) return NNB_OK;
	if (!dst || !src) return nnb::fail(NNB_ERR_INVALID, "copy_async: null pointer");
	NNB_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
	return NNB_OK;
}

nnb_status nnb_ipc_close(void* ptr, size_t offset) {
	if (!ptr) return NNB_OK;
	NNB_CUDA_TRY(cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset));
	return NNB_OK;
}

int nnb_device_error(void* stream) {
	nnb::DeviceState* st = nullptr;
	if (nnb::device_state(&st) != NNB_OK) return -1;
	if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess) return -1;
	int v = 0;
	if (cudaMemcpy(&v, st->error_word, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
	if (v != 0) cudaMemset(st->error_word, 0, sizeof(int));
	return v;
}

}  // extern "C"
