// nnb_internal.h -- host-side plumbing shared by the C-ABI translation units: error text, status
// helpers, per-device state (error word, SM count, tensor-map encoder) and stream-ordered
// scratch allocation.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>

#include "../../include/nnb.h"

namespace nnb {

// Records printf-style text as this thread's last error and returns `st`.
nnb_status fail(nnb_status st, const char* fmt, ...);

// Maps a CUDA error to NNB_ERR_CUDA with a message naming `what`; cudaSuccess -> NNB_OK.
nnb_status cuda_status(cudaError_t e, const char* what);

#define NNB_CUDA_TRY(expr)                                            \
	do {                                                              \
		cudaError_t nnb_e_ = (expr);                                  \
		if (nnb_e_ != cudaSuccess) return ::nnb::cuda_status(nnb_e_, #expr); \
	} while (0)

#define NNB_TRY(expr)                          \
	do {                                       \
		nnb_status nnb_s_ = (expr);            \
		if (nnb_s_ != NNB_OK) return nnb_s_;   \
	} while (0)

struct DeviceState {
	int device = -1;
	int sm_count = 0;
	int* error_word = nullptr;   // device int, first kernel error code wins
	bool ready = false;
};

// State of the current device, created on first use (checks for an sm_100 device).
nnb_status device_state(DeviceState** out);

// cuTensorMapEncodeTiled, fetched once through the runtime's driver entry point.
nnb_status encode_tiled_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
		uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
		CUtensorMapSwizzle swizzle);
// The same for a float32 tensor of `rank` (2..5) dimensions: dims[0] innermost, strides[i] the byte
// stride of dimension i + 1, box[i] the box extent along dimension i.
nnb_status encode_tiled_nd(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
		const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle);

// Stream-ordered scratch from the device's default memory pool (kept cached by the pool).
nnb_status scratch_alloc(void** p, size_t bytes, cudaStream_t s);
nnb_status scratch_free(void* p, cudaStream_t s);

// Process default math mode.
int math_mode();

}  // namespace nnb
