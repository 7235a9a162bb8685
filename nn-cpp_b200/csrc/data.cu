// data.cu -- batch assembly for the DataLoader (src/data/dataloader.cpp:76-96, src/data/text.cpp:60-70)
// from datasets held in HBM.
//
// The reference stacks dataset.get(index) tensors on the host for every batch. Here a dataset that
// fits the device (TensorDataset rows, a SequenceDataset's token stream) is uploaded once, the
// epoch's sample order (shuffled or weighted-drawn on the host, exactly as the reference draws it)
// is uploaded once per epoch, and each batch is one gather launch: no host work, no H2D copy per
// step, and the launch can sit inside a CUDA graph.
//
//   gather_rows:    dst[r] = src[index[r]], rows of row_bytes bytes (a TensorDataset's inputs or
//                   targets); one warp per row, 16-, 4- or 1-byte moves by alignment.
//   gather_windows: x[b][t] = tokens[start[b] + t], y[b][t] = tokens[start[b] + 1 + t] (the next-token
//                   windows of SequenceDataset), int32 tokens widened to int64 ids.
// Both are HBM-bound copies (bytes moved = 2 x bytes gathered). An index outside the dataset
// writes zeros for that row and sets the device error word (the reference throws TensorIndexError).
#include "nnb_internal.h"
#include "nnb_ops.h"
#include "nnb_trace.h"

namespace nnb {

namespace {

constexpr int kDevBadSample = 17;      // device error word: a sample index outside the dataset
constexpr int kGatherThreads = 256;

template <typename V>
__global__ void gather_rows_kernel(const V* __restrict__ src, long long vec_per_row, long long rows,
		const int64_t* __restrict__ index, long long count, V* __restrict__ dst, int* err) {
	const int lane = threadIdx.x & 31;
	const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
	for (long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; r < count; r += warps) {
		const int64_t i = index[r];
		V* out = dst + r * vec_per_row;
		if (i < 0 || i >= rows) {
			for (long long c = lane; c < vec_per_row; c += 32) out[c] = V{};
			if (lane == 0) atomicCAS(err, 0, kDevBadSample);
			continue;
		}
		const V* in = src + i * vec_per_row;
		for (long long c = lane; c < vec_per_row; c += 32) out[c] = in[c];
	}
}

__global__ void gather_windows_kernel(const int32_t* __restrict__ tokens, long long n_windows,
		const int64_t* __restrict__ start, long long count, long long block, int64_t* __restrict__ x,
		int64_t* __restrict__ y, int* err) {
	const int lane = threadIdx.x & 31;
	const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
	for (long long b = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; b < count; b += warps) {
		const int64_t s = start[b];
		int64_t* xr = x + b * block;
		int64_t* yr = y + b * block;
		if (s < 0 || s >= n_windows) {
			for (long long t = lane; t < block; t += 32) xr[t] = yr[t] = 0;
			if (lane == 0) atomicCAS(err, 0, kDevBadSample);
			continue;
		}
		const int32_t* w = tokens + s;
		for (long long t = lane; t < block; t += 32) {
			xr[t] = w[t];
			yr[t] = w[t + 1];
		}
	}
}

unsigned gather_grid(long long count) {
	const long long warps_per_block = kGatherThreads / 32;
	long long b = (count + warps_per_block - 1) / warps_per_block;
	if (b < 1) b = 1;
	if (b > 148 * 16) b = 148 * 16;
	return (unsigned)b;
}

}  // namespace

}  // namespace nnb

extern "C" {

nnb_status nnb_gather_rows(void* stream, const void* src, size_t row_bytes, size_t rows, const int64_t* index,
		size_t count, void* dst) {
	if (count == 0 || row_bytes == 0) return NNB_OK;
	if (!src || !index || !dst) return nnb::fail(NNB_ERR_INVALID, "gather_rows: null pointer");
	nnb::DeviceState* dev = nullptr;
	NNB_TRY(nnb::device_state(&dev));
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const uintptr_t align = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | row_bytes;
	const unsigned grid = nnb::gather_grid((long long)count);
	nnb::TraceScope ts(s, nnb::kTraceAux);
	if (align % 16 == 0)
		nnb::gather_rows_kernel<uint4><<<grid, nnb::kGatherThreads, 0, s>>>(static_cast<const uint4*>(src),
			(long long)(row_bytes / 16), (long long)rows, index, (long long)count, static_cast<uint4*>(dst), dev->error_word);
	else if (align % 4 == 0)
		nnb::gather_rows_kernel<uint32_t><<<grid, nnb::kGatherThreads, 0, s>>>(static_cast<const uint32_t*>(src),
			(long long)(row_bytes / 4), (long long)rows, index, (long long)count, static_cast<uint32_t*>(dst),
			dev->error_word);
	else
		nnb::gather_rows_kernel<unsigned char><<<grid, nnb::kGatherThreads, 0, s>>>(
			static_cast<const unsigned char*>(src), (long long)row_bytes, (long long)rows, index, (long long)count,
			static_cast<unsigned char*>(dst), dev->error_word);
	return nnb::cuda_status(cudaGetLastError(), "gather_rows launch");
}

nnb_status nnb_gather_windows(void* stream, const int32_t* tokens, size_t n_tokens, const int64_t* start, size_t count,
		size_t block, int64_t* x, int64_t* y) {
	if (block == 0 || n_tokens <= block)
		return nnb::fail(NNB_ERR_INVALID, "gather_windows: need block >= 1 and more than block tokens");
	if (count == 0) return NNB_OK;
	if (!tokens || !start || !x || !y) return nnb::fail(NNB_ERR_INVALID, "gather_windows: null pointer");
	nnb::DeviceState* dev = nullptr;
	NNB_TRY(nnb::device_state(&dev));
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	nnb::TraceScope ts(s, nnb::kTraceAux);
	nnb::gather_windows_kernel<<<nnb::gather_grid((long long)count), nnb::kGatherThreads, 0, s>>>(tokens,
		(long long)(n_tokens - block), start, (long long)count, (long long)block, x, y, dev->error_word);
	return nnb::cuda_status(cudaGetLastError(), "gather_windows launch");
}

}  // extern "C"
