// nnb_ops.h -- library-internal helpers shared between the op translation units.
#pragma once

#include <cuda_runtime.h>

#include "../../include/nnb.h"

namespace nnb {

// out[j] (+)= sum over rows of g[r][j] in the fixed chunked order of ops_linear.cu.
nnb_status colsum(cudaStream_t s, const float* g, long long rows, long long cols, float* out, int first);
// dX (+)= G W and dW_z (+)= G_z^T X_z (per group of rows) of a linear backward; either may be null.
nnb_status linear_bwd_gemms(cudaStream_t s, long long rows, long long K, long long n, long long groups, const float* g,
		const float* x, const void* x_pack, int x_pack_mode, const float* w, float* dx, int dx_first, float* dw,
		long long dw_stride, int dw_first);
// The same per group of rows/groups consecutive rows: out[z*out_stride + j] (+)= sum over group z's rows.
nnb_status colsum_grouped(cudaStream_t s, const float* g, long long rows, long long cols, long long groups, float* out,
		long long out_stride, int first);

// Inverted dropout's factor for kept elements, 1 / (1 - p) in float (dropout.cpp:24); 0 for p == 1.
float dropout_keep_scale(float p);

// Elementwise ceiling for 1-D grids: enough blocks for n items, at most 148 * 64 blocks.
inline unsigned grid_for(long long n, int threads) {
	long long b = (n + threads - 1) / threads;
	if (b < 1) b = 1;
	if (b > 148 * 64) b = 148 * 64;
	return (unsigned)b;
}

}  // namespace nnb
