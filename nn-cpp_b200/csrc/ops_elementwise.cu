// ops_elementwise.cu -- the support ops the CNN and transformer configs need so that nothing on
// their path runs on the host: relu, gelu, residual add / gradient accumulation, maxpool2d,
// cross_entropy_loss, sequence_cross_entropy, embedding and the AdamW step.
//
// Each kernel keeps the reference's expression and, where the reference's order of operations is
// sequential per output element, that order too, so relu, gelu (Cephes tanh), add, maxpool2d,
// embedding (forward and backward) and AdamW give the reference's bits on the same inputs.
// The loss ops use CUDA's expf/logf and a fixed warp-tree order for the row sums, so they agree
// within tolerance rather than bit for bit.
#include <algorithm>
#include <cmath>

#include "nnb_internal.h"
#include "nnb_math.cuh"
#include "nnb_ops.h"
#include "nnb_trace.h"

namespace nnb {

namespace {

constexpr int kDevBadIndex = 16;   // device error word: a target or token id outside its range

#define GRID_STRIDE(i, n) \
	for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (n); i += (long long)gridDim.x * blockDim.x)

__global__ void relu_fwd_kernel(long long n, const float* __restrict__ x, float* __restrict__ y) {
	GRID_STRIDE(i, n) y[i] = x[i] > 0.0f ? x[i] : 0.0f;          // ops.cpp:780
}

__global__ void relu_bwd_kernel(long long n, const float* __restrict__ x, const float* __restrict__ g,
		float* __restrict__ dx, int first) {
	GRID_STRIDE(i, n) {
		const float v = x[i] > 0.0f ? g[i] : 0.0f;                  // ops.cpp:790
		dx[i] = first ? v + 0.0f : dx[i] + v;
	}
}

__global__ void gelu_fwd_kernel(long long n, const float* __restrict__ x, float* __restrict__ y,
		float* __restrict__ th) {
	GRID_STRIDE(i, n) {
		const float t = tanh_one(gelu_tanh_arg(x[i]));            // ops.cpp:462-464
		th[i] = t;
		y[i] = gelu_fwd(x[i], t);
	}
}

// th may be null: the tanh is then recomputed from x (same bits as the saved one)
__global__ void gelu_bwd_kernel(long long n, const float* __restrict__ x, const float* __restrict__ th,
		const float* __restrict__ g, float* __restrict__ dx, int first) {
	GRID_STRIDE(i, n) {
		const float t = th ? th[i] : tanh_one(gelu_tanh_arg(x[i]));
		const float v = gelu_bwd(g[i], x[i], t);                  // ops.cpp:474-477
		dx[i] = first ? v + 0.0f : dx[i] + v;
	}
}

__global__ void fill_kernel(long long n, float value, float* __restrict__ y) {
	GRID_STRIDE(i, n) y[i] = value;
}

__global__ void scale_kernel(long long n, float alpha, const float* __restrict__ x, float* __restrict__ y) {
	GRID_STRIDE(i, n) y[i] = x[i] * alpha;                      // Tensor scale, src/tensor.cpp:558-566
}

// y = a + b with b broadcast along the leading axis when b_period < n (b has b_period elements)
__global__ void add_kernel(long long n, const float* __restrict__ a, const float* __restrict__ b, long long b_period,
		float* __restrict__ y) {
	GRID_STRIDE(i, n) y[i] = a[i] + b[i % b_period];
}

// the grad_accum convention (ops.cpp:67-73): first stores src + 0, otherwise adds; negate subtracts
__global__ void accumulate_kernel(long long n, const float* __restrict__ src, float* __restrict__ dst, int first,
		int negate) {
	GRID_STRIDE(i, n) {
		if (negate) dst[i] = first ? 0.0f - src[i] : dst[i] - src[i];
		else dst[i] = first ? src[i] + 0.0f : dst[i] + src[i];
	}
}

// Vector (float4) forms of the elementwise kernels, used when the length is a multiple of 4 and
// every pointer is 16-byte aligned: four elements per thread and 16-byte accesses, each element
// getting exactly the scalar kernel's operations.
__device__ __forceinline__ float4 ld4(const float* p, long long i) { return __ldg(reinterpret_cast<const float4*>(p) + i); }

__device__ __forceinline__ float4 store_rule(float4 v, const float4* dst, int first) {
	if (first) return make_float4(v.x + 0.0f, v.y + 0.0f, v.z + 0.0f, v.w + 0.0f);
	const float4 c = *dst;
	return make_float4(c.x + v.x, c.y + v.y, c.z + v.z, c.w + v.w);
}

__global__ void gelu_bwd_vec_kernel(long long n4, const float* __restrict__ x, const float* __restrict__ th,
		const float* __restrict__ g, float* __restrict__ dx, int first) {
	GRID_STRIDE(i, n4) {
		const float4 xv = ld4(x, i), gv = ld4(g, i);
		const float4 tv = th ? ld4(th, i)
			: make_float4(tanh_one(gelu_tanh_arg(xv.x)), tanh_one(gelu_tanh_arg(xv.y)), tanh_one(gelu_tanh_arg(xv.z)),
				tanh_one(gelu_tanh_arg(xv.w)));
		const float4 v = make_float4(gelu_bwd(gv.x, xv.x, tv.x), gelu_bwd(gv.y, xv.y, tv.y), gelu_bwd(gv.z, xv.z, tv.z),
			gelu_bwd(gv.w, xv.w, tv.w));
		float4* d = reinterpret_cast<float4*>(dx) + i;
		*d = store_rule(v, d, first);
	}
}

__global__ void add_same_vec_kernel(long long n4, const float* __restrict__ a, const float* __restrict__ b,
		float* __restrict__ y) {
	GRID_STRIDE(i, n4) {
		const float4 u = ld4(a, i), v = ld4(b, i);
		reinterpret_cast<float4*>(y)[i] = make_float4(u.x + v.x, u.y + v.y, u.z + v.z, u.w + v.w);
	}
}

// b broadcast over the rows of a [rows, period]: rows over grid.y, float4 columns over grid.x
__global__ void add_bcast_vec_kernel(long long rows, long long period4, const float* __restrict__ a,
		const float* __restrict__ b, float* __restrict__ y) {
	for (long long r = blockIdx.y; r < rows; r += gridDim.y)
		for (long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x; c < period4; c += (long long)gridDim.x * blockDim.x) {
			const float4 u = ld4(a, r * period4 + c), v = ld4(b, c);
			reinterpret_cast<float4*>(y)[r * period4 + c] = make_float4(u.x + v.x, u.y + v.y, u.z + v.z, u.w + v.w);
		}
}

__global__ void accumulate_vec_kernel(long long n4, const float* __restrict__ src, float* __restrict__ dst, int first,
		int negate) {
	GRID_STRIDE(i, n4) {
		const float4 v = ld4(src, i);
		float4* d = reinterpret_cast<float4*>(dst) + i;
		if (negate) {
			if (first) {
				*d = make_float4(0.0f - v.x, 0.0f - v.y, 0.0f - v.z, 0.0f - v.w);
			} else {
				const float4 c = *d;
				*d = make_float4(c.x - v.x, c.y - v.y, c.z - v.z, c.w - v.w);
			}
		} else {
			*d = store_rule(v, d, first);
		}
	}
}

// rows over grid.y (at most 65535, the kernel loops), enough column blocks for about 32 blocks per SM
inline dim3 ce_bwd_grid(long long rows, int C) {
	const unsigned bx = (unsigned)std::max(1, (C + 255) / 256);
	const long long by = std::min<long long>(rows, std::max<long long>(1, 148 * 32 / bx));
	return dim3(bx, (unsigned)std::min<long long>(by, 65535));
}

__host__ __device__ inline bool vec4_ok(long long n, const void* p0, const void* p1 = nullptr, const void* p2 = nullptr,
		const void* p3 = nullptr) {
	const uintptr_t m = reinterpret_cast<uintptr_t>(p0) | reinterpret_cast<uintptr_t>(p1) |
		reinterpret_cast<uintptr_t>(p2) | reinterpret_cast<uintptr_t>(p3);
	return n % 4 == 0 && (m & 15) == 0;
}

// ---------------------------------------------------------------------------------------------
// maxpool2d (ops.cpp:1609-1705): first maximum wins, offset 0 when nothing beats -inf
// ---------------------------------------------------------------------------------------------

__global__ void maxpool_fwd_kernel(long long planes, int H, int W, int k, int stride, int ho, int wo,
		const float* __restrict__ x, float* __restrict__ y, uint32_t* __restrict__ arg) {
	GRID_STRIDE(i, planes * ho * wo) {
		const long long p = i / ((long long)ho * wo);
		const int oh = (int)((i / wo) % ho), ow = (int)(i % wo);
		const float* plane = x + p * (long long)H * W;
		float best = -INFINITY;
		uint32_t at = 0;
		for (int ph = 0; ph < k; ++ph) {
			const int r = oh * stride + ph;
			for (int pw = 0; pw < k; ++pw) {
				const int c = ow * stride + pw;
				const float v = plane[(long long)r * W + c];
				if (v > best) {
					best = v;
					at = (uint32_t)(r * W + c);
				}
			}
		}
		y[i] = best;
		arg[i] = at;
	}
}

// Gather form of the reference's scatter `plane[arg[i]] += g[i]` in output order: each input
// element adds, in increasing output index, the gradients of the windows whose argmax it is.
__global__ void maxpool_bwd_kernel(long long planes, int H, int W, int k, int stride, int ho, int wo,
		const float* __restrict__ g, const uint32_t* __restrict__ arg, float* __restrict__ dx, int first) {
	GRID_STRIDE(i, planes * (long long)H * W) {
		const long long p = i / ((long long)H * W);
		const int off = (int)(i % ((long long)H * W));
		const int r = off / W, c = off % W;
		// windows (oh, ow) with oh*stride <= r < oh*stride + k
		const int oh_lo = r >= k ? (r - k) / stride + 1 : 0, oh_hi = min(ho - 1, r / stride);
		const int ow_lo = c >= k ? (c - k) / stride + 1 : 0, ow_hi = min(wo - 1, c / stride);
		float acc = first ? 0.0f : dx[i];
		const long long obase = p * (long long)ho * wo;
		for (int oh = oh_lo; oh <= oh_hi; ++oh)
			for (int ow = ow_lo; ow <= ow_hi; ++ow) {
				const long long o = obase + (long long)oh * wo + ow;
				if (arg[o] == (uint32_t)off) acc += g[o];
			}
		dx[i] = acc;
	}
}

// ---------------------------------------------------------------------------------------------
// avgpool2d (ops.cpp:1707-1772): window sum in (row, column) order from +0, times 1 / k^2
// ---------------------------------------------------------------------------------------------

__global__ void avgpool_fwd_kernel(long long planes, int H, int W, int k, int stride, int ho, int wo, float inv_area,
		const float* __restrict__ x, float* __restrict__ y) {
	GRID_STRIDE(i, planes * ho * wo) {
		const long long p = i / ((long long)ho * wo);
		const int oh = (int)((i / wo) % ho), ow = (int)(i % wo);
		const float* plane = x + p * (long long)H * W;
		float acc = 0.0f;
		for (int ph = 0; ph < k; ++ph) {
			const float* row = plane + (long long)(oh * stride + ph) * W + ow * stride;
			for (int pw = 0; pw < k; ++pw) acc += row[pw];
		}
		y[i] = acc * inv_area;
	}
}

// the reference scatters share = g * (1/k^2) into every window element, windows in (oh, ow) order;
// gathered here per input element over the windows that contain it, in that order
__global__ void avgpool_bwd_kernel(long long planes, int H, int W, int k, int stride, int ho, int wo, float inv_area,
		const float* __restrict__ g, float* __restrict__ dx, int first) {
	GRID_STRIDE(i, planes * (long long)H * W) {
		const long long p = i / ((long long)H * W);
		const int off = (int)(i % ((long long)H * W));
		const int r = off / W, c = off % W;
		const int oh_lo = r >= k ? (r - k) / stride + 1 : 0, oh_hi = min(ho - 1, r / stride);
		const int ow_lo = c >= k ? (c - k) / stride + 1 : 0, ow_hi = min(wo - 1, c / stride);
		float acc = first ? 0.0f : dx[i];
		const long long obase = p * (long long)ho * wo;
		for (int oh = oh_lo; oh <= oh_hi; ++oh)
			for (int ow = ow_lo; ow <= ow_hi; ++ow) acc += g[obase + (long long)oh * wo + ow] * inv_area;
		dx[i] = acc;
	}
}

// ---------------------------------------------------------------------------------------------
// sum / mean over one axis (reduce_axis, ops.cpp:284-376): x viewed as [outer, n, inner]
// ---------------------------------------------------------------------------------------------

__global__ void reduce_axis_fwd_kernel(long long outer, long long n, long long inner, const float* __restrict__ x,
		int average, float factor, float* __restrict__ y) {
	GRID_STRIDE(j, outer * inner) {
		const long long base = (j / inner) * n * inner + j % inner;
		float total = 0.0f;
		for (long long k = 0; k < n; ++k) total += x[base + k * inner];
		y[j] = average ? total * factor : total;
	}
}

__global__ void reduce_axis_bwd_kernel(long long outer, long long n, long long inner, const float* __restrict__ g,
		float factor, float* __restrict__ dx, int first) {
	GRID_STRIDE(j, outer * inner) {
		const long long base = (j / inner) * n * inner + j % inner;
		const float v = g[j] * factor;
		for (long long k = 0; k < n; ++k) {
			float* d = dx + base + k * inner;
			*d = first ? v + 0.0f : *d + v;
		}
	}
}

// ---------------------------------------------------------------------------------------------
// Cross entropy over rows (ops.cpp:1774-1840) and sequences (ops.cpp:1908-1979)
// ---------------------------------------------------------------------------------------------

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

// One warp per row: softmax row and the row's loss (ignored rows: loss 0, softmax untouched).
// label smoothing ls: loss = (1-ls)*nll + ls*mean_nll (ls = 0 for cross_entropy_loss).
__global__ void ce_rows_kernel(long long rows, int C, const float* __restrict__ logits,
		const int64_t* __restrict__ targets, int64_t ignore_index, int use_ignore, float ls,
		float* __restrict__ softmax, float* __restrict__ row_loss, int* __restrict__ valid, int* err) {
	const int lane = threadIdx.x & 31;
	const long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
	if (r >= rows) return;
	const int64_t t = targets[r];
	if (use_ignore && t == ignore_index) {
		if (lane == 0) {
			row_loss[r] = 0.0f;
			valid[r] = 0;
		}
		return;
	}
	if (t < 0 || t >= C) {
		if (lane == 0) {
			row_loss[r] = __int_as_float(0x7fc00000);
			valid[r] = 0;
			atomicCAS(err, 0, kDevBadIndex);
		}
		return;
	}
	const float* row = logits + r * C;
	float m = -INFINITY;
	for (int c = lane; c < C; c += 32) m = fmaxf(m, row[c]);
	m = warp_max(m);
	float se = 0.0f;
	for (int c = lane; c < C; c += 32) se += expf(row[c] - m);
	se = warp_sum(se);
	const float lse = logf(se);
	float* sm = softmax + r * C;
	float mean_nll = 0.0f;
	const float inv_c = 1.0f / (float)C;
	for (int c = lane; c < C; c += 32) {
		const float lp = row[c] - m - lse;
		sm[c] = expf(lp);
		mean_nll -= lp * inv_c;
	}
	mean_nll = warp_sum(mean_nll);
	if (lane == 0) {
		const float nll = -(row[t] - m - lse);
		row_loss[r] = ls == 0.0f ? nll : (1.0f - ls) * nll + ls * mean_nll;
		valid[r] = 1;
	}
}

// The same row results for wide rows (C % 4 == 0, 16-byte aligned, C <= 4096): one 128-thread block
// per row keeps the row in registers (up to eight float4 per thread), so the logits are read from HBM
// once instead of three times; the max and the sums are combined in a fixed order (each thread's
// elements in order, then the warp's xor tree, then the four warps in order), so the results are
// deterministic. The operations per element are those of ce_rows_kernel.
constexpr int kCeBlock = 128, kCeV4 = 8;
__global__ void __launch_bounds__(kCeBlock) ce_rows_block_kernel(long long rows, int C,
		const float* __restrict__ logits, const int64_t* __restrict__ targets, int64_t ignore_index, int use_ignore,
		float ls, float* __restrict__ softmax, float* __restrict__ row_loss, int* __restrict__ valid, int* err) {
	__shared__ float red[2][kCeBlock / 32];
	const long long r = blockIdx.x;
	const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
	const int64_t t = targets[r];
	if (use_ignore && t == ignore_index) {
		if (tid == 0) {
			row_loss[r] = 0.0f;
			valid[r] = 0;
		}
		return;
	}
	if (t < 0 || t >= C) {
		if (tid == 0) {
			row_loss[r] = __int_as_float(0x7fc00000);
			valid[r] = 0;
			atomicCAS(err, 0, kDevBadIndex);
		}
		return;
	}
	const int C4 = C >> 2;
	const float4* row = reinterpret_cast<const float4*>(logits + r * C);
	float4 v[kCeV4];
	float m = -INFINITY;
#pragma unroll
	for (int u = 0; u < kCeV4; ++u) {
		const int i = tid + u * kCeBlock;
		v[u] = i < C4 ? __ldg(row + i) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
		m = fmaxf(fmaxf(fmaxf(m, v[u].x), fmaxf(v[u].y, v[u].z)), v[u].w);
	}
	m = warp_max(m);
	if (lane == 0) red[0][warp] = m;
	__syncthreads();
	m = fmaxf(fmaxf(red[0][0], red[0][1]), fmaxf(red[0][2], red[0][3]));
	float se = 0.0f;
#pragma unroll
	for (int u = 0; u < kCeV4; ++u)
		if (tid + u * kCeBlock < C4) {
			se += expf(v[u].x - m);
			se += expf(v[u].y - m);
			se += expf(v[u].z - m);
			se += expf(v[u].w - m);
		}
	se = warp_sum(se);
	if (lane == 0) red[1][warp] = se;
	__syncthreads();
	se = ((red[1][0] + red[1][1]) + red[1][2]) + red[1][3];
	const float lse = logf(se);
	float4* sm = reinterpret_cast<float4*>(softmax + r * C);
	float mean_nll = 0.0f;
	const float inv_c = 1.0f / (float)C;
#pragma unroll
	for (int u = 0; u < kCeV4; ++u) {
		const int i = tid + u * kCeBlock;
		if (i < C4) {
			const float l0 = v[u].x - m - lse, l1 = v[u].y - m - lse, l2 = v[u].z - m - lse, l3 = v[u].w - m - lse;
			sm[i] = make_float4(expf(l0), expf(l1), expf(l2), expf(l3));
			mean_nll -= l0 * inv_c;
			mean_nll -= l1 * inv_c;
			mean_nll -= l2 * inv_c;
			mean_nll -= l3 * inv_c;
		}
	}
	mean_nll = warp_sum(mean_nll);
	__syncthreads();                          // red[0] is reused below
	if (lane == 0) red[0][warp] = mean_nll;
	__syncthreads();
	if (tid == 0) {
		mean_nll = ((red[0][0] + red[0][1]) + red[0][2]) + red[0][3];
		const float nll = -(logits[r * C + t] - m - lse);
		row_loss[r] = ls == 0.0f ? nll : (1.0f - ls) * nll + ls * mean_nll;
		valid[r] = 1;
	}
}

// loss = sum(row_loss) / count in fixed order: 256 threads sum contiguous slices serially
// (fp64 for sequences, as the reference; fp32 otherwise), then thread 0 sums the slices in order.
// norm: the backward scale's divisor N (rows) or multiplier 1/count (sequences)
__global__ void ce_total_kernel(long long rows, const float* __restrict__ row_loss, const int* __restrict__ valid,
		int as_double, float* __restrict__ loss, float* __restrict__ norm) {
	__shared__ double part_d[256];
	__shared__ float part_f[256];
	__shared__ long long part_n[256];
	const int t = threadIdx.x;
	const long long per = (rows + 255) / 256, r0 = t * per, r1 = min(rows, r0 + per);
	double sd = 0.0;
	float sf = 0.0f;
	long long cnt = 0;
	for (long long r = r0; r < r1; ++r) {
		sd += (double)row_loss[r];
		sf += row_loss[r];
		cnt += valid[r];
	}
	part_d[t] = sd;
	part_f[t] = sf;
	part_n[t] = cnt;
	__syncthreads();
	if (t == 0) {
		double td = 0.0;
		float tf = 0.0f;
		long long tn = 0;
		for (int i = 0; i < 256; ++i) {
			td += part_d[i];
			tf += part_f[i];
			tn += part_n[i];
		}
		if (as_double) {
			*loss = tn ? (float)(td / (double)tn) : __int_as_float(0x7fc00000);
			*norm = tn ? 1.0f / (float)tn : 0.0f;
		} else {
			*loss = tf / (float)rows;
			*norm = (float)rows;
		}
	}
}

// dlogits (+)= (softmax - ls/C - [c == t](1 - ls)) * scale (ignored rows: 0), where
// scale = grad_loss / N for rows (ops.cpp:1830) and grad_loss * (1/count) for sequences (ops.cpp:1968)
__global__ void ce_bwd_kernel(long long rows, int C, const float* __restrict__ softmax,
		const int64_t* __restrict__ targets, int64_t ignore_index, int use_ignore, float ls,
		const float* __restrict__ grad_loss, const float* __restrict__ norm, float* __restrict__ dlogits,
		int first) {
	const float scale = use_ignore ? grad_loss[0] * norm[0] : grad_loss[0] / norm[0];
	// rows over grid.y, columns over grid.x
	for (long long r = blockIdx.y; r < rows; r += gridDim.y) {
		const int64_t t = targets[r];
		const bool live = !(use_ignore && t == ignore_index) && t >= 0 && t < C;
		for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < C; c += gridDim.x * blockDim.x) {
			const long long i = r * C + c;
			float v = 0.0f;
			if (live) {
				if (ls == 0.0f && !use_ignore) {
					v = (c == t ? softmax[i] - 1.0f : softmax[i]) * scale;            // ops.cpp:1835
				} else {
					float q = softmax[i] - ls / (float)C;                             // ops.cpp:1972-1974
					if (c == t) q -= 1.0f - ls;
					v = q * scale;
				}
			}
			dlogits[i] = first ? v + 0.0f : dlogits[i] + v;
		}
	}
}

// The same gradient four columns at a time (C % 4 == 0, 16-byte aligned pointers): a grid-stride walk
// over the float4 groups of the whole [rows, C] array, each element getting ce_bwd_kernel's operations.
__global__ void ce_bwd_vec_kernel(long long n4, int C, const float* __restrict__ softmax,
		const int64_t* __restrict__ targets, int64_t ignore_index, int use_ignore, float ls,
		const float* __restrict__ grad_loss, const float* __restrict__ norm, float* __restrict__ dlogits,
		int first) {
	const float scale = use_ignore ? grad_loss[0] * norm[0] : grad_loss[0] / norm[0];
	const int C4 = C >> 2;
	GRID_STRIDE(i, n4) {
		const long long r = i / C4;
		const int c0 = (int)(i - r * C4) * 4;
		const int64_t t = __ldg(targets + r);
		const bool live = !(use_ignore && t == ignore_index) && t >= 0 && t < C;
		float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
		if (live) {
			const float4 p = ld4(softmax, i);
			const float pv[4] = {p.x, p.y, p.z, p.w};
			float o[4];
#pragma unroll
			for (int j = 0; j < 4; ++j) {
				const int c = c0 + j;
				if (ls == 0.0f && !use_ignore) {
					o[j] = (c == t ? pv[j] - 1.0f : pv[j]) * scale;                // ops.cpp:1835
				} else {
					float q = pv[j] - ls / (float)C;                               // ops.cpp:1972-1974
					if (c == t) q -= 1.0f - ls;
					o[j] = q * scale;
				}
			}
			v = make_float4(o[0], o[1], o[2], o[3]);
		}
		float4* d = reinterpret_cast<float4*>(dlogits) + i;
		*d = store_rule(v, d, first);
	}
}

// ---------------------------------------------------------------------------------------------
// embedding (ops.cpp:1991-2015)
// ---------------------------------------------------------------------------------------------

__global__ void embedding_fwd_kernel(long long count, int V, int D, const float* __restrict__ w,
		const int64_t* __restrict__ ids, float* __restrict__ out, int* err) {
	GRID_STRIDE(i, count * (long long)D) {
		const long long tok = i / D;
		const int d = (int)(i % D);
		const int64_t id = ids[tok];
		if (id < 0 || id >= V) {
			out[i] = __int_as_float(0x7fc00000);
			if (d == 0) atomicCAS(err, 0, kDevBadIndex);
		} else {
			out[i] = w[id * D + d];
		}
	}
}

constexpr int kEmbChunk = 1024;

// hist[chunk][v] = tokens of id v in chunk
__global__ void embedding_hist_kernel(long long count, int V, const int64_t* __restrict__ ids, int* __restrict__ hist) {
	GRID_STRIDE(i, count) {
		const int64_t id = ids[i];
		if (id >= 0 && id < V) atomicAdd(&hist[(i / kEmbChunk) * V + id], 1);
	}
}

// start[v][chunk] = position of the first token of (id v, chunk) in the id-major, token-order
// layout, id_begin[v] = first position of id v. One block of 1024 threads: per-thread totals of a
// slice of ids, an integer scan across threads (exact in any order), then the per-chunk starts.
__global__ void __launch_bounds__(1024) embedding_scan_kernel(int V, int chunks, const int* __restrict__ hist,
		int* __restrict__ start, int* __restrict__ id_begin) {
	__shared__ int part[1024];
	const int t = threadIdx.x;
	const int per = (V + 1023) / 1024, v0 = min(V, t * per), v1 = min(V, v0 + per);
	int tot = 0;
	for (int v = v0; v < v1; ++v)
		for (int c = 0; c < chunks; ++c) tot += hist[(long long)c * V + v];
	part[t] = tot;
	__syncthreads();
	for (int off = 1; off < 1024; off <<= 1) {
		const int x = t >= off ? part[t - off] : 0;
		__syncthreads();
		part[t] += x;
		__syncthreads();
	}
	int pos = t ? part[t - 1] : 0;
	for (int v = v0; v < v1; ++v) {
		id_begin[v] = pos;
		for (int c = 0; c < chunks; ++c) {
			start[(long long)v * chunks + c] = pos;
			pos += hist[(long long)c * V + v];
		}
	}
	if (t == 1023) id_begin[V] = part[1023];
}

// Stable placement: block c copies its chunk's ids and the V slot counters into shared memory,
// then one thread walks the chunk's tokens in order, so tokens of one id keep their order.
__global__ void embedding_place_kernel(long long count, int V, int chunks, const int64_t* __restrict__ ids,
		const int* __restrict__ start, int* __restrict__ order) {
	extern __shared__ int slots[];
	__shared__ int sid[kEmbChunk];
	const long long c = blockIdx.x, t0 = c * kEmbChunk, t1 = min(count, t0 + kEmbChunk);
	for (int v = threadIdx.x; v < V; v += blockDim.x) slots[v] = start[(long long)v * chunks + c];
	for (long long t = t0 + threadIdx.x; t < t1; t += blockDim.x) {
		const int64_t id = ids[t];
		sid[t - t0] = (id >= 0 && id < V) ? (int)id : -1;
	}
	__syncthreads();
	if (threadIdx.x >= 32) return;
	// warp 0 places the chunk's tokens in token order, 32 at a time: lanes holding the same id take
	// consecutive slots in lane (= token) order, and the group's first lane advances the id's slot,
	// which gives exactly the serial placement
	const int lane = threadIdx.x;
	for (long long base = t0; base < t1; base += 32) {
		const long long t = base + lane;
		const int id = t < t1 ? sid[t - t0] : -1;
		const unsigned same = __match_any_sync(0xffffffffu, id);
		const int leader = __ffs(same) - 1;
		const int rank = __popc(same & ((1u << lane) - 1u));
		int pos = 0;
		if (id >= 0 && lane == leader) pos = slots[id];
		pos = __shfl_sync(0xffffffffu, pos, leader);
		if (id >= 0) order[pos + rank] = (int)t;
		__syncwarp();
		if (id >= 0 && lane == leader) slots[id] = pos + __popc(same);
		__syncwarp();
	}
}

// dweight[v][d] (+)= g[t][d] for the tokens t of id v in token order (ops.cpp:2012-2013); with
// first set the row starts from 0, as the reference's zero-on-demand grad() does
__global__ void embedding_bwd_kernel(int V, int D, const int* __restrict__ id_begin, const int* __restrict__ order,
		const float* __restrict__ g, float* __restrict__ dw, int first) {
	GRID_STRIDE(i, (long long)V * D) {
		const int v = (int)(i / D), d = (int)(i % D);
		const int b = id_begin[v], e = id_begin[v + 1];
		if (b == e) {
			if (first) dw[i] = 0.0f;
			continue;
		}
		float acc = first ? 0.0f : dw[i];
		for (int k = b; k < e; ++k) acc += g[(long long)order[k] * D + d];
		dw[i] = acc;
	}
}

// ---------------------------------------------------------------------------------------------
// AdamW (src/optim/adamw.cpp:15-24 then src/optim/adam.cpp:24-43)
// ---------------------------------------------------------------------------------------------

__global__ void adamw_kernel(long long n, float* __restrict__ w, const float* __restrict__ g, float* __restrict__ m,
		float* __restrict__ v, float shrink, float lr, float b1, float b2, float eps, float c1, float c2) {
	GRID_STRIDE(k, n) {
		float wk = w[k] * shrink;
		const float gk = g[k];
		const float mk = b1 * m[k] + (1.0f - b1) * gk;
		const float vk = b2 * v[k] + (1.0f - b2) * gk * gk;
		m[k] = mk;
		v[k] = vk;
		wk -= lr * (mk / c1) / (sqrtf(vk / c2) + eps);
		w[k] = wk;
	}
}

// The same update with its per-step scalars in device memory, so a captured CUDA graph replays it:
// hyper = {shrink, lr, beta1, beta2, eps}; (c1, c2) = table[min(t, len) - 1] for t = *step (the
// corrections saturate at exactly 1.0f, where the table ends).
__global__ void adamw_device_kernel(long long n, float* __restrict__ w, const float* __restrict__ g,
		float* __restrict__ m, float* __restrict__ v, const float* __restrict__ hyper,
		const float* __restrict__ table, long long table_len, const int64_t* __restrict__ step) {
	const float shrink = hyper[0], lr = hyper[1], b1 = hyper[2], b2 = hyper[3], eps = hyper[4];
	long long t = *step;
	if (t < 1) return;
	if (t > table_len) t = table_len;
	const float c1 = table[2 * (t - 1)], c2 = table[2 * (t - 1) + 1];
	GRID_STRIDE(k, n) {
		float wk = w[k] * shrink;
		const float gk = g[k];
		const float mk = b1 * m[k] + (1.0f - b1) * gk;
		const float vk = b2 * v[k] + (1.0f - b2) * gk * gk;
		m[k] = mk;
		v[k] = vk;
		wk -= lr * (mk / c1) / (sqrtf(vk / c2) + eps);
		w[k] = wk;
	}
}

__global__ void step_advance_kernel(int64_t* step) {
	if (threadIdx.x == 0 && blockIdx.x == 0) *step += 1;
}

}  // namespace

}  // namespace nnb

using nnb::grid_for;

extern "C" {

#define NNB_LAUNCH(kind, grid, block, kernel, ...)                 \
	do {                                                           \
		nnb::TraceScope nnb_ts_(s, nnb::kind);                     \
		kernel<<<grid, block, 0, s>>>(__VA_ARGS__);                \
	} while (0)

nnb_status nnb_relu_fwd(void* stream, size_t n, const float* x, float* y) {
	if (n == 0) return NNB_OK;
	if (!x || !y) return nnb::fail(NNB_ERR_INVALID, "relu_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	NNB_LAUNCH(kTraceRowwise, grid_for(n, 256), 256, nnb::relu_fwd_kernel, (long long)n, x, y);
	return nnb::cuda_status(cudaGetLastError(), "relu_fwd launch");
}

nnb_status nnb_relu_bwd(void* stream, size_t n, const float* x, const float* g, float* dx, int dx_first) {
	if (n == 0) return NNB_OK;
	if (!x || !g || !dx) return nnb::fail(NNB_ERR_INVALID, "relu_bwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	NNB_LAUNCH(kTraceRowwise, grid_for(n, 256), 256, nnb::relu_bwd_kernel, (long long)n, x, g, dx, dx_first);
	return nnb::cuda_status(cudaGetLastError(), "relu_bwd launch");
}

nnb_status nnb_gelu_fwd(void* stream, size_t n, const float* x, float* y, float* tanh_saved) {
	if (n == 0) return NNB_OK;
	if (!x || !y || !tanh_saved) return nnb::fail(NNB_ERR_INVALID, "gelu_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	NNB_LAUNCH(kTraceRowwise, grid_for(n, 256), 256, nnb::gelu_fwd_kernel, (long long)n, x, y, tanh_saved);
	return nnb::cuda_status(cudaGetLastError(), "gelu_fwd launch");
}

nnb_status nnb_gelu_bwd(void* stream, size_t n, const float* x, const float* tanh_saved, const float* g, float* dx,
		int dx_first) {
	if (n == 0) return NNB_OK;
	if (!x || !g || !dx) return nnb::fail(NNB_ERR_INVALID, "gelu_bwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	if (nnb::vec4_ok((long long)n, x, tanh_saved, g, dx))
		NNB_LAUNCH(kTraceRowwise, grid_for(n / 4, 256), 256, nnb::gelu_bwd_vec_kernel, (long long)n / 4, x, tanh_saved, g,
			dx, dx_first);
	else
		NNB_LAUNCH(kTraceRowwise, grid_for(n, 256), 256, nnb::gelu_bwd_kernel, (long long)n, x, tanh_saved, g, dx, dx_first);
	return nnb::cuda_status(cudaGetLastError(), "gelu_bwd launch");
}

nnb_status nnb_fill(void* stream, size_t n, float value, float* y) {
	if (n == 0) return NNB_OK;
	if (!y) return nnb::fail(NNB_ERR_INVALID, "fill: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	NNB_LAUNCH(kTraceAux, grid_for(n, 256), 256, nnb::fill_kernel, (long long)n, value, y);
	return nnb::cuda_status(cudaGetLastError(), "fill launch");
}

nnb_status nnb_scale(void* stream, size_t n, float alpha, const float* x, float* y) {
	if (n == 0) return NNB_OK;
	if (!x || !y) return nnb::fail(NNB_ERR_INVALID, "scale: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	NNB_LAUNCH(kTraceRowwise, grid_for(n, 256), 256, nnb::scale_kernel, (long long)n, alpha, x, y);
	return nnb::cuda_status(cudaGetLastError(), "scale launch");
}

nnb_status nnb_add_fwd(void* stream, size_t n, const float* a, const float* b, size_t b_period, float* y) {
	if (n == 0) return NNB_OK;
	if (!a || !b || !y) return nnb::fail(NNB_ERR_INVALID, "add_fwd: null pointer");
	if (b_period == 0 || n % b_period != 0) return nnb::fail(NNB_ERR_SHAPE, "add_fwd: %zu is not a multiple of %zu", n, b_period);
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	if (b_period == n && nnb::vec4_ok((long long)n, a, b, y)) {
		NNB_LAUNCH(kTraceRowwise, grid_for(n / 4, 256), 256, nnb::add_same_vec_kernel, (long long)n / 4, a, b, y);
	} else if (nnb::vec4_ok((long long)b_period, a, b, y)) {
		const long long rows = (long long)(n / b_period), p4 = (long long)b_period / 4;
		const unsigned bx = (unsigned)std::min<long long>((p4 + 255) / 256, 64);
		const unsigned by = (unsigned)std::min<long long>(rows, 65535);
		NNB_LAUNCH(kTraceRowwise, dim3(bx, by), 256, nnb::add_bcast_vec_kernel, rows, p4, a, b, y);
	} else {
		NNB_LAUNCH(kTraceRowwise, grid_for(n, 256), 256, nnb::add_kernel, (long long)n, a, b, (long long)b_period, y);
	}
	return nnb::cuda_status(cudaGetLastError(), "add_fwd launch");
}

nnb_status nnb_accumulate(void* stream, size_t n, const float* src, float* dst, int first, int negate) {
	if (n == 0) return NNB_OK;
	if (!src || !dst) return nnb::fail(NNB_ERR_INVALID, "accumulate: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	if (nnb::vec4_ok((long long)n, src, dst))
		NNB_LAUNCH(kTraceRowwise, grid_for(n / 4, 256), 256, nnb::accumulate_vec_kernel, (long long)n / 4, src, dst, first,
			negate);
	else
		NNB_LAUNCH(kTraceRowwise, grid_for(n, 256), 256, nnb::accumulate_kernel, (long long)n, src, dst, first, negate);
	return nnb::cuda_status(cudaGetLastError(), "accumulate launch");
}

nnb_status nnb_maxpool2d_fwd(void* stream, size_t N, size_t C, size_t H, size_t W, size_t kernel, size_t stride,
		const float* x, float* y, uint32_t* argmax) {
	if (kernel == 0 || stride == 0 || kernel > H || kernel > W) return nnb::fail(NNB_ERR_SHAPE, "maxpool2d: bad window");
	if ((unsigned long long)H * W > 0xffffffffull) return nnb::fail(NNB_ERR_SHAPE, "maxpool2d: plane too large");
	const long long ho = (long long)(H - kernel) / stride + 1, wo = (long long)(W - kernel) / stride + 1;
	const long long planes = (long long)N * C;
	if (planes == 0) return NNB_OK;
	if (!x || !y || !argmax) return nnb::fail(NNB_ERR_INVALID, "maxpool2d_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	NNB_LAUNCH(kTraceRowwise, grid_for(planes * ho * wo, 256), 256, nnb::maxpool_fwd_kernel, planes, (int)H, (int)W,
		(int)kernel, (int)stride, (int)ho, (int)wo, x, y, argmax);
	return nnb::cuda_status(cudaGetLastError(), "maxpool2d_fwd launch");
}

nnb_status nnb_maxpool2d_bwd(void* stream, size_t N, size_t C, size_t H, size_t W, size_t kernel, size_t stride,
		const float* g, const uint32_t* argmax, float* dx, int dx_first) {
	if (kernel == 0 || stride == 0 || kernel > H || kernel > W) return nnb::fail(NNB_ERR_SHAPE, "maxpool2d: bad window");
	const long long ho = (long long)(H - kernel) / stride + 1, wo = (long long)(W - kernel) / stride + 1;
	const long long planes = (long long)N * C;
	if (planes == 0) return NNB_OK;
	if (!g || !argmax || !dx) return nnb::fail(NNB_ERR_INVALID, "maxpool2d_bwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	NNB_LAUNCH(kTraceRowwise, grid_for(planes * H * W, 256), 256, nnb::maxpool_bwd_kernel, planes, (int)H, (int)W,
		(int)kernel, (int)stride, (int)ho, (int)wo, g, argmax, dx, dx_first);
	return nnb::cuda_status(cudaGetLastError(), "maxpool2d_bwd launch");
}

nnb_status nnb_avgpool2d_fwd(void* stream, size_t N, size_t C, size_t H, size_t W, size_t kernel, size_t stride,
		const float* x, float* y) {
	if (kernel == 0 || stride == 0 || kernel > H || kernel > W) return nnb::fail(NNB_ERR_SHAPE, "avgpool2d: bad window");
	const long long ho = (long long)(H - kernel) / stride + 1, wo = (long long)(W - kernel) / stride + 1;
	const long long planes = (long long)N * C;
	if (planes == 0) return NNB_OK;
	if (!x || !y) return nnb::fail(NNB_ERR_INVALID, "avgpool2d_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const float inv_area = 1.0f / static_cast<float>(kernel * kernel);      // ops.cpp:1727
	NNB_LAUNCH(kTraceRowwise, grid_for(planes * ho * wo, 256), 256, nnb::avgpool_fwd_kernel, planes, (int)H, (int)W,
		(int)kernel, (int)stride, (int)ho, (int)wo, inv_area, x, y);
	return nnb::cuda_status(cudaGetLastError(), "avgpool2d_fwd launch");
}

nnb_status nnb_avgpool2d_bwd(void* stream, size_t N, size_t C, size_t H, size_t W, size_t kernel, size_t stride,
		const float* g, float* dx, int dx_first) {
	if (kernel == 0 || stride == 0 || kernel > H || kernel > W) return nnb::fail(NNB_ERR_SHAPE, "avgpool2d: bad window");
	const long long ho = (long long)(H - kernel) / stride + 1, wo = (long long)(W - kernel) / stride + 1;
	const long long planes = (long long)N * C;
	if (planes == 0) return NNB_OK;
	if (!g || !dx) return nnb::fail(NNB_ERR_INVALID, "avgpool2d_bwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const float inv_area = 1.0f / static_cast<float>(kernel * kernel);
	NNB_LAUNCH(kTraceRowwise, grid_for(planes * H * W, 256), 256, nnb::avgpool_bwd_kernel, planes, (int)H, (int)W,
		(int)kernel, (int)stride, (int)ho, (int)wo, inv_area, g, dx, dx_first);
	return nnb::cuda_status(cudaGetLastError(), "avgpool2d_bwd launch");
}

nnb_status nnb_reduce_axis_fwd(void* stream, size_t outer, size_t n, size_t inner, const float* x, int average,
		float* y) {
	if (n == 0) return nnb::fail(NNB_ERR_SHAPE, "reduce_axis: empty axis");
	if (outer == 0 || inner == 0) return NNB_OK;
	if (!x || !y) return nnb::fail(NNB_ERR_INVALID, "reduce_axis_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const float factor = average ? 1.0f / static_cast<float>(n) : 1.0f;   // ops.cpp:300
	NNB_LAUNCH(kTraceRowwise, grid_for((long long)(outer * inner), 256), 256, nnb::reduce_axis_fwd_kernel,
		(long long)outer, (long long)n, (long long)inner, x, average, factor, y);
	return nnb::cuda_status(cudaGetLastError(), "reduce_axis_fwd launch");
}

nnb_status nnb_reduce_axis_bwd(void* stream, size_t outer, size_t n, size_t inner, const float* g, int average,
		float* dx, int dx_first) {
	if (n == 0) return nnb::fail(NNB_ERR_SHAPE, "reduce_axis: empty axis");
	if (outer == 0 || inner == 0) return NNB_OK;
	if (!g || !dx) return nnb::fail(NNB_ERR_INVALID, "reduce_axis_bwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const float factor = average ? 1.0f / static_cast<float>(n) : 1.0f;
	NNB_LAUNCH(kTraceRowwise, grid_for((long long)(outer * inner), 256), 256, nnb::reduce_axis_bwd_kernel,
		(long long)outer, (long long)n, (long long)inner, g, factor, dx, dx_first);
	return nnb::cuda_status(cudaGetLastError(), "reduce_axis_bwd launch");
}

// Shared body of the two cross-entropy forwards. `scratch` must hold rows floats + rows ints.
static nnb_status ce_forward(cudaStream_t s, long long rows, int C, const float* logits, const int64_t* targets,
		int64_t ignore_index, int use_ignore, float ls, int as_double, float* softmax, float* loss, float* norm) {
	nnb::DeviceState* dev = nullptr;
	NNB_TRY(nnb::device_state(&dev));
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, rows * (sizeof(float) + sizeof(int)), s));
	float* row_loss = static_cast<float*>(ws);
	int* valid = reinterpret_cast<int*>(row_loss + rows);
	const long long threads = rows * 32;
	if (C > 1024 && C <= 4 * nnb::kCeBlock * nnb::kCeV4 && rows <= 0x7fffffffLL && nnb::vec4_ok(C, logits, softmax))
		NNB_LAUNCH(kTraceRowwise, (unsigned)rows, nnb::kCeBlock, nnb::ce_rows_block_kernel, rows, C, logits, targets,
			ignore_index, use_ignore, ls, softmax, row_loss, valid, dev->error_word);
	else
		NNB_LAUNCH(kTraceRowwise, (unsigned)((threads + 255) / 256), 256, nnb::ce_rows_kernel, rows, C, logits, targets,
			ignore_index, use_ignore, ls, softmax, row_loss, valid, dev->error_word);
	NNB_LAUNCH(kTraceRowwise, 1, 256, nnb::ce_total_kernel, rows, row_loss, valid, as_double, loss, norm);
	nnb_status st = nnb::cuda_status(cudaGetLastError(), "cross entropy launch");
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

nnb_status nnb_cross_entropy_fwd(void* stream, size_t N, size_t C, const float* logits, const int64_t* targets,
		float* softmax, float* loss, float* norm) {
	if (N == 0 || C == 0) return nnb::fail(NNB_ERR_SHAPE, "cross_entropy: empty logits");
	if (!logits || !targets || !softmax || !loss || !norm) return nnb::fail(NNB_ERR_INVALID, "cross_entropy_fwd: null pointer");
	return ce_forward(static_cast<cudaStream_t>(stream), (long long)N, (int)C, logits, targets, 0, 0, 0.0f, 0, softmax,
		loss, norm);
}

nnb_status nnb_cross_entropy_bwd(void* stream, size_t N, size_t C, const float* softmax, const int64_t* targets,
		const float* grad_loss, const float* norm, float* dlogits, int first) {
	if (N == 0 || C == 0) return NNB_OK;
	if (!softmax || !targets || !grad_loss || !norm || !dlogits)
		return nnb::fail(NNB_ERR_INVALID, "cross_entropy_bwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long n = (long long)N * C;
	if (nnb::vec4_ok(n, softmax, dlogits) && C % 4 == 0)
		NNB_LAUNCH(kTraceRowwise, nnb::grid_for(n / 4, 256), 256, nnb::ce_bwd_vec_kernel, n / 4, (int)C, softmax, targets, 0,
			0, 0.0f, grad_loss, norm, dlogits, first);
	else
		NNB_LAUNCH(kTraceRowwise, nnb::ce_bwd_grid((long long)N, (int)C), 256, nnb::ce_bwd_kernel, (long long)N, (int)C,
			softmax, targets, 0, 0, 0.0f, grad_loss, norm, dlogits, first);
	return nnb::cuda_status(cudaGetLastError(), "cross_entropy_bwd launch");
}

nnb_status nnb_sequence_ce_fwd(void* stream, size_t P, size_t V, const float* logits, const int64_t* targets,
		int64_t ignore_index, float label_smoothing, float* softmax, float* loss, float* norm) {
	if (P == 0 || V == 0) return nnb::fail(NNB_ERR_SHAPE, "sequence_cross_entropy: empty logits");
	if (!(label_smoothing >= 0.0f && label_smoothing < 1.0f))
		return nnb::fail(NNB_ERR_INVALID, "sequence_cross_entropy: label_smoothing must be in [0, 1)");
	if (!logits || !targets || !softmax || !loss || !norm) return nnb::fail(NNB_ERR_INVALID, "sequence_ce_fwd: null pointer");
	return ce_forward(static_cast<cudaStream_t>(stream), (long long)P, (int)V, logits, targets, ignore_index, 1,
		label_smoothing, 1, softmax, loss, norm);
}

nnb_status nnb_sequence_ce_bwd(void* stream, size_t P, size_t V, const float* softmax, const int64_t* targets,
		int64_t ignore_index, float label_smoothing, const float* grad_loss, const float* norm, float* dlogits,
		int first) {
	if (P == 0 || V == 0) return NNB_OK;
	if (!softmax || !targets || !grad_loss || !norm || !dlogits)
		return nnb::fail(NNB_ERR_INVALID, "sequence_ce_bwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long n = (long long)P * V;
	if (nnb::vec4_ok(n, softmax, dlogits) && V % 4 == 0)
		NNB_LAUNCH(kTraceRowwise, nnb::grid_for(n / 4, 256), 256, nnb::ce_bwd_vec_kernel, n / 4, (int)V, softmax, targets,
			ignore_index, 1, label_smoothing, grad_loss, norm, dlogits, first);
	else
		NNB_LAUNCH(kTraceRowwise, nnb::ce_bwd_grid((long long)P, (int)V), 256, nnb::ce_bwd_kernel, (long long)P, (int)V,
			softmax, targets, ignore_index, 1, label_smoothing, grad_loss, norm, dlogits, first);
	return nnb::cuda_status(cudaGetLastError(), "sequence_ce_bwd launch");
}

nnb_status nnb_embedding_fwd(void* stream, size_t V, size_t D, const float* weight, const int64_t* ids, size_t count,
		float* out) {
	if (count == 0 || D == 0) return NNB_OK;
	if (!weight || !ids || !out) return nnb::fail(NNB_ERR_INVALID, "embedding_fwd: null pointer");
	nnb::DeviceState* dev = nullptr;
	NNB_TRY(nnb::device_state(&dev));
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	NNB_LAUNCH(kTraceRowwise, grid_for((long long)count * D, 256), 256, nnb::embedding_fwd_kernel, (long long)count,
		(int)V, (int)D, weight, ids, out, dev->error_word);
	return nnb::cuda_status(cudaGetLastError(), "embedding_fwd launch");
}

nnb_status nnb_embedding_bwd(void* stream, size_t V, size_t D, const int64_t* ids, size_t count, const float* g,
		float* dweight, int first) {
	if (D == 0 || V == 0) return NNB_OK;
	if (count == 0) {
		if (first && dweight) NNB_CUDA_TRY(cudaMemsetAsync(dweight, 0, V * D * sizeof(float), static_cast<cudaStream_t>(stream)));
		return NNB_OK;
	}
	if (!ids || !g || !dweight) return nnb::fail(NNB_ERR_INVALID, "embedding_bwd: null pointer");
	if (V > 40000) return nnb::fail(NNB_ERR_UNSUPPORTED, "embedding_bwd: vocabulary above 40000 rows");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long chunks = ((long long)count + nnb::kEmbChunk - 1) / nnb::kEmbChunk;
	const size_t hist_n = (size_t)(chunks * V);
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, (2 * hist_n + V + 1 + count) * sizeof(int), s));
	int* hist = static_cast<int*>(ws);
	int* start = hist + hist_n;
	int* id_begin = start + hist_n;
	int* order = id_begin + V + 1;
	nnb_status st = nnb::cuda_status(cudaMemsetAsync(hist, 0, hist_n * sizeof(int), s), "embedding_bwd memset");
	if (st == NNB_OK) {
		NNB_LAUNCH(kTraceAux, grid_for((long long)count, 256), 256, nnb::embedding_hist_kernel, (long long)count, (int)V,
			ids, hist);
		NNB_LAUNCH(kTraceAux, 1, 1024, nnb::embedding_scan_kernel, (int)V, (int)chunks, hist, start, id_begin);
		{
			nnb::TraceScope ts(s, nnb::kTraceAux);
			nnb::embedding_place_kernel<<<(unsigned)chunks, 256, V * sizeof(int), s>>>((long long)count, (int)V,
				(int)chunks, ids, start, order);
		}
		NNB_LAUNCH(kTraceRowwise, grid_for((long long)V * D, 256), 256, nnb::embedding_bwd_kernel, (int)V, (int)D,
			id_begin, order, g, dweight, first);
		st = nnb::cuda_status(cudaGetLastError(), "embedding_bwd launch");
	}
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

nnb_status nnb_embedding_bwd_grouped(void* stream, size_t V, size_t D, size_t groups, const int64_t* ids, size_t count,
		const float* g, float* dweight, size_t dweight_stride, int first) {
	if (groups == 0 || count % groups != 0)
		return nnb::fail(NNB_ERR_SHAPE, "embedding_bwd_grouped: %zu ids in %zu groups", count, groups);
	const size_t per = count / groups;
	for (size_t z = 0; z < groups; ++z)
		NNB_TRY(nnb_embedding_bwd(stream, V, D, ids + z * per, per, g + z * per * D,
			dweight + z * (dweight_stride ? dweight_stride : V * D), first));
	return NNB_OK;
}

nnb_status nnb_adamw_step(void* stream, size_t n, float* w, const float* g, float* m, float* v, float lr, float beta1,
		float beta2, float eps, float weight_decay, long long step) {
	if (n == 0) return NNB_OK;
	if (!w || !g || !m || !v) return nnb::fail(NNB_ERR_INVALID, "adamw_step: null pointer");
	if (step < 1) return nnb::fail(NNB_ERR_INVALID, "adamw_step: step counts from 1");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	// host scalars exactly as Adam::step computes them (adam.cpp:25-27) and AdamW::step (adamw.cpp:16)
	const float c1 = 1.0f - std::pow(beta1, static_cast<float>(step));
	const float c2 = 1.0f - std::pow(beta2, static_cast<float>(step));
	const float shrink = 1.0f - lr * weight_decay;
	NNB_LAUNCH(kTraceRowwise, grid_for((long long)n, 256), 256, nnb::adamw_kernel, (long long)n, w, g, m, v, shrink, lr,
		beta1, beta2, eps, c1, c2);
	return nnb::cuda_status(cudaGetLastError(), "adamw launch");
}

size_t nnb_adam_bias_table(float beta1, float beta2, float* out, size_t max_len) {
	if (!out || max_len == 0) return 0;
	if (max_len > (size_t(1) << 24)) max_len = size_t(1) << 24;     // t is exact as a float up to 2^24
	size_t len = 0;
	for (size_t t = 1; t <= max_len; ++t) {
		const float c1 = 1.0f - std::pow(beta1, static_cast<float>(t));
		const float c2 = 1.0f - std::pow(beta2, static_cast<float>(t));
		out[2 * (t - 1)] = c1;
		out[2 * (t - 1) + 1] = c2;
		len = t;
		if (c1 == 1.0f && c2 == 1.0f) break;       // both saturated: every later step has these values
	}
	return len;
}

nnb_status nnb_step_advance(void* stream, int64_t* step) {
	if (!step) return nnb::fail(NNB_ERR_INVALID, "step_advance: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	NNB_LAUNCH(kTraceAux, 1, 32, nnb::step_advance_kernel, step);
	return nnb::cuda_status(cudaGetLastError(), "step_advance launch");
}

nnb_status nnb_adamw_step_device(void* stream, size_t n, float* w, const float* g, float* m, float* v,
		const float* hyper, const float* bias_table, size_t table_len, const int64_t* step) {
	if (n == 0) return NNB_OK;
	if (!w || !g || !m || !v || !hyper || !bias_table || !step || table_len == 0)
		return nnb::fail(NNB_ERR_INVALID, "adamw_step_device: null pointer or empty table");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	NNB_LAUNCH(kTraceRowwise, grid_for((long long)n, 256), 256, nnb::adamw_device_kernel, (long long)n, w, g, m, v,
		hyper, bias_table, (long long)table_len, step);
	return nnb::cuda_status(cudaGetLastError(), "adamw_device launch");
}

}  // extern "C"
