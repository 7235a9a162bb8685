// ops_norm.cu -- `layernorm` (src/autograd/ops.cpp:1003-1078) and training-mode `batchnorm`
// (ops.cpp:900-1001), forward and backward.
//
// LayerNorm: one warp per row. Each lane sums a strided slice of the row serially and a fixed
// xor-shuffle tree combines the 32 partials, so every lane holds the same bits and the result
// depends only on D. mean and 1/std are kept per row for the backward pass, as the reference
// keeps them. dgamma/dbeta are column sums over rows in the fixed chunked order of
// ops_linear.cu (serial within 256-row chunks, then over chunks).
//
// BatchNorm: the reference's statistics are reproduced bit for bit: per (sample, channel) an
// 8-lane fp32 partial sum over the plane (lane_sum / lane_sq / lane_dot, ops.cpp:804-898), then
// per channel an fp64 sum of those partials in sample order; the normalisation, the folded ReLU
// with its 1-byte alive mask, and the backward formulas use the reference's expressions with
// correctly rounded operations only (no FMA contraction).
#include "nnb_internal.h"
#include "nnb_ops.h"
#include "nnb_trace.h"

namespace nnb {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
	for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
	return v;
}

// ---------------------------------------------------------------------------------------------
// LayerNorm
// ---------------------------------------------------------------------------------------------

__global__ void layernorm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
		const float* __restrict__ beta, float eps, long long R, int D, float* __restrict__ y,
		float* __restrict__ mean, float* __restrict__ inv_std) {
	const int lane = threadIdx.x & 31;
	const long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
	if (r >= R) return;
	const float* row = x + r * D;
	float s = 0.0f;
	for (int j = lane; j < D; j += 32) s += row[j];
	s = warp_sum(s);
	const float mu = s / (float)D;
	float q = 0.0f;
	for (int j = lane; j < D; j += 32) {
		const float d = row[j] - mu;
		q += d * d;
	}
	q = warp_sum(q);
	const float inv = 1.0f / sqrtf(q / (float)D + eps);
	float* o = y + r * D;
	for (int j = lane; j < D; j += 32) o[j] = (row[j] - mu) * inv * gamma[j] + beta[j];
	if (lane == 0) {
		mean[r] = mu;
		inv_std[r] = inv;
	}
}

__global__ void layernorm_bwd_dx_kernel(const float* __restrict__ g, const float* __restrict__ x,
		const float* __restrict__ gamma, const float* __restrict__ mean, const float* __restrict__ inv_std,
		long long R, int D, float* __restrict__ dx, int first) {
	const int lane = threadIdx.x & 31;
	const long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
	if (r >= R) return;
	const float mu = mean[r], inv = inv_std[r];
	const float* gr = g + r * D;
	const float* xr = x + r * D;
	float a = 0.0f, b = 0.0f;
	for (int j = lane; j < D; j += 32) {
		const float dxhat = gr[j] * gamma[j];
		a += dxhat;
		b += dxhat * ((xr[j] - mu) * inv);
	}
	a = warp_sum(a);
	b = warp_sum(b);
	const float k = inv / (float)D, fd = (float)D;
	float* o = dx + r * D;
	for (int j = lane; j < D; j += 32) {
		const float dxhat = gr[j] * gamma[j];
		const float v = k * (fd * dxhat - a - ((xr[j] - mu) * inv) * b);
		o[j] = first ? v + 0.0f : o[j] + v;
	}
}

// Four-per-lane forms for 16-byte aligned rows with D % 4 == 0 and D <= 128 kV: one warp per row as
// above, the row held in registers (read from HBM once) and moved as float4; lane l owns the 16-byte
// groups l, l + 32, ... and sums its elements in order before the same xor-shuffle tree. The
// per-element expressions are those of the scalar kernels; the sums' grouping differs from theirs
// (it is fixed by D, so the results are deterministic).
template <int kV>
__global__ void layernorm_fwd_vec_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
		const float* __restrict__ beta, float eps, long long R, int D, float* __restrict__ y,
		float* __restrict__ mean, float* __restrict__ inv_std) {
	const int lane = threadIdx.x & 31;
	const long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
	if (r >= R) return;
	const int D4 = D >> 2;
	const float4* row = reinterpret_cast<const float4*>(x + r * D);
	float4 v[kV];
	float s = 0.0f;
#pragma unroll
	for (int u = 0; u < kV; ++u) {
		const int j = lane + 32 * u;
		v[u] = j < D4 ? __ldg(row + j) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
		if (j < D4) {
			s += v[u].x;
			s += v[u].y;
			s += v[u].z;
			s += v[u].w;
		}
	}
	s = warp_sum(s);
	const float mu = s / (float)D;
	float q = 0.0f;
#pragma unroll
	for (int u = 0; u < kV; ++u)
		if (lane + 32 * u < D4) {
			const float d0 = v[u].x - mu, d1 = v[u].y - mu, d2 = v[u].z - mu, d3 = v[u].w - mu;
			q += d0 * d0;
			q += d1 * d1;
			q += d2 * d2;
			q += d3 * d3;
		}
	q = warp_sum(q);
	const float inv = 1.0f / sqrtf(q / (float)D + eps);
	float4* o = reinterpret_cast<float4*>(y + r * D);
	const float4* g4 = reinterpret_cast<const float4*>(gamma);
	const float4* b4 = reinterpret_cast<const float4*>(beta);
#pragma unroll
	for (int u = 0; u < kV; ++u) {
		const int j = lane + 32 * u;
		if (j < D4) {
			const float4 gm = __ldg(g4 + j), bt = __ldg(b4 + j);
			o[j] = make_float4((v[u].x - mu) * inv * gm.x + bt.x, (v[u].y - mu) * inv * gm.y + bt.y,
				(v[u].z - mu) * inv * gm.z + bt.z, (v[u].w - mu) * inv * gm.w + bt.w);
		}
	}
	if (lane == 0) {
		mean[r] = mu;
		inv_std[r] = inv;
	}
}

template <int kV>
__global__ void layernorm_bwd_dx_vec_kernel(const float* __restrict__ g, const float* __restrict__ x,
		const float* __restrict__ gamma, const float* __restrict__ mean, const float* __restrict__ inv_std,
		long long R, int D, float* __restrict__ dx, int first) {
	const int lane = threadIdx.x & 31;
	const long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
	if (r >= R) return;
	const int D4 = D >> 2;
	const float mu = mean[r], inv = inv_std[r];
	const float4* gr = reinterpret_cast<const float4*>(g + r * D);
	const float4* xr = reinterpret_cast<const float4*>(x + r * D);
	const float4* g4 = reinterpret_cast<const float4*>(gamma);
	float4 dh[kV], xh[kV];
	float a = 0.0f, b = 0.0f;
#pragma unroll
	for (int u = 0; u < kV; ++u) {
		const int j = lane + 32 * u;
		if (j < D4) {
			const float4 gv = __ldg(gr + j), xv = __ldg(xr + j), gm = __ldg(g4 + j);
			dh[u] = make_float4(gv.x * gm.x, gv.y * gm.y, gv.z * gm.z, gv.w * gm.w);
			xh[u] = make_float4((xv.x - mu) * inv, (xv.y - mu) * inv, (xv.z - mu) * inv, (xv.w - mu) * inv);
			a += dh[u].x;
			b += dh[u].x * xh[u].x;
			a += dh[u].y;
			b += dh[u].y * xh[u].y;
			a += dh[u].z;
			b += dh[u].z * xh[u].z;
			a += dh[u].w;
			b += dh[u].w * xh[u].w;
		}
	}
	a = warp_sum(a);
	b = warp_sum(b);
	const float k = inv / (float)D, fd = (float)D;
	float4* o = reinterpret_cast<float4*>(dx + r * D);
#pragma unroll
	for (int u = 0; u < kV; ++u) {
		const int j = lane + 32 * u;
		if (j < D4) {
			float4 v = make_float4(k * (fd * dh[u].x - a - xh[u].x * b), k * (fd * dh[u].y - a - xh[u].y * b),
				k * (fd * dh[u].z - a - xh[u].z * b), k * (fd * dh[u].w - a - xh[u].w * b));
			if (first) {
				v = make_float4(v.x + 0.0f, v.y + 0.0f, v.z + 0.0f, v.w + 0.0f);
			} else {
				const float4 c = o[j];
				v = make_float4(c.x + v.x, c.y + v.y, c.z + v.z, c.w + v.w);
			}
			o[j] = v;
		}
	}
}

// Chooses the four-per-lane form (its register count kV) for a row length and pointers; 0: scalar.
inline int layernorm_vec_width(int D, const void* p0, const void* p1, const void* p2, const void* p3) {
	const uintptr_t m = reinterpret_cast<uintptr_t>(p0) | reinterpret_cast<uintptr_t>(p1) |
		reinterpret_cast<uintptr_t>(p2) | reinterpret_cast<uintptr_t>(p3);
	if (D % 4 != 0 || (m & 15) != 0 || D > 1024) return 0;
	const int d4 = D / 4;
	return d4 <= 32 ? 1 : d4 <= 64 ? 2 : d4 <= 128 ? 4 : 8;
}

constexpr int kChunk = 256;

// Chunk partials of sum_r g*xhat (dgamma) and sum_r g (dbeta), serial within the chunk; group z
// (blockIdx.z) covers rows [z*R, (z+1)*R).
__global__ void layernorm_bwd_param_partial(const float* __restrict__ g, const float* __restrict__ x,
		const float* __restrict__ mean, const float* __restrict__ inv_std, long long R, int D,
		float* __restrict__ pg, float* __restrict__ pb) {
	const int j = blockIdx.x * blockDim.x + threadIdx.x;
	const long long c = blockIdx.y, chunks = gridDim.y, z = blockIdx.z;
	if (j >= D) return;
	const long long base = z * R;
	const long long r0 = base + c * kChunk, r1 = base + min(R, (c + 1) * kChunk);
	// serial in row order, with 16 rows' loads issued ahead of their adds
	float sg = 0.0f, sb = 0.0f;
	long long r = r0;
	for (; r + 16 <= r1; r += 16) {
		float gv[16], xv[16], mv[16], iv[16];
#pragma unroll
		for (int u = 0; u < 16; ++u) {
			gv[u] = __ldg(g + (r + u) * D + j);
			xv[u] = __ldg(x + (r + u) * D + j);
			mv[u] = __ldg(mean + r + u);
			iv[u] = __ldg(inv_std + r + u);
		}
#pragma unroll
		for (int u = 0; u < 16; ++u) {
			sg += gv[u] * ((xv[u] - mv[u]) * iv[u]);
			sb += gv[u];
		}
	}
	for (; r < r1; ++r) {
		const float gv = g[r * D + j];
		sg += gv * ((x[r * D + j] - mean[r]) * inv_std[r]);
		sb += gv;
	}
	pg[(z * chunks + c) * D + j] = sg;
	pb[(z * chunks + c) * D + j] = sb;
}

// The same partials with the chunk staged in shared memory (256 threads keep every load in flight),
// then warp 0 accumulates each column serially in row order: the additions and their order are those
// of layernorm_bwd_param_partial.
__global__ void __launch_bounds__(256) layernorm_bwd_param_partial_staged(const float* __restrict__ g,
		const float* __restrict__ x, const float* __restrict__ mean, const float* __restrict__ inv_std, long long R, int D,
		float* __restrict__ pg, float* __restrict__ pb) {
	constexpr int kPass = kChunk / 2;                // rows staged at a time (shared memory < 48 KB)
	__shared__ __align__(16) float tg[kPass][32], tx[kPass][32];
	__shared__ float tm[kPass], ti[kPass];
	const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
	const int j = blockIdx.x * 32 + lane;
	const long long c = blockIdx.y, chunks = gridDim.y, z = blockIdx.z;
	const long long r0 = z * R + c * kChunk;
	const int n = (int)min(R - c * kChunk, (long long)kChunk);
	float sg = 0.0f, sb = 0.0f;
	for (int p0 = 0; p0 < n; p0 += kPass) {
		const int m = min(kPass, n - p0);
		const int j0 = blockIdx.x * 32;
		if (m == kPass && j0 + 32 <= D && D % 4 == 0 &&
				((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(x)) & 15) == 0) {
			// a whole pass of 32 full columns: every thread's 16-byte loads issued before any store
			constexpr int kLoads = kPass * 32 / 4 / 256;
			const int c4 = (threadIdx.x & 7) * 4, rq = threadIdx.x >> 3;
			float4 vg[kLoads], vx[kLoads];
#pragma unroll
			for (int u = 0; u < kLoads; ++u) {
				const long long off = (r0 + p0 + rq + 32 * u) * D + j0 + c4;
				vg[u] = __ldg(reinterpret_cast<const float4*>(g + off));
				vx[u] = __ldg(reinterpret_cast<const float4*>(x + off));
			}
#pragma unroll
			for (int u = 0; u < kLoads; ++u) {
				*reinterpret_cast<float4*>(&tg[rq + 32 * u][c4]) = vg[u];
				*reinterpret_cast<float4*>(&tx[rq + 32 * u][c4]) = vx[u];
			}
		} else {
			for (int rr = warp; rr < m; rr += 8) {
				tg[rr][lane] = j < D ? __ldg(g + (r0 + p0 + rr) * D + j) : 0.0f;
				tx[rr][lane] = j < D ? __ldg(x + (r0 + p0 + rr) * D + j) : 0.0f;
			}
		}
		for (int rr = threadIdx.x; rr < m; rr += 256) {
			tm[rr] = __ldg(mean + r0 + p0 + rr);
			ti[rr] = __ldg(inv_std + r0 + p0 + rr);
		}
		__syncthreads();
		if (warp == 0) {                              // serial in row order, continuing across the passes
			for (int rr = 0; rr < m; ++rr) {
				const float gv = tg[rr][lane];
				sg += gv * ((tx[rr][lane] - tm[rr]) * ti[rr]);
				sb += gv;
			}
		}
		__syncthreads();                              // the pass is read before the next one is written
	}
	if (warp != 0 || j >= D) return;
	pg[(z * chunks + c) * D + j] = sg;
	pb[(z * chunks + c) * D + j] = sb;
}

__global__ void layernorm_bwd_param_final(const float* __restrict__ pg, const float* __restrict__ pb,
		long long chunks, int D, float* __restrict__ dgamma, long long dg_stride, int dg_first,
		float* __restrict__ dbeta, long long db_stride, int db_first) {
	const int j = blockIdx.x * blockDim.x + threadIdx.x;
	const long long z = blockIdx.y;
	if (j >= D) return;
	float sg = 0.0f, sb = 0.0f;
	for (long long c = 0; c < chunks; ++c) {
		sg += pg[(z * chunks + c) * D + j];
		sb += pb[(z * chunks + c) * D + j];
	}
	if (dgamma) dgamma[z * dg_stride + j] = dg_first ? sg + 0.0f : dgamma[z * dg_stride + j] + sg;
	if (dbeta) dbeta[z * db_stride + j] = db_first ? sb + 0.0f : dbeta[z * db_stride + j] + sb;
}

// ---------------------------------------------------------------------------------------------
// BatchNorm (training statistics)
// ---------------------------------------------------------------------------------------------

// ops.cpp:804-812
__device__ __forceinline__ float lane_sum(const float* p, long long n) {
	float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
	long long i = 0;
	for (; i + 8 <= n; i += 8)
#pragma unroll
		for (int k = 0; k < 8; ++k) a[k] += p[i + k];
	float t = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
	for (; i < n; ++i) t += p[i];
	return t;
}

// ops.cpp:824-835
__device__ __forceinline__ float lane_sq(const float* p, long long n, float mu) {
	float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
	long long i = 0;
	for (; i + 8 <= n; i += 8)
#pragma unroll
		for (int k = 0; k < 8; ++k) {
			const float d = p[i + k] - mu;
			a[k] += d * d;
		}
	float t = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
	for (; i < n; ++i) t += (p[i] - mu) * (p[i] - mu);
	return t;
}

// lane_sum of g (masked by `alive` when given) and lane_dot of g with (x - mu): ops.cpp:848-898
__device__ __forceinline__ void lane_sum_dot(const float* g, const unsigned char* alive, const float* x,
		long long n, float mu, float& sum_out, float& dot_out) {
	float a[8] = {0, 0, 0, 0, 0, 0, 0, 0}, b[8] = {0, 0, 0, 0, 0, 0, 0, 0};
	long long i = 0;
	for (; i + 8 <= n; i += 8)
#pragma unroll
		for (int k = 0; k < 8; ++k) {
			const float gv = alive ? (alive[i + k] ? g[i + k] : 0.0f) : g[i + k];
			a[k] += gv;
			b[k] += gv * (x[i + k] - mu);
		}
	float t = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
	float u = ((b[0] + b[1]) + (b[2] + b[3])) + ((b[4] + b[5]) + (b[6] + b[7]));
	for (; i < n; ++i) {
		const float gv = alive ? (alive[i] ? g[i] : 0.0f) : g[i];
		t += gv;
		u += gv * (x[i] - mu);
	}
	sum_out = t;
	dot_out = u;
}

// part[n*C + c] = lane_sum (pass 0) or lane_sq around mean[c] (pass 1) of plane (n, c)
__global__ void bn_plane_kernel(const float* __restrict__ x, long long N, long long C, long long S,
		const float* __restrict__ mean, int pass, float* __restrict__ part) {
	const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
	if (idx >= N * C) return;
	const long long c = idx % C;
	const float* p = x + idx * S;
	part[idx] = pass == 0 ? lane_sum(p, S) : lane_sq(p, S, mean[c]);
}

// per channel: double sum of the plane partials in sample order; pass 0 -> mean, pass 1 -> var, inv_std
__global__ void bn_channel_kernel(const float* __restrict__ part, long long N, long long C, long long M,
		float eps, int pass, float* __restrict__ mean, float* __restrict__ var, float* __restrict__ inv_std) {
	const long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x;
	if (c >= C) return;
	double s = 0.0;
	for (long long n = 0; n < N; ++n) s += (double)part[n * C + c];
	const float v = (float)(s / (double)M);
	if (pass == 0) {
		mean[c] = v;
	} else {
		var[c] = v;
		inv_std[c] = 1.0f / sqrtf(v + eps);
	}
}

__global__ void bn_apply_kernel(const float* __restrict__ x, long long N, long long C, long long S,
		const float* __restrict__ w, const float* __restrict__ b, const float* __restrict__ mean,
		const float* __restrict__ inv_std, float* __restrict__ y, unsigned char* __restrict__ alive) {
	const long long total = N * C * S;
	for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
			i += (long long)gridDim.x * blockDim.x) {
		const long long c = (i / S) % C;
		const float scale = w[c] * inv_std[c];
		const float v = (x[i] - mean[c]) * scale + b[c];
		if (alive) {
			alive[i] = v > 0.0f;
			y[i] = v > 0.0f ? v : 0.0f;
		} else {
			y[i] = v;
		}
	}
}

__global__ void bn_bwd_plane_kernel(const float* __restrict__ g, const unsigned char* __restrict__ alive,
		const float* __restrict__ x, long long N, long long C, long long S, const float* __restrict__ mean,
		float* __restrict__ psum, float* __restrict__ pdot) {
	const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
	if (idx >= N * C) return;
	const long long c = idx % C, base = idx * S;
	float su, du;
	lane_sum_dot(g + base, alive ? alive + base : nullptr, x + base, S, mean[c], su, du);
	psum[idx] = su;
	pdot[idx] = du;
}

// per channel: sdy, sdg in fp64 (sample order); db/dw update; scalars for the dx pass
__global__ void bn_bwd_channel_kernel(const float* __restrict__ psum, const float* __restrict__ pdot,
		long long N, long long C, const float* __restrict__ inv_std, float* __restrict__ dw, int dw_first,
		float* __restrict__ db, int db_first, float* __restrict__ a_out, float* __restrict__ b_out) {
	const long long c = blockIdx.x * (long long)blockDim.x + threadIdx.x;
	if (c >= C) return;
	double sdy = 0.0, sdg = 0.0;
	for (long long n = 0; n < N; ++n) {
		sdy += (double)psum[n * C + c];
		sdg += (double)pdot[n * C + c];
	}
	const double sdyx = sdg * (double)inv_std[c];
	if (db) db[c] = db_first ? (float)sdy + 0.0f : db[c] + (float)sdy;
	if (dw) dw[c] = dw_first ? (float)sdyx + 0.0f : dw[c] + (float)sdyx;
	a_out[c] = (float)sdy;
	b_out[c] = (float)sdyx;
}

__global__ void bn_bwd_dx_kernel(const float* __restrict__ g, const unsigned char* __restrict__ alive,
		const float* __restrict__ x, long long N, long long C, long long S, const float* __restrict__ w,
		const float* __restrict__ mean, const float* __restrict__ inv_std, const float* __restrict__ a_c,
		const float* __restrict__ b_c, float* __restrict__ dx, int first) {
	const long long total = N * C * S;
	const float fm = (float)(N * S);
	for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
			i += (long long)gridDim.x * blockDim.x) {
		const long long c = (i / S) % C;
		const float mu = mean[c], inv = inv_std[c];
		const float k = w[c] * inv / fm;
		const float gv = alive ? (alive[i] ? g[i] : 0.0f) : g[i];
		const float v = k * (fm * gv - a_c[c] - ((x[i] - mu) * inv) * b_c[c]);
		dx[i] = first ? v + 0.0f : dx[i] + v;
	}
}

}  // namespace

}  // namespace nnb

extern "C" {

nnb_status nnb_layernorm_fwd(void* stream, size_t R, size_t D, const float* x, const float* gamma,
		const float* beta, float eps, float* y, float* mean, float* inv_std) {
	if (R == 0) return NNB_OK;
	if (D == 0) return nnb::fail(NNB_ERR_SHAPE, "layernorm: empty rows");
	if (!x || !gamma || !beta || !y || !mean || !inv_std) return nnb::fail(NNB_ERR_INVALID, "layernorm_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long threads = (long long)R * 32;
	nnb::TraceScope ts(s, nnb::kTraceRowwise);
	const unsigned blocks = (unsigned)((threads + 255) / 256);
	switch (nnb::layernorm_vec_width((int)D, x, y, gamma, beta)) {
	case 1: nnb::layernorm_fwd_vec_kernel<1><<<blocks, 256, 0, s>>>(x, gamma, beta, eps, (long long)R, (int)D, y, mean, inv_std); break;
	case 2: nnb::layernorm_fwd_vec_kernel<2><<<blocks, 256, 0, s>>>(x, gamma, beta, eps, (long long)R, (int)D, y, mean, inv_std); break;
	case 4: nnb::layernorm_fwd_vec_kernel<4><<<blocks, 256, 0, s>>>(x, gamma, beta, eps, (long long)R, (int)D, y, mean, inv_std); break;
	case 8: nnb::layernorm_fwd_vec_kernel<8><<<blocks, 256, 0, s>>>(x, gamma, beta, eps, (long long)R, (int)D, y, mean, inv_std); break;
	default:
		nnb::layernorm_fwd_kernel<<<blocks, 256, 0, s>>>(x, gamma, beta, eps, (long long)R, (int)D, y, mean, inv_std);
	}
	return nnb::cuda_status(cudaGetLastError(), "layernorm_fwd launch");
}

nnb_status nnb_layernorm_bwd_grouped(void* stream, size_t R, size_t D, size_t groups, const float* g, const float* x,
		const float* gamma, const float* mean, const float* inv_std, float* dx, int dx_first, float* dgamma,
		size_t dgamma_stride, int dgamma_first, float* dbeta, size_t dbeta_stride, int dbeta_first) {
	if (R == 0 || D == 0) return NNB_OK;
	if (!g || !x || !gamma || !mean || !inv_std) return nnb::fail(NNB_ERR_INVALID, "layernorm_bwd: null input");
	if (groups == 0 || R % groups != 0) return nnb::fail(NNB_ERR_SHAPE, "layernorm_bwd: %zu rows in %zu groups", R, groups);
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	if (dx) {
		const long long threads = (long long)R * 32;
		nnb::TraceScope ts(s, nnb::kTraceRowwise);
		const unsigned blocks = (unsigned)((threads + 255) / 256);
		const int vw = nnb::layernorm_vec_width((int)D, g, x, gamma, dx);
		if (vw == 1)
			nnb::layernorm_bwd_dx_vec_kernel<1><<<blocks, 256, 0, s>>>(g, x, gamma, mean, inv_std, (long long)R, (int)D, dx, dx_first);
		else if (vw == 2)
			nnb::layernorm_bwd_dx_vec_kernel<2><<<blocks, 256, 0, s>>>(g, x, gamma, mean, inv_std, (long long)R, (int)D, dx, dx_first);
		else if (vw == 4)
			nnb::layernorm_bwd_dx_vec_kernel<4><<<blocks, 256, 0, s>>>(g, x, gamma, mean, inv_std, (long long)R, (int)D, dx, dx_first);
		else if (vw == 8)
			nnb::layernorm_bwd_dx_vec_kernel<8><<<blocks, 256, 0, s>>>(g, x, gamma, mean, inv_std, (long long)R, (int)D, dx, dx_first);
		else
			nnb::layernorm_bwd_dx_kernel<<<blocks, 256, 0, s>>>(g, x, gamma, mean, inv_std, (long long)R, (int)D, dx,
				dx_first);
		NNB_CUDA_TRY(cudaGetLastError());
	}
	if (dgamma || dbeta) {
		const long long Rg = (long long)(R / groups);
		const long long chunks = (Rg + nnb::kChunk - 1) / nnb::kChunk;
		if (chunks > 65535 || groups > 65535) return nnb::fail(NNB_ERR_UNSUPPORTED, "layernorm_bwd: too many rows");
		void* ws = nullptr;
		NNB_TRY(nnb::scratch_alloc(&ws, 2 * groups * chunks * D * sizeof(float), s));
		float* pg = static_cast<float*>(ws);
		float* pb = pg + groups * chunks * D;
		// 32 columns per block (the chunking, and so every sum's order, depends only on the rows)
		const unsigned bx = (unsigned)((D + 31) / 32);
		{
			nnb::TraceScope ts(s, nnb::kTraceRowwise);
			if (Rg >= 64)           // tall sums: chunk staged in shared memory (same order, loads in flight)
				nnb::layernorm_bwd_param_partial_staged<<<dim3(bx, (unsigned)chunks, (unsigned)groups), 256, 0, s>>>(g, x,
					mean, inv_std, Rg, (int)D, pg, pb);
			else
				nnb::layernorm_bwd_param_partial<<<dim3(bx, (unsigned)chunks, (unsigned)groups), 32, 0, s>>>(g, x, mean,
					inv_std, Rg, (int)D, pg, pb);
		}
		{
			nnb::TraceScope ts(s, nnb::kTraceRowwise);
			nnb::layernorm_bwd_param_final<<<dim3(bx, (unsigned)groups), 32, 0, s>>>(pg, pb, chunks, (int)D, dgamma,
				dgamma_stride ? (long long)dgamma_stride : (long long)D, dgamma_first, dbeta,
				dbeta_stride ? (long long)dbeta_stride : (long long)D, dbeta_first);
		}
		nnb_status st = nnb::cuda_status(cudaGetLastError(), "layernorm_bwd launch");
		nnb_status st2 = nnb::scratch_free(ws, s);
		NNB_TRY(st);
		NNB_TRY(st2);
	}
	return NNB_OK;
}

nnb_status nnb_layernorm_bwd(void* stream, size_t R, size_t D, const float* g, const float* x, const float* gamma,
		const float* mean, const float* inv_std, float* dx, int dx_first, float* dgamma, int dgamma_first,
		float* dbeta, int dbeta_first) {
	return nnb_layernorm_bwd_grouped(stream, R, D, 1, g, x, gamma, mean, inv_std, dx, dx_first, dgamma, D, dgamma_first,
		dbeta, D, dbeta_first);
}

nnb_status nnb_batchnorm_fwd(void* stream, size_t N, size_t C, size_t S, const float* x, const float* weight,
		const float* bias, float eps, int fuse_relu, float* y, unsigned char* alive, float* mean, float* var,
		float* inv_std) {
	if (N == 0 || C == 0) return nnb::fail(NNB_ERR_SHAPE, "batchnorm: empty batch or no channels");
	if (!x || !weight || !bias || !y || !mean || !var || !inv_std || (fuse_relu && !alive))
		return nnb::fail(NNB_ERR_INVALID, "batchnorm_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long NC = (long long)N * C, M = (long long)N * S;
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, NC * sizeof(float), s));
	float* part = static_cast<float*>(ws);
	const unsigned gp = (unsigned)((NC + 127) / 128), gc = (unsigned)((C + 127) / 128);
	{
		nnb::TraceScope ts(s, nnb::kTraceRowwise);
		nnb::bn_plane_kernel<<<gp, 128, 0, s>>>(x, N, C, S, nullptr, 0, part);
	}
	{
		nnb::TraceScope ts(s, nnb::kTraceRowwise);
		nnb::bn_channel_kernel<<<gc, 128, 0, s>>>(part, N, C, M, eps, 0, mean, var, inv_std);
	}
	{
		nnb::TraceScope ts(s, nnb::kTraceRowwise);
		nnb::bn_plane_kernel<<<gp, 128, 0, s>>>(x, N, C, S, mean, 1, part);
	}
	{
		nnb::TraceScope ts(s, nnb::kTraceRowwise);
		nnb::bn_channel_kernel<<<gc, 128, 0, s>>>(part, N, C, M, eps, 1, mean, var, inv_std);
	}
	{
		nnb::TraceScope ts(s, nnb::kTraceRowwise);
		nnb::bn_apply_kernel<<<nnb::grid_for(NC * S, 256), 256, 0, s>>>(x, N, C, S, weight, bias, mean, inv_std, y,
			fuse_relu ? alive : nullptr);
	}
	nnb_status st = nnb::cuda_status(cudaGetLastError(), "batchnorm_fwd launch");
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

nnb_status nnb_batchnorm_bwd(void* stream, size_t N, size_t C, size_t S, const float* g, const float* x,
		const float* weight, const float* mean, const float* inv_std, const unsigned char* alive, float* dx,
		int dx_first, float* dweight, int dweight_first, float* dbias, int dbias_first) {
	if (N == 0 || C == 0) return NNB_OK;
	if (!g || !x || !weight || !mean || !inv_std) return nnb::fail(NNB_ERR_INVALID, "batchnorm_bwd: null input");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long NC = (long long)N * C;
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, (2 * NC + 2 * C) * sizeof(float), s));
	float* psum = static_cast<float*>(ws);
	float* pdot = psum + NC;
	float* a_c = pdot + NC;
	float* b_c = a_c + C;
	{
		nnb::TraceScope ts(s, nnb::kTraceRowwise);
		nnb::bn_bwd_plane_kernel<<<(unsigned)((NC + 127) / 128), 128, 0, s>>>(g, alive, x, N, C, S, mean, psum, pdot);
	}
	{
		nnb::TraceScope ts(s, nnb::kTraceRowwise);
		nnb::bn_bwd_channel_kernel<<<(unsigned)((C + 127) / 128), 128, 0, s>>>(psum, pdot, N, C, inv_std, dweight,
			dweight_first, dbias, dbias_first, a_c, b_c);
	}
	if (dx) {
		nnb::TraceScope ts(s, nnb::kTraceRowwise);
		nnb::bn_bwd_dx_kernel<<<nnb::grid_for(NC * S, 256), 256, 0, s>>>(g, alive, x, N, C, S, weight, mean, inv_std,
			a_c, b_c, dx, dx_first);
	}
	nnb_status st = nnb::cuda_status(cudaGetLastError(), "batchnorm_bwd launch");
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// BatchNorm module pieces (src/nn/batchnorm.cpp): the running statistics update after a training
// step, and the evaluation-mode transform built from the running statistics.
// ---------------------------------------------------------------------------------------------
namespace nnb {
namespace {

// batchnorm.cpp:38-47: float arithmetic in the reference's order
__global__ void bn_running_update_kernel(int C, long long n, const float* __restrict__ mean,
		const float* __restrict__ var, float momentum, float* __restrict__ rmean, float* __restrict__ rvar) {
	const int c = blockIdx.x * blockDim.x + threadIdx.x;
	if (c >= C) return;
	rmean[c] = (1.0f - momentum) * rmean[c] + momentum * mean[c];
	if (n > 1) {
		const float unbiased = static_cast<float>(n) / static_cast<float>(n - 1);
		rvar[c] = (1.0f - momentum) * rvar[c] + momentum * var[c] * unbiased;
	}
}

// eval transform (batchnorm.cpp:51-55): inv = 1 / sqrt(rv + eps); y = ((x - rm) * inv) * w + b
__device__ __forceinline__ float bn_eval_inv(const float* rvar, int c, float eps) {
	return 1.0f / sqrtf(rvar[c] + eps);
}

__global__ void bn_eval_fwd_kernel(long long total, long long C, long long S, const float* __restrict__ x,
		const float* __restrict__ rmean, const float* __restrict__ rvar, float eps, const float* __restrict__ w,
		const float* __restrict__ b, int fuse_relu, float* __restrict__ y, unsigned char* __restrict__ alive) {
	for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
		const int c = (int)((i / S) % C);
		const float v = ((x[i] - rmean[c]) * bn_eval_inv(rvar, c, eps)) * w[c] + b[c];
		if (fuse_relu) {
			const bool on = v > 0.0f;
			y[i] = on ? v : 0.0f;
			alive[i] = on ? 1 : 0;
		} else {
			y[i] = v;
		}
	}
}

// dx: the gradient through the reference's op graph add(mul(normed, w), b) then mul(x - mean, inv),
// each node's gradient stored with its +0 (ops.cpp:67-73): g1 = g (0 where the fused ReLU was off),
// dx = ((g1 * w) + 0) * inv + 0, stored (first) or added.
__global__ void bn_eval_dx_kernel(long long total, long long C, long long S, const float* __restrict__ g,
		const unsigned char* __restrict__ alive, const float* __restrict__ rvar, float eps, const float* __restrict__ w,
		float* __restrict__ dx, int first) {
	for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
		const int c = (int)((i / S) % C);
		const float gv = ((alive && !alive[i]) ? 0.0f : g[i]) + 0.0f;
		const float v = ((gv * w[c]) + 0.0f) * bn_eval_inv(rvar, c, eps) + 0.0f;
		dx[i] = first ? v + 0.0f : dx[i] + v;
	}
}

// dweight and dbias: per element terms g1 * normed and g1, reduced to the {1, C, 1, 1} parameter
// shape as the reference's sum_to_shape does it (ops.cpp:35-53): over the sample axis first (one
// sum from 0 for every (c, h, w)), then over h, then over w, each axis only when its size is not 1;
// the result is stored with +0 (first) or added. One block per channel; each thread owns columns
// w = tid, tid + blockDim, ... and the column totals are added in w order by thread 0.
__global__ void bn_eval_param_kernel(long long N, long long C, long long H, long long W, const float* __restrict__ g,
		const unsigned char* __restrict__ alive, const float* __restrict__ x, const float* __restrict__ rmean,
		const float* __restrict__ rvar, float eps, float* __restrict__ dw, int dw_first, float* __restrict__ db,
		int db_first) {
	__shared__ float col_w[256], col_b[256];
	const long long c = blockIdx.x;
	const float inv = bn_eval_inv(rvar, (int)c, eps);
	const float mu = rmean[c];
	float red_w = 0.0f, red_b = 0.0f;
	float one_w = 0.0f, one_b = 0.0f;           // the single column's total when W == 1
	for (long long w0 = 0; w0 < W; w0 += blockDim.x) {
		const long long w = w0 + threadIdx.x;
		if (w < W) {
			float hw = 0.0f, hb = 0.0f;
			for (long long h = 0; h < H; ++h) {
				float nw = 0.0f, nb = 0.0f;
				for (long long n = 0; n < N; ++n) {
					const long long i = ((n * C + c) * H + h) * W + w;
					const float gv = ((alive && !alive[i]) ? 0.0f : g[i]) + 0.0f;
					const float tw = gv * ((x[i] - mu) * inv);
					if (N == 1) { nw = tw; nb = gv; }
					else { nw += tw; nb += gv; }
				}
				if (H == 1) { hw = nw; hb = nb; }
				else { hw += nw; hb += nb; }
			}
			col_w[threadIdx.x] = hw;
			col_b[threadIdx.x] = hb;
		}
		__syncthreads();
		if (threadIdx.x == 0) {
			const long long cnt = min((long long)blockDim.x, W - w0);
			if (W == 1) {
				one_w = col_w[0];
				one_b = col_b[0];
			} else {
				for (long long j = 0; j < cnt; ++j) {
					red_w += col_w[j];
					red_b += col_b[j];
				}
			}
		}
		__syncthreads();
	}
	if (threadIdx.x == 0) {
		const float tw = W == 1 ? one_w : red_w, tb = W == 1 ? one_b : red_b;
		if (dw) dw[c] = dw_first ? tw + 0.0f : dw[c] + (tw + 0.0f);
		if (db) db[c] = db_first ? tb + 0.0f : db[c] + (tb + 0.0f);
	}
}

}  // namespace
}  // namespace nnb

extern "C" {

nnb_status nnb_batchnorm_running_update(void* stream, size_t C, size_t count, const float* mean, const float* var,
		float momentum, float* running_mean, float* running_var) {
	if (C == 0) return NNB_OK;
	if (!mean || !var || !running_mean || !running_var)
		return nnb::fail(NNB_ERR_INVALID, "batchnorm_running_update: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	nnb::TraceScope ts(s, nnb::kTraceRowwise);
	nnb::bn_running_update_kernel<<<(unsigned)((C + 127) / 128), 128, 0, s>>>((int)C, (long long)count, mean, var, momentum,
		running_mean, running_var);
	return nnb::cuda_status(cudaGetLastError(), "batchnorm_running_update launch");
}

nnb_status nnb_batchnorm_eval_fwd(void* stream, size_t N, size_t C, size_t S, const float* x, const float* running_mean,
		const float* running_var, float eps, const float* weight, const float* bias, int fuse_relu, float* y,
		unsigned char* alive) {
	const long long total = (long long)N * C * S;
	if (total == 0) return NNB_OK;
	if (!x || !running_mean || !running_var || !weight || !bias || !y || (fuse_relu && !alive))
		return nnb::fail(NNB_ERR_INVALID, "batchnorm_eval_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	nnb::TraceScope ts(s, nnb::kTraceRowwise);
	nnb::bn_eval_fwd_kernel<<<nnb::grid_for(total, 256), 256, 0, s>>>(total, (long long)C, (long long)S, x, running_mean,
		running_var, eps, weight, bias, fuse_relu, y, alive);
	return nnb::cuda_status(cudaGetLastError(), "batchnorm_eval_fwd launch");
}

nnb_status nnb_batchnorm_eval_bwd(void* stream, size_t N, size_t C, size_t H, size_t W, const float* g,
		const float* x, const float* running_mean, const float* running_var, float eps, const float* weight,
		const unsigned char* alive, float* dx, int dx_first, float* dweight, int dweight_first, float* dbias,
		int dbias_first) {
	const long long S = (long long)H * W;
	const long long total = (long long)N * C * S;
	if (total == 0) return NNB_OK;
	if (!g || !x || !running_mean || !running_var || !weight)
		return nnb::fail(NNB_ERR_INVALID, "batchnorm_eval_bwd: null input");
	if (C > 0x7fffffffLL) return nnb::fail(NNB_ERR_UNSUPPORTED, "batchnorm_eval_bwd: too many channels");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	if (dx) {
		nnb::TraceScope ts(s, nnb::kTraceRowwise);
		nnb::bn_eval_dx_kernel<<<nnb::grid_for(total, 256), 256, 0, s>>>(total, (long long)C, S, g, alive,
			running_var, eps, weight, dx, dx_first);
	}
	if (dweight || dbias) {
		nnb::TraceScope ts(s, nnb::kTraceRowwise);
		nnb::bn_eval_param_kernel<<<(unsigned)C, 256, 0, s>>>((long long)N, (long long)C, (long long)H, (long long)W, g,
			alive, x, running_mean, running_var, eps, dweight, dweight_first, dbias, dbias_first);
	}
	return nnb::cuda_status(cudaGetLastError(), "batchnorm_eval_bwd launch");
}

}  // extern "C"
