// ops_conv.cu -- `conv2d` / `conv2d_relu` (src/autograd/ops.cpp:1345-1472) as im2col + the
// tensor-core GEMM, with the reference's per-sample structure kept where it fixes the order of a sum.
//
// Forward: every sample is unrolled (im2col_sample, ops.cpp:188-212) into col[n] (K x hw,
// K = Cin*kh*kw), then ONE batched GEMM over the samples computes y[n] = W col[n] with the bias
// (per output channel = per row of y[n]) and the folded ReLU + 1-byte alive mask in its epilogue
// (ops.cpp:1395-1408).
// Backward: the gradient masked by `alive`; db per channel = sum over samples, in sample order, of
// the 8-lane sum of the channel's plane (ops.cpp:1441-1442, 1461); dW = sum over samples, in sample
// order, of g[n] col[n]^T (one batched GEMM into per-sample buffers, then an ordered sum,
// ops.cpp:1449, 1462); dX = col2im(W^T g[n]) (ops.cpp:1452-1455), written as a gather that adds each
// input element's contributions in the reference's (kernel row, kernel column) order.
#include "nnb_gemm.h"
#include "nnb_internal.h"
#include "nnb_ops.h"
#include "nnb_trace.h"

namespace nnb {

namespace {

struct Geo {
	int N, Cin, H, W, Cout, kh, kw, stride, pad, ho, wo;
	int dil = 1, groups = 1;
	// im2col rows of all groups together: group g's rows are [g * K/groups, (g+1) * K/groups)
	__host__ __device__ long long K() const { return (long long)Cin * kh * kw; }
	__host__ __device__ long long hw() const { return (long long)ho * wo; }
};

#define GRID_STRIDE(i, n) \
	for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (n); i += (long long)gridDim.x * blockDim.x)

// col[n][(c*kh + ph)*kw + pw][oh*wo + ow] = x[n][c][oh*s + ph - p][ow*s + pw - p] (0 in the padding)
__global__ void im2col_kernel(Geo g, const float* __restrict__ x, float* __restrict__ col) {
	const long long K = g.K(), hw = g.hw();
	GRID_STRIDE(i, (long long)g.N * K * hw) {
		const long long n = i / (K * hw);
		const long long rem = i - n * K * hw;
		const int kr = (int)(rem / hw), o = (int)(rem % hw);
		const int c = kr / (g.kh * g.kw), ph = (kr / g.kw) % g.kh, pw = kr % g.kw;
		const int oh = o / g.wo, ow = o % g.wo;
		const int ih = oh * g.stride + ph * g.dil - g.pad, iw = ow * g.stride + pw * g.dil - g.pad;
		float v = 0.0f;
		if (ih >= 0 && ih < g.H && iw >= 0 && iw < g.W)
			v = x[((n * g.Cin + c) * (long long)g.H + ih) * g.W + iw];
		col[i] = v;
	}
}

// grad_x[n][c][ih][iw] = sum over (ph, pw), in that order, from +0, of dcol[n][(c*kh+ph)*kw+pw][oh*wo+ow]
// for the window position (oh, ow) that reads (ih, iw), if any; then dx = grad_x + 0 (first) or
// dx + grad_x, as the reference builds grad_x and adds it to x.grad() (ops.cpp:1452-1455, 1604)
__global__ void col2im_kernel(Geo g, const float* __restrict__ dcol, float* __restrict__ dx, int first) {
	const long long K = g.K(), hw = g.hw();
	GRID_STRIDE(i, (long long)g.N * g.Cin * g.H * g.W) {
		const long long n = i / ((long long)g.Cin * g.H * g.W);
		const int c = (int)((i / ((long long)g.H * g.W)) % g.Cin);
		const int ih = (int)((i / g.W) % g.H), iw = (int)(i % g.W);
		float acc = 0.0f;
		const float* base = dcol + n * K * hw;
		for (int ph = 0; ph < g.kh; ++ph) {
			const int th = ih + g.pad - ph * g.dil;
			if (th < 0 || th % g.stride != 0) continue;
			const int oh = th / g.stride;
			if (oh >= g.ho) continue;
			for (int pw = 0; pw < g.kw; ++pw) {
				const int tw = iw + g.pad - pw * g.dil;
				if (tw < 0 || tw % g.stride != 0) continue;
				const int ow = tw / g.stride;
				if (ow >= g.wo) continue;
				acc += base[((long long)(c * g.kh + ph) * g.kw + pw) * hw + (long long)oh * g.wo + ow];
			}
		}
		dx[i] = first ? acc + 0.0f : dx[i] + acc;
	}
}

// y[n][c][i] += b[c] after the product, as the general conv path adds its bias (ops.cpp:1556-1557)
__global__ void conv_add_bias_kernel(long long total, long long hw, int Cout, const float* __restrict__ b,
		float* __restrict__ y) {
	GRID_STRIDE(i, total) y[i] += b[(i / hw) % Cout];
}

// db[c] (+)= sum over samples n, then positions i, serially from +0 (ops.cpp:1595-1599)
__global__ void conv_bias_grad_serial_kernel(const float* __restrict__ g, int N, int Cout, long long hw,
		float* __restrict__ db, int first) {
	const int c = blockIdx.x * blockDim.x + threadIdx.x;
	if (c >= Cout) return;
	float acc = 0.0f;
	for (int n = 0; n < N; ++n) {
		const float* p = g + ((long long)n * Cout + c) * hw;
		for (long long i = 0; i < hw; ++i) acc += p[i];
	}
	db[c] = first ? acc + 0.0f : db[c] + acc;
}

__global__ void mask_grad_kernel(long long n, const float* __restrict__ g, const unsigned char* __restrict__ alive,
		float* __restrict__ out) {
	GRID_STRIDE(i, n) out[i] = alive[i] ? g[i] : 0.0f;
}

// gb[n*Cout + c] = lane_sum(g[n][c][:]) (ops.cpp:804-812, 1441-1442): one thread per (sample, channel)
__global__ void conv_plane_sum_kernel(const float* __restrict__ g, long long planes, long long hw, float* __restrict__ gb) {
	const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
	if (idx >= planes) return;
	const float* p = g + idx * hw;
	float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
	long long i = 0;
	for (; i + 8 <= hw; i += 8)
#pragma unroll
		for (int k = 0; k < 8; ++k) a[k] += p[i + k];
	float t = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
	for (; i < hw; ++i) t += p[i];
	gb[idx] = t;
}

// db[c] (+)= sum_n gb[n][c] in sample order (Tensor::sum(0), src/tensor.cpp:448-453; ops.cpp:1461)
__global__ void conv_bias_grad_kernel(const float* __restrict__ gb, int N, int Cout, float* __restrict__ db, int first) {
	const int c = blockIdx.x * blockDim.x + threadIdx.x;
	if (c >= Cout) return;
	float acc = 0.0f;
	for (int n = 0; n < N; ++n) acc += gb[(long long)n * Cout + c];
	db[c] = first ? acc + 0.0f : db[c] + acc;
}

// dw[j] (+)= sum_n gw[n][j] in sample order (Tensor::sum(0), src/tensor.cpp:448-453)
__global__ void sum_samples_kernel(const float* __restrict__ gw, int N, long long per, float* __restrict__ dw, int first) {
	GRID_STRIDE(j, per) {
		float acc = 0.0f;
		for (int n = 0; n < N; ++n) acc += gw[(long long)n * per + j];
		dw[j] = first ? acc + 0.0f : dw[j] + acc;
	}
}

nnb_status make_geo(size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh, size_t kw, int stride, int padding,
		Geo& g) {
	if (stride <= 0 || padding < 0) return fail(NNB_ERR_SHAPE, "conv2d: stride %d / padding %d", stride, padding);
	if (kh == 0 || kw == 0 || kh > H + 2 * (size_t)padding || kw > W + 2 * (size_t)padding)
		return fail(NNB_ERR_SHAPE, "conv2d: kernel %zux%zu larger than the padded input", kh, kw);
	g.N = (int)N; g.Cin = (int)Cin; g.H = (int)H; g.W = (int)W; g.Cout = (int)Cout;
	g.kh = (int)kh; g.kw = (int)kw; g.stride = stride; g.pad = padding;
	g.ho = (int)((H + 2 * padding - kh) / stride + 1);
	g.wo = (int)((W + 2 * padding - kw) / stride + 1);
	return NNB_OK;
}

nnb_status make_geo_ex(size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t Cg, size_t kh, size_t kw,
		int stride, int padding, int dilation, int groups, Geo& g) {
	if (stride <= 0 || padding < 0 || dilation <= 0 || groups <= 0)
		return fail(NNB_ERR_SHAPE, "conv2d: stride %d, padding %d, dilation %d, groups %d", stride, padding, dilation,
			groups);
	const size_t G = (size_t)groups;
	if (Cin % G != 0 || Cout % G != 0 || Cg != Cin / G || kh == 0 || kw == 0)
		return fail(NNB_ERR_SHAPE, "conv2d: %zu input / %zu output channels do not split into %d groups of %zu", Cin, Cout,
			groups, Cg);
	const size_t ekh = (size_t)dilation * (kh - 1) + 1, ekw = (size_t)dilation * (kw - 1) + 1;
	if (ekh > H + 2 * (size_t)padding || ekw > W + 2 * (size_t)padding)
		return fail(NNB_ERR_SHAPE, "conv2d: dilated kernel %zux%zu larger than the padded input", ekh, ekw);
	g.N = (int)N; g.Cin = (int)Cin; g.H = (int)H; g.W = (int)W; g.Cout = (int)Cout;
	g.kh = (int)kh; g.kw = (int)kw; g.stride = stride; g.pad = padding; g.dil = dilation; g.groups = groups;
	g.ho = (int)((H + 2 * padding - ekh) / stride + 1);
	g.wo = (int)((W + 2 * padding - ekw) / stride + 1);
	return NNB_OK;
}

}  // namespace

}  // namespace nnb

extern "C" {

nnb_status nnb_conv2d_fwd(void* stream, size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh, size_t kw,
		int stride, int padding, const float* x, const float* weight, const float* bias, int fuse_relu, float* y,
		unsigned char* alive) {
	nnb::Geo g;
	NNB_TRY(nnb::make_geo(N, Cin, H, W, Cout, kh, kw, stride, padding, g));
	if (N == 0 || Cout == 0) return NNB_OK;
	if (!x || !weight || !bias || !y || (fuse_relu && !alive)) return nnb::fail(NNB_ERR_INVALID, "conv2d_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long K = g.K(), hw = g.hw();
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, (size_t)N * K * hw * sizeof(float), s));
	float* col = static_cast<float*>(ws);
	nnb_status st = NNB_OK;
	{
		nnb::TraceScope ts(s, nnb::kTraceConv);
		nnb::im2col_kernel<<<nnb::grid_for((long long)N * K * hw, 256), 256, 0, s>>>(g, x, col);
	}
	st = nnb::cuda_status(cudaGetLastError(), "im2col launch");
	if (st == NNB_OK) {
		nnb::GemmDesc d;
		d.m = (long long)Cout; d.n = hw; d.k = K;
		d.a = weight; d.lda = K; d.b = col; d.ldb = hw; d.c = y; d.ldc = hw;
		d.batch_outer = (long long)N; d.sa_outer = 0; d.sb_outer = K * hw; d.sc_outer = (long long)Cout * hw;
		d.mode = nnb::math_mode();
		d.epi.bias = bias; d.epi.bias_mode = nnb::kBiasRow;
		if (fuse_relu) {
			d.epi.act = nnb::kActRelu;
			d.epi.mask = alive;
			d.epi.ld_aux = hw;
			d.epi.s_aux_outer = (long long)Cout * hw;
		}
		st = nnb::gemm_run(s, d);
	}
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

nnb_status nnb_conv2d_bwd(void* stream, size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh, size_t kw,
		int stride, int padding, const float* grad, const float* x, const float* weight, const unsigned char* alive,
		float* dx, int dx_first, float* dweight, int dweight_first, float* dbias, int dbias_first) {
	nnb::Geo g;
	NNB_TRY(nnb::make_geo(N, Cin, H, W, Cout, kh, kw, stride, padding, g));
	if (N == 0 || Cout == 0) return NNB_OK;
	if (!grad || !x || !weight) return nnb::fail(NNB_ERR_INVALID, "conv2d_bwd: null input");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long K = g.K(), hw = g.hw(), out_n = (long long)N * Cout * hw;
	const bool need_col = dweight || dx;
	const size_t col_f = need_col ? (size_t)N * K * hw : 0, gm_f = alive ? (size_t)out_n : 0,
		gw_f = dweight ? (size_t)N * Cout * K : 0;
	void* ws = nullptr;
	const size_t gb_f = (size_t)N * Cout;
	NNB_TRY(nnb::scratch_alloc(&ws, (col_f + gm_f + gw_f + gb_f + 64) * sizeof(float), s));
	float* col = static_cast<float*>(ws);
	float* gm = col + col_f;
	float* gw = gm + gm_f;
	float* gb = gw + gw_f;
	nnb_status st = NNB_OK;
	do {
		const float* gg = grad;
		if (alive) {
			nnb::TraceScope ts(s, nnb::kTraceConv);
			nnb::mask_grad_kernel<<<nnb::grid_for(out_n, 256), 256, 0, s>>>(out_n, grad, alive, gm);
			gg = gm;
		}
		if (dbias) {
			const long long planes = (long long)N * Cout;
			{
				nnb::TraceScope ts(s, nnb::kTraceConv);
				nnb::conv_plane_sum_kernel<<<(unsigned)((planes + 127) / 128), 128, 0, s>>>(gg, planes, hw, gb);
			}
			nnb::TraceScope ts(s, nnb::kTraceConv);
			nnb::conv_bias_grad_kernel<<<(unsigned)((Cout + 127) / 128), 128, 0, s>>>(gb, (int)N, (int)Cout, dbias,
				dbias_first);
		}
		if ((st = nnb::cuda_status(cudaGetLastError(), "conv bias grad launch")) != NNB_OK) break;
		if (dweight) {
			{
				nnb::TraceScope ts(s, nnb::kTraceConv);
				nnb::im2col_kernel<<<nnb::grid_for((long long)N * K * hw, 256), 256, 0, s>>>(g, x, col);
			}
			nnb::GemmDesc d;     // gw[n] = g[n] col[n]^T : [Cout, hw] x [hw, K]
			d.tb = 1;
			d.m = (long long)Cout; d.n = K; d.k = hw;
			d.a = gg; d.lda = hw; d.b = col; d.ldb = hw; d.c = gw; d.ldc = K;
			d.batch_outer = (long long)N; d.sa_outer = (long long)Cout * hw; d.sb_outer = K * hw; d.sc_outer = (long long)Cout * K;
			d.mode = nnb::math_mode();
			if ((st = nnb::gemm_run(s, d)) != NNB_OK) break;
			const long long per = (long long)Cout * K;
			nnb::TraceScope ts(s, nnb::kTraceConv);
			nnb::sum_samples_kernel<<<nnb::grid_for(per, 256), 256, 0, s>>>(gw, (int)N, per, dweight, dweight_first);
		}
		if (dx) {
			nnb::GemmDesc d;     // dcol[n] = W^T g[n] : [K, Cout] x [Cout, hw], into the col buffer
			d.ta = 1;
			d.m = K; d.n = hw; d.k = (long long)Cout;
			d.a = weight; d.lda = K; d.b = gg; d.ldb = hw; d.c = col; d.ldc = hw;
			d.batch_outer = (long long)N; d.sa_outer = 0; d.sb_outer = (long long)Cout * hw; d.sc_outer = K * hw;
			d.mode = nnb::math_mode();
			if ((st = nnb::gemm_run(s, d)) != NNB_OK) break;
			nnb::TraceScope ts(s, nnb::kTraceConv);
			nnb::col2im_kernel<<<nnb::grid_for((long long)N * Cin * H * W, 256), 256, 0, s>>>(g, col, dx, dx_first);
		}
		st = nnb::cuda_status(cudaGetLastError(), "conv2d_bwd launch");
	} while (0);
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

nnb_status nnb_conv2d_ex_fwd(void* stream, size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh, size_t kw,
		int stride, int padding, int dilation, int groups, const float* x, const float* weight, const float* bias,
		float* y) {
	nnb::Geo g;
	NNB_TRY(nnb::make_geo_ex(N, Cin, H, W, Cout, Cin / (groups > 0 ? (size_t)groups : 1), kh, kw, stride, padding, dilation,
		groups, g));
	if (N == 0 || Cout == 0) return NNB_OK;
	if (!x || !weight || !bias || !y) return nnb::fail(NNB_ERR_INVALID, "conv2d_ex_fwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long K = g.K(), hw = g.hw(), G = groups, Kg = K / G, Cog = (long long)Cout / G;
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, (size_t)N * K * hw * sizeof(float), s));
	float* col = static_cast<float*>(ws);
	nnb_status st = NNB_OK;
	do {
		{
			nnb::TraceScope ts(s, nnb::kTraceConv);
			nnb::im2col_kernel<<<nnb::grid_for((long long)N * K * hw, 256), 256, 0, s>>>(g, x, col);
		}
		if ((st = nnb::cuda_status(cudaGetLastError(), "im2col launch")) != NNB_OK) break;
		// y[n][g] = W_g col[n][g] for every (sample, group): ops.cpp:1552-1555
		nnb::GemmDesc d;
		d.m = Cog; d.n = hw; d.k = Kg;
		d.a = weight; d.lda = Kg; d.b = col; d.ldb = hw; d.c = y; d.ldc = hw;
		d.batch_outer = (long long)N; d.batch_inner = G;
		d.sa_outer = 0; d.sa_inner = Cog * Kg;
		d.sb_outer = K * hw; d.sb_inner = Kg * hw;
		d.sc_outer = (long long)Cout * hw; d.sc_inner = Cog * hw;
		d.mode = nnb::math_mode();
		if ((st = nnb::gemm_run(s, d)) != NNB_OK) break;
		const long long total = (long long)N * Cout * hw;
		nnb::TraceScope ts(s, nnb::kTraceConv);
		nnb::conv_add_bias_kernel<<<nnb::grid_for(total, 256), 256, 0, s>>>(total, hw, (int)Cout, bias, y);
		st = nnb::cuda_status(cudaGetLastError(), "conv bias launch");
	} while (0);
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

nnb_status nnb_conv2d_ex_bwd(void* stream, size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh, size_t kw,
		int stride, int padding, int dilation, int groups, const float* grad, const float* x, const float* weight,
		float* dx, int dx_first, float* dweight, int dweight_first, float* dbias, int dbias_first) {
	nnb::Geo g;
	NNB_TRY(nnb::make_geo_ex(N, Cin, H, W, Cout, Cin / (groups > 0 ? (size_t)groups : 1), kh, kw, stride, padding, dilation,
		groups, g));
	if (N == 0 || Cout == 0) return NNB_OK;
	if (!grad || !x || !weight) return nnb::fail(NNB_ERR_INVALID, "conv2d_ex_bwd: null input");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const long long K = g.K(), hw = g.hw(), G = groups, Kg = K / G, Cog = (long long)Cout / G;
	const size_t col_f = (dweight || dx) ? (size_t)N * K * hw : 0, gw_f = dweight ? (size_t)N * Cout * Kg : 0;
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, (col_f + gw_f + 64) * sizeof(float), s));
	float* col = static_cast<float*>(ws);
	float* gw = col + col_f;
	nnb_status st = NNB_OK;
	do {
		if (dbias) {
			nnb::TraceScope ts(s, nnb::kTraceConv);
			nnb::conv_bias_grad_serial_kernel<<<(unsigned)((Cout + 127) / 128), 128, 0, s>>>(grad, (int)N, (int)Cout, hw,
				dbias, dbias_first);
		}
		if ((st = nnb::cuda_status(cudaGetLastError(), "conv bias grad launch")) != NNB_OK) break;
		if (dweight) {
			{
				nnb::TraceScope ts(s, nnb::kTraceConv);
				nnb::im2col_kernel<<<nnb::grid_for((long long)N * K * hw, 256), 256, 0, s>>>(g, x, col);
			}
			nnb::GemmDesc d;     // gw[n][g] = g[n][g] col[n][g]^T : [Cog, hw] x [hw, Kg]  (ops.cpp:1580-1581)
			d.tb = 1;
			d.m = Cog; d.n = Kg; d.k = hw;
			d.a = grad; d.lda = hw; d.b = col; d.ldb = hw; d.c = gw; d.ldc = Kg;
			d.batch_outer = (long long)N; d.batch_inner = G;
			d.sa_outer = (long long)Cout * hw; d.sa_inner = Cog * hw;
			d.sb_outer = K * hw; d.sb_inner = Kg * hw;
			d.sc_outer = (long long)Cout * Kg; d.sc_inner = Cog * Kg;
			d.mode = nnb::math_mode();
			if ((st = nnb::gemm_run(s, d)) != NNB_OK) break;
			const long long per = (long long)Cout * Kg;
			nnb::TraceScope ts(s, nnb::kTraceConv);
			nnb::sum_samples_kernel<<<nnb::grid_for(per, 256), 256, 0, s>>>(gw, (int)N, per, dweight, dweight_first);
		}
		if (dx) {
			nnb::GemmDesc d;     // dcol[n][g] = W_g^T g[n][g] : [Kg, Cog] x [Cog, hw]  (ops.cpp:1584-1585)
			d.ta = 1;
			d.m = Kg; d.n = hw; d.k = Cog;
			d.a = weight; d.lda = Kg; d.b = grad; d.ldb = hw; d.c = col; d.ldc = hw;
			d.batch_outer = (long long)N; d.batch_inner = G;
			d.sa_outer = 0; d.sa_inner = Cog * Kg;
			d.sb_outer = (long long)Cout * hw; d.sb_inner = Cog * hw;
			d.sc_outer = K * hw; d.sc_inner = Kg * hw;
			d.mode = nnb::math_mode();
			if ((st = nnb::gemm_run(s, d)) != NNB_OK) break;
			nnb::TraceScope ts(s, nnb::kTraceConv);
			nnb::col2im_kernel<<<nnb::grid_for((long long)N * Cin * H * W, 256), 256, 0, s>>>(g, col, dx, dx_first);
		}
		st = nnb::cuda_status(cudaGetLastError(), "conv2d_ex_bwd launch");
	} while (0);
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

}  // extern "C"
