// ops_conv.cu -- `conv2d` / `conv2d_relu` (src/autograd/ops.cpp:1345-1472) and the general conv
// (dilation, groups; ops.cpp:1525-1607) as implicit GEMMs on the tensor-core kernel: the kernel's
// gather warps build the column operand straight into its shared-memory stages from the activation
// (or the output gradient), so no column matrix [K, N*hw] is ever written to global memory.
//
// Forward: y[n][g] = W_g im2col(x[n][g]) for every (sample, group) in ONE launch, the im2col of the
// reference (im2col_sample, ops.cpp:188-212) gathered per stage (kGatherIm2col); bias (per output
// channel = per row), ReLU and the 1-byte alive mask in the epilogue (ops.cpp:1395-1408). The grouped
// path adds its bias afterwards, as the reference's general path does (ops.cpp:1556-1557).
// Backward: the gradient masked by `alive`; db per channel = sum over samples, in sample order, of the
// 8-lane sum of the channel's plane (ops.cpp:1441-1442, 1461); dW = sum over samples, in sample order,
// of g[n] im2col(x[n])^T (one launch into per-sample buffers, the column rows gathered per stage:
// kGatherIm2colRows; then an ordered sum, ops.cpp:1449, 1462); dX = col2im(W^T g[n]) (ops.cpp:1452-1455)
// as ONE product per (sample, group): rows = input channels, columns = input positions, depth =
// (kernel row, kernel column, output channel) over W rearranged to [c][(ph, pw, co)] and the output
// gradient gathered at the window position that reads each input position (kGatherTransposed). Each
// dX element is one k-ordered chain over the taps and channels, where the reference adds per-tap
// products in (kernel row, kernel column) order: the same terms, fp32-bound apart.
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

// wt[g][c][(ph*kw + pw)*Cog + co] = w[g*Cog + co][c][ph][pw]: the A operand of the input gradient
__global__ void conv_weight_taps_kernel(long long total, int Cg, int Cog, int khw, const float* __restrict__ w,
		float* __restrict__ wt) {
	GRID_STRIDE(i, total) {
		const long long per_group = (long long)Cg * khw * Cog;
		const long long grp = i / per_group;
		const long long r = i - grp * per_group;
		const int c = (int)(r / ((long long)khw * Cog));
		const int rem = (int)(r - (long long)c * khw * Cog);
		const int t = rem / Cog, co = rem - t * Cog;
		wt[i] = w[((grp * Cog + co) * Cg + c) * khw + t];
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

GemmGather gather_of(const Geo& g, int mode, const float* src) {
	GemmGather q;
	q.mode = mode;
	q.src = src;
	const int Cg = g.Cin / g.groups, Cog = g.Cout / g.groups;
	if (mode == kGatherTransposed) {          // the output gradient [N][Cout][ho][wo], per (sample, group)
		q.s_outer = (long long)g.Cout * g.hw();
		q.s_inner = (long long)Cog * g.hw();
		q.C = Cog;
	} else {                                  // the input [N][Cin][H][W], per (sample, group)
		q.s_outer = (long long)g.Cin * g.H * g.W;
		q.s_inner = (long long)Cg * g.H * g.W;
		q.C = Cg;
	}
	q.H = g.H; q.W = g.W; q.ho = g.ho; q.wo = g.wo; q.kh = g.kh; q.kw = g.kw;
	q.stride = g.stride; q.pad = g.pad; q.dil = g.dil; q.cout = Cog;
	return q;
}

// y[n][g] = W_g im2col(x[n][g]) (+ the epilogue in d.epi), one launch over every (sample, group)
nnb_status conv_forward(cudaStream_t s, const Geo& g, const float* x, const float* w, float* y, const GemmEpilogue& epi) {
	const long long G = g.groups, Kg = g.K() / G, Cog = g.Cout / G, hw = g.hw();
	GemmDesc d;
	d.m = Cog; d.n = hw; d.k = Kg;
	d.a = w; d.lda = Kg;
	d.c = y; d.ldc = hw;
	d.batch_outer = g.N; d.batch_inner = G;
	d.sa_outer = 0; d.sa_inner = Cog * Kg;
	d.sc_outer = (long long)g.Cout * hw; d.sc_inner = Cog * hw;
	d.mode = math_mode();
	d.epi = epi;
	d.gather = gather_of(g, kGatherIm2col, x);
	return gemm_run(s, d);
}

// gw[n][g] = gg[n][g] im2col(x[n][g])^T : [Cog, hw] x [hw, Kg], per (sample, group)
nnb_status conv_weight_grad(cudaStream_t s, const Geo& g, const float* gg, const float* x, float* gw) {
	const long long G = g.groups, Kg = g.K() / G, Cog = g.Cout / G, hw = g.hw();
	GemmDesc d;
	d.m = Cog; d.n = Kg; d.k = hw;
	d.a = gg; d.lda = hw;
	d.c = gw; d.ldc = Kg;
	d.batch_outer = g.N; d.batch_inner = G;
	d.sa_outer = (long long)g.Cout * hw; d.sa_inner = Cog * hw;
	d.sc_outer = (long long)g.Cout * Kg; d.sc_inner = Cog * Kg;
	d.mode = math_mode();
	d.gather = gather_of(g, kGatherIm2colRows, x);
	return gemm_run(s, d);
}

// dx[n][g] (+)= Wt_g gather(gg[n][g]) : [Cg, khw*Cog] x [khw*Cog, H*W], per (sample, group)
nnb_status conv_input_grad(cudaStream_t s, const Geo& g, const float* gg, const float* wt, float* dx, int first) {
	const long long G = g.groups, Cg = g.Cin / G, Cog = g.Cout / G, khw = (long long)g.kh * g.kw;
	const long long plane = (long long)g.H * g.W;
	GemmDesc d;
	d.m = Cg; d.n = plane; d.k = khw * Cog;
	d.a = wt; d.lda = khw * Cog;
	d.c = dx; d.ldc = plane;
	d.batch_outer = g.N; d.batch_inner = G;
	d.sa_outer = 0; d.sa_inner = Cg * khw * Cog;
	d.sc_outer = (long long)g.Cin * plane; d.sc_inner = Cg * plane;
	d.accumulate = first ? 0 : 1;
	d.mode = math_mode();
	d.gather = gather_of(g, kGatherTransposed, gg);
	return gemm_run(s, d);
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
	nnb::GemmEpilogue epi;
	epi.bias = bias;
	epi.bias_mode = nnb::kBiasRow;
	if (fuse_relu) {
		epi.act = nnb::kActRelu;
		epi.mask = alive;
		epi.ld_aux = g.hw();
		epi.s_aux_outer = (long long)Cout * g.hw();
	}
	return nnb::conv_forward(static_cast<cudaStream_t>(stream), g, x, weight, y, epi);
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
	const size_t gm_f = alive ? (size_t)out_n : 0, gw_f = dweight ? (size_t)N * Cout * K : 0;
	const size_t wt_f = dx ? (size_t)Cout * K : 0, gb_f = (size_t)N * Cout;
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, (gm_f + gw_f + wt_f + gb_f + 64) * sizeof(float), s));
	float* gm = static_cast<float*>(ws);
	float* gw = gm + gm_f;
	float* wt = gw + gw_f;
	float* gb = wt + wt_f;
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
			if ((st = nnb::conv_weight_grad(s, g, gg, x, gw)) != NNB_OK) break;
			const long long per = (long long)Cout * K;
			nnb::TraceScope ts(s, nnb::kTraceConv);
			nnb::sum_samples_kernel<<<nnb::grid_for(per, 256), 256, 0, s>>>(gw, (int)N, per, dweight, dweight_first);
		}
		if (dx) {
			{
				nnb::TraceScope ts(s, nnb::kTraceConv);
				nnb::conv_weight_taps_kernel<<<nnb::grid_for((long long)Cout * K, 256), 256, 0, s>>>((long long)Cout * K,
					(int)Cin, (int)Cout, (int)(kh * kw), weight, wt);
			}
			if ((st = nnb::cuda_status(cudaGetLastError(), "conv weight taps launch")) != NNB_OK) break;
			if ((st = nnb::conv_input_grad(s, g, gg, wt, dx, dx_first)) != NNB_OK) break;
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
	// y[n][g] = W_g col[n][g] for every (sample, group) (ops.cpp:1552-1555), then the bias
	NNB_TRY(nnb::conv_forward(s, g, x, weight, y, nnb::GemmEpilogue()));
	const long long total = (long long)N * Cout * g.hw();
	nnb::TraceScope ts(s, nnb::kTraceConv);
	nnb::conv_add_bias_kernel<<<nnb::grid_for(total, 256), 256, 0, s>>>(total, g.hw(), (int)Cout, bias, y);
	return nnb::cuda_status(cudaGetLastError(), "conv bias launch");
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
	const long long K = g.K(), G = groups, Kg = K / G;
	const size_t gw_f = dweight ? (size_t)N * Cout * Kg : 0, wt_f = dx ? (size_t)Cout * Kg : 0;
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, (gw_f + wt_f + 64) * sizeof(float), s));
	float* gw = static_cast<float*>(ws);
	float* wt = gw + gw_f;
	nnb_status st = NNB_OK;
	do {
		if (dbias) {
			nnb::TraceScope ts(s, nnb::kTraceConv);
			nnb::conv_bias_grad_serial_kernel<<<(unsigned)((Cout + 127) / 128), 128, 0, s>>>(grad, (int)N, (int)Cout,
				g.hw(), dbias, dbias_first);
		}
		if ((st = nnb::cuda_status(cudaGetLastError(), "conv bias grad launch")) != NNB_OK) break;
		if (dweight) {      // gw[n][g] = g[n][g] col[n][g]^T (ops.cpp:1580-1581), then the sample-order sum
			if ((st = nnb::conv_weight_grad(s, g, grad, x, gw)) != NNB_OK) break;
			const long long per = (long long)Cout * Kg;
			nnb::TraceScope ts(s, nnb::kTraceConv);
			nnb::sum_samples_kernel<<<nnb::grid_for(per, 256), 256, 0, s>>>(gw, (int)N, per, dweight, dweight_first);
		}
		if (dx) {           // dcol[n][g] = W_g^T g[n][g] folded back (ops.cpp:1584-1587), one product
			{
				nnb::TraceScope ts(s, nnb::kTraceConv);
				nnb::conv_weight_taps_kernel<<<nnb::grid_for((long long)Cout * Kg, 256), 256, 0, s>>>((long long)Cout * Kg,
					(int)(Cin / G), (int)(Cout / G), (int)(kh * kw), weight, wt);
			}
			if ((st = nnb::cuda_status(cudaGetLastError(), "conv weight taps launch")) != NNB_OK) break;
			if ((st = nnb::conv_input_grad(s, g, grad, wt, dx, dx_first)) != NNB_OK) break;
		}
		st = nnb::cuda_status(cudaGetLastError(), "conv2d_ex_bwd launch");
	} while (0);
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

}  // extern "C"
