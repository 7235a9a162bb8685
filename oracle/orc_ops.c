/*
 * orc_ops.c -- CPU oracle for the fused ops on the GEMM path. TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs load this
 * code, to check the CUDA path; no product path calls it.
 *
 * Each function restates one op of nn-cpp v2.0.0 in plain C, in the reference's own order of
 * floating-point operations (serial loops as written there), citing the lines it follows. GEMMs
 * inside the ops use the plain fp32 triple loop of tests/reference_gemm.hpp (orc_sgemm_f32). It is
 * compiled with -ffp-contract=off, as the reference is. Pinned against the reference build itself
 * by tests/test_oracle_ops.py.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

void orc_sgemm_f32(int ta, int tb, size_t m, size_t n, size_t k, const float* a, size_t lda, const float* b,
		size_t ldb, float* c, size_t ldc, int accumulate);

/* grad_accum convention (ops.cpp:67-73): first stores v + 0, otherwise adds */
static inline float acc_store(float old, float v, int first) { return first ? v + 0.0f : old + v; }

/* ---- vmath (src/kernels/vmath.cpp:79-109): Cephes expf and tanh from mul/add/div only ---- */

float orc_exp_one(float x) {
	const float kExpLo = -87.3f, kExpHi = 88.3f, kLog2e = 1.44269504088896341f;
	const float kLn2Hi = 0.693359375f, kLn2Lo = -2.12194440e-4f;
	const float kP0 = 1.9875691500e-4f, kP1 = 1.3981999507e-3f, kP2 = 8.3334519073e-3f;
	const float kP3 = 4.1665795894e-2f, kP4 = 1.6666665459e-1f, kP5 = 5.0000001201e-1f;
	if (x != x) return x;
	if (x < kExpLo) return 0.0f;
	if (x > kExpHi) return HUGE_VALF;
	float n = nearbyintf(x * kLog2e);
	float r = x - n * kLn2Hi;
	r = r - n * kLn2Lo;
	float p = kP0;
	p = p * r + kP1;
	p = p * r + kP2;
	p = p * r + kP3;
	p = p * r + kP4;
	p = p * r + kP5;
	float e = (p * (r * r) + r) + 1.0f;
	uint32_t bits = (uint32_t)((int32_t)n + 127) << 23;
	float pow2;
	memcpy(&pow2, &bits, sizeof pow2);
	return e * pow2;
}

float orc_tanh_one(float x) {
	if (x != x) return x;
	float z = x < -9.0f ? -9.0f : x;
	z = 9.0f < z ? 9.0f : z;
	float e = orc_exp_one(z + z);
	return (e - 1.0f) / (e + 1.0f);
}

/* ---- gelu (ops.cpp:451-481) ---- */
void orc_gelu_fwd(size_t n, const float* x, float* y, float* th) {
	const float k = 0.7978845608f, c = 0.044715f;
	for (size_t i = 0; i < n; i++) th[i] = k * (x[i] + c * x[i] * x[i] * x[i]);
	for (size_t i = 0; i < n; i++) th[i] = orc_tanh_one(th[i]);
	for (size_t i = 0; i < n; i++) y[i] = 0.5f * x[i] * (1.0f + th[i]);
}

void orc_gelu_bwd(size_t n, const float* x, const float* th, const float* g, float* dx, int first) {
	const float k = 0.7978845608f, c = 0.044715f;
	for (size_t i = 0; i < n; i++) {
		const float v = x[i], t = th[i];
		dx[i] = acc_store(dx[i], g[i] * (0.5f * (1.0f + t) + 0.5f * v * (1.0f - t * t) * k * (1.0f + 3.0f * c * v * v)), first);
	}
}

/* ---- relu (ops.cpp:775-793) ---- */
void orc_relu_fwd(size_t n, const float* x, float* y) {
	for (size_t i = 0; i < n; i++) y[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

void orc_relu_bwd(size_t n, const float* x, const float* g, float* dx, int first) {
	for (size_t i = 0; i < n; i++) dx[i] = acc_store(dx[i], x[i] > 0.0f ? g[i] : 0.0f, first);
}

/* ---- column sum = Tensor::sum(0) of a 2-D tensor (src/tensor.cpp:448-453) into a grad ---- */
void orc_colsum(size_t rows, size_t cols, const float* g, float* out, int first) {
	float* acc = (float*)calloc(cols ? cols : 1, sizeof(float));
	for (size_t r = 0; r < rows; r++)
		for (size_t j = 0; j < cols; j++) acc[j] += g[r * cols + j];
	for (size_t j = 0; j < cols; j++) out[j] = acc_store(out[j], acc[j], first);
	free(acc);
}

/* ---- linear (ops.cpp:714-745) ---- */
void orc_linear_fwd(size_t M, size_t K, size_t n, const float* x, const float* w, const float* b, float* y) {
	orc_sgemm_f32(0, 1, M, n, K, x, K, w, K, y, n, 0);
	for (size_t r = 0; r < M; r++)
		for (size_t j = 0; j < n; j++) y[r * n + j] += b[j];
}

void orc_linear_bwd(size_t M, size_t K, size_t n, const float* g, const float* x, const float* w, float* dx,
		int dx_first, float* dw, int dw_first, float* db, int db_first) {
	if (dx) orc_sgemm_f32(0, 0, M, K, n, g, n, w, K, dx, K, !dx_first);
	if (dw) orc_sgemm_f32(1, 0, n, K, M, g, n, x, K, dw, K, !dw_first);
	if (db) orc_colsum(M, n, g, db, db_first);
}

/* ---- layernorm (ops.cpp:1003-1078) ---- */
void orc_layernorm_fwd(size_t R, size_t D, const float* x, const float* gm, const float* bt, float eps, float* y,
		float* mean, float* inv_std) {
	for (size_t r = 0; r < R; r++) {
		const float* row = x + r * D;
		float sum = 0.0f;
		for (size_t j = 0; j < D; j++) sum += row[j];
		const float mu = sum / (float)D;
		float sq = 0.0f;
		for (size_t j = 0; j < D; j++) sq += (row[j] - mu) * (row[j] - mu);
		const float inv = 1.0f / sqrtf(sq / (float)D + eps);
		mean[r] = mu;
		inv_std[r] = inv;
		for (size_t j = 0; j < D; j++) y[r * D + j] = (row[j] - mu) * inv * gm[j] + bt[j];
	}
}

void orc_layernorm_bwd(size_t R, size_t D, const float* g, const float* x, const float* gm, const float* mean,
		const float* inv_std, float* dx, int dx_first, float* dg, int dg_first, float* db, int db_first) {
	if (dx) {
		for (size_t r = 0; r < R; r++) {
			const float mu = mean[r], inv = inv_std[r];
			float a = 0.0f, b = 0.0f;
			for (size_t j = 0; j < D; j++) {
				const float dxhat = g[r * D + j] * gm[j];
				a += dxhat;
				b += dxhat * ((x[r * D + j] - mu) * inv);
			}
			const float k = inv / (float)D, fd = (float)D;
			for (size_t j = 0; j < D; j++) {
				const float dxhat = g[r * D + j] * gm[j];
				dx[r * D + j] = acc_store(dx[r * D + j], k * (fd * dxhat - a - ((x[r * D + j] - mu) * inv) * b), dx_first);
			}
		}
	}
	for (size_t j = 0; j < D; j++) {
		float sg = 0.0f, sb = 0.0f;
		for (size_t r = 0; r < R; r++) {
			const float gv = g[r * D + j];
			sg += gv * ((x[r * D + j] - mean[r]) * inv_std[r]);
			sb += gv;
		}
		if (dg) dg[j] = acc_store(dg[j], sg, dg_first);
		if (db) db[j] = acc_store(db[j], sb, db_first);
	}
}

/* ---- batchnorm, training statistics (ops.cpp:804-1001) ---- */
static float lane_sum(const float* p, size_t n) {
	float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
	size_t i = 0;
	for (; i + 8 <= n; i += 8)
		for (size_t k = 0; k < 8; k++) a[k] += p[i + k];
	float t = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
	for (; i < n; i++) t += p[i];
	return t;
}

static float lane_sq(const float* p, size_t n, float mu) {
	float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
	size_t i = 0;
	for (; i + 8 <= n; i += 8)
		for (size_t k = 0; k < 8; k++) {
			const float d = p[i + k] - mu;
			a[k] += d * d;
		}
	float t = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
	for (; i < n; i++) t += (p[i] - mu) * (p[i] - mu);
	return t;
}

static float lane_sum_m(const float* g, const unsigned char* alive, size_t n) {
	float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
	size_t i = 0;
	for (; i + 8 <= n; i += 8)
		for (size_t k = 0; k < 8; k++) a[k] += alive ? (alive[i + k] ? g[i + k] : 0.0f) : g[i + k];
	float t = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
	for (; i < n; i++) t += alive ? (alive[i] ? g[i] : 0.0f) : g[i];
	return t;
}

static float lane_dot_m(const float* g, const unsigned char* alive, const float* x, size_t n, float mu) {
	float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
	size_t i = 0;
	for (; i + 8 <= n; i += 8)
		for (size_t k = 0; k < 8; k++) a[k] += (alive ? (alive[i + k] ? g[i + k] : 0.0f) : g[i + k]) * (x[i + k] - mu);
	float t = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
	for (; i < n; i++) t += (alive ? (alive[i] ? g[i] : 0.0f) : g[i]) * (x[i] - mu);
	return t;
}

void orc_batchnorm_fwd(size_t N, size_t C, size_t S, const float* x, const float* w, const float* b, float eps,
		int fuse_relu, float* y, unsigned char* alive, float* mean, float* var, float* inv_std) {
	const size_t M = N * S;
	for (size_t c = 0; c < C; c++) {
		double sum = 0.0;
		for (size_t n = 0; n < N; n++) sum += lane_sum(x + (n * C + c) * S, S);
		const float mu = (float)(sum / (double)M);
		double sq = 0.0;
		for (size_t n = 0; n < N; n++) sq += lane_sq(x + (n * C + c) * S, S, mu);
		const float v = (float)(sq / (double)M);
		const float inv = 1.0f / sqrtf(v + eps);
		mean[c] = mu;
		var[c] = v;
		inv_std[c] = inv;
		const float scale = w[c] * inv;
		for (size_t n = 0; n < N; n++)
			for (size_t s = 0; s < S; s++) {
				const size_t i = (n * C + c) * S + s;
				const float o = (x[i] - mu) * scale + b[c];
				if (fuse_relu) {
					alive[i] = o > 0.0f;
					y[i] = o > 0.0f ? o : 0.0f;
				} else {
					y[i] = o;
				}
			}
	}
}

void orc_batchnorm_bwd(size_t N, size_t C, size_t S, const float* g, const float* x, const float* w,
		const float* mean, const float* inv_std, const unsigned char* alive, float* dx, int dx_first, float* dw,
		int dw_first, float* db, int db_first) {
	const size_t M = N * S;
	for (size_t c = 0; c < C; c++) {
		const float mu = mean[c], inv = inv_std[c];
		double sdy = 0.0, sdg = 0.0;
		for (size_t n = 0; n < N; n++) {
			const size_t base = (n * C + c) * S;
			sdy += lane_sum_m(g + base, alive ? alive + base : NULL, S);
			sdg += lane_dot_m(g + base, alive ? alive + base : NULL, x + base, S, mu);
		}
		const double sdyx = sdg * inv;
		if (db) db[c] = acc_store(db[c], (float)sdy, db_first);
		if (dw) dw[c] = acc_store(dw[c], (float)sdyx, dw_first);
		if (dx) {
			const float k = w[c] * inv / (float)M;
			const float fm = (float)M, a = (float)sdy, bb = (float)sdyx;
			for (size_t n = 0; n < N; n++)
				for (size_t s = 0; s < S; s++) {
					const size_t i = (n * C + c) * S + s;
					const float gv = alive ? (alive[i] ? g[i] : 0.0f) : g[i];
					dx[i] = acc_store(dx[i], k * (fm * gv - a - ((x[i] - mu) * inv) * bb), dx_first);
				}
		}
	}
}

/* ---- attention (ops.cpp:1183-1296) ---- */
static void softmax_row(const float* row, float* o, size_t Tk, size_t i, const float* ph, int causal, float scale) {
	for (size_t j = 0; j < Tk; j++) {
		float v = row[j] * scale;
		if (ph && ph[j] == 0.0f) v = -1e9f;
		if (causal && j > i) v = -2e9f;
		o[j] = v;
	}
	float m = o[0];
	for (size_t j = 1; j < Tk; j++) m = fmaxf(m, o[j]);
	const size_t live = causal ? (Tk < i + 1 ? Tk : i + 1) : Tk;
	float sum = 0.0f;
	for (size_t j = 0; j < live; j++) {
		o[j] = expf(o[j] - m);
		sum += o[j];
	}
	for (size_t j = live; j < Tk; j++) o[j] = 0.0f;
	for (size_t j = 0; j < Tk; j++) o[j] /= sum;
}

static void softmax_row_bwd(const float* y, float* g, size_t Tk, size_t i, const float* ph, int causal, float scale) {
	float dot = 0.0f;
	for (size_t j = 0; j < Tk; j++) dot += g[j] * y[j];
	for (size_t j = 0; j < Tk; j++) {
		const int masked = (ph && ph[j] == 0.0f) || (causal && j > i);
		g[j] = masked ? 0.0f : scale * (y[j] * (g[j] - dot)) + 0.0f;
	}
}

void orc_attention_fwd(size_t N, size_t Tq, size_t Tk, size_t D, size_t H, const float* q, const float* k,
		const float* v, const float* pad, int causal, float* out, float* probs) {
	const size_t Dh = D / H;
	const float scale = 1.0f / sqrtf((float)Dh);
	for (size_t nh = 0; nh < N * H; nh++) {
		const size_t n = nh / H, h = nh % H;
		float* p = probs + nh * Tq * Tk;
		orc_sgemm_f32(0, 1, Tq, Tk, Dh, q + n * Tq * D + h * Dh, D, k + n * Tk * D + h * Dh, D, p, Tk, 0);
		for (size_t i = 0; i < Tq; i++) softmax_row(p + i * Tk, p + i * Tk, Tk, i, pad ? pad + n * Tk : NULL, causal, scale);
		orc_sgemm_f32(0, 0, Tq, Dh, Tk, p, Tk, v + n * Tk * D + h * Dh, D, out + n * Tq * D + h * Dh, D, 0);
	}
}

void orc_attention_bwd(size_t N, size_t Tq, size_t Tk, size_t D, size_t H, const float* g, const float* q,
		const float* k, const float* v, const float* probs, const float* pad, int causal, float* dq, int dq_first,
		float* dk, int dk_first, float* dv, int dv_first) {
	const size_t Dh = D / H;
	const float scale = 1.0f / sqrtf((float)Dh);
	float* ds = (float*)malloc(Tq * Tk * sizeof(float));
	for (size_t nh = 0; nh < N * H; nh++) {
		const size_t n = nh / H, h = nh % H;
		const float* p = probs + nh * Tq * Tk;
		const float* gh = g + n * Tq * D + h * Dh;
		orc_sgemm_f32(0, 1, Tq, Tk, Dh, gh, D, v + n * Tk * D + h * Dh, D, ds, Tk, 0);
		if (dv) orc_sgemm_f32(1, 0, Tk, Dh, Tq, p, Tk, gh, D, dv + n * Tk * D + h * Dh, D, !dv_first);
		if (!dq && !dk) continue;
		for (size_t i = 0; i < Tq; i++)
			softmax_row_bwd(p + i * Tk, ds + i * Tk, Tk, i, pad ? pad + n * Tk : NULL, causal, scale);
		if (dq) orc_sgemm_f32(0, 0, Tq, Dh, Tk, ds, Tk, k + n * Tk * D + h * Dh, D, dq + n * Tq * D + h * Dh, D, !dq_first);
		if (dk) orc_sgemm_f32(1, 0, Tk, Dh, Tq, ds, Tk, q + n * Tq * D + h * Dh, D, dk + n * Tk * D + h * Dh, D, !dk_first);
	}
	free(ds);
}

/* ---- BatchNorm module: running statistics and evaluation mode (batchnorm.cpp:27-60) ----
 * Training forwards update rm = (1-m)*rm + m*mean and rv = (1-m)*rv + (m*var)*(n/(n-1)) (only rm
 * when n = 1), from the batch statistics of orc_batchnorm_fwd. Evaluation composes the reference's
 * broadcasting ops: inv = 1/sqrt(rv + eps), normed = (x - rm)*inv, y = normed*w + b (ReLU on top when
 * fused). Its backward, for Y's gradient gy (the caller's seed, stored as g + 0), follows the op graph:
 * every node's gradient is stored as v + 0, ReLU passes g or +0, and the broadcast parameters' gradients
 * are reduced to [1, C, 1, 1] as sum_to_shape does (ops.cpp:35-53): over axis 0, then 2, then 3, each
 * only when its extent is not 1, each a serial sum from zero. */
void orc_bn_running_update(size_t C, size_t n, float momentum, const float* mean, const float* var, float* rm,
		float* rv) {
	const float unbiased = n > 1 ? (float)n / (float)(n - 1) : 0.0f;
	for (size_t c = 0; c < C; c++) {
		rm[c] = (1.0f - momentum) * rm[c] + momentum * mean[c];
		if (n > 1) rv[c] = (1.0f - momentum) * rv[c] + momentum * var[c] * unbiased;
	}
}

void orc_reduce_axis_fwd(size_t outer, size_t n, size_t inner, int average, const float* x, float* y);

static void sum_to_channels(size_t N, size_t C, size_t H, size_t W, const float* t, float* out) {
	float* a = (float*)malloc(N * C * H * W * sizeof(float));
	float* b = (float*)malloc(N * C * H * W * sizeof(float));
	memcpy(a, t, N * C * H * W * sizeof(float));
	size_t n0 = N, h = H, w = W;
	if (n0 != 1) { orc_reduce_axis_fwd(1, n0, C * h * w, 0, a, b); memcpy(a, b, C * h * w * sizeof(float)); n0 = 1; }
	if (h != 1) { orc_reduce_axis_fwd(C, h, w, 0, a, b); memcpy(a, b, C * w * sizeof(float)); h = 1; }
	if (w != 1) { orc_reduce_axis_fwd(C, w, 1, 0, a, b); memcpy(a, b, C * sizeof(float)); w = 1; }
	memcpy(out, a, C * sizeof(float));
	free(a);
	free(b);
}

void orc_batchnorm_eval_fwd(size_t N, size_t C, size_t S, const float* x, const float* w, const float* b,
		const float* rm, const float* rv, float eps, int fuse_relu, float* y) {
	for (size_t c = 0; c < C; c++) {
		const float inv = 1.0f / sqrtf(rv[c] + eps);
		for (size_t n = 0; n < N; n++)
			for (size_t s = 0; s < S; s++) {
				const size_t i = (n * C + c) * S + s;
				const float o = ((x[i] - rm[c]) * inv) * w[c] + b[c];
				y[i] = fuse_relu ? (o > 0.0f ? o : 0.0f) : o;
			}
	}
}

void orc_batchnorm_eval_bwd(size_t N, size_t C, size_t H, size_t W, const float* gy, const float* x, const float* w,
		const float* b, const float* rm, const float* rv, float eps, int fuse_relu, float* dx, float* dw, float* db) {
	const size_t S = H * W, T = N * C * S;
	float* r = (float*)malloc(T * sizeof(float));
	float* t = (float*)malloc(T * sizeof(float));
	float* red = (float*)malloc(C * sizeof(float));
	for (size_t c = 0; c < C; c++) {
		const float inv = 1.0f / sqrtf(rv[c] + eps);
		for (size_t n = 0; n < N; n++)
			for (size_t s = 0; s < S; s++) {
				const size_t i = (n * C + c) * S + s;
				const float normed = (x[i] - rm[c]) * inv;
				const float g = gy[i] + 0.0f;                                  /* Y's gradient */
				const float ri = fuse_relu ? ((normed * w[c] + b[c] > 0.0f ? g : 0.0f) + 0.0f) : g;
				r[i] = ri;                                                     /* the add node's gradient */
				const float g1 = ri + 0.0f;                                    /* normed * w */
				t[i] = g1 * normed;
				const float g2 = g1 * w[c] + 0.0f;                             /* normed */
				const float g3 = g2 * inv + 0.0f;                              /* x - rm */
				dx[i] = g3 + 0.0f;
			}
	}
	sum_to_channels(N, C, H, W, t, red);
	for (size_t c = 0; c < C; c++) dw[c] = red[c] + 0.0f;
	sum_to_channels(N, C, H, W, r, red);
	for (size_t c = 0; c < C; c++) db[c] = red[c] + 0.0f;
	free(r);
	free(t);
	free(red);
}

/* ---- conv2d / conv2d_relu (ops.cpp:188-243, 1345-1472) ---- */
/* column matrix [Cin*kh*kw, ho*wo] of one sample (or one group's channels); tap (ph, pw) reads input
 * row oh*st + ph*dl - pd and column ow*st + pw*dl - pd, zero outside (ops.cpp:1486-1500 with dl > 1) */
static void im2col(const float* x, float* col, size_t Cin, size_t H, size_t W, size_t kh, size_t kw, size_t st,
		size_t pd, size_t dl, size_t ho, size_t wo) {
	for (size_t c = 0; c < Cin; c++)
		for (size_t ph = 0; ph < kh; ph++)
			for (size_t pw = 0; pw < kw; pw++)
				for (size_t oh = 0; oh < ho; oh++)
					for (size_t ow = 0; ow < wo; ow++) {
						const long ih = (long)(oh * st + ph * dl) - (long)pd, iw = (long)(ow * st + pw * dl) - (long)pd;
						float v = 0.0f;
						if (ih >= 0 && ih < (long)H && iw >= 0 && iw < (long)W) v = x[(c * H + (size_t)ih) * W + (size_t)iw];
						col[((c * kh + ph) * kw + pw) * ho * wo + oh * wo + ow] = v;
					}
}

static void col2im_add(const float* col, float* x, size_t Cin, size_t H, size_t W, size_t kh, size_t kw, size_t st,
		size_t pd, size_t dl, size_t ho, size_t wo) {
	for (size_t c = 0; c < Cin; c++)
		for (size_t ph = 0; ph < kh; ph++)
			for (size_t pw = 0; pw < kw; pw++)
				for (size_t oh = 0; oh < ho; oh++)
					for (size_t ow = 0; ow < wo; ow++) {
						const long ih = (long)(oh * st + ph * dl) - (long)pd, iw = (long)(ow * st + pw * dl) - (long)pd;
						if (ih >= 0 && ih < (long)H && iw >= 0 && iw < (long)W)
							x[(c * H + (size_t)ih) * W + (size_t)iw] += col[((c * kh + ph) * kw + pw) * ho * wo + oh * wo + ow];
					}
}

void orc_conv2d_fwd(size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh, size_t kw, size_t st,
		size_t pd, const float* x, const float* w, const float* b, int fuse_relu, float* y, unsigned char* alive) {
	const size_t ho = (H + 2 * pd - kh) / st + 1, wo = (W + 2 * pd - kw) / st + 1, K = Cin * kh * kw, hw = ho * wo;
	float* col = (float*)malloc(K * hw * sizeof(float));
	for (size_t n = 0; n < N; n++) {
		im2col(x + n * Cin * H * W, col, Cin, H, W, kh, kw, st, pd, 1, ho, wo);
		float* yn = y + n * Cout * hw;
		orc_sgemm_f32(0, 0, Cout, hw, K, w, K, col, hw, yn, hw, 0);
		for (size_t c = 0; c < Cout; c++)
			for (size_t i = 0; i < hw; i++) {
				const float v = yn[c * hw + i] + b[c];
				if (fuse_relu) {
					alive[(n * Cout + c) * hw + i] = v > 0.0f;
					yn[c * hw + i] = v > 0.0f ? v : 0.0f;
				} else {
					yn[c * hw + i] = v;
				}
			}
	}
	free(col);
}

void orc_conv2d_bwd(size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh, size_t kw, size_t st,
		size_t pd, const float* grad, const float* x, const float* w, const unsigned char* alive, float* dx,
		int dx_first, float* dw, int dw_first, float* db, int db_first) {
	const size_t ho = (H + 2 * pd - kh) / st + 1, wo = (W + 2 * pd - kw) / st + 1, K = Cin * kh * kw, hw = ho * wo;
	float* col = (float*)malloc(K * hw * sizeof(float));
	float* gm = (float*)malloc(Cout * hw * sizeof(float));
	float* gw = (float*)malloc(N * Cout * K * sizeof(float));
	float* gb = (float*)malloc(N * Cout * sizeof(float));
	for (size_t n = 0; n < N; n++) {
		const float* g = grad + n * Cout * hw;
		for (size_t i = 0; i < Cout * hw; i++) gm[i] = alive ? (alive[n * Cout * hw + i] ? g[i] : 0.0f) : g[i];
		for (size_t c = 0; c < Cout; c++) gb[n * Cout + c] = lane_sum(gm + c * hw, hw);
		im2col(x + n * Cin * H * W, col, Cin, H, W, kh, kw, st, pd, 1, ho, wo);
		orc_sgemm_f32(0, 1, Cout, K, hw, gm, hw, col, hw, gw + n * Cout * K, K, 0);
		if (dx) {
			orc_sgemm_f32(1, 0, K, hw, Cout, w, K, gm, hw, col, hw, 0);
			float* dxn = dx + n * Cin * H * W;
			if (dx_first) memset(dxn, 0, Cin * H * W * sizeof(float));
			col2im_add(col, dxn, Cin, H, W, kh, kw, st, pd, 1, ho, wo);
		}
	}
	if (db)
		for (size_t c = 0; c < Cout; c++) {
			float s = 0.0f;
			for (size_t n = 0; n < N; n++) s += gb[n * Cout + c];
			db[c] = acc_store(db[c], s, db_first);
		}
	if (dw)
		for (size_t j = 0; j < Cout * K; j++) {
			float s = 0.0f;
			for (size_t n = 0; n < N; n++) s += gw[n * Cout * K + j];
			dw[j] = acc_store(dw[j], s, dw_first);
		}
	free(col);
	free(gm);
	free(gw);
	free(gb);
}

/* ---- conv2d with dilation and groups (ops.cpp:1525-1607) ----
 * Per sample n and group g: the group's Cg = Cin/G input channels go through the dilated im2col, its
 * Cog = Cout/G filters (w rows g*Cog..) multiply the column matrix, then the bias is added. Backward:
 * dW per sample, summed over samples in order; dX by the transposed product and col2im per group into
 * a zeroed per-sample buffer; the bias gradient sums, per channel, samples then positions in order. */
void orc_conv2d_ex_fwd(size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh, size_t kw, size_t st,
		size_t pd, size_t dl, size_t G, const float* x, const float* w, const float* b, float* y) {
	const size_t Cg = Cin / G, Cog = Cout / G, K = Cg * kh * kw;
	const size_t ho = (H + 2 * pd - (dl * (kh - 1) + 1)) / st + 1, wo = (W + 2 * pd - (dl * (kw - 1) + 1)) / st + 1;
	const size_t hw = ho * wo;
	float* col = (float*)malloc(K * hw * sizeof(float));
	for (size_t n = 0; n < N; n++)
		for (size_t g = 0; g < G; g++) {
			im2col(x + (n * Cin + g * Cg) * H * W, col, Cg, H, W, kh, kw, st, pd, dl, ho, wo);
			float* yg = y + (n * Cout + g * Cog) * hw;
			orc_sgemm_f32(0, 0, Cog, hw, K, w + g * Cog * K, K, col, hw, yg, hw, 0);
			for (size_t c = 0; c < Cog; c++)
				for (size_t i = 0; i < hw; i++) yg[c * hw + i] += b[g * Cog + c];
		}
	free(col);
}

void orc_conv2d_ex_bwd(size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh, size_t kw, size_t st,
		size_t pd, size_t dl, size_t G, const float* grad, const float* x, const float* w, float* dx, float* dw,
		float* db) {
	const size_t Cg = Cin / G, Cog = Cout / G, K = Cg * kh * kw;
	const size_t ho = (H + 2 * pd - (dl * (kh - 1) + 1)) / st + 1, wo = (W + 2 * pd - (dl * (kw - 1) + 1)) / st + 1;
	const size_t hw = ho * wo, wsz = Cout * K;
	float* col = (float*)malloc(K * hw * sizeof(float));
	float* gw = (float*)malloc(N * wsz * sizeof(float));
	memset(dx, 0, N * Cin * H * W * sizeof(float));
	for (size_t n = 0; n < N; n++)
		for (size_t g = 0; g < G; g++) {
			const float* gy = grad + (n * Cout + g * Cog) * hw;
			im2col(x + (n * Cin + g * Cg) * H * W, col, Cg, H, W, kh, kw, st, pd, dl, ho, wo);
			orc_sgemm_f32(0, 1, Cog, K, hw, gy, hw, col, hw, gw + n * wsz + g * Cog * K, K, 0);
			orc_sgemm_f32(1, 0, K, hw, Cog, w + g * Cog * K, K, gy, hw, col, hw, 0);
			col2im_add(col, dx + (n * Cin + g * Cg) * H * W, Cg, H, W, kh, kw, st, pd, dl, ho, wo);
		}
	for (size_t c = 0; c < Cout; c++) {
		float s = 0.0f;
		for (size_t n = 0; n < N; n++)
			for (size_t i = 0; i < hw; i++) s += grad[(n * Cout + c) * hw + i];
		db[c] = s + 0.0f;
	}
	for (size_t j = 0; j < wsz; j++) {
		float s = 0.0f;
		for (size_t n = 0; n < N; n++) s += gw[n * wsz + j];
		dw[j] = s + 0.0f;
	}
	free(col);
	free(gw);
}

/* ---- maxpool2d (ops.cpp:1609-1705) ---- */
void orc_maxpool2d_fwd(size_t N, size_t C, size_t H, size_t W, size_t k, size_t st, const float* x, float* y,
		uint32_t* arg) {
	const size_t ho = (H - k) / st + 1, wo = (W - k) / st + 1;
	for (size_t p = 0; p < N * C; p++)
		for (size_t oh = 0; oh < ho; oh++)
			for (size_t ow = 0; ow < wo; ow++) {
				float best = -INFINITY;
				uint32_t at = 0;
				for (size_t ph = 0; ph < k; ph++)
					for (size_t pw = 0; pw < k; pw++) {
						const float v = x[p * H * W + (oh * st + ph) * W + ow * st + pw];
						if (v > best) {
							best = v;
							at = (uint32_t)((oh * st + ph) * W + ow * st + pw);
						}
					}
				y[p * ho * wo + oh * wo + ow] = best;
				arg[p * ho * wo + oh * wo + ow] = at;
			}
}

void orc_maxpool2d_bwd(size_t N, size_t C, size_t H, size_t W, size_t k, size_t st, const float* g,
		const uint32_t* arg, float* dx, int first) {
	const size_t ho = (H - k) / st + 1, wo = (W - k) / st + 1;
	for (size_t p = 0; p < N * C; p++) {
		float* plane = dx + p * H * W;
		if (first) memset(plane, 0, H * W * sizeof(float));
		for (size_t i = p * ho * wo; i < (p + 1) * ho * wo; i++) plane[arg[i]] += g[i];
	}
}

/* ---- avgpool2d (ops.cpp:1707-1770) ----
 * y = (window sum from 0, rows then columns) * (1 / (k*k)); the backward adds g * (1 / (k*k)) to
 * every element of each window, windows in (oh, ow) order, into dx (zeroed first when `first`). */
void orc_avgpool2d_fwd(size_t N, size_t C, size_t H, size_t W, size_t k, size_t st, const float* x, float* y) {
	const size_t ho = (H - k) / st + 1, wo = (W - k) / st + 1;
	const float inv = 1.0f / (float)(k * k);
	for (size_t p = 0; p < N * C; p++)
		for (size_t oh = 0; oh < ho; oh++)
			for (size_t ow = 0; ow < wo; ow++) {
				float acc = 0.0f;
				for (size_t ph = 0; ph < k; ph++)
					for (size_t pw = 0; pw < k; pw++) acc += x[p * H * W + (oh * st + ph) * W + ow * st + pw];
				y[p * ho * wo + oh * wo + ow] = acc * inv;
			}
}

void orc_avgpool2d_bwd(size_t N, size_t C, size_t H, size_t W, size_t k, size_t st, const float* g, float* dx,
		int first) {
	const size_t ho = (H - k) / st + 1, wo = (W - k) / st + 1;
	const float inv = 1.0f / (float)(k * k);
	for (size_t p = 0; p < N * C; p++) {
		float* plane = dx + p * H * W;
		if (first) memset(plane, 0, H * W * sizeof(float));
		for (size_t oh = 0; oh < ho; oh++)
			for (size_t ow = 0; ow < wo; ow++) {
				const float share = g[p * ho * wo + oh * wo + ow] * inv;
				for (size_t ph = 0; ph < k; ph++)
					for (size_t pw = 0; pw < k; pw++) plane[(oh * st + ph) * W + ow * st + pw] += share;
			}
	}
}

/* ---- sum / mean over one axis (ops.cpp:284-327) ----
 * x viewed as [outer, n, inner]; y[o, i] = sum over j in order from 0 (times 1/n for the mean); the
 * backward stores g * factor + 0 (first) or adds g * factor to every x element of the reduced line. */
void orc_reduce_axis_fwd(size_t outer, size_t n, size_t inner, int average, const float* x, float* y) {
	const float factor = average ? 1.0f / (float)n : 1.0f;
	for (size_t o = 0; o < outer; o++)
		for (size_t i = 0; i < inner; i++) {
			float total = 0.0f;
			for (size_t j = 0; j < n; j++) total += x[(o * n + j) * inner + i];
			y[o * inner + i] = average ? total * factor : total;
		}
}

void orc_reduce_axis_bwd(size_t outer, size_t n, size_t inner, int average, const float* g, float* dx, int first) {
	const float factor = average ? 1.0f / (float)n : 1.0f;
	for (size_t o = 0; o < outer; o++)
		for (size_t i = 0; i < inner; i++) {
			const float v = g[o * inner + i] * factor;
			for (size_t j = 0; j < n; j++) {
				float* d = dx + (o * n + j) * inner + i;
				*d = first ? v + 0.0f : *d + v;
			}
		}
}

/* ---- cross entropy (ops.cpp:1774-1840) ---- */
void orc_cross_entropy_fwd(size_t N, size_t C, const float* logits, const int64_t* t, float* sm, float* loss) {
	float total = 0.0f;
	for (size_t n = 0; n < N; n++) {
		const float* row = logits + n * C;
		float* s = sm + n * C;
		float mx = -INFINITY;
		for (size_t c = 0; c < C; c++) mx = fmaxf(mx, row[c]);
		float se = 0.0f;
		for (size_t c = 0; c < C; c++) {
			s[c] = row[c] - mx;
			se += expf(s[c]);
		}
		const float lse = logf(se);
		total += -(s[t[n]] - lse);
		for (size_t c = 0; c < C; c++) s[c] = expf(s[c] - lse);
	}
	*loss = total / (float)N;
}

void orc_cross_entropy_bwd(size_t N, size_t C, const float* sm, const int64_t* t, float grad_loss, float* dl, int first) {
	const float scale = grad_loss / (float)N;
	for (size_t n = 0; n < N; n++)
		for (size_t c = 0; c < C; c++) {
			const float v = ((int64_t)c == t[n] ? sm[n * C + c] - 1.0f : sm[n * C + c]) * scale;
			dl[n * C + c] = acc_store(dl[n * C + c], v, first);
		}
}

/* ---- sequence cross entropy (ops.cpp:1908-1979) ---- */
void orc_sequence_ce_fwd(size_t P, size_t V, const float* logits, const int64_t* t, int64_t ignore, float ls,
		float* sm, float* loss) {
	const float inv_v = 1.0f / (float)V;
	double total = 0.0;
	size_t count = 0;
	for (size_t p = 0; p < P; p++) {
		if (t[p] == ignore) continue;
		count++;
		const float* row = logits + p * V;
		float* s = sm + p * V;
		float mx = row[0];
		for (size_t c = 1; c < V; c++) mx = fmaxf(mx, row[c]);
		float se = 0.0f;
		for (size_t c = 0; c < V; c++) se += expf(row[c] - mx);
		const float lse = logf(se);
		float mean_nll = 0.0f;
		for (size_t c = 0; c < V; c++) {
			const float lp = row[c] - mx - lse;
			s[c] = expf(lp);
			mean_nll -= lp * inv_v;
		}
		const float nll = -(row[t[p]] - mx - lse);
		total += (double)((1.0f - ls) * nll + ls * mean_nll);
	}
	*loss = (float)(total / (double)count);
}

void orc_sequence_ce_bwd(size_t P, size_t V, const float* sm, const int64_t* t, int64_t ignore, float ls,
		float grad_loss, size_t count, float* dl, int first) {
	const float g = grad_loss * (1.0f / (float)count);
	for (size_t p = 0; p < P; p++)
		for (size_t c = 0; c < V; c++) {
			float v = 0.0f;
			if (t[p] != ignore) {
				v = sm[p * V + c] - ls / (float)V;
				if ((int64_t)c == t[p]) v -= 1.0f - ls;
				v *= g;
			}
			dl[p * V + c] = acc_store(dl[p * V + c], v, first);
		}
}

/* ---- embedding (ops.cpp:1991-2015); backward adds into dweight ---- */
void orc_embedding_fwd(size_t D, const float* w, const int64_t* ids, size_t count, float* out) {
	for (size_t i = 0; i < count; i++) memcpy(out + i * D, w + ids[i] * D, D * sizeof(float));
}

void orc_embedding_bwd(size_t D, const int64_t* ids, size_t count, const float* g, float* dw) {
	for (size_t i = 0; i < count; i++)
		for (size_t d = 0; d < D; d++) dw[ids[i] * D + d] += g[i * D + d];
}

/* ---- AdamW step (src/optim/adamw.cpp:15-24, src/optim/adam.cpp:24-43) ---- */
void orc_adamw_step(size_t n, float* w, const float* g, float* m, float* v, float lr, float b1, float b2, float eps,
		float wd, long long step) {
	const float shrink = 1.0f - lr * wd;
	for (size_t k = 0; k < n; k++) w[k] *= shrink;
	const float c1 = 1.0f - powf(b1, (float)step);
	const float c2 = 1.0f - powf(b2, (float)step);
	for (size_t k = 0; k < n; k++) {
		m[k] = b1 * m[k] + (1.0f - b1) * g[k];
		v[k] = b2 * v[k] + (1.0f - b2) * g[k] * g[k];
		w[k] -= lr * (m[k] / c1) / (sqrtf(v[k] / c2) + eps);
	}
}
