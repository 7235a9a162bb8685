/*
 * ref_shim.cpp -- a C-ABI over the reference library itself, for checking and timing only.
 * TEST INFRASTRUCTURE ONLY (tests/, smoke() and bench.py's cpu_baseline / reference legs).
 *
 * oracle/Makefile compiles this file together with the reference's own, unmodified sources
 * (read in place from the reference tree, compiled with the reference's flags: C++17,
 * -ffp-contract=off, AVX2+FMA) into oracle/_ref/libnnref.so. Nothing here re-implements the
 * reference: every function forwards to the reference's public API so that Python (ctypes)
 * can run it on the same host buffers the CUDA path sees.
 */
#include "nn/autograd/ops.hpp"
#include "nn/checkpoint.hpp"
#include "nn/data/dataloader.hpp"
#include "nn/data/subset.hpp"
#include "nn/data/tensor_dataset.hpp"
#include "nn/nn/attention.hpp"
#include "nn/nn/dropout.hpp"
#include "nn/random.hpp"
#include "nn/nn/linear.hpp"
#include "nn/autograd/value.hpp"
#include "nn/kernels/gemm.hpp"
#include "nn/kernels/vmath.hpp"
#include "nn/nn/batchnorm.hpp"
#include "nn/nn/pool2d.hpp"
#include "nn/nn/sequential.hpp"
#include "nn/nn/transformer.hpp"
#include "nn/optim/adamw.hpp"
#include "nn/kernels/parallel.hpp"
#include "nn/tensor.hpp"
#include "reference_gemm.hpp"   // the reference's own test oracle, tests/reference_gemm.hpp

#include <chrono>
#include <cmath>
#include <cstddef>
#include <cstring>
#include <vector>

namespace {

using nn::Tensor;
using nn::Value;

size_t count_of(const std::vector<size_t>& shape) {
	size_t n = 1;
	for (size_t d : shape) n *= d;
	return n;
}

Tensor tensor(std::vector<size_t> shape, const float* p) {
	const size_t n = count_of(shape);
	return Tensor(std::move(shape), std::vector<float>(p, p + n));
}

Value leaf(std::vector<size_t> shape, const float* p) { return Value::leaf(tensor(std::move(shape), p), true); }

void copy_out(const Tensor& t, float* dst) {
	if (dst) std::memcpy(dst, t.data().data(), t.size() * sizeof(float));
}

// Runs a node's backward rule once with the given upstream gradient (the leaves' gradients start
// at zero, so every contribution lands as 0 + term).
void backward_with(const Value& out, const float* g) { out.impl()->backward_fn(tensor(out.data().shape(), g)); }

// Backpropagates an upstream gradient g of y through y's whole graph: d sum(y * G) / dy = G exactly.
void backward_through(const Value& y, const float* g) {
	Value G = Value::leaf(tensor(y.data().shape(), g), false);
	nn::sum(nn::mul(y, G)).backward();
}

Tensor ids_tensor(std::vector<size_t> shape, const int64_t* ids) {
	std::vector<float> v(count_of(shape));
	for (size_t i = 0; i < v.size(); ++i) v[i] = static_cast<float>(ids[i]);
	return Tensor(std::move(shape), std::move(v));
}

}  // namespace

extern "C" {

/* nn::kernels::sgemm (include/nn/kernels/gemm.hpp:57) */
void ref_sgemm(int ta, int tb, size_t m, size_t n, size_t k, const float* a, size_t lda,
		const float* b, size_t ldb, float* c, size_t ldc, int accumulate) {
	nn::kernels::sgemm(ta != 0, tb != 0, m, n, k, a, lda, b, ldb, c, ldc, accumulate != 0);
}

/* nn::kernels::sgemm_portable (gemm.hpp:69) */
void ref_sgemm_portable(int ta, int tb, size_t m, size_t n, size_t k, const float* a, size_t lda,
		const float* b, size_t ldb, float* c, size_t ldc, int accumulate) {
	nn::kernels::sgemm_portable(ta != 0, tb != 0, m, n, k, a, lda, b, ldb, c, ldc, accumulate != 0);
}

/* reference_sgemm, the plain triple loop of tests/reference_gemm.hpp:30-45, compiled as is */
void ref_reference_sgemm(int ta, int tb, size_t m, size_t n, size_t k, const float* a, size_t lda,
		const float* b, size_t ldb, float* c, size_t ldc, int accumulate) {
	reference_sgemm(ta != 0, tb != 0, m, n, k, a, lda, b, ldb, c, ldc, accumulate != 0);
}

int ref_sgemm_uses_avx2() { return nn::kernels::sgemm_uses_avx2() ? 1 : 0; }

/* parallel.hpp:23,34 */
size_t ref_num_threads() { return nn::kernels::num_threads(); }
void ref_set_threads(size_t n) { nn::kernels::set_num_threads(n); }

/*
 * nn::matmul on [batch..., m, k] x [k, n] tensors (tensor.cpp:571-641), with the result copied
 * out. a has a_batch*m*k floats, b has k*n, c receives a_batch*m*n.
 */
void ref_matmul(size_t a_batch, size_t m, size_t k, size_t n, const float* a, const float* b,
		float* c) {
	std::vector<size_t> ashape;
	if (a_batch > 1) ashape.push_back(a_batch);
	ashape.push_back(m);
	ashape.push_back(k);
	nn::Tensor ta(ashape, std::vector<float>(a, a + a_batch * m * k));
	nn::Tensor tb({k, n}, std::vector<float>(b, b + k * n));
	nn::Tensor tc = nn::matmul(ta, tb);
	std::memcpy(c, tc.data().data(), a_batch * m * n * sizeof(float));
}

/*
 * Times `reps` calls of nn::matmul(a, b) on [m,k] x [k,n] tensors built once, the way
 * apps/bench/runner.cpp:80-96 times its matmul suite; returns the median seconds per call.
 */
double ref_time_matmul(size_t m, size_t k, size_t n, const float* a, const float* b, int reps) {
	nn::Tensor ta({m, k}, std::vector<float>(a, a + m * k));
	nn::Tensor tb({k, n}, std::vector<float>(b, b + k * n));
	std::vector<double> t;
	for (int r = 0; r < reps; ++r) {
		auto t0 = std::chrono::steady_clock::now();
		nn::Tensor tc = nn::matmul(ta, tb);
		auto t1 = std::chrono::steady_clock::now();
		t.push_back(std::chrono::duration<double>(t1 - t0).count());
		if (tc.data().empty()) return -1.0;
	}
	std::vector<double> s = t;
	for (size_t i = 1; i < s.size(); ++i)
		for (size_t j = i; j > 0 && s[j - 1] > s[j]; --j) std::swap(s[j - 1], s[j]);
	return s.empty() ? 0.0 : s[s.size() / 2];
}

/*
 * Median seconds of `reps` calls (after one untimed call) of nn::kernels::sgemm(false, false, m, n,
 * k, a, k, b, n, c, n, false): the reference's lowest seam (gemm.hpp:57) on row-major operands.
 */
double ref_time_sgemm(size_t m, size_t n, size_t k, const float* a, const float* b, float* c, int reps) {
	nn::kernels::sgemm(false, false, m, n, k, a, k, b, n, c, n, false);
	std::vector<double> t;
	for (int r = 0; r < reps; ++r) {
		auto t0 = std::chrono::steady_clock::now();
		nn::kernels::sgemm(false, false, m, n, k, a, k, b, n, c, n, false);
		auto t1 = std::chrono::steady_clock::now();
		t.push_back(std::chrono::duration<double>(t1 - t0).count());
	}
	for (size_t i = 1; i < t.size(); ++i)
		for (size_t j = i; j > 0 && t[j - 1] > t[j]; --j) std::swap(t[j - 1], t[j]);
	return t.empty() ? 0.0 : t[t.size() / 2];
}

/*
 * nn::matmul(a, b, trans_a, trans_b) (tensor.cpp:571) on N-D tensors; c receives the result
 * (sized by the caller). Returns 0, or 1 when the reference throws a shape error.
 */
int ref_matmul_nd(const float* a, const int64_t* as, int an, const float* b, const int64_t* bs, int bn, int ta,
		int tb, float* c) {
	try {
		std::vector<size_t> sa(as, as + an), sb(bs, bs + bn);
		Tensor A = tensor(sa, a), B = tensor(sb, b);
		Tensor C = nn::matmul(A, B, ta != 0, tb != 0);
		copy_out(C, c);
		return 0;
	} catch (const std::exception&) {
		return 1;
	}
}

/* ---- the reference's autograd ops, forward then one backward with upstream gradient g ---- */

/*
 * nn::matmul / nn::matmul_bt on Values (ops.cpp:683-712, 747-773): y = op(a, b), or with `twice`
 * y = add(op(a, b), op(a, b)) so each gradient is stored by one backward rule and added to by the
 * other; then d sum(y * g) through the graph. Returns 0, or 1 when the reference throws.
 */
int ref_matmul_value(const float* a, const int64_t* as, int an, const float* b, const int64_t* bs, int bn, int bt,
		int twice, const float* g, float* y, float* da, float* db) {
	try {
		Value A = leaf(std::vector<size_t>(as, as + an), a), B = leaf(std::vector<size_t>(bs, bs + bn), b);
		Value Y = bt ? nn::matmul_bt(A, B) : nn::matmul(A, B);
		if (twice) Y = nn::add(Y, bt ? nn::matmul_bt(A, B) : nn::matmul(A, B));
		copy_out(Y.data(), y);
		backward_through(Y, g);
		copy_out(A.grad(), da);
		copy_out(B.grad(), db);
		return 0;
	} catch (const std::exception&) {
		return 1;
	}
}

/* nn::scaled_masked_softmax (ops.cpp:1298-1343) on x [N, H, Tq, Tk], then the backward of g. */
void ref_scaled_masked_softmax(size_t N, size_t H, size_t Tq, size_t Tk, const float* x, float scale,
		const float* pad, int causal, const float* g, float* y, float* dx) {
	Value X = leaf({N, H, Tq, Tk}, x);
	Tensor mask = pad ? tensor({N, Tk}, pad) : Tensor({0});
	Value Y = nn::scaled_masked_softmax(X, scale, mask, causal != 0);
	copy_out(Y.data(), y);
	backward_with(Y, g);
	copy_out(X.grad(), dx);
}


void ref_linear(size_t M, size_t K, size_t n, const float* x, const float* w, const float* b, const float* g,
		float* y, float* dx, float* dw, float* db) {
	Value X = leaf({M, K}, x), W = leaf({n, K}, w), B = leaf({n}, b);
	Value Y = nn::linear(X, W, B);
	copy_out(Y.data(), y);
	backward_with(Y, g);
	copy_out(X.grad(), dx);
	copy_out(W.grad(), dw);
	copy_out(B.grad(), db);
}

void ref_layernorm(size_t R, size_t D, const float* x, const float* gm, const float* bt, float eps, const float* g,
		float* y, float* dx, float* dg, float* db) {
	Value X = leaf({R, D}, x), G = leaf({D}, gm), B = leaf({D}, bt);
	Value Y = nn::layernorm(X, G, B, eps);
	copy_out(Y.data(), y);
	backward_with(Y, g);
	copy_out(X.grad(), dx);
	copy_out(G.grad(), dg);
	copy_out(B.grad(), db);
}

void ref_batchnorm(size_t N, size_t C, size_t S, const float* x, const float* w, const float* b, float eps,
		int fuse_relu, const float* g, float* y, float* mean, float* var, float* dx, float* dw, float* db) {
	Value X = leaf({N, C, S}, x), W = leaf({C}, w), B = leaf({C}, b);
	Tensor mo({1}), vo({1});
	Value Y = nn::batchnorm(X, W, B, eps, &mo, &vo, fuse_relu != 0);
	copy_out(Y.data(), y);
	copy_out(mo, mean);
	copy_out(vo, var);
	backward_with(Y, g);
	copy_out(X.grad(), dx);
	copy_out(W.grad(), dw);
	copy_out(B.grad(), db);
}

void ref_attention(size_t N, size_t Tq, size_t Tk, size_t D, size_t heads, const float* q, const float* k,
		const float* v, const float* pad, int causal, const float* g, float* out, float* dq, float* dk, float* dv) {
	Value Q = leaf({N, Tq, D}, q), K = leaf({N, Tk, D}, k), V = leaf({N, Tk, D}, v);
	Tensor mask = pad ? tensor({N, Tk}, pad) : Tensor({0});
	Value O = nn::attention(Q, K, V, heads, mask, causal != 0);
	copy_out(O.data(), out);
	backward_with(O, g);
	copy_out(Q.grad(), dq);
	copy_out(K.grad(), dk);
	copy_out(V.grad(), dv);
}

void ref_conv2d(size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh, size_t kw, int stride,
		int padding, const float* x, const float* w, const float* b, int fuse_relu, const float* g, float* y, float* dx,
		float* dw, float* db) {
	Value X = leaf({N, Cin, H, W}, x), Wt = leaf({Cout, Cin, kh, kw}, w), B = leaf({Cout}, b);
	Value Y = fuse_relu ? nn::conv2d_relu(X, Wt, B, stride, padding) : nn::conv2d(X, Wt, B, stride, padding);
	copy_out(Y.data(), y);
	backward_with(Y, g);
	copy_out(X.grad(), dx);
	copy_out(Wt.grad(), dw);
	copy_out(B.grad(), db);
}

void ref_maxpool2d(size_t N, size_t C, size_t H, size_t W, size_t k, size_t stride, const float* x, const float* g,
		float* y, float* dx) {
	Value X = leaf({N, C, H, W}, x);
	Value Y = nn::maxpool2d(X, k, stride);
	copy_out(Y.data(), y);
	backward_with(Y, g);
	copy_out(X.grad(), dx);
}

void ref_conv2d_ex(size_t N, size_t Cin, size_t H, size_t W, size_t Cout, size_t kh, size_t kw, int stride,
		int padding, int dilation, int groups, const float* x, const float* w, const float* b, const float* g, float* y,
		float* dx, float* dw, float* db) {
	Value X = leaf({N, Cin, H, W}, x), Wt = leaf({Cout, Cin / (size_t)groups, kh, kw}, w), B = leaf({Cout}, b);
	Value Y = nn::conv2d(X, Wt, B, stride, padding, dilation, groups);
	copy_out(Y.data(), y);
	backward_with(Y, g);
	copy_out(X.grad(), dx);
	copy_out(Wt.grad(), dw);
	copy_out(B.grad(), db);
}

void ref_avgpool2d(size_t N, size_t C, size_t H, size_t W, size_t k, size_t stride, const float* x, const float* g,
		float* y, float* dx) {
	Value X = leaf({N, C, H, W}, x);
	Value Y = nn::avgpool2d(X, k, stride);
	copy_out(Y.data(), y);
	backward_with(Y, g);
	copy_out(X.grad(), dx);
}

// sum (average = 0) or mean over one axis of a 4-D x
void ref_reduce4(size_t n0, size_t n1, size_t n2, size_t n3, int axis, int average, const float* x, const float* g,
		float* y, float* dx) {
	Value X = leaf({n0, n1, n2, n3}, x);
	Value Y = average ? nn::mean(X, axis) : nn::sum(X, axis);
	copy_out(Y.data(), y);
	backward_with(Y, g);
	copy_out(X.grad(), dx);
}

void ref_global_avgpool(size_t N, size_t C, size_t H, size_t W, const float* x, const float* g, float* y, float* dx) {
	Value X = leaf({N, C, H, W}, x);
	nn::GlobalAvgPool2d pool;
	Value Y = pool.forward(X);
	copy_out(Y.data(), y);
	backward_through(Y, g);
	copy_out(X.grad(), dx);
}

// BatchNorm2d(C) module: `train_steps` training-mode forwards on x, then (eval = 1) one
// evaluation-mode forward, or (eval = 0) the last training forward, is returned with its backward
// for the upstream gradient g; the running statistics are copied out after.
void ref_bn2d_module_ex(size_t N, size_t C, size_t H, size_t W, int train_steps, int eval, int fuse_relu, const float* x,
		const float* g, const float* w_in, const float* b_in, float* y, float* dx, float* dw, float* db,
		float* running_mean, float* running_var);

void ref_bn2d_module(size_t N, size_t C, size_t H, size_t W, int train_steps, int eval, int fuse_relu, const float* x,
		const float* g, float* y, float* dx, float* dw, float* db, float* running_mean, float* running_var) {
	ref_bn2d_module_ex(N, C, H, W, train_steps, eval, fuse_relu, x, g, nullptr, nullptr, y, dx, dw, db, running_mean,
		running_var);
}

// The same with the module's weight and bias set from w_in and b_in (C floats each; null keeps the
// defaults 1 and 0).
void ref_bn2d_module_ex(size_t N, size_t C, size_t H, size_t W, int train_steps, int eval, int fuse_relu, const float* x,
		const float* g, const float* w_in, const float* b_in, float* y, float* dx, float* dw, float* db,
		float* running_mean, float* running_var) {
	nn::BatchNorm2d bn(C);
	std::vector<Value> params = bn.parameters();
	if (w_in) std::memcpy(params[0].data().data().data(), w_in, C * sizeof(float));
	if (b_in) std::memcpy(params[1].data().data().data(), b_in, C * sizeof(float));
	Value X = leaf({N, C, H, W}, x);
	Value Y = fuse_relu ? bn.forward_relu(X) : bn.forward(X);
	for (int s = 1; s < train_steps; ++s) {
		X = leaf({N, C, H, W}, x);
		Y = fuse_relu ? bn.forward_relu(X) : bn.forward(X);
	}
	if (eval) {
		bn.train(false);
		X = leaf({N, C, H, W}, x);
		Y = fuse_relu ? bn.forward_relu(X) : bn.forward(X);
	}
	for (Value& p : params) p.zero_grad();
	copy_out(Y.data(), y);
	backward_through(Y, g);
	copy_out(X.grad(), dx);
	copy_out(params[0].grad(), dw);
	copy_out(params[1].grad(), db);
	auto buffers = bn.named_buffers();
	copy_out(*buffers[0].second, running_mean);
	copy_out(*buffers[1].second, running_var);
}

// Sequential{Linear(3, 2)} with weight w [2, 3] and bias b [2]; with grads given, one AdamW step
// (lr, weight_decay, other settings default) first; then save_checkpoint(path, model, optim?, step).
// Returns 0, or 1 when the reference threw.
int ref_linear_checkpoint_save(const char* path, const float* w, const float* b, const float* gw, const float* gb,
		float lr, float wd, int64_t step) {
	try {
		nn::Sequential m;
		m.add(std::make_unique<nn::Linear>(3, 2));
		auto p = m.named_parameters();
		p[0].second.data().data().assign(w, w + 6);
		p[1].second.data().data().assign(b, b + 2);
		if (gw) {
			nn::AdamW opt(m.parameters(), lr, 0.9f, 0.999f, 1e-8f, wd);
			p[0].second.grad().data().assign(gw, gw + 6);
			p[1].second.grad().data().assign(gb, gb + 2);
			opt.step();
			nn::save_checkpoint(path, m, &opt, step);
		} else {
			nn::save_checkpoint(path, m, nullptr, step);
		}
		return 0;
	} catch (...) {
		return 1;
	}
}

// load_checkpoint(path) into Sequential{Linear(3, 2)} (optimizer entries ignored); the step, or -1
// when the reference threw (a malformed or mismatching file).
int64_t ref_linear_checkpoint_load(const char* path, float* w, float* b) {
	try {
		nn::Sequential m;
		m.add(std::make_unique<nn::Linear>(3, 2));
		const int64_t step = nn::load_checkpoint(path, m, nullptr);
		auto p = m.named_parameters();
		copy_out(p[0].second.data(), w);
		copy_out(p[1].second.data(), b);
		return step;
	} catch (...) {
		return -1;
	}
}

// TensorDataset of n samples whose input and target rows are [i] (so a batch shows its indices).
nn::TensorDataset index_dataset(size_t n) {
	std::vector<float> v(n);
	for (size_t i = 0; i < n; i++) v[i] = static_cast<float>(i);
	return nn::TensorDataset(Tensor({n, 1}, v), Tensor({n, 1}, v));
}

// manual_seed(seed), `skip` loaders built first, then DataLoader(index dataset of n, batch, shuffle,
// drop_last); for `epochs` epochs (reset_epoch before each but the first) every batch's inputs in
// order go to out. Returns the number written.
size_t ref_loader_orders(uint64_t seed, int skip, size_t n, size_t batch, int shuffle, int drop_last, int epochs,
		float* out) {
	nn::TensorDataset ds = index_dataset(n);
	nn::manual_seed(seed);
	for (int i = 0; i < skip; i++) nn::DataLoader unused(ds, batch, shuffle != 0);
	nn::DataLoader loader(ds, batch, shuffle != 0, drop_last != 0);
	size_t o = 0;
	for (int e = 0; e < epochs; e++) {
		if (e) loader.reset_epoch();
		for (size_t b = 0; b < loader.num_batches(); b++) {
			auto batch_xy = loader.get_batch(b);
			for (float v : batch_xy.first.data().data()) out[o++] = v;
		}
	}
	return o;
}

// The weighted form: DataLoader(index dataset of n, batch, weights, num_samples, drop_last); the
// targets of every batch of `epochs` epochs. Returns the number written, or -1 when it threw.
long long ref_loader_weighted(uint64_t seed, const double* w, size_t n, size_t batch, size_t num_samples,
		int drop_last, int epochs, float* out) {
	try {
		nn::TensorDataset ds = index_dataset(n);
		nn::manual_seed(seed);
		std::vector<double> weights(w, w + n);
		nn::DataLoader loader(ds, batch, weights, num_samples, drop_last != 0);
		long long o = 0;
		for (int e = 0; e < epochs; e++) {
			if (e) loader.reset_epoch();
			for (size_t b = 0; b < loader.num_batches(); b++) {
				auto batch_xy = loader.get_batch(b);
				for (float v : batch_xy.second.data()) out[o++] = v;
			}
		}
		return o;
	} catch (...) {
		return -1;
	}
}

// random_split(index dataset of n, fractions[0..k), seed): sizes[j] and the subsets' indices in
// order to out. Returns 0, or 1 when it threw.
int ref_random_split(size_t n, const double* fractions, int k, uint64_t seed, size_t* sizes, float* out) {
	try {
		nn::TensorDataset ds = index_dataset(n);
		auto parts = nn::random_split(ds, std::vector<double>(fractions, fractions + k), seed);
		size_t o = 0;
		for (size_t j = 0; j < parts.size(); j++) {
			sizes[j] = parts[j].size();
			for (size_t i = 0; i < parts[j].size(); i++) out[o++] = parts[j].get(i).first.data()[0];
		}
		return 0;
	} catch (...) {
		return 1;
	}
}

// balanced_sample_weights(labels, classes) into out; 0, or 1 when it threw.
int ref_balanced_weights(const size_t* labels, size_t n, size_t classes, double* out) {
	try {
		auto w = nn::balanced_sample_weights(std::vector<size_t>(labels, labels + n), classes);
		std::memcpy(out, w.data(), n * sizeof(double));
		return 0;
	} catch (...) {
		return 1;
	}
}

// Seconds for `batches` get_batch calls of a DataLoader(batch, shuffle) over a TensorDataset of n
// rows of `row` floats (targets one float per row): the reference's host-side batch assembly.
double ref_time_loader(size_t n, size_t row, size_t batch, size_t batches) {
	std::vector<float> x(n * row), y(n);
	for (size_t i = 0; i < x.size(); i++) x[i] = static_cast<float>(i % 251);
	for (size_t i = 0; i < n; i++) y[i] = static_cast<float>(i % 10);
	nn::TensorDataset ds(Tensor({n, row}, x), Tensor({n, 1}, y));
	nn::manual_seed(1);
	nn::DataLoader loader(ds, batch, true);
	const auto t0 = std::chrono::steady_clock::now();
	float sink = 0.0f;
	for (size_t b = 0; b < batches; b++) sink += loader.get_batch(b % loader.num_batches()).second.data()[0];
	const double sec = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
	return sink < -1.0f ? -sec : sec;
}

// Seconds for one save_checkpoint and one load_checkpoint (model and AdamW state) of
// Sequential{Linear(in, out)} at `path`.
double ref_time_checkpoint(const char* path, size_t in, size_t out) {
	nn::Sequential m;
	m.add(std::make_unique<nn::Linear>(in, out));
	nn::AdamW opt(m.parameters(), 1e-3f);
	for (auto& p : m.parameters()) p.grad() = Tensor(p.data().shape(), 0.5f);
	opt.step();
	const auto t0 = std::chrono::steady_clock::now();
	nn::save_checkpoint(path, m, &opt, 1);
	nn::load_checkpoint(path, m, &opt);
	return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

// n outputs of std::mt19937 seeded from std::seed_seq{seeds[0..count)}.
void ref_mt19937_outputs(const uint32_t* seeds, size_t count, size_t n, uint32_t* out) {
	std::seed_seq seq(seeds, seeds + count);
	std::mt19937 g(seq);
	for (size_t i = 0; i < n; i++) out[i] = g();
}

// manual_seed(seed), `skip` derive_generator(stream) calls, then n outputs of the next one.
void ref_derive_outputs(uint64_t seed, const char* stream, int skip, size_t n, uint32_t* out) {
	nn::manual_seed(seed);
	for (int i = 0; i < skip; i++) nn::derive_generator(stream);
	std::mt19937 g = nn::derive_generator(stream);
	for (size_t i = 0; i < n; i++) out[i] = g();
}

// manual_seed(seed), `skip` Dropout layers constructed and dropped, then Dropout(p) applied to
// ones of sizes[0], sizes[1], ... in turn: out gets the masks one after another.
void ref_dropout_masks(uint64_t seed, int skip, float p, const size_t* sizes, int count, float* out) {
	nn::manual_seed(seed);
	for (int i = 0; i < skip; i++) nn::Dropout unused(p);
	nn::Dropout d(p);
	size_t off = 0;
	for (int c = 0; c < count; c++) {
		std::vector<float> ones(sizes[c], 1.0f);
		Value y = d.forward(Value::leaf(Tensor({sizes[c]}, ones), false));
		copy_out(y.data(), out + off);
		off += sizes[c];
	}
}

// The core of MultiHeadAttention::attend's dropout branch (src/nn/attention.cpp:36-47) on q, k, v
// [N, T, D]: split heads, matmul_bt, scaled_masked_softmax, Dropout(p) (taken after
// manual_seed(seed)), matmul, merge heads; then the backward of upstream g. Any output may be null.
void ref_attention_dropout(uint64_t seed, size_t N, size_t T, size_t D, size_t heads, int causal, float p,
		const float* q, const float* k, const float* v, const float* g, float* out, float* dq, float* dk, float* dv) {
	nn::manual_seed(seed);
	nn::Dropout drop(p);
	const size_t Dh = D / heads;
	Value Q = leaf({N, T, D}, q), K = leaf({N, T, D}, k), V = leaf({N, T, D}, v);
	auto split = [&](const Value& x) { return nn::transpose(nn::reshape(x, {N, T, heads, Dh}), {0, 2, 1, 3}); };
	Value scores = nn::matmul_bt(split(Q), split(K));
	Value w = drop.forward(nn::scaled_masked_softmax(scores, 1.0f / std::sqrt(static_cast<float>(Dh)), Tensor({0}),
		causal != 0));
	Value merged = nn::reshape(nn::transpose(nn::matmul(w, split(V)), {0, 2, 1, 3}), {N, T, D});
	backward_through(merged, g);
	copy_out(merged.data(), out);
	copy_out(Q.grad(), dq);
	copy_out(K.grad(), dk);
	copy_out(V.grad(), dv);
}

// manual_seed(seed); MultiHeadAttention(D, heads, causal, p) with params = q.w, q.b, k.w, k.b, v.w,
// v.b, o.w, o.b (flat); `calls` forward + backward passes of x [N, T, D] with upstream gradient g
// (the dropout stream advances between them); y, dx and dparams (flat, same order) of the last.
void ref_mha_dropout(uint64_t seed, size_t N, size_t T, size_t D, size_t heads, int causal, float p, int calls,
		const float* params, const float* x, const float* g, float* y, float* dx, float* dparams) {
	nn::manual_seed(seed);
	nn::MultiHeadAttention mha(D, heads, causal != 0, p);
	auto named = mha.named_parameters();
	size_t off = 0;
	for (auto& q : named) {
		Tensor& d = q.second.data();
		std::memcpy(d.data().data(), params + off, d.size() * sizeof(float));
		off += d.size();
	}
	for (int c = 0; c < calls; c++) {
		for (auto& q : named) q.second.grad() = Tensor(q.second.data().shape(), 0.0f);
		Value X = leaf({N, T, D}, x);
		Value Y = mha.forward(X);
		backward_through(Y, g);
		if (c + 1 == calls) {
			copy_out(Y.data(), y);
			copy_out(X.grad(), dx);
			size_t o = 0;
			for (auto& q : named) {
				copy_out(q.second.grad(), dparams + o);
				o += q.second.data().size();
			}
		}
	}
}

void ref_gelu(size_t n, const float* x, const float* g, float* y, float* dx) {
	Value X = leaf({n}, x);
	Value Y = nn::gelu(X);
	copy_out(Y.data(), y);
	backward_with(Y, g);
	copy_out(X.grad(), dx);
}

void ref_relu(size_t n, const float* x, const float* g, float* y, float* dx) {
	Value X = leaf({n}, x);
	Value Y = nn::relu(X);
	copy_out(Y.data(), y);
	backward_with(Y, g);
	copy_out(X.grad(), dx);
}

void ref_tanh_inplace(float* x, size_t n) { nn::kernels::tanh_inplace(x, n); }

void ref_cross_entropy(size_t N, size_t C, const float* logits, const int64_t* targets, float grad_loss, float* loss,
		float* dlogits) {
	Value L = leaf({N, C}, logits);
	Value out = nn::cross_entropy_loss(L, ids_tensor({N}, targets));
	copy_out(out.data(), loss);
	backward_with(out, &grad_loss);
	copy_out(L.grad(), dlogits);
}

void ref_sequence_ce(size_t N, size_t T, size_t V, const float* logits, const int64_t* targets, int ignore_index,
		float ls, float grad_loss, float* loss, float* dlogits) {
	Value L = leaf({N, T, V}, logits);
	Value out = nn::sequence_cross_entropy(L, ids_tensor({N, T}, targets), ignore_index, ls);
	copy_out(out.data(), loss);
	backward_with(out, &grad_loss);
	copy_out(L.grad(), dlogits);
}

void ref_embedding(size_t V, size_t D, const float* w, const int64_t* ids, size_t count, const float* g, float* out,
		float* dw) {
	Value Wt = leaf({V, D}, w);
	Value Y = nn::embedding(Wt, ids_tensor({count}, ids));
	copy_out(Y.data(), out);
	backward_with(Y, g);
	copy_out(Wt.grad(), dw);
}

/* `steps` AdamW steps on one parameter with the same gradient each step; w updated in place */
void ref_adamw(size_t n, float* w, const float* g, float lr, float b1, float b2, float eps, float wd, int steps) {
	Value P = leaf({n}, w);
	nn::AdamW opt({P}, lr, b1, b2, eps, wd);
	for (int s = 0; s < steps; ++s) {
		std::memcpy(P.grad().data().data(), g, n * sizeof(float));
		opt.step();
	}
	copy_out(P.data(), w);
}

/*
 * Builds nn::Transformer (src/nn/transformer.cpp) with the given parameters (flat, in
 * named_parameters order), then runs `steps` training steps on one batch: zero_grad, forward,
 * sequence_cross_entropy, backward, AdamW step. losses[s] gets each step's loss, grads the first
 * step's gradients (flat), params_out the parameters after the last step. Returns the number of
 * parameter floats, or -1 if the sizes do not match.
 */
long long ref_transformer_train_ex(uint64_t seed, float dropout, size_t vocab, size_t dim, size_t heads, size_t layers,
		size_t max_len, size_t N, size_t T, const float* params_in, const int64_t* ids, const int64_t* targets, float lr,
		float wd, int steps, float* losses, float* grads, float* params_out);

long long ref_transformer_train(size_t vocab, size_t dim, size_t heads, size_t layers, size_t max_len, size_t N,
		size_t T, const float* params_in, const int64_t* ids, const int64_t* targets, float lr, float wd, int steps,
		float* losses, float* grads, float* params_out) {
	return ref_transformer_train_ex(0, 0.0f, vocab, dim, heads, layers, max_len, N, T, params_in, ids, targets, lr, wd,
		steps, losses, grads, params_out);
}

// The same with manual_seed(seed) before the model is built and dropout in its config.
long long ref_transformer_train_ex(uint64_t seed, float dropout, size_t vocab, size_t dim, size_t heads, size_t layers,
		size_t max_len, size_t N, size_t T, const float* params_in, const int64_t* ids, const int64_t* targets, float lr,
		float wd, int steps, float* losses, float* grads, float* params_out) {
	nn::manual_seed(seed);
	nn::TransformerConfig c{vocab, dim, heads, layers, max_len};
	c.dropout = dropout;
	nn::Transformer model(c);
	std::vector<std::pair<std::string, Value>> named = model.named_parameters();
	size_t off = 0;
	for (auto& p : named) {
		Tensor& d = p.second.data();
		std::memcpy(d.data().data(), params_in + off, d.size() * sizeof(float));
		off += d.size();
	}
	nn::AdamW opt(model.parameters(), lr, 0.9f, 0.999f, 1e-8f, wd);
	Value idv = Value::leaf(ids_tensor({N, T}, ids), false);
	Tensor tg = ids_tensor({N, T}, targets);
	for (int st = 0; st < steps; ++st) {
		opt.zero_grad();
		Value logits = model.forward(idv);
		Value loss = nn::sequence_cross_entropy(logits, tg);
		loss.backward();
		losses[st] = loss.data().data()[0];
		if (st == 0 && grads) {
			size_t g = 0;
			for (auto& p : named) {
				Tensor& gr = p.second.grad();
				std::memcpy(grads + g, gr.data().data(), gr.size() * sizeof(float));
				g += gr.size();
			}
		}
		opt.step();
	}
	size_t o = 0;
	for (auto& p : named) {
		Tensor& d = p.second.data();
		std::memcpy(params_out + o, d.data().data(), d.size() * sizeof(float));
		o += d.size();
	}
	return static_cast<long long>(off);
}

/*
 * The config-2 CNN (conv2d_relu 1->32, maxpool 2, conv2d_relu 32->64, maxpool 2, flatten,
 * linear 3136->128, relu, linear 128->10, cross_entropy_loss) composed from the reference's ops,
 * as Sequential runs it (src/nn/sequential.cpp:16-28): one forward and backward. params and grads
 * are flat in order conv1.w, conv1.b, conv2.w, conv2.b, fc1.w, fc1.b, fc2.w, fc2.b.
 */
void ref_cnn_fwd_bwd_ex(size_t N, const float* x, const int64_t* labels, const float* params, float* loss,
		float* logits_out, float* grads, float* fc1_out);

void ref_cnn_fwd_bwd(size_t N, const float* x, const int64_t* labels, const float* params, float* loss,
		float* logits_out, float* grads) {
	ref_cnn_fwd_bwd_ex(N, x, labels, params, loss, logits_out, grads, nullptr);
}

// The same, also giving fc1's output before its ReLU (N x 128) in fc1_out when not null.
void ref_cnn_fwd_bwd_ex(size_t N, const float* x, const int64_t* labels, const float* params, float* loss,
		float* logits_out, float* grads, float* fc1_out) {
	const std::vector<std::vector<size_t>> shapes = {{32, 1, 3, 3}, {32}, {64, 32, 3, 3}, {64}, {128, 3136}, {128},
		{10, 128}, {10}};
	std::vector<Value> P;
	size_t off = 0;
	for (const auto& sh : shapes) {
		P.push_back(leaf(sh, params + off));
		off += count_of(sh);
	}
	Value X = Value::leaf(tensor({N, 1, 28, 28}, x), false);
	Value h = nn::conv2d_relu(X, P[0], P[1], 1, 1);
	h = nn::maxpool2d(h, 2, 2);
	h = nn::conv2d_relu(h, P[2], P[3], 1, 1);
	h = nn::maxpool2d(h, 2, 2);
	h = nn::reshape(h, {N, 3136});
	h = nn::linear(h, P[4], P[5]);
	copy_out(h.data(), fc1_out);
	h = nn::relu(h);
	Value logits = nn::linear(h, P[6], P[7]);
	Value L = nn::cross_entropy_loss(logits, ids_tensor({N}, labels));
	L.backward();
	copy_out(L.data(), loss);
	copy_out(logits.data(), logits_out);
	size_t g = 0;
	for (const Value& p : P) {
		copy_out(p.grad(), grads + g);
		g += p.data().size();
	}
}

}  // extern "C"
