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
#include "nn/kernels/gemm.hpp"
#include "nn/kernels/parallel.hpp"
#include "nn/tensor.hpp"
#include "reference_gemm.hpp"   // the reference's own test oracle, tests/reference_gemm.hpp

#include <chrono>
#include <cstddef>
#include <cstring>
#include <vector>

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

}  // extern "C"
