/*
 * orc_gen.cpp -- seeded input generators for the parity tests and the CPU baseline.
 * TEST INFRASTRUCTURE ONLY (tests/, smoke() and bench.py's cpu_baseline / reference legs).
 *
 * The reference draws every synthetic input from libstdc++'s std::mt19937 through
 * std::uniform_real_distribution<float> or std::normal_distribution<float>:
 *   - tests/test_kernels.cpp:68-86 (make_problem: U[-1,1], A then B then C, row by row,
 *     padding columns of every leading dimension filled with the sentinel 1e30f);
 *   - apps/bench/runner.cpp:80-96 (run_matmul: mt19937(seed), U[-1,1], A then B).
 * Generating through the same library objects gives the CUDA path, the oracle and the
 * reference build bit-identical inputs.
 */
#include <cstddef>
#include <cstdint>
#include <random>

extern "C" {

/* n draws of U[lo, hi) from mt19937(seed), in order (runner.cpp:81-85 pattern) */
void orc_fill_uniform(uint32_t seed, size_t n, float lo, float hi, float* out) {
	std::mt19937 gen(seed);
	std::uniform_real_distribution<float> dist(lo, hi);
	for (size_t i = 0; i < n; ++i) out[i] = dist(gen);
}

/* n draws of N(mean, stddev) from mt19937(seed) */
void orc_fill_normal(uint32_t seed, size_t n, float mean, float stddev, float* out) {
	std::mt19937 gen(seed);
	std::normal_distribution<float> dist(mean, stddev);
	for (size_t i = 0; i < n; ++i) out[i] = dist(gen);
}

/* n draws of U{lo..hi} (inclusive) from mt19937(seed), e.g. class labels and token ids */
void orc_fill_int(uint32_t seed, size_t n, int64_t lo, int64_t hi, int64_t* out) {
	std::mt19937 gen(seed);
	std::uniform_int_distribution<int64_t> dist(lo, hi);
	for (size_t i = 0; i < n; ++i) out[i] = dist(gen);
}

/*
 * test_kernels.cpp:68-86: one GEMM problem. a has (ta ? k : m) rows of lda = cols + pad,
 * b has (tb ? n : k) rows of ldb = cols + pad, c has m rows of ldc = n + pad; the caller
 * sizes the buffers. Values in [-1, 1], padding = 1e30f.
 */
void orc_make_problem(int ta, int tb, size_t m, size_t n, size_t k, size_t pad, uint32_t seed,
		float* a, float* b, float* c) {
	const float sentinel = 1e30f;
	std::mt19937 gen(seed);
	std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
	auto fill = [&](float* v, size_t rows, size_t cols, size_t ld) {
		for (size_t i = 0; i < rows * ld; ++i) v[i] = sentinel;
		for (size_t r = 0; r < rows; ++r)
			for (size_t col = 0; col < cols; ++col) v[r * ld + col] = dist(gen);
	};
	const size_t a_rows = ta ? k : m, a_cols = ta ? m : k;
	const size_t b_rows = tb ? n : k, b_cols = tb ? k : n;
	fill(a, a_rows, a_cols, a_cols + pad);
	fill(b, b_rows, b_cols, b_cols + pad);
	fill(c, m, n, n + pad);
}

}  // extern "C"
