/*
 * orc_gemm.c -- CPU oracle for the GEMM path. TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and the cpu_baseline / reference legs of
 * bench.py load this code, and only to check or to time beside the CUDA path.
 * No product code path calls it.
 *
 * Restates the ground truth of the reference's kernel tests:
 *   - orc_sgemm_f32 is the plain triple loop of tests/reference_gemm.hpp:30-45
 *     (fp32 accumulator, same op(A)/op(B) indexing, "accumulate" adds the sum to C);
 *   - orc_sgemm_f64 is the same loop with a double accumulator and double output,
 *     the fp64 evaluation the accuracy bound (1e-5*sqrt(K), TF32 5e-3) is taken against;
 *   - orc_magnitude is tests/test_kernels.cpp:101-109: sum over p of |op(A)(i,p)*op(B)(p,j)|
 *     (+|C(i,j)| when accumulating), the scale every relative tolerance is measured in.
 *
 * Pinned against the reference itself: tests/test_oracle.py compares orc_sgemm_f32 with the
 * reference's own nn::kernels::sgemm (built from its sources by oracle/Makefile into
 * oracle/_ref/) and with the committed golden vectors in tests/golden/.
 *
 * Compiled with -ffp-contract=off like the reference (CMakeLists.txt:63-65), so no FMA
 * contraction changes the fp32 loop's bits.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

/* op(A)(i,p): A stored m x k (row-major, ld lda), or k x m read transposed (reference_gemm.hpp:34) */
static inline float op_a(int ta, const float* a, size_t lda, size_t i, size_t p) {
	return ta ? a[p * lda + i] : a[i * lda + p];
}

/* op(B)(p,j): B stored k x n, or n x k read transposed (reference_gemm.hpp:35) */
static inline float op_b(int tb, const float* b, size_t ldb, size_t p, size_t j) {
	return tb ? b[j * ldb + p] : b[p * ldb + j];
}

/* fp32 triple loop, bit-for-bit the reference's reference_sgemm (tests/reference_gemm.hpp:30-45) */
void orc_sgemm_f32(int ta, int tb, size_t m, size_t n, size_t k,
		const float* a, size_t lda, const float* b, size_t ldb,
		float* c, size_t ldc, int accumulate) {
	for (size_t i = 0; i < m; ++i) {
		for (size_t j = 0; j < n; ++j) {
			float sum = 0.0f;
			for (size_t p = 0; p < k; ++p) sum += op_a(ta, a, lda, i, p) * op_b(tb, b, ldb, p, j);
			c[i * ldc + j] = accumulate ? c[i * ldc + j] + sum : sum;
		}
	}
}

/*
 * fp64 twin of the loop above. c_in (may be NULL when !accumulate) holds the prior C with
 * leading dimension ldc; out receives m x n doubles with leading dimension n.
 */
void orc_sgemm_f64(int ta, int tb, size_t m, size_t n, size_t k,
		const float* a, size_t lda, const float* b, size_t ldb,
		const float* c_in, size_t ldc, int accumulate, double* out) {
	for (size_t i = 0; i < m; ++i) {
		for (size_t j = 0; j < n; ++j) {
			double sum = 0.0;
			for (size_t p = 0; p < k; ++p)
				sum += (double)op_a(ta, a, lda, i, p) * (double)op_b(tb, b, ldb, p, j);
			out[i * n + j] = accumulate ? (double)c_in[i * ldc + j] + sum : sum;
		}
	}
}

/* test_kernels.cpp:101-109, evaluated in double; out is m x n with leading dimension n */
void orc_magnitude(int ta, int tb, size_t m, size_t n, size_t k,
		const float* a, size_t lda, const float* b, size_t ldb,
		const float* c_in, size_t ldc, int accumulate, double* out) {
	for (size_t i = 0; i < m; ++i) {
		for (size_t j = 0; j < n; ++j) {
			double s = accumulate ? fabs((double)c_in[i * ldc + j]) : 0.0;
			for (size_t p = 0; p < k; ++p)
				s += fabs((double)op_a(ta, a, lda, i, p) * (double)op_b(tb, b, ldb, p, j));
			out[i * n + j] = s;
		}
	}
}

/*
 * fp64 values and magnitudes of a sample of C elements: (rows[s], cols[s]) for s < count.
 * Used at sizes where the full triple loop is too slow (the sampled check of large shapes).
 */
void orc_sgemm_f64_sample(int ta, int tb, size_t k,
		const float* a, size_t lda, const float* b, size_t ldb,
		const float* c_in, size_t ldc, int accumulate,
		const int64_t* rows, const int64_t* cols, size_t count, double* val, double* mag) {
	for (size_t s = 0; s < count; ++s) {
		const size_t i = (size_t)rows[s], j = (size_t)cols[s];
		double sum = 0.0, m = 0.0;
		for (size_t p = 0; p < k; ++p) {
			const double t = (double)op_a(ta, a, lda, i, p) * (double)op_b(tb, b, ldb, p, j);
			sum += t;
			m += fabs(t);
		}
		if (accumulate) {
			sum += (double)c_in[i * ldc + j];
			m += fabs((double)c_in[i * ldc + j]);
		}
		val[s] = sum;
		mag[s] = m;
	}
}
