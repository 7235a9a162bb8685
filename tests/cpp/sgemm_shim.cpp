// A driver for the drop-in a maintainer of nn-cpp would add for its GEMM seam, nn::kernels::sgemm
// (include/nn/kernels/gemm.hpp:57-59, src/kernels/gemm.cpp:546-556; the drop-in itself is
// nn-cpp_b200/host/nn_kernels_gemm.cpp): the same signature, host buffers in and C written on
// return, forwarded to the C ABI's host-buffer entry. Compiled as C++17 against include/nnb.h together
// with the drop-in and linked with libnnb.so by tests/test_cpp_host.py:
//
//   sgemm_shim checks
//       host-side paths only, no GPU needed: the library's version, the empty products the
//       reference returns from at once (gemm.cpp:345), and the argument errors the library rejects
//       before any device work (thrown as std::invalid_argument by the shim)
//   sgemm_shim run ta tb m n k lda ldb ldc accumulate in.bin out.bin
//       A, B and C (float32, row-major with the given leading dimensions, one after the other) from
//       in.bin; one nn::kernels::sgemm; C to out.bin
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <vector>

#include "nnb.h"

// nn::kernels::sgemm as include/nn/kernels/gemm.hpp:57-59 declares it; the definition is the
// drop-in nn-cpp_b200/host/nn_kernels_gemm.cpp, compiled with this file.
namespace nn {
namespace kernels {
void sgemm(bool trans_a, bool trans_b, size_t m, size_t n, size_t k, const float* a, size_t lda, const float* b,
		size_t ldb, float* c, size_t ldc, bool accumulate);
}  // namespace kernels
}  // namespace nn

namespace {

int checks() {
	std::printf("version %s\n", nnb_version());
	float a[4] = {1, 2, 3, 4}, b[4] = {5, 6, 7, 8}, c[4] = {-1, -1, -1, -1};
	nn::kernels::sgemm(false, false, 0, 2, 2, a, 2, b, 2, c, 2, false);     // m == 0: nothing
	nn::kernels::sgemm(false, false, 2, 0, 2, a, 2, b, 2, c, 2, false);     // n == 0: nothing
	for (float v : c)
		if (v != -1.0f) {
			std::printf("empty product wrote C\n");
			return 1;
		}
	int rejected = 0;
	try {
		nn::kernels::sgemm(false, false, 2, 2, 2, a, 2, b, 2, c, 1, false);  // ldc < n
	} catch (const std::invalid_argument& e) {
		std::printf("invalid_argument: %s\n", e.what());
		++rejected;
	}
	try {
		nn::kernels::sgemm(false, true, 2, 2, 3, a, 2, b, 2, c, 2, false);   // B stored n x k: ldb < k
	} catch (const std::invalid_argument& e) {
		std::printf("invalid_argument: %s\n", e.what());
		++rejected;
	}
	try {
		nn::kernels::sgemm(false, false, 2, 2, 2, nullptr, 2, b, 2, c, 2, false);
	} catch (const std::invalid_argument& e) {
		std::printf("invalid_argument: %s\n", e.what());
		++rejected;
	}
	if (rejected != 3) {
		std::printf("expected 3 rejections, got %d\n", rejected);
		return 1;
	}
	std::printf("checks ok\n");
	return 0;
}

int run(char** argv) {
	const bool ta = std::atoi(argv[0]) != 0, tb = std::atoi(argv[1]) != 0;
	const size_t m = std::strtoull(argv[2], nullptr, 10), n = std::strtoull(argv[3], nullptr, 10);
	const size_t k = std::strtoull(argv[4], nullptr, 10), lda = std::strtoull(argv[5], nullptr, 10);
	const size_t ldb = std::strtoull(argv[6], nullptr, 10), ldc = std::strtoull(argv[7], nullptr, 10);
	const bool acc = std::atoi(argv[8]) != 0;
	const size_t na = (ta ? k : m) * lda, nb = (tb ? n : k) * ldb, nc = m * ldc;
	std::vector<float> a(na), b(nb), c(nc);
	FILE* in = std::fopen(argv[9], "rb");
	if (!in) return 2;
	const bool read_ok = std::fread(a.data(), sizeof(float), na, in) == na &&
		std::fread(b.data(), sizeof(float), nb, in) == nb && std::fread(c.data(), sizeof(float), nc, in) == nc;
	std::fclose(in);
	if (!read_ok) return 2;
	nn::kernels::sgemm(ta, tb, m, n, k, a.data(), lda, b.data(), ldb, c.data(), ldc, acc);
	FILE* out = std::fopen(argv[10], "wb");
	if (!out) return 2;
	const bool write_ok = std::fwrite(c.data(), sizeof(float), nc, out) == nc;
	std::fclose(out);
	return write_ok ? 0 : 2;
}

}  // namespace

int main(int argc, char** argv) {
	try {
		if (argc == 2 && std::string(argv[1]) == "checks") return checks();
		if (argc == 13 && std::string(argv[1]) == "run") return run(argv + 2);
	} catch (const std::exception& e) {
		std::printf("error: %s\n", e.what());
		return 3;
	}
	std::fprintf(stderr, "usage: %s checks | run ta tb m n k lda ldb ldc accumulate in.bin out.bin\n", argv[0]);
	return 2;
}
