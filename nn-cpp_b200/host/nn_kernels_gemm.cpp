// nn_kernels_gemm.cpp -- the drop-in for nn-cpp's GEMM translation unit (src/kernels/gemm.cpp):
// every function include/nn/kernels/gemm.hpp declares, with the same signatures and contract, on the
// B200 through the C ABI's host-buffer entry (nnb_sgemm_host: host pointers in, C written on return).
//
// Built in place of the reference's src/kernels/gemm.cpp and linked with libnnb.so, it puts every
// caller of the seam on the GPU unchanged: Tensor::matmul (src/tensor.cpp:593,622), linear
// (src/autograd/ops.cpp:725-741), the matmul / matmul_bt backward folds (ops.cpp:695-760), attention
// (ops.cpp:1256-1292) and the convolutions (ops.cpp:1395-1452, 1557-1587) -- and through them the
// Linear, MultiHeadAttention, Conv2d and TransformerBlock modules.
//
// - sgemm: 3xTF32 by default (fp32-grade; nnb_set_math_mode(NNB_MATH_TF32) selects the fast mode).
//   m == 0 or n == 0 returns at once and k == 0 stores zeros (or leaves C when accumulating), as
//   gemm.cpp:345-350; only the m x n region of C is written.
// - sgemm_portable / sgemm_unpacked: the reference keeps them as alternative CPU kernels with the same
//   contract for its tests; here they take the same GPU path.
// - sgemm_uses_avx2: false (no CPU microkernel is compiled).
// - Errors: arguments the C ABI rejects (a leading dimension below the row width, a null operand)
//   throw std::invalid_argument before any device work; a device failure throws std::runtime_error.
//   The reference's sgemm reports no errors, so its callers never see either for valid arguments.
// - Threads: callable from any thread; the library orders calls per device, as the reference's pool
//   serialises jobs.
#include <cstddef>
#include <stdexcept>

#include "nnb.h"

namespace nn {
namespace kernels {

namespace {

void on_device(bool trans_a, bool trans_b, size_t m, size_t n, size_t k, const float* a, size_t lda, const float* b,
		size_t ldb, float* c, size_t ldc, bool accumulate) {
	const nnb_status st = nnb_sgemm_host(trans_a, trans_b, m, n, k, a, lda, b, ldb, c, ldc, accumulate);
	if (st == NNB_ERR_INVALID || st == NNB_ERR_SHAPE) throw std::invalid_argument(nnb_last_error());
	if (st != NNB_OK) throw std::runtime_error(nnb_last_error());
}

}  // namespace

void sgemm(bool trans_a, bool trans_b, size_t m, size_t n, size_t k, const float* a, size_t lda, const float* b,
		size_t ldb, float* c, size_t ldc, bool accumulate) {
	on_device(trans_a, trans_b, m, n, k, a, lda, b, ldb, c, ldc, accumulate);
}

void sgemm_portable(bool trans_a, bool trans_b, size_t m, size_t n, size_t k, const float* a, size_t lda,
		const float* b, size_t ldb, float* c, size_t ldc, bool accumulate) {
	on_device(trans_a, trans_b, m, n, k, a, lda, b, ldb, c, ldc, accumulate);
}

void sgemm_unpacked(bool trans_a, bool trans_b, size_t m, size_t n, size_t k, const float* a, size_t lda,
		const float* b, size_t ldb, float* c, size_t ldc, bool accumulate) {
	on_device(trans_a, trans_b, m, n, k, a, lda, b, ldb, c, ldc, accumulate);
}

bool sgemm_uses_avx2() { return false; }

}  // namespace kernels
}  // namespace nn
