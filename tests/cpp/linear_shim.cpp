// The op-level seam as C++17 host code over device-resident storage: nn-cpp's `linear` forward and
// backward (include/nn/autograd/ops.hpp:304, src/autograd/ops.cpp:714-745) through the C ABI's
// nnb_linear_fwd / nnb_linear_bwd, the buffers allocated with cudaMalloc and the calls ordered on
// one CUDA stream, each gradient stored as a first write (Value::grad_accum, src/autograd/value.cpp:60-64).
// Compiled against include/nnb.h and the CUDA runtime by tests/test_cpp_host.py:
//
//   linear_shim M K n in.bin out.bin
//       x (M x K), w (n x K), b (n), g (M x n) as float32 from in.bin;
//       y = x w^T + b, then dx, dw, db for the upstream gradient g; y, dx, dw, db to out.bin
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime_api.h>

#include "nnb.h"

namespace {

void check(nnb_status st) {
	if (st == NNB_ERR_INVALID) throw std::invalid_argument(nnb_last_error());
	if (st == NNB_ERR_SHAPE) throw std::length_error(nnb_last_error());
	if (st != NNB_OK) throw std::runtime_error(nnb_last_error());
}

void cuda(cudaError_t e) {
	if (e != cudaSuccess) throw std::runtime_error(cudaGetErrorString(e));
}

// A device-resident float buffer: the Storage of a Tensor living in HBM.
struct DeviceBuffer {
	float* ptr = nullptr;
	size_t n = 0;
	explicit DeviceBuffer(size_t count) : n(count) { cuda(cudaMalloc(reinterpret_cast<void**>(&ptr), count * 4 + 4)); }
	~DeviceBuffer() { cudaFree(ptr); }
	DeviceBuffer(const DeviceBuffer&) = delete;
	DeviceBuffer& operator=(const DeviceBuffer&) = delete;
	void upload(const float* src, cudaStream_t s) { cuda(cudaMemcpyAsync(ptr, src, n * 4, cudaMemcpyHostToDevice, s)); }
	void download(float* dst, cudaStream_t s) const {
		cuda(cudaMemcpyAsync(dst, ptr, n * 4, cudaMemcpyDeviceToHost, s));
	}
};

int run(size_t M, size_t K, size_t n, const char* in_path, const char* out_path) {
	std::vector<float> x(M * K), w(n * K), b(n), g(M * n);
	FILE* in = std::fopen(in_path, "rb");
	if (!in) return 2;
	bool ok = std::fread(x.data(), 4, x.size(), in) == x.size() && std::fread(w.data(), 4, w.size(), in) == w.size() &&
		std::fread(b.data(), 4, b.size(), in) == b.size() && std::fread(g.data(), 4, g.size(), in) == g.size();
	std::fclose(in);
	if (!ok) return 2;

	cudaStream_t s = nullptr;
	cuda(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
	std::vector<float> y(M * n), dx(M * K), dw(n * K), db(n);
	{
		DeviceBuffer dx_d(M * K), dw_d(n * K), db_d(n), x_d(M * K), w_d(n * K), b_d(n), g_d(M * n), y_d(M * n);
		x_d.upload(x.data(), s);
		w_d.upload(w.data(), s);
		b_d.upload(b.data(), s);
		g_d.upload(g.data(), s);
		check(nnb_linear_fwd(s, M, K, n, x_d.ptr, w_d.ptr, b_d.ptr, y_d.ptr));
		check(nnb_linear_bwd(s, M, K, n, g_d.ptr, x_d.ptr, w_d.ptr, dx_d.ptr, 1, dw_d.ptr, 1, db_d.ptr, 1));
		y_d.download(y.data(), s);
		dx_d.download(dx.data(), s);
		dw_d.download(dw.data(), s);
		db_d.download(db.data(), s);
		cuda(cudaStreamSynchronize(s));
	}
	cuda(cudaStreamDestroy(s));

	FILE* out = std::fopen(out_path, "wb");
	if (!out) return 2;
	ok = std::fwrite(y.data(), 4, y.size(), out) == y.size() && std::fwrite(dx.data(), 4, dx.size(), out) == dx.size() &&
		std::fwrite(dw.data(), 4, dw.size(), out) == dw.size() && std::fwrite(db.data(), 4, db.size(), out) == db.size();
	std::fclose(out);
	return ok ? 0 : 2;
}

}  // namespace

int main(int argc, char** argv) {
	if (argc != 6) {
		std::fprintf(stderr, "usage: %s M K n in.bin out.bin\n", argv[0]);
		return 2;
	}
	try {
		return run(std::strtoull(argv[1], nullptr, 10), std::strtoull(argv[2], nullptr, 10),
			std::strtoull(argv[3], nullptr, 10), argv[4], argv[5]);
	} catch (const std::exception& e) {
		std::printf("error: %s\n", e.what());
		return 3;
	}
}
