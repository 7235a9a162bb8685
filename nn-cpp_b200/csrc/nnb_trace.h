// nnb_trace.h -- RAII scope placed around every kernel launch of the library (see trace.cu).
#pragma once

#include <cuda_runtime.h>

namespace nnb {

// Kernel kinds, the `kind` argument of nnb_trace_query (values fixed by include/nnb.h).
enum TraceKind : int {
	kTraceGemm = 0,       // tcgen05 GEMM main kernel
	kTracePack = 1,       // operand pack / TF32 split
	kTraceAux = 2,        // fills and other small helpers
	kTraceRowwise = 3,    // layernorm / batchnorm / softmax / elementwise kernels
	kTraceAttention = 4,  // fused attention kernels
	kTraceConv = 5,       // convolution helpers (im2col / col2im style gathers)
	kTraceKinds = 6
};

class TraceScope {
public:
	// enabled = false: the scope does nothing at all (no event, no count), for entry points that
	// must not create CUDA objects.
	TraceScope(cudaStream_t s, int kind, bool enabled = true);
	~TraceScope();
	TraceScope(const TraceScope&) = delete;
	TraceScope& operator=(const TraceScope&) = delete;

private:
	cudaStream_t s_;
	int kind_;
	cudaEvent_t start_ = nullptr, stop_ = nullptr;
};

}  // namespace nnb
