// nnb_math.cuh -- element functions shared by the epilogues and the elementwise kernels.
//
// exp_one / tanh_one restate nn-cpp's own vector-math method (src/kernels/vmath.cpp:22-109): the
// Cephes expf reduction x = n*ln2 + r with ln2 split in two, a degree-5 polynomial, the 2^n scale
// built in the exponent bits, and tanh(x) = (e^{2x} - 1) / (e^{2x} + 1) on x clamped to +-9. They
// are built only from correctly rounded multiply, add and divide (the library is compiled with
// --fmad=false, the counterpart of the reference's -ffp-contract=off), so every value has the
// reference's bits.
#pragma once

#include <cstdint>

namespace nnb {

__device__ __forceinline__ float exp_one(float x) {
	constexpr float kExpLo = -87.3f, kExpHi = 88.3f;
	constexpr float kLog2e = 1.44269504088896341f;
	constexpr float kLn2Hi = 0.693359375f, kLn2Lo = -2.12194440e-4f;
	constexpr float kP0 = 1.9875691500e-4f, kP1 = 1.3981999507e-3f, kP2 = 8.3334519073e-3f;
	constexpr float kP3 = 4.1665795894e-2f, kP4 = 1.6666665459e-1f, kP5 = 5.0000001201e-1f;
	if (x != x) return x;
	if (x < kExpLo) return 0.0f;
	if (x > kExpHi) return __int_as_float(0x7f800000);
	const float n = rintf(x * kLog2e);   // round half to even, as nearbyint in the default mode
	float r = x - n * kLn2Hi;
	r = r - n * kLn2Lo;
	float p = kP0;
	p = p * r + kP1;
	p = p * r + kP2;
	p = p * r + kP3;
	p = p * r + kP4;
	p = p * r + kP5;
	const float e = (p * (r * r) + r) + 1.0f;
	const float pow2 = __int_as_float(((int)n + 127) << 23);
	return e * pow2;
}

__device__ __forceinline__ float tanh_one(float x) {
	constexpr float kTanhMax = 9.0f;
	if (x != x) return x;
	float z = x < -kTanhMax ? -kTanhMax : x;
	z = kTanhMax < z ? kTanhMax : z;
	const float e = exp_one(z + z);
	return (e - 1.0f) / (e + 1.0f);
}

// tanh-GELU of src/autograd/ops.cpp:451-466: th = tanh(k * (x + c*x*x*x)), y = 0.5*x*(1 + th).
constexpr float kGeluK = 0.7978845608f;
constexpr float kGeluC = 0.044715f;

__device__ __forceinline__ float gelu_tanh_arg(float x) { return kGeluK * (x + kGeluC * x * x * x); }

__device__ __forceinline__ float gelu_fwd(float x, float th) { return 0.5f * x * (1.0f + th); }

// d gelu / dx given the saved tanh (ops.cpp:474-477), times the incoming gradient g
__device__ __forceinline__ float gelu_bwd(float g, float x, float th) {
	return g * (0.5f * (1.0f + th) + 0.5f * x * (1.0f - th * th) * kGeluK * (1.0f + 3.0f * kGeluC * x * x));
}

}  // namespace nnb
