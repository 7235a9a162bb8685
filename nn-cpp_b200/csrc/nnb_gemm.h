// nnb_gemm.h -- the library-internal GEMM interface used by every op built on the tensor-core
// GEMM (linear, attention, convolution, batched matmul).
#pragma once

#include <cuda_runtime.h>

#include "../../include/nnb.h"

namespace nnb {

enum GemmBias : int { kBiasNone = 0, kBiasCol = 1, kBiasRow = 2 };
enum GemmAct : int { kActNone = 0, kActRelu = 1, kActGelu = 2 };

// What the epilogue does to each element v = sum_p op(A)(i,p) op(B)(p,j) before it is stored:
//   v = v + 0                 (so a zero result is +0, as the reference's zero-started sums)
//   v = v + bias[j] or bias[i]              (bias_mode)
//   relu: alive = v > 0, v = alive ? v : 0, mask(i,j) = alive
//   gelu: pre(i,j) = v, v = 0.5 v (1 + tanh_one(k (v + c v^3)))
//   C(i,j) = accumulate ? C(i,j) + v : v
struct GemmEpilogue {
	const float* bias = nullptr;
	int bias_mode = kBiasNone;
	int act = kActNone;
	unsigned char* mask = nullptr;      // relu alive flags, same (i, j) layout as C with ld_aux
	float* pre = nullptr;               // gelu pre-activation, same (i, j) layout as C with ld_aux
	long long ld_aux = 0, s_aux_outer = 0, s_aux_inner = 0;
	long long s_bias_outer = 0;         // floats between the biases of consecutive outer batch entries
};

// A B operand gathered on the fly from a 4-D tensor [N, C, H, W] into the GEMM's shared-memory stages
// (implicit GEMM: no column matrix in global memory). Batch entry e = (o, i) reads
// src + o * s_outer + i * s_inner; op(B)^T element (j, k) of that entry is, by mode:
//   kGatherIm2col     conv forward, j = output position (oh, ow), k = (c, ph, pw):
//                     src[c][oh*stride + ph*dil - pad][ow*stride + pw*dil - pad], 0 outside
//   kGatherTransposed conv input gradient, j = input position (ih, iw), k = (ph, pw, co), src the
//                     output gradient [co][oh][ow] at oh = (ih + pad - ph*dil) / stride (and ow
//                     likewise) when that divides exactly and lands inside, else 0
//   kGatherIm2colRows conv weight gradient, j = (c, ph, pw), k = output position (oh, ow):
//                     src[c][oh*stride + ph*dil - pad][ow*stride + pw*dil - pad], 0 outside
// C, H, W are the gathered tensor's channels (per batch entry) and plane; ho, wo the conv output plane.
enum GatherMode : int { kGatherNone = 0, kGatherIm2col = 1, kGatherTransposed = 2, kGatherIm2colRows = 3 };
struct GemmGather {
	int mode = kGatherNone;
	const float* src = nullptr;
	long long s_outer = 0, s_inner = 0;
	int C = 0, H = 0, W = 0, ho = 0, wo = 0, kh = 1, kw = 1, stride = 1, pad = 0, dil = 1, cout = 0;
};

// A row pack kept by an earlier product (GemmDesc::keep_a): the panels of a row-major matrix X
// [rows x cols] (leading dimension ld, first element `base`) packed as that product's A operand, in
// math mode `mode`. Buffer layout (gemm_row_pack_bytes): the panels of round_up(rows, 256) rows x
// round_up(cols, 32) depths (128-row panels, 32 floats wide, hi[, lo]), then one non-finite flag per
// padded row, then the any-non-finite flag.
struct GemmRowPack {
	const void* buf = nullptr;
	const float* base = nullptr;
	long long ld = 0, rows = 0, cols = 0;
	int mode = NNB_MATH_FP32X3;
};

// C_e = op(A_e) op(B_e) for batch entries e = (o, i), o < batch_outer, i < batch_inner, where
// X_e = x + o * sx_outer + i * sx_inner (floats). A zero stride shares the operand.
struct GemmDesc {
	int ta = 0, tb = 0;
	long long m = 0, n = 0, k = 0;
	const float* a = nullptr;
	long long lda = 0;
	const float* b = nullptr;
	long long ldb = 0;
	float* c = nullptr;
	long long ldc = 0;
	long long batch_outer = 1, batch_inner = 1;
	long long sa_outer = 0, sa_inner = 0, sb_outer = 0, sb_inner = 0, sc_outer = 0, sc_inner = 0;
	int accumulate = 0;
	int mode = NNB_MATH_FP32X3;
	GemmEpilogue epi;
	// B already in the packed panel layout, written by gemm_pack_b for this n, k, math mode and tile
	// width (one batch entry, no depth cut); b/ldb stay the unpacked operand (non-finite fix-ups)
	const void* packed_b = nullptr;
	int bn = 0;                         // tile width: 0 chooses it from the shape; 64, 128 or 256
	// B gathered by the GEMM kernel itself (b, ldb, sb_*, tb unused); never cut along its depth
	GemmGather gather;
	// A (not transposed, shared by every batch entry) packed into this caller buffer of
	// gemm_row_pack_bytes(m, k, mode) bytes instead of the scratch, and left there for later products
	// (mn_a / mn_b)
	void* keep_a = nullptr;
	// Operands read from a kept row pack instead of being packed: A = X^T (ta = 1, a and lda inside
	// X) through mn_a, B = X (tb = 0, b and ldb inside X) through mn_b. The tensor core reads them
	// MN-major straight from the 32-wide panels, so a weight gradient G^T X reuses the packs the
	// forward product (X) and the input-gradient product (G) already wrote. Used only when every
	// batch entry starts on a 16-row boundary of X and k % 16 == 0 (otherwise packed as usual); the
	// result has the same bits either way.
	GemmRowPack mn_a, mn_b;
	// A (ta = 0) read K-major from a kept row pack of the matrix it lies in, at a column offset of
	// whole 16-column blocks (a depth piece of a product whose A was kept: gemm_run packs a kept A
	// once and hands every piece its columns this way). Ignored when A does not lie so.
	GemmRowPack pre_a;
};

// Bytes of a kept row pack of a rows x cols matrix in math mode `mode` (GemmDesc::keep_a).
size_t gemm_row_pack_bytes(long long rows, long long cols, int mode);

// Validates and enqueues the product (pack kernels + one persistent tensor-core kernel).
nnb_status gemm_run(cudaStream_t s, const GemmDesc& d);

// Tile width gemm_run picks for d on a device with `sms` SMs (it never changes the result's bits).
int gemm_tile_width(const GemmDesc& d, int sms);

// Depth pieces gemm_run cuts d's k into (1: none); the cut depends on n, k and the epilogue only.
int gemm_depth_pieces(const GemmDesc& d);

// Packed form of d's B operand for tile width bn: its size in bytes, and the pack itself (panels,
// then one non-finite flag per padded row of op(B)^T, then the any-non-finite flag).
size_t gemm_packed_b_bytes(const GemmDesc& d, int bn);
nnb_status gemm_pack_b(cudaStream_t s, const GemmDesc& d, int bn, void* buf);

}  // namespace nnb
