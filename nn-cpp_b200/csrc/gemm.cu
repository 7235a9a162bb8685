// gemm.cu -- the fp32 GEMM of nn-cpp (nn::kernels::sgemm, include/nn/kernels/gemm.hpp:57-59)
// rebuilt for B200 (sm_100a): a pack kernel plus a persistent tcgen05 tensor-core kernel.
//
// Pack (the counterpart of pack_a / pack_b, src/kernels/gemm.cpp:79,126): op(A) and op(B)^T are
// rewritten, whatever their transpose flag and leading dimension, into K-major "panels",
// contiguous and zero-padded to whole panels: 128 rows x 32 floats for A (each stage loads the
// 16-float half that holds its k-block), 128 (or the tile width) rows x 16 floats for B. A pack of
// A can be kept in a caller's buffer and read again by a later product: K-major at a column offset
// (the depth pieces of a cut product), or MN-major, as the transposed operand of a weight gradient
// (32 consecutive packed depths of a row are one 128-byte row of a tcgen05 MN-major tile). In 3xTF32 mode each value
// x is stored twice, as hi = tf32(x) and lo = tf32(x - hi) (the split-precision method of
// Ootomo & Yokota, 2022), so C = Ahi*Bhi + Ahi*Blo + Alo*Bhi carries about 21 mantissa bits.
// Rows holding Inf or NaN are flagged; the epilogue recomputes the IEEE result of those
// elements (+-Inf or NaN) so non-finite inputs propagate exactly as the reference's fp32 loop.
//
// Main kernel, one CTA per SM, 6 warps:
//   warp 0     TMA producer: each stage = the A panels (hi[,lo]) of a 128-row tile and the B
//              panels of a BN-column tile (BN = 64, 128 or 256) for one 16-wide k-block,
//              64-byte swizzled;
//   warp 1     MMA issuer: tcgen05.mma.kind::tf32 128xBNx8 into a TMEM accumulator, two
//              accumulators so the epilogue of tile i overlaps tile i+1;
//   warps 2-5  epilogue: tcgen05.ld -> (+bias, ReLU/GELU) -> (C +) -> global, bounds-checked.
// There is no split-K and the k order is fixed, so every element of C is produced by the same
// sequence of operations whatever the grid size, the number of GPUs or the M-shard it sits in.
#include <algorithm>
#include <mutex>

#include "nnb_gemm.h"
#include "nnb_internal.h"
#include "nnb_math.cuh"
#include "nnb_ptx.cuh"
#include "nnb_trace.h"

namespace nnb {
namespace gemm {

constexpr int kBM = 128;                 // rows of C per tile (MMA M)
constexpr int kBK = 16;                  // floats of depth per pipeline stage (one 64 B row)
constexpr int kAPanelRows = 128;         // rows per packed panel of A
constexpr int kAPanelWidth = 32;         // floats per packed row of A (two 16-deep k-blocks; B rows hold one)
constexpr int kGroupM = 16;              // tiles of M walked together for L2 reuse of B
constexpr int kThreads = 192;            // TMA producer, MMA issuer, 4 epilogue warps
constexpr int kGatherThreads = 128;      // + 4 warps that gather B into the stages (implicit GEMM)
__host__ __device__ constexpr int threads_for(int gather) { return gather ? kThreads + kGatherThreads : kThreads; }
constexpr int kSmemBudget = 200 * 1024;  // dynamic shared memory for the stage ring

// Rows per packed B panel (one TMA box): 128 for the widths that are multiples of 128, else the width.
__host__ __device__ constexpr int b_panel_rows(int bn) { return bn % 128 == 0 ? 128 : bn; }
__host__ __device__ constexpr int tmem_cols_pow2(int cols) { return cols <= 32 ? 32 : 2 * tmem_cols_pow2((cols + 1) / 2); }

// 16-deep k-blocks per pipeline stage. A TF32-mode k-block carries two MMAs, against six in 3xTF32,
// so its stages take two k-blocks: each full / empty barrier round trip then covers four MMAs. (The
// gathered-operand path keeps one: its gather warps fill a stage per k-block.)
// A 256-row ("wide") tile, TF32 mode only, holds two 128-row A panels per k-block instead (below).
__host__ __device__ constexpr int kblocks_per_stage(int split, int gather, int wide = 0) {
	return (!split && !gather && !wide) ? 2 : 1;
}

template <int kSplit, int kBN, int kKPS = 1, int kAM = 1>
struct Cfg {
	static constexpr int S = kSplit ? 2 : 1;                 // hi[, lo]
	static constexpr int kABytes = kAM * S * kBM * kBK * 4;  // kAM 128-row A panels, each hi[, lo]
	static constexpr int kBPartBytes = kBN * kBK * 4;        // one part (hi or lo) of the B tile
	static constexpr int kBBytes = S * kBPartBytes;
	static constexpr int kKBlockBytes = kABytes + kBBytes;   // one k-block: A parts, then B parts
	static constexpr int kStageBytes = kKPS * kKBlockBytes;
	static constexpr int kStagesRaw = kSmemBudget / kStageBytes;
	static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
	static constexpr int kEpiBytes = 4 * 32 * 32 * 4;        // one 32 x 32 staging tile per epilogue warp
	static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 1024;
	static constexpr int kTmemCols = tmem_cols_pow2(2 * kBN); // two accumulators (allocations are powers of 2)
	static constexpr int kBPanelRows = b_panel_rows(kBN);
	static constexpr int kBPanels = kBN / kBPanelRows;
};

struct Params {
	int M, N, K, KB;
	int tiles_m, tiles_n;
	int batch, batch_inner;
	int a_batched, b_batched;        // 0: operand shared by every batch entry
	int Mp, Np;                      // padded row counts of the packed operands
	float* C;
	long long ldc, sc_outer, sc_inner;
	int accumulate;
	// epilogue
	const float* bias;
	long long s_bias_outer;          // bias offset per outer batch entry
	int bias_mode, act;
	unsigned char* mask;
	float* pre;
	long long ld_aux, s_aux_outer, s_aux_inner;
	// exact IEEE handling of non-finite inputs
	const int* any_nonfinite;
	const int* any_b;                // B's any-flag
	const int* flags_a;              // [a_batches][Mp]
	const int* flags_b;              // [b_batches][Np]
	const float* A;
	long long lda, sa_outer, sa_inner;
	const float* B;
	long long ldb, sb_outer, sb_inner;
	int ta, tb;
	int* err;
	// B gathered by the kernel (implicit GEMM); its non-finite flags are set by the gathering warps
	GemmGather g;
	int* gflags_b;                   // writable view of flags_b
	int* gany_b;                     // writable view of any_b
	// operands read MN-major from kept row packs (kernel variant kMn): batch entry bi's depth q is
	// row r0 + (bi / batch_inner) * r_outer + (bi % batch_inner) * r_inner + q of the packed matrix
	long long ra0, ra_outer, ra_inner, rb0, rb_outer, rb_inner;
	// A's packed columns: a_kw 32-wide columns per 128-row panel; batch entry bi's k-block kb is packed
	// k-block kb + a_kb0 + (bi / batch_inner) * a_kb_outer + (bi % batch_inner) * a_kb_inner (offsets
	// nonzero only for an A read from a kept row pack at a column offset, GemmDesc::pre_a)
	int a_kw, a_kb0, a_kb_outer, a_kb_inner;
};

// ---------------------------------------------------------------------------------------------
// Pack
// ---------------------------------------------------------------------------------------------

// Panel layout: panels of `panel_rows` rows x `pw` floats (pw = 16 for B, 32 for A), panel (rb, c)
// holding rows rb*panel_rows .. and depths c*pw .., stored as panel index (rb * KW + c) * S + part
// (part 0 = hi, 1 = lo); KW = panel columns over the padded depth (zero beyond K).
// One block: 32 rows x 64 depth of op(X) (X stored rows x K, or K x rows when trans), written
// as 4 k-blocks of the packed panel layout with `panel_rows`-row panels.
// grid = (Rp/32, ceil(KW*pw/64), batch entries); entry e reads X + (e / inner)*s_outer + (e % inner)*s_inner.
template <int kSplit>
__global__ void __launch_bounds__(256) pack_kernel(const float* __restrict__ X, long long ldx,
		long long s_outer, long long s_inner, int inner, int trans, int R, int K, int Rp, int KW, int pw,
		int panel_rows, float* __restrict__ out, int* __restrict__ flags, int* __restrict__ any_flag) {
	constexpr int S = kSplit ? 2 : 1;
	__shared__ float tile[32][65];
	const int t = threadIdx.x;
	const int r0 = blockIdx.x * 32, k0 = blockIdx.y * 64, e = blockIdx.z;
	const float* Xb = X + (long long)(e / inner) * s_outer + (long long)(e % inner) * s_inner;
	if (!trans) {
		const int kk = t & 63, rr = t >> 6;
#pragma unroll
		for (int i = 0; i < 8; ++i) {
			const int r = rr + 4 * i, gr = r0 + r, gk = k0 + kk;
			tile[r][kk] = (gr < R && gk < K) ? __ldg(Xb + (long long)gr * ldx + gk) : 0.0f;
		}
	} else {
		const int rr = t & 31, kk = t >> 5;
#pragma unroll
		for (int i = 0; i < 8; ++i) {
			const int k = kk + 8 * i, gr = r0 + rr, gk = k0 + k;
			tile[rr][k] = (gr < R && gk < K) ? __ldg(Xb + (long long)gk * ldx + gr) : 0.0f;
		}
	}
	__syncthreads();
	const int q = 2 * t;                 // element pair inside a 32 x 16 k-block slab
	const int rl = q >> 4, kl = q & 15;
	const long long batch_off = (long long)e * Rp * KW * pw * S;
	const int panel_floats = panel_rows * pw;
	const int kbs = KW * pw / 16;        // 16-deep blocks of the padded depth
	bool bad = false;
#pragma unroll
	for (int w = 0; w < 4; ++w) {
		const int kb = (k0 >> 4) + w;
		if (kb >= kbs) break;
		const float x0 = tile[rl][w * 16 + kl], x1 = tile[rl][w * 16 + kl + 1];
		const bool f0 = isfinite(x0), f1 = isfinite(x1);
		bad |= !(f0 && f1);
		float h0, l0, h1, l1;
		if (kSplit) {
			split_tf32(f0 ? x0 : 0.0f, h0, l0);
			split_tf32(f1 ? x1 : 0.0f, h1, l1);
		} else {
			h0 = to_tf32(f0 ? x0 : 0.0f);
			h1 = to_tf32(f1 ? x1 : 0.0f);
			l0 = l1 = 0.0f;
		}
		const int k = kb * 16 + kl;
		const long long panel = ((long long)(r0 / panel_rows) * KW + k / pw) * S;
		float* dst = out + batch_off + panel * panel_floats + (r0 % panel_rows + rl) * pw + (k % pw);
		*reinterpret_cast<float2*>(dst) = make_float2(h0, h1);
		if (kSplit) *reinterpret_cast<float2*>(dst + panel_floats) = make_float2(l0, l1);
	}
	if (bad) {
		atomicOr(flags + (long long)e * Rp + r0 + rl, 1);
		atomicOr(any_flag, 1);
	}
}

// Vectorised pack for X stored rows x K (K contiguous) with 16-byte aligned rows and K % 4 == 0:
// every thread moves float4 groups straight from X into the panels (4 consecutive k of one row are
// 16 contiguous bytes in both layouts). grid = (blocks, batch entries), grid-stride over Rp * KB * 4.
template <int kSplit>
__global__ void __launch_bounds__(256) pack_rows_vec_kernel(const float* __restrict__ X, long long ldx,
		long long s_outer, long long s_inner, int inner, int R, int K, int Rp, int KW, int pw, int panel_rows,
		float* __restrict__ out, int* __restrict__ flags, int* __restrict__ any_flag) {
	constexpr int S = kSplit ? 2 : 1;
	const int e = blockIdx.y;
	const float* Xb = X + (long long)(e / inner) * s_outer + (long long)(e % inner) * s_inner;
	// Rp * KW * pw / 4 < 2^31 (checked on the host), so the index arithmetic stays in 32 bits
	const unsigned K4 = (unsigned)(KW * pw / 4), total = (unsigned)Rp * K4;
	const long long batch_off = (long long)e * Rp * KW * pw * S;
	const int panel_floats = panel_rows * pw;
	for (unsigned idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
		const int r = (int)(idx / K4), q = (int)(idx - (unsigned)r * K4), k = q * 4;
		float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
		if (r < R && k < K) v = __ldg(reinterpret_cast<const float4*>(Xb + (long long)r * ldx + k));
		const bool ok = isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
		if (!ok) {
			atomicOr(flags + (long long)e * Rp + r, 1);
			atomicOr(any_flag, 1);
			v.x = isfinite(v.x) ? v.x : 0.0f;
			v.y = isfinite(v.y) ? v.y : 0.0f;
			v.z = isfinite(v.z) ? v.z : 0.0f;
			v.w = isfinite(v.w) ? v.w : 0.0f;
		}
		float4 h, l;
		if (kSplit) {
			split_tf32(v.x, h.x, l.x);
			split_tf32(v.y, h.y, l.y);
			split_tf32(v.z, h.z, l.z);
			split_tf32(v.w, h.w, l.w);
		} else {
			h = make_float4(to_tf32(v.x), to_tf32(v.y), to_tf32(v.z), to_tf32(v.w));
		}
		const long long panel = ((long long)(r / panel_rows) * KW + k / pw) * S;
		float* dst = out + batch_off + panel * panel_floats + (r % panel_rows) * pw + (k % pw);
		*reinterpret_cast<float4*>(dst) = h;
		if (kSplit) *reinterpret_cast<float4*>(dst + panel_floats) = l;
	}
}

// Vectorised pack for X stored K x rows (rows contiguous) with 16-byte aligned k-rows and R % 4 == 0:
// a 64-row x 32-depth tile is read with float4 loads along the rows, transposed in shared memory,
// and written as float4 groups of 4 consecutive k. grid = (ceil(Rp/64), ceil(Kp/32), batch entries).
template <int kSplit>
__global__ void __launch_bounds__(256) pack_cols_vec_kernel(const float* __restrict__ X, long long ldx,
		long long s_outer, long long s_inner, int inner, int R, int K, int Rp, int KW, int pw, int panel_rows,
		float* __restrict__ out, int* __restrict__ flags, int* __restrict__ any_flag) {
	constexpr int S = kSplit ? 2 : 1;
	__shared__ float tile[64][33];
	const int t = threadIdx.x;
	const int r0 = blockIdx.x * 64, k0 = blockIdx.y * 32, e = blockIdx.z;
	const float* Xb = X + (long long)(e / inner) * s_outer + (long long)(e % inner) * s_inner;
#pragma unroll
	for (int i = 0; i < 2; ++i) {
		const int f = t + 256 * i;                // float4 index in the 32 x 16 float4 tile
		const int kk = f >> 4, r4 = (f & 15) * 4;
		const int gk = k0 + kk, gr = r0 + r4;
		float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
		if (gk < K && gr < R) v = __ldg(reinterpret_cast<const float4*>(Xb + (long long)gk * ldx + gr));
		tile[r4][kk] = v.x;
		tile[r4 + 1][kk] = v.y;
		tile[r4 + 2][kk] = v.z;
		tile[r4 + 3][kk] = v.w;
	}
	__syncthreads();
	const long long batch_off = (long long)e * Rp * KW * pw * S;
	const int panel_floats = panel_rows * pw;
#pragma unroll
	for (int i = 0; i < 2; ++i) {
		const int f = t + 256 * i;                // (row, k-quad) pairs: 64 rows x 8 quads
		const int rl = f >> 3, q = f & 7;
		const int gr = r0 + rl, k = k0 + q * 4;
		if (k >= KW * pw || gr >= Rp) continue;
		float4 v = make_float4(tile[rl][q * 4], tile[rl][q * 4 + 1], tile[rl][q * 4 + 2], tile[rl][q * 4 + 3]);
		const bool ok = isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w);
		if (!ok) {
			atomicOr(flags + (long long)e * Rp + gr, 1);
			atomicOr(any_flag, 1);
			v.x = isfinite(v.x) ? v.x : 0.0f;
			v.y = isfinite(v.y) ? v.y : 0.0f;
			v.z = isfinite(v.z) ? v.z : 0.0f;
			v.w = isfinite(v.w) ? v.w : 0.0f;
		}
		float4 h, l;
		if (kSplit) {
			split_tf32(v.x, h.x, l.x);
			split_tf32(v.y, h.y, l.y);
			split_tf32(v.z, h.z, l.z);
			split_tf32(v.w, h.w, l.w);
		} else {
			h = make_float4(to_tf32(v.x), to_tf32(v.y), to_tf32(v.z), to_tf32(v.w));
		}
		const long long panel = ((long long)(gr / panel_rows) * KW + k / pw) * S;
		float* dst = out + batch_off + panel * panel_floats + (gr % panel_rows) * pw + (k % pw);
		*reinterpret_cast<float4*>(dst) = h;
		if (kSplit) *reinterpret_cast<float4*>(dst + panel_floats) = l;
	}
}

// ---------------------------------------------------------------------------------------------
// Main kernel
// ---------------------------------------------------------------------------------------------

// Work item t -> batch entry, row tile and column tile. A work item is kAM consecutive 128-row tiles
// (1, or 2 for the wide TF32 tile) of one column tile; mt is its first 128-row tile.
template <int kAM = 1>
__device__ __forceinline__ void tile_coords(int t, const Params& p, int& bi, int& mt, int& nt) {
	const int tiles_m = p.tiles_m / kAM;
	const int per_batch = tiles_m * p.tiles_n;
	bi = t / per_batch;
	const int r = t - bi * per_batch;
	const int group = r / (kGroupM * p.tiles_n);
	const int first_m = group * kGroupM;
	const int gsz = min(tiles_m - first_m, kGroupM);
	const int in = r - group * kGroupM * p.tiles_n;
	mt = (first_m + in % gsz) * kAM;
	nt = in / gsz;
}

__device__ __forceinline__ long long batch_offset(int bi, int inner, long long s_outer, long long s_inner) {
	return (long long)(bi / inner) * s_outer + (long long)(bi % inner) * s_inner;
}

// ---------------------------------------------------------------------------------------------
// Gathered B (implicit GEMM for the convolutions; the modes are described in nnb_gemm.h)
// ---------------------------------------------------------------------------------------------

// The gather geometry copied into registers once by each gather thread (the hot loops read no kernel
// parameter memory).
struct GatherRegs {
	const float* src;
	long long s_outer, s_inner;
	int mode, N, K, inner, H, W, ho, wo, kh, kw, stride, pad, dil, cout;
};

__device__ __forceinline__ GatherRegs gather_regs(const Params& p) {
	GatherRegs r;
	r.src = p.g.src; r.s_outer = p.g.s_outer; r.s_inner = p.g.s_inner;
	r.mode = p.g.mode; r.N = p.N; r.K = p.K; r.inner = p.batch_inner;
	r.H = p.g.H; r.W = p.g.W; r.ho = p.g.ho; r.wo = p.g.wo; r.kh = p.g.kh; r.kw = p.g.kw;
	r.stride = p.g.stride; r.pad = p.g.pad; r.dil = p.g.dil; r.cout = p.g.cout;
	return r;
}

__device__ __forceinline__ const float* gather_src(const Params& p, int bi) {
	return p.g.src + (long long)(bi / p.batch_inner) * p.g.s_outer + (long long)(bi % p.batch_inner) * p.g.s_inner;
}

// Element (j, k) of op(B)^T of batch entry bi, decoded from scratch (the non-finite fix-up path).
__device__ float gather_elem(const Params& p, int bi, int j, int k) {
	const GemmGather& g = p.g;
	const float* src = gather_src(p, bi);
	if (j >= p.N || k >= p.K) return 0.0f;
	const int khw = g.kh * g.kw;
	if (g.mode == kGatherTransposed) {
		const int ih = j / g.W, iw = j % g.W;
		const int t = k / g.cout, co = k % g.cout, ph = t / g.kw, pw = t % g.kw;
		const int th = ih + g.pad - ph * g.dil, tw = iw + g.pad - pw * g.dil;
		if (th < 0 || tw < 0 || th % g.stride || tw % g.stride) return 0.0f;
		const int oh = th / g.stride, ow = tw / g.stride;
		if (oh >= g.ho || ow >= g.wo) return 0.0f;
		return src[((long long)co * g.ho + oh) * g.wo + ow];
	}
	const int kk = g.mode == kGatherIm2col ? k : j, pos = g.mode == kGatherIm2col ? j : k;
	const int c = kk / khw, r = kk % khw, ph = r / g.kw, pw = r % g.kw;
	const int oh = pos / g.wo, ow = pos % g.wo;
	const int ih = oh * g.stride + ph * g.dil - g.pad, iw = ow * g.stride + pw * g.dil - g.pad;
	if (ih < 0 || ih >= g.H || iw < 0 || iw >= g.W) return 0.0f;
	return src[((long long)c * g.H + ih) * g.W + iw];
}

// Smem byte offset of element (row r, depth q) of a 16-deep K-major tile in the 64-byte swizzle the
// TMA loads would write: 16-byte unit u = q / 4 of row r sits at u ^ ((r >> 1) & 3).
__device__ __forceinline__ uint32_t sw64_offset(int r, int q) {
	return (uint32_t)(r * (kBK * 4) + ((((q >> 2) ^ (r >> 1)) & 3) << 4) + ((q & 3) << 2));
}

// Issues the 4-byte asynchronous copies of row j, depths k0 .. k0 + 15, of op(B)^T into the hi part of
// a stage (raw fp32, at the positions hi will occupy); positions outside the tensor are zero-filled.
// The index is decoded once, then stepped.
__device__ __forceinline__ void gather_issue_row(const GatherRegs& g, const float* __restrict__ src, int j, int k0,
		uint32_t row_base, int rr) {
	const bool row_ok = j < g.N;
	if (g.mode == kGatherIm2col) {
		const int oh = j / g.wo, ow = j - (j / g.wo) * g.wo;
		const int khw = g.kh * g.kw;
		int c = k0 / khw, r = k0 - c * khw, ph = r / g.kw, pw = r - (r / g.kw) * g.kw;
#pragma unroll
		for (int q = 0; q < 16; ++q) {
			const int ih = oh * g.stride + ph * g.dil - g.pad, iw = ow * g.stride + pw * g.dil - g.pad;
			const bool in = row_ok && k0 + q < g.K && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
			cp_async_4(row_base + sw64_offset(rr, q), in ? src + ((long long)c * g.H + ih) * g.W + iw : src, in ? 4u : 0u);
			if (++pw == g.kw) {
				pw = 0;
				if (++ph == g.kh) { ph = 0; ++c; }
			}
		}
	} else if (g.mode == kGatherTransposed && g.cout % 16 == 0) {
		// 16 consecutive output channels of one kernel tap: one window position for the whole stage
		const int ih = j / g.W, iw = j - (j / g.W) * g.W;
		const int t = k0 / g.cout, co0 = k0 - t * g.cout, ph = t / g.kw, pw = t - (t / g.kw) * g.kw;
		const int th = ih + g.pad - ph * g.dil, tw = iw + g.pad - pw * g.dil;
		const int oh = th / g.stride, ow = tw / g.stride;
		const bool in = k0 < g.K && th >= 0 && tw >= 0 && oh * g.stride == th && ow * g.stride == tw && oh < g.ho &&
			ow < g.wo;
		const long long plane = (long long)g.ho * g.wo;
		const float* base = in ? src + co0 * plane + (long long)oh * g.wo + ow : src;
#pragma unroll
		for (int q = 0; q < 16; ++q)
			cp_async_4(row_base + sw64_offset(rr, q), in ? base + q * plane : src, in ? 4u : 0u);
	} else if (g.mode == kGatherTransposed) {
		const int ih = j / g.W, iw = j - (j / g.W) * g.W;
		const int t = k0 / g.cout;
		int co = k0 - t * g.cout, ph = t / g.kw, pw = t - (t / g.kw) * g.kw;
#pragma unroll
		for (int q = 0; q < 16; ++q) {
			const int th = ih + g.pad - ph * g.dil, tw = iw + g.pad - pw * g.dil;
			const int oh = th / g.stride, ow = tw / g.stride;
			const bool in = row_ok && k0 + q < g.K && th >= 0 && tw >= 0 && oh * g.stride == th && ow * g.stride == tw &&
				oh < g.ho && ow < g.wo;
			cp_async_4(row_base + sw64_offset(rr, q), in ? src + ((long long)co * g.ho + oh) * g.wo + ow : src, in ? 4u : 0u);
			if (++co == g.cout) {
				co = 0;
				if (++pw == g.kw) { pw = 0; ++ph; }
			}
		}
	} else {                                   // kGatherIm2colRows
		const int khw = g.kh * g.kw;
		const int c = j / khw, r = j - c * khw, ph = r / g.kw, pw = r - (r / g.kw) * g.kw;
		int oh = k0 / g.wo, ow = k0 - (k0 / g.wo) * g.wo;
#pragma unroll
		for (int q = 0; q < 16; ++q) {
			const int ih = oh * g.stride + ph * g.dil - g.pad, iw = ow * g.stride + pw * g.dil - g.pad;
			const bool in = row_ok && k0 + q < g.K && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
			cp_async_4(row_base + sw64_offset(rr, q), in ? src + ((long long)c * g.H + ih) * g.W + iw : src, in ? 4u : 0u);
			if (++ow == g.wo) { ow = 0; ++oh; }
		}
	}
}

// Gathered B, step 1: the 128 gather threads (thread gt owns rows gt, gt + 128, ...) issue the copies
// of one stage's B tile (kBN rows x 16 depth) into its hi part, as one copy group.
template <int kBN>
__device__ __forceinline__ void gather_issue(const GatherRegs& g, int bi, int nt, int kb, int gt, uint32_t bpart) {
	const float* src = g.src + (long long)(bi / g.inner) * g.s_outer + (long long)(bi % g.inner) * g.s_inner;
#pragma unroll
	for (int i = 0; i < (kBN + kGatherThreads - 1) / kGatherThreads; ++i) {
		const int rr = gt + kGatherThreads * i;
		// columns of C past N are never stored, so their B rows are left as they are
		if (rr >= kBN || nt * kBN + rr >= g.N) break;
		gather_issue_row(g, src, nt * kBN + rr, kb * kBK, bpart, rr);
	}
	cp_async_commit();
}

// Gathered B, step 2 (once this thread's copies of the stage have landed): each row is read back,
// non-finite values are zeroed and flag their row (as the pack kernels do), and the values are split
// into hi (in place) and lo, in the layout the MMA reads.
template <int kSplit, int kBN>
__device__ __forceinline__ void gather_finish(int* __restrict__ flags_b, int* __restrict__ any_b, int rows_valid, int nt,
		int gt, uint8_t* bpart) {
#pragma unroll
	for (int i = 0; i < (kBN + kGatherThreads - 1) / kGatherThreads; ++i) {
		const int rr = gt + kGatherThreads * i;
		if (rr >= kBN || rr >= rows_valid) break;
		const int sw = (rr >> 1) & 3;
		float4* hrow = reinterpret_cast<float4*>(bpart + rr * (kBK * 4));
		float4* lrow = reinterpret_cast<float4*>(bpart + Cfg<kSplit, kBN>::kBPartBytes + rr * (kBK * 4));
		float4 x[4];
		bool bad = false;
#pragma unroll
		for (int u = 0; u < 4; ++u) {
			x[u] = hrow[u ^ sw];
			const bool f = isfinite(x[u].x) && isfinite(x[u].y) && isfinite(x[u].z) && isfinite(x[u].w);
			if (!f) {
				bad = true;
				x[u].x = isfinite(x[u].x) ? x[u].x : 0.0f;
				x[u].y = isfinite(x[u].y) ? x[u].y : 0.0f;
				x[u].z = isfinite(x[u].z) ? x[u].z : 0.0f;
				x[u].w = isfinite(x[u].w) ? x[u].w : 0.0f;
			}
		}
		if (bad) {
			atomicOr(flags_b + nt * kBN + rr, 1);
			atomicOr(any_b, 1);
			__threadfence();
		}
#pragma unroll
		for (int u = 0; u < 4; ++u) {
			float4 h, l;
			if (kSplit) {
				split_tf32(x[u].x, h.x, l.x);
				split_tf32(x[u].y, h.y, l.y);
				split_tf32(x[u].z, h.z, l.z);
				split_tf32(x[u].w, h.w, l.w);
				lrow[u ^ sw] = l;
			} else {
				h = make_float4(to_tf32(x[u].x), to_tf32(x[u].y), to_tf32(x[u].z), to_tf32(x[u].w));
			}
			hrow[u ^ sw] = h;
		}
	}
}

// IEEE value of sum_p op(A)(i,p)*op(B)(p,j) for an element whose row or column holds Inf/NaN:
// NaN if any product is NaN or both infinities occur, else the infinity that occurs.
__device__ __noinline__ float nonfinite_result(const Params& p, int bi, int i, int j, float v) {
	const float* A = p.A + batch_offset(bi, p.batch_inner, p.sa_outer, p.sa_inner);
	const float* B = p.B + batch_offset(bi, p.batch_inner, p.sb_outer, p.sb_inner);
	bool nan = false, pinf = false, ninf = false;
	for (int q = 0; q < p.K; ++q) {
		const float a = p.ta ? A[(long long)q * p.lda + i] : A[(long long)i * p.lda + q];
		const float b = p.g.mode != kGatherNone ? gather_elem(p, bi, j, q)
			: p.tb ? B[(long long)j * p.ldb + q] : B[(long long)q * p.ldb + j];
		const float pr = a * b;
		if (pr != pr) nan = true;
		else if (isinf(pr)) (pr > 0.0f ? pinf : ninf) = true;
	}
	if (nan || (pinf && ninf)) return __int_as_float(0x7fc00000);
	if (pinf) return __int_as_float(0x7f800000);
	if (ninf) return __int_as_float(0xff800000);
	return v;
}

// kWide (TF32 mode, no gather, BN = 256): each work item is a 256 x 256 tile, two 128-row halves that
// share every B stage, one half per TMEM accumulator. Per 16-deep k-block the CTA then loads 32 KB for
// four 128 x 256 x 8 MMAs instead of 24 KB for two: a third less operand traffic per MMA, and the
// 192 KB of stages hold 1.5x the tensor time. The cost: no accumulator double buffering (the next
// tile's MMAs wait for both halves' epilogues). Each element's arithmetic is the narrow kernel's.
// kMn (no gather, no wide tiles): bit 0 -- A is read MN-major from a kept row pack (its 128 rows are
// 4 chunks of 32 packed depths, each chunk 16 packed rows of 128 bytes, the 128-byte swizzle with
// 32-byte atoms that TMA writes with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B); bit 1 -- the same for B.
// Such an operand has no per-row flags: when its pack saw a non-finite value every element is
// recomputed by nonfinite_result.
template <int kSplit, int kBN, int kGather, int kWide = 0, int kMn = 0>
__global__ void __launch_bounds__(threads_for(kGather), 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a,
		const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ Params p) {
	static_assert(!kWide || (!kGather && kBN == 256), "wide tiles: no gather, 256 columns");
	static_assert(!kMn || (!kGather && !kWide), "MN-major operands: no gather, no wide tiles");
	constexpr int kAM = kWide ? 2 : 1;
	constexpr int kKPS = kblocks_per_stage(kSplit, kGather, kWide);
	using C = Cfg<kSplit, kBN, kKPS, kAM>;
	constexpr int S = C::S;
	constexpr int kStages = C::kStages;
	extern __shared__ uint8_t smem_raw[];
	uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
	__shared__ __align__(8) uint64_t full_bar[kStages], empty_bar[kStages], accf_bar[2], acce_bar[2];
	__shared__ uint32_t tmem_base_sh;
	__shared__ int abort_sh;

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	if (threadIdx.x == 0) {
		for (int s = 0; s < kStages; ++s) {
			// the TMA producer's arrival (+ one per gather warp when B is gathered)
			mbar_init(smem_u32(&full_bar[s]), kGather ? 1 + kGatherThreads / 32 : 1);
			mbar_init(smem_u32(&empty_bar[s]), 1);
		}
		for (int b = 0; b < 2; ++b) {
			mbar_init(smem_u32(&accf_bar[b]), 1);
			mbar_init(smem_u32(&acce_bar[b]), 4);
		}
		abort_sh = 0;
		fence_mbar_init();
		tma_prefetch_desc(&tm_a);
		if (!kGather) tma_prefetch_desc(&tm_b);
	}
	if (warp == 1) {
		tmem_alloc(smem_u32(&tmem_base_sh), C::kTmemCols);
		tmem_relinquish();
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem_base = tmem_base_sh;
	volatile int* abort_flag = &abort_sh;

	const int num_tiles = p.batch * (p.tiles_m / kAM) * p.tiles_n;      // work items
	const int a_panels = p.Mp / kAPanelRows, b_panels = p.Np / C::kBPanelRows;
	const int kwa = p.a_kw;                   // packed 32-wide columns of A

	if (warp == 0) {
		if (lane == 0) {
			// ------------------------------ TMA producer ------------------------------
			int stage = 0;
			uint32_t phase = 0;
			for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
				int bi, mt, nt;
				tile_coords<kAM>(t, p, bi, mt, nt);
				const int ab = p.a_batched ? bi : 0, bb = p.b_batched ? bi : 0;
				bool ok = true;
				for (int kb0 = 0; kb0 < p.KB; kb0 += kKPS) {
					if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1, p.err, kDevTimeoutEmpty, abort_flag)) {
						ok = false;
						break;
					}
					const int nkb = min(kKPS, p.KB - kb0);
					const uint32_t fb = smem_u32(&full_bar[stage]);
					mbar_arrive_expect_tx(fb, kGather ? C::kABytes : nkb * C::kKBlockBytes);
#pragma unroll
					for (int g = 0; g < kKPS; ++g) {
						if (g >= nkb) break;
						const int kb = kb0 + g;
						const uint32_t base = smem_u32(smem + stage * C::kStageBytes + g * C::kKBlockBytes);
						if (kMn & 1) {
							// 4 chunks of 32 depths of the kept pack = this tile's 128 rows, at 16 packed rows
							const long long r = p.ra0 + (long long)(bi / p.batch_inner) * p.ra_outer +
								(long long)(bi % p.batch_inner) * p.ra_inner + (long long)kb * kBK;
#pragma unroll
							for (int s = 0; s < S; ++s)
								tma_load_5d(base + s * (kAPanelRows * kBK * 4), &tm_a, fb, 0, (int)(r % kAPanelRows), s,
									mt * (kBM / 32), (int)(r / kAPanelRows));
						} else {
#pragma unroll
							for (int h = 0; h < kAM; ++h) {
								// 32-wide A rows: packed k-block akb is the (akb & 1) half of packed column akb / 2
								const int akb = kb + p.a_kb0 + (bi / p.batch_inner) * p.a_kb_outer +
									(bi % p.batch_inner) * p.a_kb_inner;
								const int ya = (int)((((long long)ab * a_panels + mt + h) * kwa + (akb >> 1)) * S * kAPanelRows);
#pragma unroll
								for (int s = 0; s < S; ++s)
									tma_load_2d(base + (h * S + s) * (kAPanelRows * kBK * 4), &tm_a, fb, (akb & 1) * kBK,
										ya + s * kAPanelRows);
							}
						}
						if (kMn & 2) {
							const long long r = p.rb0 + (long long)(bi / p.batch_inner) * p.rb_outer +
								(long long)(bi % p.batch_inner) * p.rb_inner + (long long)kb * kBK;
#pragma unroll
							for (int s = 0; s < S; ++s)
								tma_load_5d(base + C::kABytes + s * C::kBPartBytes, &tm_b, fb, 0, (int)(r % kAPanelRows), s,
									nt * (kBN / 32), (int)(r / kAPanelRows));
						}
#pragma unroll
						for (int q = 0; q < ((kGather || (kMn & 2)) ? 0 : C::kBPanels); ++q) {
							const long long panel = (long long)bb * b_panels + (long long)nt * C::kBPanels + q;
							const int yb = (int)((panel * p.KB + kb) * S * C::kBPanelRows);
#pragma unroll
							for (int s = 0; s < S; ++s)
								tma_load_2d(base + C::kABytes + s * C::kBPartBytes + q * (C::kBPanelRows * kBK * 4), &tm_b,
									fb, 0, yb + s * C::kBPanelRows);
						}
					}
					if (++stage == kStages) {
						stage = 0;
						phase ^= 1;
					}
				}
				if (!ok) break;
			}
		}
	} else if (warp == 1) {
		// --------------------- MMA issuer (the whole warp; one elected lane issues) ---------------------
		// accumulator v (the v-th 128-row tile this CTA hands to the epilogue) lives in buffer v & 1; a
		// wide work item fills two of them, one per 128-row half
		constexpr uint32_t idesc = idesc_tf32(kBM, kBN) | ((kMn & 1) ? kIdescAMajorMN : 0u) |
			((kMn & 2) ? kIdescBMajorMN : 0u);
		int stage = 0;
		uint32_t phase = 0;
		int it = 0;
		for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, it += kAM) {
			bool ok = true;
#pragma unroll
			for (int h = 0; h < kAM; ++h) {
				const int v = it + h;
				if (ok && !mbar_wait_warp(smem_u32(&acce_bar[v & 1]), ((v >> 1) & 1) ^ 1, p.err, kDevTimeoutAccumFree,
						abort_flag))
					ok = false;
			}
			if (!ok) break;
			tc_fence_after();
			for (int kb0 = 0; kb0 < p.KB; kb0 += kKPS) {
				if (!mbar_wait_warp(smem_u32(&full_bar[stage]), phase, p.err, kDevTimeoutFull, abort_flag)) {
					ok = false;
					break;
				}
				tc_fence_after();
#pragma unroll
				for (int g = 0; g < kKPS; ++g) {
					const int kb = kb0 + g;
					if (kb >= p.KB) break;
					const uint32_t base = smem_u32(smem + stage * C::kStageBytes + g * C::kKBlockBytes);
#pragma unroll
					for (int kk = 0; kk < kBK / 8; ++kk) {
						// K-major: 8 tf32 = 32 bytes along the swizzled row; MN-major: 8 rows of 128 bytes,
						// the next 32 rows (or columns) of C one 2 KB chunk further on
						const uint32_t off = kk * 32, off_mn = kk * 1024;
						const uint64_t b_hi = (kMn & 2) ? smem_desc_mn_sw128b32(base + C::kABytes + off_mn, 2048)
							: smem_desc_k_sw64(base + C::kABytes + off);
						const uint32_t first = (kb == 0 && kk == 0) ? 0u : 1u;
#pragma unroll
						for (int h = 0; h < kAM; ++h) {
							const uint32_t d_tmem = tmem_base + ((it + h) & 1) * kBN;
							const uint32_t abase = base + h * S * (kAPanelRows * kBK * 4);
							const uint64_t a_hi = (kMn & 1) ? smem_desc_mn_sw128b32(abase + off_mn, 2048)
								: smem_desc_k_sw64(abase + off);
							if (kSplit) {
								const uint64_t a_lo = (kMn & 1)
									? smem_desc_mn_sw128b32(abase + kAPanelRows * kBK * 4 + off_mn, 2048)
									: smem_desc_k_sw64(abase + kAPanelRows * kBK * 4 + off);
								const uint64_t b_lo = (kMn & 2)
									? smem_desc_mn_sw128b32(base + C::kABytes + C::kBPartBytes + off_mn, 2048)
									: smem_desc_k_sw64(base + C::kABytes + C::kBPartBytes + off);
								mma_tf32_elect(d_tmem, a_lo, b_hi, idesc, first);
								mma_tf32_elect(d_tmem, a_hi, b_lo, idesc, 1u);
								mma_tf32_elect(d_tmem, a_hi, b_hi, idesc, 1u);
							} else {
								mma_tf32_elect(d_tmem, a_hi, b_hi, idesc, first);
							}
						}
					}
				}
				mma_commit_elect(smem_u32(&empty_bar[stage]));
				if (++stage == kStages) {
					stage = 0;
					phase ^= 1;
				}
			}
			if (!ok) break;
#pragma unroll
			for (int h = 0; h < kAM; ++h) mma_commit_elect(smem_u32(&accf_bar[(it + h) & 1]));
		}
	} else if (kGather && warp >= kThreads / 32) {
		// ------------------------- B gatherers (implicit GEMM) -------------------------
		// Copies of up to kAhead stages are in flight per thread; a stage is split and handed to the MMA
		// issuer once its own copies have landed (cp.async.wait_group), so the gather's load latency
		// overlaps the stages before it. kAhead < kStages: a stage still being gathered is never needed
		// free before it is finished.
		constexpr int kAhead = kStages - 1;
		const int gt = threadIdx.x - kThreads;
		const GatherRegs gr = gather_regs(p);
		int* const gflags = p.gflags_b;
		int* const gany = p.gany_b;
		const long long flag_stride = p.b_batched ? p.Np : 0;
		int pend_stage[kAhead], pend_bi[kAhead], pend_nt[kAhead];
		int head = 0, count = 0;
		int stage = 0;
		uint32_t phase = 0;
		bool ok = true;
		for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
			int bi, mt, nt;
			tile_coords(t, p, bi, mt, nt);
			for (int kb = 0; kb < p.KB; ++kb) {
				const bool got = mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1, p.err, kDevTimeoutEmpty, abort_flag);
				if (!__all_sync(0xffffffffu, got)) {
					ok = false;
					break;
				}
				gather_issue<kBN>(gr, bi, nt, kb, gt, smem_u32(smem + stage * C::kStageBytes + C::kABytes));
				int slot = head + count;
				if (slot >= kAhead) slot -= kAhead;
				pend_stage[slot] = stage;
				pend_bi[slot] = bi;
				pend_nt[slot] = nt;
				if (++count == kAhead) {
					cp_async_wait<kAhead - 1>();
					gather_finish<kSplit, kBN>(gflags + pend_bi[head] * flag_stride, gany, gr.N - pend_nt[head] * kBN, pend_nt[head], gt,
						smem + pend_stage[head] * C::kStageBytes + C::kABytes);
					fence_proxy_async_smem();
					__syncwarp();
					if (lane == 0) mbar_arrive(smem_u32(&full_bar[pend_stage[head]]));
					head = head + 1 == kAhead ? 0 : head + 1;
					--count;
				}
				if (++stage == kStages) {
					stage = 0;
					phase ^= 1;
				}
			}
		}
		// the stages still pending: all copies landed, finished in order (also on the abort path, so no
		// copy is in flight when the CTA exits)
		cp_async_wait<0>();
		while (count > 0) {
			gather_finish<kSplit, kBN>(gflags + pend_bi[head] * flag_stride, gany, gr.N - pend_nt[head] * kBN, pend_nt[head], gt,
				smem + pend_stage[head] * C::kStageBytes + C::kABytes);
			fence_proxy_async_smem();
			__syncwarp();
			if (lane == 0) mbar_arrive(smem_u32(&full_bar[pend_stage[head]]));
			head = head + 1 == kAhead ? 0 : head + 1;
			--count;
		}
	} else {
		// ---------------------------------- epilogue ----------------------------------
		const int quad = warp & 3;                 // TMEM lanes this warp may access
		const int row = quad * 32 + lane;
		// the auxiliary output of a fused activation (ReLU's 1-byte mask, GELU's pre-activation) goes out
		// through the staging tile too when its rows are 4-element aligned
		const bool aux_ok = p.act == kActNone ||
			((p.ld_aux % 4 == 0) && (p.s_aux_outer % 4 == 0) && (p.s_aux_inner % 4 == 0) &&
			 (p.act == kActRelu ? (reinterpret_cast<uintptr_t>(p.mask) & 3) == 0
			                    : (reinterpret_cast<uintptr_t>(p.pre) & 15) == 0));
		const bool vec_ok = aux_ok && (p.ldc % 4 == 0) && (p.sc_outer % 4 == 0) &&
			(p.sc_inner % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
		// 32 x 32 staging tile of this warp: element (r, c) at float r*32 + 4*((c/4) ^ (r & 7)) + c%4, so that
		// both the row-per-lane writes and the 4-rows-per-instruction reads are free of bank conflicts
		float* stage = reinterpret_cast<float*>(smem + (size_t)kStages * C::kStageBytes) + quad * 1024;
		// the it-th 128-row tile of this CTA: half it % kAM of work item blockIdx.x + (it / kAM) * gridDim.x
		for (int it = 0;; ++it) {
			const int t = blockIdx.x + (it / kAM) * gridDim.x;
			if (t >= num_tiles) break;
			const int buf = it & 1;
			const uint32_t acc_phase = (it >> 1) & 1;
			if (!mbar_wait(smem_u32(&accf_bar[buf]), acc_phase, p.err, kDevTimeoutAccum, abort_flag)) break;
			tc_fence_after();
			int bi, mt, nt;
			tile_coords<kAM>(t, p, bi, mt, nt);
			mt += it % kAM;
			const int gm = mt * kBM + row;
			const bool row_ok = gm < p.M;
			float* cbase = p.C + batch_offset(bi, p.batch_inner, p.sc_outer, p.sc_inner);
			float* crow = cbase + (long long)gm * p.ldc;
			const long long aux_base = batch_offset(bi, p.batch_inner, p.s_aux_outer, p.s_aux_inner);
			const long long aux_row = aux_base + (long long)gm * p.ld_aux;
			float4* st4 = reinterpret_cast<float4*>(stage);
			// the warp's 32 x 32 values v (row per lane) to rows of dst (row stride ld) at column gn0, as
			// 128-byte row segments: lane (row) writes into the staging tile, then 8 lanes per row read
			// 16-byte pieces back and store them (rows past M are skipped)
			auto stage_rows = [&](float* dst, long long ld, int gn0, const float (&v)[32], bool acc) {
#pragma unroll
				for (int g = 0; g < 8; ++g)
					st4[lane * 8 + (g ^ (lane & 7))] = make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
				__syncwarp();
				const int g = lane & 7;
#pragma unroll
				for (int k = 0; k < 8; ++k) {
					const int rr = 4 * k + (lane >> 3);
					const int grow = mt * kBM + quad * 32 + rr;
					float4 o = st4[rr * 8 + (g ^ (rr & 7))];
					if (grow < p.M) {
						float4* d4 = reinterpret_cast<float4*>(dst + (long long)grow * ld + gn0) + g;
						if (acc) {
							const float4 c = *d4;
							o.x = c.x + o.x; o.y = c.y + o.y; o.z = c.z + o.z; o.w = c.w + o.w;
						}
						*d4 = o;
					}
				}
				__syncwarp();                       // the tile is read before it is written again
			};
			// a gathered B's flags are set during this kernel (by atomics, at L2): read them past L1
			const bool fix = (*p.any_nonfinite | (kGather ? __ldcg(p.any_b) : *p.any_b)) != 0;
			const bool row_bad = fix && row_ok && ((kMn & 1) || p.flags_a[(long long)(p.a_batched ? bi : 0) * p.Mp + gm] != 0);
			const int* fcol = p.flags_b + (long long)(p.b_batched ? bi : 0) * p.Np;
			const float* bias_e = p.bias + (long long)(bi / p.batch_inner) * p.s_bias_outer;
			const float row_bias = (p.bias_mode == kBiasRow && row_ok) ? bias_e[gm] : 0.0f;
#pragma unroll 1
			for (int ch = 0; ch < kBN / 32; ++ch) {
				const int gn0 = nt * kBN + ch * 32;
				if (gn0 >= p.N) break;                 // warp-uniform
				uint32_t r[32];
				tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + buf * kBN + ch * 32, r);
				tmem_wait_ld();
				// whole 32-column chunks of a vector-friendly C go out through the staging tile as
				// 128-byte row segments (coalesced: one line per 8 lanes, also over NVLink when C is a
				// peer's memory); every lane takes part, rows past M only skip the global stores
				const bool staged = vec_ok && gn0 + 32 <= p.N;       // warp-uniform
				if (!row_ok && !staged) continue;
				float v[32];
#pragma unroll
				for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
				if (fix && row_ok) {
#pragma unroll
					for (int j = 0; j < 32; ++j) {
						const int gn = gn0 + j;
						if (gn < p.N && (row_bad || (kMn & 2) || (kGather ? __ldcg(fcol + gn) : fcol[gn]) != 0))
							v[j] = nonfinite_result(p, bi, gm, gn, v[j]);
					}
				}
#pragma unroll
				for (int j = 0; j < 32; ++j) v[j] = v[j] + 0.0f;
				if (p.bias_mode == kBiasRow) {
#pragma unroll
					for (int j = 0; j < 32; ++j) v[j] = v[j] + row_bias;
				} else if (p.bias_mode == kBiasCol) {
#pragma unroll
					for (int j = 0; j < 32; ++j) {
						const int gn = gn0 + j;
						v[j] = v[j] + (gn < p.N ? __ldg(bias_e + gn) : 0.0f);
					}
				}
				uint32_t alive_bits = 0;
				if (p.act == kActRelu) {
#pragma unroll
					for (int j = 0; j < 32; ++j) {
						const bool alive = v[j] > 0.0f;
						v[j] = alive ? v[j] : 0.0f;
						alive_bits |= (alive ? 1u : 0u) << j;
					}
					if (!staged) {
#pragma unroll
						for (int j = 0; j < 32; ++j)
							if (gn0 + j < p.N) p.mask[aux_row + gn0 + j] = (alive_bits >> j) & 1u;
					}
				} else if (p.act == kActGelu) {
					if (staged) {
						stage_rows(p.pre + aux_base, p.ld_aux, gn0, v, false);
					} else {
#pragma unroll
						for (int j = 0; j < 32; ++j)
							if (gn0 + j < p.N) p.pre[aux_row + gn0 + j] = v[j];
					}
#pragma unroll
					for (int j = 0; j < 32; ++j) v[j] = gelu_fwd(v[j], tanh_one(gelu_tanh_arg(v[j])));
				}
				if (staged) {
					stage_rows(cbase, p.ldc, gn0, v, p.accumulate != 0);
					if (p.act == kActRelu) {
						// the 32 x 32 alive bytes: row per lane into the tile (8 words of 4 bytes, the
						// same XOR placement), then 4 rows of 32 bytes per store instruction
						uint32_t* st = reinterpret_cast<uint32_t*>(stage);
#pragma unroll
						for (int w = 0; w < 8; ++w) {
							const uint32_t b = alive_bits >> (4 * w);
							st[lane * 8 + (w ^ (lane & 7))] = (b & 1u) | ((b >> 1) & 1u) << 8 | ((b >> 2) & 1u) << 16 |
								((b >> 3) & 1u) << 24;
						}
						__syncwarp();
						const int w = lane & 7;
#pragma unroll
						for (int k = 0; k < 4; ++k) {
							const int rr = 8 * k + (lane >> 3) * 2;
#pragma unroll
							for (int h2 = 0; h2 < 2; ++h2) {
								const int r2 = rr + h2;
								const int grow = mt * kBM + quad * 32 + r2;
								if (grow < p.M)
									*reinterpret_cast<uint32_t*>(p.mask + aux_base + (long long)grow * p.ld_aux + gn0 + 4 * w) =
										st[r2 * 8 + (w ^ (r2 & 7))];
							}
						}
						__syncwarp();
					}
				} else {
#pragma unroll
					for (int j = 0; j < 32; ++j) {
						const int gn = gn0 + j;
						if (gn < p.N) crow[gn] = p.accumulate ? crow[gn] + v[j] : v[j];
					}
				}
			}
			tc_fence_before();
			__syncwarp();
			if (lane == 0) mbar_arrive(smem_u32(&acce_bar[buf]));
		}
	}

	tc_fence_before();
	__syncthreads();
	if (warp == 1) {
		__syncwarp();
		tc_fence_after();
		tmem_dealloc(tmem_base, C::kTmemCols);
	}
}

// Zero fill of an m x n region per batch entry: the k == 0 product (gemm.cpp:346-348).
__global__ void zero_fill_kernel(float* c, long long ldc, long long s_outer, long long s_inner, int inner,
		int m, int n) {
	float* cb = c + (long long)(blockIdx.z / inner) * s_outer + (long long)(blockIdx.z % inner) * s_inner;
	for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < (long long)m * n;
			idx += (long long)gridDim.x * blockDim.x) {
		const long long i = idx / n, j = idx - i * n;
		cb[i * ldc + j] = 0.0f;
	}
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------

inline long long round_up(long long x, long long a) { return (x + a - 1) / a * a; }

// Tile width. A tile's time is its MMA instruction count (the same for every width) times the cost of
// one tf32 instruction, measured at about 44 + 0.38 N cycles, and the persistent grid works through
// the tiles in waves of one per SM: the width with the fewest waves x instruction cost wins, a
// narrower one only when clearly better. Big products keep 256; a product whose 256-wide tiles leave
// its last wave part-empty may take 224 (a 1024 x 8192 row band: 296 tiles, two full waves on 148 SMs,
// against 256 tiles in two waves at 256); products with few tiles (a rank's share of a data-parallel
// batch) get narrower tiles that fill the SMs. The width does not change any
// element's arithmetic (each is one k-ordered chain in the accumulator), so results stay bitwise
// independent of it, of the batch size and of the GPU count.
static int choose_bn(long long m, long long n, long long entries, int sms) {
	const long long mt = entries * (round_up(m, kBM) / kBM);
	int best = 256;
	double best_cost = 0.0;
	for (int bn : {256, 224, 128, 64}) {
		const long long tiles = mt * (round_up(n, bn) / bn);
		const long long waves = (tiles + sms - 1) / sms;
		const double cost = (double)waves * (44.0 + 0.38 * bn);
		if (bn == 256 || cost < best_cost * 0.97) {
			best = bn;
			best_cost = cost;
		}
	}
	return best;
}

static bool g_attr_set[64][2][4][2][2][4];
static std::mutex g_attr_mutex;

template <int kSplit, int kBN, int kGather, int kWide>
using KernelCfg = Cfg<kSplit, kBN, kblocks_per_stage(kSplit, kGather, kWide), kWide ? 2 : 1>;

template <int kSplit, int kBN, int kGather = 0, int kWide = 0, int kMn = 0>
static nnb_status set_smem_attr(int dev) {
	const int bi = kBN == 64 ? 0 : kBN == 128 ? 1 : kBN == 224 ? 3 : 2;
	std::lock_guard<std::mutex> lock(g_attr_mutex);
	if (g_attr_set[dev & 63][kSplit][bi][kGather][kWide][kMn]) return NNB_OK;
	NNB_CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel<kSplit, kBN, kGather, kWide, kMn>,
		cudaFuncAttributeMaxDynamicSharedMemorySize, KernelCfg<kSplit, kBN, kGather, kWide>::kSmemBytes));
	g_attr_set[dev & 63][kSplit][bi][kGather][kWide][kMn] = true;
	return NNB_OK;
}

// Scratch layout of one product: packed A, packed B, then the non-finite flags (A's, B's, then the
// two any-flags) -- each part only when it lives in the scratch (not in a kept, pre-packed or
// MN-major-read pack).
struct Plan {
	int S, bn, b_panel_rows;
	int wide;                                 // 256 x 256 TF32 tiles (rows padded to 256)
	int mn;                                   // bit 0: A, bit 1: B read MN-major from kept row packs
	int pre_a;                                // A read K-major from a kept row pack (GemmDesc::pre_a)
	long long a_kb0, a_kb_outer, a_kb_inner;  // its packed k-block offsets (Params::a_kb0 ...)
	long long Mp, Np, Kp, KB, KWA, entries, a_entries, b_entries;
	long long rows_a, rows_b;                 // packed rows of each operand (A: 32 floats, B: 16 floats)
	long long ra0, ra_outer, ra_inner, rb0, rb_outer, rb_inner;
	size_t off_b, off_f, flag_ints, total;
};

// Kept row pack of a rows x cols matrix: panel bytes, then round_up(rows, 256) flags and the any-flag.
static long long row_pack_rows(long long rows) { return round_up(rows, 2 * kBM); }
static size_t row_pack_panel_bytes(long long rows, long long cols, int S) {
	return (size_t)round_up(row_pack_rows(rows) * round_up(cols, kAPanelWidth) * S * 4, 1024);
}
static int* row_pack_flags(const void* buf, long long rows, long long cols, int S) {
	return reinterpret_cast<int*>(static_cast<unsigned char*>(const_cast<void*>(buf)) + row_pack_panel_bytes(rows, cols, S));
}

// Whether operand X (A through mn_a, stored K x m with ta = 1; B through mn_b, stored K x n with
// tb = 0) can be read from the kept row pack r: every batch entry X_e = x + o*s_outer + i*s_inner
// must start in column 0 of the packed matrix on a 16-row boundary, the depth must be whole
// 16-row blocks (so no k-block reaches past its entry), and the rows and `width` columns it covers
// must lie inside the pack. Gives the entries' first rows.
static bool mn_usable(const GemmDesc& d, const GemmRowPack& r, const float* x, long long ld, long long s_outer,
		long long s_inner, long long width, long long& r0, long long& r_outer, long long& r_inner) {
	if (!r.buf || !r.base || !x || r.mode != d.mode || ld != r.ld || x < r.base || d.k % kBK != 0) return false;
	const long long off = x - r.base;
	if (off % ld != 0 || s_outer % ld != 0 || s_inner % ld != 0 || s_outer < 0 || s_inner < 0) return false;
	r0 = off / ld;
	r_outer = s_outer / ld;
	r_inner = s_inner / ld;
	if (r0 % kBK != 0 || r_outer % kBK != 0 || r_inner % kBK != 0 || width > r.cols) return false;
	const long long last = r0 + (d.batch_outer - 1) * r_outer + (d.batch_inner - 1) * r_inner + d.k;
	return last <= r.rows && r.rows <= INT32_MAX;
}

// Whether A (ta = 0) can be read K-major from the kept row pack r of the matrix it lies in: every
// batch entry A_e = a + o*sa_outer + i*sa_inner starts in row 0 of the packed matrix at a column
// offset that is whole 16-column blocks, and its k columns lie inside (k whole 16-column blocks, or a
// single entry ending at the last column, where the pack's zero padding completes the block).
static bool pre_a_usable(const GemmDesc& d, const GemmRowPack& r, long long& kb0, long long& kb_outer,
		long long& kb_inner) {
	if (!r.buf || !r.base || !d.a || d.ta || r.mode != d.mode || d.lda != r.ld || d.a < r.base) return false;
	const long long c0 = d.a - r.base;
	if (c0 >= r.ld || c0 % kBK != 0 || d.sa_outer % kBK != 0 || d.sa_inner % kBK != 0 || d.sa_outer < 0 ||
			d.sa_inner < 0 || d.m > r.rows ||
			row_pack_rows(r.rows) * (round_up(r.cols, kAPanelWidth) / kAPanelWidth) * (r.mode == NNB_MATH_FP32X3 ? 2 : 1) >
				INT32_MAX)
		return false;
	const long long end = c0 + (d.batch_outer - 1) * d.sa_outer + (d.batch_inner - 1) * d.sa_inner + d.k;
	const bool single = d.batch_outer * d.batch_inner == 1;
	if (end > r.cols || (d.k % kBK != 0 && !(single && end == r.cols))) return false;
	kb0 = c0 / kBK;
	kb_outer = d.sa_outer / kBK;
	kb_inner = d.sa_inner / kBK;
	return true;
}

static nnb_status make_plan(const GemmDesc& d, Plan& pl, int force_bn = 0, int sms = 148) {
	pl.S = d.mode == NNB_MATH_FP32X3 ? 2 : 1;
	pl.bn = force_bn ? force_bn : choose_bn(d.m, d.n, d.batch_outer * d.batch_inner, sms > 0 ? sms : 148);
	if (d.gather.mode != kGatherNone && pl.bn == 224) pl.bn = 256;
	pl.b_panel_rows = b_panel_rows(pl.bn);
	pl.entries = d.batch_outer * d.batch_inner;
	pl.KB = round_up(d.k, kBK) / kBK;
	// Wide tiles in TF32 mode when the width was left to the plan, the 256-wide tiles are chosen, the
	// 256 x 256 work items still fill the SMs and the depth amortises the unoverlapped epilogue
	pl.mn = 0;
	pl.ra0 = pl.ra_outer = pl.ra_inner = pl.rb0 = pl.rb_outer = pl.rb_inner = 0;
	pl.a_kb0 = pl.a_kb_outer = pl.a_kb_inner = 0;
	pl.pre_a = !d.keep_a && pre_a_usable(d, d.pre_a, pl.a_kb0, pl.a_kb_outer, pl.a_kb_inner) ? 1 : 0;
	if (d.gather.mode == kGatherNone && !d.packed_b && !d.keep_a) {
		if (!pl.pre_a && d.ta && mn_usable(d, d.mn_a, d.a, d.lda, d.sa_outer, d.sa_inner, d.m, pl.ra0, pl.ra_outer, pl.ra_inner))
			pl.mn |= 1;
		if (!d.tb && mn_usable(d, d.mn_b, d.b, d.ldb, d.sb_outer, d.sb_inner, d.n, pl.rb0, pl.rb_outer, pl.rb_inner))
			pl.mn |= 2;
	}
	pl.wide = (force_bn == 0 && pl.mn == 0 && d.gather.mode == kGatherNone && pl.bn == 256 &&
		pl.KB >= 64 && pl.entries * (round_up(d.m, 2 * kBM) / (2 * kBM)) * (round_up(d.n, 256) / 256) >= (sms > 0 ? sms : 148))
		? 1 : 0;
	pl.Mp = round_up(d.m, pl.wide ? 2 * kBM : kBM);
	pl.Np = round_up(d.n, pl.bn);
	pl.Kp = round_up(d.k, kBK);
	pl.KB = pl.Kp / kBK;
	pl.entries = d.batch_outer * d.batch_inner;
	pl.a_entries = (!pl.pre_a && (d.sa_outer || d.sa_inner)) ? pl.entries : 1;
	const bool gathered = d.gather.mode != kGatherNone;
	pl.b_entries = (gathered ? (d.gather.s_outer || d.gather.s_inner) : (d.sb_outer || d.sb_inner)) ? pl.entries : 1;
	pl.KWA = (pl.KB + 1) / 2;
	pl.rows_a = pl.a_entries * pl.Mp * pl.KWA * pl.S;
	pl.rows_b = pl.b_entries * pl.Np * pl.KB * pl.S;
	if (pl.rows_a > INT32_MAX || pl.rows_b > INT32_MAX)
		return fail(NNB_ERR_UNSUPPORTED, "gemm: operands too large for one launch (packed rows %lld, %lld)",
			pl.rows_a, pl.rows_b);
	if (pl.entries > 65535) return fail(NNB_ERR_UNSUPPORTED, "gemm: more than 65535 batch entries");
	if (pl.entries * (pl.Mp / kBM) * (pl.Np / pl.bn) > INT32_MAX) return fail(NNB_ERR_UNSUPPORTED, "gemm: too many tiles");
	// a B that arrives packed (GemmDesc::packed_b) has its panels and flags outside the workspace; a
	// gathered B has no panels at all, only its flags
	const bool pre_b = d.packed_b != nullptr;
	const bool a_ws = !(pl.mn & 1) && !d.keep_a && !pl.pre_a;   // A's panels and flags in the scratch
	const bool b_flags_ws = !(pl.mn & 2) && !pre_b;        // B's flags (a gathered B has flags, no panels)
	const size_t bytes_a = a_ws ? (size_t)pl.rows_a * kAPanelWidth * 4 : 0,
		bytes_b = (pre_b || gathered || (pl.mn & 2)) ? 0 : (size_t)pl.rows_b * kBK * 4;
	pl.flag_ints = (size_t)((a_ws ? pl.a_entries * pl.Mp : 0) + (b_flags_ws ? pl.b_entries * pl.Np : 0) + 2);
	pl.off_b = round_up(bytes_a, 1024);
	pl.off_f = pl.off_b + round_up(bytes_b, 1024);
	pl.total = pl.off_f + pl.flag_ints * sizeof(int);
	return NNB_OK;
}

// Packs one operand with the fastest kernel its layout allows (16-byte aligned rows and a multiple of
// 4 along the contiguous axis: float4 paths; anything else: the scalar tile kernel).
// Panels are `pw` floats wide (16: B operands; 32: A operands, see kAPanelWidth) and KW = padded depth / pw.
template <int kSplit>
static void launch_pack(cudaStream_t s, const float* X, long long ldx, long long s_outer, long long s_inner, int inner,
		int trans, long long R, long long K, long long Rp, long long KW, int pw, int panel_rows, long long entries,
		float* out, int* flags, int* any) {
	const bool base16 = (reinterpret_cast<uintptr_t>(X) & 15) == 0;
	const bool strides4 = ldx % 4 == 0 && s_outer % 4 == 0 && s_inner % 4 == 0;
	const long long width = KW * pw;
	if (!trans && base16 && strides4 && K % 4 == 0 && Rp * width / 4 < (1LL << 31)) {
		const long long work = Rp * width / 4;
		const unsigned blocks = (unsigned)std::max<long long>(1, std::min<long long>((work + 255) / 256, 148 * 16));
		pack_rows_vec_kernel<kSplit><<<dim3(blocks, (unsigned)entries), 256, 0, s>>>(X, ldx, s_outer, s_inner, inner,
			(int)R, (int)K, (int)Rp, (int)KW, pw, panel_rows, out, flags, any);
	} else if (trans && base16 && strides4 && R % 4 == 0) {
		dim3 g((unsigned)((Rp + 63) / 64), (unsigned)((width + 31) / 32), (unsigned)entries);
		pack_cols_vec_kernel<kSplit><<<g, 256, 0, s>>>(X, ldx, s_outer, s_inner, inner, (int)R, (int)K, (int)Rp, (int)KW,
			pw, panel_rows, out, flags, any);
	} else {
		dim3 g((unsigned)(Rp / 32), (unsigned)((width + 63) / 64), (unsigned)entries);
		pack_kernel<kSplit><<<g, 256, 0, s>>>(X, ldx, s_outer, s_inner, inner, trans, (int)R, (int)K, (int)Rp, (int)KW,
			pw, panel_rows, out, flags, any);
	}
}

// Tensor map of a kept row pack read MN-major: (32 depths, 128 panel rows, part, panel column,
// 128-row block), boxes of 16 rows x `chunks` panel columns (32 rows or columns of C each).
static nnb_status encode_row_pack_mn(CUtensorMap* map, const GemmRowPack& r, int chunks) {
	const int S = r.mode == NNB_MATH_FP32X3 ? 2 : 1;
	const uint64_t kw = (uint64_t)(round_up(r.cols, kAPanelWidth) / kAPanelWidth);
	const uint64_t panel = (uint64_t)kAPanelRows * kAPanelWidth * 4;
	const uint64_t dims[5] = {(uint64_t)kAPanelWidth, (uint64_t)kAPanelRows, (uint64_t)S, kw,
		(uint64_t)(row_pack_rows(r.rows) / kAPanelRows)};
	const uint64_t strides[4] = {(uint64_t)kAPanelWidth * 4, panel, S * panel, kw * S * panel};
	const uint32_t box[5] = {(uint32_t)kAPanelWidth, (uint32_t)kBK, 1, (uint32_t)chunks, 1};
	return encode_tiled_nd(map, r.buf, 5, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}

template <int kSplit, int kBN, int kGather = 0, int kWide = 0, int kMn = 0>
static nnb_status launch_main(cudaStream_t s, int dev, int sm_count, int* err, const GemmDesc& d, const Plan& pl,
		unsigned char* ws, bool traced) {
	using Cf = KernelCfg<kSplit, kBN, kGather, kWide>;   // the kernel's own stage layout
	const bool pre_b = d.packed_b != nullptr;
	// the scratch's flags: A's (when packed into the scratch), B's (when not pre-packed or MN-major),
	// then A's and B's any-flags
	int* wsf = reinterpret_cast<int*>(ws + pl.off_f);
	long long nf = 0;
	float* pa = nullptr;
	float* pb = reinterpret_cast<float*>(ws + pl.off_b);
	int *flags_a = nullptr, *flags_b = nullptr;
	const int *any_a = nullptr, *any_b = nullptr;
	int *any_a_w = nullptr, *any_b_w = nullptr;          // the words the pack kernels set
	int* kept_flags = nullptr;
	const int* pre_flags = nullptr;
	if (kMn & 1) {
		any_a = row_pack_flags(d.mn_a.buf, d.mn_a.rows, d.mn_a.cols, pl.S) + row_pack_rows(d.mn_a.rows);
	} else if (pl.pre_a) {                                 // panels, flags and any-flag of the kept pack
		pa = static_cast<float*>(const_cast<void*>(d.pre_a.buf));
		pre_flags = row_pack_flags(d.pre_a.buf, d.pre_a.rows, d.pre_a.cols, pl.S);
		flags_a = const_cast<int*>(pre_flags);
		any_a = pre_flags + row_pack_rows(d.pre_a.rows);
	} else if (d.keep_a) {                                 // panels, flags and any-flag in the caller's buffer
		pa = static_cast<float*>(d.keep_a);
		kept_flags = flags_a = row_pack_flags(d.keep_a, d.m, d.k, pl.S);
	} else {
		pa = reinterpret_cast<float*>(ws);
		flags_a = wsf;
		nf += pl.a_entries * pl.Mp;
	}
	if (kMn & 2) {
		any_b = row_pack_flags(d.mn_b.buf, d.mn_b.rows, d.mn_b.cols, pl.S) + row_pack_rows(d.mn_b.rows);
	} else if (pre_b) {                                    // panels, then Np flags, then B's any-flag
		unsigned char* buf = static_cast<unsigned char*>(const_cast<void*>(d.packed_b));
		pb = reinterpret_cast<float*>(buf);
		flags_b = reinterpret_cast<int*>(buf + round_up((long long)pl.rows_b * kBK * 4, 1024));
		any_b = flags_b + pl.Np;
	} else {
		flags_b = wsf + nf;
		nf += pl.b_entries * pl.Np;
	}
	if (!(kMn & 1) && !pl.pre_a) any_a = any_a_w = kept_flags ? kept_flags + row_pack_rows(d.m) : wsf + nf;
	if (!(kMn & 2) && !pre_b) any_b = any_b_w = wsf + nf + 1;
	const int inner = (int)d.batch_inner;

	NNB_CUDA_TRY(cudaMemsetAsync(wsf, 0, pl.flag_ints * sizeof(int), s));
	if (kept_flags) NNB_CUDA_TRY(cudaMemsetAsync(kept_flags, 0, (row_pack_rows(d.m) + 1) * sizeof(int), s));
	if (!(kMn & 1) && !pl.pre_a) {
		TraceScope ts(s, kTracePack, traced);
		launch_pack<kSplit>(s, d.a, d.lda, d.sa_outer, d.sa_inner, inner, d.ta, d.m, d.k, pl.Mp, pl.KWA, kAPanelWidth,
			kAPanelRows, pl.a_entries, pa, flags_a, any_a_w);
	}
	if (!pre_b && !kGather && !(kMn & 2)) {
		TraceScope ts(s, kTracePack, traced);
		launch_pack<kSplit>(s, d.b, d.ldb, d.sb_outer, d.sb_inner, inner, !d.tb, d.n, d.k, pl.Np, pl.KB, kBK,
			Cf::kBPanelRows, pl.b_entries, pb, flags_b, any_b_w);
	}
	NNB_CUDA_TRY(cudaGetLastError());

	CUtensorMap tma, tmb;
	if (kMn & 1)
		NNB_TRY(encode_row_pack_mn(&tma, d.mn_a, kBM / 32));
	else if (pl.pre_a)
		NNB_TRY(encode_tiled_2d(&tma, pa, kAPanelWidth,
			(uint64_t)(row_pack_rows(d.pre_a.rows) * (round_up(d.pre_a.cols, kAPanelWidth) / kAPanelWidth) * pl.S),
			kAPanelWidth * 4, kBK, kAPanelRows, CU_TENSOR_MAP_SWIZZLE_64B));
	else      // 16-deep halves of the 32-wide rows, written to shared memory as today's 64-byte rows
		NNB_TRY(encode_tiled_2d(&tma, pa, kAPanelWidth, (uint64_t)pl.rows_a, kAPanelWidth * 4, kBK, kAPanelRows,
			CU_TENSOR_MAP_SWIZZLE_64B));
	if (kGather)
		tmb = tma;                               // not read: B is gathered by the kernel
	else if (kMn & 2)
		NNB_TRY(encode_row_pack_mn(&tmb, d.mn_b, kBN / 32));
	else
		NNB_TRY(encode_tiled_2d(&tmb, pb, kBK, (uint64_t)pl.rows_b, kBK * 4, kBK, Cf::kBPanelRows,
			CU_TENSOR_MAP_SWIZZLE_64B));

	Params p;
	p.M = (int)d.m; p.N = (int)d.n; p.K = (int)d.k; p.KB = (int)pl.KB;
	p.tiles_m = (int)(pl.Mp / kBM); p.tiles_n = (int)(pl.Np / kBN);
	p.batch = (int)pl.entries; p.batch_inner = inner;
	p.a_batched = pl.a_entries > 1; p.b_batched = pl.b_entries > 1;
	p.Mp = (int)pl.Mp; p.Np = (int)pl.Np;
	p.C = d.c; p.ldc = d.ldc; p.sc_outer = d.sc_outer; p.sc_inner = d.sc_inner; p.accumulate = d.accumulate;
	p.bias = d.epi.bias; p.s_bias_outer = d.epi.s_bias_outer; p.bias_mode = d.epi.bias_mode; p.act = d.epi.act;
	p.mask = d.epi.mask; p.pre = d.epi.pre;
	p.ld_aux = d.epi.ld_aux; p.s_aux_outer = d.epi.s_aux_outer; p.s_aux_inner = d.epi.s_aux_inner;
	p.any_nonfinite = any_a; p.any_b = any_b; p.flags_a = flags_a; p.flags_b = flags_b;
	p.ra0 = pl.ra0; p.ra_outer = pl.ra_outer; p.ra_inner = pl.ra_inner;
	p.a_kw = (int)(pl.pre_a ? round_up(d.pre_a.cols, kAPanelWidth) / kAPanelWidth : pl.KWA);
	p.a_kb0 = (int)pl.a_kb0; p.a_kb_outer = (int)pl.a_kb_outer; p.a_kb_inner = (int)pl.a_kb_inner;
	p.rb0 = pl.rb0; p.rb_outer = pl.rb_outer; p.rb_inner = pl.rb_inner;
	p.A = d.a; p.lda = d.lda; p.sa_outer = d.sa_outer; p.sa_inner = d.sa_inner;
	p.B = d.b; p.ldb = d.ldb; p.sb_outer = d.sb_outer; p.sb_inner = d.sb_inner;
	p.ta = d.ta; p.tb = d.tb; p.err = err;
	p.g = d.gather;
	p.gflags_b = flags_b;
	p.gany_b = any_b_w;

	NNB_TRY((set_smem_attr<kSplit, kBN, kGather, kWide, kMn>(dev)));
	const long long tiles = pl.entries * (p.tiles_m / (kWide ? 2 : 1)) * p.tiles_n;     // work items
	const int grid = (int)std::min<long long>(tiles, sm_count);
	{
		TraceScope ts(s, kGather ? kTraceConv : kTraceGemm, traced);
		gemm_tc_kernel<kSplit, kBN, kGather, kWide, kMn><<<grid, threads_for(kGather), Cf::kSmemBytes, s>>>(tma, tmb, p);
	}
	return cuda_status(cudaGetLastError(), "gemm launch");
}

template <int kSplit, int kMn>
static nnb_status dispatch_mn_bn(cudaStream_t s, int dev, int sm_count, int* err, const GemmDesc& d, const Plan& pl,
		unsigned char* ws, bool traced) {
	if (pl.bn == 256) return launch_main<kSplit, 256, 0, 0, kMn>(s, dev, sm_count, err, d, pl, ws, traced);
	if (pl.bn == 224) return launch_main<kSplit, 224, 0, 0, kMn>(s, dev, sm_count, err, d, pl, ws, traced);
	if (pl.bn == 128) return launch_main<kSplit, 128, 0, 0, kMn>(s, dev, sm_count, err, d, pl, ws, traced);
	return launch_main<kSplit, 64, 0, 0, kMn>(s, dev, sm_count, err, d, pl, ws, traced);
}

template <int kSplit>
static nnb_status dispatch_mn(cudaStream_t s, int dev, int sm_count, int* err, const GemmDesc& d, const Plan& pl,
		unsigned char* ws, bool traced) {
	if (pl.mn == 3) return dispatch_mn_bn<kSplit, 3>(s, dev, sm_count, err, d, pl, ws, traced);
	if (pl.mn == 2) return dispatch_mn_bn<kSplit, 2>(s, dev, sm_count, err, d, pl, ws, traced);
	return dispatch_mn_bn<kSplit, 1>(s, dev, sm_count, err, d, pl, ws, traced);
}

template <int kSplit>
static nnb_status dispatch_bn(cudaStream_t s, int dev, int sm_count, int* err, const GemmDesc& d, const Plan& pl,
		unsigned char* ws, bool traced) {
	if (d.gather.mode != kGatherNone) {         // widths 64, 128, 256 (make_plan never gives 224 here)
		if (pl.bn == 256) return launch_main<kSplit, 256, 1>(s, dev, sm_count, err, d, pl, ws, traced);
		if (pl.bn == 128) return launch_main<kSplit, 128, 1>(s, dev, sm_count, err, d, pl, ws, traced);
		return launch_main<kSplit, 64, 1>(s, dev, sm_count, err, d, pl, ws, traced);
	}
	if (pl.wide) return launch_main<kSplit, 256, 0, 1>(s, dev, sm_count, err, d, pl, ws, traced);
	if (pl.mn) return dispatch_mn<kSplit>(s, dev, sm_count, err, d, pl, ws, traced);
	if (pl.bn == 256) return launch_main<kSplit, 256>(s, dev, sm_count, err, d, pl, ws, traced);
	if (pl.bn == 224) return launch_main<kSplit, 224>(s, dev, sm_count, err, d, pl, ws, traced);
	if (pl.bn == 128) return launch_main<kSplit, 128>(s, dev, sm_count, err, d, pl, ws, traced);
	return launch_main<kSplit, 64>(s, dev, sm_count, err, d, pl, ws, traced);
}

static nnb_status validate(const GemmDesc& d) {
	if (d.mode != NNB_MATH_FP32X3 && d.mode != NNB_MATH_TF32) return fail(NNB_ERR_INVALID, "gemm: unknown math mode %d", d.mode);
	if (d.m < 0 || d.n < 0 || d.k < 0 || d.batch_outer < 0 || d.batch_inner < 1) return fail(NNB_ERR_INVALID, "gemm: negative size");
	if (d.m == 0 || d.n == 0 || d.batch_outer == 0) return NNB_OK;
	if (!d.c) return fail(NNB_ERR_INVALID, "gemm: C is null");
	if (d.ldc < d.n) return fail(NNB_ERR_INVALID, "gemm: ldc %lld < n %lld", d.ldc, d.n);
	const long long lim = 1ll << 30;
	if (d.m > lim || d.n > lim || d.k > lim || d.batch_outer * d.batch_inner > lim)
		return fail(NNB_ERR_UNSUPPORTED, "gemm: dimension above 2^30");
	if (d.k > 0) {
		if (!d.a || (!d.b && d.gather.mode == kGatherNone)) return fail(NNB_ERR_INVALID, "gemm: A or B is null");
		if (d.lda < (d.ta ? d.m : d.k)) return fail(NNB_ERR_INVALID, "gemm: lda %lld too small", d.lda);
		if (d.gather.mode == kGatherNone && d.ldb < (d.tb ? d.k : d.n))
			return fail(NNB_ERR_INVALID, "gemm: ldb %lld too small", d.ldb);
	}
	if (d.epi.bias_mode != kBiasNone && !d.epi.bias) return fail(NNB_ERR_INVALID, "gemm: bias is null");
	if (d.epi.act == kActRelu && !d.epi.mask) return fail(NNB_ERR_INVALID, "gemm: relu mask is null");
	if (d.epi.act == kActGelu && !d.epi.pre) return fail(NNB_ERR_INVALID, "gemm: gelu pre-activation is null");
	if ((d.epi.act != kActNone || d.epi.bias_mode != kBiasNone) && d.k == 0)
		return fail(NNB_ERR_UNSUPPORTED, "gemm: fused epilogue with k == 0");
	if (d.bn != 0 && d.bn != 64 && d.bn != 128 && d.bn != 224 && d.bn != 256)
		return fail(NNB_ERR_INVALID, "gemm: tile width %d", d.bn);
	if (d.packed_b && (d.bn == 0 || d.batch_outer * d.batch_inner != 1))
		return fail(NNB_ERR_INVALID, "gemm: a packed B needs its tile width and a single batch entry");
	if (d.keep_a && (d.ta || d.sa_outer || d.sa_inner || d.packed_b || d.gather.mode != kGatherNone))
		return fail(NNB_ERR_INVALID, "gemm: a kept A pack needs an untransposed A shared by every batch entry");
	if (d.gather.mode != kGatherNone) {
		const GemmGather& g = d.gather;
		if (d.packed_b || d.bn == 224 || !g.src || g.kh < 1 || g.kw < 1 || g.stride < 1 || g.dil < 1 || g.pad < 0 ||
				g.H < 1 || g.W < 1 || g.ho < 1 || g.wo < 1 || (g.mode == kGatherTransposed && g.cout < 1))
			return fail(NNB_ERR_INVALID, "gemm: bad gather geometry");
	}
	return NNB_OK;
}

}  // namespace gemm

namespace gemm {

// Depth cut (the counterpart of the reference's `blocked`, src/kernels/gemm.cpp:453-485): a product
// with a long depth relative to its output width -- a weight gradient, a 512 x 512 output summed over
// thousands of rows -- is computed as P products over consecutive depth pieces into separate buffers,
// which one kernel then adds in piece order. P is planned from (n, k) alone: never from m, the batch,
// the device, the grid or the number of GPUs. A row of C therefore gets the same sequence of
// operations however many rows the call has, which keeps row-sharded products (and the data-parallel
// training step) bitwise identical at any GPU count.
// Pieces are at least 1024 deep and at least n deep (the partial slabs, pieces x m x n, stay small next
// to the operands): a 512-wide weight gradient summed over 4096 rows (one shard of a data-parallel
// batch) is cut into 4 pieces, so it fills the GPU even when a rank computes it for a single shard.
constexpr long long kCutMinDepth = 1024;
constexpr long long kCutMaxPieces = 32;

static int depth_pieces(const GemmDesc& d) {
	if (d.batch_inner != 1 || d.epi.bias_mode != kBiasNone || d.epi.act != kActNone) return 1;
	const long long p = std::min<long long>(kCutMaxPieces, d.k / std::max<long long>(kCutMinDepth, d.n));
	return p >= 2 ? (int)p : 1;
}

// c_e = (accumulate ? c_e : 0) + (((part_e0 + part_e1) + part_e2) + ...), part_ep an m x n slab;
// entry e = blockIdx.y, c_e = c + e * sc
__device__ __forceinline__ float4 f4_add(float4 a, float4 b) {
	return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

__device__ __forceinline__ float depth_v(float x) { return x; }
__device__ __forceinline__ float4 depth_v(float4 x) { return x; }
__device__ __forceinline__ float depth_add(float a, float b) { return a + b; }
__device__ __forceinline__ float4 depth_add(float4 a, float4 b) { return f4_add(a, b); }
__device__ __forceinline__ float depth_zero_fix(float a) { return a + 0.0f; }
__device__ __forceinline__ float4 depth_zero_fix(float4 a) { return f4_add(a, make_float4(0.0f, 0.0f, 0.0f, 0.0f)); }

// c_e = (accumulate ? c_e : 0) + (((part_e0 + part_e1) + part_e2) + ...), part_ep an m x n slab;
// entry e = blockIdx.y, c_e = c + e * sc. V = float or float4 (4 consecutive columns, when n, ldc and
// the pointers allow). A grid-stride walk over the entry's m x (n / W) vectors, so every thread is busy
// whatever the width; up to 8 pieces' loads are issued before their adds, which stay in piece order.
template <typename V>
__global__ void depth_sum_kernel(const float* __restrict__ part, int pieces, long long m, long long n,
		float* __restrict__ c, long long ldc, long long sc, int accumulate) {
	constexpr int W = sizeof(V) / sizeof(float);
	const long long mn = m * n, nv = n / W, total = m * nv;
	part += (long long)blockIdx.y * pieces * mn;
	c += (long long)blockIdx.y * sc;
	const long long stride = mn / W;                 // one slab, in V units
	for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
			idx += (long long)gridDim.x * blockDim.x) {
		const long long i = idx / nv, jv = idx - i * nv;
		const V* src = reinterpret_cast<const V*>(part + i * n) + jv;
		V acc{};
		for (int p = 0; p < pieces; p += 8) {
			V v[8];
#pragma unroll
			for (int u = 0; u < 8; ++u)
				if (p + u < pieces) v[u] = __ldg(src + (long long)(p + u) * stride);
#pragma unroll
			for (int u = 0; u < 8; ++u)
				if (p + u < pieces) acc = (p + u == 0) ? depth_v(v[u]) : depth_add(acc, v[u]);
		}
		V* dst = reinterpret_cast<V*>(c + i * ldc) + jv;
		*dst = accumulate ? depth_add(*dst, acc) : depth_zero_fix(acc);
	}
}

static nnb_status gemm_direct(cudaStream_t s, const DeviceState* dev, const GemmDesc& d) {
	Plan pl;
	NNB_TRY(make_plan(d, pl, d.bn, dev->sm_count));
	void* ws = nullptr;
	NNB_TRY(scratch_alloc(&ws, pl.total, s));
	nnb_status st = d.mode == NNB_MATH_FP32X3
		? dispatch_bn<1>(s, dev->device, dev->sm_count, dev->error_word, d, pl, static_cast<unsigned char*>(ws), true)
		: dispatch_bn<0>(s, dev->device, dev->sm_count, dev->error_word, d, pl, static_cast<unsigned char*>(ws), true);
	nnb_status st2 = scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

// A (ta = 0, one batch entry) packed on its own into d.keep_a, in the kept row-pack layout.
static nnb_status pack_rows_kept(cudaStream_t s, const GemmDesc& d) {
	const int S = d.mode == NNB_MATH_FP32X3 ? 2 : 1;
	const long long rp = row_pack_rows(d.m), kw = round_up(d.k, kAPanelWidth) / kAPanelWidth;
	if (rp * kw * S > INT32_MAX) return fail(NNB_ERR_UNSUPPORTED, "gemm: operand too large to keep packed");
	int* flags = row_pack_flags(d.keep_a, d.m, d.k, S);
	NNB_CUDA_TRY(cudaMemsetAsync(flags, 0, (size_t)(rp + 1) * sizeof(int), s));
	float* out = static_cast<float*>(d.keep_a);
	{
		TraceScope ts(s, kTracePack);
		if (S == 2)
			launch_pack<1>(s, d.a, d.lda, 0, 0, 1, 0, d.m, d.k, rp, kw, kAPanelWidth, kAPanelRows, 1, out, flags, flags + rp);
		else
			launch_pack<0>(s, d.a, d.lda, 0, 0, 1, 0, d.m, d.k, rp, kw, kAPanelWidth, kAPanelRows, 1, out, flags, flags + rp);
	}
	return cuda_status(cudaGetLastError(), "kept pack launch");
}

static nnb_status gemm_depth_cut(cudaStream_t s, const DeviceState* dev, const GemmDesc& d, int pieces) {
	const long long kp = round_up((d.k + pieces - 1) / pieces, kBK);
	pieces = (int)((d.k + kp - 1) / kp);
	const long long full = d.k / kp;                      // pieces of exactly kp
	const long long mn = d.m * d.n, E = d.batch_outer;
	if (E > 65535) return fail(NNB_ERR_UNSUPPORTED, "gemm: more than 65535 batch entries");
	void* ws = nullptr;
	NNB_TRY(scratch_alloc(&ws, (size_t)E * pieces * mn * sizeof(float), s));
	float* part = static_cast<float*>(ws);
	const long long a_step = d.ta ? kp * d.lda : kp, b_step = d.tb ? kp : kp * d.ldb;
	nnb_status st = NNB_OK;
	do {
		GemmDesc e = d;                                     // entries x full pieces, two-level batch
		e.k = kp; e.c = part; e.ldc = d.n; e.accumulate = 0;
		e.batch_outer = E; e.batch_inner = full;
		e.sa_outer = d.sa_outer; e.sa_inner = a_step;
		e.sb_outer = d.sb_outer; e.sb_inner = b_step;
		e.sc_outer = (long long)pieces * mn; e.sc_inner = mn;
		if ((st = gemm_direct(s, dev, e)) != NNB_OK) break;
		if (full < pieces) {                                 // the shorter last piece of every entry
			GemmDesc t = d;
			t.k = d.k - full * kp;
			t.a = d.a + full * a_step; t.b = d.b + full * b_step;
			t.c = part + full * mn; t.ldc = d.n; t.accumulate = 0;
			t.batch_outer = E; t.batch_inner = 1;
			t.sc_outer = (long long)pieces * mn;
			if ((st = gemm_direct(s, dev, t)) != NNB_OK) break;
		}
		const bool vec = d.n % 4 == 0 && d.ldc % 4 == 0 && d.sc_outer % 4 == 0 &&
			(reinterpret_cast<uintptr_t>(d.c) & 15) == 0;
		const long long nv = vec ? d.n / 4 : d.n;
		// about 16 blocks per SM over all entries, no more blocks than an entry has vectors
		const unsigned bx = (unsigned)std::max<long long>(1, std::min<long long>((d.m * nv + 255) / 256,
			std::max<long long>(1, (148 * 16) / E)));
		{
			TraceScope ts(s, kTraceAux);
			if (vec)
				depth_sum_kernel<float4><<<dim3(bx, (unsigned)E), 256, 0, s>>>(part, pieces, d.m, d.n, d.c, d.ldc,
					d.sc_outer, d.accumulate);
			else
				depth_sum_kernel<float><<<dim3(bx, (unsigned)E), 256, 0, s>>>(part, pieces, d.m, d.n, d.c, d.ldc,
					d.sc_outer, d.accumulate);
		}
		st = cuda_status(cudaGetLastError(), "depth sum launch");
	} while (0);
	nnb_status st2 = scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

}  // namespace gemm

nnb_status gemm_run(cudaStream_t s, const GemmDesc& d) {
	using namespace gemm;
	NNB_TRY(validate(d));
	if (d.m == 0 || d.n == 0 || d.batch_outer == 0) return NNB_OK;
	DeviceState* dev = nullptr;
	NNB_TRY(device_state(&dev));
	if (d.k == 0) {
		if (d.accumulate) return NNB_OK;
		const long long entries = d.batch_outer * d.batch_inner;
		dim3 g((unsigned)std::min<long long>((d.m * d.n + 255) / 256, 4096), 1, (unsigned)entries);
		TraceScope ts(s, kTraceAux);
		zero_fill_kernel<<<g, 256, 0, s>>>(d.c, d.ldc, d.sc_outer, d.sc_inner, (int)d.batch_inner, (int)d.m, (int)d.n);
		return cuda_status(cudaGetLastError(), "zero fill launch");
	}
	const int pieces = d.gather.mode != kGatherNone ? 1 : depth_pieces(d);
	if (pieces > 1 && d.packed_b) return fail(NNB_ERR_INVALID, "gemm: a packed B with a depth cut");
	if (pieces > 1 && d.keep_a) {
		// the whole of A packed once into the kept buffer, every depth piece reading its columns from it
		NNB_TRY(pack_rows_kept(s, d));
		GemmDesc e = d;
		e.keep_a = nullptr;
		e.pre_a.buf = d.keep_a; e.pre_a.base = d.a; e.pre_a.ld = d.lda; e.pre_a.rows = d.m; e.pre_a.cols = d.k;
		e.pre_a.mode = d.mode;
		return gemm_depth_cut(s, dev, e, pieces);
	}
	if (pieces > 1) return gemm_depth_cut(s, dev, d, pieces);
	return gemm_direct(s, dev, d);
}

int gemm_tile_width(const GemmDesc& d, int sms) {
	return gemm::choose_bn(d.m, d.n, d.batch_outer * d.batch_inner, sms > 0 ? sms : 148);
}

int gemm_depth_pieces(const GemmDesc& d) { return gemm::depth_pieces(d); }

size_t gemm_row_pack_bytes(long long rows, long long cols, int mode) {
	const int S = mode == NNB_MATH_FP32X3 ? 2 : 1;
	return gemm::row_pack_panel_bytes(rows, cols, S) + (size_t)(gemm::row_pack_rows(rows) + 1) * sizeof(int);
}

size_t gemm_packed_b_bytes(const GemmDesc& d, int bn) {
	gemm::Plan pl;
	if (gemm::make_plan(d, pl, bn) != NNB_OK) return 0;
	return (size_t)gemm::round_up((long long)pl.rows_b * gemm::kBK * 4, 1024) + (size_t)(pl.Np + 1) * sizeof(int);
}

nnb_status gemm_pack_b(cudaStream_t s, const GemmDesc& d, int bn, void* buf) {
	using namespace gemm;
	NNB_TRY(validate(d));
	if (bn != 64 && bn != 128 && bn != 224 && bn != 256) return fail(NNB_ERR_INVALID, "gemm_pack_b: tile width %d", bn);
	if (d.batch_outer * d.batch_inner != 1 || d.k == 0 || d.n == 0)
		return fail(NNB_ERR_INVALID, "gemm_pack_b: needs one batch entry and k, n > 0");
	if (!buf) return fail(NNB_ERR_INVALID, "gemm_pack_b: buffer is null");
	Plan pl;
	NNB_TRY(make_plan(d, pl, bn));
	float* pb = static_cast<float*>(buf);
	int* flags = reinterpret_cast<int*>(static_cast<unsigned char*>(buf) + round_up((long long)pl.rows_b * kBK * 4, 1024));
	NNB_CUDA_TRY(cudaMemsetAsync(flags, 0, (size_t)(pl.Np + 1) * sizeof(int), s));
	{
		TraceScope ts(s, kTracePack);
		if (d.mode == NNB_MATH_FP32X3)
			launch_pack<1>(s, d.b, d.ldb, 0, 0, 1, !d.tb, d.n, d.k, pl.Np, pl.KB, kBK, b_panel_rows(bn), 1, pb, flags,
				flags + pl.Np);
		else
			launch_pack<0>(s, d.b, d.ldb, 0, 0, 1, !d.tb, d.n, d.k, pl.Np, pl.KB, kBK, b_panel_rows(bn), 1, pb, flags,
				flags + pl.Np);
	}
	return cuda_status(cudaGetLastError(), "gemm_pack_b launch");
}

}  // namespace nnb

extern "C" {

nnb_status nnb_sgemm(void* stream, int trans_a, int trans_b, size_t m, size_t n, size_t k,
		const float* a, size_t lda, const float* b, size_t ldb, float* c, size_t ldc, int accumulate) {
	return nnb_sgemm_ex(stream, trans_a, trans_b, m, n, k, a, lda, b, ldb, c, ldc, accumulate, nnb::math_mode());
}

nnb_status nnb_sgemm_ex(void* stream, int trans_a, int trans_b, size_t m, size_t n, size_t k,
		const float* a, size_t lda, const float* b, size_t ldb, float* c, size_t ldc, int accumulate,
		int math_mode) {
	nnb::GemmDesc d;
	d.ta = trans_a != 0; d.tb = trans_b != 0;
	d.m = (long long)m; d.n = (long long)n; d.k = (long long)k;
	d.a = a; d.lda = (long long)lda; d.b = b; d.ldb = (long long)ldb; d.c = c; d.ldc = (long long)ldc;
	d.accumulate = accumulate != 0; d.mode = math_mode;
	return nnb::gemm_run(static_cast<cudaStream_t>(stream), d);
}

nnb_status nnb_sgemm_strided_batched(void* stream, int trans_a, int trans_b, size_t m, size_t n,
		size_t k, const float* a, size_t lda, size_t stride_a, const float* b, size_t ldb,
		size_t stride_b, float* c, size_t ldc, size_t stride_c, size_t batch, int accumulate,
		int math_mode) {
	if (batch > 1 && stride_c == 0)
		return nnb::fail(NNB_ERR_INVALID, "sgemm_strided_batched: stride_c must be nonzero for batch > 1");
	nnb::GemmDesc d;
	d.ta = trans_a != 0; d.tb = trans_b != 0;
	d.m = (long long)m; d.n = (long long)n; d.k = (long long)k;
	d.a = a; d.lda = (long long)lda; d.b = b; d.ldb = (long long)ldb; d.c = c; d.ldc = (long long)ldc;
	d.batch_outer = (long long)batch;
	d.sa_outer = (long long)stride_a; d.sb_outer = (long long)stride_b; d.sc_outer = (long long)stride_c;
	d.accumulate = accumulate != 0; d.mode = math_mode;
	return nnb::gemm_run(static_cast<cudaStream_t>(stream), d);
}

}  // extern "C"

// =============================================================================================
// Allocation-free GEMM entry point (nnb_sgemm_noalloc)
//
// Some callers of this library cannot allocate device memory on the call path: a host that has
// already handed every byte of the GPU to its own arena, a real-time loop that must not enter the
// driver's allocator (cudaMalloc synchronises the device and cudaMallocAsync can grow a pool at an
// unpredictable moment), or a host whose allocator hooks are off limits. For them this entry point
// runs the same pack and tcgen05 kernels as nnb_sgemm_ex, with the packed operands and flags in a
// fixed, file-scope device array instead of scratch from the memory pool.
//
// - The array holds kNoAllocScratchBytes (32 MiB). Every GPU that loads this library keeps it
//   until the process exits.
// - The first call on a device, with that device current, looks up the array's device address
//   (cudaGetSymbolAddress) and sets the kernels' shared-memory limit. Make that first call before
//   any stream capture.
// - All calls share the array and it keeps the last call's contents; the non-finite flags that must
//   start at zero are cleared on the stream at every call. Calls that overlap on the GPU (different
//   streams, or different host threads, without ordering between them) race on the array.
// - Calls needing more scratch than the array holds are rejected with NNB_ERR_UNSUPPORTED before
//   anything is enqueued. The column tile is always 256 wide here, so the limit is exactly the
//   one stated in include/nnb.h.
// =============================================================================================

namespace nnb {
namespace gemm {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ int g_noalloc_error;

struct NoAllocDevice {
	bool ready = false;
	unsigned char* scratch = nullptr;   // device address of g_noalloc_scratch on this device
	int* error = nullptr;               // device address of g_noalloc_error on this device
	int sm_count = 0;
};

static NoAllocDevice g_noalloc_devices[64];
static std::mutex g_noalloc_mutex;

// Once per device, with that device current: resolve the array's device address (in host code
// the symbol itself is only a host-side stand-in) and set the kernels' shared-memory limit.
static nnb_status noalloc_setup(NoAllocDevice** out, int* dev_out) {
	int dev = 0;
	NNB_CUDA_TRY(cudaGetDevice(&dev));
	if (dev < 0 || dev >= 64) return fail(NNB_ERR_UNSUPPORTED, "sgemm_noalloc: device index %d out of range", dev);
	*dev_out = dev;
	std::lock_guard<std::mutex> lock(g_noalloc_mutex);
	NoAllocDevice& d = g_noalloc_devices[dev];
	if (!d.ready) {
		int major = 0, sms = 0;
		NNB_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
		if (major != 10) return fail(NNB_ERR_UNSUPPORTED, "sgemm_noalloc: device %d is not sm_100", dev);
		NNB_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
		void* scratch = nullptr;
		void* error = nullptr;
		cudaError_t e = cudaGetSymbolAddress(&scratch, g_noalloc_scratch);
		if (e != cudaSuccess) return cuda_status(e, "sgemm_noalloc: cudaGetSymbolAddress(scratch)");
		e = cudaGetSymbolAddress(&error, g_noalloc_error);
		if (e != cudaSuccess) return cuda_status(e, "sgemm_noalloc: cudaGetSymbolAddress(error word)");
		NNB_TRY((set_smem_attr<1, 256>(dev)));
		NNB_TRY((set_smem_attr<0, 256>(dev)));
		d.scratch = static_cast<unsigned char*>(scratch);
		d.error = static_cast<int*>(error);
		d.sm_count = sms;
		d.ready = true;
	}
	*out = &d;
	return NNB_OK;
}

}  // namespace gemm
}  // namespace nnb

extern "C" nnb_status nnb_sgemm_noalloc(void* stream, int trans_a, int trans_b, size_t m, size_t n,
		size_t k, const float* a, size_t lda, const float* b, size_t ldb, float* c, size_t ldc,
		int accumulate, int math_mode) {
	using namespace nnb;
	using namespace nnb::gemm;
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	GemmDesc d;
	d.ta = trans_a != 0; d.tb = trans_b != 0;
	d.m = (long long)m; d.n = (long long)n; d.k = (long long)k;
	d.a = a; d.lda = (long long)lda; d.b = b; d.ldb = (long long)ldb; d.c = c; d.ldc = (long long)ldc;
	d.accumulate = accumulate != 0; d.mode = math_mode;
	NNB_TRY(validate(d));
	if (d.m == 0 || d.n == 0) return NNB_OK;
	NoAllocDevice* nd = nullptr;
	int dev = 0;
	NNB_TRY(noalloc_setup(&nd, &dev));
	if (d.k == 0) {
		if (d.accumulate) return NNB_OK;
		dim3 g((unsigned)std::min<long long>((d.m * d.n + 255) / 256, 4096), 1, 1);
		zero_fill_kernel<<<g, 256, 0, s>>>(d.c, d.ldc, 0, 0, 1, (int)d.m, (int)d.n);
		return cuda_status(cudaGetLastError(), "sgemm_noalloc: zero fill launch");
	}
	Plan pl;
	NNB_TRY(make_plan(d, pl, 256));
	if (pl.total > kNoAllocScratchBytes)
		return fail(NNB_ERR_UNSUPPORTED,
			"sgemm_noalloc: %lld x %lld x %lld needs %zu bytes of scratch; the static buffer holds %zu "
			"(packed operands take (roundup(m,128) * roundup(k,32) + roundup(n,256) * roundup(k,16)) * %d * 4 bytes)",
			d.m, d.n, d.k, pl.total, kNoAllocScratchBytes, pl.S);
	if (d.mode == NNB_MATH_FP32X3)
		return launch_main<1, 256>(s, dev, nd->sm_count, nd->error, d, pl, nd->scratch, false);
	return launch_main<0, 256>(s, dev, nd->sm_count, nd->error, d, pl, nd->scratch, false);
}

extern "C" nnb_status nnb_sgemm_noalloc_error(void* stream, int* out, int clear) {
	using namespace nnb;
	using namespace nnb::gemm;
	if (!out) return fail(NNB_ERR_INVALID, "sgemm_noalloc_error: out is null");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	NoAllocDevice* nd = nullptr;
	int dev = 0;
	NNB_TRY(noalloc_setup(&nd, &dev));
	// Plain copies from and to the symbol on the caller's stream: no allocation; the host value is
	// read once the stream has reached this point.
	int word = 0;
	NNB_CUDA_TRY(cudaMemcpyFromSymbolAsync(&word, g_noalloc_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s));
	NNB_CUDA_TRY(cudaStreamSynchronize(s));
	*out = word;
	if (clear && word != 0) {
		static const int zero = 0;
		NNB_CUDA_TRY(cudaMemcpyToSymbolAsync(g_noalloc_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s));
		NNB_CUDA_TRY(cudaStreamSynchronize(s));
	}
	return NNB_OK;
}
