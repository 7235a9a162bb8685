// gemm.cu -- the fp32 GEMM of nn-cpp (nn::kernels::sgemm, include/nn/kernels/gemm.hpp:57-59)
// rebuilt for B200 (sm_100a): a pack kernel plus a persistent tcgen05 tensor-core kernel.
//
// Pack (the counterpart of pack_a / pack_b, src/kernels/gemm.cpp:79,126): op(A) and op(B)^T are
// rewritten, whatever their transpose flag and leading dimension, into K-major "panels" of
// 128 rows x 16 floats (8 KB, contiguous), zero-padded to whole panels. In 3xTF32 mode each
// value x is stored twice, as hi = tf32(x) and lo = tf32(x - hi) (the split-precision method of
// Ootomo & Yokota, 2022), so C = Ahi*Bhi + Ahi*Blo + Alo*Bhi carries about 21 mantissa bits.
// Rows holding Inf or NaN are flagged; the epilogue recomputes the IEEE result of those
// elements (+-Inf or NaN) so non-finite inputs propagate exactly as the reference's fp32 loop.
//
// Main kernel, one CTA per SM, 6 warps:
//   warp 0     TMA producer: each stage = the A panels (hi[,lo]) of a 128-row tile and the B
//              panels of a 256-column tile for one 16-wide k-block, 64-byte swizzled;
//   warp 1     MMA issuer: tcgen05.mma.kind::tf32 128x256x8 into a TMEM accumulator, two
//              accumulators (512 TMEM columns) so the epilogue of tile i overlaps tile i+1;
//   warps 2-5  epilogue: tcgen05.ld -> (C +) acc -> global, with bounds checks.
// There is no split-K and the k order is fixed, so every element of C is produced by the same
// sequence of operations whatever the grid size, the number of GPUs or the M-shard it sits in.
#include <algorithm>

#include "nnb_internal.h"
#include "nnb_ptx.cuh"
#include "nnb_trace.h"

namespace nnb {
namespace gemm {

constexpr int kBM = 128;                 // rows of C per tile (MMA M)
constexpr int kBN = 256;                 // columns of C per tile (MMA N)
constexpr int kBK = 16;                  // floats of depth per pipeline stage (one 64 B row)
constexpr int kPanelRows = 128;          // rows per packed panel
constexpr int kPanelFloats = kPanelRows * kBK;
constexpr int kPanelBytes = kPanelFloats * 4;   // 8 KB
constexpr int kGroupM = 16;              // tiles of M walked together for L2 reuse of B
constexpr int kThreads = 192;

template <int kSplit>
struct Cfg {
	static constexpr int S = kSplit ? 2 : 1;                 // hi[, lo]
	static constexpr int kABytes = S * kBM * kBK * 4;        // 16 KB / 8 KB
	static constexpr int kBBytes = S * kBN * kBK * 4;        // 32 KB / 16 KB
	static constexpr int kStageBytes = kABytes + kBBytes;
	static constexpr int kStages = kSplit ? 4 : 8;
	static constexpr int kSmemBytes = kStages * kStageBytes + 1024;
};

struct Params {
	int M, N, K, KB;
	int tiles_m, tiles_n, batch;
	int a_batched, b_batched;        // 0: operand shared by every batch entry
	int Mp, Np;                      // padded row counts of the packed operands
	float* C;
	long long ldc, stride_c;
	int accumulate;
	// Exact IEEE handling of non-finite inputs
	const int* any_nonfinite;
	const int* flags_a;              // [a_batches][Mp]
	const int* flags_b;              // [b_batches][Np]
	const float* A;
	long long lda, stride_a;
	const float* B;
	long long ldb, stride_b;
	int ta, tb;
	int* err;
};

// ---------------------------------------------------------------------------------------------
// Pack
// ---------------------------------------------------------------------------------------------

__device__ __forceinline__ float to_tf32(float x) {
	uint32_t r;
	asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
	return __uint_as_float(r);
}

// hi + lo ~= x with hi, lo both TF32; finite x never gives a non-finite part.
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
	hi = to_tf32(x);
	if (isinf(hi)) hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);  // |x| near FLT_MAX
	lo = to_tf32(x - hi);
}

// One block: 32 rows x 64 depth of op(X) (X stored rows x K, or K x rows when trans), written
// as 4 k-blocks of the packed panel layout. grid = (Rp/32, ceil(Kp/64), batches).
template <int kSplit>
__global__ void __launch_bounds__(256) pack_kernel(const float* __restrict__ X, long long ldx,
		long long stride_x, int trans, int R, int K, int Rp, int KB, float* __restrict__ out,
		int* __restrict__ flags, int* __restrict__ any_flag) {
	constexpr int S = kSplit ? 2 : 1;
	__shared__ float tile[32][65];
	const int t = threadIdx.x;
	const int r0 = blockIdx.x * 32, k0 = blockIdx.y * 64, bi = blockIdx.z;
	const float* Xb = X + (long long)bi * stride_x;
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
	const int e = 2 * t;                 // element pair inside a 32 x 16 k-block slab
	const int rl = e >> 4, kl = e & 15;
	const long long batch_off = (long long)bi * Rp * KB * 16 * S;
	bool bad = false;
#pragma unroll
	for (int w = 0; w < 4; ++w) {
		const int kb = (k0 >> 4) + w;
		if (kb >= KB) break;
		float x0 = tile[rl][w * 16 + kl], x1 = tile[rl][w * 16 + kl + 1];
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
		const long long panel = ((long long)(r0 / kPanelRows) * KB + kb) * S;
		float* dst = out + batch_off + panel * kPanelFloats + (r0 % kPanelRows) * 16 + e;
		*reinterpret_cast<float2*>(dst) = make_float2(h0, h1);
		if (kSplit) *reinterpret_cast<float2*>(dst + kPanelFloats) = make_float2(l0, l1);
	}
	if (bad) {
		atomicOr(flags + (long long)bi * Rp + r0 + rl, 1);
		atomicOr(any_flag, 1);
	}
}

// ---------------------------------------------------------------------------------------------
// Main kernel
// ---------------------------------------------------------------------------------------------

__device__ __forceinline__ void tile_coords(int t, const Params& p, int& bi, int& mt, int& nt) {
	const int per_batch = p.tiles_m * p.tiles_n;
	bi = t / per_batch;
	const int r = t - bi * per_batch;
	const int group = r / (kGroupM * p.tiles_n);
	const int first_m = group * kGroupM;
	const int gsz = min(p.tiles_m - first_m, kGroupM);
	const int in = r - group * kGroupM * p.tiles_n;
	mt = first_m + in % gsz;
	nt = in / gsz;
}

// IEEE value of sum_p op(A)(i,p)*op(B)(p,j) for an element whose row or column holds Inf/NaN:
// NaN if any product is NaN or both infinities occur, else the infinity that occurs.
__device__ __noinline__ float nonfinite_result(const Params& p, int bi, int i, int j, float v) {
	const float* A = p.A + (p.a_batched ? (long long)bi * p.stride_a : 0);
	const float* B = p.B + (p.b_batched ? (long long)bi * p.stride_b : 0);
	bool nan = false, pinf = false, ninf = false;
	for (int q = 0; q < p.K; ++q) {
		const float a = p.ta ? A[(long long)q * p.lda + i] : A[(long long)i * p.lda + q];
		const float b = p.tb ? B[(long long)j * p.ldb + q] : B[(long long)q * p.ldb + j];
		const float pr = a * b;
		if (pr != pr) nan = true;
		else if (isinf(pr)) (pr > 0.0f ? pinf : ninf) = true;
	}
	if (nan || (pinf && ninf)) return __int_as_float(0x7fc00000);
	if (pinf) return __int_as_float(0x7f800000);
	if (ninf) return __int_as_float(0xff800000);
	return v;
}

template <int kSplit>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a,
		const __grid_constant__ CUtensorMap tm_b, const Params p) {
	using C = Cfg<kSplit>;
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
			mbar_init(smem_u32(&full_bar[s]), 1);
			mbar_init(smem_u32(&empty_bar[s]), 1);
		}
		for (int b = 0; b < 2; ++b) {
			mbar_init(smem_u32(&accf_bar[b]), 1);
			mbar_init(smem_u32(&acce_bar[b]), 4);
		}
		abort_sh = 0;
		fence_mbar_init();
		tma_prefetch_desc(&tm_a);
		tma_prefetch_desc(&tm_b);
	}
	if (warp == 1) {
		tmem_alloc(smem_u32(&tmem_base_sh), 512);
		tmem_relinquish();
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem_base = tmem_base_sh;
	volatile int* abort_flag = &abort_sh;

	const int num_tiles = p.batch * p.tiles_m * p.tiles_n;
	const int a_panels = p.Mp / kPanelRows, b_panels = p.Np / kPanelRows;

	if (warp == 0) {
		if (lane == 0) {
			// ------------------------------ TMA producer ------------------------------
			int stage = 0;
			uint32_t phase = 0;
			for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
				int bi, mt, nt;
				tile_coords(t, p, bi, mt, nt);
				const int ab = p.a_batched ? bi : 0, bb = p.b_batched ? bi : 0;
				bool ok = true;
				for (int kb = 0; kb < p.KB; ++kb) {
					if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1, p.err, kDevTimeoutEmpty, abort_flag)) {
						ok = false;
						break;
					}
					const uint32_t fb = smem_u32(&full_bar[stage]);
					mbar_arrive_expect_tx(fb, C::kStageBytes);
					const uint32_t base = smem_u32(smem + stage * C::kStageBytes);
					const int ya = (int)((((long long)ab * a_panels + mt) * p.KB + kb) * S * kPanelRows);
#pragma unroll
					for (int s = 0; s < S; ++s) tma_load_2d(base + s * kPanelBytes, &tm_a, fb, 0, ya + s * kPanelRows);
#pragma unroll
					for (int q = 0; q < 2; ++q) {
						const int yb = (int)((((long long)bb * b_panels + 2 * nt + q) * p.KB + kb) * S * kPanelRows);
#pragma unroll
						for (int s = 0; s < S; ++s)
							tma_load_2d(base + C::kABytes + s * (kBN * kBK * 4) + q * kPanelBytes, &tm_b, fb, 0,
								yb + s * kPanelRows);
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
		if (lane == 0) {
			// ------------------------------ MMA issuer --------------------------------
			constexpr uint32_t idesc = idesc_tf32(kBM, kBN);
			int stage = 0;
			uint32_t phase = 0;
			int it = 0;
			for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
				const int buf = it & 1;
				const uint32_t acc_phase = (it >> 1) & 1;
				if (!mbar_wait(smem_u32(&acce_bar[buf]), acc_phase ^ 1, p.err, kDevTimeoutAccumFree, abort_flag)) break;
				tc_fence_after();
				const uint32_t d_tmem = tmem_base + buf * kBN;
				bool ok = true;
				for (int kb = 0; kb < p.KB; ++kb) {
					if (!mbar_wait(smem_u32(&full_bar[stage]), phase, p.err, kDevTimeoutFull, abort_flag)) {
						ok = false;
						break;
					}
					tc_fence_after();
					const uint32_t base = smem_u32(smem + stage * C::kStageBytes);
#pragma unroll
					for (int kk = 0; kk < kBK / 8; ++kk) {
						const uint32_t off = kk * 32;    // 8 tf32 = 32 bytes along the swizzled row
						const uint64_t a_hi = smem_desc_k_sw64(base + off);
						const uint64_t b_hi = smem_desc_k_sw64(base + C::kABytes + off);
						const uint32_t first = (kb == 0 && kk == 0) ? 0u : 1u;
						if (kSplit) {
							const uint64_t a_lo = smem_desc_k_sw64(base + kPanelBytes + off);
							const uint64_t b_lo = smem_desc_k_sw64(base + C::kABytes + kBN * kBK * 4 + off);
							mma_tf32(d_tmem, a_lo, b_hi, idesc, first);
							mma_tf32(d_tmem, a_hi, b_lo, idesc, 1u);
							mma_tf32(d_tmem, a_hi, b_hi, idesc, 1u);
						} else {
							mma_tf32(d_tmem, a_hi, b_hi, idesc, first);
						}
					}
					mma_commit(smem_u32(&empty_bar[stage]));
					if (++stage == kStages) {
						stage = 0;
						phase ^= 1;
					}
				}
				if (!ok) break;
				mma_commit(smem_u32(&accf_bar[buf]));
			}
		}
	} else {
		// ---------------------------------- epilogue ----------------------------------
		const int quad = warp & 3;                 // TMEM lanes this warp may access
		const int row = quad * 32 + lane;
		const bool vec_ok = (p.ldc % 4 == 0) && (p.stride_c % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0);
		int it = 0;
		for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
			const int buf = it & 1;
			const uint32_t acc_phase = (it >> 1) & 1;
			if (!mbar_wait(smem_u32(&accf_bar[buf]), acc_phase, p.err, kDevTimeoutAccum, abort_flag)) break;
			tc_fence_after();
			int bi, mt, nt;
			tile_coords(t, p, bi, mt, nt);
			const int gm = mt * kBM + row;
			const bool row_ok = gm < p.M;
			float* crow = p.C + (long long)bi * p.stride_c + (long long)gm * p.ldc;
			const bool fix = *p.any_nonfinite != 0;
			const bool row_bad = fix && row_ok && p.flags_a[(long long)(p.a_batched ? bi : 0) * p.Mp + gm] != 0;
			const int* fcol = p.flags_b + (long long)(p.b_batched ? bi : 0) * p.Np;
#pragma unroll 1
			for (int ch = 0; ch < kBN / 32; ++ch) {
				const int gn0 = nt * kBN + ch * 32;
				if (gn0 >= p.N) break;                 // warp-uniform
				uint32_t r[32];
				tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + buf * kBN + ch * 32, r);
				tmem_wait_ld();
				if (!row_ok) continue;
				float v[32];
#pragma unroll
				for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
				if (fix) {
#pragma unroll
					for (int j = 0; j < 32; ++j) {
						const int gn = gn0 + j;
						if (gn < p.N && (row_bad || fcol[gn] != 0)) v[j] = nonfinite_result(p, bi, gm, gn, v[j]);
					}
				}
				if (vec_ok && gn0 + 32 <= p.N) {
					float4* c4 = reinterpret_cast<float4*>(crow + gn0);
#pragma unroll
					for (int j = 0; j < 8; ++j) {
						float4 o = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
						if (p.accumulate) {
							const float4 c = c4[j];
							o.x = c.x + o.x; o.y = c.y + o.y; o.z = c.z + o.z; o.w = c.w + o.w;
						} else {
							o.x += 0.0f; o.y += 0.0f; o.z += 0.0f; o.w += 0.0f;
						}
						c4[j] = o;
					}
				} else {
#pragma unroll
					for (int j = 0; j < 32; ++j) {
						const int gn = gn0 + j;
						if (gn < p.N) crow[gn] = p.accumulate ? crow[gn] + v[j] : v[j] + 0.0f;
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
		tmem_dealloc(tmem_base, 512);
	}
}

// Zero fill of an m x n region per batch entry: the k == 0 product (gemm.cpp:346-348).
__global__ void zero_fill_kernel(float* c, long long ldc, long long stride_c, int m, int n) {
	float* cb = c + (long long)blockIdx.z * stride_c;
	for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < (long long)m * n;
			idx += (long long)gridDim.x * blockDim.x) {
		const long long i = idx / n, j = idx - i * n;
		cb[i * ldc + j] = 0.0f;
	}
}

inline long long round_up(long long x, long long a) { return (x + a - 1) / a * a; }

template <int kSplit>
nnb_status launch(cudaStream_t s, const DeviceState* dev, int ta, int tb, long long m, long long n,
		long long k, const float* a, long long lda, long long sa, const float* b, long long ldb,
		long long sb, float* c, long long ldc, long long sc, long long batch, int acc) {
	using Cf = Cfg<kSplit>;
	constexpr int S = Cf::S;
	const long long Mp = round_up(m, kBM), Np = round_up(n, kBN), Kp = round_up(k, kBK);
	const long long KB = Kp / kBK;
	const long long a_b = sa ? batch : 1, b_b = sb ? batch : 1;
	const long long rows_a = a_b * Mp * KB * S, rows_b = b_b * Np * KB * S;   // packed 16-float rows
	if (rows_a > INT32_MAX || rows_b > INT32_MAX)
		return fail(NNB_ERR_UNSUPPORTED, "sgemm: operands too large for one launch (packed rows %lld, %lld)",
			rows_a, rows_b);
	const long long tiles = batch * (Mp / kBM) * (Np / kBN);
	if (tiles > INT32_MAX) return fail(NNB_ERR_UNSUPPORTED, "sgemm: too many tiles");

	const size_t bytes_a = (size_t)rows_a * kBK * 4, bytes_b = (size_t)rows_b * kBK * 4;
	const size_t flag_ints = (size_t)(a_b * Mp + b_b * Np + 1);
	const size_t off_b = round_up(bytes_a, 1024), off_f = off_b + round_up(bytes_b, 1024);
	const size_t total = off_f + flag_ints * sizeof(int);
	void* ws = nullptr;
	NNB_TRY(scratch_alloc(&ws, total, s));
	float* pa = static_cast<float*>(ws);
	float* pb = reinterpret_cast<float*>(static_cast<char*>(ws) + off_b);
	int* flags = reinterpret_cast<int*>(static_cast<char*>(ws) + off_f);
	int* flags_a = flags;
	int* flags_b = flags + a_b * Mp;
	int* any = flags + a_b * Mp + b_b * Np;

	nnb_status st = NNB_OK;
	do {
		if ((st = cuda_status(cudaMemsetAsync(flags, 0, flag_ints * sizeof(int), s), "memset flags")) != NNB_OK) break;
		dim3 ga((unsigned)(Mp / 32), (unsigned)((Kp + 63) / 64), (unsigned)a_b);
		{
			TraceScope ts(s, kTracePack);
			pack_kernel<kSplit><<<ga, 256, 0, s>>>(a, lda, sa, ta, (int)m, (int)k, (int)Mp, (int)KB, pa, flags_a, any);
		}
		dim3 gb((unsigned)(Np / 32), (unsigned)((Kp + 63) / 64), (unsigned)b_b);
		{
			TraceScope ts(s, kTracePack);
			pack_kernel<kSplit><<<gb, 256, 0, s>>>(b, ldb, sb, !tb, (int)n, (int)k, (int)Np, (int)KB, pb, flags_b, any);
		}
		if ((st = cuda_status(cudaGetLastError(), "pack launch")) != NNB_OK) break;

		CUtensorMap tma, tmb;
		if ((st = encode_tiled_2d(&tma, pa, kBK, (uint64_t)rows_a, kBK * 4, kBK, kPanelRows,
				CU_TENSOR_MAP_SWIZZLE_64B)) != NNB_OK) break;
		if ((st = encode_tiled_2d(&tmb, pb, kBK, (uint64_t)rows_b, kBK * 4, kBK, kPanelRows,
				CU_TENSOR_MAP_SWIZZLE_64B)) != NNB_OK) break;

		Params p;
		p.M = (int)m; p.N = (int)n; p.K = (int)k; p.KB = (int)KB;
		p.tiles_m = (int)(Mp / kBM); p.tiles_n = (int)(Np / kBN); p.batch = (int)batch;
		p.a_batched = sa != 0; p.b_batched = sb != 0;
		p.Mp = (int)Mp; p.Np = (int)Np;
		p.C = c; p.ldc = ldc; p.stride_c = sc; p.accumulate = acc;
		p.any_nonfinite = any; p.flags_a = flags_a; p.flags_b = flags_b;
		p.A = a; p.lda = lda; p.stride_a = sa; p.B = b; p.ldb = ldb; p.stride_b = sb;
		p.ta = ta; p.tb = tb; p.err = dev->error_word;

		static bool attr_set[64][2] = {};
		if (!attr_set[dev->device & 63][kSplit]) {
			if ((st = cuda_status(cudaFuncSetAttribute(gemm_tc_kernel<kSplit>,
					cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::kSmemBytes), "smem attribute")) != NNB_OK) break;
			attr_set[dev->device & 63][kSplit] = true;
		}
		const int grid = (int)std::min<long long>(tiles, dev->sm_count);
		{
			TraceScope ts(s, kTraceGemm);
			gemm_tc_kernel<kSplit><<<grid, kThreads, Cf::kSmemBytes, s>>>(tma, tmb, p);
		}
		st = cuda_status(cudaGetLastError(), "gemm launch");
	} while (0);
	nnb_status st2 = scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

nnb_status sgemm_entry(void* stream, int ta, int tb, size_t m, size_t n, size_t k, const float* a,
		size_t lda, size_t sa, const float* b, size_t ldb, size_t sb, float* c, size_t ldc,
		size_t sc, size_t batch, int acc, int mode) {
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	if (mode != NNB_MATH_FP32X3 && mode != NNB_MATH_TF32)
		return fail(NNB_ERR_INVALID, "sgemm: unknown math mode %d", mode);
	if (m == 0 || n == 0 || batch == 0) return NNB_OK;
	if (!c) return fail(NNB_ERR_INVALID, "sgemm: C is null");
	if (ldc < n) return fail(NNB_ERR_INVALID, "sgemm: ldc %zu < n %zu", ldc, n);
	const size_t lim = (size_t)1 << 30;
	if (m > lim || n > lim || k > lim || batch > lim)
		return fail(NNB_ERR_UNSUPPORTED, "sgemm: dimension above 2^30");
	DeviceState* dev = nullptr;
	NNB_TRY(device_state(&dev));
	if (k == 0) {
		if (acc) return NNB_OK;
		dim3 g((unsigned)std::min<size_t>((m * n + 255) / 256, 4096), 1, (unsigned)batch);
		TraceScope ts(s, kTraceAux);
		zero_fill_kernel<<<g, 256, 0, s>>>(c, (long long)ldc, (long long)sc, (int)m, (int)n);
		return cuda_status(cudaGetLastError(), "zero fill launch");
	}
	if (!a || !b) return fail(NNB_ERR_INVALID, "sgemm: A or B is null");
	if (lda < (ta ? m : k)) return fail(NNB_ERR_INVALID, "sgemm: lda %zu too small", lda);
	if (ldb < (tb ? k : n)) return fail(NNB_ERR_INVALID, "sgemm: ldb %zu too small", ldb);
	if (mode == NNB_MATH_FP32X3)
		return launch<1>(s, dev, ta, tb, m, n, k, a, lda, sa, b, ldb, sb, c, ldc, sc, batch, acc);
	return launch<0>(s, dev, ta, tb, m, n, k, a, lda, sa, b, ldb, sb, c, ldc, sc, batch, acc);
}

}  // namespace gemm
}  // namespace nnb

extern "C" {

nnb_status nnb_sgemm(void* stream, int trans_a, int trans_b, size_t m, size_t n, size_t k,
		const float* a, size_t lda, const float* b, size_t ldb, float* c, size_t ldc, int accumulate) {
	return nnb::gemm::sgemm_entry(stream, trans_a != 0, trans_b != 0, m, n, k, a, lda, 0, b, ldb, 0, c,
		ldc, 0, 1, accumulate != 0, nnb::math_mode());
}

nnb_status nnb_sgemm_ex(void* stream, int trans_a, int trans_b, size_t m, size_t n, size_t k,
		const float* a, size_t lda, const float* b, size_t ldb, float* c, size_t ldc, int accumulate,
		int math_mode) {
	return nnb::gemm::sgemm_entry(stream, trans_a != 0, trans_b != 0, m, n, k, a, lda, 0, b, ldb, 0, c,
		ldc, 0, 1, accumulate != 0, math_mode);
}

nnb_status nnb_sgemm_strided_batched(void* stream, int trans_a, int trans_b, size_t m, size_t n,
		size_t k, const float* a, size_t lda, size_t stride_a, const float* b, size_t ldb,
		size_t stride_b, float* c, size_t ldc, size_t stride_c, size_t batch, int accumulate,
		int math_mode) {
	if (batch > 1 && stride_c == 0)
		return nnb::fail(NNB_ERR_INVALID, "sgemm_strided_batched: stride_c must be nonzero for batch > 1");
	return nnb::gemm::sgemm_entry(stream, trans_a != 0, trans_b != 0, m, n, k, a, lda, stride_a, b, ldb,
		stride_b, c, ldc, stride_c, batch, accumulate != 0, math_mode);
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
//   anything is enqueued.
// =============================================================================================

#include <mutex>

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
static nnb_status noalloc_setup(NoAllocDevice** out) {
	int dev = 0;
	NNB_CUDA_TRY(cudaGetDevice(&dev));
	if (dev < 0 || dev >= 64) return fail(NNB_ERR_UNSUPPORTED, "sgemm_noalloc: device index %d out of range", dev);
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
		NNB_CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
			Cfg<1>::kSmemBytes));
		NNB_CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
			Cfg<0>::kSmemBytes));
		d.scratch = static_cast<unsigned char*>(scratch);
		d.error = static_cast<int*>(error);
		d.sm_count = sms;
		d.ready = true;
	}
	*out = &d;
	return NNB_OK;
}

template <int kSplit>
static nnb_status launch_noalloc(cudaStream_t s, const NoAllocDevice* dev, int ta, int tb, long long m,
		long long n, long long k, const float* a, long long lda, const float* b, long long ldb, float* c,
		long long ldc, int acc) {
	constexpr int S = Cfg<kSplit>::S;
	const long long Mp = round_up(m, kBM), Np = round_up(n, kBN), Kp = round_up(k, kBK);
	const long long KB = Kp / kBK;
	const long long rows_a = Mp * KB * S, rows_b = Np * KB * S;
	const size_t bytes_a = (size_t)rows_a * kBK * 4, bytes_b = (size_t)rows_b * kBK * 4;
	const size_t flag_ints = (size_t)(Mp + Np + 1);
	const size_t off_b = round_up(bytes_a, 1024), off_f = off_b + round_up(bytes_b, 1024);
	const size_t total = off_f + flag_ints * sizeof(int);
	if (total > kNoAllocScratchBytes)
		return fail(NNB_ERR_UNSUPPORTED,
			"sgemm_noalloc: %lld x %lld x %lld needs %zu bytes of scratch; the static buffer holds %zu "
			"(packed operands take (roundup(m,128) + roundup(n,256)) * roundup(k,16) * %d * 4 bytes)",
			m, n, k, total, kNoAllocScratchBytes, S);
	float* pa = reinterpret_cast<float*>(dev->scratch);
	float* pb = reinterpret_cast<float*>(dev->scratch + off_b);
	int* flags_a = reinterpret_cast<int*>(dev->scratch + off_f);
	int* flags_b = flags_a + Mp;
	int* any = flags_b + Np;

	NNB_CUDA_TRY(cudaMemsetAsync(flags_a, 0, flag_ints * sizeof(int), s));
	dim3 ga((unsigned)(Mp / 32), (unsigned)((Kp + 63) / 64), 1);
	pack_kernel<kSplit><<<ga, 256, 0, s>>>(a, lda, 0, ta, (int)m, (int)k, (int)Mp, (int)KB, pa, flags_a, any);
	dim3 gb((unsigned)(Np / 32), (unsigned)((Kp + 63) / 64), 1);
	pack_kernel<kSplit><<<gb, 256, 0, s>>>(b, ldb, 0, !tb, (int)n, (int)k, (int)Np, (int)KB, pb, flags_b, any);
	NNB_CUDA_TRY(cudaGetLastError());

	CUtensorMap tma, tmb;
	NNB_TRY(encode_tiled_2d(&tma, pa, kBK, (uint64_t)rows_a, kBK * 4, kBK, kPanelRows, CU_TENSOR_MAP_SWIZZLE_64B));
	NNB_TRY(encode_tiled_2d(&tmb, pb, kBK, (uint64_t)rows_b, kBK * 4, kBK, kPanelRows, CU_TENSOR_MAP_SWIZZLE_64B));

	Params p;
	p.M = (int)m; p.N = (int)n; p.K = (int)k; p.KB = (int)KB;
	p.tiles_m = (int)(Mp / kBM); p.tiles_n = (int)(Np / kBN); p.batch = 1;
	p.a_batched = 0; p.b_batched = 0;
	p.Mp = (int)Mp; p.Np = (int)Np;
	p.C = c; p.ldc = ldc; p.stride_c = 0; p.accumulate = acc;
	p.any_nonfinite = any; p.flags_a = flags_a; p.flags_b = flags_b;
	p.A = a; p.lda = lda; p.stride_a = 0; p.B = b; p.ldb = ldb; p.stride_b = 0;
	p.ta = ta; p.tb = tb; p.err = dev->error;
	const long long tiles = (Mp / kBM) * (Np / kBN);
	const int grid = (int)std::min<long long>(tiles, dev->sm_count);
	gemm_tc_kernel<kSplit><<<grid, kThreads, Cfg<kSplit>::kSmemBytes, s>>>(tma, tmb, p);
	return cuda_status(cudaGetLastError(), "sgemm_noalloc: gemm launch");
}

}  // namespace gemm
}  // namespace nnb

extern "C" nnb_status nnb_sgemm_noalloc(void* stream, int trans_a, int trans_b, size_t m, size_t n,
		size_t k, const float* a, size_t lda, const float* b, size_t ldb, float* c, size_t ldc,
		int accumulate, int math_mode) {
	using namespace nnb;
	using namespace nnb::gemm;
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	const int ta = trans_a != 0, tb = trans_b != 0, acc = accumulate != 0;
	if (math_mode != NNB_MATH_FP32X3 && math_mode != NNB_MATH_TF32)
		return fail(NNB_ERR_INVALID, "sgemm_noalloc: unknown math mode %d", math_mode);
	if (m == 0 || n == 0) return NNB_OK;
	if (!c) return fail(NNB_ERR_INVALID, "sgemm_noalloc: C is null");
	if (ldc < n) return fail(NNB_ERR_INVALID, "sgemm_noalloc: ldc %zu < n %zu", ldc, n);
	const size_t lim = (size_t)1 << 30;
	if (m > lim || n > lim || k > lim) return fail(NNB_ERR_UNSUPPORTED, "sgemm_noalloc: dimension above 2^30");
	NoAllocDevice* dev = nullptr;
	NNB_TRY(noalloc_setup(&dev));
	if (k == 0) {
		if (acc) return NNB_OK;
		dim3 g((unsigned)std::min<size_t>((m * n + 255) / 256, 4096), 1, 1);
		zero_fill_kernel<<<g, 256, 0, s>>>(c, (long long)ldc, 0, (int)m, (int)n);
		return cuda_status(cudaGetLastError(), "sgemm_noalloc: zero fill launch");
	}
	if (!a || !b) return fail(NNB_ERR_INVALID, "sgemm_noalloc: A or B is null");
	if (lda < (ta ? m : k)) return fail(NNB_ERR_INVALID, "sgemm_noalloc: lda %zu too small", lda);
	if (ldb < (tb ? k : n)) return fail(NNB_ERR_INVALID, "sgemm_noalloc: ldb %zu too small", ldb);
	if (math_mode == NNB_MATH_FP32X3)
		return launch_noalloc<1>(s, dev, ta, tb, m, n, k, a, lda, b, ldb, c, ldc, acc);
	return launch_noalloc<0>(s, dev, ta, tb, m, n, k, a, lda, b, ldb, c, ldc, acc);
}
