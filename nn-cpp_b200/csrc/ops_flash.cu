// ops_flash.cu -- fused multi-head attention for head size 64: the `attention` op of
// src/autograd/ops.cpp:1226-1296 (scores Q_h K_h^T, the masked softmax of ops.cpp:1183-1224 with
// scale 1/sqrt(Dh), then P V_h) and its backward (ops.cpp:1280-1293), without materialising the
// {N, H, Tq, Tk} probability matrix.
//
// The reference runs two sgemm calls per (sample, head) and keeps P for the backward pass. Here one
// CTA owns 128 query rows of one (sample, head) and streams the keys through the tensor cores:
//   forward   S = Q K^T (TS MMA: Q hi/lo resident in tensor memory), online softmax in registers
//             (one thread per query row), P split into TF32 hi/lo and stored to tensor memory, then
//             O += P V (TS MMA, V read as an MN-major B operand). Only O and the row statistics
//             (max m and sum l of exp(score - m)) are written.
//   backward  two kernels, each output written by exactly one CTA (no atomics, fixed order):
//             dQ kernel  (128 query rows): S, dP = dO V^T recomputed, dS = P (dP - D) scale,
//                        dQ += dS K; it also writes D = rowsum(dO o O) and padded copies of m, l.
//             dKdV kernel (128 keys): S^T = K Q^T, dP^T = V dO^T, P^T and dS^T in tensor memory,
//                        dV += P^T dO and dK += dS^T Q accumulated in tensor memory.
// Every product is 3xTF32 (lo*hi + hi*lo + hi*hi) in the fp32x3 math mode, one TF32 MMA in the
// tf32 mode, as the GEMM does.
//
// Operand images. The tensor cores read a 32-bit operand either K-major with the 64-byte swizzle
// (rows of 16 depth elements; a Q K^T style product reads Q, K, V, dO this way) or MN-major with the
// 128-byte / 32-byte-atom swizzle (rows of 32 output columns for one depth index; P V, dS K, P^T dO
// and dS^T Q read V, K, dO, Q this way). Each operand is packed once per call, in the form(s) its
// consumers need, per (sample, head):
//   K-major  [hi/lo][4 panels of 16 head columns][Tp rows][16 floats], 16-byte unit u of row r
//            stored at u ^ ((r >> 1) & 3);
//   MN-major [hi/lo][2 blocks of 32 head columns][Tp rows][32 floats], 32-byte chunk c of row r
//            stored at c ^ (r & 3).
// These are the images TMA's 64-byte and 128-byte-with-32-byte-atom swizzles would write, so a plain
// bulk copy of any 8-row-aligned row range of a panel or block is a valid operand tile.
//
// Masking follows the reference: scaled scores of key-padded keys become -1e9 (they still take part
// in the softmax), causally hidden keys (key > query) get probability exactly 0; in the backward,
// both kinds get a zero score gradient.
#include <algorithm>
#include <cmath>
#include <mutex>

#include "nnb_internal.h"
#include "nnb_ops.h"
#include "nnb_ptx.cuh"
#include "nnb_trace.h"

namespace nnb {

namespace {

constexpr int kDh = 64;                       // head size these kernels handle
constexpr int kPanels = kDh / 16;             // K-major image: 16-float (64-byte) panels
constexpr int kBlocks = kDh / 32;             // MN-major image: 32-float (128-byte) blocks
constexpr int kRowAlign = 128;                // packed rows per (sample, head) are padded to this
constexpr uint32_t kTmemCols = 512;
// warp 0 loads, warp 1 issues MMAs, warps 2-9 do the per-element math: two warps per tensor-memory
// lane quarter (warp w reaches lanes 32 (w % 4) .. +31), each taking half of a row's columns
constexpr int kMathWarps = 8;
constexpr int kMathThreads = 32 * kMathWarps;
constexpr int kThreadsFa = 64 + kMathThreads;
constexpr float kLog2e = 1.4426950408889634f;   // exp(x) = 2^(x log2 e)

// Floats of one (sample, head) image of Tp rows, either form: hi and lo, 64 floats per row each.
__host__ __device__ inline long long packed_head_floats(long long Tp) { return 2LL * kDh * Tp; }

// Float offset, inside one head's image, of the 16-byte unit u (head columns 4u .. 4u+3) of row r.
__device__ __forceinline__ long long kmajor_offset(int hl, int u, long long r, long long Tp) {
	return ((long long)(hl * kPanels + (u >> 2)) * Tp + r) * 16 + (((u & 3) ^ (int)((r >> 1) & 3)) << 2);
}
__device__ __forceinline__ long long mnmajor_offset(int hl, int u, long long r, long long Tp) {
	const int e = (u & 7) * 4;                 // column inside the 32-float block
	return ((long long)(hl * kBlocks + (u >> 3)) * Tp + r) * 32 + ((((e >> 3) ^ (int)(r & 3)) << 3) | (e & 7));
}

// Every thread of the warp waits; the result is made warp-uniform so that the .sync.aligned
// tensor-memory instructions that follow run with the whole warp or not at all.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, int* err, volatile int* abort) {
	const bool ok = mbar_wait(bar, parity, err, kDevTimeoutAttn, abort);
	return __all_sync(0xffffffffu, ok);
}

// Waits (bounded, ignoring the abort flag) for a barrier phase before the CTA exits: used so that
// no bulk copy or MMA of this CTA is still in flight when its shared / tensor memory is released.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity, int* err) {
	mbar_wait(bar, parity, err, kDevTimeoutDrain, nullptr);
}

__device__ __forceinline__ void split4(float4 x, float4& hi, float4& lo) {
	split_tf32(x.x, hi.x, lo.x);
	split_tf32(x.y, hi.y, lo.y);
	split_tf32(x.z, hi.z, lo.z);
	split_tf32(x.w, hi.w, lo.w);
}

// Loads 32 consecutive floats of a head row (zeros when !valid), splits them and stores hi to the
// 32 columns at taddr_hi and lo to those at taddr_lo of this thread's tensor-memory lane.
__device__ __forceinline__ void half_row_to_tmem(const float* src, bool valid, uint32_t taddr_hi, uint32_t taddr_lo) {
	uint32_t hi[32], lo[32];
#pragma unroll
	for (int u = 0; u < 8; ++u) {
		float4 x = valid ? __ldg(reinterpret_cast<const float4*>(src) + u) : make_float4(0.f, 0.f, 0.f, 0.f);
		float4 h, l;
		split4(x, h, l);
		hi[4 * u] = __float_as_uint(h.x); hi[4 * u + 1] = __float_as_uint(h.y);
		hi[4 * u + 2] = __float_as_uint(h.z); hi[4 * u + 3] = __float_as_uint(h.w);
		lo[4 * u] = __float_as_uint(l.x); lo[4 * u + 1] = __float_as_uint(l.y);
		lo[4 * u + 2] = __float_as_uint(l.z); lo[4 * u + 3] = __float_as_uint(l.w);
	}
	tmem_st_32x32b_x32(taddr_hi, hi);
	tmem_st_32x32b_x32(taddr_lo, lo);
}

// The two math threads that share a row (one per half) swap a value through shared memory:
// each writes its own, arrives on the pair's mbarrier (count 64) and waits, bounded, for the phase.
// Returns false (warp-uniform) when the wait ran out.
__device__ __forceinline__ bool pair_swap(float* slot_mine, const float* slot_other, float v, float& other,
		uint32_t bar, uint32_t parity, int* err, volatile int* abort) {
	*slot_mine = v;
	mbar_arrive(bar);
	if (!warp_wait(bar, parity, err, abort)) return false;
	other = *slot_other;
	return true;
}

// Splits 16 values and stores hi / lo to two 16-column groups of this thread's lane.
__device__ __forceinline__ void vals_to_tmem16(const float (&v)[16], uint32_t taddr_hi, uint32_t taddr_lo) {
	uint32_t hi[16], lo[16];
#pragma unroll
	for (int c = 0; c < 16; ++c) {
		const float h = to_tf32(v[c]);
		hi[c] = __float_as_uint(h);
		lo[c] = __float_as_uint(to_tf32(v[c] - h));
	}
	tmem_st_32x32b_x16(taddr_hi, hi);
	tmem_st_32x32b_x16(taddr_lo, lo);
}

// Splits 32 values and stores hi / lo to two 32-column groups of this thread's lane.
__device__ __forceinline__ void vals_to_tmem(const float (&v)[32], uint32_t taddr_hi, uint32_t taddr_lo) {
	uint32_t hi[32], lo[32];
#pragma unroll
	for (int c = 0; c < 32; ++c) {        // finite values well inside the fp32 range
		const float h = to_tf32(v[c]);
		hi[c] = __float_as_uint(h);
		lo[c] = __float_as_uint(to_tf32(v[c] - h));
	}
	tmem_st_32x32b_x32(taddr_hi, hi);
	tmem_st_32x32b_x32(taddr_lo, lo);
}

// Issues one MMA step (depth 8) of D (+)= A B in the given split: A from tensor memory (hi, lo
// columns), B from the shared-memory descriptors (hi, lo).
__device__ __forceinline__ void mma_step(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint64_t b_hi, uint64_t b_lo,
		uint32_t idesc, uint32_t acc, int split) {
	if (split) {
		mma_tf32_ts(d, a_lo, b_hi, idesc, acc);
		mma_tf32_ts(d, a_hi, b_lo, idesc, 1u);
		mma_tf32_ts(d, a_hi, b_hi, idesc, 1u);
	} else {
		mma_tf32_ts(d, a_hi, b_hi, idesc, acc);
	}
}

// ---------------------------------------------------------------------------------------------
// Pack: x [N, T, D] (head h in columns h*64 .. h*64+63) -> the K-major and / or MN-major image of
// every (sample, head), as described above (a null destination skips that form).
// ---------------------------------------------------------------------------------------------
struct PackSet {
	const float* src[4];
	float* kdst[4];
	float* mdst[4];
	int T[4];
	int Tp[4];
};

__global__ void __launch_bounds__(256) attn_pack_kernel(const PackSet ps, long long NH, int H, long long D, int with_lo) {
	const int t = blockIdx.y;
	const float* __restrict__ x = ps.src[t];
	float* __restrict__ kd = ps.kdst[t];
	float* __restrict__ md = ps.mdst[t];
	const int T = ps.T[t], Tp = ps.Tp[t];
	const long long per_head = (long long)Tp * 16;     // 16 float4 units per row
	const long long total = NH * per_head;
	for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
		const long long nh = i / per_head;
		const int rem = (int)(i - nh * per_head);
		const int row = rem >> 4, u = rem & 15;
		const long long n = nh / H;
		const int h = (int)(nh - n * H);
		float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
		if (row < T) v = __ldg(reinterpret_cast<const float4*>(x + ((long long)n * T + row) * D + h * kDh) + u);
		float4 hi, lo;
		split4(v, hi, lo);
		const long long base = nh * packed_head_floats(Tp);
		if (kd) {
			*reinterpret_cast<float4*>(kd + base + kmajor_offset(0, u, row, Tp)) = hi;
			if (with_lo) *reinterpret_cast<float4*>(kd + base + kmajor_offset(1, u, row, Tp)) = lo;
		}
		if (md) {
			*reinterpret_cast<float4*>(md + base + mnmajor_offset(0, u, row, Tp)) = hi;
			if (with_lo) *reinterpret_cast<float4*>(md + base + mnmajor_offset(1, u, row, Tp)) = lo;
		}
	}
}

// Bulk copies of rows [r0, r0 + R) of one head's image (hi or lo part) into shared memory, laid out
// as the operand tile: K-major -> 4 panels of R x 64 bytes, MN-major -> 2 blocks of R x 128 bytes.
__device__ __forceinline__ void copy_kmajor(uint32_t dst, const float* img, int hl, long long Tp, long long r0, int R,
		uint32_t bar) {
#pragma unroll
	for (int pp = 0; pp < kPanels; ++pp)
		bulk_load(dst + pp * (R * 64), img + ((long long)(hl * kPanels + pp) * Tp + r0) * 16, R * 64, bar);
}
__device__ __forceinline__ void copy_mnmajor(uint32_t dst, const float* img, int hl, long long Tp, long long r0, int R,
		uint32_t bar) {
#pragma unroll
	for (int b = 0; b < kBlocks; ++b)
		bulk_load(dst + b * (R * 128), img + ((long long)(hl * kBlocks + b) * Tp + r0) * 32, R * 128, bar);
}

// ---------------------------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------------------------
struct FwdParams {
	const float* pk;     // K, K-major image, Tpk rows per head
	const float* pv;     // V, MN-major image
	const float* q;      // [N, Tq, D]
	const float* pad;    // [N, Tk] key-padding mask (0 = padded) or null
	float* out;          // [N, Tq, D]
	float* stats;        // [N, H, Tq, 2]: row max m, row sum l of exp(score - m)
	int* err;
	long long D;
	int N, H, Tq, Tk, Tpk, q_tiles, causal, split;
	float scale;
};

constexpr int kFwdRows = 128;                               // query rows per CTA (MMA M)
constexpr int kFwdKeys = 64;                                // keys per tile (S columns, PV depth)
constexpr int kFwdStages = 3;
constexpr uint32_t kFwdOpBytes = kPanels * kFwdKeys * 64;   // 16 KB: one of K hi, K lo, V hi, V lo
constexpr uint32_t kFwdStageBytes = 4 * kFwdOpBytes;
constexpr uint32_t kFwdSmem = kFwdStages * kFwdStageBytes + 1024;
// tensor-memory columns: Q hi | Q lo | S/P-hi 0 | P-lo 0 | S/P-hi 1 | P-lo 1 | PV 0 | PV 1
constexpr uint32_t kFColQhi = 0, kFColQlo = 64, kFColS = 128, kFColPV = 384;

__global__ void __launch_bounds__(kThreadsFa, 1) flash_fwd_kernel(const FwdParams p) {
	extern __shared__ uint8_t smem_raw[];
	uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
	__shared__ __align__(8) uint64_t kv_full[kFwdStages], kv_empty[kFwdStages], s_full[2], p_full[2], pv_full[2],
		pv_empty[2], q_ready, drain, xbar[4][2];
	__shared__ float xval[2][2][kFwdRows];          // [tile parity][half][row]: partial row max / sum
	__shared__ uint32_t tmem_base_sh;
	__shared__ int abort_sh;

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int NH = p.N * p.H;
	const int qt = p.q_tiles - 1 - (int)(blockIdx.x / NH);     // longest causal rows first
	const int nh = (int)(blockIdx.x % NH);
	const int n = nh / p.H, h = nh % p.H;
	const int q0 = qt * kFwdRows;
	const int key_end = p.causal ? min(q0 + kFwdRows, p.Tq) : p.Tk;
	const int J = (key_end + kFwdKeys - 1) / kFwdKeys;

	if (threadIdx.x == 0) {
		for (int s = 0; s < kFwdStages; ++s) {
			mbar_init(smem_u32(&kv_full[s]), 1);
			mbar_init(smem_u32(&kv_empty[s]), 1);
		}
		for (int b = 0; b < 2; ++b) {
			mbar_init(smem_u32(&s_full[b]), 1);
			mbar_init(smem_u32(&p_full[b]), kMathThreads);
			mbar_init(smem_u32(&pv_full[b]), 1);
			mbar_init(smem_u32(&pv_empty[b]), kMathThreads);
		}
		for (int qd = 0; qd < 4; ++qd) {
			mbar_init(smem_u32(&xbar[qd][0]), 64);
			mbar_init(smem_u32(&xbar[qd][1]), 64);
		}
		mbar_init(smem_u32(&q_ready), kMathThreads);
		mbar_init(smem_u32(&drain), 1);
		abort_sh = 0;
		fence_mbar_init();
	}
	if (warp == 1) {
		tmem_alloc(smem_u32(&tmem_base_sh), kTmemCols);
		tmem_relinquish();
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = tmem_base_sh;
	volatile int* abort_flag = &abort_sh;

	if (warp == 0) {
		if (lane == 0) {
			// ---------------------------- bulk-copy producer ----------------------------
			const float* kb = p.pk + (long long)nh * packed_head_floats(p.Tpk);
			const float* vb = p.pv + (long long)nh * packed_head_floats(p.Tpk);
			const int parts = p.split ? 2 : 1;
			int issued = 0;
			for (int j = 0; j < J; ++j) {
				const int s = j % kFwdStages;
				if (j >= kFwdStages &&
						!mbar_wait(smem_u32(&kv_empty[s]), ((j / kFwdStages) & 1) ^ 1, p.err, kDevTimeoutAttn, abort_flag))
					break;
				const uint32_t fb = smem_u32(&kv_full[s]);
				mbar_arrive_expect_tx(fb, parts * 2 * kFwdOpBytes);
				const uint32_t dst = smem_u32(smem + s * kFwdStageBytes);
				for (int hl = 0; hl < parts; ++hl) {
					copy_kmajor(dst + hl * kFwdOpBytes, kb, hl, p.Tpk, (long long)j * kFwdKeys, kFwdKeys, fb);
					copy_mnmajor(dst + 2 * kFwdOpBytes + hl * kFwdOpBytes, vb, hl, p.Tpk, (long long)j * kFwdKeys, kFwdKeys,
						fb);
				}
				issued = j + 1;
			}
			// every issued copy has landed before the CTA can exit
			for (int j = max(0, issued - kFwdStages); j < issued; ++j)
				drain_wait(smem_u32(&kv_full[j % kFwdStages]), (j / kFwdStages) & 1, p.err);
		}
	} else if (warp == 1) {
		if (lane == 0) {
			// -------------------------------- MMA issuer --------------------------------
			const uint32_t id_s = idesc_tf32(kFwdRows, kFwdKeys);
			const uint32_t id_pv = idesc_tf32(kFwdRows, kDh) | kIdescBMajorMN;
			bool ok = mbar_wait(smem_u32(&q_ready), 0, p.err, kDevTimeoutAttn, abort_flag);
			tc_fence_after();
			for (int j = 0; ok && j <= J; ++j) {
				if (j < J) {
					const int s = j % kFwdStages;
					if (!mbar_wait(smem_u32(&kv_full[s]), (j / kFwdStages) & 1, p.err, kDevTimeoutAttn, abort_flag)) break;
					tc_fence_after();
					const uint32_t kbase = smem_u32(smem + s * kFwdStageBytes);
					const uint32_t d = tmem + kFColS + (j & 1) * 128;
#pragma unroll
					for (int ks = 0; ks < kDh / 8; ++ks) {
						const uint32_t off = (ks >> 1) * (kFwdKeys * 64) + (ks & 1) * 32;
						mma_step(d, tmem + kFColQhi + ks * 8, tmem + kFColQlo + ks * 8, smem_desc_k_sw64(kbase + off),
							smem_desc_k_sw64(kbase + kFwdOpBytes + off), id_s, ks > 0, p.split);
					}
					mma_commit(smem_u32(&s_full[j & 1]));
				}
				if (j >= 1) {
					const int jj = j - 1, b = jj & 1, s = jj % kFwdStages;
					if (!mbar_wait(smem_u32(&p_full[b]), (jj >> 1) & 1, p.err, kDevTimeoutAttn, abort_flag)) break;
					if (jj >= 2 && !mbar_wait(smem_u32(&pv_empty[b]), ((jj >> 1) - 1) & 1, p.err, kDevTimeoutAttn, abort_flag))
						break;
					tc_fence_after();
					const uint32_t vbase = smem_u32(smem + s * kFwdStageBytes + 2 * kFwdOpBytes);
					const uint32_t d = tmem + kFColPV + b * 64, pc = tmem + kFColS + b * 128;
#pragma unroll
					for (int ks = 0; ks < kFwdKeys / 8; ++ks)
						mma_step(d, pc + ks * 8, pc + 64 + ks * 8, smem_desc_mn_sw128b32(vbase + ks * 1024, kFwdKeys * 128),
							smem_desc_mn_sw128b32(vbase + kFwdOpBytes + ks * 1024, kFwdKeys * 128), id_pv, ks > 0, p.split);
					mma_commit(smem_u32(&pv_full[b]));
					mma_commit(smem_u32(&kv_empty[s]));
				}
			}
			// every issued MMA has completed before tensor memory is released
			mma_commit(smem_u32(&drain));
			drain_wait(smem_u32(&drain), 0, p.err);
		}
	} else {
		// ------------- softmax: two threads per query row, 32 key columns each -------------
		const int quad = warp & 3, half = (warp - 2) >> 2;
		const int row = quad * 32 + lane, qrow = q0 + row;
		const bool row_ok = qrow < p.Tq;
		const uint32_t lb = tmem + ((uint32_t)(quad * 32) << 16);
		const long long roff = ((long long)n * p.Tq + (row_ok ? qrow : 0)) * p.D + h * kDh + half * 32;
		half_row_to_tmem(p.q + roff, row_ok, lb + kFColQhi + half * 32, lb + kFColQlo + half * 32);
		tmem_wait_st();
		tc_fence_before();
		mbar_arrive(smem_u32(&q_ready));

		const float* padn = p.pad ? p.pad + (long long)n * p.Tk : nullptr;
		const float c1 = p.scale * kLog2e;
		float m = -INFINITY, l = 0.0f, alpha_prev = 0.0f;
		float o[32];
#pragma unroll
		for (int c = 0; c < 32; ++c) o[c] = 0.0f;
		int xuse = 0;                                // exchanges so far (phase of the pair barriers)
		auto swap = [&](float v, float& other) -> bool {
			const int par = xuse & 1;
			const bool r = pair_swap(&xval[par][half][row], &xval[par][half ^ 1][row], v, other,
				smem_u32(&xbar[quad][par]), (xuse >> 1) & 1, p.err, abort_flag);
			++xuse;
			return r;
		};
		// O = alpha O + PV_jj (this thread's 32 head columns) for the finished tile jj
		auto fold = [&](int jj) -> bool {
			const int b = jj & 1;
			if (!warp_wait(smem_u32(&pv_full[b]), (jj >> 1) & 1, p.err, abort_flag)) return false;
			tc_fence_after();
			uint32_t r[32];
			tmem_ld_32x32b_x32(lb + kFColPV + b * 64 + half * 32, r);
			tmem_wait_ld();
#pragma unroll
			for (int c = 0; c < 32; ++c) o[c] = o[c] * alpha_prev + __uint_as_float(r[c]);
			tc_fence_before();
			mbar_arrive(smem_u32(&pv_empty[b]));
			return true;
		};
		bool ok = true;
		for (int j = 0; j < J; ++j) {
			const int b = j & 1;
			if (!warp_wait(smem_u32(&s_full[b]), (j >> 1) & 1, p.err, abort_flag)) {
				ok = false;
				break;
			}
			tc_fence_after();
			float sv[32];
			{
				uint32_t r[32];
				tmem_ld_32x32b_x32(lb + kFColS + b * 128 + half * 32, r);
				tmem_wait_ld();
#pragma unroll
				for (int c = 0; c < 32; ++c) sv[c] = __uint_as_float(r[c]);
			}
			// tiles on the causal diagonal, past the last key, or under a padding mask take the
			// masked path (the same for every thread of the CTA)
			const int key0 = j * kFwdKeys + half * 32;
			const bool general = padn || (p.causal && j * kFwdKeys + kFwdKeys - 1 > q0) || (j * kFwdKeys + kFwdKeys > p.Tk);
			float mt = -INFINITY;
			if (!general) {
#pragma unroll
				for (int c = 0; c < 32; ++c) mt = fmaxf(mt, sv[c]);
				mt = mt * p.scale;                   // scale > 0: max of the scaled scores
			} else {
#pragma unroll
				for (int c = 0; c < 32; ++c) {
					const int key = key0 + c;
					const bool live = key < p.Tk && (!p.causal || key <= qrow);
					const bool padded = padn && live && padn[key] == 0.0f;
					mt = fmaxf(mt, !live ? -INFINITY : padded ? -1e9f : sv[c] * p.scale);
				}
			}
			float mo;
			if (!swap(mt, mo)) {
				ok = false;
				break;
			}
			const float m_new = fmaxf(m, fmaxf(mt, mo));
			const float alpha = exp2_hw((m - m_new) * kLog2e);     // 0 on the first tile (m = -inf)
			const float mlog = m_new * kLog2e;
			float sum = 0.0f;
			if (!general) {
#pragma unroll
				for (int c = 0; c < 32; ++c) {
					const float e = exp2_hw(__fmaf_rn(sv[c], c1, -mlog));
					sv[c] = e;
					sum += e;
				}
			} else {
#pragma unroll
				for (int c = 0; c < 32; ++c) {
					const int key = key0 + c;
					const bool live = key < p.Tk && (!p.causal || key <= qrow);
					const bool padded = padn && live && padn[key] == 0.0f;
					// a padded key's exponent is formed from -1e9 - m, exact when the whole row is padded
					const float e = !live ? 0.0f : exp2_hw(padded ? (-1e9f - m_new) * kLog2e : __fmaf_rn(sv[c], c1, -mlog));
					sv[c] = e;
					sum += e;
				}
			}
			l = l * alpha + sum;
			m = m_new;
			vals_to_tmem(sv, lb + kFColS + b * 128 + half * 32, lb + kFColS + b * 128 + 64 + half * 32);
			tmem_wait_st();
			tc_fence_before();
			mbar_arrive(smem_u32(&p_full[b]));
			if (j >= 1 && !fold(j - 1)) {
				ok = false;
				break;
			}
			alpha_prev = alpha;
		}
		if (ok && J >= 1) ok = fold(J - 1);
		float lo_other = 0.0f;
		if (ok) ok = swap(l, lo_other);
		if (ok && row_ok) {
			const float lt = l + lo_other;
			const float inv_l = 1.0f / lt;
			float4* orow = reinterpret_cast<float4*>(p.out + roff);
#pragma unroll
			for (int u = 0; u < 8; ++u)
				orow[u] = make_float4(o[4 * u] * inv_l, o[4 * u + 1] * inv_l, o[4 * u + 2] * inv_l, o[4 * u + 3] * inv_l);
			if (half == 0) {
				// m and l are kept apart: with the reference's -1e9 padding scores, m + log(l) would lose
				// log(l) to rounding for a row whose keys are all padded
				p.stats[((long long)nh * p.Tq + qrow) * 2] = m;
				p.stats[((long long)nh * p.Tq + qrow) * 2 + 1] = lt;
			}
		}
	}

	tc_fence_before();
	__syncthreads();
	if (warp == 1) {
		__syncwarp();
		tc_fence_after();
		tmem_dealloc(tmem, kTmemCols);
	}
}

// ---------------------------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------------------------
struct BwdParams {
	const float* pq;     // Q, K-major image, Tpq rows per head
	const float* pq_mn;  // Q, MN-major image
	const float* pdo;    // dO (upstream gradient), K-major image, Tpq rows
	const float* pdo_mn; // dO, MN-major image
	const float* pk;     // K, K-major image, Tpk rows
	const float* pk_mn;  // K, MN-major image
	const float* pv;     // V, K-major image
	const float* q;      // raw [N, Tq, D]
	const float* k;      // raw [N, Tk, D]
	const float* v;
	const float* dout;   // [N, Tq, D]
	const float* out;    // forward output [N, Tq, D]
	const float* stats;  // [N, H, Tq, 2] from the forward
	const float* pad;    // [N, Tk] or null
	float* rowstat;      // [N*H][3][Tpq]: m, l (padded copies) and D = rowsum(dO o O)
	float* dq;
	float* dk;
	float* dv;
	int dq_first, dk_first, dv_first;
	int* err;
	long long D;
	int N, H, Tq, Tk, Tpq, Tpk, q_tiles, k_tiles, causal, split;
	float scale;
};

// Stores (first) or adds 64 values to a head row.
__device__ __forceinline__ void store_row(float* dst, const float (&v)[kDh], int first) {
	float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
	for (int u = 0; u < kDh / 4; ++u) {
		float4 o = make_float4(v[4 * u] + 0.0f, v[4 * u + 1] + 0.0f, v[4 * u + 2] + 0.0f, v[4 * u + 3] + 0.0f);
		if (!first) {
			const float4 c = d4[u];
			o.x = c.x + o.x; o.y = c.y + o.y; o.z = c.z + o.z; o.w = c.w + o.w;
		}
		d4[u] = o;
	}
}

// -------- dQ kernel: 128 query rows per CTA, 64-key tiles streamed --------
// stage: K (K-major hi, lo) | V (K-major hi, lo) | K (MN-major hi, lo), 16 KB each
constexpr int kDqStages = 2;
constexpr uint32_t kDqStageBytes = 6 * kFwdOpBytes;
constexpr uint32_t kDqSmem = kDqStages * kDqStageBytes + 1024;
// tensor-memory columns: Q hi | Q lo | dO hi | dO lo | S/dS-hi | dS-lo | dP | dQ
constexpr uint32_t kQColQhi = 0, kQColQlo = 64, kQColOhi = 128, kQColOlo = 192, kQColS = 256, kQColSlo = 320,
	kQColP = 384, kQColAcc = 448;

__global__ void __launch_bounds__(kThreadsFa, 1) flash_bwd_dq_kernel(const BwdParams p) {
	extern __shared__ uint8_t smem_raw[];
	uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
	__shared__ __align__(8) uint64_t kv_full[kDqStages], kv_empty[kDqStages], sdp_full, ds_full, acc_full, q_ready,
		drain, xbar[4];
	__shared__ float xval[2][kFwdRows];
	__shared__ uint32_t tmem_base_sh;
	__shared__ int abort_sh;

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int NH = p.N * p.H;
	const int qt = p.q_tiles - 1 - (int)(blockIdx.x / NH);
	const int nh = (int)(blockIdx.x % NH);
	const int n = nh / p.H, h = nh % p.H;
	const int q0 = qt * kFwdRows;
	const int key_end = p.causal ? min(q0 + kFwdRows, p.Tq) : p.Tk;
	const int J = (key_end + kFwdKeys - 1) / kFwdKeys;

	if (threadIdx.x == 0) {
		for (int s = 0; s < kDqStages; ++s) {
			mbar_init(smem_u32(&kv_full[s]), 1);
			mbar_init(smem_u32(&kv_empty[s]), 1);
		}
		mbar_init(smem_u32(&sdp_full), 1);
		mbar_init(smem_u32(&ds_full), kMathThreads);
		mbar_init(smem_u32(&acc_full), 1);
		mbar_init(smem_u32(&q_ready), kMathThreads);
		for (int qd = 0; qd < 4; ++qd) mbar_init(smem_u32(&xbar[qd]), 64);
		mbar_init(smem_u32(&drain), 1);
		abort_sh = 0;
		fence_mbar_init();
	}
	if (warp == 1) {
		tmem_alloc(smem_u32(&tmem_base_sh), kTmemCols);
		tmem_relinquish();
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = tmem_base_sh;
	volatile int* abort_flag = &abort_sh;

	if (warp == 0) {
		if (lane == 0) {
			const long long img = (long long)nh * packed_head_floats(p.Tpk);
			const float* kb = p.pk + img;
			const float* vb = p.pv + img;
			const float* km = p.pk_mn + img;
			const int parts = p.split ? 2 : 1;
			int issued = 0;
			for (int j = 0; j < J; ++j) {
				const int s = j % kDqStages;
				if (j >= kDqStages &&
						!mbar_wait(smem_u32(&kv_empty[s]), ((j / kDqStages) & 1) ^ 1, p.err, kDevTimeoutAttn, abort_flag))
					break;
				const uint32_t fb = smem_u32(&kv_full[s]);
				mbar_arrive_expect_tx(fb, parts * 3 * kFwdOpBytes);
				const uint32_t dst = smem_u32(smem + s * kDqStageBytes);
				const long long r0 = (long long)j * kFwdKeys;
				for (int hl = 0; hl < parts; ++hl) {
					copy_kmajor(dst + hl * kFwdOpBytes, kb, hl, p.Tpk, r0, kFwdKeys, fb);
					copy_kmajor(dst + 2 * kFwdOpBytes + hl * kFwdOpBytes, vb, hl, p.Tpk, r0, kFwdKeys, fb);
					copy_mnmajor(dst + 4 * kFwdOpBytes + hl * kFwdOpBytes, km, hl, p.Tpk, r0, kFwdKeys, fb);
				}
				issued = j + 1;
			}
			for (int j = max(0, issued - kDqStages); j < issued; ++j)
				drain_wait(smem_u32(&kv_full[j % kDqStages]), (j / kDqStages) & 1, p.err);
		}
	} else if (warp == 1) {
		if (lane == 0) {
			const uint32_t id_s = idesc_tf32(kFwdRows, kFwdKeys);
			const uint32_t id_dq = idesc_tf32(kFwdRows, kDh) | kIdescBMajorMN;
			bool ok = mbar_wait(smem_u32(&q_ready), 0, p.err, kDevTimeoutAttn, abort_flag);
			tc_fence_after();
			for (int j = 0; ok && j < J; ++j) {
				const int s = j % kDqStages;
				if (!mbar_wait(smem_u32(&kv_full[s]), (j / kDqStages) & 1, p.err, kDevTimeoutAttn, abort_flag)) break;
				tc_fence_after();
				const uint32_t kbase = smem_u32(smem + s * kDqStageBytes);
				const uint32_t vbase = kbase + 2 * kFwdOpBytes, kmn = kbase + 4 * kFwdOpBytes;
#pragma unroll
				for (int ks = 0; ks < kDh / 8; ++ks) {      // S = Q K^T
					const uint32_t off = (ks >> 1) * (kFwdKeys * 64) + (ks & 1) * 32;
					mma_step(tmem + kQColS, tmem + kQColQhi + ks * 8, tmem + kQColQlo + ks * 8,
						smem_desc_k_sw64(kbase + off), smem_desc_k_sw64(kbase + kFwdOpBytes + off), id_s, ks > 0, p.split);
				}
#pragma unroll
				for (int ks = 0; ks < kDh / 8; ++ks) {      // dP = dO V^T
					const uint32_t off = (ks >> 1) * (kFwdKeys * 64) + (ks & 1) * 32;
					mma_step(tmem + kQColP, tmem + kQColOhi + ks * 8, tmem + kQColOlo + ks * 8,
						smem_desc_k_sw64(vbase + off), smem_desc_k_sw64(vbase + kFwdOpBytes + off), id_s, ks > 0, p.split);
				}
				mma_commit(smem_u32(&sdp_full));
				if (!mbar_wait(smem_u32(&ds_full), j & 1, p.err, kDevTimeoutAttn, abort_flag)) break;
				tc_fence_after();
#pragma unroll
				for (int ks = 0; ks < kFwdKeys / 8; ++ks)   // dQ += dS K
					mma_step(tmem + kQColAcc, tmem + kQColS + ks * 8, tmem + kQColSlo + ks * 8,
						smem_desc_mn_sw128b32(kmn + ks * 1024, kFwdKeys * 128),
						smem_desc_mn_sw128b32(kmn + kFwdOpBytes + ks * 1024, kFwdKeys * 128), id_dq, (j > 0 || ks > 0),
						p.split);
				mma_commit(smem_u32(&kv_empty[s]));
				if (j == J - 1) mma_commit(smem_u32(&acc_full));
			}
			mma_commit(smem_u32(&drain));
			drain_wait(smem_u32(&drain), 0, p.err);
		}
	} else {
		// ------------- score gradients: two threads per query row, 32 key columns each -------------
		const int quad = warp & 3, half = (warp - 2) >> 2;
		const int row = quad * 32 + lane, qrow = q0 + row;
		const bool row_ok = qrow < p.Tq;
		const uint32_t lb = tmem + ((uint32_t)(quad * 32) << 16);
		const long long roff = ((long long)n * p.Tq + (row_ok ? qrow : 0)) * p.D + h * kDh + half * 32;
		half_row_to_tmem(p.q + roff, row_ok, lb + kQColQhi + half * 32, lb + kQColQlo + half * 32);
		half_row_to_tmem(p.dout + roff, row_ok, lb + kQColOhi + half * 32, lb + kQColOlo + half * 32);
		// D = rowsum(dO o O): the reference's dot = sum_j dP_j P_j of the softmax backward, as
		// sum_j P_j (dO . v_j) = dO . O (this thread's 32 columns, then the pair's sum)
		float dpart = 0.0f, mrow = 0.0f, inv_l = 1.0f;
		if (row_ok) {
			const float4* g4 = reinterpret_cast<const float4*>(p.dout + roff);
			const float4* o4 = reinterpret_cast<const float4*>(p.out + roff);
#pragma unroll
			for (int u = 0; u < 8; ++u) {
				const float4 a = __ldg(g4 + u), b = __ldg(o4 + u);
				dpart += a.x * b.x;
				dpart += a.y * b.y;
				dpart += a.z * b.z;
				dpart += a.w * b.w;
			}
			mrow = p.stats[((long long)nh * p.Tq + qrow) * 2];
			inv_l = 1.0f / p.stats[((long long)nh * p.Tq + qrow) * 2 + 1];
		}
		float dother = 0.0f;
		bool ok = pair_swap(&xval[half][row], &xval[half ^ 1][row], dpart, dother, smem_u32(&xbar[quad]), 0, p.err,
			abort_flag);
		const float drow = half == 0 ? dpart + dother : dother + dpart;      // same order in both threads
		if (half == 0) {
			// rows past Tq get neutral statistics (m 0, 1/l 1, D 0): their Q and dO rows are zero
			float* rs_out = p.rowstat + (long long)nh * 3 * p.Tpq;
			rs_out[qrow] = mrow;
			rs_out[p.Tpq + qrow] = inv_l;
			rs_out[2 * p.Tpq + qrow] = drow;
		}
		tmem_wait_st();
		tc_fence_before();
		mbar_arrive(smem_u32(&q_ready));

		const float* padn = p.pad ? p.pad + (long long)n * p.Tk : nullptr;
		const float c1 = p.scale * kLog2e, mlog = mrow * kLog2e;
		for (int j = 0; ok && j < J; ++j) {
			if (!warp_wait(smem_u32(&sdp_full), j & 1, p.err, abort_flag)) {
				ok = false;
				break;
			}
			tc_fence_after();
			uint32_t rs[32], rp[32];
			tmem_ld_32x32b_x32(lb + kQColS + half * 32, rs);
			tmem_ld_32x32b_x32(lb + kQColP + half * 32, rp);
			tmem_wait_ld();
			const int key0 = j * kFwdKeys + half * 32;
			const bool general = padn || (p.causal && j * kFwdKeys + kFwdKeys - 1 > q0) || (j * kFwdKeys + kFwdKeys > p.Tk);
			float ds[32];
			if (!general) {
#pragma unroll
				for (int c = 0; c < 32; ++c) {
					const float pr = exp2_hw(__fmaf_rn(__uint_as_float(rs[c]), c1, -mlog)) * inv_l;
					ds[c] = p.scale * (pr * (__uint_as_float(rp[c]) - drow));
				}
			} else {
#pragma unroll
				for (int c = 0; c < 32; ++c) {
					const int key = key0 + c;
					const bool live = row_ok && key < p.Tk && (!p.causal || key <= qrow);
					const bool padded = padn && live && padn[key] == 0.0f;
					const float pr = exp2_hw(__fmaf_rn(__uint_as_float(rs[c]), c1, -mlog)) * inv_l;
					ds[c] = (live && !padded) ? p.scale * (pr * (__uint_as_float(rp[c]) - drow)) : 0.0f;
				}
			}
			vals_to_tmem(ds, lb + kQColS + half * 32, lb + kQColSlo + half * 32);
			tmem_wait_st();
			tc_fence_before();
			mbar_arrive(smem_u32(&ds_full));
		}
		if (ok && J > 0) ok = warp_wait(smem_u32(&acc_full), 0, p.err, abort_flag);
		if (ok && J > 0) {
			tc_fence_after();
			uint32_t r[32];
			tmem_ld_32x32b_x32(lb + kQColAcc + half * 32, r);
			tmem_wait_ld();
			if (row_ok && p.dq) {
				float4* d4 = reinterpret_cast<float4*>(p.dq + roff);
#pragma unroll
				for (int u = 0; u < 8; ++u) {
					float4 v = make_float4(__uint_as_float(r[4 * u]) + 0.0f, __uint_as_float(r[4 * u + 1]) + 0.0f,
						__uint_as_float(r[4 * u + 2]) + 0.0f, __uint_as_float(r[4 * u + 3]) + 0.0f);
					if (!p.dq_first) {
						const float4 c = d4[u];
						v.x = c.x + v.x; v.y = c.y + v.y; v.z = c.z + v.z; v.w = c.w + v.w;
					}
					d4[u] = v;
				}
			}
		}
	}

	tc_fence_before();
	__syncthreads();
	if (warp == 1) {
		__syncwarp();
		tc_fence_after();
		tmem_dealloc(tmem, kTmemCols);
	}
}

// -------- dKdV kernel: 128 keys per CTA, 32-query tiles streamed --------
constexpr int kKvRows = 128;                                   // keys per CTA (MMA M)
constexpr int kKvQ = 32;                                       // queries per tile
constexpr int kKvStages = 3;
// stage: Q K-major (hi, lo) | dO K-major (hi, lo) | Q MN-major (hi, lo) | dO MN-major (hi, lo), 8 KB
// each, then m[32], l[32], D[32] of the tile's queries
constexpr uint32_t kKvOpBytes = kPanels * kKvQ * 64;
constexpr uint32_t kKvStatOff = 8 * kKvOpBytes;
constexpr uint32_t kKvStageBytes = 8 * kKvOpBytes + 1024;      // keeps every stage 1024-byte aligned
constexpr uint32_t kKvSmem = kKvStages * kKvStageBytes + 1024;
// tensor-memory columns: K hi | K lo | V hi | V lo | S^T/P^T-hi | P^T-lo | dP^T/dS^T-hi | dS^T-lo | dV | dK
constexpr uint32_t kKColKhi = 0, kKColKlo = 64, kKColVhi = 128, kKColVlo = 192, kKColS = 256, kKColSlo = 288,
	kKColP = 320, kKColPlo = 352, kKColDv = 384, kKColDk = 448;

__global__ void __launch_bounds__(kThreadsFa, 1) flash_bwd_dkdv_kernel(const BwdParams p) {
	extern __shared__ uint8_t smem_raw[];
	uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
	__shared__ __align__(8) uint64_t q_full[kKvStages], q_empty[kKvStages], sdp_full, pds_full, acc_full, kv_ready,
		drain;
	__shared__ uint32_t tmem_base_sh;
	__shared__ int abort_sh;

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int NH = p.N * p.H;
	const int kt = (int)(blockIdx.x / NH);                       // causal: first key tiles have the most queries
	const int nh = (int)(blockIdx.x % NH);
	const int n = nh / p.H, h = nh % p.H;
	const int k0 = kt * kKvRows;
	const int qt_end = (p.Tq + kKvQ - 1) / kKvQ;
	const int qt_begin = p.causal ? min(k0 / kKvQ, qt_end) : 0;
	const int J = qt_end - qt_begin;

	if (threadIdx.x == 0) {
		for (int s = 0; s < kKvStages; ++s) {
			mbar_init(smem_u32(&q_full[s]), 1);
			mbar_init(smem_u32(&q_empty[s]), 1);
		}
		mbar_init(smem_u32(&sdp_full), 1);
		mbar_init(smem_u32(&pds_full), kMathThreads);
		mbar_init(smem_u32(&acc_full), 1);
		mbar_init(smem_u32(&kv_ready), kMathThreads);
		mbar_init(smem_u32(&drain), 1);
		abort_sh = 0;
		fence_mbar_init();
	}
	if (warp == 1) {
		tmem_alloc(smem_u32(&tmem_base_sh), kTmemCols);
		tmem_relinquish();
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = tmem_base_sh;
	volatile int* abort_flag = &abort_sh;

	if (warp == 0) {
		if (lane == 0) {
			const long long img = (long long)nh * packed_head_floats(p.Tpq);
			const float* qb = p.pq + img;
			const float* ob = p.pdo + img;
			const float* qm = p.pq_mn + img;
			const float* om = p.pdo_mn + img;
			const float* st = p.rowstat + (long long)nh * 3 * p.Tpq;
			const int parts = p.split ? 2 : 1;
			int issued = 0;
			for (int j = 0; j < J; ++j) {
				const int s = j % kKvStages;
				if (j >= kKvStages &&
						!mbar_wait(smem_u32(&q_empty[s]), ((j / kKvStages) & 1) ^ 1, p.err, kDevTimeoutAttn, abort_flag))
					break;
				const uint32_t fb = smem_u32(&q_full[s]);
				mbar_arrive_expect_tx(fb, parts * 4 * kKvOpBytes + 3 * kKvQ * 4);
				const uint32_t dst = smem_u32(smem + s * kKvStageBytes);
				const long long r0 = (long long)(qt_begin + j) * kKvQ;
				for (int hl = 0; hl < parts; ++hl) {
					copy_kmajor(dst + hl * kKvOpBytes, qb, hl, p.Tpq, r0, kKvQ, fb);
					copy_kmajor(dst + 2 * kKvOpBytes + hl * kKvOpBytes, ob, hl, p.Tpq, r0, kKvQ, fb);
					copy_mnmajor(dst + 4 * kKvOpBytes + hl * kKvOpBytes, qm, hl, p.Tpq, r0, kKvQ, fb);
					copy_mnmajor(dst + 6 * kKvOpBytes + hl * kKvOpBytes, om, hl, p.Tpq, r0, kKvQ, fb);
				}
				for (int w = 0; w < 3; ++w) bulk_load(dst + kKvStatOff + w * kKvQ * 4, st + w * p.Tpq + r0, kKvQ * 4, fb);
				issued = j + 1;
			}
			for (int j = max(0, issued - kKvStages); j < issued; ++j)
				drain_wait(smem_u32(&q_full[j % kKvStages]), (j / kKvStages) & 1, p.err);
		}
	} else if (warp == 1) {
		if (lane == 0) {
			const uint32_t id_s = idesc_tf32(kKvRows, kKvQ);
			const uint32_t id_acc = idesc_tf32(kKvRows, kDh) | kIdescBMajorMN;
			bool ok = mbar_wait(smem_u32(&kv_ready), 0, p.err, kDevTimeoutAttn, abort_flag);
			tc_fence_after();
			for (int j = 0; ok && j < J; ++j) {
				const int s = j % kKvStages;
				if (!mbar_wait(smem_u32(&q_full[s]), (j / kKvStages) & 1, p.err, kDevTimeoutAttn, abort_flag)) break;
				tc_fence_after();
				const uint32_t qbase = smem_u32(smem + s * kKvStageBytes);
				const uint32_t obase = qbase + 2 * kKvOpBytes, qmn = qbase + 4 * kKvOpBytes, omn = qbase + 6 * kKvOpBytes;
#pragma unroll
				for (int ks = 0; ks < kDh / 8; ++ks) {      // S^T = K Q^T
					const uint32_t off = (ks >> 1) * (kKvQ * 64) + (ks & 1) * 32;
					mma_step(tmem + kKColS, tmem + kKColKhi + ks * 8, tmem + kKColKlo + ks * 8,
						smem_desc_k_sw64(qbase + off), smem_desc_k_sw64(qbase + kKvOpBytes + off), id_s, ks > 0, p.split);
				}
#pragma unroll
				for (int ks = 0; ks < kDh / 8; ++ks) {      // dP^T = V dO^T
					const uint32_t off = (ks >> 1) * (kKvQ * 64) + (ks & 1) * 32;
					mma_step(tmem + kKColP, tmem + kKColVhi + ks * 8, tmem + kKColVlo + ks * 8,
						smem_desc_k_sw64(obase + off), smem_desc_k_sw64(obase + kKvOpBytes + off), id_s, ks > 0, p.split);
				}
				mma_commit(smem_u32(&sdp_full));
				if (!mbar_wait(smem_u32(&pds_full), j & 1, p.err, kDevTimeoutAttn, abort_flag)) break;
				tc_fence_after();
#pragma unroll
				for (int ks = 0; ks < kKvQ / 8; ++ks) {
					const uint32_t acc = (j > 0 || ks > 0);
					// dV += P^T dO
					mma_step(tmem + kKColDv, tmem + kKColS + ks * 8, tmem + kKColSlo + ks * 8,
						smem_desc_mn_sw128b32(omn + ks * 1024, kKvQ * 128),
						smem_desc_mn_sw128b32(omn + kKvOpBytes + ks * 1024, kKvQ * 128), id_acc, acc, p.split);
					// dK += dS^T Q
					mma_step(tmem + kKColDk, tmem + kKColP + ks * 8, tmem + kKColPlo + ks * 8,
						smem_desc_mn_sw128b32(qmn + ks * 1024, kKvQ * 128),
						smem_desc_mn_sw128b32(qmn + kKvOpBytes + ks * 1024, kKvQ * 128), id_acc, acc, p.split);
				}
				mma_commit(smem_u32(&q_empty[s]));
				if (j == J - 1) mma_commit(smem_u32(&acc_full));
			}
			mma_commit(smem_u32(&drain));
			drain_wait(smem_u32(&drain), 0, p.err);
		}
	} else {
		// ------------- P^T and dS^T: two threads per key row, 16 query columns each -------------
		const int quad = warp & 3, half = (warp - 2) >> 2;
		const int row = quad * 32 + lane, key = k0 + row;
		const bool key_ok = key < p.Tk;
		const uint32_t lb = tmem + ((uint32_t)(quad * 32) << 16);
		const long long roff = ((long long)n * p.Tk + (key_ok ? key : 0)) * p.D + h * kDh;
		half_row_to_tmem(p.k + roff + half * 32, key_ok, lb + kKColKhi + half * 32, lb + kKColKlo + half * 32);
		half_row_to_tmem(p.v + roff + half * 32, key_ok, lb + kKColVhi + half * 32, lb + kKColVlo + half * 32);
		tmem_wait_st();
		tc_fence_before();
		mbar_arrive(smem_u32(&kv_ready));

		const bool padded = p.pad && key_ok && p.pad[(long long)n * p.Tk + key] == 0.0f;
		const float c1 = p.scale * kLog2e;
		bool ok = true;
		for (int j = 0; j < J; ++j) {
			const int s = j % kKvStages;
			// the stage's m / (1/l) / D words were written by the bulk copy: observe its barrier too
			if (!warp_wait(smem_u32(&q_full[s]), (j / kKvStages) & 1, p.err, abort_flag) ||
					!warp_wait(smem_u32(&sdp_full), j & 1, p.err, abort_flag)) {
				ok = false;
				break;
			}
			tc_fence_after();
			const float* m_j = reinterpret_cast<const float*>(smem + s * kKvStageBytes + kKvStatOff) + half * 16;
			const float* il_j = m_j + kKvQ;
			const float* d_j = m_j + 2 * kKvQ;
			const int qbeg = (qt_begin + j) * kKvQ + half * 16;
			uint32_t rs[16], rp[16];
			tmem_ld_32x32b_x16(lb + kKColS + half * 16, rs);
			tmem_ld_32x32b_x16(lb + kKColP + half * 16, rp);
			tmem_wait_ld();
			// queries past Tq have zero Q / dO rows and neutral statistics, keys past Tk zero K / V
			// rows (their dK / dV rows are not stored): only the causal diagonal and padding need masks
			const bool general = padded || (p.causal && k0 + kKvRows - 1 > (qt_begin + j) * kKvQ);
			float pr[16], ds[16];
			if (!general) {
#pragma unroll
				for (int c = 0; c < 16; ++c) {
					pr[c] = exp2_hw(__fmaf_rn(__uint_as_float(rs[c]), c1, -(m_j[c] * kLog2e))) * il_j[c];
					ds[c] = p.scale * (pr[c] * (__uint_as_float(rp[c]) - d_j[c]));
				}
			} else {
#pragma unroll
				for (int c = 0; c < 16; ++c) {
					const bool live = !p.causal || key <= qbeg + c;
					const float x = padded ? (-1e9f - m_j[c]) * kLog2e : __fmaf_rn(__uint_as_float(rs[c]), c1, -(m_j[c] * kLog2e));
					pr[c] = live ? exp2_hw(x) * il_j[c] : 0.0f;
					ds[c] = (live && !padded) ? p.scale * (pr[c] * (__uint_as_float(rp[c]) - d_j[c])) : 0.0f;
				}
			}
			vals_to_tmem16(pr, lb + kKColS + half * 16, lb + kKColSlo + half * 16);
			vals_to_tmem16(ds, lb + kKColP + half * 16, lb + kKColPlo + half * 16);
			tmem_wait_st();
			tc_fence_before();
			mbar_arrive(smem_u32(&pds_full));
		}
		if (ok && J > 0) ok = warp_wait(smem_u32(&acc_full), 0, p.err, abort_flag);
		if (ok) {
			tc_fence_after();
			// half 0 writes dV, half 1 writes dK (64 columns each)
			float* dst = half == 0 ? p.dv : p.dk;
			const int first = half == 0 ? p.dv_first : p.dk_first;
			const uint32_t col = half == 0 ? kKColDv : kKColDk;
			float acc[kDh];
#pragma unroll
			for (int hh = 0; hh < 2; ++hh) {
				uint32_t r[32];
				if (J > 0) {
					tmem_ld_32x32b_x32(lb + col + hh * 32, r);
					tmem_wait_ld();
				}
#pragma unroll
				for (int c = 0; c < 32; ++c) acc[hh * 32 + c] = J > 0 ? __uint_as_float(r[c]) : 0.0f;
			}
			if (key_ok && dst) store_row(dst + roff, acc, first);
		}
	}

	tc_fence_before();
	__syncthreads();
	if (warp == 1) {
		__syncwarp();
		tc_fence_after();
		tmem_dealloc(tmem, kTmemCols);
	}
}

}  // namespace

static std::mutex g_fa_mutex;
static bool g_fa_attr[64];

static nnb_status fa_set_attrs(int dev) {
	std::lock_guard<std::mutex> lock(g_fa_mutex);
	if (g_fa_attr[dev & 63]) return NNB_OK;
	NNB_CUDA_TRY(cudaFuncSetAttribute(flash_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem));
	NNB_CUDA_TRY(cudaFuncSetAttribute(flash_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDqSmem));
	NNB_CUDA_TRY(cudaFuncSetAttribute(flash_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kKvSmem));
	g_fa_attr[dev & 63] = true;
	return NNB_OK;
}

static long long round_up(long long x, long long a) { return (x + a - 1) / a * a; }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static nnb_status fa_check(size_t N, size_t Tq, size_t Tk, size_t D, size_t heads, int causal) {
	if (heads == 0 || D % heads != 0 || Tq == 0 || Tk == 0 || (causal && Tq != Tk))
		return fail(NNB_ERR_SHAPE, "flash attention: bad shapes (N %zu, Tq %zu, Tk %zu, D %zu, heads %zu, causal %d)", N,
			Tq, Tk, D, heads, causal);
	if (D / heads != (size_t)kDh)
		return fail(NNB_ERR_UNSUPPORTED, "flash attention: head size %zu (only %d is fused; use nnb_attention_*)",
			D / heads, kDh);
	const unsigned long long ctas = (unsigned long long)N * heads * ((std::max(Tq, Tk) + kRowAlign - 1) / kRowAlign);
	if (Tq > (1u << 28) || Tk > (1u << 28) || ctas >= (1ull << 31))
		return fail(NNB_ERR_UNSUPPORTED, "flash attention: problem too large (N %zu, Tq %zu, Tk %zu, heads %zu)", N, Tq,
			Tk, heads);
	return NNB_OK;
}

static nnb_status fa_pack(cudaStream_t s, int count, const PackSet& ps, long long NH, int H, long long D, int with_lo) {
	TraceScope ts(s, kTracePack);
	long long most = 0;
	for (int t = 0; t < count; ++t) most = std::max(most, NH * ps.Tp[t] * 16);
	const unsigned blocks = grid_for(most, 256);
	attn_pack_kernel<<<dim3(blocks, count), 256, 0, s>>>(ps, NH, H, D, with_lo);
	return cuda_status(cudaGetLastError(), "attention pack launch");
}

}  // namespace nnb

extern "C" {

int nnb_flash_attention_supported(size_t D, size_t heads) {
	return heads != 0 && D % heads == 0 && D / heads == (size_t)nnb::kDh;
}

nnb_status nnb_flash_attention_fwd(void* stream, size_t N, size_t Tq, size_t Tk, size_t D, size_t heads, const float* q,
		const float* k, const float* v, const float* key_padding_mask, int causal, float* out, float* stats) {
	NNB_TRY(nnb::fa_check(N, Tq, Tk, D, heads, causal));
	if (N == 0) return NNB_OK;
	if (!q || !k || !v || !out || !stats) return nnb::fail(NNB_ERR_INVALID, "flash_attention_fwd: null pointer");
	if (!nnb::aligned16(q) || !nnb::aligned16(k) || !nnb::aligned16(v) || !nnb::aligned16(out))
		return nnb::fail(NNB_ERR_INVALID, "flash_attention_fwd: q, k, v and out must be 16-byte aligned");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	nnb::DeviceState* dev = nullptr;
	NNB_TRY(nnb::device_state(&dev));
	NNB_TRY(nnb::fa_set_attrs(dev->device));
	const int split = nnb::math_mode() == NNB_MATH_FP32X3 ? 1 : 0;
	const long long NH = (long long)N * heads;
	const long long Tpk = nnb::round_up((long long)Tk, nnb::kRowAlign);
	const size_t head_bytes = (size_t)nnb::packed_head_floats(Tpk) * sizeof(float);
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, 2 * NH * head_bytes, s));
	float* pk = static_cast<float*>(ws);
	float* pv = pk + NH * nnb::packed_head_floats(Tpk);
	nnb_status st = NNB_OK;
	do {
		nnb::PackSet ps{};
		ps.src[0] = k; ps.kdst[0] = pk; ps.T[0] = (int)Tk; ps.Tp[0] = (int)Tpk;       // S = Q K^T
		ps.src[1] = v; ps.mdst[1] = pv; ps.T[1] = (int)Tk; ps.Tp[1] = (int)Tpk;       // O += P V
		if ((st = nnb::fa_pack(s, 2, ps, NH, (int)heads, (long long)D, split)) != NNB_OK) break;
		nnb::FwdParams p{};
		p.pk = pk; p.pv = pv; p.q = q; p.pad = key_padding_mask; p.out = out; p.stats = stats; p.err = dev->error_word;
		p.D = (long long)D; p.N = (int)N; p.H = (int)heads; p.Tq = (int)Tq; p.Tk = (int)Tk; p.Tpk = (int)Tpk;
		p.q_tiles = (int)((Tq + nnb::kFwdRows - 1) / nnb::kFwdRows);
		p.causal = causal ? 1 : 0; p.split = split;
		p.scale = 1.0f / std::sqrt(static_cast<float>(nnb::kDh));     // ops.cpp:1236
		nnb::TraceScope ts(s, nnb::kTraceAttention);
		nnb::flash_fwd_kernel<<<(unsigned)(NH * p.q_tiles), nnb::kThreadsFa, nnb::kFwdSmem, s>>>(p);
		st = nnb::cuda_status(cudaGetLastError(), "flash attention forward launch");
	} while (0);
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

nnb_status nnb_flash_attention_bwd(void* stream, size_t N, size_t Tq, size_t Tk, size_t D, size_t heads, const float* g,
		const float* q, const float* k, const float* v, const float* out, const float* stats,
		const float* key_padding_mask, int causal, float* dq, int dq_first, float* dk, int dk_first, float* dv,
		int dv_first) {
	NNB_TRY(nnb::fa_check(N, Tq, Tk, D, heads, causal));
	if (N == 0 || (!dq && !dk && !dv)) return NNB_OK;
	if (!g || !q || !k || !v || !out || !stats) return nnb::fail(NNB_ERR_INVALID, "flash_attention_bwd: null input");
	const float* al[] = {g, q, k, v, out, dq, dk, dv};
	for (const float* a : al)
		if (a && !nnb::aligned16(a)) return nnb::fail(NNB_ERR_INVALID, "flash_attention_bwd: tensors must be 16-byte aligned");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	nnb::DeviceState* dev = nullptr;
	NNB_TRY(nnb::device_state(&dev));
	NNB_TRY(nnb::fa_set_attrs(dev->device));
	const int split = nnb::math_mode() == NNB_MATH_FP32X3 ? 1 : 0;
	const long long NH = (long long)N * heads;
	const long long Tpq = nnb::round_up((long long)Tq, nnb::kRowAlign), Tpk = nnb::round_up((long long)Tk, nnb::kRowAlign);
	const long long fq = NH * nnb::packed_head_floats(Tpq), fk = NH * nnb::packed_head_floats(Tpk);
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, (size_t)(4 * fq + 3 * fk + NH * 3 * Tpq) * sizeof(float), s));
	float* pq = static_cast<float*>(ws);
	float* pq_mn = pq + fq;
	float* pdo = pq_mn + fq;
	float* pdo_mn = pdo + fq;
	float* pk = pdo_mn + fq;
	float* pk_mn = pk + fk;
	float* pv = pk_mn + fk;
	float* rowstat = pv + fk;
	nnb_status st = NNB_OK;
	do {
		nnb::PackSet ps{};
		ps.src[0] = q; ps.kdst[0] = pq; ps.mdst[0] = pq_mn; ps.T[0] = (int)Tq; ps.Tp[0] = (int)Tpq;
		ps.src[1] = g; ps.kdst[1] = pdo; ps.mdst[1] = pdo_mn; ps.T[1] = (int)Tq; ps.Tp[1] = (int)Tpq;
		ps.src[2] = k; ps.kdst[2] = pk; ps.mdst[2] = pk_mn; ps.T[2] = (int)Tk; ps.Tp[2] = (int)Tpk;
		ps.src[3] = v; ps.kdst[3] = pv; ps.T[3] = (int)Tk; ps.Tp[3] = (int)Tpk;
		if ((st = nnb::fa_pack(s, 4, ps, NH, (int)heads, (long long)D, split)) != NNB_OK) break;
		nnb::BwdParams p{};
		p.pq = pq; p.pq_mn = pq_mn; p.pdo = pdo; p.pdo_mn = pdo_mn; p.pk = pk; p.pk_mn = pk_mn; p.pv = pv;
		p.q = q; p.k = k; p.v = v; p.dout = g; p.out = out; p.stats = stats; p.pad = key_padding_mask;
		p.rowstat = rowstat; p.dq = dq; p.dk = dk; p.dv = dv;
		p.dq_first = dq_first; p.dk_first = dk_first; p.dv_first = dv_first;
		p.err = dev->error_word;
		p.D = (long long)D; p.N = (int)N; p.H = (int)heads; p.Tq = (int)Tq; p.Tk = (int)Tk;
		p.Tpq = (int)Tpq; p.Tpk = (int)Tpk;
		p.q_tiles = (int)((Tq + nnb::kFwdRows - 1) / nnb::kFwdRows);
		p.k_tiles = (int)((Tk + nnb::kKvRows - 1) / nnb::kKvRows);
		p.causal = causal ? 1 : 0; p.split = split;
		p.scale = 1.0f / std::sqrt(static_cast<float>(nnb::kDh));
		nnb::TraceScope ts(s, nnb::kTraceAttention);
		// the dQ kernel also writes the row statistics the dKdV kernel reads
		nnb::flash_bwd_dq_kernel<<<(unsigned)(NH * p.q_tiles), nnb::kThreadsFa, nnb::kDqSmem, s>>>(p);
		if ((st = nnb::cuda_status(cudaGetLastError(), "flash attention dQ launch")) != NNB_OK) break;
		if (dk || dv) {
			nnb::flash_bwd_dkdv_kernel<<<(unsigned)(NH * p.k_tiles), nnb::kThreadsFa, nnb::kKvSmem, s>>>(p);
			st = nnb::cuda_status(cudaGetLastError(), "flash attention dKdV launch");
		}
	} while (0);
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

}  // extern "C"
