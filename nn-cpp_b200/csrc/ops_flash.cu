// ops_flash.cu -- fused multi-head attention for head size 64: the `attention` op of
// src/autograd/ops.cpp:1226-1296 (scores Q_h K_h^T, the masked softmax of ops.cpp:1183-1224 with
// scale 1/sqrt(Dh), then P V_h) and its backward (ops.cpp:1280-1293), without materialising the
// {N, H, Tq, Tk} probability matrix.
//
// The reference runs two sgemm calls per (sample, head) and keeps P for the backward pass. Here the
// work is split into items -- 128 query rows (or 128 keys) of one (sample, head) -- and a persistent
// grid of one CTA per SM walks the items, heaviest causal items first, with every barrier phase
// carried from item to item so that one item's loads and MMAs overlap the previous item's tail.
//   forward   S = Q K^T (Q in tensor memory, K tiles in shared memory), online softmax in registers
//             (four threads per query row, 16 keys each), P split into TF32 hi/lo and stored to tensor memory,
//             then O += P V (TS MMA: P from tensor memory, V an MN-major B operand). Only O and the
//             row statistics (max m, sum l of exp(score - m)) are written.
//   backward  two kernels, each output element written by exactly one CTA (no atomics, fixed order):
//             dQ kernel  (128 query rows): S and dP = dO V^T recomputed (Q, dO in tensor memory),
//                        dS = scale P (dP - D), dQ += dS K; it also writes m and 1/l per row.
//             dKdV kernel (128 keys): S^T = K Q^T, dP^T = V dO^T (K, V in tensor memory), P^T and
//                        dS^T to tensor memory, dV += P^T dO and dK += dS^T Q in tensor memory.
//             D = rowsum(dO o O) comes from the pack kernel.
// Every product is 3xTF32 (lo*hi + hi*lo + hi*hi) in the fp32x3 math mode, one TF32 MMA in the
// tf32 mode, as the GEMM does. exp(x) is evaluated as 2^(x log2 e) with the hardware ex2.
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
// Every kernel here: warp 0 loads, warp 1 issues MMAs, warps 2-17 do the per-element math, four warps
// per tensor-memory lane quarter (warp w reaches lanes 32 (w % 4) .. +31), each taking a quarter of a
// row's columns (kFwdParts, kDqParts, kKvParts below).
constexpr float kLog2e = 1.4426950408889634f;   // exp(x) = 2^(x log2 e)

// Floats of one (sample, head) image of Tp rows, either form: hi and lo, 64 floats per row each.
__host__ __device__ inline long long packed_head_floats(long long Tp) { return 2LL * kDh * Tp; }

// Float offset, inside one head's image, of the 16-byte unit u (head columns 4u .. 4u+3) of row r.
__device__ __forceinline__ int kmajor_offset(int hl, int u, int r, int Tp) {
	return ((hl * kPanels + (u >> 2)) * Tp + r) * 16 + (((u & 3) ^ ((r >> 1) & 3)) << 2);
}
__device__ __forceinline__ int mnmajor_offset(int hl, int u, int r, int Tp) {
	const int e = (u & 7) * 4;                 // column inside the 32-float block
	return ((hl * kBlocks + (u >> 3)) * Tp + r) * 32 + ((((e >> 3) ^ (r & 3)) << 3) | (e & 7));
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

__device__ __forceinline__ void prefetch_l2(const void* p) {
	asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<uint64_t>(p)));
}

// hi / lo split of an even count of per-tile values (probabilities, score gradients), two at a time
// with packed fp32 instructions. hi is Veltkamp's splitting (Dekker 1971) with the constant 2^13 + 1:
// p = 8193 v, hi = (v - p) + p keeps the top 11 significant bits of v rounded to nearest (a TF32
// value, low 13 bits zero) and lo = v - hi is exact. p is formed as the single fused operation
// fma(v, 8192, v), which is 8193 v rounded once, so no compiler contraction of a multiply into the
// following add can change it (the splitting needs p rounded before v - p is taken). lo keeps up to 13
// significant bits, of which the TF32 MMA reads the top 11 (it ignores an operand's low 13 bits), so
// lo is not rounded here: the products' error stays near 2^-21 of |v| (against 2^-22 for a rounded
// lo), and the split costs four fp32 operations per value instead of two conversions. |v| must stay
// below 2^128 / 8193.
template <int kN>
__device__ __forceinline__ void split_pairs(const float (&v)[kN], uint32_t (&hi)[kN], uint32_t (&lo)[kN]) {
	const float2 k8192 = make_float2(8192.0f, 8192.0f);
#pragma unroll
	for (int c = 0; c < kN; c += 2) {
		const float2 x = make_float2(v[c], v[c + 1]);
		const float2 p = fma2_rn(x, k8192, x);
		const float2 h = add2_rn(add2_rn(x, make_float2(-p.x, -p.y)), p);
		const float2 l = add2_rn(x, make_float2(-h.x, -h.y));
		hi[c] = __float_as_uint(h.x);
		hi[c + 1] = __float_as_uint(h.y);
		lo[c] = __float_as_uint(l.x);
		lo[c + 1] = __float_as_uint(l.y);
	}
}

// Splits 16 values (|v| < 2^128 / 8193) and stores hi / lo to two column groups of this thread's lane.
__device__ __forceinline__ void vals_to_tmem16(const float (&v)[16], uint32_t taddr_hi, uint32_t taddr_lo) {
	uint32_t hi[16], lo[16];
	split_pairs<16>(v, hi, lo);
	tmem_st_32x32b_x16(taddr_hi, hi);
	tmem_st_32x32b_x16(taddr_lo, lo);
}

// Bit c set when key key0 + c takes part in query row qrow's softmax: below Tk and, causal, not after
// the row. Built arithmetically so that the masked paths below select per column without branching (a
// per-column test of a lane-dependent condition around the padding load made every column a divergent
// branch: the masked tiles ran about six times slower than the others).
__device__ __forceinline__ uint32_t live_bits32(int key0, int qrow, int Tk, int causal) {
	int n = Tk - key0;
	if (causal) n = min(n, qrow - key0 + 1);
	return n <= 0 ? 0u : n >= 32 ? 0xffffffffu : (1u << n) - 1u;
}

// Bit c set when key key0 + c is live and marked as padding (0) in the key-padding row padn (null: none).
__device__ __forceinline__ uint32_t padded_bits32(const float* padn, int key0, uint32_t live) {
	uint32_t bits = 0;
	if (padn) {
#pragma unroll
		for (int c = 0; c < 32; ++c) {
			const bool on = (live >> c) & 1u;
			const float f = on ? padn[key0 + c] : 1.0f;
			bits |= (f == 0.0f ? 1u : 0u) << c;
		}
	}
	return bits;
}

// One MMA step (depth 8) of D (+)= A B, three TF32 MMAs (lo*hi, hi*lo, hi*hi) in the 3xTF32 split
// or one (hi*hi) in TF32; A from tensor memory (hi, lo columns) or shared memory (hi, lo
// descriptors), B from shared-memory descriptors (hi, lo). The caller passes descriptors built once
// per tile plus compile-time offsets, so issuing an MMA costs a few instructions. Warp-collective:
// the whole MMA warp calls it and one elected lane issues.
template <int kSplit>
__device__ __forceinline__ void mma_step(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint64_t b_hi, uint64_t b_lo,
		uint32_t idesc, uint32_t acc) {
	if (kSplit) {
		mma_tf32_ts_elect(d, a_lo, b_hi, idesc, acc);
		mma_tf32_ts_elect(d, a_hi, b_lo, idesc, 1u);
		mma_tf32_ts_elect(d, a_hi, b_hi, idesc, 1u);
	} else {
		mma_tf32_ts_elect(d, a_hi, b_hi, idesc, acc);
	}
}
template <int kSplit>
__device__ __forceinline__ void mma_step_ss(uint32_t d, uint64_t a_hi, uint64_t a_lo, uint64_t b_hi, uint64_t b_lo,
		uint32_t idesc, uint32_t acc) {
	if (kSplit) {
		mma_tf32_elect(d, a_lo, b_hi, idesc, acc);
		mma_tf32_elect(d, a_hi, b_lo, idesc, 1u);
		mma_tf32_elect(d, a_hi, b_hi, idesc, 1u);
	} else {
		mma_tf32_elect(d, a_hi, b_hi, idesc, acc);
	}
}

// Descriptor of (tile base + byte offset): the start-address field holds address / 16 in its low 14
// bits, and every tile here lies below 256 KB, so an offset is a plain add.
__device__ __forceinline__ uint64_t desc_at(uint64_t d, uint32_t byte_offset) { return d + (byte_offset >> 4); }

// ---------------------------------------------------------------------------------------------
// Pack: x [N, T, D] (head h in columns h*64 .. h*64+63) -> the K-major and / or MN-major image of
// every (sample, head), as described above (a null destination skips that form). With dot_with
// set, it also writes dot_out[nh * dot_stride + row] = sum over the head row of x * dot_with (the
// backward's D = rowsum(dO o O); zero for padding rows).
// grid = (Tp_max * 16 / 256, min(N*H, 65535), tensors); one thread per 16-byte unit of a row.
// ---------------------------------------------------------------------------------------------
struct PackSet {
	const float* src[4];
	float* kdst[4];
	float* mdst[4];
	const float* dot_with[4];
	float* dot_out[4];
	long long dot_stride[4];
	int T[4];
	int Tp[4];
};

__global__ void __launch_bounds__(256) attn_pack_kernel(const PackSet ps, int NH, int H, long long D, int with_lo) {
	const int t = blockIdx.z;
	const int Tp = ps.Tp[t];
	if ((int)(blockIdx.x * 16) >= Tp) return;          // whole block past this tensor's rows
	const int i = blockIdx.x * 256 + threadIdx.x;
	const int row = i >> 4, u = i & 15;
	const float* __restrict__ x = ps.src[t];
	float* __restrict__ kd = ps.kdst[t];
	float* __restrict__ md = ps.mdst[t];
	const float* __restrict__ ow = ps.dot_with[t];
	const int T = ps.T[t];
	for (int nh = blockIdx.y; nh < NH; nh += gridDim.y) {
		const int n = nh / H, h = nh - n * H;
		const long long src_off = ((long long)n * T + row) * D + h * kDh + u * 4;
		float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
		if (row < T) v = __ldg(reinterpret_cast<const float4*>(x + src_off));
		float4 hi, lo;
		split4(v, hi, lo);
		const long long base = (long long)nh * packed_head_floats(Tp);
		if (kd) {
			*reinterpret_cast<float4*>(kd + base + kmajor_offset(0, u, row, Tp)) = hi;
			if (with_lo) *reinterpret_cast<float4*>(kd + base + kmajor_offset(1, u, row, Tp)) = lo;
		}
		if (md) {
			*reinterpret_cast<float4*>(md + base + mnmajor_offset(0, u, row, Tp)) = hi;
			if (with_lo) *reinterpret_cast<float4*>(md + base + mnmajor_offset(1, u, row, Tp)) = lo;
		}
		if (ow) {
			float part = 0.0f;
			if (row < T) {
				const float4 o = __ldg(reinterpret_cast<const float4*>(ow + src_off));
				part = v.x * o.x;
				part += v.y * o.y;
				part += v.z * o.z;
				part += v.w * o.w;
			}
#pragma unroll
			for (int off = 8; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
			if (u == 0) ps.dot_out[t][(long long)nh * ps.dot_stride[t] + row] = part;
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

// Tensor-memory allocation by warp 1, then a block-wide sync with the tcgen05 fences around it (the
// caller's thread 0 has initialised the barriers before).
__device__ __forceinline__ uint32_t fa_setup_tmem(uint32_t* tmem_base_sh, int warp) {
	if (warp == 1) {
		tmem_alloc(smem_u32(tmem_base_sh), kTmemCols);
		tmem_relinquish();
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	return *tmem_base_sh;
}

__device__ __forceinline__ void fa_release_tmem(uint32_t tmem, int warp) {
	tc_fence_before();
	__syncthreads();
	if (warp == 1) {
		__syncwarp();
		tc_fence_after();
		tmem_dealloc(tmem, kTmemCols);
	}
}

// ---------------------------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------------------------
struct FwdParams {
	const float* q;      // [N, Tq, D]
	const float* pk;     // K, K-major image, Tpk rows per head
	const float* pv;     // V, MN-major image
	const float* pad;    // [N, Tk] key-padding mask (0 = padded) or null
	float* out;          // [N, Tq, D]
	float* stats;        // [N, H, Tq, 2]: row max m, row sum l of exp(score - m)
	int* err;
	long long D;
	int N, H, Tq, Tk, Tpk, q_tiles, causal, split;
	float scale;
};

constexpr int kFwdRows = 128;                               // query rows per item (MMA M)
constexpr int kFwdKeys = 64;                                // keys per tile (S columns, PV depth)
constexpr uint32_t kFwdOpBytes = kPanels * kFwdKeys * 64;   // 16 KB: one of K hi, K lo, V hi, V lo
// K and V tiles stream through separate rings: a K slot is free once the tile's score MMAs are done,
// a V slot once its P V MMAs are, so the K loads run further ahead
constexpr int kFwdSlots = 3;
constexpr uint32_t kFwdSlotBytes = 2 * kFwdOpBytes;         // hi, lo
constexpr uint32_t kFwdVBase = kFwdSlots * kFwdSlotBytes;
constexpr uint32_t kFwdSmem = 2 * kFwdSlots * kFwdSlotBytes + 1024;
// tensor-memory columns: Q hi | Q lo | S/P-hi b, P-lo b (b = 0, 1; 128 columns per buffer) | PV 0 | PV 1
constexpr uint32_t kFColQhi = 0, kFColQlo = 64, kFColS = 128, kFColPV = 384;

// Work item w -> (sample, head) and query tile; key tiles it streams. A head's query tiles are
// consecutive items (heaviest causal tile first), so the CTAs that run them at the same time share
// that head's K / V tiles through L2.
__device__ __forceinline__ void fwd_item(const FwdParams& p, int w, int& q0, int& nh, int& J) {
	nh = w / p.q_tiles;
	q0 = (p.q_tiles - 1 - w % p.q_tiles) * kFwdRows;
	const int key_end = p.causal ? min(q0 + kFwdRows, p.Tq) : p.Tk;
	J = (key_end + kFwdKeys - 1) / kFwdKeys;
}

// The forward's softmax is its critical path (about 2400 cycles per 64-key tile with two math warps
// per lane quarter against about 1400 of MMA issue), so it runs four math warps per lane quarter, each
// thread a quarter of a row's columns: twice the warps per scheduler to hide the latencies of the same
// instruction stream.
constexpr int kFwdParts = 4;                                // math threads per query row
constexpr int kFwdMathThreads = 32 * 4 * kFwdParts;
constexpr int kFwdThreads = 64 + kFwdMathThreads;
constexpr int kFwdCols = kFwdKeys / kFwdParts;             // score columns per math thread
constexpr int kFwdHeadCols = kDh / kFwdParts;              // output columns per math thread

// The kFwdParts math threads of a row exchange one value each through shared memory (mbarrier
// count kFwdMathThreads / 4 per lane quarter); returns false (warp-uniform) if the wait ran out.
__device__ __forceinline__ bool row_exchange(float (*slots)[kFwdRows], int part, int row, float v, float (&all)[kFwdParts],
		uint32_t bar, uint32_t parity, int* err, volatile int* abort) {
	slots[part][row] = v;
	mbar_arrive(bar);
	if (!warp_wait(bar, parity, err, abort)) return false;
#pragma unroll
	for (int q = 0; q < kFwdParts; ++q) all[q] = slots[q][row];
	return true;
}

template <int kSplit>
__global__ void __launch_bounds__(kFwdThreads, 1) flash_fwd_kernel(const FwdParams p) {
	extern __shared__ uint8_t smem_raw[];
	uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
	__shared__ __align__(8) uint64_t k_full[kFwdSlots], k_empty[kFwdSlots], v_full[kFwdSlots], v_empty[kFwdSlots],
		s_full[2], p_full[2], pv_full[2], pv_empty[2], q_ready, xbar[4][2], drain;
	__shared__ float xval[2][kFwdParts][kFwdRows];  // [exchange parity][part][row]
	__shared__ uint32_t tmem_base_sh;
	__shared__ int abort_sh;

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int W = p.N * p.H * p.q_tiles;
	if (threadIdx.x == 0) {
		for (int s = 0; s < kFwdSlots; ++s) {
			mbar_init(smem_u32(&k_full[s]), 1);
			mbar_init(smem_u32(&k_empty[s]), 1);
			mbar_init(smem_u32(&v_full[s]), 1);
			mbar_init(smem_u32(&v_empty[s]), 1);
		}
		for (int b = 0; b < 2; ++b) {
			mbar_init(smem_u32(&s_full[b]), 1);
			mbar_init(smem_u32(&p_full[b]), kFwdMathThreads);
			mbar_init(smem_u32(&pv_full[b]), 1);
			mbar_init(smem_u32(&pv_empty[b]), kFwdMathThreads);
		}
		for (int qd = 0; qd < 4; ++qd) {
			mbar_init(smem_u32(&xbar[qd][0]), 32 * kFwdParts);
			mbar_init(smem_u32(&xbar[qd][1]), 32 * kFwdParts);
		}
		mbar_init(smem_u32(&q_ready), kFwdMathThreads);
		mbar_init(smem_u32(&drain), 1);
		abort_sh = 0;
		fence_mbar_init();
	}
	const uint32_t tmem = fa_setup_tmem(&tmem_base_sh, warp);
	volatile int* abort_flag = &abort_sh;
	constexpr int parts = kSplit ? 2 : 1;

	if (warp == 0) {
		if (lane == 0) {
			// ------------------------------ bulk-copy producer ------------------------------
			int t = 0;
			bool ok = true;
			for (int w = blockIdx.x; ok && w < W; w += gridDim.x) {
				int q0, nh, J;
				fwd_item(p, w, q0, nh, J);
				const float* kb = p.pk + (long long)nh * packed_head_floats(p.Tpk);
				const float* vb = p.pv + (long long)nh * packed_head_floats(p.Tpk);
				for (int j = 0; j < J; ++j, ++t) {
					const int s = t % kFwdSlots, use = t / kFwdSlots;
					const long long r0 = (long long)j * kFwdKeys;
					if (use >= 1 && !mbar_wait(smem_u32(&k_empty[s]), (use - 1) & 1, p.err, kDevTimeoutAttn, abort_flag)) {
						ok = false;
						break;
					}
					mbar_arrive_expect_tx(smem_u32(&k_full[s]), parts * kFwdOpBytes);
					for (int hl = 0; hl < parts; ++hl)
						copy_kmajor(smem_u32(smem + s * kFwdSlotBytes + hl * kFwdOpBytes), kb, hl, p.Tpk, r0, kFwdKeys,
							smem_u32(&k_full[s]));
					if (use >= 1 && !mbar_wait(smem_u32(&v_empty[s]), (use - 1) & 1, p.err, kDevTimeoutAttn, abort_flag)) {
						ok = false;
						break;
					}
					mbar_arrive_expect_tx(smem_u32(&v_full[s]), parts * kFwdOpBytes);
					for (int hl = 0; hl < parts; ++hl)
						copy_mnmajor(smem_u32(smem + kFwdVBase + s * kFwdSlotBytes + hl * kFwdOpBytes), vb, hl, p.Tpk, r0,
							kFwdKeys, smem_u32(&v_full[s]));
				}
			}
			// every issued copy has landed before the CTA can exit (a V copy is issued after its K copy)
			for (int tt = max(0, t - kFwdSlots); tt < t; ++tt) {
				drain_wait(smem_u32(&k_full[tt % kFwdSlots]), (tt / kFwdSlots) & 1, p.err);
				drain_wait(smem_u32(&v_full[tt % kFwdSlots]), (tt / kFwdSlots) & 1, p.err);
			}
		}
	} else if (warp == 1) {
		// ---------------------------------- MMA issuer ----------------------------------
		const uint32_t id_s = idesc_tf32(kFwdRows, kFwdKeys);
		const uint32_t id_pv = idesc_tf32(kFwdRows, kDh) | kIdescBMajorMN;
		int t = 0, i = 0;
		bool ok = true;
		for (int w = blockIdx.x; ok && w < W; w += gridDim.x, ++i) {
			int q0, nh, J;
			fwd_item(p, w, q0, nh, J);
			// this item's Q is in tensor memory (written after the previous item's last score MMA)
			if (!warp_wait(smem_u32(&q_ready), i & 1, p.err, abort_flag)) break;
			tc_fence_after();
			for (int j = 0; j <= J; ++j) {
				if (j < J) {                       // S_t = Q K_t^T
					const int tt = t + j, s = tt % kFwdSlots;
					if (!warp_wait(smem_u32(&k_full[s]), (tt / kFwdSlots) & 1, p.err, abort_flag)) {
						ok = false;
						break;
					}
					tc_fence_after();
					const uint64_t kd = smem_desc_k_sw64(smem_u32(smem + s * kFwdSlotBytes));
					const uint32_t d = tmem + kFColS + (tt & 1) * 128;
#pragma unroll
					for (int ks = 0; ks < kDh / 8; ++ks) {
						const uint32_t ko = (ks >> 1) * (kFwdKeys * 64) + (ks & 1) * 32;
						mma_step<kSplit>(d, tmem + kFColQhi + ks * 8, tmem + kFColQlo + ks * 8, desc_at(kd, ko),
							desc_at(kd, kFwdOpBytes + ko), id_s, ks > 0);
					}
					mma_commit_elect(smem_u32(&s_full[tt & 1]));
					mma_commit_elect(smem_u32(&k_empty[s]));
				}
				if (j >= 1) {                      // O_t-1 part = P_t-1 V_t-1
					const int tp = t + j - 1, b = tp & 1, s = tp % kFwdSlots;
					if (!warp_wait(smem_u32(&p_full[b]), (tp >> 1) & 1, p.err, abort_flag) ||
							(tp >= 2 && !warp_wait(smem_u32(&pv_empty[b]), ((tp >> 1) - 1) & 1, p.err,
								abort_flag)) ||
							!warp_wait(smem_u32(&v_full[s]), (tp / kFwdSlots) & 1, p.err, abort_flag)) {
						ok = false;
						break;
					}
					tc_fence_after();
					const uint64_t vd = smem_desc_mn_sw128b32(smem_u32(smem + kFwdVBase + s * kFwdSlotBytes), kFwdKeys * 128);
					const uint32_t d = tmem + kFColPV + b * 64, pc = tmem + kFColS + b * 128;
#pragma unroll
					for (int ks = 0; ks < kFwdKeys / 8; ++ks)
						mma_step<kSplit>(d, pc + ks * 8, pc + 64 + ks * 8, desc_at(vd, ks * 1024),
							desc_at(vd, kFwdOpBytes + ks * 1024), id_pv, ks > 0);
					mma_commit_elect(smem_u32(&pv_full[b]));
					mma_commit_elect(smem_u32(&v_empty[s]));
				}
			}
			t += J;
		}
		// every issued MMA has completed before tensor memory is released
		mma_commit_elect(smem_u32(&drain));
		drain_wait(smem_u32(&drain), 0, p.err);
	} else {
		// ------------- softmax: kFwdParts threads per query row, kFwdCols key columns each -------------
		const int quad = warp & 3, part = (warp - 2) >> 2;
		const int row = quad * 32 + lane;
		const uint32_t lb = tmem + ((uint32_t)(quad * 32) << 16);
		const float c1 = p.scale * kLog2e;
		int t = 0, xuse = 0;
		auto exchange = [&](float v, float (&all)[kFwdParts]) -> bool {
			const int par = xuse & 1;
			const bool r = row_exchange(xval[par], part, row, v, all, smem_u32(&xbar[quad][par]), (xuse >> 1) & 1,
				p.err, abort_flag);
			++xuse;
			return r;
		};
		// this thread's kFwdHeadCols columns of the query row of item w (row index `row`), or null past Tq
		auto q_src = [&](int w) -> const float* {
			int q0w, nhw, Jw;
			fwd_item(p, w, q0w, nhw, Jw);
			if (q0w + row >= p.Tq) return nullptr;
			return p.q + ((long long)(nhw / p.H) * p.Tq + q0w + row) * p.D + (nhw % p.H) * kDh + part * kFwdHeadCols;
		};
		// Q of item w into tensor memory (zeros past Tq), then the MMA warp may issue its scores
		auto load_q = [&](int w) {
			const float* src = q_src(w);
			uint32_t hi[kFwdHeadCols], lo[kFwdHeadCols];
#pragma unroll
			for (int u = 0; u < kFwdHeadCols / 4; ++u) {
				const float4 x = src ? __ldg(reinterpret_cast<const float4*>(src) + u) : make_float4(0.f, 0.f, 0.f, 0.f);
				float4 h4, l4;
				split4(x, h4, l4);
				hi[4 * u] = __float_as_uint(h4.x); hi[4 * u + 1] = __float_as_uint(h4.y);
				hi[4 * u + 2] = __float_as_uint(h4.z); hi[4 * u + 3] = __float_as_uint(h4.w);
				lo[4 * u] = __float_as_uint(l4.x); lo[4 * u + 1] = __float_as_uint(l4.y);
				lo[4 * u + 2] = __float_as_uint(l4.z); lo[4 * u + 3] = __float_as_uint(l4.w);
			}
			tmem_st_32x32b_x16(lb + kFColQhi + part * kFwdHeadCols, hi);
			tmem_st_32x32b_x16(lb + kFColQlo + part * kFwdHeadCols, lo);
			tmem_wait_st();
			tc_fence_before();
			mbar_arrive(smem_u32(&q_ready));
		};
		if (blockIdx.x < W) load_q(blockIdx.x);
		bool ok = true;
		for (int w = blockIdx.x; ok && w < W; w += gridDim.x) {
			int q0, nh, J;
			fwd_item(p, w, q0, nh, J);
			const int n = nh / p.H, h = nh % p.H;
			const int qrow = q0 + row;
			const bool row_ok = qrow < p.Tq;
			const int wn = w + (int)gridDim.x;
			if (wn < W) {
				const float* nq = q_src(wn);
				if (nq) prefetch_l2(nq);
			}
			const float* padn = p.pad ? p.pad + (long long)n * p.Tk : nullptr;
			float m = -INFINITY, l = 0.0f, alpha_prev = 0.0f;
			float o[kFwdHeadCols];
#pragma unroll
			for (int c = 0; c < kFwdHeadCols; ++c) o[c] = 0.0f;
			// O = alpha O + PV_tt (this thread's head columns) for the finished tile tt
			auto fold = [&](int tt) -> bool {
				const int b = tt & 1;
				if (!warp_wait(smem_u32(&pv_full[b]), (tt >> 1) & 1, p.err, abort_flag)) return false;
				tc_fence_after();
				uint32_t r[kFwdHeadCols];
				tmem_ld_32x32b_x16(lb + kFColPV + b * 64 + part * kFwdHeadCols, r);
				tmem_wait_ld();
				// o * alpha + PV with one rounding, two columns per instruction
				const float2 av = make_float2(alpha_prev, alpha_prev);
#pragma unroll
				for (int c = 0; c < kFwdHeadCols; c += 2) {
					const float2 y = fma2_rn(make_float2(o[c], o[c + 1]), av,
						make_float2(__uint_as_float(r[c]), __uint_as_float(r[c + 1])));
					o[c] = y.x;
					o[c + 1] = y.y;
				}
				tc_fence_before();
				mbar_arrive(smem_u32(&pv_empty[b]));
				return true;
			};
			for (int j = 0; j < J; ++j) {
				const int tt = t + j, b = tt & 1;
				if (!warp_wait(smem_u32(&s_full[b]), (tt >> 1) & 1, p.err, abort_flag)) {
					ok = false;
					break;
				}
				tc_fence_after();
				float sv[kFwdCols];
				{
					uint32_t r[kFwdCols];
					tmem_ld_32x32b_x16(lb + kFColS + b * 128 + part * kFwdCols, r);
					tmem_wait_ld();
#pragma unroll
					for (int c = 0; c < kFwdCols; ++c) sv[c] = __uint_as_float(r[c]);
				}
				// tiles on the causal diagonal, past the last key, or under a padding mask take the
				// masked path (the same for every thread of the CTA)
				const int key0 = j * kFwdKeys + part * kFwdCols;
				const bool general =
					padn || (p.causal && j * kFwdKeys + kFwdKeys - 1 > q0) || (j * kFwdKeys + kFwdKeys > p.Tk);
				float mt = -INFINITY;
				uint32_t live = 0xffffffffu, padb = 0u;
				if (!general) {
#pragma unroll
					for (int c = 0; c < kFwdCols; ++c) mt = fmaxf(mt, sv[c]);
					mt = mt * p.scale;                 // scale > 0: the max of the scaled scores
				} else {
					live = live_bits32(key0, qrow, p.Tk, p.causal);
					padb = padded_bits32(padn, key0, live & ((1u << kFwdCols) - 1u));
#pragma unroll
					for (int c = 0; c < kFwdCols; ++c) {
						const bool lv = (live >> c) & 1u, pd = (padb >> c) & 1u;
						mt = fmaxf(mt, !lv ? -INFINITY : pd ? -1e9f : sv[c] * p.scale);
					}
				}
				float all[kFwdParts];
				if (!exchange(mt, all)) {
					ok = false;
					break;
				}
				const float m_new = fmaxf(m, fmaxf(fmaxf(all[0], all[1]), fmaxf(all[2], all[3])));
				const float alpha = exp2_hw((m - m_new) * kLog2e);     // 0 on the first tile (m = -inf)
				const float mlog = m_new * kLog2e;
				float sum = 0.0f;
				if (!general) {
					// the exponents' FMAs two columns at a time (packed fp32), the sum in column order
					const float2 c1v = make_float2(c1, c1), mv = make_float2(-mlog, -mlog);
#pragma unroll
					for (int c = 0; c < kFwdCols; c += 2) {
						const float2 x = fma2_rn(make_float2(sv[c], sv[c + 1]), c1v, mv);
						const float e0 = exp2_hw(x.x), e1 = exp2_hw(x.y);
						sv[c] = e0;
						sv[c + 1] = e1;
						sum += e0;
						sum += e1;
					}
				} else {
					// a padded key's exponent is formed from -1e9 - m, exact when the whole row is padded
					const float xpad = (-1e9f - m_new) * kLog2e;
					const float2 c1v = make_float2(c1, c1), mv = make_float2(-mlog, -mlog);
#pragma unroll
					for (int c = 0; c < kFwdCols; c += 2) {
						const float2 x = fma2_rn(make_float2(sv[c], sv[c + 1]), c1v, mv);
						const bool lv0 = (live >> c) & 1u, pd0 = (padb >> c) & 1u;
						const bool lv1 = (live >> (c + 1)) & 1u, pd1 = (padb >> (c + 1)) & 1u;
						const float e0 = !lv0 ? 0.0f : exp2_hw(pd0 ? xpad : x.x);
						const float e1 = !lv1 ? 0.0f : exp2_hw(pd1 ? xpad : x.y);
						sv[c] = e0;
						sv[c + 1] = e1;
						sum += e0;
						sum += e1;
					}
				}
				l = l * alpha + sum;
				m = m_new;
				vals_to_tmem16(sv, lb + kFColS + b * 128 + part * kFwdCols, lb + kFColS + b * 128 + 64 + part * kFwdCols);
				tmem_wait_st();
				tc_fence_before();
				mbar_arrive(smem_u32(&p_full[b]));
				// after the item's last tile every score MMA of the item has completed (s_full was
				// observed), so the next item's Q can replace this one while P V and the epilogue run
				if (j == J - 1 && wn < W) load_q(wn);
				if (j >= 1 && !fold(tt - 1)) {
					ok = false;
					break;
				}
				alpha_prev = alpha;
			}
			if (ok) ok = fold(t + J - 1);
			float ls[kFwdParts];
			if (ok) ok = exchange(l, ls);
			if (ok && row_ok) {
				// the row sum in part order: the same bits in every thread of the row
				const float lt = ((ls[0] + ls[1]) + ls[2]) + ls[3];
				const float inv_l = 1.0f / lt;
				float4* orow = reinterpret_cast<float4*>(p.out + ((long long)n * p.Tq + qrow) * p.D + h * kDh +
					part * kFwdHeadCols);
				const float2 il2 = make_float2(inv_l, inv_l);
#pragma unroll
				for (int u = 0; u < kFwdHeadCols / 4; ++u) {
					const float2 a = mul2_rn(make_float2(o[4 * u], o[4 * u + 1]), il2);
					const float2 b2 = mul2_rn(make_float2(o[4 * u + 2], o[4 * u + 3]), il2);
					orow[u] = make_float4(a.x, a.y, b2.x, b2.y);
				}
				if (part == 0) {
					// m and l are kept apart: with the reference's -1e9 padding scores, m + log(l) would
					// lose log(l) to rounding for a row whose keys are all padded
					p.stats[((long long)nh * p.Tq + qrow) * 2] = m;
					p.stats[((long long)nh * p.Tq + qrow) * 2 + 1] = lt;
				}
			}
			t += J;
		}
	}

	fa_release_tmem(tmem, warp);
}

// ---------------------------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------------------------
struct BwdParams {
	const float* pq_mn;  // Q, MN-major image, Tpq rows per head
	const float* pdo;    // dO (upstream gradient), K-major image, Tpq rows
	const float* pdo_mn; // dO, MN-major image
	const float* pq;     // Q, K-major image
	const float* pk;     // K, K-major image, Tpk rows
	const float* pk_mn;  // K, MN-major image
	const float* pv;     // V, K-major image
	const float* q;      // raw [N, Tq, D]
	const float* k;      // raw [N, Tk, D]
	const float* v;
	const float* dout;   // [N, Tq, D]
	const float* stats;  // [N, H, Tq, 2] from the forward
	const float* pad;    // [N, Tk] or null
	float* rowstat;      // [N*H][3][Tpq]: m, 1/l (this kernel) and D = rowsum(dO o O) (the pack)
	float* dq;
	float* dk;
	float* dv;
	int dq_first, dk_first, dv_first;
	int* err;
	long long D;
	int N, H, Tq, Tk, Tpq, Tpk, q_tiles, k_tiles, causal, split;
	float scale;
};

// Stores (first) or adds 32 values to a head row segment.
__device__ __forceinline__ void store32(float* dst, const uint32_t (&r)[32], int first) {
	float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
	for (int u = 0; u < 8; ++u) {
		float4 v = make_float4(__uint_as_float(r[4 * u]) + 0.0f, __uint_as_float(r[4 * u + 1]) + 0.0f,
			__uint_as_float(r[4 * u + 2]) + 0.0f, __uint_as_float(r[4 * u + 3]) + 0.0f);
		if (!first) {
			const float4 c = d4[u];
			v.x = c.x + v.x; v.y = c.y + v.y; v.z = c.z + v.z; v.w = c.w + v.w;
		}
		d4[u] = v;
	}
}

// -------- dQ kernel: 128 query rows per item, 64-key tiles streamed --------
// stage: K (K-major hi, lo) | V (K-major hi, lo) | K (MN-major hi, lo), 16 KB each
constexpr int kDqStages = 2;
constexpr uint32_t kDqStageBytes = 6 * kFwdOpBytes;
constexpr uint32_t kDqSmem = kDqStages * kDqStageBytes + 1024;
// tensor-memory columns: Q hi | Q lo | dO hi | dO lo | S/dS-hi | dS-lo | dP | dQ
constexpr uint32_t kQColQhi = 0, kQColQlo = 64, kQColOhi = 128, kQColOlo = 192, kQColS = 256, kQColSlo = 320,
	kQColP = 384, kQColAcc = 448;

__device__ __forceinline__ void dq_item(const BwdParams& p, int w, int& q0, int& nh, int& J) {
	nh = w / p.q_tiles;
	q0 = (p.q_tiles - 1 - w % p.q_tiles) * kFwdRows;
	const int key_end = p.causal ? min(q0 + kFwdRows, p.Tq) : p.Tk;
	J = (key_end + kFwdKeys - 1) / kFwdKeys;
}

// Four math warps per lane quarter here too, each thread a quarter of a row's columns: the per-tile math
// sits on the critical path between the score MMAs and the dQ MMAs.
constexpr int kDqParts = 4;
constexpr int kDqMathThreads = 32 * 4 * kDqParts;
constexpr int kDqThreads = 64 + kDqMathThreads;
constexpr int kDqCols = kFwdKeys / kDqParts;               // score columns per math thread (16)
constexpr int kDqHeadCols = kDh / kDqParts;                // head columns per math thread (16)

// 16 consecutive floats of a head row (zeros when !valid), split into hi and lo, stored to 16 columns
// each at taddr_hi / taddr_lo of this thread's tensor-memory lane.
__device__ __forceinline__ void row16_to_tmem(const float* src, bool valid, uint32_t taddr_hi, uint32_t taddr_lo) {
	uint32_t hi[16], lo[16];
#pragma unroll
	for (int u = 0; u < 4; ++u) {
		const float4 x = valid ? __ldg(reinterpret_cast<const float4*>(src) + u) : make_float4(0.f, 0.f, 0.f, 0.f);
		float4 h4, l4;
		split4(x, h4, l4);
		hi[4 * u] = __float_as_uint(h4.x); hi[4 * u + 1] = __float_as_uint(h4.y);
		hi[4 * u + 2] = __float_as_uint(h4.z); hi[4 * u + 3] = __float_as_uint(h4.w);
		lo[4 * u] = __float_as_uint(l4.x); lo[4 * u + 1] = __float_as_uint(l4.y);
		lo[4 * u + 2] = __float_as_uint(l4.z); lo[4 * u + 3] = __float_as_uint(l4.w);
	}
	tmem_st_32x32b_x16(taddr_hi, hi);
	tmem_st_32x32b_x16(taddr_lo, lo);
}

// Stores (first: value + 0) or adds 16 values to a head row segment.
__device__ __forceinline__ void store16(float* dst, const uint32_t (&r)[16], int first) {
	float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
	for (int u = 0; u < 4; ++u) {
		float4 v = make_float4(__uint_as_float(r[4 * u]) + 0.0f, __uint_as_float(r[4 * u + 1]) + 0.0f,
			__uint_as_float(r[4 * u + 2]) + 0.0f, __uint_as_float(r[4 * u + 3]) + 0.0f);
		if (!first) {
			const float4 c = d4[u];
			v.x = c.x + v.x; v.y = c.y + v.y; v.z = c.z + v.z; v.w = c.w + v.w;
		}
		d4[u] = v;
	}
}

template <int kSplit>
__global__ void __launch_bounds__(kDqThreads, 1) flash_bwd_dq_kernel(const BwdParams p) {
	extern __shared__ uint8_t smem_raw[];
	uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
	__shared__ __align__(8) uint64_t kv_full[kDqStages], kv_empty[kDqStages], sdp_full, ds_full, acc_full, q_ready,
		drain;
	__shared__ uint32_t tmem_base_sh;
	__shared__ int abort_sh;

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int W = p.N * p.H * p.q_tiles;
	if (threadIdx.x == 0) {
		for (int s = 0; s < kDqStages; ++s) {
			mbar_init(smem_u32(&kv_full[s]), 1);
			mbar_init(smem_u32(&kv_empty[s]), 1);
		}
		mbar_init(smem_u32(&sdp_full), 1);
		mbar_init(smem_u32(&ds_full), kDqMathThreads);
		mbar_init(smem_u32(&acc_full), 1);
		mbar_init(smem_u32(&q_ready), kDqMathThreads);
		mbar_init(smem_u32(&drain), 1);
		abort_sh = 0;
		fence_mbar_init();
	}
	const uint32_t tmem = fa_setup_tmem(&tmem_base_sh, warp);
	volatile int* abort_flag = &abort_sh;
	constexpr int parts = kSplit ? 2 : 1;

	if (warp == 0) {
		if (lane == 0) {
			int t = 0;
			bool ok = true;
			for (int w = blockIdx.x; ok && w < W; w += gridDim.x) {
				int q0, nh, J;
				dq_item(p, w, q0, nh, J);
				const long long img = (long long)nh * packed_head_floats(p.Tpk);
				for (int j = 0; j < J; ++j, ++t) {
					const int s = t % kDqStages, use = t / kDqStages;
					if (use >= 1 &&
							!mbar_wait(smem_u32(&kv_empty[s]), (use - 1) & 1, p.err, kDevTimeoutAttn, abort_flag)) {
						ok = false;
						break;
					}
					const uint32_t fb = smem_u32(&kv_full[s]);
					mbar_arrive_expect_tx(fb, parts * 3 * kFwdOpBytes);
					const uint32_t dst = smem_u32(smem + s * kDqStageBytes);
					const long long r0 = (long long)j * kFwdKeys;
					for (int hl = 0; hl < parts; ++hl) {
						copy_kmajor(dst + hl * kFwdOpBytes, p.pk + img, hl, p.Tpk, r0, kFwdKeys, fb);
						copy_kmajor(dst + 2 * kFwdOpBytes + hl * kFwdOpBytes, p.pv + img, hl, p.Tpk, r0, kFwdKeys, fb);
						copy_mnmajor(dst + 4 * kFwdOpBytes + hl * kFwdOpBytes, p.pk_mn + img, hl, p.Tpk, r0, kFwdKeys, fb);
					}
				}
			}
			for (int tt = max(0, t - kDqStages); tt < t; ++tt)
				drain_wait(smem_u32(&kv_full[tt % kDqStages]), (tt / kDqStages) & 1, p.err);
		}
	} else if (warp == 1) {
		const uint32_t id_s = idesc_tf32(kFwdRows, kFwdKeys);
		const uint32_t id_dq = idesc_tf32(kFwdRows, kDh) | kIdescBMajorMN;
		int t = 0, i = 0;
		bool ok = true;
		for (int w = blockIdx.x; ok && w < W; w += gridDim.x, ++i) {
			int q0, nh, J;
			dq_item(p, w, q0, nh, J);
			if (!warp_wait(smem_u32(&q_ready), i & 1, p.err, abort_flag)) break;
			tc_fence_after();
			for (int j = 0; j < J; ++j) {
				const int tt = t + j, s = tt % kDqStages;
				if (!warp_wait(smem_u32(&kv_full[s]), (tt / kDqStages) & 1, p.err, abort_flag)) {
					ok = false;
					break;
				}
				tc_fence_after();
				const uint32_t kbase = smem_u32(smem + s * kDqStageBytes);
				const uint64_t kd = smem_desc_k_sw64(kbase), vd = smem_desc_k_sw64(kbase + 2 * kFwdOpBytes);
				const uint64_t kmd = smem_desc_mn_sw128b32(kbase + 4 * kFwdOpBytes, kFwdKeys * 128);
				// S = Q K^T and dP = dO V^T, their depth steps interleaved: two independent accumulator
				// chains keep the tensor pipe busy while one step's result feeds the next of its chain
#pragma unroll
				for (int ks = 0; ks < kDh / 8; ++ks) {
					const uint32_t off = (ks >> 1) * (kFwdKeys * 64) + (ks & 1) * 32;
					mma_step<kSplit>(tmem + kQColS, tmem + kQColQhi + ks * 8, tmem + kQColQlo + ks * 8, desc_at(kd, off),
						desc_at(kd, kFwdOpBytes + off), id_s, ks > 0);
					mma_step<kSplit>(tmem + kQColP, tmem + kQColOhi + ks * 8, tmem + kQColOlo + ks * 8, desc_at(vd, off),
						desc_at(vd, kFwdOpBytes + off), id_s, ks > 0);
				}
				mma_commit_elect(smem_u32(&sdp_full));
				if (!warp_wait(smem_u32(&ds_full), tt & 1, p.err, abort_flag)) {
					ok = false;
					break;
				}
				tc_fence_after();
#pragma unroll
				for (int ks = 0; ks < kFwdKeys / 8; ++ks)   // dQ += dS K
					mma_step<kSplit>(tmem + kQColAcc, tmem + kQColS + ks * 8, tmem + kQColSlo + ks * 8,
						desc_at(kmd, ks * 1024), desc_at(kmd, kFwdOpBytes + ks * 1024), id_dq, (j > 0 || ks > 0));
				mma_commit_elect(smem_u32(&kv_empty[s]));
			}
			if (!ok) break;
			mma_commit_elect(smem_u32(&acc_full));
			t += J;
		}
		mma_commit_elect(smem_u32(&drain));
		drain_wait(smem_u32(&drain), 0, p.err);
	} else {
		// ------------- score gradients: kDqParts threads per query row, kDqCols key columns each -------------
		const int quad = warp & 3, part = (warp - 2) >> 2;
		const int row = quad * 32 + lane;
		const uint32_t lb = tmem + ((uint32_t)(quad * 32) << 16);
		const float c1 = p.scale * kLog2e;
		int t = 0, i = 0;
		bool ok = true;
		for (int w = blockIdx.x; ok && w < W; w += gridDim.x, ++i) {
			int q0, nh, J;
			dq_item(p, w, q0, nh, J);
			const int n = nh / p.H, h = nh % p.H;
			const int qrow = q0 + row;
			const bool row_ok = qrow < p.Tq;
			const long long roff = ((long long)n * p.Tq + (row_ok ? qrow : 0)) * p.D + h * kDh + part * kDqHeadCols;
			// this item's Q and dO rows go to tensor memory (the previous item's MMAs have all
			// completed: its dQ was read after acc_full); the next item's rows are prefetched to L2
			row16_to_tmem(p.q + roff, row_ok, lb + kQColQhi + part * kDqHeadCols, lb + kQColQlo + part * kDqHeadCols);
			row16_to_tmem(p.dout + roff, row_ok, lb + kQColOhi + part * kDqHeadCols, lb + kQColOlo + part * kDqHeadCols);
			if (w + (int)gridDim.x < W) {
				int nq0, nnh, nJ;
				dq_item(p, w + gridDim.x, nq0, nnh, nJ);
				const int nn = nnh / p.H, nhh = nnh % p.H;
				if (nq0 + row < p.Tq) {
					const long long noff = ((long long)nn * p.Tq + nq0 + row) * p.D + nhh * kDh + part * kDqHeadCols;
					prefetch_l2(p.q + noff);
					prefetch_l2(p.dout + noff);
				}
			}
			tmem_wait_st();
			tc_fence_before();
			mbar_arrive(smem_u32(&q_ready));
			// the row's statistics (not needed by the MMAs, so loaded after the hand-off)
			float* rs = p.rowstat + (long long)nh * 3 * p.Tpq;
			float mrow = 0.0f, inv_l = 1.0f;
			const float drow = rs[2 * p.Tpq + qrow];
			if (row_ok) {
				mrow = p.stats[((long long)nh * p.Tq + qrow) * 2];
				inv_l = 1.0f / p.stats[((long long)nh * p.Tq + qrow) * 2 + 1];
			}
			if (part == 0) {
				// rows past Tq get neutral statistics (m 0, 1/l 1; D is 0): their Q and dO rows are zero
				rs[qrow] = mrow;
				rs[p.Tpq + qrow] = inv_l;
			}

			const float* padn = p.pad ? p.pad + (long long)n * p.Tk : nullptr;
			const float mlog = mrow * kLog2e;
			for (int j = 0; j < J; ++j) {
				const int tt = t + j;
				if (!warp_wait(smem_u32(&sdp_full), tt & 1, p.err, abort_flag)) {
					ok = false;
					break;
				}
				tc_fence_after();
				uint32_t rsv[kDqCols], rp[kDqCols];
				tmem_ld_32x32b_x16(lb + kQColS + part * kDqCols, rsv);
				tmem_ld_32x32b_x16(lb + kQColP + part * kDqCols, rp);
				tmem_wait_ld();
				const int key0 = j * kFwdKeys + part * kDqCols;
				const bool general =
					padn || (p.causal && j * kFwdKeys + kFwdKeys - 1 > q0) || (j * kFwdKeys + kFwdKeys > p.Tk);
				float ds[kDqCols];
				if (!general) {
					// the same operations as the masked form below, two columns per packed instruction
					const float2 c1v = make_float2(c1, c1), mv = make_float2(-mlog, -mlog), ilv = make_float2(inv_l, inv_l),
						dv = make_float2(-drow, -drow), sc = make_float2(p.scale, p.scale);
#pragma unroll
					for (int c = 0; c < kDqCols; c += 2) {
						const float2 x = fma2_rn(make_float2(__uint_as_float(rsv[c]), __uint_as_float(rsv[c + 1])), c1v, mv);
						const float2 pr = mul2_rn(make_float2(exp2_hw(x.x), exp2_hw(x.y)), ilv);
						const float2 t2 = add2_rn(make_float2(__uint_as_float(rp[c]), __uint_as_float(rp[c + 1])), dv);
						const float2 d2 = mul2_rn(sc, mul2_rn(pr, t2));
						ds[c] = d2.x;
						ds[c + 1] = d2.y;
					}
				} else {
					const uint32_t live = (row_ok ? live_bits32(key0, qrow, p.Tk, p.causal) : 0u) & ((1u << kDqCols) - 1u);
					const uint32_t use = live & ~padded_bits32(padn, key0, live);
					const float2 c1v = make_float2(c1, c1), mv = make_float2(-mlog, -mlog), ilv = make_float2(inv_l, inv_l),
						dv = make_float2(-drow, -drow), sc = make_float2(p.scale, p.scale);
#pragma unroll
					for (int c = 0; c < kDqCols; c += 2) {
						const float2 x = fma2_rn(make_float2(__uint_as_float(rsv[c]), __uint_as_float(rsv[c + 1])), c1v, mv);
						const float2 pr = mul2_rn(make_float2(exp2_hw(x.x), exp2_hw(x.y)), ilv);
						const float2 t2 = add2_rn(make_float2(__uint_as_float(rp[c]), __uint_as_float(rp[c + 1])), dv);
						const float2 d2 = mul2_rn(sc, mul2_rn(pr, t2));
						ds[c] = ((use >> c) & 1u) ? d2.x : 0.0f;
						ds[c + 1] = ((use >> (c + 1)) & 1u) ? d2.y : 0.0f;
					}
				}
				vals_to_tmem16(ds, lb + kQColS + part * kDqCols, lb + kQColSlo + part * kDqCols);
				tmem_wait_st();
				tc_fence_before();
				mbar_arrive(smem_u32(&ds_full));
			}
			if (ok) ok = warp_wait(smem_u32(&acc_full), i & 1, p.err, abort_flag);
			if (ok) {
				tc_fence_after();
				uint32_t r[kDqHeadCols];
				tmem_ld_32x32b_x16(lb + kQColAcc + part * kDqHeadCols, r);
				tmem_wait_ld();
				if (row_ok && p.dq) store16(p.dq + roff, r, p.dq_first);
			}
			t += J;
		}
	}

	fa_release_tmem(tmem, warp);
}

// -------- dKdV kernel: 128 keys per item, 32-query tiles streamed --------
constexpr int kKvRows = 128;                                   // keys per item (MMA M)
constexpr int kKvQ = 32;                                       // queries per tile
constexpr int kKvStages = 3;
// stage: Q K-major (hi, lo) | dO K-major (hi, lo) | Q MN-major (hi, lo) | dO MN-major (hi, lo), 8 KB
// each, then m[32], 1/l[32], D[32] of the tile's queries
constexpr uint32_t kKvOpBytes = kPanels * kKvQ * 64;
constexpr uint32_t kKvStatOff = 8 * kKvOpBytes;
constexpr uint32_t kKvStageBytes = 8 * kKvOpBytes + 1024;      // keeps every stage 1024-byte aligned
constexpr uint32_t kKvSmem = kKvStages * kKvStageBytes + 1024;
// tensor-memory columns: K hi | K lo | V hi | V lo | S^T/P^T-hi | P^T-lo | dP^T/dS^T-hi | dS^T-lo | dV | dK
constexpr uint32_t kKColKhi = 0, kKColKlo = 64, kKColVhi = 128, kKColVlo = 192, kKColS = 256, kKColSlo = 288,
	kKColP = 320, kKColPlo = 352, kKColDv = 384, kKColDk = 448;

// Work item w -> (sample, head) and key tile (causal: the first key tiles see the most queries and
// go first), and the range of 32-query tiles it streams; a head's key tiles are consecutive items.
__device__ __forceinline__ void kv_item(const BwdParams& p, int w, int& k0, int& nh, int& qt_begin, int& J) {
	nh = w / p.k_tiles;
	k0 = (w % p.k_tiles) * kKvRows;
	const int qt_end = (p.Tq + kKvQ - 1) / kKvQ;
	qt_begin = p.causal ? min(k0 / kKvQ, qt_end) : 0;
	J = qt_end - qt_begin;
}

// Four math warps per lane quarter, each thread a quarter of a tile's 32 query columns (8).
constexpr int kKvParts = 4;
constexpr int kKvMathThreads = 32 * 4 * kKvParts;
constexpr int kKvThreads = 64 + kKvMathThreads;
constexpr int kKvCols = kKvQ / kKvParts;                   // query columns per math thread (8)

// Splits 8 values (|v| < 2^128 / 8193) and stores hi / lo to two column groups of this thread's lane.
__device__ __forceinline__ void vals_to_tmem8(const float (&v)[8], uint32_t taddr_hi, uint32_t taddr_lo) {
	uint32_t hi[8], lo[8];
	split_pairs<8>(v, hi, lo);
	tmem_st_32x32b_x8(taddr_hi, hi);
	tmem_st_32x32b_x8(taddr_lo, lo);
}

template <int kSplit>
__global__ void __launch_bounds__(kKvThreads, 1) flash_bwd_dkdv_kernel(const BwdParams p) {
	extern __shared__ uint8_t smem_raw[];
	uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
	__shared__ __align__(8) uint64_t q_full[kKvStages], q_empty[kKvStages], sdp_full, pds_full, acc_full, kv_ready,
		drain;
	__shared__ uint32_t tmem_base_sh;
	__shared__ int abort_sh;

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int W = p.N * p.H * p.k_tiles;
	if (threadIdx.x == 0) {
		for (int s = 0; s < kKvStages; ++s) {
			mbar_init(smem_u32(&q_full[s]), 1);
			mbar_init(smem_u32(&q_empty[s]), 1);
		}
		mbar_init(smem_u32(&sdp_full), 1);
		mbar_init(smem_u32(&pds_full), kKvMathThreads);
		mbar_init(smem_u32(&acc_full), 1);
		mbar_init(smem_u32(&kv_ready), kKvMathThreads);
		mbar_init(smem_u32(&drain), 1);
		abort_sh = 0;
		fence_mbar_init();
	}
	const uint32_t tmem = fa_setup_tmem(&tmem_base_sh, warp);
	volatile int* abort_flag = &abort_sh;
	constexpr int parts = kSplit ? 2 : 1;

	if (warp == 0) {
		if (lane == 0) {
			int t = 0;
			bool ok = true;
			for (int w = blockIdx.x; ok && w < W; w += gridDim.x) {
				int k0, nh, qt_begin, J;
				kv_item(p, w, k0, nh, qt_begin, J);
				const long long img = (long long)nh * packed_head_floats(p.Tpq);
				const float* st = p.rowstat + (long long)nh * 3 * p.Tpq;
				for (int j = 0; j < J; ++j, ++t) {
					const int s = t % kKvStages, use = t / kKvStages;
					if (use >= 1 &&
							!mbar_wait(smem_u32(&q_empty[s]), (use - 1) & 1, p.err, kDevTimeoutAttn, abort_flag)) {
						ok = false;
						break;
					}
					const uint32_t fb = smem_u32(&q_full[s]);
					mbar_arrive_expect_tx(fb, parts * 4 * kKvOpBytes + 3 * kKvQ * 4);
					const uint32_t dst = smem_u32(smem + s * kKvStageBytes);
					const long long r0 = (long long)(qt_begin + j) * kKvQ;
					for (int hl = 0; hl < parts; ++hl) {
						copy_kmajor(dst + hl * kKvOpBytes, p.pq + img, hl, p.Tpq, r0, kKvQ, fb);
						copy_kmajor(dst + 2 * kKvOpBytes + hl * kKvOpBytes, p.pdo + img, hl, p.Tpq, r0, kKvQ, fb);
						copy_mnmajor(dst + 4 * kKvOpBytes + hl * kKvOpBytes, p.pq_mn + img, hl, p.Tpq, r0, kKvQ, fb);
						copy_mnmajor(dst + 6 * kKvOpBytes + hl * kKvOpBytes, p.pdo_mn + img, hl, p.Tpq, r0, kKvQ, fb);
					}
					for (int wd = 0; wd < 3; ++wd)
						bulk_load(dst + kKvStatOff + wd * kKvQ * 4, st + wd * p.Tpq + r0, kKvQ * 4, fb);
				}
			}
			for (int tt = max(0, t - kKvStages); tt < t; ++tt)
				drain_wait(smem_u32(&q_full[tt % kKvStages]), (tt / kKvStages) & 1, p.err);
		}
	} else if (warp == 1) {
		const uint32_t id_s = idesc_tf32(kKvRows, kKvQ);
		const uint32_t id_acc = idesc_tf32(kKvRows, kDh) | kIdescBMajorMN;
		int t = 0, i = 0;
		bool ok = true;
		for (int w = blockIdx.x; ok && w < W; w += gridDim.x, ++i) {
			int k0, nh, qt_begin, J;
			kv_item(p, w, k0, nh, qt_begin, J);
			if (!warp_wait(smem_u32(&kv_ready), i & 1, p.err, abort_flag)) break;
			tc_fence_after();
			for (int j = 0; j < J; ++j) {
				const int tt = t + j, s = tt % kKvStages;
				if (!warp_wait(smem_u32(&q_full[s]), (tt / kKvStages) & 1, p.err, abort_flag)) {
					ok = false;
					break;
				}
				tc_fence_after();
				const uint32_t qbase = smem_u32(smem + s * kKvStageBytes);
				const uint64_t qd = smem_desc_k_sw64(qbase), od = smem_desc_k_sw64(qbase + 2 * kKvOpBytes);
				const uint64_t qmd = smem_desc_mn_sw128b32(qbase + 4 * kKvOpBytes, kKvQ * 128);
				const uint64_t omd = smem_desc_mn_sw128b32(qbase + 6 * kKvOpBytes, kKvQ * 128);
				// S^T = K Q^T and dP^T = V dO^T, depth steps interleaved (two independent chains)
#pragma unroll
				for (int ks = 0; ks < kDh / 8; ++ks) {
					const uint32_t off = (ks >> 1) * (kKvQ * 64) + (ks & 1) * 32;
					mma_step<kSplit>(tmem + kKColS, tmem + kKColKhi + ks * 8, tmem + kKColKlo + ks * 8, desc_at(qd, off),
						desc_at(qd, kKvOpBytes + off), id_s, ks > 0);
					mma_step<kSplit>(tmem + kKColP, tmem + kKColVhi + ks * 8, tmem + kKColVlo + ks * 8, desc_at(od, off),
						desc_at(od, kKvOpBytes + off), id_s, ks > 0);
				}
				mma_commit_elect(smem_u32(&sdp_full));
				if (!warp_wait(smem_u32(&pds_full), tt & 1, p.err, abort_flag)) {
					ok = false;
					break;
				}
				tc_fence_after();
#pragma unroll
				for (int ks = 0; ks < kKvQ / 8; ++ks) {
					const uint32_t acc = (j > 0 || ks > 0);
					// dV += P^T dO
					mma_step<kSplit>(tmem + kKColDv, tmem + kKColS + ks * 8, tmem + kKColSlo + ks * 8, desc_at(omd, ks * 1024),
						desc_at(omd, kKvOpBytes + ks * 1024), id_acc, acc);
					// dK += dS^T Q
					mma_step<kSplit>(tmem + kKColDk, tmem + kKColP + ks * 8, tmem + kKColPlo + ks * 8, desc_at(qmd, ks * 1024),
						desc_at(qmd, kKvOpBytes + ks * 1024), id_acc, acc);
				}
				mma_commit_elect(smem_u32(&q_empty[s]));
			}
			if (!ok) break;
			mma_commit_elect(smem_u32(&acc_full));
			t += J;
		}
		mma_commit_elect(smem_u32(&drain));
		drain_wait(smem_u32(&drain), 0, p.err);
	} else {
		// ------------- P^T and dS^T: kKvParts threads per key row, kKvCols query columns each -------------
		const int quad = warp & 3, part = (warp - 2) >> 2;
		const int row = quad * 32 + lane;
		const uint32_t lb = tmem + ((uint32_t)(quad * 32) << 16);
		const float c1 = p.scale * kLog2e;
		int t = 0, i = 0;
		bool ok = true;
		for (int w = blockIdx.x; ok && w < W; w += gridDim.x, ++i) {
			int k0, nh, qt_begin, J;
			kv_item(p, w, k0, nh, qt_begin, J);
			const int n = nh / p.H, h = nh % p.H;
			const int key = k0 + row;
			const bool key_ok = key < p.Tk;
			const long long roff = ((long long)n * p.Tk + (key_ok ? key : 0)) * p.D + h * kDh;
			// this item's K and V rows go to tensor memory (the previous item's MMAs have all
			// completed: its dK / dV were read after acc_full); the next item's rows go to L2
			const int hc = part * (kDh / kKvParts);
			row16_to_tmem(p.k + roff + hc, key_ok, lb + kKColKhi + hc, lb + kKColKlo + hc);
			row16_to_tmem(p.v + roff + hc, key_ok, lb + kKColVhi + hc, lb + kKColVlo + hc);
			if (w + (int)gridDim.x < W) {
				int nk0, nnh, nqb, nJ;
				kv_item(p, w + gridDim.x, nk0, nnh, nqb, nJ);
				const int nn = nnh / p.H, nhh = nnh % p.H;
				if (nk0 + row < p.Tk) {
					const long long noff = ((long long)nn * p.Tk + nk0 + row) * p.D + nhh * kDh + hc;
					prefetch_l2(p.k + noff);
					prefetch_l2(p.v + noff);
				}
			}
			tmem_wait_st();
			tc_fence_before();
			mbar_arrive(smem_u32(&kv_ready));

			const bool padded = p.pad && key_ok && p.pad[(long long)n * p.Tk + key] == 0.0f;
			for (int j = 0; j < J; ++j) {
				const int tt = t + j, s = tt % kKvStages;
				// the stage's m / (1/l) / D words were written by the bulk copy: observe its barrier too
				if (!warp_wait(smem_u32(&q_full[s]), (tt / kKvStages) & 1, p.err, abort_flag) ||
						!warp_wait(smem_u32(&sdp_full), tt & 1, p.err, abort_flag)) {
					ok = false;
					break;
				}
				tc_fence_after();
				const float* m_j = reinterpret_cast<const float*>(smem + s * kKvStageBytes + kKvStatOff) + part * kKvCols;
				const float* il_j = m_j + kKvQ;
				const float* d_j = m_j + 2 * kKvQ;
				const int qbeg = (qt_begin + j) * kKvQ + part * kKvCols;
				uint32_t rs[kKvCols], rp[kKvCols];
				tmem_ld_32x32b_x8(lb + kKColS + part * kKvCols, rs);
				tmem_ld_32x32b_x8(lb + kKColP + part * kKvCols, rp);
				tmem_wait_ld();
				// queries past Tq have zero Q / dO rows and neutral statistics, keys past Tk zero K / V
				// rows (their dK / dV rows are not stored): only the causal diagonal and padding need masks
				const bool general = padded || (p.causal && k0 + kKvRows - 1 > (qt_begin + j) * kKvQ);
				float pr[kKvCols], ds[kKvCols];
				if (!general) {
					// the same operations as the masked form below, two columns per packed instruction
					const float2 c1v = make_float2(c1, c1), l2e = make_float2(kLog2e, kLog2e), sc = make_float2(p.scale, p.scale);
#pragma unroll
					for (int c = 0; c < kKvCols; c += 2) {
						const float2 ml = mul2_rn(make_float2(m_j[c], m_j[c + 1]), l2e);
						const float2 x = fma2_rn(make_float2(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1])), c1v,
							make_float2(-ml.x, -ml.y));
						const float2 pv = mul2_rn(make_float2(exp2_hw(x.x), exp2_hw(x.y)), make_float2(il_j[c], il_j[c + 1]));
						const float2 t2 = add2_rn(make_float2(__uint_as_float(rp[c]), __uint_as_float(rp[c + 1])),
							make_float2(-d_j[c], -d_j[c + 1]));
						const float2 d2 = mul2_rn(sc, mul2_rn(pv, t2));
						pr[c] = pv.x;
						pr[c + 1] = pv.y;
						ds[c] = d2.x;
						ds[c + 1] = d2.y;
					}
				} else {
					const float2 c1v = make_float2(c1, c1), l2e = make_float2(kLog2e, kLog2e), sc = make_float2(p.scale, p.scale);
#pragma unroll
					for (int c = 0; c < kKvCols; c += 2) {
						const bool live0 = !p.causal || key <= qbeg + c, live1 = !p.causal || key <= qbeg + c + 1;
						float2 x;
						if (padded) {
							x = mul2_rn(add2_rn(make_float2(-1e9f, -1e9f), make_float2(-m_j[c], -m_j[c + 1])), l2e);
						} else {
							const float2 ml = mul2_rn(make_float2(m_j[c], m_j[c + 1]), l2e);
							x = fma2_rn(make_float2(__uint_as_float(rs[c]), __uint_as_float(rs[c + 1])), c1v,
								make_float2(-ml.x, -ml.y));
						}
						const float2 pv = mul2_rn(make_float2(exp2_hw(x.x), exp2_hw(x.y)), make_float2(il_j[c], il_j[c + 1]));
						const float2 t2 = add2_rn(make_float2(__uint_as_float(rp[c]), __uint_as_float(rp[c + 1])),
							make_float2(-d_j[c], -d_j[c + 1]));
						const float2 d2 = mul2_rn(sc, mul2_rn(pv, t2));
						pr[c] = live0 ? pv.x : 0.0f;
						pr[c + 1] = live1 ? pv.y : 0.0f;
						ds[c] = (live0 && !padded) ? d2.x : 0.0f;
						ds[c + 1] = (live1 && !padded) ? d2.y : 0.0f;
					}
				}
				vals_to_tmem8(pr, lb + kKColS + part * kKvCols, lb + kKColSlo + part * kKvCols);
				vals_to_tmem8(ds, lb + kKColP + part * kKvCols, lb + kKColPlo + part * kKvCols);
				tmem_wait_st();
				tc_fence_before();
				mbar_arrive(smem_u32(&pds_full));
			}
			if (ok) ok = warp_wait(smem_u32(&acc_full), i & 1, p.err, abort_flag);
			if (ok) {
				tc_fence_after();
				// parts 0, 1 write dV, parts 2, 3 dK: 32 of the 64 columns each
				float* dst = part < 2 ? p.dv : p.dk;
				const int first = part < 2 ? p.dv_first : p.dk_first;
				const int hh = part & 1;
				const uint32_t col = (part < 2 ? kKColDv : kKColDk) + hh * 32;
				uint32_t r[32];
				tmem_ld_32x32b_x32(lb + col, r);
				tmem_wait_ld();
				if (key_ok && dst) store32(dst + roff + hh * 32, r, first);
			}
			t += J;
		}
	}

	fa_release_tmem(tmem, warp);
}

}  // namespace

static std::mutex g_fa_mutex;
static bool g_fa_attr[64];

static nnb_status fa_set_attrs(int dev) {
	std::lock_guard<std::mutex> lock(g_fa_mutex);
	if (g_fa_attr[dev & 63]) return NNB_OK;
	NNB_CUDA_TRY(cudaFuncSetAttribute(flash_fwd_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem));
	NNB_CUDA_TRY(cudaFuncSetAttribute(flash_fwd_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem));
	NNB_CUDA_TRY(cudaFuncSetAttribute(flash_bwd_dq_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kDqSmem));
	NNB_CUDA_TRY(cudaFuncSetAttribute(flash_bwd_dq_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kDqSmem));
	NNB_CUDA_TRY(cudaFuncSetAttribute(flash_bwd_dkdv_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kKvSmem));
	NNB_CUDA_TRY(cudaFuncSetAttribute(flash_bwd_dkdv_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kKvSmem));
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
	// item counts and in-head float offsets stay inside 32-bit integers
	const unsigned long long items = (unsigned long long)N * heads * ((std::max(Tq, Tk) + kRowAlign - 1) / kRowAlign);
	if (Tq > (1u << 20) || Tk > (1u << 20) || items >= (1ull << 31))
		return fail(NNB_ERR_UNSUPPORTED, "flash attention: problem too large (N %zu, Tq %zu, Tk %zu, heads %zu)", N, Tq,
			Tk, heads);
	return NNB_OK;
}

static nnb_status fa_pack(cudaStream_t s, int count, const PackSet& ps, long long NH, int H, long long D, int with_lo) {
	TraceScope ts(s, kTracePack);
	int most = 0;
	for (int t = 0; t < count; ++t) most = std::max(most, ps.Tp[t]);
	const dim3 grid((unsigned)(most * 16 / 256), (unsigned)std::min<long long>(NH, 65535), (unsigned)count);
	attn_pack_kernel<<<grid, 256, 0, s>>>(ps, (int)NH, H, D, with_lo);
	return cuda_status(cudaGetLastError(), "attention pack launch");
}

static unsigned persistent_grid(long long items, int sm_count) {
	return (unsigned)std::max<long long>(1, std::min<long long>(items, sm_count));
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
	const long long Tpq = nnb::round_up((long long)Tq, nnb::kRowAlign), Tpk = nnb::round_up((long long)Tk, nnb::kRowAlign);
	const long long fk = NH * nnb::packed_head_floats(Tpk);
	void* ws = nullptr;
	NNB_TRY(nnb::scratch_alloc(&ws, (size_t)(2 * fk) * sizeof(float), s));
	float* pk = static_cast<float*>(ws);
	float* pv = pk + fk;
	nnb_status st = NNB_OK;
	do {
		nnb::PackSet ps{};
		ps.src[0] = k; ps.kdst[0] = pk; ps.T[0] = (int)Tk; ps.Tp[0] = (int)Tpk;       // S = Q K^T
		ps.src[1] = v; ps.mdst[1] = pv; ps.T[1] = (int)Tk; ps.Tp[1] = (int)Tpk;       // O += P V
		if ((st = nnb::fa_pack(s, 2, ps, NH, (int)heads, (long long)D, split)) != NNB_OK) break;
		nnb::FwdParams p{};
		p.q = q; p.pk = pk; p.pv = pv; p.pad = key_padding_mask; p.out = out; p.stats = stats;
		p.err = dev->error_word;
		p.D = (long long)D; p.N = (int)N; p.H = (int)heads; p.Tq = (int)Tq; p.Tk = (int)Tk;
		p.Tpk = (int)Tpk;
		p.q_tiles = (int)((Tq + nnb::kFwdRows - 1) / nnb::kFwdRows);
		p.causal = causal ? 1 : 0; p.split = split;
		p.scale = 1.0f / std::sqrt(static_cast<float>(nnb::kDh));     // ops.cpp:1236
		nnb::TraceScope ts(s, nnb::kTraceAttention);
		const unsigned grid = nnb::persistent_grid(NH * p.q_tiles, dev->sm_count);
		if (split) nnb::flash_fwd_kernel<1><<<grid, nnb::kFwdThreads, nnb::kFwdSmem, s>>>(p);
		else nnb::flash_fwd_kernel<0><<<grid, nnb::kFwdThreads, nnb::kFwdSmem, s>>>(p);
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
		ps.dot_with[1] = out; ps.dot_out[1] = rowstat + 2 * Tpq; ps.dot_stride[1] = 3 * Tpq;   // D = rowsum(dO o O)
		ps.src[2] = k; ps.kdst[2] = pk; ps.mdst[2] = pk_mn; ps.T[2] = (int)Tk; ps.Tp[2] = (int)Tpk;
		ps.src[3] = v; ps.kdst[3] = pv; ps.T[3] = (int)Tk; ps.Tp[3] = (int)Tpk;
		if ((st = nnb::fa_pack(s, 4, ps, NH, (int)heads, (long long)D, split)) != NNB_OK) break;
		nnb::BwdParams p{};
		p.pq = pq; p.pq_mn = pq_mn; p.pdo = pdo; p.pdo_mn = pdo_mn; p.pk = pk; p.pk_mn = pk_mn; p.pv = pv;
		p.q = q; p.k = k; p.v = v; p.dout = g; p.stats = stats; p.pad = key_padding_mask;
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
		// the dQ kernel also writes the m, 1/l statistics the dKdV kernel reads
		const unsigned gq = nnb::persistent_grid(NH * p.q_tiles, dev->sm_count);
		if (split) nnb::flash_bwd_dq_kernel<1><<<gq, nnb::kDqThreads, nnb::kDqSmem, s>>>(p);
		else nnb::flash_bwd_dq_kernel<0><<<gq, nnb::kDqThreads, nnb::kDqSmem, s>>>(p);
		if ((st = nnb::cuda_status(cudaGetLastError(), "flash attention dQ launch")) != NNB_OK) break;
		if (dk || dv) {
			const unsigned gk = nnb::persistent_grid(NH * p.k_tiles, dev->sm_count);
			if (split) nnb::flash_bwd_dkdv_kernel<1><<<gk, nnb::kKvThreads, nnb::kKvSmem, s>>>(p);
			else nnb::flash_bwd_dkdv_kernel<0><<<gk, nnb::kKvThreads, nnb::kKvSmem, s>>>(p);
			st = nnb::cuda_status(cudaGetLastError(), "flash attention dKdV launch");
		}
	} while (0);
	nnb_status st2 = nnb::scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

}  // extern "C"
