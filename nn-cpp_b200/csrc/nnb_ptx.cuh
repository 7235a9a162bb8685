// nnb_ptx.cuh -- thin inline-PTX wrappers for the sm_100a features the kernels use:
// mbarriers, TMA tensor copies (no multicast anywhere), tcgen05 MMA / TMEM, and bounded waits.
//
// Every wait on an mbarrier is bounded by wall-clock time (%globaltimer). When the bound is hit
// the waiter records an error code in the caller's device error word and returns false, so no
// kernel in this library can spin forever.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace nnb {

// Status codes written into the device error word (first writer wins).
enum DeviceError : int {
	kDevOk = 0,
	kDevTimeoutFull = 1,      // consumer waited too long for a TMA stage
	kDevTimeoutEmpty = 2,     // producer waited too long for a free stage
	kDevTimeoutAccum = 3,     // epilogue waited too long for an accumulator
	kDevTimeoutAccumFree = 4, // MMA issuer waited too long for an accumulator to drain
	kDevTimeoutAttn = 5,      // a fused-attention role waited too long for another role
	kDevTimeoutDrain = 6,     // a CTA waited too long for its own copies / MMAs before exiting
};

// Upper bound on any single mbarrier wait: 2 s. A healthy wait is a few microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
	return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
	uint64_t t;
	asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
	return t;
}

__device__ __forceinline__ void record_error(int* err, int code) {
	if (err) atomicCAS(err, 0, code);
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
	asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
	asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
	asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
		"r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
	asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// 4-byte asynchronous copy global -> shared (L1-allocating); src_bytes 0 writes a zero instead of
// reading (the source address is then not dereferenced but must still be a valid pointer).
__device__ __forceinline__ void cp_async_4(uint32_t smem_dst, const void* src, uint32_t src_bytes) {
	asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Waits until at most N of this thread's committed copy groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Orders this thread's ordinary shared-memory stores before later reads of that memory by the async
// proxy (tensor-core operand reads): each writing thread fences, then signals the MMA issuer.
__device__ __forceinline__ void fence_proxy_async_smem() {
	asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
	uint32_t ok;
	asm volatile(
		"{\n\t.reg .pred p;\n\t"
		"mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
		"selp.u32 %0, 1, 0, p;\n\t}"
		: "=r"(ok)
		: "r"(bar), "r"(parity)
		: "memory");
	return ok != 0;
}

// Waits for the phase with the given parity to complete. Returns false (after recording `code`)
// if that takes longer than kWaitLimitNs, or if *abort is already set by another role.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code,
		volatile int* abort) {
	if (mbar_try_wait(bar, parity)) return true;
	const uint64_t t0 = global_timer_ns();
	for (uint32_t i = 1;; ++i) {
		if (mbar_try_wait(bar, parity)) return true;
		if ((i & 255u) == 0) {
			if (abort && *abort) return false;
			if (global_timer_ns() - t0 > kWaitLimitNs) {
				record_error(err, code);
				if (abort) *abort = 1;
				return false;
			}
		}
	}
}

// mbar_wait by every lane of a converged warp, with a warp-uniform result (false if any lane's wait
// gave up), for roles whose whole warp runs the loop.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, int* err, int code, volatile int* abort) {
	return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, code, abort));
}

// ---------------------------------------------------------------------------------------------
// TMA (bulk tensor copies, global -> shared, completion counted on an mbarrier). No multicast.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
	asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t smem_dst, const void* tmap, uint32_t bar,
		int32_t x, int32_t y) {
	asm volatile(
		"cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
		" [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_dst),
		"l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar)
		: "memory");
}

// The same for a 5-D tensor map, coordinates innermost first.
__device__ __forceinline__ void tma_load_5d(uint32_t smem_dst, const void* tmap, uint32_t bar,
		int32_t c0, int32_t c1, int32_t c2, int32_t c3, int32_t c4) {
	asm volatile(
		"cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
		" [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(smem_dst),
		"l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(bar)
		: "memory");
}

// ---------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads, fences
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t smem_result, uint32_t ncols) {
	asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_result),
		"r"(ncols) : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
	asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
	asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
		: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
	asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
	asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::tf32, issued by one thread.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
		uint32_t idesc, uint32_t accumulate) {
	asm volatile(
		"{\n\t.reg .pred p;\n\t"
		"setp.ne.b32 p, %4, 0;\n\t"
		"tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
		"l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
		: "memory");
}

// Arrives once on the mbarrier when every tcgen05 op issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
	asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
		: "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
	asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives lane (base + t).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
	asm volatile(
		"tcgen05.ld.sync.aligned.32x32b.x32.b32 "
		"{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
		"%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
		: "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
		"=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
		"=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
		"=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
		"=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
		: "r"(taddr)
		: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored as rows of 64 bytes with the
// 64-byte swizzle (the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_64B): 8-row core groups
// 512 bytes apart (stride byte offset), descriptor version 1, layout type 4 (SWIZZLE_64B).
// The tile base must be 512-byte aligned; `byte_offset` moves along K inside the 64-byte row.
__device__ __forceinline__ uint64_t smem_desc_k_sw64(uint32_t smem_addr) {
	uint64_t d = 0;
	d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);   // start address, 16-byte units
	d |= (uint64_t)(512u >> 4) << 32;               // stride byte offset
	d |= (uint64_t)1 << 46;                         // descriptor version (sm_100)
	d |= (uint64_t)4 << 61;                         // SWIZZLE_64B
	return d;
}

// Instruction descriptor for kind::tf32: F32 accumulator, TF32 A and B, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
	return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Instruction-descriptor bit selecting an MN-major B operand (N contiguous for each k).
constexpr uint32_t kIdescBMajorMN = 1u << 16;
// The same for A (M contiguous for each k).
constexpr uint32_t kIdescAMajorMN = 1u << 15;

// Shared-memory descriptor for an MN-major 32-bit (tf32) operand. The one layout tcgen05 offers for
// MN-major 32-bit operands is the 128-byte swizzle with 32-byte atoms (layout type 1): each 128-byte
// row holds 32 consecutive N elements of one k, its four 32-byte chunks permuted as chunk c at
// c ^ (k & 3); 4 k-rows form a 512-byte group (stride byte offset 512 to the next group) and the
// next 32 N elements sit `lbo_bytes` further on (leading byte offset). One tf32 MMA step (K = 8)
// reads two groups, so the k step moves the start by 1024 bytes.
__device__ __forceinline__ uint64_t smem_desc_mn_sw128b32(uint32_t smem_addr, uint32_t lbo_bytes) {
	uint64_t d = 0;
	d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
	d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
	d |= (uint64_t)(512u >> 4) << 32;
	d |= (uint64_t)1 << 46;
	d |= (uint64_t)1 << 61;                         // SWIZZLE_128B_BASE32B
	return d;
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::tf32, with A (M rows x K) read from tensor memory:
// row i in lane i, K consecutive 32-bit columns starting at a_tmem's column.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
		uint32_t idesc, uint32_t accumulate) {
	asm volatile(
		"{\n\t.reg .pred p;\n\t"
		"setp.ne.b32 p, %4, 0;\n\t"
		"tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
		"r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
		: "memory");
}

// Warp-collective forms of the MMA and commit: every lane of a converged warp executes them with the
// same (warp-uniform) operands and the lane that elect.sync picks -- always the lowest, so the same
// lane for every call -- issues the instruction. A role that runs its whole loop this way keeps its
// descriptors and tensor-memory addresses warp-uniform: measured with clock stamps in the attention
// kernels, issuing took about 50 cycles per MMA from a loop run by one lane of a diverged warp and
// about 25-30 from the whole warp -- the tensor core needs about 16-32 cycles for a 128 x 32..64 x 8
// tf32 MMA, so the one-lane loop, not the tensor core, set the pace.
__device__ __forceinline__ void mma_tf32_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
		uint32_t accumulate) {
	asm volatile(
		"{\n\t.reg .pred p, e;\n\t"
		"elect.sync _|e, 0xffffffff;\n\t"
		"setp.ne.b32 p, %4, 0;\n\t"
		"@e tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
		"l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
		: "memory");
}
__device__ __forceinline__ void mma_tf32_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
		uint32_t accumulate) {
	asm volatile(
		"{\n\t.reg .pred p, e;\n\t"
		"elect.sync _|e, 0xffffffff;\n\t"
		"setp.ne.b32 p, %4, 0;\n\t"
		"@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
		"r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
		: "memory");
}
__device__ __forceinline__ void mma_commit_elect(uint32_t bar) {
	asm volatile(
		"{\n\t.reg .pred e;\n\t"
		"elect.sync _|e, 0xffffffff;\n\t"
		"@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
		: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp writes lane (base + t).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
	asm volatile(
		"tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
		"{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
		"%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
		"r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
		"r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
		"r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
		"r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
		"r"(r[29]), "r"(r[30]), "r"(r[31])
		: "memory");
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
	asm volatile(
		"tcgen05.ld.sync.aligned.32x32b.x16.b32 "
		"{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
		: "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
		"=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
		"=r"(r[14]), "=r"(r[15])
		: "r"(taddr)
		: "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
	asm volatile(
		"tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
		"{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
		"r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
		"r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
		"r"(r[15])
		: "memory");
}

// 32 lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
	asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
		: "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
		: "r"(taddr)
		: "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x8(uint32_t taddr, const uint32_t (&r)[8]) {
	asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
		"r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
		: "memory");
}

// Barrier over `count` threads (a multiple of 32) with id 1..15; id 0 is __syncthreads.
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
	asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// 2^x with the hardware base-2 exponential (ex2.approx: relative error about 2^-22; 2^-inf = +0).
__device__ __forceinline__ float exp2_hw(float x) {
	float y;
	asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
	return y;
}

__device__ __forceinline__ void tmem_wait_st() {
	asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Plain (untiled) bulk copy global -> this CTA's shared memory, completion counted on an
// mbarrier. Both addresses 16-byte aligned, size a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_load(uint32_t smem_dst, const void* src, uint32_t bytes, uint32_t bar) {
	asm volatile(
		"cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_dst),
		"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
		: "memory");
}

// TF32 rounding (round to nearest, ties away) and the 3xTF32 split x ~= hi + lo.
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

// Packed fp32 pairs (the f32x2 instructions of sm_100: one instruction for two lanes' operations),
// round to nearest. A multiply whose result feeds an add is not guaranteed to stay two roundings
// (measured: a packed GELU built from such pairs, or from the __fmul2_rn / __fadd2_rn intrinsics, did
// not reproduce the separately rounded scalar results bit for bit), so code that needs two roundings
// does not rely on a mul2_rn -> add2_rn pair: it writes the fused form explicitly or avoids the pattern.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
	float2 d;
	asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
	    "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
	    : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
	return d;
}

__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
	float2 d;
	asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
	    "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
	    : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
	return d;
}

// d = a * b + c with one rounding per lane
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
	float2 d;
	asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
	    "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
	    : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
	return d;
}

}  // namespace nnb
