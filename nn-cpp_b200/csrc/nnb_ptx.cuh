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

}  // namespace nnb
