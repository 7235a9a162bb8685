// rng.cu -- the library's random streams (src/random.cpp) and inverted dropout (src/nn/dropout.cpp).
//
// Host side: the seeding registry. manual_seed(seed) fixes a base and resets the per-stream
// counters; the k-th derive_generator(name) after it seeds an mt19937 from
// splitmix64(base ^ fnv1a(name) ^ k * golden-ratio) split into two 32-bit words fed through a
// seed_seq, exactly as src/random.cpp:67-79 does, so a given seed yields the reference's streams.
// seed_seq::generate and mt19937's seed(seed_seq&) follow their definitions in the C++ standard
// ([rand.util.seedseq], [rand.eng.mers]); SplitMix64 (Steele, Lea & Flood 2014) and FNV-1a 64
// (Fowler, Noll & Vo) are the published functions.
//
// Device side: one generator state = 624 untempered words + the index of the next word to temper
// (625 uint32 in HBM), so successive draws continue the stream across launches and inside CUDA
// graphs. A draw of n outputs is two launches per 2^24 outputs: ONE CTA advances the twist, read as
// the linear recurrence it is, 454 words per barrier (227 threads, two chained words each) and
// streams the raw words out; then a grid-wide kernel tempers them, compares with p and packs one
// keep word per 32 outputs (warp ballot). The stream is serial by definition (the reference draws
// output i for element i in row-major order); the masks are 1 bit per element (the reference keeps
// a float per element).
//
// Dropout (dropout.cpp:20-31): u = float(x >> 8) * 2^-24 per element, dropped when u < p, kept
// elements scaled by 1/(1-p); p == 1 drops everything without drawing, p == 0 keeps everything
// without drawing.
#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <random>
#include <string>
#include <utility>

#include "nnb_internal.h"
#include "nnb_trace.h"

namespace nnb {

namespace {

constexpr int kMtN = 624;
constexpr int kMtShift = 397;
constexpr int kMtHalf = kMtN - kMtShift;     // 227: words before this index read only old words
constexpr uint32_t kMtMatrix = 0x9908b0dfu;

// ---- host: seed_seq + mt19937 seeding ------------------------------------------------------------

// seed_seq{seeds...}.generate(out, out + n) per [rand.util.seedseq]
void seed_seq_generate(const uint32_t* seeds, size_t s, uint32_t* out, size_t n) {
	for (size_t i = 0; i < n; i++) out[i] = 0x8b8b8b8bu;
	const size_t t = n >= 623 ? 11 : n >= 68 ? 7 : n >= 39 ? 5 : n >= 7 ? 3 : (n - 1) / 2;
	const size_t p = (n - t) / 2, q = p + t, m = std::max(s + 1, n);
	auto T = [](uint32_t x) { return x ^ (x >> 27); };
	for (size_t k = 0; k < m; k++) {
		const uint32_t r1 = 1664525u * T(out[k % n] ^ out[(k + p) % n] ^ out[(k + n - 1) % n]);
		uint32_t r2 = r1;
		if (k == 0) r2 += static_cast<uint32_t>(s);
		else if (k <= s) r2 += static_cast<uint32_t>(k % n) + seeds[k - 1];
		else r2 += static_cast<uint32_t>(k % n);
		out[(k + p) % n] += r1;
		out[(k + q) % n] += r2;
		out[k % n] = r2;
	}
	for (size_t k = m; k < m + n; k++) {
		const uint32_t r3 = 1566083941u * T(out[k % n] + out[(k + p) % n] + out[(k + n - 1) % n]);
		const uint32_t r4 = r3 - static_cast<uint32_t>(k % n);
		out[(k + p) % n] ^= r3;
		out[(k + q) % n] ^= r4;
		out[k % n] = r4;
	}
}

// mt19937::seed(seed_seq&) per [rand.eng.mers]: the 624 generated words are the state; an all-zero
// state (ignoring the low 31 bits of word 0) becomes 2^31 in word 0. The index starts at 624, so
// the first draw twists.
void mt_seed_from_seq(const uint32_t* seeds, size_t s, uint32_t* state) {
	seed_seq_generate(seeds, s, state, kMtN);
	bool zero = (state[0] & 0x80000000u) == 0;
	for (int i = 1; i < kMtN && zero; i++) zero = state[i] == 0;
	if (zero) state[0] = 0x80000000u;
	state[kMtN] = kMtN;
}

uint64_t splitmix64(uint64_t x) {
	x += 0x9e3779b97f4a7c15ull;
	x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
	x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
	return x ^ (x >> 31);
}

uint64_t fnv1a64(const char* s) {
	uint64_t h = 0xcbf29ce484222325ull;
	for (; *s; ++s) h = (h ^ static_cast<unsigned char>(*s)) * 0x100000001b3ull;
	return h;
}

struct Registry {
	std::mutex mu;
	bool seeded = false, has_base = false;
	uint64_t base = 0, epoch = 0;
	std::map<std::string, uint64_t> counters;
};

Registry& registry() {
	static Registry r;
	return r;
}

// ---- host: mt19937 draws, the portable shuffle and weighted draws (src/data/shuffle.hpp,
// src/data/dataloader.cpp:58-73) -------------------------------------------------------------------

uint32_t host_mix(uint32_t upper_of, uint32_t lower_of) {
	const uint32_t y = (upper_of & 0x80000000u) | (lower_of & 0x7fffffffu);
	return (y >> 1) ^ ((y & 1u) ? kMtMatrix : 0u);
}

uint32_t host_next(uint32_t* st) {
	if (st[kMtN] >= (uint32_t)kMtN) {
		for (int i = 0; i < kMtN; i++) st[i] = st[(i + kMtShift) % kMtN] ^ host_mix(st[i], st[(i + 1) % kMtN]);
		st[kMtN] = 0;
	}
	uint32_t y = st[st[kMtN]++];
	y ^= y >> 11;
	y ^= (y << 7) & 0x9d2c5680u;
	y ^= (y << 15) & 0xefc60000u;
	return y ^ (y >> 18);
}

// uniform in [0, bound) by rejecting the incomplete top bucket of 2^32 (shuffle.hpp:25-33)
uint32_t bounded(uint32_t* st, uint32_t bound) {
	const uint64_t limit = (uint64_t{1} << 32) - ((uint64_t{1} << 32) % bound);
	uint32_t r = host_next(st);
	while (r >= limit) r = host_next(st);
	return r % bound;
}

// ---- device: mt19937 blocks and the keep mask ----------------------------------------------------

__device__ __forceinline__ uint32_t mt_mix(uint32_t upper_of, uint32_t lower_of) {
	const uint32_t y = (upper_of & 0x80000000u) | (lower_of & 0x7fffffffu);
	return (y >> 1) ^ ((y & 1u) ? kMtMatrix : 0u);
}

__device__ __forceinline__ uint32_t mt_temper(uint32_t y) {
	y ^= y >> 11;
	y ^= (y << 7) & 0x9d2c5680u;
	y ^= (y << 15) & 0xefc60000u;
	return y ^ (y >> 18);
}

// The stream as one sequence: X[0..623] = the state's words, and for j >= 624
//   X[j] = X[j - 227] ^ mix(X[j - 624], X[j - 623]),
// which is exactly the twist (block b+1's word i reads block b's words i, i+1, i+397 for i < 227 and
// block b+1's word i-227 above). Output o of a draw that starts at state index p is temper(X[p + o]).
// Every word depends only on words at least 227 back, so a round computes 454 new words: thread
// t < 227 makes X[f + t] and then X[f + t + 227] (which needs X[f + t] -- its own register -- and
// words 396 / 397 back, all older than the round); one barrier per round. X lives in a 2048-word
// shared ring. This serial part only streams the raw words X[p .. p + n) to global memory; tempering,
// the comparison with p and the bit packing run afterwards over the whole GPU.
constexpr int kRing = 2048;
constexpr int kRound = 2 * kMtHalf;              // 454 words per round
constexpr int kStreamThreads = 256;
constexpr unsigned long long kChunk = 1ull << 24;  // outputs per serial launch (64 MB of raw words)

// Outputs o in [w0, w1) of this launch's n go to raw[o - w0]; the others only advance the state (a
// rank that needs a slice of a longer draw still runs the whole serial stream).
__global__ void __launch_bounds__(kStreamThreads, 1) mt_stream_kernel(uint32_t* __restrict__ state,
		unsigned long long n, uint32_t* __restrict__ raw, unsigned long long w0, unsigned long long w1) {
	__shared__ uint32_t ring[kRing];
	const int t = threadIdx.x;
	for (int i = t; i < kMtN; i += kStreamThreads) ring[i] = state[i];
	const unsigned long long p0 = state[kMtN] > (uint32_t)kMtN ? (unsigned long long)kMtN : state[kMtN];
	__syncthreads();
	const unsigned long long end = p0 + n, last = end - 1;                // outputs are X[p0 .. end)
	const unsigned long long block0 = (last / kMtN) * kMtN, need = block0 + kMtN;
	const unsigned long long lo = p0 + w0, hi = p0 + (w1 < n ? w1 : n);   // X[lo .. hi) are written
	for (unsigned long long i = lo + t; i < hi && i < (unsigned long long)kMtN; i += kStreamThreads)
		raw[i - lo] = ring[i];
	for (unsigned long long frontier = kMtN; frontier < need; frontier += kRound) {
		if (t < kMtHalf) {
			const unsigned long long j = frontier + t, j2 = j + kMtHalf;
			const uint32_t x1 = ring[(j - kMtHalf) & (kRing - 1)] ^
				mt_mix(ring[(j - kMtN) & (kRing - 1)], ring[(j - kMtN + 1) & (kRing - 1)]);
			const uint32_t x2 = x1 ^ mt_mix(ring[(j - kMtShift) & (kRing - 1)], ring[(j - kMtShift + 1) & (kRing - 1)]);
			ring[j & (kRing - 1)] = x1;
			ring[j2 & (kRing - 1)] = x2;
			if (j >= lo && j < hi) raw[j - lo] = x1;
			if (j2 >= lo && j2 < hi) raw[j2 - lo] = x2;
		}
		__syncthreads();
	}
	for (int i = t; i < kMtN; i += kStreamThreads) state[i] = ring[(block0 + i) & (kRing - 1)];
	if (t == 0) state[kMtN] = (uint32_t)(last - block0 + 1);
}

// keep[w] bit b = output 32w + b kept: temper(x) >> 8 >= threshold, where threshold = ceil(p * 2^24)
// makes the integer test equal to the reference's float test u = float(x >> 8) * 2^-24 < p (both
// sides are exact: x >> 8 < 2^24 and p * 2^24 only rescales p).
__global__ void keep_pack_kernel(const uint32_t* __restrict__ raw, unsigned long long n, uint32_t threshold,
		uint32_t* __restrict__ keep) {
	const int lane = threadIdx.x & 31;
	const unsigned long long warps = (unsigned long long)gridDim.x * (blockDim.x >> 5);
	const unsigned long long words = (n + 31) / 32;
	for (unsigned long long w = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) >> 5; w < words;
			w += warps) {
		const unsigned long long e = 32 * w + lane;
		const bool kept = e < n && (mt_temper(raw[e]) >> 8) >= threshold;
		const uint32_t word = __ballot_sync(0xffffffffu, kept);
		if (lane == 0) keep[w] = word;
	}
}

__device__ __forceinline__ float keep_factor(const uint32_t* keep, unsigned long long i, float scale) {
	return ((keep[i >> 5] >> (i & 31)) & 1u) ? scale : 0.0f;
}

// y = x * m, m = kept ? scale : 0 (mul, ops.cpp:347 on the mask tensor)
__global__ void dropout_apply_kernel(unsigned long long n, float scale, const float* __restrict__ x,
		const uint32_t* __restrict__ keep, float* __restrict__ y) {
	const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
	for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < n; i += stride)
		y[i] = x[i] * keep_factor(keep, i, scale);
}

// dx (first: =, else +=) g * m, with the grad_accum convention (ops.cpp:67-73)
__global__ void dropout_bwd_kernel(unsigned long long n, float scale, const float* __restrict__ g,
		const uint32_t* __restrict__ keep, float* __restrict__ dx, int first) {
	const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
	for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < n; i += stride) {
		const float v = g[i] * keep_factor(keep, i, scale);
		dx[i] = first ? v + 0.0f : dx[i] + v;
	}
}

nnb_status elementwise_grid(unsigned long long n, unsigned* blocks) {
	DeviceState* ds = nullptr;
	NNB_TRY(device_state(&ds));
	const unsigned long long want = (n + 255) / 256, cap = (unsigned long long)ds->sm_count * 8;
	*blocks = (unsigned)(want < cap ? want : cap);
	return NNB_OK;
}

nnb_status check_p(float p) {
	if (!(p >= 0.0f && p <= 1.0f)) return fail(NNB_ERR_INVALID, "dropout: p must be in [0, 1] (got %g)", (double)p);
	return NNB_OK;
}

}  // namespace

float dropout_keep_scale(float p) { return p < 1.0f ? 1.0f / (1.0f - p) : 0.0f; }

nnb_status dropout_mask_slice(cudaStream_t s, uint32_t* state, size_t total, size_t offset, size_t count, float p,
		uint32_t* keep) {
	NNB_TRY(check_p(p));
	if (offset > total || count > total - offset)
		return fail(NNB_ERR_INVALID, "dropout_mask: slice [%zu, +%zu) outside %zu draws", offset, count, total);
	if (offset % 32) return fail(NNB_ERR_UNSUPPORTED, "dropout_mask: slice offset %zu not a multiple of 32", offset);
	if (total == 0) return NNB_OK;
	if (!state || (count && !keep)) return fail(NNB_ERR_INVALID, "dropout_mask: null pointer");
	const size_t words = (count + 31) / 32;
	TraceScope ts(s, kTraceRowwise);
	if (p == 0.0f || p == 1.0f)        // nothing is drawn (dropout.cpp:20-23)
		return count ? cuda_status(cudaMemsetAsync(keep, p == 0.0f ? 0xff : 0, words * sizeof(uint32_t), s),
			"dropout mask fill") : NNB_OK;
	const double scaled = std::ceil(static_cast<double>(p) * 16777216.0);    // exact: p * 2^24 <= 2^24
	const uint32_t threshold = static_cast<uint32_t>(scaled);
	void* ws = nullptr;
	const size_t chunk = count < kChunk ? count : (size_t)kChunk;
	NNB_TRY(scratch_alloc(&ws, (chunk ? chunk : 1) * sizeof(uint32_t), s));
	uint32_t* raw = static_cast<uint32_t*>(ws);
	DeviceState* dev = nullptr;
	nnb_status st = device_state(&dev);
	// chunks of the whole draw are multiples of 32 outputs; the slice's part of each is tempered and
	// packed at its bit position in `keep`
	for (size_t g0 = 0; st == NNB_OK && g0 < total; g0 += kChunk) {
		const size_t c = total - g0 < kChunk ? total - g0 : (size_t)kChunk;
		// this chunk's part of the slice, [lo_g, hi_g) in output numbers (empty when they do not meet)
		const size_t lo_g = offset > g0 ? offset : g0;
		const size_t hi_g = offset + count < g0 + c ? offset + count : g0 + c;
		const bool some = lo_g < hi_g;
		const size_t a = some ? lo_g - g0 : 0, b = some ? hi_g - g0 : 0;
		if (b > c || b - a > chunk) {              // the window always fits the chunk and the raw buffer
			st = fail(NNB_ERR_INVALID, "dropout_mask: internal slice window [%zu, %zu) of %zu", a, b, c);
			break;
		}
		mt_stream_kernel<<<1, kStreamThreads, 0, s>>>(state, (unsigned long long)c, raw, a, b);
		if (some) {
			const unsigned long long wn = (unsigned long long)(b - a);
			unsigned blocks = (unsigned)(((wn + 31) / 32 + 7) / 8);
			const unsigned cap = (unsigned)dev->sm_count * 16;
			if (blocks > cap) blocks = cap;
			keep_pack_kernel<<<blocks, 256, 0, s>>>(raw, wn, threshold, keep + (lo_g - offset) / 32);
		}
		st = cuda_status(cudaGetLastError(), "dropout_mask launch");
	}
	nnb_status st2 = scratch_free(ws, s);
	return st != NNB_OK ? st : st2;
}

nnb_status dropout_mask(cudaStream_t s, uint32_t* state, size_t n, float p, uint32_t* keep) {
	return dropout_mask_slice(s, state, n, 0, n, p, keep);
}

}  // namespace nnb

extern "C" {

void nnb_manual_seed(uint64_t seed) {
	nnb::Registry& r = nnb::registry();
	std::lock_guard<std::mutex> lock(r.mu);
	r.seeded = r.has_base = true;
	r.base = seed;
	r.epoch++;
	r.counters.clear();
}

int nnb_is_seeded(void) {
	nnb::Registry& r = nnb::registry();
	std::lock_guard<std::mutex> lock(r.mu);
	return r.seeded ? 1 : 0;
}

uint64_t nnb_seed_epoch(void) {
	nnb::Registry& r = nnb::registry();
	std::lock_guard<std::mutex> lock(r.mu);
	return r.epoch;
}

nnb_status nnb_derive_generator(const char* stream_name, uint32_t* state) {
	if (!stream_name || !state) return nnb::fail(NNB_ERR_INVALID, "derive_generator: null pointer");
	nnb::Registry& r = nnb::registry();
	uint64_t s;
	{
		std::lock_guard<std::mutex> lock(r.mu);
		if (!r.has_base) {           // unseeded: a nondeterministic base, taken once
			std::random_device rd;
			r.base = (static_cast<uint64_t>(rd()) << 32) ^ rd();
			r.has_base = true;
		}
		const uint64_t k = r.counters[stream_name]++;
		s = nnb::splitmix64(r.base ^ nnb::fnv1a64(stream_name) ^ (k * 0x9e3779b97f4a7c15ull));
	}
	const uint32_t seeds[2] = {static_cast<uint32_t>(s), static_cast<uint32_t>(s >> 32)};
	nnb::mt_seed_from_seq(seeds, 2, state);
	return NNB_OK;
}

nnb_status nnb_mt19937_seed_seq(const uint32_t* seeds, size_t count, uint32_t* state) {
	if ((count && !seeds) || !state) return nnb::fail(NNB_ERR_INVALID, "mt19937_seed_seq: null pointer");
	nnb::mt_seed_from_seq(seeds, count, state);
	return NNB_OK;
}

nnb_status nnb_mt19937_seed(uint32_t seed, uint32_t* state) {
	if (!state) return nnb::fail(NNB_ERR_INVALID, "mt19937_seed: null pointer");
	state[0] = seed;          // the published linear initialisation (init_genrand; [rand.eng.mers])
	for (int i = 1; i < nnb::kMtN; i++) state[i] = 1812433253u * (state[i - 1] ^ (state[i - 1] >> 30)) + (uint32_t)i;
	state[nnb::kMtN] = nnb::kMtN;
	return NNB_OK;
}

nnb_status nnb_mt19937_next(uint32_t* state, size_t n, uint32_t* out) {
	if (!state || (n && !out)) return nnb::fail(NNB_ERR_INVALID, "mt19937_next: null pointer");
	for (size_t i = 0; i < n; i++) out[i] = nnb::host_next(state);
	return NNB_OK;
}

uint64_t nnb_fnv1a64(const char* s) { return s ? nnb::fnv1a64(s) : 0; }

uint64_t nnb_splitmix64(uint64_t x) { return nnb::splitmix64(x); }

nnb_status nnb_portable_shuffle(uint32_t* state, uint64_t* v, size_t n) {
	if (!state || (n && !v)) return nnb::fail(NNB_ERR_INVALID, "portable_shuffle: null pointer");
	if (n > 0xFFFFFFFFull) return nnb::fail(NNB_ERR_INVALID, "portable_shuffle: more than 2^32 elements");
	for (size_t i = n; i > 1; i--) std::swap(v[i - 1], v[nnb::bounded(state, (uint32_t)i)]);
	return NNB_OK;
}

nnb_status nnb_weighted_draws(uint32_t* state, const double* cumulative, size_t count, size_t num_samples,
		uint64_t* out) {
	if (!state || !cumulative || count == 0 || (num_samples && !out))
		return nnb::fail(NNB_ERR_INVALID, "weighted_draws: null pointer or no weights");
	const double total = cumulative[count - 1];
	for (size_t s = 0; s < num_samples; s++) {
		// 53 random bits from two outputs: a uniform double in [0, 1), then the first running sum above it
		const uint64_t a = nnb::host_next(state) >> 5, b = nnb::host_next(state) >> 6;
		const double u = (static_cast<double>(a) * 67108864.0 + static_cast<double>(b)) / 9007199254740992.0;
		const double target = u * total;
		size_t lo = 0, hi = count;
		while (lo < hi) {
			const size_t mid = lo + (hi - lo) / 2;
			if (cumulative[mid] > target) hi = mid;
			else lo = mid + 1;
		}
		out[s] = lo < count ? lo : count - 1;
	}
	return NNB_OK;
}

nnb_status nnb_dropout_mask(void* stream, uint32_t* state, size_t n, float p, uint32_t* keep) {
	return nnb::dropout_mask(static_cast<cudaStream_t>(stream), state, n, p, keep);
}

nnb_status nnb_dropout_mask_slice(void* stream, uint32_t* state, size_t total, size_t offset, size_t count, float p,
		uint32_t* keep) {
	return nnb::dropout_mask_slice(static_cast<cudaStream_t>(stream), state, total, offset, count, p, keep);
}

nnb_status nnb_dropout_apply(void* stream, size_t n, float p, const float* x, const uint32_t* keep, float* y) {
	NNB_TRY(nnb::check_p(p));
	if (n == 0) return NNB_OK;
	if (!x || !keep || !y) return nnb::fail(NNB_ERR_INVALID, "dropout_apply: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	unsigned blocks;
	NNB_TRY(nnb::elementwise_grid(n, &blocks));
	nnb::TraceScope ts(s, nnb::kTraceRowwise);
	nnb::dropout_apply_kernel<<<blocks, 256, 0, s>>>(n, nnb::dropout_keep_scale(p), x, keep, y);
	return nnb::cuda_status(cudaGetLastError(), "dropout_apply launch");
}

nnb_status nnb_dropout_bwd(void* stream, size_t n, float p, const float* g, const uint32_t* keep, float* dx,
		int dx_first) {
	NNB_TRY(nnb::check_p(p));
	if (n == 0) return NNB_OK;
	if (!g || !keep || !dx) return nnb::fail(NNB_ERR_INVALID, "dropout_bwd: null pointer");
	cudaStream_t s = static_cast<cudaStream_t>(stream);
	unsigned blocks;
	NNB_TRY(nnb::elementwise_grid(n, &blocks));
	nnb::TraceScope ts(s, nnb::kTraceRowwise);
	nnb::dropout_bwd_kernel<<<blocks, 256, 0, s>>>(n, nnb::dropout_keep_scale(p), g, keep, dx, dx_first);
	return nnb::cuda_status(cudaGetLastError(), "dropout_bwd launch");
}

}  // extern "C"
