// trace.cu -- per-kernel device timing and launch counting for the library's own kernels.
//
// Every kernel launch in this library goes through trace_begin / trace_end. With tracing on, a
// pair of CUDA events is recorded on the launching stream around the launch; nnb_trace_query
// later sums the elapsed times per kernel kind. The launch counter runs always, so a caller can
// tell how many of this library's kernels a region launched.
#include <atomic>
#include <mutex>
#include <vector>

#include "nnb_internal.h"
#include "nnb_trace.h"

namespace nnb {

namespace {

struct Pending {
	int kind;
	cudaEvent_t start, stop;
};

std::atomic<bool> g_on{false};
std::atomic<long long> g_launches{0};
std::mutex g_mu;
std::vector<Pending> g_pending;
std::vector<cudaEvent_t> g_free;
double g_total_ms[kTraceKinds] = {};
long long g_count[kTraceKinds] = {};

cudaEvent_t take_event() {
	if (!g_free.empty()) {
		cudaEvent_t e = g_free.back();
		g_free.pop_back();
		return e;
	}
	cudaEvent_t e = nullptr;
	cudaEventCreate(&e);
	return e;
}

// Folds every finished pair into the totals (blocks on unfinished ones).
void drain_locked() {
	for (Pending& p : g_pending) {
		float ms = 0.0f;
		if (cudaEventSynchronize(p.stop) == cudaSuccess && cudaEventElapsedTime(&ms, p.start, p.stop) == cudaSuccess) {
			g_total_ms[p.kind] += ms;
			g_count[p.kind] += 1;
		}
		g_free.push_back(p.start);
		g_free.push_back(p.stop);
	}
	g_pending.clear();
}

}  // namespace

TraceScope::TraceScope(cudaStream_t s, int kind, bool enabled) : s_(s), kind_(kind) {
	if (!enabled) return;
	g_launches.fetch_add(1, std::memory_order_relaxed);
	if (!g_on.load(std::memory_order_relaxed)) return;
	std::lock_guard<std::mutex> lock(g_mu);
	start_ = take_event();
	stop_ = take_event();
	if (start_ && stop_) cudaEventRecord(start_, s_);
}

TraceScope::~TraceScope() {
	if (!start_ || !stop_) return;
	cudaEventRecord(stop_, s_);
	std::lock_guard<std::mutex> lock(g_mu);
	g_pending.push_back({kind_, start_, stop_});
}

}  // namespace nnb

extern "C" {

void nnb_trace_enable(int on) { nnb::g_on.store(on != 0); }

void nnb_trace_reset(void) {
	std::lock_guard<std::mutex> lock(nnb::g_mu);
	nnb::drain_locked();
	for (int i = 0; i < nnb::kTraceKinds; ++i) {
		nnb::g_total_ms[i] = 0.0;
		nnb::g_count[i] = 0;
	}
	nnb::g_launches.store(0);
}

nnb_status nnb_trace_query(int kind, double* total_ms, long long* launches) {
	if (kind < 0 || kind >= nnb::kTraceKinds) return nnb::fail(NNB_ERR_INVALID, "trace kind %d out of range", kind);
	std::lock_guard<std::mutex> lock(nnb::g_mu);
	nnb::drain_locked();
	if (total_ms) *total_ms = nnb::g_total_ms[kind];
	if (launches) *launches = nnb::g_count[kind];
	return NNB_OK;
}

long long nnb_launch_count(void) { return nnb::g_launches.load(); }

}  // extern "C"
