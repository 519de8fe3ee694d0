// Launch accounting and optional per-kernel CUDA-event timing.
//
// Every kernel the library launches goes through prof_begin / prof_end. The
// launch counter is always on (one relaxed atomic add); event timing is off
// unless dd_profile_enable(1) was called, in which case an event pair is
// recorded on the launching stream around each launch and resolved by
// dd_profile_read. While timing is on, dd_cascade_decode does not fork its
// tensor-core kernel onto a side stream, so the pairs time kernels alone.
#include <atomic>
#include <mutex>
#include <vector>

#include "dd_device.cuh"
#include "dd_profile.h"

namespace dd {

static std::atomic<uint64_t> g_launches{0};
static std::atomic<int> g_prof_on{0};
static std::mutex g_mu;
struct Pending {
  int kind;
  cudaEvent_t a, b;
};
static std::vector<Pending> g_pending;
static thread_local cudaEvent_t t_open[kNumProf];

void prof_begin(int kind, cudaStream_t st) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (!g_prof_on.load(std::memory_order_relaxed)) return;
  cudaEvent_t e;
  if (cudaEventCreate(&e) != cudaSuccess) return;
  cudaEventRecord(e, st);
  t_open[kind] = e;
}

bool prof_timing_on() { return g_prof_on.load(std::memory_order_relaxed) != 0; }

void prof_end(int kind, cudaStream_t st) {
  if (!g_prof_on.load(std::memory_order_relaxed) || !t_open[kind]) return;
  cudaEvent_t e;
  if (cudaEventCreate(&e) != cudaSuccess) return;
  cudaEventRecord(e, st);
  std::lock_guard<std::mutex> lk(g_mu);
  g_pending.push_back({kind, t_open[kind], e});
  t_open[kind] = nullptr;
}

}  // namespace dd

using namespace dd;

extern "C" uint64_t dd_launch_count(void) { return g_launches.load(); }

extern "C" void dd_profile_enable(int on) { g_prof_on.store(on ? 1 : 0); }

extern "C" int dd_profile_read(double* ms, int64_t* launches, int32_t n) {
  if (n < 0) return fail(DD_ERR_INVALID_ARGUMENT, "n must be >= 0");
  std::vector<Pending> todo;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    todo.swap(g_pending);
  }
  for (int k = 0; k < n; ++k) {
    if (ms) ms[k] = 0.0;
    if (launches) launches[k] = 0;
  }
  int rc = DD_OK;
  for (const Pending& p : todo) {
    float t = 0.f;
    const cudaError_t e = cudaEventSynchronize(p.b);
    if (e == cudaSuccess && cudaEventElapsedTime(&t, p.a, p.b) == cudaSuccess) {
      if (p.kind < n) {
        if (ms) ms[p.kind] += t;
        if (launches) launches[p.kind] += 1;
      }
    } else {
      rc = fail(DD_ERR_CUDA, "profile event failed");
    }
    cudaEventDestroy(p.a);
    cudaEventDestroy(p.b);
  }
  return rc;
}
