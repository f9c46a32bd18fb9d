// Opt-in per-launch timing: when enabled, every kernel launch of the library
// is bracketed by CUDA events recorded on its own stream; gdn2_profile_read
// waits for them and reports launches and total device time per kernel.
// Off by default; a disabled check is one relaxed atomic load per launch.
#include <atomic>
#include <mutex>
#include <vector>

#include "chunk_layout.cuh"
#include "profile.cuh"

namespace gdn2 {
namespace {

const char* kNames[kNumKernels] = {"chunk_intra_kernel", "chunk_scan_fwd_kernel", "chunk_scan_bwd_kernel",
                                   "chunk_bwd_intra_kernel", "recurrent_kernel", "cp_kernel",
                                   "chunk_scan_fwd_tc_kernel", "chunk_scan_bwd_tc_kernel",
                                   "layer_prep_fwd_kernel", "layer_prep_bwd_kernel",
                                   "norm_gate_fwd_kernel", "norm_gate_bwd_kernel", "seg_fold_kernel",
                                   "chunk_bwd_fp32_kernel", "fp32_prep_epilogue_kernel"};

struct Pending {
  int id;
  cudaEvent_t start, end;
};

std::atomic<int> g_on{0};
std::mutex g_mu;
std::vector<Pending> g_pending;
std::vector<cudaEvent_t> g_pool;
thread_local cudaEvent_t t_start = nullptr;

cudaEvent_t get_event() {
  if (!g_pool.empty()) {
    cudaEvent_t e = g_pool.back();
    g_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

}  // namespace

bool prof_on() { return g_on.load(std::memory_order_relaxed) != 0; }

void prof_begin(int, cudaStream_t s) {
  if (!prof_on()) return;
  std::lock_guard<std::mutex> lk(g_mu);
  t_start = get_event();
  if (t_start) cudaEventRecord(t_start, s);
}

void prof_end(int id, cudaStream_t s) {
  if (!prof_on() || !t_start) return;
  std::lock_guard<std::mutex> lk(g_mu);
  cudaEvent_t e = get_event();
  if (!e) return;
  cudaEventRecord(e, s);
  g_pending.push_back({id, t_start, e});
  t_start = nullptr;
}

}  // namespace gdn2

using namespace gdn2;

extern "C" int gdn2_profile_enable(int on) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (auto& p : g_pending) {
    cudaEventSynchronize(p.end);
    g_pool.push_back(p.start);
    g_pool.push_back(p.end);
  }
  g_pending.clear();
  g_on.store(on ? 1 : 0);
  return GDN2_OK;
}

extern "C" int gdn2_profile_read(gdn2_kernel_stat* out, int max_entries) {
  std::lock_guard<std::mutex> lk(g_mu);
  int64_t launches[kNumKernels] = {0};
  double ms[kNumKernels] = {0.0};
  for (auto& p : g_pending) {
    cudaError_t e = cudaEventSynchronize(p.end);
    if (e != cudaSuccess) return -static_cast<int>(e);
    float t = 0.f;
    cudaEventElapsedTime(&t, p.start, p.end);
    launches[p.id] += 1;
    ms[p.id] += t;
    g_pool.push_back(p.start);
    g_pool.push_back(p.end);
  }
  g_pending.clear();
  int n = 0;
  for (int i = 0; i < kNumKernels && n < max_entries; ++i) {
    if (!launches[i]) continue;
    out[n].name = kNames[i];
    out[n].launches = launches[i];
    out[n].total_ms = ms[i];
    ++n;
  }
  return n;
}
