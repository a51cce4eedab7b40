// murm_profile.cu — launch counting and optional per-kernel CUDA-event timing.
//
// Every kernel launch in this library goes through launch_begin/launch_end
// (see MURM_LAUNCH in murm_kernels.cuh). Counting is one relaxed atomic add.
// While profiling is on, the launch is bracketed by two CUDA events recorded
// on the launch stream, so the device time of each kernel is measured on the
// stream it runs on; results are aggregated by kernel name.
#include <atomic>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "murm_kernels.cuh"

namespace murm {
namespace {
std::atomic<uint64_t> g_launches{0};
std::atomic<bool> g_profiling{false};
std::mutex g_mu;
struct Rec {
  const char* name;
  cudaEvent_t a, b;
};
std::vector<Rec> g_recs;
std::vector<cudaEvent_t> g_free;
thread_local Rec* t_open = nullptr;

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
std::mutex g_attr_mu;
std::map<std::pair<const void*, int>, int> g_attr;  // (kernel, device) -> dynamic smem opted into
}  // namespace

cudaError_t smem_opt_in_raw(const void* kernel, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  int& have = g_attr[std::make_pair(kernel, dev)];
  if (bytes <= have) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) have = bytes;
  return e;
}

bool coop_fits(const void* kernel, int threads, int smem, int blocks) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, int, int>, int> resident;  // -> blocks resident at once
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_tuple(kernel, dev, threads, smem);
  auto it = resident.find(key);
  if (it == resident.end()) {
    int coop = 0, sms = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess)
      coop = 0;
    it = resident.emplace(key, coop ? sms * per_sm : 0).first;
  }
  return blocks <= it->second;
}

void launch_begin(const char* name, cudaStream_t st) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (!g_profiling.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lk(g_mu);
  g_recs.push_back(Rec{name, take_event(), take_event()});
  cudaEventRecord(g_recs.back().a, st);
  t_open = &g_recs.back();
}

void launch_end(cudaStream_t st) {
  if (!g_profiling.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_recs.empty()) cudaEventRecord(g_recs.back().b, st);
  t_open = nullptr;
}

}  // namespace murm

using namespace murm;

extern "C" {

uint64_t murm_kernel_launches(void) { return g_launches.load(); }

murm_status murm_profile_begin(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_recs.clear();
  g_recs.reserve(1 << 16);  // records must not move while a launch is open
  g_profiling.store(true);
  return MURM_OK;
}

murm_status murm_profile_end(murm_kernel_time* out, int32_t capacity, int32_t* count) {
  g_profiling.store(false);
  std::lock_guard<std::mutex> lk(g_mu);
  std::vector<murm_kernel_time> agg;
  murm_status st = MURM_OK;
  for (Rec& r : g_recs) {
    float ms = 0.f;
    if (cudaEventSynchronize(r.b) != cudaSuccess || cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess)
      st = MURM_ERR_CUDA;
    size_t i = 0;
    for (; i < agg.size(); ++i)
      if (std::strncmp(agg[i].name, r.name, sizeof(agg[i].name) - 1) == 0) break;
    if (i == agg.size()) {
      murm_kernel_time k{};
      std::strncpy(k.name, r.name, sizeof(k.name) - 1);
      agg.push_back(k);
    }
    agg[i].launches += 1;
    agg[i].total_ms += ms;
    g_free.push_back(r.a);
    g_free.push_back(r.b);
  }
  g_recs.clear();
  if (count) *count = (int32_t)agg.size();
  for (int32_t i = 0; i < capacity && i < (int32_t)agg.size(); ++i) out[i] = agg[i];
  return st;
}

}  // extern "C"
