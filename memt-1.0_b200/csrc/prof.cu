// Optional per-launch kernel timing with CUDA events (memt_profiler_* in memt_gdn2.h).
#include <atomic>
#include <mutex>
#include <vector>

#include "launch.h"

namespace memt {
namespace {

struct Record {
  int family;
  cudaEvent_t start, end;
};

std::atomic<bool> g_enabled{false};
std::mutex g_mu;
std::vector<Record> g_records;
std::vector<cudaEvent_t> g_pool;

cudaEvent_t take_event() {
  if (!g_pool.empty()) {
    cudaEvent_t e = g_pool.back();
    g_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

}  // namespace

void prof_begin(int family, cudaStream_t s, void** token) {
  *token = nullptr;
  if (!g_enabled.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lock(g_mu);
  Record* r = new Record{family, take_event(), take_event()};
  cudaEventRecord(r->start, s);
  *token = r;
}

void prof_end(void* token, cudaStream_t s) {
  if (token == nullptr) return;
  Record* r = static_cast<Record*>(token);
  cudaEventRecord(r->end, s);
  std::lock_guard<std::mutex> lock(g_mu);
  g_records.push_back(*r);
  delete r;
}

}  // namespace memt

extern "C" {

int memt_profiler_enable(int on) {
  memt::g_enabled.store(on != 0);
  return MEMT_OK;
}

int memt_profiler_reset(void) {
  std::lock_guard<std::mutex> lock(memt::g_mu);
  for (auto& r : memt::g_records) {
    cudaEventSynchronize(r.end);
    memt::g_pool.push_back(r.start);
    memt::g_pool.push_back(r.end);
  }
  memt::g_records.clear();
  return MEMT_OK;
}

int memt_profiler_read(double* ms, int64_t* launches, int n) {
  if (ms == nullptr || launches == nullptr || n < 0) return MEMT_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < n; ++i) {
    ms[i] = 0.0;
    launches[i] = 0;
  }
  std::lock_guard<std::mutex> lock(memt::g_mu);
  for (auto& r : memt::g_records) {
    cudaError_t e = cudaEventSynchronize(r.end);
    if (e != cudaSuccess) return memt::cuda_status(e);
    float t = 0.f;
    e = cudaEventElapsedTime(&t, r.start, r.end);
    if (e != cudaSuccess) return memt::cuda_status(e);
    if (r.family >= 0 && r.family < n) {
      ms[r.family] += t;
      launches[r.family] += 1;
    }
  }
  return MEMT_OK;
}

}  // extern "C"
