// Host-mapped status word. Kernels that give up on a bounded wait store an
// error code here with a system-scope release store; the host reads it
// without synchronising the device.
#include <ATen/cuda/CUDAContext.h>
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "host_utils.h"

namespace bdion {

namespace {
volatile int* g_host_word = nullptr;
int* g_dev_word = nullptr;
std::once_flag g_once;
std::atomic<uint64_t> g_limit_ns{2000000000ull};
std::atomic<uint64_t> g_launches{0};

void init_word() {
  void* h = nullptr;
  C10_CUDA_CHECK(cudaHostAlloc(&h, 64, cudaHostAllocMapped | cudaHostAllocPortable));
  g_host_word = static_cast<volatile int*>(h);
  *g_host_word = 0;
  void* d = nullptr;
  C10_CUDA_CHECK(cudaHostGetDevicePointer(&d, h, 0));
  g_dev_word = static_cast<int*>(d);
}
}  // namespace

int* status_device_ptr() {
  std::call_once(g_once, init_word);
  return g_dev_word;
}
int status_read() {
  std::call_once(g_once, init_word);
  return *g_host_word;
}
void status_clear() {
  std::call_once(g_once, init_word);
  *g_host_word = 0;
}
uint64_t wait_limit_ns() { return g_limit_ns.load(); }
void set_wait_limit_ns(uint64_t ns) { g_limit_ns.store(ns); }
void note_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }
uint64_t launch_count() { return g_launches.load(); }

}  // namespace bdion
