#include <algorithm>
// Host-side runtime helpers shared by all launchers: last-error message, SM count.
#include <cuda_runtime.h>

#include <atomic>
#include <string>

#include "../api.h"

namespace llmt {
namespace {
thread_local std::string g_last_error;
}

const char* last_error() { return g_last_error.c_str(); }
void set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }

int sm_count() {
  static std::atomic<int> n[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  int v = n[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

// SMs left to the persistent kernels (GEMM, attention backward): all of them unless some are
// reserved for kernels that run beside them (the overlapped data-parallel step). A persistent
// kernel sized to every SM waits, whole, for any SM another stream holds.
static std::atomic<int> g_reserved_sms{0};
void set_reserved_sms(int n) { g_reserved_sms.store(n < 0 ? 0 : n); }
int reserved_sms() { return g_reserved_sms.load(); }
int persistent_sms() { return std::max(1, sm_count() - g_reserved_sms.load()); }

namespace {
std::atomic<int> g_n_readers{0};
unsigned long long (*g_readers[64])(bool) = {nullptr};
}  // namespace
// Called during static initialisation of each instrumented translation unit.
int register_bounds_reader(unsigned long long (*reader)(bool)) {
  const int i = g_n_readers.fetch_add(1);
  if (i < 64) g_readers[i] = reader;
  return i;
}
unsigned long long bounds_error(bool reset) {
  unsigned long long first = 0;
  const int n = std::min(64, g_n_readers.load());
  for (int i = 0; i < n; ++i) {
    const unsigned long long v = g_readers[i](reset);
    if (v && !first) first = v;
  }
  return first;
}
bool bounds_checking() {
#ifdef LLMT_DEBUG_BOUNDS
  return true;
#else
  return false;
#endif
}
}  // namespace llmt
