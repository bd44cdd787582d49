// Library-level entry points of libgrs_b200.so.
#include <atomic>

#include "grs_common.cuh"

namespace grs {
static std::atomic<int64_t> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace grs

extern "C" int64_t grs_launch_count(void) {
  return grs::g_launches.load(std::memory_order_relaxed);
}

extern "C" void grs_count_launches(int64_t n) {
  if (n > 0) grs::g_launches.fetch_add(n, std::memory_order_relaxed);
}

extern "C" const char* grs_version(void) {
  return "grs_b200 0.1 sm_100a";
}
