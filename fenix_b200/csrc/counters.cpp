// counters.cpp — process-wide count of kernel launches issued by this library (reported by the
// benchmark as evidence of which code ran on the GPU).
#include "counters.hpp"

#include <atomic>

namespace fxk {
namespace {
std::atomic<unsigned long long> g_launches{0};
}
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
unsigned long long launch_count() { return g_launches.load(std::memory_order_relaxed); }
}  // namespace fxk
