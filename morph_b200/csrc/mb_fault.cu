// Test-only fault injection for the bounded device waits.
//
// Kernels 1 and 2 (bulk-staged forms) and the kernel-4 GEMM wait on mbarriers
// for the copies their producer issues; every such wait gives up after a bound
// (about 2 s by default), raises the CTA's abort flag, waits (bounded) for its
// own copies in flight, frees what it holds and reports MB_ERR_TIMEOUT (or the
// GEMM's error flag). mb_debug_arm_fault lets a test make that happen without
// faulting anything: the next launch of the named kernel in this process
// withholds one unit's load and uses a short bound, so the consumers' wait for
// that unit expires and the abort path runs. Nothing else changes; a launch
// that finds nothing armed behaves exactly as before.
#include <atomic>
#include <mutex>

#include "mb_async.cuh"
#include "mb_common.cuh"

namespace mb {
namespace {

struct Armed {
  bool on = false;
  int64_t unit = -1;
  uint64_t limit_ns = kWaitLimitNs;
};

std::mutex g_fault_mu;
Armed g_armed[3];                   // kFaultApply, kFaultStats, kFaultGemm
std::atomic<int> g_any_armed{0};

int slot_of(int kernel) {
  switch (kernel) {
    case kFaultApply: return 0;
    case kFaultStats: return 1;
    case kFaultGemm: return 2;
    default: return -1;
  }
}

}  // namespace

void take_fault(int kernel, int64_t* unit, uint64_t* limit_ns) {
  *unit = -1;
  *limit_ns = kWaitLimitNs;
  if (g_any_armed.load(std::memory_order_acquire) == 0) return;
  const int s = slot_of(kernel);
  if (s < 0) return;
  std::lock_guard<std::mutex> lock(g_fault_mu);
  if (!g_armed[s].on) return;
  *unit = g_armed[s].unit;
  *limit_ns = g_armed[s].limit_ns;
  g_armed[s] = Armed{};
  g_any_armed.fetch_sub(1, std::memory_order_acq_rel);
}

}  // namespace mb

extern "C" MB_API int mb_debug_arm_fault(int32_t kernel, int64_t unit, int64_t wait_limit_ns) {
  if (kernel == 0) {  // disarm everything
    std::lock_guard<std::mutex> lock(mb::g_fault_mu);
    for (auto& a : mb::g_armed) a = mb::Armed{};
    mb::g_any_armed.store(0, std::memory_order_release);
    return MB_OK;
  }
  const int s = mb::slot_of(kernel);
  if (s < 0 || unit < 0 || wait_limit_ns < 1000 || wait_limit_ns > (int64_t)mb::kWaitLimitNs) return MB_ERR_ARG;
  std::lock_guard<std::mutex> lock(mb::g_fault_mu);
  if (!mb::g_armed[s].on) mb::g_any_armed.fetch_add(1, std::memory_order_acq_rel);
  mb::g_armed[s].on = true;
  mb::g_armed[s].unit = unit;
  mb::g_armed[s].limit_ns = (uint64_t)wait_limit_ns;
  return MB_OK;
}
