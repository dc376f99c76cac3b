// launch_util.cu — host helpers shared by the kernel launchers.
#include <map>
#include <mutex>
#include <utility>

#include "kernels.h"

namespace moe {

// Opt the kernel in to `smem` bytes of dynamic shared memory and check that
// one CTA of `threads` threads fits an SM.  The driver calls cost a few
// microseconds of host time, so each (kernel, device) pair does them once per
// new maximum: the opt-in only ever grows, and a smaller request fits it.
bool ensure_dynamic_smem(const void* kern, size_t smem, int threads) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> granted;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(kern, dev);
  const auto it = granted.find(key);
  if (it != granted.end() && it->second >= smem) return true;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
      cudaSuccess)
    return false;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess || per_sm < 1)
    return false;
  granted[key] = smem;
  return true;
}

}  // namespace moe
