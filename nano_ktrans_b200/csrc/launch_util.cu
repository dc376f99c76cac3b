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

// True for page-locked host memory registered with CUDA (cudaHostAlloc /
// cudaHostRegister), which device code may read through the same pointer.
bool host_mapped(const void* p) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeHost && at.devicePointer == p;
}

// Inputs of moe_forward_host read from mapped host memory into the workspace:
// 16-byte loads, one grid of 256-thread blocks over both buffers.
__global__ void __launch_bounds__(256) stage_in_kernel(const uint4* __restrict__ x, int nx, const uint4* __restrict__ l,
                                                       int nl, uint4* __restrict__ xd, uint4* __restrict__ ld) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the previous step's kernels are done with the workspace
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < nx)
    xd[i] = x[i];
  else if (i < nx + nl)
    ld[i - nx] = l[i - nx];
}

void launch_stage_in(const void* x, size_t xbytes, const void* l, size_t lbytes, void* xd, void* ld,
                     cudaStream_t st) {
  const int nx = static_cast<int>(xbytes / 16), nl = static_cast<int>(lbytes / 16);
  const int n = nx + nl;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((n + 255) / 256);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, stage_in_kernel, static_cast<const uint4*>(x), nx, static_cast<const uint4*>(l), nl,
                     static_cast<uint4*>(xd), static_cast<uint4*>(ld));
}

}  // namespace moe
