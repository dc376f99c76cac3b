// async_copy.cuh — mbarrier, bulk-copy and grid-barrier primitives (sm_100a).
//
// Every wait here is bounded: it gives up after a fixed number of polls and
// reports failure, so a kernel can record a timeout status and unwind instead
// of hanging the GPU.
#pragma once

#include <cuda/atomic>
#include <stdint.h>

#include "common.cuh"

namespace moe {
namespace ac {

constexpr uint32_t kSpinLimit = 1u << 22;

MOE_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

MOE_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Arrive once and add `bytes` to the transaction count of the current phase.
MOE_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

MOE_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

MOE_DEV bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Bulk copy global -> this CTA's shared memory, completion counted on `bar`.
// dst, src 16-byte aligned, bytes a multiple of 16.
MOE_DEV void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

MOE_DEV unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Grid-wide barrier for a cooperative launch.  The 64-bit arrival counter only
// grows: launch n's barrier is complete when the counter reaches (n + 1) * G.
// The arrival is kept off the critical path.  grid_epoch_read
// reads the counter once, after griddepcontrol.wait and before this CTA
// arrives: every CTA of the launch then sees a value in [n * G, n * G + G - 1]
// (the previous launch's G arrivals are complete, this launch's are not all in)
// and grid_sync_epoch derives the same target (n + 1) * G from it.  The
// arrival is a posted release-add, with no round trip for its return value.
// Issue the read after the CTA's first copies: its result is only needed at
// the barrier.
MOE_DEV unsigned long long grid_epoch_read(const unsigned long long* bar) {
  cuda::atomic_ref<const unsigned long long, cuda::thread_scope_device> count(*bar);
  return count.load(cuda::memory_order_relaxed);
}

MOE_DEV bool grid_sync_epoch(unsigned long long* bar, unsigned long long seen, int* ok_smem) {
  __syncthreads();  // the CTA's writes are ordered before thread 0's release (cumulativity)
  if (threadIdx.x == 0) {
    const unsigned long long g = gridDim.x, target = (seen / g + 1) * g;
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(bar) : "memory");
    cuda::atomic_ref<unsigned long long, cuda::thread_scope_device> count(*bar);
    int ok = 1;
    for (uint32_t i = 0; count.load(cuda::memory_order_acquire) < target; ++i) {
      if (i > kSpinLimit) {
        ok = 0;
        break;
      }
    }
    *ok_smem = ok;
  }
  __syncthreads();
  return *ok_smem != 0;
}

}  // namespace ac
}  // namespace moe
