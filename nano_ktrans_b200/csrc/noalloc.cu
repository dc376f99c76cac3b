// noalloc.cu — the single-launch decode step without any allocation.
//
// moe_forward() needs a handle from moe_create(), and moe_create() calls
// cudaMalloc for its workspace.  Some callers cannot allocate device memory
// at the point where they run a layer: code running under a memory budget
// that was fixed up front, an allocator-free embedding (for example an
// inference server that hands out only pre-registered buffers), or a caller
// that must not touch the driver's allocator while other work is in flight.
// moe_decode_noalloc() serves them: it takes the layer description, the
// weight pointers, the inputs and the outputs directly, and keeps its scratch
// (the per-pair SiLU(gate)*up intermediate, the grid-barrier counter and a
// status word) in one file-scope device array of fixed size.
//
// Limits and sharing:
//   * scratch holds at most kNoAllocMaxH floats of intermediate:
//     num_tokens * top_k * inter_size <= kNoAllocMaxH (24576 floats = 96 KiB,
//     the most the single-launch kernel stages); larger calls are rejected
//     with MOE_ERANGE before anything is launched;
//   * the batch must also fit the single-launch kernel (at most 4 tokens and
//     32 (token, expert) pairs, at most 256 experts);
//   * every call on a device uses the same array, which keeps the previous
//     call's contents.  Nothing in it needs clearing between calls: the
//     intermediate is written before it is read, and the barrier counter
//     only grows (it starts at zero when the module loads).  Two calls whose
//     kernels overlap on the GPU (different streams, or concurrent host
//     threads) race on the array and produce wrong results; serialise them.
//   * the first call on each device looks up the array's device address with
//     cudaGetSymbolAddress; make that first call outside any stream capture.
//     The address is remembered per device ordinal for the life of the
//     process: after cudaDeviceReset (which unloads the module) this entry
//     point must not be used again in the process;
//   * a null status_dev discards the kernel's status bits (bounded-wait
//     timeouts, bad expert ids); pass a zeroed int32 to receive them - bits
//     accumulate across calls until the caller clears the word.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/moe_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace {

constexpr size_t kNoAllocMaxH = 24576;  // floats of SiLU(gate)*up intermediate (96 KiB, the kernel's cap)
constexpr size_t kNoAllocHeader = 256;  // barrier counter (8 B) + status word (4 B), padded
constexpr size_t kNoAllocBytes = kNoAllocHeader + kNoAllocMaxH * sizeof(float);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

std::mutex g_mu;
unsigned char* g_scratch_addr[kMaxDevices] = {};

void put_err(char* buf, size_t len, const char* f, ...) {
  if (buf == nullptr || len == 0) return;
  va_list ap;
  va_start(ap, f);
  vsnprintf(buf, len, f, ap);
  va_end(ap);
}

// Device address of the scratch array on the current device (looked up once).
int scratch_address(unsigned char** out, char* err, size_t err_len) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    put_err(err, err_len, "moe_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return MOE_ECUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    put_err(err, err_len, "moe_decode_noalloc: device ordinal %d not supported", dev);
    return MOE_EINVAL;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      put_err(err, err_len, "moe_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return MOE_ECUDA;
    }
    g_scratch_addr[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_scratch_addr[dev];
  return MOE_OK;
}

moe::QuantProj proj(const moe_layer_desc& d, const void* q, const void* s, int n, int k) {
  moe::QuantProj p;
  p.q = static_cast<const uint8_t*>(q);
  p.s = static_cast<const uint16_t*>(s);
  p.n = n;
  p.k = k;
  p.group = d.group_size > 0 ? d.group_size : k;
  p.sstride = (k / p.group + 7) / 8 * 8;
  return p;
}

}  // namespace

extern "C" int moe_decode_noalloc(const moe_layer_desc* desc, const moe_weights* w, const uint16_t* x_dev,
                                  const uint16_t* logits_dev, int32_t num_tokens, uint16_t* out_dev,
                                  int64_t* topk_ids_dev, uint16_t* topk_weights_dev, int32_t* status_dev,
                                  void* stream, char* err, size_t err_len) {
  if (desc == nullptr || w == nullptr) {
    put_err(err, err_len, "moe_decode_noalloc: null description or weights");
    return MOE_EINVAL;
  }
  const moe_layer_desc& d = *desc;
  if ((d.bits != 4 && d.bits != 8) || d.top_k < 1 || d.num_experts < 1 || d.top_k > d.num_experts ||
      d.hidden_size <= 0 || d.inter_size <= 0 || d.group_size < 0) {
    put_err(err, err_len, "moe_decode_noalloc: invalid layer description");
    return MOE_EINVAL;
  }
  const int align = d.bits == 4 ? 32 : 16;
  if (d.hidden_size % align || d.inter_size % align ||
      (d.group_size > 0 && (d.group_size % align || d.hidden_size % d.group_size || d.inter_size % d.group_size))) {
    put_err(err, err_len, "moe_decode_noalloc: hidden/inter/group sizes must be multiples of %d codes", align);
    return MOE_EINVAL;
  }
  if (num_tokens < 0) {
    put_err(err, err_len, "moe_decode_noalloc: negative token count");
    return MOE_EINVAL;
  }
  if (num_tokens == 0) return MOE_OK;
  if (x_dev == nullptr || logits_dev == nullptr || out_dev == nullptr || topk_ids_dev == nullptr ||
      topk_weights_dev == nullptr) {
    put_err(err, err_len, "moe_decode_noalloc: null input or output pointer");
    return MOE_EINVAL;
  }
  const void* need[] = {w->gate_q_dev, w->gate_s_dev, w->up_q_dev, w->up_s_dev, w->down_q_dev, w->down_s_dev};
  for (const void* p : need) {
    if (p == nullptr || reinterpret_cast<uintptr_t>(p) % 16) {
      put_err(err, err_len, "moe_decode_noalloc: routed-expert weight pointers must be non-null and 16-byte aligned");
      return MOE_EINVAL;
    }
  }
  const size_t h_floats = static_cast<size_t>(num_tokens) * d.top_k * d.inter_size;
  if (h_floats > kNoAllocMaxH) {
    put_err(err, err_len,
            "moe_decode_noalloc: num_tokens * top_k * inter_size = %zu exceeds the fixed scratch of %zu floats",
            h_floats, kNoAllocMaxH);
    return MOE_ERANGE;
  }
  int num_sms = 0, dev = 0;
  cudaError_t ce = cudaGetDevice(&dev);
  if (ce == cudaSuccess) ce = cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev);
  if (ce != cudaSuccess || num_sms < 1) {
    put_err(err, err_len, "moe_decode_noalloc: device query failed: %s", cudaGetErrorString(ce));
    return MOE_ECUDA;
  }
  moe::DecodeFusedParams p{};
  p.gate = proj(d, w->gate_q_dev, w->gate_s_dev, d.inter_size, d.hidden_size);
  p.up = proj(d, w->up_q_dev, w->up_s_dev, d.inter_size, d.hidden_size);
  p.down = proj(d, w->down_q_dev, w->down_s_dev, d.hidden_size, d.inter_size);
  if (!moe::decode_fused_eligible(d.bits, num_tokens, d.num_experts, d.top_k, p.gate, p.down, num_sms)) {
    put_err(err, err_len,
            "moe_decode_noalloc: batch outside the single-launch kernel's limits (<= 4 tokens, <= 32 "
            "(token, expert) pairs, <= 256 experts)");
    return MOE_ERANGE;
  }
  unsigned char* scratch = nullptr;
  if (int rc = scratch_address(&scratch, err, err_len)) return rc;
  p.x = x_dev;
  p.logits = logits_dev;
  p.ids_out = topk_ids_dev;
  p.w_out = topk_weights_dev;
  p.T = num_tokens;
  p.E = d.num_experts;
  p.top_k = d.top_k;
  p.use_softmax = d.router_use_softmax;
  p.renorm = d.normalize_topk_prob;
  p.bar = reinterpret_cast<unsigned long long*>(scratch);
  p.status = status_dev != nullptr ? status_dev : reinterpret_cast<int*>(scratch + 8);
  p.hbuf = reinterpret_cast<float*>(scratch + kNoAllocHeader);
  p.out = out_dev;
  p.num_sms = num_sms;
  const int rc = moe::launch_decode_fused(d.bits, p, static_cast<cudaStream_t>(stream));
  const cudaError_t e = cudaGetLastError();
  if (rc < 0 || e != cudaSuccess) {
    put_err(err, err_len, "moe_decode_noalloc: launch failed: %s",
            e != cudaSuccess ? cudaGetErrorString(e) : "launch configuration refused");
    return MOE_ECUDA;
  }
  return MOE_OK;
}
