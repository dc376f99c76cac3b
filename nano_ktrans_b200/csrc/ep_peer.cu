// ep_peer.cu — expert parallelism with the exchanges done over peer memory.
//
// The routed experts of a layer are split over the ranks (one process per
// GPU, all GPUs in one NVLink / NVSwitch domain) as in ep.cu; the difference
// is how rows move.  Instead of two collective all-to-alls whose split sizes
// must first be read back to the host, every rank publishes its token rows
// and their expert slots in its own region, and the other ranks' kernels
// read them through CUDA IPC mappings (plain loads over NVLink) and store the
// fp32 expert outputs straight into the token's rank's region (plain stores
// over NVLink).  Ranks hand over with epoch flags: the last block of the
// publishing (or storing) kernel makes the rank's writes visible at system
// scope and stores the epoch into a flag slot of every rank's region with
// release semantics; a consumer kernel's blocks wait for every rank's flag
// with acquire loads (bounded: 5 s, then the group's status word gets
// MOE_EP_STATUS_TIMEOUT and every later wait of the group gives up at once).
// Buffers are reused without extra handshakes: a rank republishes its rows
// only after its own combine, which waited for every rank's "done", which
// each rank signals after it has read those rows; a rank's y is rewritten
// only after it signalled "ready" for the next step, which follows its own
// combine of the previous one.
//
// Token rows are gathered whole (every rank's x into x_all): with top-8
// routing over 8 ranks two thirds of the tokens touch each rank, and a dense
// layout needs no prefix sums across ranks.  The owners' expert kernels then
// see x_all with ids_all (local expert of each pair, -1 for pairs owned
// elsewhere, skipped by the permute).
//
// No counterpart in the reference (its offload backends are single-device);
// the combine is the single-GPU combine (nano_ktrans/kernels/cpu_moe.py:515-538
// order: experts ascending, fp32, one bf16 rounding).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "../../include/moe_b200.h"
#include "async_copy.cuh"
#include "common.cuh"
#include "ep_peer.h"

namespace moe {
namespace ep {

constexpr unsigned long long kPeerWaitNs = 5000000000ull;
constexpr int kMaxTopK = 16;

MOE_DEV unsigned long long* flag_ptr(unsigned char* region, int which, int slot) {
  return reinterpret_cast<unsigned long long*>(region) + which * kEpMaxWorld + slot;
}

MOE_DEV unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

MOE_DEV void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Thread 0 of the block waits until flag `which` of every rank has reached
// `epoch`; the block then proceeds (true) or gives up (false) together.
MOE_DEV bool wait_all(const PeerView& v, int which, unsigned long long epoch, int* ok_smem) {
  if (threadIdx.x == 0) {
    int ok = (atomicOr(v.status, 0) & kStatusTimeout) ? 0 : 1;
    const unsigned long long* f = flag_ptr(v.region[v.rank], which, 0);
    const unsigned long long t0 = ac::global_ns();
    for (int s = 0; ok && s < v.world; ++s) {
      while (ld_acquire_sys(f + s) < epoch) {
        if (ac::global_ns() - t0 > kPeerWaitNs) {
          atomicOr(v.status, kStatusTimeout);
          ok = 0;
          break;
        }
        __nanosleep(128);
      }
    }
    *ok_smem = ok;
  }
  __syncthreads();
  return *ok_smem != 0;
}

// Called by every thread of every block at the end of a producing kernel: the
// block's writes are fenced at system scope, and the last block to arrive
// stores the epoch (advanced first when `advance`) into flag `which`, slot
// `rank`, of every rank's region.  The counter is back at 0 afterwards.
MOE_DEV void signal_last(const PeerView& v, int which, unsigned long long* epoch, unsigned int* counter,
                         bool advance) {
  __shared__ unsigned int s_last;
  __shared__ unsigned long long s_epoch;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    s_last = atomicAdd(counter, 1u) == gridDim.x - 1 ? 1u : 0u;
    if (s_last) {
      __threadfence_system();
      unsigned long long e = *reinterpret_cast<volatile unsigned long long*>(epoch);
      if (advance) {
        e += 1;
        *reinterpret_cast<volatile unsigned long long*>(epoch) = e;
      }
      s_epoch = e;
      *reinterpret_cast<volatile unsigned int*>(counter) = 0u;
    }
  }
  __syncthreads();
  if (s_last && threadIdx.x < v.world) {
    __threadfence_system();
    st_release_sys(flag_ptr(v.region[threadIdx.x], which, v.rank), s_epoch);
  }
}

__global__ void __launch_bounds__(256) publish_kernel(PeerView v, const uint16_t* __restrict__ x,
                                                      const int64_t* __restrict__ ids, int T,
                                                      const int32_t* __restrict__ slot_of_expert,
                                                      unsigned long long* epoch, unsigned int* counter) {
  unsigned char* mine = v.region[v.rank];
  const int nthreads = gridDim.x * blockDim.x;
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
  const int vec = v.hidden / 8;
  const uint4* src = reinterpret_cast<const uint4*>(x);
  uint4* dst = reinterpret_cast<uint4*>(mine + v.off_x);
  const long n = static_cast<long>(T) * vec;
  for (long i = gtid; i < n; i += nthreads) dst[i] = src[i];
  int32_t* slots = reinterpret_cast<int32_t*>(mine + v.off_slots);
  bool bad = false;
  for (int p = gtid; p < T * v.top_k; p += nthreads) {
    const int64_t e = ids[p];
    int slot = -1;
    if (e >= 0 && e < v.num_experts) {
      const int g = slot_of_expert[e];
      if (g >= 0 && g < v.num_experts) slot = g;
    }
    bad |= slot < 0;
    slots[p] = slot;
  }
  if (bad) atomicOr(v.status, kStatusBadExpertId);
  if (gtid == 0) *reinterpret_cast<volatile int32_t*>(mine + kEpOffHdr) = T;
  signal_last(v, kEpFlagReady, epoch, counter, true);
}

// x_all [world][bound][hidden] and ids_all [world][bound][top_k]: rank s's
// token t at row s * bound + t (bound = the step's tokens-per-rank limit).
__global__ void __launch_bounds__(256) collect_kernel(PeerView v, const unsigned long long* epoch, int bound,
                                                      uint16_t* __restrict__ x_all, int64_t* __restrict__ ids_all) {
  __shared__ int ok;
  __shared__ int ts[kEpMaxWorld];
  const bool ready = wait_all(v, kEpFlagReady, *epoch, &ok);
  if (threadIdx.x < v.world) {
    const int t = *reinterpret_cast<const volatile int32_t*>(v.region[threadIdx.x] + kEpOffHdr);
    if (ready && t > bound && blockIdx.x == 0) atomicOr(v.status, kEpStatusOverflow);
    // a step whose wait ran out selects no pairs, so the expert kernels do nothing
    ts[threadIdx.x] = !ready || t < 0 ? 0 : (t > bound ? bound : t);
  }
  __syncthreads();
  const int nthreads = gridDim.x * blockDim.x;
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
  const int k = v.top_k, per = bound * k, epr = v.experts_per_rank;
  for (int i = gtid; i < v.world * per; i += nthreads) {
    const int s = i / per, q = i - s * per;
    int64_t loc = -1;
    if (q / k < ts[s]) {
      const int slot = reinterpret_cast<const int32_t*>(v.region[s] + v.off_slots)[q];
      if (slot >= 0 && slot / epr == v.rank) loc = slot - v.rank * epr;
    }
    ids_all[i] = loc;
  }
  const int vec = v.hidden / 8;
  const long rows = static_cast<long>(v.world) * bound;
  uint4* dst = reinterpret_cast<uint4*>(x_all);
  for (long i = gtid; i < rows * vec; i += nthreads) {
    const long r = i / vec;
    const int c = static_cast<int>(i - r * vec);
    const int s = static_cast<int>(r / bound), t = static_cast<int>(r - static_cast<long>(s) * bound);
    if (t < ts[s]) dst[i] = reinterpret_cast<const uint4*>(v.region[s] + v.off_x)[static_cast<long>(t) * vec + c];
  }
}

// One warp per pair: the pair's fp32 output row into its token's rank's y
// (pair p = (s * bound + t) * top_k + j goes to rank s's y[t][j]).
__global__ void __launch_bounds__(256) scatter_kernel(PeerView v, const int32_t* __restrict__ pair_pos, int P,
                                                      int bound, const float* __restrict__ y,
                                                      unsigned long long* epoch, unsigned int* counter) {
  const int lane = threadIdx.x & 31;
  const int per = bound * v.top_k;
  const int vec = v.hidden / 4;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int p = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < P; p += warps) {
    const int pos = pair_pos[p];
    if (pos < 0) continue;
    const int s = p / per, q = p - s * per;
    const float4* src = reinterpret_cast<const float4*>(y + static_cast<size_t>(pos) * v.hidden);
    float4* dst = reinterpret_cast<float4*>(v.region[s] + v.off_y) + static_cast<size_t>(q) * vec;
    for (int i = lane; i < vec; i += 32) dst[i] = src[i];
  }
  signal_last(v, kEpFlagDone, epoch, counter, false);
}

// The single-GPU combine (expert_matvec.cu combine_kernel) over y[t][j] of
// this rank's region.
__global__ void __launch_bounds__(256) combine_kernel(PeerView v, const unsigned long long* epoch,
                                                      const int64_t* __restrict__ ids,
                                                      const uint16_t* __restrict__ weights, int T,
                                                      uint16_t* __restrict__ out) {
  __shared__ int ok;
  const bool done = wait_all(v, kEpFlagDone, *epoch, &ok);
  const int H = v.hidden, top_k = v.top_k, cols4 = H / 4;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= T * cols4) return;
  const int t = idx / cols4, c4 = idx - t * cols4;
  if (!done) {  // the status word says why; the output is zeros
    reinterpret_cast<uint2*>(out + static_cast<size_t>(t) * H)[c4] = make_uint2(0u, 0u);
    return;
  }
  const float* y = reinterpret_cast<const float*>(v.region[v.rank] + v.off_y);
  int ex[kMaxTopK], ps[kMaxTopK];
  float wt[kMaxTopK];
  int n = 0;
  for (int j = 0; j < top_k; ++j) {
    const int p = t * top_k + j;
    const int64_t e64 = ids[p];
    if (e64 < 0 || e64 >= v.num_experts) continue;
    const int e = static_cast<int>(e64);
    const float w = bf16_to_f32(weights[p]);
    int i = n++;
    while (i > 0 && ex[i - 1] > e) {
      ex[i] = ex[i - 1];
      ps[i] = ps[i - 1];
      wt[i] = wt[i - 1];
      --i;
    }
    ex[i] = e;
    ps[i] = p;
    wt[i] = w;
  }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i = 0; i < n; ++i) {
    const float4 val = reinterpret_cast<const float4*>(y + static_cast<size_t>(ps[i]) * H)[c4];
    acc.x = __fadd_rn(acc.x, __fmul_rn(val.x, wt[i]));
    acc.y = __fadd_rn(acc.y, __fmul_rn(val.y, wt[i]));
    acc.z = __fadd_rn(acc.z, __fmul_rn(val.z, wt[i]));
    acc.w = __fadd_rn(acc.w, __fmul_rn(val.w, wt[i]));
  }
  uint2 o;
  o.x = static_cast<uint32_t>(f32_to_bf16(acc.x)) | (static_cast<uint32_t>(f32_to_bf16(acc.y)) << 16);
  o.y = static_cast<uint32_t>(f32_to_bf16(acc.z)) | (static_cast<uint32_t>(f32_to_bf16(acc.w)) << 16);
  reinterpret_cast<uint2*>(out + static_cast<size_t>(t) * H)[c4] = o;
}

}  // namespace ep

static size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

void ep_region_layout(int max_tokens, int top_k, int hidden, size_t& off_slots, size_t& off_x, size_t& off_y,
                      size_t& total) {
  const size_t T = static_cast<size_t>(max_tokens), k = static_cast<size_t>(top_k), H = static_cast<size_t>(hidden);
  off_slots = kEpOffSlots;
  off_x = align256(off_slots + T * k * sizeof(int32_t));
  off_y = align256(off_x + T * H * sizeof(uint16_t));
  total = align256(off_y + T * k * H * sizeof(float));
}

void launch_ep_peer_publish(const PeerView& v, const uint16_t* x, const int64_t* ids, int T,
                            const int32_t* slot_of_expert, unsigned long long* epoch, unsigned int* counter,
                            int num_sms, cudaStream_t st) {
  const long work = std::max(static_cast<long>(T) * (v.hidden / 8), 1L);
  const int grid = static_cast<int>(std::min<long>((work + 255) / 256, 2L * num_sms));
  ep::publish_kernel<<<grid, 256, 0, st>>>(v, x, ids, T, slot_of_expert, epoch, counter);
}

void launch_ep_peer_collect(const PeerView& v, const unsigned long long* epoch, int bound, uint16_t* x_all,
                            int64_t* ids_all, int num_sms, cudaStream_t st) {
  const long work = static_cast<long>(v.world) * bound * (v.hidden / 8);
  const int grid = static_cast<int>(std::max(1L, std::min<long>((work + 255) / 256, 8L * num_sms)));
  ep::collect_kernel<<<grid, 256, 0, st>>>(v, epoch, bound, x_all, ids_all);
}

void launch_ep_peer_scatter(const PeerView& v, const int32_t* pair_pos, int P, int bound, const float* y,
                            const unsigned long long* epoch, unsigned int* counter, int num_sms, cudaStream_t st) {
  const int grid = std::max(1, std::min((P + 7) / 8, 8 * num_sms));
  ep::scatter_kernel<<<grid, 256, 0, st>>>(v, pair_pos, P, bound, y, const_cast<unsigned long long*>(epoch),
                                           counter);
}

void launch_ep_peer_combine(const PeerView& v, const unsigned long long* epoch, const int64_t* ids,
                            const uint16_t* weights, int T, uint16_t* out, cudaStream_t st) {
  const int n = T * (v.hidden / 4);
  ep::combine_kernel<<<std::max(1, (n + 255) / 256), 256, 0, st>>>(v, epoch, ids, weights, T, out);
}

}  // namespace moe

// ---------------------------------------------------------------------------
// C ABI: group lifetime and the publish / combine phases (moe_ep_peer_experts,
// which needs a layer handle, is in capi.cu)
// ---------------------------------------------------------------------------

namespace {

using moe::PeerGroup;

static_assert(sizeof(cudaIpcMemHandle_t) == MOE_EP_IPC_HANDLE_BYTES, "IPC handle size");

int gfail(PeerGroup* g, int code, const char* f, ...) {
  char tmp[512];
  va_list ap;
  va_start(ap, f);
  vsnprintf(tmp, sizeof(tmp), f, ap);
  va_end(ap);
  if (g) g->err = tmp;
  return code;
}

int gcheck(PeerGroup* g, cudaError_t e, const char* what) {
  if (e != cudaSuccess) return gfail(g, MOE_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return MOE_OK;
}

bool all_known(const PeerGroup* g) {
  for (int s = 0; s < g->v.world; ++s)
    if (!g->have[s]) return false;
  return true;
}

}  // namespace

extern "C" {

int moe_ep_group_create(int32_t rank, int32_t world, int32_t max_tokens, int32_t top_k, int32_t hidden_size,
                        int32_t num_experts, void** group, char* err, size_t err_len) {
  auto bad = [&](const char* m) {
    if (err && err_len) snprintf(err, err_len, "moe_ep_group_create: %s", m);
    return MOE_EINVAL;
  };
  if (group == nullptr) return bad("null group pointer");
  *group = nullptr;
  if (world < 1 || world > moe::kEpMaxWorld) return bad("world must be in [1, 8]");
  if (rank < 0 || rank >= world) return bad("rank must be in [0, world)");
  if (max_tokens < 1) return bad("max_tokens must be >= 1");
  if (top_k < 1 || top_k > 16) return bad("top_k must be in [1, 16]");
  if (hidden_size < 8 || hidden_size % 8) return bad("hidden_size must be a positive multiple of 8");
  if (num_experts < top_k || num_experts > 1024 || num_experts % world)
    return bad("num_experts must be in [top_k, 1024] and a multiple of world");
  if (static_cast<int64_t>(world) * max_tokens * top_k > (1LL << 30)) return bad("world * max_tokens * top_k too large");
  auto* g = new PeerGroup();
  cudaGetDevice(&g->device);
  cudaDeviceGetAttribute(&g->num_sms, cudaDevAttrMultiProcessorCount, g->device);
  size_t off_slots, off_x, off_y, total;
  moe::ep_region_layout(max_tokens, top_k, hidden_size, off_slots, off_x, off_y, total);
  g->region_bytes = total;
  const size_t x_all = static_cast<size_t>(world) * max_tokens * hidden_size * sizeof(uint16_t);
  const size_t ids_all = static_cast<size_t>(world) * max_tokens * top_k * sizeof(int64_t);
  const size_t small = 256;  // epoch u64, counters u32[2], status i32
  const size_t x_off = 0, ids_off = moe::align256(x_all), small_off = moe::align256(ids_off + ids_all);
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&g->region), total);
  if (e == cudaSuccess) e = cudaMalloc(&g->local, small_off + small);
  if (e == cudaSuccess) e = cudaMemset(g->region, 0, moe::kEpOffSlots);
  if (e == cudaSuccess) e = cudaMemset(static_cast<unsigned char*>(g->local) + small_off, 0, small);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (err && err_len) snprintf(err, err_len, "moe_ep_group_create: %s", cudaGetErrorString(e));
    if (g->region) cudaFree(g->region);
    if (g->local) cudaFree(g->local);
    delete g;
    return MOE_ECUDA;
  }
  unsigned char* base = static_cast<unsigned char*>(g->local);
  g->x_all = reinterpret_cast<uint16_t*>(base + x_off);
  g->ids_all = reinterpret_cast<int64_t*>(base + ids_off);
  g->epoch = reinterpret_cast<unsigned long long*>(base + small_off);
  g->counters = reinterpret_cast<unsigned int*>(base + small_off + 8);
  moe::PeerView& v = g->v;
  v.status = reinterpret_cast<int32_t*>(base + small_off + 16);
  v.rank = rank;
  v.world = world;
  v.max_tokens = max_tokens;
  v.top_k = top_k;
  v.hidden = hidden_size;
  v.num_experts = num_experts;
  v.experts_per_rank = num_experts / world;
  v.off_slots = off_slots;
  v.off_x = off_x;
  v.off_y = off_y;
  v.region[rank] = g->region;
  g->have[rank] = true;
  *group = g;
  return MOE_OK;
}

int moe_ep_group_ipc_handle(void* group, void* handle_out) {
  PeerGroup* g = static_cast<PeerGroup*>(group);
  if (g == nullptr || handle_out == nullptr) return MOE_EINVAL;
  return gcheck(g, cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), g->region),
                "cudaIpcGetMemHandle");
}

int moe_ep_group_open_peer(void* group, int32_t peer, const void* ipc_handle) {
  PeerGroup* g = static_cast<PeerGroup*>(group);
  if (g == nullptr) return MOE_EINVAL;
  if (peer < 0 || peer >= g->v.world || peer == g->v.rank) return gfail(g, MOE_EINVAL, "open_peer: bad peer %d", peer);
  if (ipc_handle == nullptr) return gfail(g, MOE_EINVAL, "open_peer: null handle");
  if (g->have[peer]) return gfail(g, MOE_EINVAL, "open_peer: peer %d already set", peer);
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  if (int rc = gcheck(g, cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle"))
    return rc;
  g->v.region[peer] = static_cast<unsigned char*>(p);
  g->opened[peer] = true;
  g->have[peer] = true;
  return MOE_OK;
}

int moe_ep_group_region(void* group, void** region_dev) {
  PeerGroup* g = static_cast<PeerGroup*>(group);
  if (g == nullptr || region_dev == nullptr) return MOE_EINVAL;
  *region_dev = g->region;
  return MOE_OK;
}

int moe_ep_group_set_peer(void* group, int32_t peer, void* region_dev) {
  PeerGroup* g = static_cast<PeerGroup*>(group);
  if (g == nullptr) return MOE_EINVAL;
  if (peer < 0 || peer >= g->v.world || peer == g->v.rank) return gfail(g, MOE_EINVAL, "set_peer: bad peer %d", peer);
  if (region_dev == nullptr || reinterpret_cast<uintptr_t>(region_dev) % 256)
    return gfail(g, MOE_EINVAL, "set_peer: region must be a 256-byte aligned device pointer");
  if (g->have[peer]) return gfail(g, MOE_EINVAL, "set_peer: peer %d already set", peer);
  g->v.region[peer] = static_cast<unsigned char*>(region_dev);
  g->have[peer] = true;
  return MOE_OK;
}

int moe_ep_peer_publish(void* group, const uint16_t* x_dev, const int64_t* topk_ids_dev, int32_t num_tokens,
                        const int32_t* slot_of_expert_dev, void* stream) {
  PeerGroup* g = static_cast<PeerGroup*>(group);
  if (g == nullptr) return MOE_EINVAL;
  if (!all_known(g)) return gfail(g, MOE_EINVAL, "publish: not every rank's region is known");
  if (g->phase != 0) return gfail(g, MOE_EINVAL, "publish: the previous step has not been combined");
  if (num_tokens < 0 || num_tokens > g->v.max_tokens)
    return gfail(g, MOE_ERANGE, "publish: %d tokens outside [0, %d]", num_tokens, g->v.max_tokens);
  if (slot_of_expert_dev == nullptr || (num_tokens > 0 && (x_dev == nullptr || topk_ids_dev == nullptr)))
    return gfail(g, MOE_EINVAL, "publish: null device pointer");
  if (reinterpret_cast<uintptr_t>(x_dev) % 16) return gfail(g, MOE_EINVAL, "publish: x must be 16-byte aligned");
  cudaGetLastError();
  moe::launch_ep_peer_publish(g->v, x_dev, topk_ids_dev, num_tokens, slot_of_expert_dev, g->epoch, g->counters,
                              g->num_sms, static_cast<cudaStream_t>(stream));
  if (int rc = gcheck(g, cudaGetLastError(), "publish launch")) return rc;
  g->published_tokens = num_tokens;
  g->phase = 1;
  return MOE_OK;
}

int moe_ep_peer_combine(void* group, const int64_t* topk_ids_dev, const uint16_t* topk_weights_dev,
                        int32_t num_tokens, uint16_t* out_dev, void* stream) {
  PeerGroup* g = static_cast<PeerGroup*>(group);
  if (g == nullptr) return MOE_EINVAL;
  if (g->phase != 2) return gfail(g, MOE_EINVAL, "combine: moe_ep_peer_experts has not run for this step");
  if (num_tokens != g->published_tokens)
    return gfail(g, MOE_EINVAL, "combine: %d tokens, %d published", num_tokens, g->published_tokens);
  if (num_tokens > 0 && (topk_ids_dev == nullptr || topk_weights_dev == nullptr || out_dev == nullptr))
    return gfail(g, MOE_EINVAL, "combine: null device pointer");
  if (reinterpret_cast<uintptr_t>(out_dev) % 8) return gfail(g, MOE_EINVAL, "combine: out must be 8-byte aligned");
  cudaGetLastError();
  moe::launch_ep_peer_combine(g->v, g->epoch, topk_ids_dev, topk_weights_dev, num_tokens, out_dev,
                              static_cast<cudaStream_t>(stream));
  if (int rc = gcheck(g, cudaGetLastError(), "combine launch")) return rc;
  g->phase = 0;
  return MOE_OK;
}

int moe_ep_group_read_status(void* group, int32_t* status, void* stream) {
  PeerGroup* g = static_cast<PeerGroup*>(group);
  if (g == nullptr || status == nullptr) return MOE_EINVAL;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, g->v.status, sizeof(v), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(g->v.status, 0, sizeof(int32_t), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (int rc = gcheck(g, e, "read_status")) return rc;
  *status = v;
  return MOE_OK;
}

int moe_ep_group_last_error(void* group, char* buf, size_t len) {
  PeerGroup* g = static_cast<PeerGroup*>(group);
  if (g == nullptr) return MOE_EINVAL;
  if (buf && len) snprintf(buf, len, "%s", g->err.c_str());
  return MOE_OK;
}

int moe_ep_group_close_peers(void* group) {
  PeerGroup* g = static_cast<PeerGroup*>(group);
  if (g == nullptr) return MOE_EINVAL;
  int rc = MOE_OK;
  for (int s = 0; s < moe::kEpMaxWorld; ++s) {
    if (g->opened[s]) {
      if (cudaIpcCloseMemHandle(g->v.region[s]) != cudaSuccess) rc = MOE_ECUDA;
      g->opened[s] = false;
    }
    if (s != g->v.rank) {
      g->have[s] = false;
      g->v.region[s] = nullptr;
    }
  }
  return rc;
}

int moe_ep_group_destroy(void* group) {
  PeerGroup* g = static_cast<PeerGroup*>(group);
  if (g == nullptr) return MOE_EINVAL;
  const int rc = moe_ep_group_close_peers(g);
  cudaFree(g->region);
  cudaFree(g->local);
  delete g;
  return rc;
}

}  // extern "C"
