// ep.cu — expert-parallel dispatch/combine helpers.
//
// Expert parallelism splits the routed experts of a layer across the ranks
// of a process group.  Each expert e lives on one rank as a "slot"
// g = owner(e) * experts_per_rank + local(e).  A rank routes its own tokens,
// then sends every (token, slot) pair to the slot's owner: the pairs are
// sorted by slot (so by destination rank, then local expert) with the same
// stable counting sort as the single-GPU path, and the token rows are
// gathered into that order.  The owners run their experts on the rows they
// received and send one fp32 output row back per pair, in the order received;
// the token's rank then combines them exactly as the single-GPU path does
// (slots in ascending global expert order, fp32, one bf16 rounding).
//
// No counterpart in the reference (its offload backends are single-device);
// the combine order follows nano_ktrans/kernels/cpu_moe.py:515-538.
#include "common.cuh"
#include "kernels.h"

namespace moe {

// g[p] = slot_of_expert[ids[p]]; ids outside [0, E) become `num_slots` (flagged
// and excluded by the permute kernel).
__global__ void ep_remap_kernel(const int64_t* __restrict__ ids, int P, const int32_t* __restrict__ slot_of_expert,
                                int E, int num_slots, int64_t* __restrict__ g) {
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < P; p += gridDim.x * blockDim.x) {
    const int64_t e = ids[p];
    g[p] = (e >= 0 && e < E) ? static_cast<int64_t>(slot_of_expert[e]) : static_cast<int64_t>(num_slots);
  }
}

// send_rows[s] = x[token of sorted pair s]; send_local[s] = local expert of
// that pair's slot.  One warp per row, 16-byte copies.
__global__ void ep_gather_kernel(const uint16_t* __restrict__ x, const int32_t* __restrict__ sorted_pair,
                                 const int32_t* __restrict__ offsets, int num_slots, const int64_t* __restrict__ g,
                                 int top_k, int H, int experts_per_rank, uint16_t* __restrict__ send_rows,
                                 int64_t* __restrict__ send_local) {
  const int P = offsets[num_slots];
  const int lane = threadIdx.x & 31;
  const int vec = H / 8;  // uint4 per row
  for (int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < P; s += (gridDim.x * blockDim.x) >> 5) {
    const int p = sorted_pair[s];
    const int t = p / top_k;
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H);
    uint4* dst = reinterpret_cast<uint4*>(send_rows + static_cast<size_t>(s) * H);
    for (int i = lane; i < vec; i += 32) dst[i] = src[i];
    if (lane == 0) send_local[s] = g[p] % experts_per_rank;
  }
}

// rows[r] = y[pos[r]] (fp32 rows, float4 copies).
__global__ void ep_scatter_rows_kernel(const int32_t* __restrict__ pos, int n, int H, const float* __restrict__ y,
                                       float* __restrict__ rows) {
  const int v = H / 4;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n * v; i += gridDim.x * blockDim.x) {
    const int r = i / v, c = i - r * v;
    const int s = pos[r];
    float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
    if (s >= 0) val = reinterpret_cast<const float4*>(y + static_cast<size_t>(s) * H)[c];
    reinterpret_cast<float4*>(rows + static_cast<size_t>(r) * H)[c] = val;
  }
}

void launch_ep_remap(const int64_t* ids, int P, const int32_t* slot_of_expert, int E, int num_slots, int64_t* g,
                     cudaStream_t st) {
  if (P <= 0) return;
  const int grid = (P + 255) / 256 < 1024 ? (P + 255) / 256 : 1024;
  ep_remap_kernel<<<grid, 256, 0, st>>>(ids, P, slot_of_expert, E, num_slots, g);
}

void launch_ep_gather(const uint16_t* x, const RouteTables& rt, int num_slots, const int64_t* g, int top_k, int H,
                      int experts_per_rank, int max_pairs, uint16_t* send_rows, int64_t* send_local, int num_sms,
                      cudaStream_t st) {
  if (max_pairs <= 0) return;
  const int warps = max_pairs < num_sms * 32 ? max_pairs : num_sms * 32;
  ep_gather_kernel<<<(warps + 7) / 8, 256, 0, st>>>(x, rt.sorted_pair, rt.offsets, num_slots, g, top_k, H,
                                                     experts_per_rank, send_rows, send_local);
}

void launch_scatter_rows(const int32_t* pos, int n, int H, const float* y, float* rows, int num_sms,
                         cudaStream_t st) {
  const long long work = static_cast<long long>(n) * (H / 4);
  if (work <= 0) return;
  const long long blocks = (work + 255) / 256;
  const int grid = static_cast<int>(blocks < num_sms * 16LL ? blocks : num_sms * 16LL);
  ep_scatter_rows_kernel<<<grid, 256, 0, st>>>(pos, n, H, y, rows);
}

}  // namespace moe
