// route.cu — router top-k (K1) and the token -> expert permutation (K1b).
//
// K1 follows nano_ktrans/layers/hybrid_moe.py:3321-3329 with one warp per
// token (route_warp.cuh holds the arithmetic and the tie rule).
//
// K1b replaces the reference's per-expert scan `topk_ids == e` over all E
// experts (nano_ktrans/kernels/cpu_moe.py:515-527) with one stable counting
// sort: pairs p = t*k + j are grouped by expert in ascending expert order and,
// within an expert, in ascending p (so ascending token, the reference's
// `torch.where(match.any(1))` order).
#include <math.h>

#include "common.cuh"
#include "kernels.h"
#include "route_warp.cuh"

namespace moe {

template <int EPL>
__global__ void __launch_bounds__(256) route_kernel(const uint16_t* __restrict__ logits, int T, int E, int top_k,
                                                    int use_softmax, int renorm, int64_t* __restrict__ ids,
                                                    uint16_t* __restrict__ weights) {
  const int token = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (token >= T) return;
  int id;
  float w;
  route_token_warp<EPL>(logits + static_cast<size_t>(token) * E, E, top_k, use_softmax != 0, renorm != 0, id, w);
  if (lane < top_k) {
    ids[static_cast<size_t>(token) * top_k + lane] = id;
    weights[static_cast<size_t>(token) * top_k + lane] = f32_to_bf16(w);
  }
}

void launch_route(const uint16_t* logits, int T, int E, int top_k, bool use_softmax, bool renorm, int64_t* ids,
                  uint16_t* weights, cudaStream_t st) {
  if (T <= 0) return;
  const dim3 block(256), grid((T + 7) / 8);
  const int sm = use_softmax ? 1 : 0, rn = renorm ? 1 : 0;
  if (E <= 32)
    route_kernel<1><<<grid, block, 0, st>>>(logits, T, E, top_k, sm, rn, ids, weights);
  else if (E <= 64)
    route_kernel<2><<<grid, block, 0, st>>>(logits, T, E, top_k, sm, rn, ids, weights);
  else if (E <= 128)
    route_kernel<4><<<grid, block, 0, st>>>(logits, T, E, top_k, sm, rn, ids, weights);
  else if (E <= 256)
    route_kernel<8><<<grid, block, 0, st>>>(logits, T, E, top_k, sm, rn, ids, weights);
  else if (E <= 512)
    route_kernel<16><<<grid, block, 0, st>>>(logits, T, E, top_k, sm, rn, ids, weights);
  else
    route_kernel<32><<<grid, block, 0, st>>>(logits, T, E, top_k, sm, rn, ids, weights);
}

// ---------------------------------------------------------------------------
// K0: router logits = bf16(x . Wr^T), the reference's `self.gate(hidden)`
// (nano_ktrans/models/mixtral.py:127, :212: nn.Linear(H, E, bias=False) in
// bf16, fp32 accumulation, one bf16 rounding).
//
// Warp-level tensor-core GEMM: a CTA owns 16 tokens x 8 experts (one
// m16n8k16 output tile, tokens = M, experts = N) and its 16 warps split K in
// 32-wide blocks (block b to warp b % 16); the 16 partial tiles are added in
// warp order in shared memory.  Lane (g, t) takes the 8 consecutive k of
// block b starting at 8t, from token rows g and g + 8 (A) and expert row g
// (B); the two mma steps of the block use pairs (0,1),(2,3) and (4,5),(6,7) of
// those 8 values, the same permutation of K on both operands.
//
// Latency: a warp's first kRouterPrefetch blocks of Wr are loaded before the
// programmatic-dependency wait (the router weights are not written by the
// kernel this launch may overlap: only this library's kernels trigger an early
// launch, and none of them writes router weights), so their DRAM round trip
// overlaps the previous kernel's tail; x, which the previous kernel may have
// written, is read after the wait, all of a warp's blocks at once.
// ---------------------------------------------------------------------------

constexpr int kRouterWarps = 16;
constexpr int kRouterPrefetch = 4;  // blocks per warp per round: H <= 16 * 4 * 32 = 2048 in one round

__global__ void __launch_bounds__(kRouterWarps * 32) router_logits_kernel(const uint16_t* __restrict__ x,
                                                                         const uint16_t* __restrict__ wr, int T,
                                                                         int E, int H,
                                                                         uint16_t* __restrict__ logits) {
  __shared__ float part[kRouterWarps][16][9];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int tok0 = blockIdx.y * 16, e0 = blockIdx.x * 8;
  const bool ok_a = tok0 + g < T, ok_b = tok0 + g + 8 < T, ok_w = e0 + g < E;
  const uint16_t* xa = x + static_cast<size_t>(ok_a ? tok0 + g : 0) * H + 8 * t;
  const uint16_t* xb = x + static_cast<size_t>(ok_b ? tok0 + g + 8 : 0) * H + 8 * t;
  const uint16_t* wp = wr + static_cast<size_t>(ok_w ? e0 + g : 0) * H + 8 * t;
  const int nb = H / 32;
  const uint4 z = make_uint4(0, 0, 0, 0);
  uint4 pre[kRouterPrefetch];
#pragma unroll
  for (int i = 0; i < kRouterPrefetch; ++i) {
    const int b = warp + i * kRouterWarps;
    pre[i] = ok_w && b < nb ? *reinterpret_cast<const uint4*>(wp + 32 * b) : z;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
  for (int r = 0; r * kRouterWarps * kRouterPrefetch < nb; ++r) {
    uint4 va[kRouterPrefetch], vb[kRouterPrefetch];
#pragma unroll
    for (int i = 0; i < kRouterPrefetch; ++i) {
      const int b = warp + (r * kRouterPrefetch + i) * kRouterWarps;
      const bool in = b < nb;
      va[i] = ok_a && in ? *reinterpret_cast<const uint4*>(xa + 32 * b) : z;
      vb[i] = ok_b && in ? *reinterpret_cast<const uint4*>(xb + 32 * b) : z;
      if (r > 0) pre[i] = ok_w && in ? *reinterpret_cast<const uint4*>(wp + 32 * b) : z;
    }
    uint4* vw = pre;
#pragma unroll
    for (int i = 0; i < kRouterPrefetch; ++i) {
      if (warp + (r * kRouterPrefetch + i) * kRouterWarps >= nb) break;  // warp-uniform
      asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
          "{%0,%1,%2,%3};"
          : "+f"(c0[0]), "+f"(c0[1]), "+f"(c0[2]), "+f"(c0[3])
          : "r"(va[i].x), "r"(vb[i].x), "r"(va[i].y), "r"(vb[i].y), "r"(vw[i].x), "r"(vw[i].y));
      asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
          "{%0,%1,%2,%3};"
          : "+f"(c1[0]), "+f"(c1[1]), "+f"(c1[2]), "+f"(c1[3])
          : "r"(va[i].z), "r"(vb[i].z), "r"(va[i].w), "r"(vb[i].w), "r"(vw[i].z), "r"(vw[i].w));
    }
  }
  // c[0] = (token g, expert 2t), c[1] = (g, 2t+1), c[2] = (g+8, 2t), c[3] = (g+8, 2t+1)
  part[warp][g][2 * t] = c0[0] + c1[0];
  part[warp][g][2 * t + 1] = c0[1] + c1[1];
  part[warp][g + 8][2 * t] = c0[2] + c1[2];
  part[warp][g + 8][2 * t + 1] = c0[3] + c1[3];
  __syncthreads();
  if (threadIdx.x < 128) {
    const int r = threadIdx.x >> 3, c = threadIdx.x & 7;
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kRouterWarps; ++w) v += part[w][r][c];
    if (tok0 + r < T && e0 + c < E) logits[static_cast<size_t>(tok0 + r) * E + e0 + c] = f32_to_bf16(v);
  }
}

bool router_shape_ok(int E, int H, const void* x, const void* wr) {
  return E >= 1 && H >= 32 && H % 32 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(wr) % 16 == 0;
}

void launch_router_logits(const uint16_t* x, const uint16_t* wr, int T, int E, int H, uint16_t* logits,
                          cudaStream_t st) {
  if (T <= 0) return;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((E + 7) / 8, (T + 15) / 16);
  cfg.blockDim = dim3(kRouterWarps * 32);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, router_logits_kernel, x, wr, T, E, H, logits);
}

// ---------------------------------------------------------------------------
// K1b: stable counting sort of (token, slot) pairs by expert.  One CTA of
// 1024 threads.  Shared memory: cnt[E], run[E], off[E+1], warp_sums[32],
// wcnt[32][E].
// ---------------------------------------------------------------------------

__device__ int block_incl_scan(int v, int* warp_sums) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int n = __shfl_up_sync(kFullMask, v, off);
    if (lane >= off) v += n;
  }
  if (lane == 31) warp_sums[wid] = v;
  __syncthreads();
  if (wid == 0) {
    int w = lane < static_cast<int>(blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int n = __shfl_up_sync(kFullMask, w, off);
      if (lane >= off) w += n;
    }
    warp_sums[lane] = w;
  }
  __syncthreads();
  if (wid > 0) v += warp_sums[wid - 1];
  __syncthreads();
  return v;
}

__global__ void __launch_bounds__(1024) permute_kernel(const int64_t* __restrict__ ids, int P, int E,
                                                       const uint8_t* __restrict__ mask, int skip_negative,
                                                       RouteTables rt) {
  extern __shared__ int sm[];
  int* cnt = sm;                // [E]
  int* run = cnt + E;           // [E]
  int* off = run + E;           // [E+1]
  int* warp_sums = off + E + 1; // [32]
  int* wcnt = warp_sums + 32;   // [32][E]
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;

  for (int e = tid; e < E; e += blockDim.x) {
    cnt[e] = 0;
    run[e] = 0;
  }
  for (int i = tid; i < 32 * E; i += blockDim.x) wcnt[i] = 0;
  __syncthreads();

  bool bad = false;
  for (int p = tid; p < P; p += blockDim.x) {
    const int64_t e = ids[p];
    if (e < 0 || e >= E) {
      bad |= e >= E || !skip_negative;  // negative ids mark unrouted pairs when skip_negative
      continue;
    }
    if (mask == nullptr || mask[e]) atomicAdd(&cnt[e], 1);
  }
  if (bad) atomicOr(rt.status, kStatusBadExpertId);
  __syncthreads();

  // exclusive offsets and the ascending list of active experts (E <= 1024)
  const int c = tid < E ? cnt[tid] : 0;
  const int incl = block_incl_scan(c, warp_sums);
  const int act_incl = block_incl_scan(c > 0 ? 1 : 0, warp_sums);
  if (tid < E) {
    off[tid] = incl - c;
    rt.counts[tid] = c;
    rt.offsets[tid] = incl - c;
    if (c > 0) rt.active[act_incl - 1] = tid;
  }
  if (tid == E - 1) {
    off[E] = incl;
    rt.offsets[E] = incl;
    *rt.n_active = act_incl;
  }
  __syncthreads();

  for (int base = 0; base < P; base += blockDim.x) {
    const int p = base + tid;
    int e = -1;
    if (p < P) {
      const int64_t e0 = ids[p];
      if (e0 >= 0 && e0 < E && (mask == nullptr || mask[e0])) e = static_cast<int>(e0);
    }
    const uint32_t peers = __match_any_sync(kFullMask, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank == 0) wcnt[wid * E + e] = __popc(peers);
    __syncthreads();
    for (int ee = tid; ee < E; ee += blockDim.x) {
      int r = run[ee];
      for (int w = 0; w < 32; ++w) {
        const int t = wcnt[w * E + ee];
        wcnt[w * E + ee] = r;
        r += t;
      }
      run[ee] = r;
    }
    __syncthreads();
    if (e >= 0) {
      const int pos = off[e] + wcnt[wid * E + e] + rank;
      rt.sorted_pair[pos] = p;
      rt.pair_pos[p] = pos;
    } else if (p < P) {
      rt.pair_pos[p] = -1;
    }
    __syncthreads();
    for (int i = tid; i < 32 * E; i += blockDim.x) wcnt[i] = 0;
    __syncthreads();
  }
}

void launch_permute(const int64_t* ids, int T, int top_k, int E, const uint8_t* offload_mask, const RouteTables& rt,
                    cudaStream_t st, bool skip_negative) {
  const size_t smem = sizeof(int) * (3 * static_cast<size_t>(E) + 1 + 32 + 32 * static_cast<size_t>(E));
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    configured = true;
  }
  permute_kernel<<<1, 1024, smem, st>>>(ids, T * top_k, E, offload_mask, skip_negative ? 1 : 0, rt);
}

}  // namespace moe
