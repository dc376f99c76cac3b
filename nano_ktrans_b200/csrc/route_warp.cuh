// route_warp.cuh — one warp routes one token (nano_ktrans/layers/hybrid_moe.py:3321-3329).
//
//   softmax routing (Qwen2/Qwen3): p = bf16(softmax_fp32(logits)),
//     (w, ids) = topk(p, k), and if normalize_topk_prob:
//     w = bf16(w / bf16(sum(w)))   (bf16 tensor ops: fp32 math, bf16 result)
//   Mixtral routing: (w, ids) = topk(logits, k); w = bf16(softmax_fp32(w)).
//
// Each lane holds experts lane, lane+32, ...; the k picks are made by
// repeated warp arg-max with ties broken by (value desc, expert index asc);
// NaN ranks above every number, as in torch.topk.  Lane j < k returns the
// j-th pick (expert id and bf16-rounded weight as fp32).
#pragma once

#include <math.h>

#include <type_traits>

#include "common.cuh"

namespace moe {

MOE_DEV bool rank_before(float a, int ia, float b, int ib) {
  const bool na = isnan(a), nb = isnan(b);
  if (na != nb) return na;
  if (!na && a != b) return a > b;
  return ia < ib;
}

template <int EPL>
MOE_DEV void route_token_warp(const uint16_t* __restrict__ row, int E, int top_k, bool use_softmax, bool renorm,
                              int& my_id, float& my_w) {
  const int lane = threadIdx.x & 31;
  float v[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < E ? bf16_to_f32(row[e]) : 0.0f;
  }
  if (use_softmax) {
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (i * 32 + lane < E) m = fmaxf(m, v[i]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, off));
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      if (i * 32 + lane < E) {
        v[i] = expf(v[i] - m);
        s += v[i];
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(kFullMask, s, off);
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = round_bf16(v[i] / s);
  }

  uint32_t taken = 0;
  float my_val = 0.0f;
  my_id = 0;
  for (int j = 0; j < top_k; ++j) {
    float bv = 0.0f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = i * 32 + lane;
      if (e < E && !((taken >> i) & 1u) && (bi == 0x7fffffff || rank_before(v[i], e, bv, bi))) {
        bv = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(kFullMask, bv, off);
      const int oi = __shfl_xor_sync(kFullMask, bi, off);
      if (oi != 0x7fffffff && (bi == 0x7fffffff || rank_before(ov, oi, bv, bi))) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (lane == j) {
      my_val = bv;
      my_id = bi;
    }
  }

  float w = my_val;
  if (use_softmax) {
    if (renorm) {
      float s = 0.0f;  // sequential sum in slot order (a bf16 sum accumulates in fp32)
      for (int j = 0; j < top_k; ++j) s += __shfl_sync(kFullMask, my_val, j);
      w = my_val / round_bf16(s);
    }
  } else {
    const float m = __shfl_sync(kFullMask, my_val, 0);
    const float ex = lane < top_k ? expf(my_val - m) : 0.0f;
    float s = 0.0f;
    for (int j = 0; j < top_k; ++j) s += __shfl_sync(kFullMask, ex, j);
    w = ex / s;
  }
  my_w = round_bf16(w);
}

// Dispatch on experts-per-lane.  F is called as F(integral_constant<EPL>).
template <typename F>
MOE_DEV void with_epl(int E, F&& f) {
  if (E <= 32) f(std::integral_constant<int, 1>{});
  else if (E <= 64) f(std::integral_constant<int, 2>{});
  else if (E <= 128) f(std::integral_constant<int, 4>{});
  else if (E <= 256) f(std::integral_constant<int, 8>{});
  else if (E <= 512) f(std::integral_constant<int, 16>{});
  else f(std::integral_constant<int, 32>{});
}

}  // namespace moe
