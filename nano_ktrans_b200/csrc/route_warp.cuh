// route_warp.cuh — one warp routes one token (nano_ktrans/layers/hybrid_moe.py:3321-3329).
//
//   softmax routing (Qwen2/Qwen3): p = bf16(softmax_fp32(logits)),
//     (w, ids) = topk(p, k), and if normalize_topk_prob:
//     w = bf16(w / bf16(sum(w)))   (bf16 tensor ops: fp32 math, bf16 result)
//   Mixtral routing: (w, ids) = topk(logits, k); w = bf16(softmax_fp32(w)).
//
// Ranking.  Every candidate becomes one unique 32-bit key: the high 16 bits
// are an order-preserving image of its bf16 value (NaN mapped to the top, as
// torch.topk ranks NaN first), the low 16 bits are 0xFFFF - expert, so equal
// values rank by ascending expert index.  Each of the k picks is one
// warp-wide `redux.sync.max` over the lanes' best remaining keys, instead of
// a shuffle tree of compare-and-select steps.  Lane j < k returns the j-th
// pick (expert id and bf16-rounded weight as fp32).
#pragma once

#include <math.h>

#include <type_traits>

#include "common.cuh"

namespace moe {

// Monotonic map fp32 -> uint32 (a < b  <=>  key(a) < key(b) for non-NaN).
MOE_DEV uint32_t order_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

MOE_DEV float order_key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Key of a bf16-valued fp32 candidate `v` for expert `e`.
MOE_DEV uint32_t rank_key(float v, int e) {
  const uint32_t hi = isnan(v) ? 0xffff0000u : (order_key(v) & 0xffff0000u);
  return hi | static_cast<uint32_t>(0xffff - e);
}

// bf16 value carried by a rank key (NaN keys return a NaN).
MOE_DEV float rank_key_value(uint32_t key) {
  const uint32_t hi = key & 0xffff0000u;
  return __uint_as_float((hi & 0x80000000u) ? (hi & 0x7fff0000u) : (~hi & 0xffff0000u));
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
    uint32_t mk = 0;
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (i * 32 + lane < E) mk = max(mk, order_key(v[i]));
    const float m = order_key_value(__reduce_max_sync(kFullMask, mk));
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
  uint32_t key[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    key[i] = e < E ? rank_key(v[i], e) : 0u;  // valid keys are never 0
  }

  // each lane's keys in descending order (compare-exchange passes on registers)
#pragma unroll
  for (int p = 0; p < EPL - 1; ++p) {
#pragma unroll
    for (int i = 0; i < EPL - 1 - p; ++i) {
      const uint32_t hi = max(key[i], key[i + 1]), lo = min(key[i], key[i + 1]);
      key[i] = hi;
      key[i + 1] = lo;
    }
  }
  float my_val = 0.0f, sum = 0.0f, v0 = 0.0f, exsum = 0.0f;
  my_id = 0;
#pragma unroll 1
  for (int j = 0; j < top_k; ++j) {
    const uint32_t m = __reduce_max_sync(kFullMask, key[0]);
    if (key[0] == m) {  // keys are unique: exactly one lane owns the pick and drops it
#pragma unroll
      for (int i = 0; i < EPL - 1; ++i) key[i] = key[i + 1];
      key[EPL - 1] = 0;
    }
    const float val = rank_key_value(m);
    if (lane == j) {
      my_val = val;
      my_id = 0xffff - static_cast<int>(m & 0xffffu);
    }
    sum += val;  // slot-order fp32 sum (a bf16 sum accumulates in fp32)
    if (j == 0) v0 = val;
    if (!use_softmax) exsum += expf(val - v0);  // Mixtral: softmax over the picks
  }

  float w = my_val;
  if (use_softmax) {
    if (renorm) w = my_val / round_bf16(sum);
  } else {
    w = expf(my_val - v0) / exsum;
  }
  my_w = round_bf16(w);
}

}  // namespace moe
