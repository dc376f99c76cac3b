// mma_gemv.cuh — W4 matrix-vector products on the warp-level tensor-core path
// (mma.sync m16n8k16, bf16 operands, fp32 accumulate; sm_100a).
//
// A 16-row weight tile is the A operand, the activation vector is broadcast to
// all 8 columns of B, so every column of D carries the same 16 row sums and no
// cross-lane reduction is needed afterwards.  One mma covers 16 rows x 16 codes;
// a warp turns its 32 lanes' share of a 128-code group into 8 of them.
//
// Lane (g = lane / 4, t = lane % 4) owns the codes [32t, 32t + 32) of the group
// in tile rows g and g + 8 (16 bytes of each row) and the operand words of the
// same 32 activations.  The logical K order inside an mma is a permutation of
// the physical one that both operands share: for word q of the lane's 16 bytes,
// step 2q pairs nibbles (0,4) and (1,5), step 2q + 1 pairs (2,6) and (3,7) —
// exactly the activation pairs w4_pack_x (common.cuh) produces.
//
// Every code enters as the exact bf16 value 128 + q (the nibble OR-ed into the
// pattern of 128.0, as in w4_chunk_dot_bf16), every product is exact, and the
// caller subtracts 136 * sum(x) per group, so the group sum equals
// sum (q - 8) x up to fp32 accumulation.
#pragma once

#include "common.cuh"

namespace moe {

// D += A (16 x 16) * B (16 x 8), bf16 x bf16 -> fp32.
MOE_DEV void mma16816_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                           uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 128-code group of a W4 tile.  wlo / whi: the lane's 16 code bytes of
// tile rows g and g + 8; xr: the operand words of its 32 activations (read
// one word at a time).  Returns in d[0] (= d[1]) the group sum
// sum (128 + q) x of row g and in d[2] (= d[3]) that of row g + 8 (per column
// of B when B differs by column, see the callers).  A dependent mma costs a
// few hundred cycles of latency, so the 8 steps go to 4 independent
// accumulators (chains of 2), added in a fixed order at the end.
MOE_DEV void w4_group_mma(uint4 wlo, uint4 whi, const uint4* xr, float (&d)[4]) {
  const uint32_t u[4] = {wlo.x, wlo.y, wlo.z, wlo.w};
  const uint32_t v[4] = {whi.x, whi.y, whi.z, whi.w};
  float e[4][4];
#pragma unroll
  for (int s = 0; s < 4; ++s) e[s][0] = e[s][1] = e[s][2] = e[s][3] = 0.0f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 x = xr[q];
    mma16816_bf16(e[(2 * q) & 3], nib_bf16(u[q]), nib_bf16(v[q]), nib_bf16(u[q] >> 4), nib_bf16(v[q] >> 4),
                  x.x, x.y);
    mma16816_bf16(e[(2 * q + 1) & 3], nib_bf16(u[q] >> 8), nib_bf16(v[q] >> 8), nib_bf16(u[q] >> 12),
                  nib_bf16(v[q] >> 12), x.z, x.w);
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) d[r] = (e[0][r] + e[1][r]) + (e[2][r] + e[3][r]);
}

// fp32 value -> (hi, lo) bf16 with hi + lo == v to 16 significant bits.
MOE_DEV void split_bf16(float v, uint16_t& hi, uint16_t& lo) {
  hi = f32_to_bf16(v);
  lo = f32_to_bf16(v - bf16_to_f32(hi));
}

}  // namespace moe
