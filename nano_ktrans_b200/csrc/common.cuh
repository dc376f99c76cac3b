// common.cuh — device helpers shared by the routed-expert kernels (sm_100a).
//
// Dequantization arithmetic.  A quantized weight is (q - 2^(bits-1)) * s with
// q an unsigned code and s a bf16 group scale (nano_ktrans/kernels/
// weight_loader.py:57-69).  The kernels never build that product: they form
// (q - z) exactly in fp32 and fold s in once per 16-byte chunk, so every
// partial product is exact and only the fp32 accumulation rounds — the same
// arithmetic class as the reference's fp32 F.linear over exactly dequantized
// weights (quantized_ops.py:86-124).
//
// W4 unpack (per 32-bit word, 8 codes along K, code j at bits 4j):
//   OR-ing a code, left where it sits, into the exponent pattern of 2^23
//   gives the float 2^23 + q * 16^p, where p is the code's nibble position in
//   the word.  Subtracting 2^23 + 8 * 16^p is exact and leaves
//   (q - 8) * 16^p.  Codes 0..4 sit at p = 0..4; codes 5..7 are first moved
//   down by 12 bits (p = 2..4) so every code stays inside the 23-bit
//   mantissa.  The matching activation is pre-scaled by 16^-p (a power of two,
//   exact), so (q - 8) * 16^p * x * 16^-p == (q - 8) * x with no rounding in
//   the product.  Cost: 8 LOP3 + 1 shift + 4 packed adds + 4 packed FMAs per
//   8 weights.
// W8 unpack (per word, 4 codes, code j at bits 8j): a byte permute places the
//   code in the low byte of 2^23's bit pattern (2^23 + q); subtracting
//   2^23 + 128 leaves (q - 128) exactly; activations are not pre-scaled.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define MOE_DEV __device__ __forceinline__

namespace moe {

constexpr uint32_t kFullMask = 0xffffffffu;
constexpr int kStatusBadExpertId = 1;  // an expert id outside [0, E) was skipped
constexpr int kStatusTimeout = 2;      // a bounded wait expired; outputs of that call are invalid

MOE_DEV float bf16_to_f32(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }

MOE_DEV uint16_t f32_to_bf16(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }

// Round an fp32 value to the nearest bf16 value, returned as fp32.
MOE_DEV float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

// 16-byte streaming load that does not allocate in L1: expert weights are
// read once per launch.
MOE_DEV uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ---------------------------------------------------------------------------
// W4
// ---------------------------------------------------------------------------

// Nibble position p of code j (0..7) after the (w, w >> 12) split.
__host__ __device__ constexpr int w4_pos(int j) { return j < 5 ? j : j - 3; }

// Activation pre-scale 16^-p for code j of a word.
__host__ __device__ constexpr float w4_prescale(int j) {
  return w4_pos(j) == 0   ? 1.0f
         : w4_pos(j) == 1 ? 0.0625f
         : w4_pos(j) == 2 ? 0.00390625f
         : w4_pos(j) == 3 ? 0.000244140625f
                          : 0.0000152587890625f;
}

// (q_j - 8) * 16^p_j for the 8 codes of a word, as 4 float2 pairs (j, j+1).
MOE_DEV void w4_unpack(uint32_t w, float2& d01, float2& d23, float2& d45, float2& d67) {
  constexpr uint32_t E = 0x4B000000u;  // bit pattern of 2^23
  const uint32_t w2 = w >> 12;
  const float a0 = __uint_as_float((w & 0x0000000Fu) | E);
  const float a1 = __uint_as_float((w & 0x000000F0u) | E);
  const float a2 = __uint_as_float((w & 0x00000F00u) | E);
  const float a3 = __uint_as_float((w & 0x0000F000u) | E);
  const float a4 = __uint_as_float((w & 0x000F0000u) | E);
  const float a5 = __uint_as_float((w2 & 0x00000F00u) | E);
  const float a6 = __uint_as_float((w2 & 0x0000F000u) | E);
  const float a7 = __uint_as_float((w2 & 0x000F0000u) | E);
  // 2^23 + 8 * 16^p for p = 0..4: 8388616, 8388736, 8390656, 8421376, 8912896
  d01 = __fadd2_rn(make_float2(a0, a1), make_float2(-8388616.0f, -8388736.0f));
  d23 = __fadd2_rn(make_float2(a2, a3), make_float2(-8390656.0f, -8421376.0f));
  d45 = __fadd2_rn(make_float2(a4, a5), make_float2(-8912896.0f, -8390656.0f));
  d67 = __fadd2_rn(make_float2(a6, a7), make_float2(-8421376.0f, -8912896.0f));
}

// acc += sum_j (q_j - 8) * x_j for one word, activations pre-scaled by
// w4_prescale: xa = (x'0..x'3), xb = (x'4..x'7).
MOE_DEV float2 w4_word_fma(uint32_t w, float4 xa, float4 xb, float2 acc) {
  float2 d01, d23, d45, d67;
  w4_unpack(w, d01, d23, d45, d67);
  acc = __ffma2_rn(d01, make_float2(xa.x, xa.y), acc);
  acc = __ffma2_rn(d23, make_float2(xa.z, xa.w), acc);
  acc = __ffma2_rn(d45, make_float2(xb.x, xb.y), acc);
  acc = __ffma2_rn(d67, make_float2(xb.z, xb.w), acc);
  return acc;
}

// ---------------------------------------------------------------------------
// W8
// ---------------------------------------------------------------------------

MOE_DEV void w8_unpack(uint32_t w, float2& d01, float2& d23) {
  constexpr uint32_t E = 0x4B000000u;
  const float a0 = __uint_as_float(__byte_perm(w, E, 0x7540));
  const float a1 = __uint_as_float(__byte_perm(w, E, 0x7541));
  const float a2 = __uint_as_float(__byte_perm(w, E, 0x7542));
  const float a3 = __uint_as_float(__byte_perm(w, E, 0x7543));
  const float2 off = make_float2(-8388736.0f, -8388736.0f);  // 2^23 + 128
  d01 = __fadd2_rn(make_float2(a0, a1), off);
  d23 = __fadd2_rn(make_float2(a2, a3), off);
}

MOE_DEV float2 w8_word_fma(uint32_t w, float4 xa, float2 acc) {
  float2 d01, d23;
  w8_unpack(w, d01, d23);
  acc = __ffma2_rn(d01, make_float2(xa.x, xa.y), acc);
  acc = __ffma2_rn(d23, make_float2(xa.z, xa.w), acc);
  return acc;
}

// ---------------------------------------------------------------------------
// Chunk-level helpers.  A chunk is 16 bytes of one weight row: 32 codes (W4)
// or 16 codes (W8).  Its activations are kQ float4 (8 for W4, 4 for W8).
// ---------------------------------------------------------------------------

template <int BITS>
struct ChunkTraits {
  static constexpr int kCodes = 128 / BITS;  // codes per 16-byte chunk
  static constexpr int kQ = kCodes / 4;      // float4 of activations per chunk
};

// Pre-scale of activation k (W4 only): depends on k mod 8.
template <int BITS>
MOE_DEV float act_prescale(int k) {
  if constexpr (BITS == 4) {
    const int j = k & 7;
    return j == 0 ? 1.0f
           : j == 1 ? 0.0625f
           : (j == 2 || j == 5) ? 0.00390625f
           : (j == 3 || j == 6) ? 0.000244140625f
                                : 0.0000152587890625f;
  } else {
    return 1.0f;
  }
}

// Dot of one chunk with its activations (read from shared memory at
// `xs4[q * stride4]`, q = 0..kQ-1), unscaled by the group scale.
template <int BITS>
MOE_DEV float chunk_dot(uint4 wv, const float4* xs4, int stride4) {
  float2 acc = make_float2(0.f, 0.f);
  if constexpr (BITS == 4) {
    acc = w4_word_fma(wv.x, xs4[0 * stride4], xs4[1 * stride4], acc);
    acc = w4_word_fma(wv.y, xs4[2 * stride4], xs4[3 * stride4], acc);
    acc = w4_word_fma(wv.z, xs4[4 * stride4], xs4[5 * stride4], acc);
    acc = w4_word_fma(wv.w, xs4[6 * stride4], xs4[7 * stride4], acc);
  } else {
    acc = w8_word_fma(wv.x, xs4[0 * stride4], acc);
    acc = w8_word_fma(wv.y, xs4[1 * stride4], acc);
    acc = w8_word_fma(wv.z, xs4[2 * stride4], acc);
    acc = w8_word_fma(wv.w, xs4[3 * stride4], acc);
  }
  return acc.x + acc.y;
}

// ---------------------------------------------------------------------------
// W4 with bf16 operands (gate/up, whose activations are bf16).
//
// Moving a nibble pair into bits 0-3 of each 16-bit half and OR-ing it into
// 0x4300 (bf16 128.0, mantissa step 1) gives two exact bf16 values 128 + q per
// logic op (a bf16 mantissa has 7 bits, so the nibble must sit in bits 0-3).
// Every product x * (128 + q) is exact in the fp32 accumulator of
// fma.rn.f32.bf16, and
//   sum_j (q_j - 8) * x_j = sum_j x_j * (128 + q_j) - 136 * sum_j x_j,
// the second term being one fp32 correction per chunk and token.
// Per 8 weights: 3 shifts + 4 logic ops + 8 mixed-precision FMAs, against
// 9 logic ops + 8 fp32 adds/FMAs for the fp32 unpack above.
//
// Activation operands of one word (codes k0..k0+7): the 4 bf16x2 registers
// (x0, x4), (x1, x5), (x2, x6), (x3, x7) — matching the nibble pairs
// (0,4) (1,5) (2,6) (3,7) of the word shifted right by 0, 4, 8 and 12 bits.
// ---------------------------------------------------------------------------

// (x & mask) | bits in one LOP3 (LUT 0xEA = (a & b) | c).  Written out because
// the compiler does not always fuse the AND and the OR, and the nibble unpacks
// of the W4 kernels are bound by this ALU work.
MOE_DEV uint32_t and_or(uint32_t x, uint32_t mask, uint32_t bits) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(x), "r"(mask), "r"(bits));
  return r;
}

// Nibble pair of x at bits 0-3 and 16-19 as two exact bf16 values 128 + q.
MOE_DEV uint32_t nib_bf16(uint32_t x) { return and_or(x, 0x000F000Fu, 0x43004300u); }

MOE_DEV uint32_t pack_bf16x2(uint16_t lo, uint16_t hi) { return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16); }

// raw = 8 consecutive bf16 activations (x0..x7, two per 32-bit word, low half
// first).  Returns the word's 4 operand registers; adds its share of the
// chunk correction to `corr`.
MOE_DEV uint4 w4_pack_x(uint4 raw, float& corr) {
  const float x0 = __uint_as_float(raw.x << 16), x1 = __uint_as_float(raw.x & 0xffff0000u);
  const float x2 = __uint_as_float(raw.y << 16), x3 = __uint_as_float(raw.y & 0xffff0000u);
  const float x4 = __uint_as_float(raw.z << 16), x5 = __uint_as_float(raw.z & 0xffff0000u);
  const float x6 = __uint_as_float(raw.w << 16), x7 = __uint_as_float(raw.w & 0xffff0000u);
  corr += 136.0f * (((x0 + x1) + (x2 + x3)) + ((x4 + x5) + (x6 + x7)));
  // (x0,x4) (x1,x5) (x2,x6) (x3,x7): byte permutes of the raw pairs
  return make_uint4(__byte_perm(raw.x, raw.z, 0x5410), __byte_perm(raw.x, raw.z, 0x7632),
                    __byte_perm(raw.y, raw.w, 0x5410), __byte_perm(raw.y, raw.w, 0x7632));
}

MOE_DEV void fma2_f32_bf16(float& a0, float& a1, uint32_t x, uint32_t v) {
  asm("{\n\t.reg .b16 xl, xh, vl, vh;\n\tmov.b32 {xl, xh}, %2;\n\tmov.b32 {vl, vh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, xl, vl, %0;\n\tfma.rn.f32.bf16 %1, xh, vh, %1;\n}"
      : "+f"(a0), "+f"(a1)
      : "r"(x), "r"(v));
}

// Dot of one 16-byte W4 chunk (4 words, 32 codes) with its bf16 operands
// (xq[q * stride4], q = 0..3), minus the chunk correction; unscaled by the
// group scale.
MOE_DEV float w4_chunk_dot_bf16(uint4 wv, const uint4* xq, int stride4, float corr) {
  float a0 = 0.0f, a1 = 0.0f;
  const uint32_t w[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t ww = w[q];
    const uint4 xv = xq[q * stride4];
    fma2_f32_bf16(a0, a1, xv.x, nib_bf16(ww));
    fma2_f32_bf16(a0, a1, xv.y, nib_bf16(ww >> 4));
    fma2_f32_bf16(a0, a1, xv.z, nib_bf16(ww >> 8));
    fma2_f32_bf16(a0, a1, xv.w, nib_bf16(ww >> 12));
  }
  return (a0 + a1) - corr;
}

MOE_DEV float silu_f32(float v) { return v / (1.0f + expf(-v)); }

MOE_DEV float sigmoid_f32(float v) { return 1.0f / (1.0f + expf(-v)); }

}  // namespace moe
