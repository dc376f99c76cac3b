// grouped_gemm.cu — prefill path: per-expert grouped GEMM on tcgen05 tensor
// cores, the quantized weights dequantized on the fly into tensor memory.
//
// Replaces, for batches with several tokens per expert, the per-expert loop of
// nano_ktrans/kernels/cpu_moe.py:515-536 (gate/up/down via the grouped W4A32
// matvec, quantized_ops.py:86-124, SiLU(gate)*up at cpu_moe.py:448).
//
// Orientation ("swap AB"): the MMA's M = 128 weight rows (output features),
// N = 16..128 tokens of one expert (the token-tile width), K = the reduction
// dimension in steps of 64.
//   A  (weights)     fp16, dequantized by CUDA cores from the W4/W8 codes and
//                    stored straight into tensor memory (tcgen05.st);
//   B  (activations) fp16 [pairs, K] in expert-sorted pair order, loaded by
//                    TMA (tensor map, 128-byte swizzle) into shared memory;
//   D               fp32 in tensor memory.
// Exactness: (q - z) * s has at most 3+8 (W4) significant bits, so it is
// exact in fp16; W8 per-channel uses (q - 128) (exact) and applies the scale
// in the epilogue.  Activations are bf16 inputs converted to fp16 (exact for
// magnitudes in [2^-14, 65504]) and the SiLU*up intermediate is rounded to
// fp16 once.  Products are exact, accumulation is fp32.
//
// K order: the dequant writes each word's codes in the order its nibble /
// byte extraction produces them (W4: 0,4,1,5,2,6,3,7 within each 8 codes;
// W8: 0,2,1,3 within each 4).  A GEMM is unchanged by a permutation of K
// applied to both operands, so the activation buffers are written in that
// same order (pack_x_kernel, and the gate/up epilogue for the down GEMM).
//
// CTA roles (320 threads): warp 0 issues the TMA loads; warp 1 owns TMEM and
// one lane issues the MMAs; warps 2-9 (two per TMEM lane quarter, thread =
// weight row x half of the K step) dequantize, then run the epilogue from
// TMEM.  Stages are handed over with mbarriers; every wait is bounded and
// records kStatusTimeout on expiry.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace moe {
namespace gg {

constexpr int BM = kGemmBM;  // weight rows per tile
constexpr int BK = kGemmBK;  // K per stage (one 128-byte fp16 row)
constexpr uint32_t kSpin = 1u << 22;  // bounded waits: the kernel records kStatusTimeout and unwinds

#ifdef MOE_GEMM_TRACE
// Instrumented builds only: per-CTA %globaltimer stamps and cycle sums of the last launch.
constexpr int kTraceCtas = 1 << 15;
__device__ unsigned long long g_gemm_trace[2][kTraceCtas][16];  // [down, gate/up][cta][stamp / cycle sum]
template <bool GATEUP>
MOE_DEV void stamp(int i) {
  if (blockIdx.x < kTraceCtas) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g_gemm_trace[GATEUP ? 1 : 0][blockIdx.x][i] = t;
  }
}
#define GG_STAMP(i) stamp<GATEUP>(i)
#define GG_SUM(i, v) \
  if (blockIdx.x < kTraceCtas) g_gemm_trace[GATEUP ? 1 : 0][blockIdx.x][i] = static_cast<unsigned long long>(v)
MOE_DEV long long gg_clock() { return clock64(); }
#else
#define GG_STAMP(i) ((void)0)
#define GG_SUM(i, v) ((void)0)
MOE_DEV long long gg_clock() { return 0; }
#endif

MOE_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

MOE_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
MOE_DEV void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
MOE_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
MOE_DEV bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpin; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// 2-D tiled TMA load, global -> this CTA's shared memory (no multicast).
MOE_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// K-major operand tile with the 128-byte swizzle: rows of 128 bytes, 8-row
// groups 1024 bytes apart (stride byte offset), descriptor version 1.
MOE_DEV uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);  // start address
  d |= static_cast<uint64_t>(1) << 16;                 // leading byte offset (unused when swizzled)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;         // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;                 // descriptor version
  d |= static_cast<uint64_t>(2) << 61;                 // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: D f32, A f16, B f16, both K-major, M x N.
template <int N>
constexpr uint32_t idesc_f16() {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
}

template <int N>
MOE_DEV void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc_f16<N>()), "r"(accumulate)
      : "memory");
}

MOE_DEV void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 16 consecutive fp32 columns of this warp's 32 TMEM lanes.
MOE_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Position, within its group of 8, at which code/feature j of that group is
// stored in the K-permuted activation layout.
template <int BITS>
MOE_DEV int kpos(int j) {
  if constexpr (BITS == 4) {
    return (j & 3) * 2 + (j >> 2);  // codes 0,4,1,5,2,6,3,7 -> j = 0..7 at 0,2,4,6,1,3,5,7
  } else {
    return (j & 4) + ((j & 1) << 1) + ((j >> 1) & 1);  // 0,2,1,3 within each 4
  }
}

// Dequantize 16 bytes of codes (32 W4 or 16 W8 codes) of one row into fp16
// in storage order; `sc` is the row's fp16 scale (ignored for W8).
template <int BITS>
MOE_DEV void dequant16(uint4 c, __half2 sc, uint4* out) {
  const uint32_t w[4] = {c.x, c.y, c.z, c.w};
  if constexpr (BITS == 4) {
    const __half2 bias = __float2half2_rn(1032.0f);  // 1024 + 8
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t v[4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const uint32_t m = and_or(w[q] >> (4 * s), 0x000F000Fu, 0x64006400u);  // fp16 (1024 + q_s, 1024 + q_{s+4})
        __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&m), bias);    // q - 8, exact
        h = __hmul2(h, sc);                                                  // (q - 8) * s, exact
        v[s] = *reinterpret_cast<uint32_t*>(&h);
      }
      out[q] = make_uint4(v[0], v[1], v[2], v[3]);
    }
  } else {
    const __half2 bias = __float2half2_rn(1152.0f);  // 1024 + 128
    uint32_t v[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t m02 = __byte_perm(w[q], 0x64646464u, 0x4240);  // fp16 (1024 + b0, 1024 + b2)
      const uint32_t m13 = __byte_perm(w[q], 0x64646464u, 0x4341);  // fp16 (1024 + b1, 1024 + b3)
      __half2 h0 = __hsub2(*reinterpret_cast<const __half2*>(&m02), bias);
      __half2 h1 = __hsub2(*reinterpret_cast<const __half2*>(&m13), bias);
      v[2 * q] = *reinterpret_cast<uint32_t*>(&h0);
      v[2 * q + 1] = *reinterpret_cast<uint32_t*>(&h1);
    }
    out[0] = make_uint4(v[0], v[1], v[2], v[3]);
    out[1] = make_uint4(v[4], v[5], v[6], v[7]);
  }
}

struct GemmArgs {
  const int32_t* offsets;   // [E+1]
  const int32_t* active;    // [E]
  const int32_t* n_active;  // [1]
  const int32_t* tile_off;  // [E+1] token-tile prefix over active experts
  const uint16_t* s0;       // scales of projection 0 (gate or down)
  const uint16_t* s1;       // scales of projection 1 (up)
  int sstride, group;
  int N, K;                 // rows per expert, reduction dim
  __half* hout;             // gate/up: SiLU*up [pairs][N] (K-permuted within 8)
  float* yout;              // down: y [pairs][N]
  int* status;
};

// Operand staging.
//   load ring (shared memory, kLS stages): activation tile [BN][64] fp16 and
//     code tile(s) [BM][64*BITS/8], filled by TMA;
//   operand ring (tensor memory, kOS stages): the dequantized weight tile(s)
//     [BM][64] fp16, written by the dequant warps with tcgen05.st, one TMEM
//     lane per weight row, two fp16 per 32-bit column along K (32 columns per
//     projection per stage).  The MMAs read A from tensor memory and B from
//     shared memory, so the dequantized weights never pass through shared
//     memory.
// Tensor memory: [accumulators kNP x BN columns][operand stages kOS x kNP x 32].
// A load stage is released when the MMAs that read it complete, which is after
// the dequant warps consumed its codes (the MMAs wait for their operands).
template <int BITS, bool GATEUP, int BN>
struct Plan {
  static constexpr int kCodeRow = BK * BITS / 8;  // code bytes per row per stage
  static constexpr int kNP = GATEUP ? 2 : 1;
  static constexpr int kX = BN * 128;             // activation tile
  static constexpr int kC = BM * kCodeRow;        // code tile, per projection
  static constexpr int kLoad = kX + kNP * kC;
  static constexpr int kACols = BK / 2;           // TMEM columns of one dequantized tile
  static constexpr int kAccCols = kNP * BN;
  // operand stages: as many as the 512 TMEM columns hold beside the accumulators (at most 12)
  static constexpr int kOSraw = (512 - kAccCols) / (kNP * kACols);
  static constexpr int kOS = kOSraw > 12 ? 12 : kOSraw;
  static constexpr int kTmemUsed = kAccCols + kOS * kNP * kACols;
  static constexpr int kTmemCols = kTmemUsed <= 32 ? 32 : kTmemUsed <= 64 ? 64 : kTmemUsed <= 128 ? 128
                                   : kTmemUsed <= 256 ? 256 : 512;  // allocation: power of two
  static constexpr int kBudget = 232448 - 2048;   // opt-in limit minus barriers and alignment slack
  static constexpr int kLSraw = kBudget / kLoad;
  static constexpr int kLS = kLSraw > 16 ? 16 : kLSraw;
  static constexpr int kBarOff = kLS * kLoad;
  static constexpr int kNumBars = 2 * kLS + 2 * kOS + 1;
  // at least 116 KB of shared memory, so one CTA per SM holds the tensor memory it allocates
  static constexpr int kBytesRaw = kBarOff + 8 * kNumBars + 16 + 1024;
  static constexpr int kBytes = kBytesRaw < 118784 ? 118784 : kBytesRaw;
  static_assert(kLS >= 4 && kOS >= 4, "rings too shallow");
  static_assert(kTmemUsed <= 512, "tensor memory plan exceeds 512 columns");
  static_assert(kLoad % 1024 == 0, "tiles must stay 1024-byte aligned");
  static_assert(kBytes <= 232448, "shared-memory plan exceeds the opt-in limit");
};

constexpr int kDqWarps = 8;                         // dequant + epilogue warps (2 per TMEM lane quarter)
constexpr int kThreadsV2 = 64 + 32 * kDqWarps;      // + producer warp + MMA warp

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16, M = 128, N = BN.
template <int N>
MOE_DEV void umma_ts_f16(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc_f16<N>()), "r"(accumulate)
      : "memory");
}

// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes from registers.
MOE_DEV void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

template <int BITS, bool GATEUP, int BN>
__global__ void __launch_bounds__(kThreadsV2, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w0,
                        const __grid_constant__ CUtensorMap tm_w1, GemmArgs a) {
  using L = Plan<BITS, GATEUP, BN>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- CTA -> (expert, feature block, token tile) ----
  // Expert-major, then feature block, token tiles fastest: the CTAs that
  // share one weight tile run side by side, so it leaves HBM once and the
  // other token tiles read it from L2.
  const int nfb = a.N / BM;
  const int n_act = *a.n_active;
  const int g = blockIdx.x;
  if (g >= a.tile_off[n_act] * nfb) return;  // CTA-uniform, before any barrier
  int lo = 0, hi = n_act;                    // tile_off[lo]*nfb <= g < tile_off[hi]*nfb
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (a.tile_off[mid] * nfb <= g) lo = mid;
    else hi = mid;
  }
  const int tiles = a.tile_off[lo + 1] - a.tile_off[lo];
  const int local = g - a.tile_off[lo] * nfb;
  const int fb = local / tiles, tt = local - fb * tiles;
  const int e = a.active[lo];
  const int s_begin = a.offsets[e] + tt * BN;
  const int ntok = min(BN, a.offsets[e + 1] - s_begin);
  const int wrow = e * a.N + fb * BM;  // first weight row (codes tensor row)
  const int nk = a.K / BK;
  if (tid == 0) GG_STAMP(0);
  const long long cta_clock0 = gg_clock();

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* load_full = bars;                   // [kLS]  TMA bytes landed
  uint64_t* load_empty = bars + L::kLS;         // [kLS]  MMAs reading the stage completed
  uint64_t* oper_full = bars + 2 * L::kLS;      // [kOS]  256 dequant threads stored the operand
  uint64_t* oper_empty = oper_full + L::kOS;    // [kOS]  MMAs reading the operand completed
  uint64_t* acc_full = oper_empty + L::kOS;     // [1]    last MMA completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  __shared__ int abort_flag_s;
  volatile int* abort_flag = &abort_flag_s;  // set by whichever role times out first

  if (tid == 0) {
    for (int s = 0; s < L::kLS; ++s) {
      mbar_init(smem_u32(&load_full[s]), 1);
      mbar_init(smem_u32(&load_empty[s]), 1);
    }
    for (int s = 0; s < L::kOS; ++s) {
      mbar_init(smem_u32(&oper_full[s]), 32 * kDqWarps);
      mbar_init(smem_u32(&oper_empty[s]), 1);
    }
    mbar_init(smem_u32(acc_full), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    *abort_flag = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(L::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) GG_STAMP(1);

  auto give_up = [&]() {
    if (!*abort_flag) {
      *abort_flag = 1;
      atomicOr(a.status, kStatusTimeout);
    }
  };
  // load stage: X | C0 | C1
  auto x_tile = [&](int s) { return smem + s * L::kLoad; };
  auto c_tile = [&](int s, int p) { return smem + s * L::kLoad + L::kX + p * L::kC; };
  // TMEM column of operand stage o, projection p
  auto a_col = [&](int o, int p) { return static_cast<uint32_t>(L::kAccCols + (o * L::kNP + p) * L::kACols); };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int issued = 0;
      long long w_empty = 0;
      for (int c = 0; c < nk && !*abort_flag; ++c) {
        const int s = c % L::kLS;
        const long long t0 = gg_clock();
        if (c >= L::kLS && !mbar_wait(smem_u32(&load_empty[s]), static_cast<uint32_t>(((c / L::kLS) - 1) & 1))) {
          give_up();
          break;
        }
        w_empty += gg_clock() - t0;
        const uint32_t full = smem_u32(&load_full[s]);
        mbar_expect_tx(full, static_cast<uint32_t>(L::kLoad));
        tma_load_2d(smem_u32(x_tile(s)), &tm_x, c * BK, s_begin, full);
        tma_load_2d(smem_u32(c_tile(s, 0)), &tm_w0, c * L::kCodeRow, wrow, full);
        if constexpr (GATEUP) tma_load_2d(smem_u32(c_tile(s, 1)), &tm_w1, c * L::kCodeRow, wrow, full);
        issued = c + 1;
      }
      GG_STAMP(4);
      GG_SUM(8, w_empty);
      if (*abort_flag) {
        // no copy may still be landing in shared memory when the CTA exits
        for (int c = max(0, issued - L::kLS); c < issued; ++c)
          mbar_wait(smem_u32(&load_full[c % L::kLS]), static_cast<uint32_t>((c / L::kLS) & 1));
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      long long w_of = 0, w_lf = 0, t_iss = 0;
      for (int c = 0; c < nk && !*abort_flag; ++c) {
        const int s = c % L::kLS, o = c % L::kOS;
        const long long t0 = gg_clock();
        const bool ok_o = mbar_wait(smem_u32(&oper_full[o]), static_cast<uint32_t>((c / L::kOS) & 1));
        const long long t1 = gg_clock();
        if (!ok_o || !mbar_wait(smem_u32(&load_full[s]), static_cast<uint32_t>((c / L::kLS) & 1))) {
          give_up();
          break;
        }
        const long long t2 = gg_clock();
        w_of += t1 - t0;
        w_lf += t2 - t1;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (c == 0) GG_STAMP(2);
        const uint64_t db = sw128_desc(smem_u32(x_tile(s)));
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint32_t acc = (c > 0 || kk > 0) ? 1u : 0u;
          // A: 16 fp16 of K = 8 TMEM columns per step; B: +32 bytes per step
          umma_ts_f16<BN>(tmem, tmem + a_col(o, 0) + 8 * kk, db + 2 * kk, acc);
          if constexpr (GATEUP) umma_ts_f16<BN>(tmem + BN, tmem + a_col(o, 1) + 8 * kk, db + 2 * kk, acc);
        }
        umma_commit(smem_u32(&load_empty[s]));
        umma_commit(smem_u32(&oper_empty[o]));
        t_iss += gg_clock() - t2;
      }
      GG_STAMP(3);
      GG_SUM(9, w_of);
      GG_SUM(10, w_lf);
      GG_SUM(15, t_iss);
      umma_commit(smem_u32(acc_full));
      // every MMA has finished (normal or aborted) before TMEM is released
      if (!mbar_wait(smem_u32(acc_full), 0u)) give_up();
    }
  } else {
    // ---------------- dequant (warps 2-9), then epilogue ----------------
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;        // which half of the K chunk / of the token columns
    const int r = quarter * 32 + lane;       // weight row within the tile = TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const size_t srow = static_cast<size_t>(wrow + r) * a.sstride;
    constexpr int kVec = L::kCodeRow / 32;   // uint4 code vectors per half row (W4 1, W8 2)
    constexpr int kOut = 4 / kVec;           // output uint4 per code vector
    // W4 group scales: the next chunk's are loaded one chunk ahead
    __half2 sc_cur[L::kNP], sc_next[L::kNP];
#pragma unroll
    for (int p = 0; p < L::kNP; ++p) {
      sc_cur[p] = sc_next[p] = __float2half2_rn(1.0f);
      if constexpr (BITS == 4)
        sc_next[p] = __float2half2_rn(bf16_to_f32(__ldg((p == 0 ? a.s0 : a.s1) + srow)));
    }
    long long w_lf = 0, w_oe = 0, t_dq = 0;
    for (int c = 0; c < nk; ++c) {
      const int s = c % L::kLS, o = c % L::kOS;
      if (__any_sync(0xffffffffu, *abort_flag)) break;
#pragma unroll
      for (int p = 0; p < L::kNP; ++p) {
        sc_cur[p] = sc_next[p];
        if constexpr (BITS == 4) {
          if (c + 1 < nk)
            sc_next[p] = __float2half2_rn(bf16_to_f32(__ldg((p == 0 ? a.s0 : a.s1) + srow + ((c + 1) * BK) / a.group)));
        }
      }
      const long long t0 = gg_clock();
      const bool ok_l = mbar_wait(smem_u32(&load_full[s]), static_cast<uint32_t>((c / L::kLS) & 1));
      const long long t1 = gg_clock();
      const bool ok_o = ok_l && (c < L::kOS ||
                                 mbar_wait(smem_u32(&oper_empty[o]), static_cast<uint32_t>(((c / L::kOS) - 1) & 1)));
      if (!__all_sync(0xffffffffu, ok_o)) {
        give_up();
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const long long t2 = gg_clock();
      w_lf += t1 - t0;
      w_oe += t2 - t1;
#pragma unroll
      for (int p = 0; p < L::kNP; ++p) {
        // this thread's half of the row: 16 code bytes (W4) or 32 (W8) -> 32 fp16 = 16 TMEM columns
        const uint4* codes = reinterpret_cast<const uint4*>(c_tile(s, p) + r * L::kCodeRow + half * (L::kCodeRow / 2));
        uint32_t cols[16];
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
          uint4 ov[kOut];
          dequant16<BITS>(codes[j], sc_cur[p], ov);
#pragma unroll
          for (int q = 0; q < kOut; ++q) {
            cols[(j * kOut + q) * 4 + 0] = ov[q].x;
            cols[(j * kOut + q) * 4 + 1] = ov[q].y;
            cols[(j * kOut + q) * 4 + 2] = ov[q].z;
            cols[(j * kOut + q) * 4 + 3] = ov[q].w;
          }
        }
        tmem_st16(tmem + lane_base + a_col(o, p) + half * 16, cols);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(smem_u32(&oper_full[o]));
      t_dq += gg_clock() - t2;
    }
    if (warp == 2 && lane == 0) {
      GG_SUM(11, w_lf);
      GG_SUM(12, w_oe);
      GG_SUM(13, t_dq);
    }
    // epilogue: this warp's 32 rows x up to 64 token columns
    bool ok = !__any_sync(0xffffffffu, *abort_flag);
    if (ok && !__all_sync(0xffffffffu, mbar_wait(smem_u32(acc_full), 0u))) {
      give_up();
      ok = false;
    }
    if (ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (warp == 2 && lane == 0) GG_STAMP(5);
      const uint32_t tl = tmem + lane_base;
      const int row = fb * BM + r;  // feature row within the expert
      float s0w = 1.0f, s1w = 1.0f;
      if constexpr (BITS == 8) {
        s0w = bf16_to_f32(__ldg(a.s0 + srow));
        if constexpr (GATEUP) s1w = bf16_to_f32(__ldg(a.s1 + srow));
      }
      const int col = GATEUP ? (row & ~7) + kpos<BITS>(row & 7) : row;
      // token columns per warp half: 16-column loads, so a 16-wide tile uses one half only
      constexpr int kHalfCols = BN / 2 < 16 ? 16 : BN / 2;
      const int n0 = half * kHalfCols;
      for (int j = 0; j < kHalfCols / 16; ++j) {
        const int nb = n0 + j * 16;
        if (nb >= ntok || nb >= BN) break;  // warp-uniform
        float d0[16], d1[16];
        tmem_ld16(tl + nb, d0);
        if constexpr (GATEUP) tmem_ld16(tl + BN + nb, d1);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int n = nb + i;
          if (n < ntok) {
            const size_t oidx = static_cast<size_t>(s_begin + n) * a.N + col;
            if constexpr (GATEUP) {
              const float gv = d0[i] * s0w;  // SiLU with the fast exponential and division: the
              // result is rounded to fp16 (11 bits), far coarser than their error
              a.hout[oidx] = __float2half_rn(__fdividef(gv, 1.0f + __expf(-gv)) * (d1[i] * s1w));
            } else {
              a.yout[oidx] = d0[i] * s0w;
            }
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::kTmemCols));
  }
#ifdef MOE_GEMM_TRACE
  if (tid == 0) {
    GG_STAMP(6);
    GG_SUM(14, gg_clock() - cta_clock0);
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    if (blockIdx.x < kTraceCtas)
      g_gemm_trace[GATEUP ? 1 : 0][blockIdx.x][7] = smid | (static_cast<unsigned long long>(ntok) << 32);
  }
#endif
}

// Token-tile prefix over the active experts: tile_off[a] = sum_{a' < a} ceil(count / BN),
// BN the tile width of the routed launches (SBN: of the shared expert's).
// With shared != nullptr also writes the one-expert tables of the shared
// expert over tokens 0..T-1: offsets {0, T}, active {0}, n_active 1,
// tile_off {0, ceil(T / BN)}.
__global__ void tile_table_kernel(const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
                                  const int32_t* __restrict__ n_active, int32_t* __restrict__ tile_off,
                                  int32_t* __restrict__ shared, int T, int BN, int SBN) {
  if (threadIdx.x != 0) return;
  const int n = *n_active;
  int acc = 0;
  for (int i = 0; i < n; ++i) {
    tile_off[i] = acc;
    const int e = active[i];
    acc += (offsets[e + 1] - offsets[e] + BN - 1) / BN;
  }
  tile_off[n] = acc;
  if (shared != nullptr) {
    shared[0] = 0;  // offsets
    shared[1] = T;
    shared[2] = 0;  // active
    shared[3] = 1;  // n_active
    shared[4] = 0;  // tile_off
    shared[5] = (T + SBN - 1) / SBN;
  }
}

// X16[s][k'] = fp16(x[token(s)][k]) with k permuted within each group of 8 (kpos).
template <int BITS>
__global__ void pack_x_kernel(const uint16_t* __restrict__ x, const int32_t* __restrict__ sorted_pair,
                              const int32_t* __restrict__ offsets, int E, int top_k, int identity_tokens, int H,
                              __half* __restrict__ x16) {
  const int P = identity_tokens > 0 ? identity_tokens : offsets[E];
  const int groups = H / 8;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < P * groups; idx += gridDim.x * blockDim.x) {
    const int s = idx / groups, g = idx - s * groups;
    const int tok = identity_tokens > 0 ? s : sorted_pair[s] / top_k;
    const uint4 raw = *reinterpret_cast<const uint4*>(x + static_cast<size_t>(tok) * H + 8 * g);
    const uint16_t v[8] = {static_cast<uint16_t>(raw.x & 0xffff), static_cast<uint16_t>(raw.x >> 16),
                           static_cast<uint16_t>(raw.y & 0xffff), static_cast<uint16_t>(raw.y >> 16),
                           static_cast<uint16_t>(raw.z & 0xffff), static_cast<uint16_t>(raw.z >> 16),
                           static_cast<uint16_t>(raw.w & 0xffff), static_cast<uint16_t>(raw.w >> 16)};
    __half o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[kpos<BITS>(j)] = __float2half_rn(bf16_to_f32(v[j]));
    *reinterpret_cast<uint4*>(x16 + static_cast<size_t>(s) * H + 8 * g) = *reinterpret_cast<uint4*>(o);
  }
}

}  // namespace gg

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool make_tmap_2d(void* out_map, const void* base, bool fp16, uint64_t inner, uint64_t rows, uint32_t box_inner,
                  uint32_t box_rows, bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const uint64_t esize = fp16 ? 2 : 1;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * esize};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r =
      fn(reinterpret_cast<CUtensorMap*>(out_map), fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8,
         2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool gemm_shape_ok(int bits, const QuantProj& p) {
  if (bits != 4 && bits != 8) return false;
  if (p.n % gg::BM || p.k % gg::BK) return false;
  if (bits == 4 && p.group % gg::BK) return false;  // a 64-wide K step must stay inside one scale group
  if (bits == 8 && p.group != p.k) return false;    // W8: per-channel scale applied in the epilogue
  return true;
}

void launch_tile_table(const RouteTables& rt, int32_t* tile_off, int32_t* shared_tables, int T, int bn, int sbn,
                       cudaStream_t st) {
  gg::tile_table_kernel<<<1, 32, 0, st>>>(rt.offsets, rt.active, rt.n_active, tile_off, shared_tables, T, bn, sbn);
}

void launch_pack_x(int bits, const uint16_t* x, const RouteTables& rt, int E, int top_k, int identity_tokens, int H,
                   int max_pairs, void* x16, int num_sms, cudaStream_t st) {
  const int work = max_pairs * (H / 8);
  const int grid = std::max(1, std::min((work + 255) / 256, num_sms * 8));
  if (bits == 4)
    gg::pack_x_kernel<4><<<grid, 256, 0, st>>>(x, rt.sorted_pair, rt.offsets, E, top_k, identity_tokens, H,
                                                static_cast<__half*>(x16));
  else
    gg::pack_x_kernel<8><<<grid, 256, 0, st>>>(x, rt.sorted_pair, rt.offsets, E, top_k, identity_tokens, H,
                                                static_cast<__half*>(x16));
}

template <int BITS, bool GATEUP, int BN>
static int launch_gemm_t(const GemmLaunch& g, cudaStream_t st) {
  using L = gg::Plan<BITS, GATEUP, BN>;
  auto kern = gg::grouped_gemm_kernel<BITS, GATEUP, BN>;
  static int configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1 << (dev & 31)))) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes) != cudaSuccess) return -1;
    configured |= 1 << (dev & 31);
  }
  gg::GemmArgs a{};
  a.offsets = g.rt.offsets;
  a.active = g.rt.active;
  a.n_active = g.rt.n_active;
  a.tile_off = g.tile_off;
  a.s0 = g.p0.s;
  a.s1 = GATEUP ? g.p1.s : nullptr;
  a.sstride = g.p0.sstride;
  a.group = g.p0.group;
  a.N = g.p0.n;
  a.K = g.p0.k;
  a.hout = static_cast<__half*>(g.hout);
  a.yout = g.yout;
  a.status = g.status;
  const int max_tiles = (g.max_pairs + BN - 1) / BN + g.max_active;
  const int grid = max_tiles * (g.p0.n / gg::BM);
  const CUtensorMap* tx = reinterpret_cast<const CUtensorMap*>(g.tmap_x);
  const CUtensorMap* t0 = reinterpret_cast<const CUtensorMap*>(g.tmap_w0);
  const CUtensorMap* t1 = reinterpret_cast<const CUtensorMap*>(GATEUP ? g.tmap_w1 : g.tmap_w0);
  kern<<<grid, gg::kThreadsV2, L::kBytes, st>>>(*tx, *t0, *t1, a);
  return 1;
}

template <int BITS, bool GATEUP>
static int launch_gemm_bn(const GemmLaunch& g, cudaStream_t st) {
  switch (g.bn) {
    case 16: return launch_gemm_t<BITS, GATEUP, 16>(g, st);
    case 32: return launch_gemm_t<BITS, GATEUP, 32>(g, st);
    case 64: return launch_gemm_t<BITS, GATEUP, 64>(g, st);
    case 128: return launch_gemm_t<BITS, GATEUP, 128>(g, st);
    default: return -2;
  }
}

int launch_grouped_gemm(int bits, bool gateup, const GemmLaunch& g, cudaStream_t st) {
  if (bits == 4) return gateup ? launch_gemm_bn<4, true>(g, st) : launch_gemm_bn<4, false>(g, st);
  return gateup ? launch_gemm_bn<8, true>(g, st) : launch_gemm_bn<8, false>(g, st);
}

}  // namespace moe

#ifdef MOE_GEMM_TRACE
extern "C" int moe_gemm_trace_copy(void* host, size_t bytes) {
  return static_cast<int>(cudaMemcpyFromSymbol(host, moe::gg::g_gemm_trace, bytes));
}
#endif
