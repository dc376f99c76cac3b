// stream.cu — weight-streaming expert projections for decode batches that
// give each routed expert a few tokens (W4, sm_100a).
//
// Replaces, for every routed (token, expert) pair, the reference's
//   gate = W4A32 matvec(x, W_gate); up = matvec(x, W_up); h = silu(gate) * up
//   y = matvec(h, W_down)
// (nano_ktrans/kernels/cpu_moe.py:419-450 over quantized_ops.py:86-124): each
// active expert's code rows leave HBM once per step, through a ring of
// shared-memory stages filled by bulk copies, and are applied there to up to 8
// of the expert's tokens at a time on the warp-level tensor-core path
// (mma.sync m16n8k16, bf16 operands, fp32 accumulate; the tokens are the N
// dimension).
//
// Arithmetic (mma_gemv.cuh): a code enters as the exact bf16 value 128 + q,
// products are exact, and per 128-code group the fp32 group sum is corrected
// by 136 * sum(x) and scaled by the group scale:
//   acc += s_g * (sum_k (128 + q_k) x_k - 136 * sum_k x_k) = s_g * sum (q - 8) x.
// Gate/up operands are the bf16 activations themselves.  The down projection's
// operand h = SiLU(gate) * up is fp32; it enters as two bf16 terms hi + lo
// (hi = bf16(h), lo = bf16(h - hi), 16 significant bits), each its own mma.
//
// Work items.  The sorted pairs of each active expert are cut into chunks of
// up to 8 tokens; an item is (chunk, block of R output rows), numbered
// chunk-major, and each CTA of the persistent grid takes one contiguous range
// of items, so a CTA sees one or two chunks and streams their rows in order.
//
// Warp roles, one CTA per SM:
//   warps 0-7  consumers.  The 8 warps are P K-parts x (8 / P) row sets; warp
//              w takes K-part w % P (the 128-code groups p, p + P, ...) of two
//              16-row tiles of set w / P.  Gate/up: a set is 16 gate rows and
//              the same 16 up rows (R = 16 * sets).  Down: a set is 32 rows
//              (R = 32 * sets).  A warp keeps its K-part's B fragments in
//              registers for the whole chunk; the P partial sums of an output
//              meet in shared memory and are added in part order, so results
//              do not depend on timing.
//   warp 8     producer.  One lane issues, per item, the bulk copies of its
//              code rows and scale rows into the next ring stage.
//   warp 9     operand stager.  Converts each chunk's activations (gate/up:
//              bf16 x rows of its tokens; down: fp32 h rows) into B-fragment
//              order with the per-group corrections, while the consumers work
//              on the previous chunk.
//
// Every wait is bounded.  A wait that runs out sets the CTA's abort flag and
// the status word (kStatusTimeout); consumers leave together through a
// reducing barrier, the producer waits (bounded) for its copies in flight.
#include <cuda_runtime.h>

#include <algorithm>

#include "async_copy.cuh"
#include "common.cuh"
#include "kernels.h"
#include "mma_gemv.cuh"

namespace moe {
namespace sm {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 64;  // + producer warp + operand warp
constexpr int kTok = 8;                    // tokens per chunk: the mma's N
constexpr int kMaxStages = 8;
constexpr int kRedPitch = 17;                      // floats per (tile, token) row of the partial-sum buffer
constexpr int kRedTile = kTok * kRedPitch;         // floats per tile
constexpr int kRedFloats = 16 * kRedTile;          // P * tiles == 16 in every configuration
constexpr int kSmemLimit = 227 * 1024;

struct Args {
  const uint16_t* x;  // gate/up: bf16 [T][K]
  const float* h;     // down: fp32 [pairs][K], row = sorted position
  const int32_t* sorted_pair;
  const int32_t* offsets;
  const int32_t* active;
  const int32_t* n_active;
  int top_k;
  QuantProj p0, p1;  // gate, up | down
  float* out;        // gate/up: SiLU(g)*u [pairs][N]; down: y [pairs][N]
  int* status;
  int parts;         // P
  int rows;          // R: output rows per item
  int stages;
  int max_active;    // capacity of the chunk table
  uint32_t stage_bytes;
  uint32_t code_bytes;   // code bytes of one item (both projections for gate/up)
  uint32_t scale_bytes;  // scale bytes of one item
};

struct Smem {
  // byte offsets into dynamic shared memory
  uint32_t tab, corr, xbuf, red, stage;
};

__host__ __device__ inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

template <bool GATEUP>
__host__ __device__ inline uint32_t xbuf_bytes(int K) {
  return static_cast<uint32_t>(kTok) * K * (GATEUP ? 2 : 4);  // bf16 x | bf16 hi + lo
}

template <bool GATEUP>
__host__ __device__ inline Smem smem_layout(int K, int max_active) {
  Smem s;
  const uint32_t bars = 160;  // (2 * kMaxStages + 2) mbarriers, then the abort flag
  s.tab = bars;
  s.corr = align_up(s.tab + 4u * 4u * (max_active + 1), 16);
  s.xbuf = align_up(s.corr + 4u * kTok * (K / 128), 128);
  s.red = align_up(s.xbuf + xbuf_bytes<GATEUP>(K), 128);
  s.stage = align_up(s.red + 2u * 4u * kRedFloats, 128);
  return s;
}

MOE_DEV uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

MOE_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Wait for phase `parity` of `bar`; false if the CTA aborted or the wait ran out
// (which aborts it).
MOE_DEV bool wait_phase(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t i = 0;; ++i) {
    if (ac::mbar_try_wait(bar, parity)) return true;
    if ((i & 31u) == 31u && *abort_flag) return false;
    if (i > ac::kSpinLimit) {
      *abort_flag = 1;
      return false;
    }
  }
}

// Barrier over the consumer warps that also ORs a flag across them.
MOE_DEV bool consumers_sync_or(bool flag) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n}"
      : "=r"(out)
      : "r"(static_cast<uint32_t>(flag)), "n"(kConsumers)
      : "memory");
  return out != 0;
}

// One 128-code group of a 16-row tile against 8 token columns: wlo / whi are
// the lane's 16 code bytes of tile rows g and g + 8, b[q] the operand words of
// step pair q (mma_gemv.cuh order).  d[0..1]: row g, tokens 2t, 2t+1; d[2..3]:
// row g + 8.
MOE_DEV void group_x(uint4 wlo, uint4 whi, uint4 b0, uint4 b1, uint4 b2, uint4 b3, float (&d)[4]) {
  constexpr uint32_t M = 0x43004300u, N = 0x000F000Fu;
  const uint4 b[4] = {b0, b1, b2, b3};
  const uint32_t u[4] = {wlo.x, wlo.y, wlo.z, wlo.w};
  const uint32_t v[4] = {whi.x, whi.y, whi.z, whi.w};
  float e[4][4];
#pragma unroll
  for (int s = 0; s < 4; ++s) e[s][0] = e[s][1] = e[s][2] = e[s][3] = 0.0f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    mma16816_bf16(e[(2 * q) & 3], (u[q] & N) | M, (v[q] & N) | M, ((u[q] >> 4) & N) | M, ((v[q] >> 4) & N) | M,
                  b[q].x, b[q].y);
    mma16816_bf16(e[(2 * q + 1) & 3], ((u[q] >> 8) & N) | M, ((v[q] >> 8) & N) | M, ((u[q] >> 12) & N) | M,
                  ((v[q] >> 12) & N) | M, b[q].z, b[q].w);
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) d[r] = (e[0][r] + e[1][r]) + (e[2][r] + e[3][r]);
}

// The same with a two-term operand: bh = bf16 hi words, bl = lo words.
MOE_DEV void group_hl(uint4 wlo, uint4 whi, const uint4* bh, const uint4* bl, float (&d)[4]) {
  constexpr uint32_t M = 0x43004300u, N = 0x000F000Fu;
  const uint32_t u[4] = {wlo.x, wlo.y, wlo.z, wlo.w};
  const uint32_t v[4] = {whi.x, whi.y, whi.z, whi.w};
  float e[4][4];
#pragma unroll
  for (int s = 0; s < 4; ++s) e[s][0] = e[s][1] = e[s][2] = e[s][3] = 0.0f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t a0 = (u[q] & N) | M, a1 = (v[q] & N) | M, a2 = ((u[q] >> 4) & N) | M, a3 = ((v[q] >> 4) & N) | M;
    const uint32_t c0 = ((u[q] >> 8) & N) | M, c1 = ((v[q] >> 8) & N) | M, c2 = ((u[q] >> 12) & N) | M,
                   c3 = ((v[q] >> 12) & N) | M;
    mma16816_bf16(e[0], a0, a1, a2, a3, bh[q].x, bh[q].y);
    mma16816_bf16(e[1], a0, a1, a2, a3, bl[q].x, bl[q].y);
    mma16816_bf16(e[2], c0, c1, c2, c3, bh[q].z, bh[q].w);
    mma16816_bf16(e[3], c0, c1, c2, c3, bl[q].z, bl[q].w);
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) d[r] = (e[0][r] + e[1][r]) + (e[2][r] + e[3][r]);
}

// (x0, x4) (x1, x5) (x2, x6) (x3, x7) operand words of 8 values given as bf16 bits.
MOE_DEV uint4 pack_pairs(uint32_t p01, uint32_t p23, uint32_t p45, uint32_t p67) {
  return make_uint4(__byte_perm(p01, p45, 0x5410), __byte_perm(p01, p45, 0x7632), __byte_perm(p23, p67, 0x5410),
                    __byte_perm(p23, p67, 0x7632));
}

struct ChunkRef {
  int e, s0, cnt;
};

// Chunk table in shared memory: for active index a, tab[a] = first global
// chunk, tab[A + 1 + a] = expert, tab[2(A + 1) + a] = first sorted position,
// tab[3(A + 1) + a] = pair count.
struct Cursor {
  const int* tab;
  int cap;  // A + 1
  int a = 0;
  MOE_DEV ChunkRef at(int gc) {
    while (tab[a + 1] <= gc) ++a;
    const int c = gc - tab[a];
    ChunkRef r;
    r.e = tab[cap + a];
    r.s0 = tab[2 * cap + a] + kTok * c;
    r.cnt = min(kTok, tab[2 * cap + a] + tab[3 * cap + a] - r.s0);
    return r;
  }
};

template <bool GATEUP, int GPW>
__global__ void __launch_bounds__(kThreads, 1) stream_kernel(Args a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int K = a.p0.k, N = a.p0.n;
  const int nG = K / 128;
  const int P = a.parts, S = a.stages, R = a.rows;
  const Smem L = smem_layout<GATEUP>(K, a.max_active);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  const uint32_t full0 = ac::smem_u32(&bars[0]), empty0 = ac::smem_u32(&bars[kMaxStages]);
  const uint32_t xfull = ac::smem_u32(&bars[2 * kMaxStages]), xempty = ac::smem_u32(&bars[2 * kMaxStages + 1]);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 8 * (2 * kMaxStages + 2));
  int* tab = reinterpret_cast<int*>(smem + L.tab);
  float* cb = reinterpret_cast<float*>(smem + L.corr);  // [kTok][nG] 136 * sum of the operand per group
  uint4* xb = reinterpret_cast<uint4*>(smem + L.xbuf);
  float* red = reinterpret_cast<float*>(smem + L.red);
  unsigned char* stages = smem + L.stage;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ac::mbar_init(full0 + 8 * s, 1);
      ac::mbar_init(empty0 + 8 * s, kConsumerWarps);
    }
    ac::mbar_init(xfull, 32);
    ac::mbar_init(xempty, kConsumerWarps);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // chunk table: prefix of ceil(count / 8) over the active experts (warp 0)
  const int n_act = min(*a.n_active, a.max_active);
  const int cap = a.max_active + 1;
  if (warp == 0) {
    int run = 0;
    for (int base = 0; base < n_act; base += 32) {
      const int i = base + lane;
      int c = 0, e = 0, off = 0, cnt = 0;
      if (i < n_act) {
        e = a.active[i];
        off = a.offsets[e];
        cnt = a.offsets[e + 1] - off;
        c = (cnt + kTok - 1) / kTok;
      }
      int inc = c;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(kFullMask, inc, d);
        if (lane >= d) inc += v;
      }
      if (i < n_act) {
        tab[i] = run + inc - c;
        tab[cap + i] = e;
        tab[2 * cap + i] = off;
        tab[3 * cap + i] = cnt;
      }
      run += __shfl_sync(kFullMask, inc, 31);
    }
    if (lane == 0) tab[n_act] = run;
  }
  __syncthreads();

  const int total_chunks = tab[n_act];
  const int blocks = N / R;
  const long long total = static_cast<long long>(total_chunks) * blocks;
  const int lo = static_cast<int>(total * blockIdx.x / gridDim.x);
  const int hi = static_cast<int>(total * (blockIdx.x + 1) / gridDim.x);
  const size_t rowb = static_cast<size_t>(K) / 2;
  const int sstride = a.p0.sstride;

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      Cursor cur{tab, cap};
      int issued = lo;
      for (int it = lo; it < hi; ++it) {
        const int k = it - lo, s = k % S;
        if (!wait_phase(empty0 + 8 * s, ((k / S) & 1) ^ 1, abort_flag)) break;
        const ChunkRef c = cur.at(it / blocks);
        const size_t row0 = static_cast<size_t>(c.e) * N + static_cast<size_t>(it % blocks) * R;
        const uint32_t dst = ac::smem_u32(stages + static_cast<size_t>(s) * a.stage_bytes);
        ac::mbar_arrive_expect_tx(full0 + 8 * s, a.code_bytes + a.scale_bytes);
        const uint32_t cpp = static_cast<uint32_t>(R * rowb), spp = static_cast<uint32_t>(R * sstride * 2);
        ac::bulk_g2s(dst, a.p0.q + row0 * rowb, cpp, full0 + 8 * s);
        if constexpr (GATEUP) {
          ac::bulk_g2s(dst + cpp, a.p1.q + row0 * rowb, cpp, full0 + 8 * s);
          ac::bulk_g2s(dst + 2 * cpp, a.p0.s + row0 * sstride, spp, full0 + 8 * s);
          ac::bulk_g2s(dst + 2 * cpp + spp, a.p1.s + row0 * sstride, spp, full0 + 8 * s);
        } else {
          ac::bulk_g2s(dst + cpp, a.p0.s + row0 * sstride, spp, full0 + 8 * s);
        }
        issued = it + 1;
      }
      // the copies still in flight land before the CTA may exit
      for (int it = max(lo, issued - S); it < issued; ++it) {
        const int k = it - lo;
        ac::mbar_wait_bounded(full0 + 8 * (k % S), (k / S) & 1);
      }
    }
    return;
  }

  if (warp == kConsumerWarps + 1) {
    // ---------------- operand stager ----------------
    if (hi <= lo) return;
    Cursor cur{tab, cap};
    const int gc0 = lo / blocks, gc1 = (hi - 1) / blocks;
    const int K8 = K / 8;  // 8-value pieces per token row
    for (int gc = gc0; gc <= gc1; ++gc) {
      const int k = gc - gc0;
      if (!wait_phase(xempty, (k & 1) ^ 1, abort_flag)) break;
      const ChunkRef c = cur.at(gc);
      int my_row = -1;  // lane n < 8: source row of token slot n
      if (lane < kTok && lane < c.cnt) my_row = GATEUP ? a.sorted_pair[c.s0 + lane] / a.top_k : c.s0 + lane;
      for (int base = 0; base < kTok * K8; base += 32 * 4) {
        uint4 raw[4][2];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int pi = base + 32 * u + lane;
          const int n = pi / K8, kq = pi - n * K8;
          const int row = __shfl_sync(kFullMask, my_row, n & 7);
          raw[u][0] = raw[u][1] = make_uint4(0, 0, 0, 0);
          if (pi < kTok * K8 && row >= 0) {
            if constexpr (GATEUP) {
              raw[u][0] = *reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(row) * K + 8 * kq);
            } else {
              const uint4* src = reinterpret_cast<const uint4*>(a.h + static_cast<size_t>(row) * K + 8 * kq);
              raw[u][0] = src[0];
              raw[u][1] = src[1];
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int pi = base + 32 * u + lane;
          if (base + 32 * u >= kTok * K8) break;  // warp-uniform
          const int n = pi / K8, kq = pi - n * K8;
          const int G = kq >> 4, t = (kq >> 2) & 3, j = kq & 3;
          float corr = 0.0f;
          if constexpr (GATEUP) {
            xb[(G * 4 + j) * 32 + n * 4 + t] = w4_pack_x(raw[u][0], corr);
          } else {
            const float v[8] = {__uint_as_float(raw[u][0].x), __uint_as_float(raw[u][0].y),
                                __uint_as_float(raw[u][0].z), __uint_as_float(raw[u][0].w),
                                __uint_as_float(raw[u][1].x), __uint_as_float(raw[u][1].y),
                                __uint_as_float(raw[u][1].z), __uint_as_float(raw[u][1].w)};
            uint16_t hb[8], lb[8];
            float sh = 0.0f, sl = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              split_bf16(v[i], hb[i], lb[i]);
              sh += bf16_to_f32(hb[i]);
              sl += bf16_to_f32(lb[i]);
            }
            corr = 136.0f * (sh + sl);
            const int slot = ((G * 4 + j) * 2) * 32 + n * 4 + t;
            xb[slot] = pack_pairs(pack_bf16x2(hb[0], hb[1]), pack_bf16x2(hb[2], hb[3]), pack_bf16x2(hb[4], hb[5]),
                                  pack_bf16x2(hb[6], hb[7]));
            xb[slot + 32] = pack_pairs(pack_bf16x2(lb[0], lb[1]), pack_bf16x2(lb[2], lb[3]),
                                       pack_bf16x2(lb[4], lb[5]), pack_bf16x2(lb[6], lb[7]));
          }
          // the 16 pieces of one (token, group) sit in one half-warp
#pragma unroll
          for (int d = 1; d < 16; d <<= 1) corr += __shfl_xor_sync(kFullMask, corr, d);
          if ((lane & 15) == 0) cb[n * nG + G] = corr;
        }
      }
      mbar_arrive(xfull);  // release: this lane's stores before the consumers' reads
    }
    return;
  }

  // ---------------- consumers ----------------
  const int part = warp % P, set = warp / P;
  const int g = lane >> 2, t = lane & 3;
  const int grp = a.p0.group;
  Cursor cur{tab, cap};
  uint4 bx[GPW][GATEUP ? 4 : 8];
  float cx[GPW][2];
  int chunk_k = -1;
  bool failed = false;
  for (int it = lo; it < hi; ++it) {
    const int k = it - lo;
    const int gc = it / blocks, rb = it - gc * blocks;
    const ChunkRef c = cur.at(gc);
    if (gc - lo / blocks != chunk_k) {  // first item of a chunk: its operands into registers
      chunk_k = gc - lo / blocks;
      failed = failed || !wait_phase(xfull, chunk_k & 1, abort_flag);
      if (!failed) {
#pragma unroll
        for (int gi = 0; gi < GPW; ++gi) {
          const int G = part + gi * P;
          if (G < nG) {
#pragma unroll
            for (int q = 0; q < (GATEUP ? 4 : 8); ++q) {
              const int j = GATEUP ? q : (q & 3), hl = GATEUP ? 0 : (q >> 2);
              bx[gi][q] = xb[((G * 4 + j) * (GATEUP ? 1 : 2) + hl) * 32 + lane];
            }
            cx[gi][0] = cb[(2 * t) * nG + G];
            cx[gi][1] = cb[(2 * t + 1) * nG + G];
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(xempty);
    }
    const int s = k % S;
    failed = failed || !wait_phase(full0 + 8 * s, (k / S) & 1, abort_flag);
    float acc[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
    if (!failed) {
      const unsigned char* st = stages + static_cast<size_t>(s) * a.stage_bytes;
      const uint16_t* sc = reinterpret_cast<const uint16_t*>(st + a.code_bytes);
#pragma unroll
      for (int gi = 0; gi < GPW; ++gi) {
        const int G = part + gi * P;
        if (G < nG) {
          const int gs = (G * 128) / grp;
#pragma unroll
          for (int tile = 0; tile < 2; ++tile) {
            // stage row of tile row g: gate/up [gate R rows][up R rows]; down [R rows]
            const int r0 = GATEUP ? tile * R + set * 16 : set * 32 + tile * 16;
            const unsigned char* wp = st + static_cast<size_t>(r0 + g) * rowb + G * 64 + 16 * t;
            const uint4 wlo = lds128(wp), whi = lds128(wp + 8 * rowb);
            float d[4];
            if constexpr (GATEUP) {
              group_x(wlo, whi, bx[gi][0], bx[gi][1], bx[gi][2], bx[gi][3], d);
            } else {
              group_hl(wlo, whi, &bx[gi][0], &bx[gi][4], d);
            }
            const float s_lo = bf16_to_f32(sc[(r0 + g) * sstride + gs]);
            const float s_hi = bf16_to_f32(sc[(r0 + g + 8) * sstride + gs]);
            acc[tile][0] = fmaf(s_lo, d[0] - cx[gi][0], acc[tile][0]);
            acc[tile][1] = fmaf(s_lo, d[1] - cx[gi][1], acc[tile][1]);
            acc[tile][2] = fmaf(s_hi, d[2] - cx[gi][0], acc[tile][2]);
            acc[tile][3] = fmaf(s_hi, d[3] - cx[gi][1], acc[tile][3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(empty0 + 8 * s);
      // partial sums of this K-part: red[buf][part][tile][token][row]
      float* rp = red + (k & 1) * kRedFloats + (part * (16 / P) + set * 2) * kRedTile;
#pragma unroll
      for (int tile = 0; tile < 2; ++tile) {
        float* r = rp + tile * kRedTile;
        r[(2 * t) * kRedPitch + g] = acc[tile][0];
        r[(2 * t + 1) * kRedPitch + g] = acc[tile][1];
        r[(2 * t) * kRedPitch + g + 8] = acc[tile][2];
        r[(2 * t + 1) * kRedPitch + g + 8] = acc[tile][3];
      }
    }
    __syncwarp();
    if (consumers_sync_or(failed || *abort_flag)) {
      failed = true;
      break;
    }
    // epilogue: add the P partial sums in part order, write the item's outputs
    const float* rb_ = red + (k & 1) * kRedFloats;
    const int tiles_per_part = 16 / P;
    const int outs = (R / 16) * 128;  // gate/up: 16-row sets; down: 16-row tiles
    for (int o = threadIdx.x; o < outs; o += kConsumers) {
      const int tl = o >> 7, n = (o >> 4) & 7, r = o & 15;
      if (n >= c.cnt) continue;
      float v;
      int row;
      if constexpr (GATEUP) {
        // tl = set: tiles 2 * set (gate) and 2 * set + 1 (up)
        float gsum = 0.0f, usum = 0.0f;
        for (int p = 0; p < P; ++p) {
          gsum += rb_[(p * tiles_per_part + 2 * tl) * kRedTile + n * kRedPitch + r];
          usum += rb_[(p * tiles_per_part + 2 * tl + 1) * kRedTile + n * kRedPitch + r];
        }
        v = silu_f32(gsum) * usum;
        row = rb * R + tl * 16 + r;
      } else {
        float ysum = 0.0f;
        for (int p = 0; p < P; ++p) ysum += rb_[(p * tiles_per_part + tl) * kRedTile + n * kRedPitch + r];
        v = ysum;
        row = rb * R + tl * 16 + r;  // tile tl = set * 2 + half: rows set * 32 + half * 16
      }
      a.out[static_cast<size_t>(c.s0 + n) * N + row] = v;
    }
  }
  if (failed && threadIdx.x == 0) atomicOr(a.status, kStatusTimeout);
}

template <bool GATEUP, int GPW>
static void* kernel_ptr() {
  return reinterpret_cast<void*>(stream_kernel<GATEUP, GPW>);
}

// P (K-parts) of a projection: gate/up always 8; down the smallest power of
// two leaving at most 3 groups per warp.
static int pick_parts(bool gateup, int nG) {
  if (gateup) return 8;
  for (int p = 1; p <= 8; p <<= 1)
    if ((nG + p - 1) / p <= 3) return p;
  return 0;
}

struct Plan {
  Args a;
  void* kern = nullptr;
  size_t smem = 0;
};

template <bool GATEUP>
static bool plan(const QuantProj& p0, int max_active, Plan& pl) {
  const int K = p0.k, N = p0.n;
  if (K % 128 || p0.group % 128 || K % p0.group) return false;
  const int nG = K / 128;
  const int P = pick_parts(GATEUP, nG);
  if (P == 0) return false;
  const int gpw = (nG + P - 1) / P;
  if (gpw > (GATEUP ? 4 : 3)) return false;
  const int sets = kConsumerWarps / P;
  const int R = GATEUP ? 16 * sets : 32 * sets;
  if (N % R) return false;
  const uint32_t rowb = static_cast<uint32_t>(K / 2);
  const uint32_t code = (GATEUP ? 2u : 1u) * R * rowb;
  const uint32_t scale = (GATEUP ? 2u : 1u) * R * p0.sstride * 2u;
  const uint32_t stage = align_up(code + scale, 128);
  const Smem L = smem_layout<GATEUP>(K, max_active);
  if (L.stage >= kSmemLimit) return false;
  const int S = std::min<int>(kMaxStages, (kSmemLimit - L.stage) / stage);
  if (S < 2) return false;
  Args& a = pl.a;
  a.parts = P;
  a.rows = R;
  a.stages = S;
  a.max_active = max_active;
  a.stage_bytes = stage;
  a.code_bytes = code;
  a.scale_bytes = scale;
  pl.smem = L.stage + static_cast<size_t>(S) * stage;
  if constexpr (GATEUP) {
    pl.kern = gpw == 1 ? kernel_ptr<true, 1>() : gpw == 2 ? kernel_ptr<true, 2>()
              : gpw == 3 ? kernel_ptr<true, 3>() : kernel_ptr<true, 4>();
  } else {
    pl.kern = gpw == 1 ? kernel_ptr<false, 1>() : gpw == 2 ? kernel_ptr<false, 2>() : kernel_ptr<false, 3>();
  }
  return true;
}

static int launch(Plan& pl, int num_sms, cudaStream_t st) {
  if (!ensure_dynamic_smem(pl.kern, pl.smem, kThreads)) return -1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {&pl.a};
  return cudaLaunchKernelExC(&cfg, pl.kern, args) == cudaSuccess ? 1 : -2;
}

}  // namespace sm

bool stream_eligible(int bits, const QuantProj& gate, const QuantProj& up, const QuantProj& down, int max_active) {
  if (bits != 4 || up.group != gate.group || up.sstride != gate.sstride) return false;
  sm::Plan a, b;
  return sm::plan<true>(gate, max_active, a) && sm::plan<false>(down, max_active, b);
}

int launch_stream_gateup(const uint16_t* x, const RouteTables& rt, int top_k, int max_active, const QuantProj& gate,
                         const QuantProj& up, float* h, int* status, int num_sms, cudaStream_t st) {
  sm::Plan pl;
  if (!sm::plan<true>(gate, max_active, pl)) return -1;
  sm::Args& a = pl.a;
  a.x = x;
  a.sorted_pair = rt.sorted_pair;
  a.offsets = rt.offsets;
  a.active = rt.active;
  a.n_active = rt.n_active;
  a.top_k = top_k;
  a.p0 = gate;
  a.p1 = up;
  a.out = h;
  a.status = status;
  return sm::launch(pl, num_sms, st);
}

int launch_stream_down(const float* h, const RouteTables& rt, int max_active, const QuantProj& down, float* y,
                       int* status, int num_sms, cudaStream_t st) {
  sm::Plan pl;
  if (!sm::plan<false>(down, max_active, pl)) return -1;
  sm::Args& a = pl.a;
  a.h = h;
  a.sorted_pair = rt.sorted_pair;
  a.offsets = rt.offsets;
  a.active = rt.active;
  a.n_active = rt.n_active;
  a.top_k = 1;
  a.p0 = down;
  a.p1 = down;
  a.out = y;
  a.status = status;
  return sm::launch(pl, num_sms, st);
}

}  // namespace moe
