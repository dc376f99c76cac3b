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
// Warp roles, one CTA per SM (gate/up: C = 16 consumer warps, E = 3 epilogue
// warps; down: C = 12, E = 7 — see Roles):
//   warps 0..C-1  consumers.  P K-parts x (C / P) 16-row tiles: warp w
//               computes tile w / P of the item over the 128-code groups p,
//               p + P, ... of K-part p = w % P.  Gate/up tiles alternate gate
//               and up rows (R = 8 * C / P); down tiles are consecutive rows
//               (R = 16 * C / P).  A warp keeps its K-part's B fragments in
//               registers for the whole chunk.
//   warp C      producer: one lane issues, per item, the bulk copies of its
//               code rows and scale rows into the next ring stage.
//   warps C+1.. rows + epilogue.  The first of them bulk-copies each chunk's
//               activation rows (gate/up: the bf16 x rows of its tokens; down:
//               the fp32 h rows) into a shared-memory area once the consumers
//               have taken the previous chunk's (each consumer warp builds its
//               B fragments and per-group corrections from those rows once per
//               chunk; down splits h into its bf16 hi + lo terms).  Per item,
//               the E warps each take part of the outputs: add the P partial
//               sums in part order (results do not depend on timing), apply
//               SiLU(g) * u for gate/up, and store.
// The consumers pass partial sums to the epilogue through a ring of
// shared-memory buffers, so no consumer waits for another.
//
// Every wait is bounded (2 s of %globaltimer; while waiting, a warp is
// suspended on the mbarrier rather than spinning).  A wait that runs out sets
// the CTA's abort flag and the status word (kStatusTimeout); every role then
// leaves, the producer and the row-copying warp after their copies in flight
// have landed (bounded as well).
#include <cuda_runtime.h>

#include <algorithm>

#include "async_copy.cuh"
#include "common.cuh"
#include "kernels.h"
#include "mma_gemv.cuh"

namespace moe {
namespace sm {

// Warp roles per projection: gate/up 16 consumer warps, 1 producer, 3 epilogue
// warps; down (whose items are small and whose every output sums P partials)
// 12 consumer warps and 7 epilogue warps.  20 warps: at most 5 share an SM
// sub-partition's 16K registers, which keeps 96 registers per thread (21 warps
// would cap them at 80).
template <bool GATEUP> struct Roles {
  static constexpr int kConsumerWarps = GATEUP ? 16 : 12;
  static constexpr int kProducerWarp = kConsumerWarps;
  static constexpr int kEpilogueWarp = kConsumerWarps + 1;
  static constexpr int kEpilogueWarps = GATEUP ? 3 : 7;
  static constexpr int kThreads = (kEpilogueWarp + kEpilogueWarps) * 32;
};
constexpr int kTok = 8;  // tokens per chunk: the mma's N
constexpr int kMaxStages = 8;
constexpr int kRedBufs = 3;
// largest K-part count: gate/up always 8; down divides its 12 consumer warps
template <bool GATEUP> struct PartsCap { static constexpr int value = GATEUP ? 8 : 12; };
// A partial-sum buffer holds red[token][K-part][item row]: the epilogue's lanes
// read consecutive rows of one part (no bank conflicts).  Item rows x P is at
// most 256 (gate/up: 2R rows, R = 128 / P; down: R = 16 * consumers / P rows).
constexpr int kRedRowParts = 256;
constexpr int kRedFloats = kTok * kRedRowParts;
constexpr int kSmemLimit = 227 * 1024;
// mbarriers: full[kMaxStages], empty[kMaxStages], red_full[kRedBufs], red_empty[kRedBufs], xempty, raw
constexpr int kBarFull = 0, kBarEmpty = kMaxStages, kBarRedFull = 2 * kMaxStages,
              kBarRedEmpty = 2 * kMaxStages + kRedBufs, kBarXEmpty = 2 * kMaxStages + 2 * kRedBufs,
              kBarRaw = kBarXEmpty + 1, kNumBars = kBarXEmpty + 2;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

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
  unsigned long long* trace;  // optional [G][16] %globaltimer stamps (gate/up launch), see STREAM_TRACE
  int parts;         // P
  int rows;          // R: output rows per item
  int stages;
  int max_active;    // capacity of the chunk table
  uint32_t stage_bytes;
  uint32_t code_bytes;   // code bytes of one item (both projections for gate/up)
  uint32_t scale_bytes;  // scale bytes of one item
};

// Trace slots per CTA (ns): 0 entry (absolute), then offsets from entry:
// 1 chunk table built, 2 first operands ready (consumer warp 0), 3 consumer
// warp 0 done, 4 producer done, 5 epilogue done; 6 the CTA's item count.
#define STREAM_TRACE(slot, t0)                                                      \
  do {                                                                            \
    if (a.trace != nullptr)                                                       \
      a.trace[blockIdx.x * 16 + (slot)] = (slot) == 0 ? (t0) : ac::global_ns() - (t0); \
  } while (0)

struct Smem {
  // byte offsets into dynamic shared memory
  uint32_t tab, raw, red, stage;
};

__host__ __device__ inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// Bytes of one activation row as stored in global memory (bf16 x | fp32 h).
template <bool GATEUP>
__host__ __device__ inline uint32_t row_bytes(int K) {
  return static_cast<uint32_t>(K) * (GATEUP ? 2 : 4);
}

template <bool GATEUP>
__host__ __device__ inline Smem smem_layout(int K, int max_active) {
  Smem s;
  s.tab = align_up(8u * kNumBars + 4u, 16);  // mbarriers, then the abort flag
  s.raw = align_up(s.tab + 4u * 4u * (max_active + 1), 128);
  s.red = align_up(s.raw + kTok * row_bytes<GATEUP>(K), 128);
  s.stage = align_up(s.red + 4u * kRedBufs * kRedFloats, 128);
  return s;
}

MOE_DEV uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }

MOE_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// try_wait with a suspend-time hint: the warp sleeps on the barrier (up to
// `ns`) instead of re-polling.
MOE_DEV bool try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar`; false if the CTA aborted or the wait ran
// out of its time limit (which aborts it).
MOE_DEV bool wait_phase_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  const unsigned long long t0 = ac::global_ns();
  for (uint32_t i = 1;; ++i) {
    if (try_wait_sleep(bar, parity, 20000u)) return true;
    if ((i & 15u) == 0) {
      if (*abort_flag) return false;
      if (ac::global_ns() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        return false;
      }
    }
  }
}

MOE_DEV bool wait_phase(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  return ac::mbar_try_wait(bar, parity) || wait_phase_slow(bar, parity, abort_flag);
}

// Bounded wait that ignores the abort flag: for copies in flight that must land
// before the CTA exits.
MOE_DEV void wait_landed(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = ac::global_ns();
  while (!try_wait_sleep(bar, parity, 20000u))
    if (ac::global_ns() - t0 > kWaitLimitNs) return;
}

// The lanes' earlier shared-memory stores, then one arrival for the warp.
MOE_DEV void warp_arrive(uint32_t bar) {
  __threadfence_block();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// (x0, x4) (x1, x5) (x2, x6) (x3, x7) operand words of 8 values given as bf16 bits.
MOE_DEV uint4 pack_pairs(uint32_t p01, uint32_t p23, uint32_t p45, uint32_t p67) {
  return make_uint4(__byte_perm(p01, p45, 0x5410), __byte_perm(p01, p45, 0x7632), __byte_perm(p23, p67, 0x5410),
                    __byte_perm(p23, p67, 0x7632));
}

// A-operand registers of code word pair (u: tile row g, v: row g + 8): steps
// 2q (nibbles 0,4 / 1,5) and 2q + 1 (nibbles 2,6 / 3,7), as 128 + q bf16.
struct AWords {
  uint32_t a0, a1, a2, a3, c0, c1, c2, c3;
};
MOE_DEV AWords unpack_a(uint32_t u, uint32_t v) {
  AWords w;
  w.a0 = nib_bf16(u);
  w.a1 = nib_bf16(v);
  w.a2 = nib_bf16(u >> 4);
  w.a3 = nib_bf16(v >> 4);
  w.c0 = nib_bf16(u >> 8);
  w.c1 = nib_bf16(v >> 8);
  w.c2 = nib_bf16(u >> 12);
  w.c3 = nib_bf16(v >> 12);
  return w;
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

// One consumer warp's share of an item: its NV groups (all valid: no per-group
// guards in the unrolled body) of one 16-row tile against the chunk's tokens.
// Reads the stage (codes + scales), then releases it (`release` runs once the
// stage's words are in registers); returns the tile's partial sums in acc.
template <bool GATEUP, int NV, int GPW, typename Release>
MOE_DEV void item_compute(const unsigned char* st, const uint16_t* sc, const uint32_t (&woff)[GPW],
                          const uint32_t (&soff)[GPW], uint32_t w8, uint32_t s8,
                          const uint4 (&bx)[GPW][GATEUP ? 4 : 8], const float (&cx)[GPW][2], Release release,
                          float (&acc)[4]) {
  uint4 wlo[NV], whi[NV];
  float slo[NV], shi[NV];
#pragma unroll
  for (int gi = 0; gi < NV; ++gi) {
    wlo[gi] = lds128(st + woff[gi]);
    whi[gi] = lds128(st + woff[gi] + w8);
    slo[gi] = bf16_to_f32(sc[soff[gi]]);
    shi[gi] = bf16_to_f32(sc[soff[gi] + s8]);
  }
  release();
  // NV independent accumulator pairs (even / odd steps), interleaved per word
  float e[NV][2][4];
#pragma unroll
  for (int gi = 0; gi < NV; ++gi)
#pragma unroll
    for (int h = 0; h < 2; ++h) e[gi][h][0] = e[gi][h][1] = e[gi][h][2] = e[gi][h][3] = 0.0f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
#pragma unroll
    for (int gi = 0; gi < NV; ++gi) {
      const uint32_t u = q == 0 ? wlo[gi].x : q == 1 ? wlo[gi].y : q == 2 ? wlo[gi].z : wlo[gi].w;
      const uint32_t v = q == 0 ? whi[gi].x : q == 1 ? whi[gi].y : q == 2 ? whi[gi].z : whi[gi].w;
      const AWords A = unpack_a(u, v);
      mma16816_bf16(e[gi][0], A.a0, A.a1, A.a2, A.a3, bx[gi][q].x, bx[gi][q].y);
      mma16816_bf16(e[gi][1], A.c0, A.c1, A.c2, A.c3, bx[gi][q].z, bx[gi][q].w);
      if constexpr (!GATEUP) {
        mma16816_bf16(e[gi][0], A.a0, A.a1, A.a2, A.a3, bx[gi][q + 4].x, bx[gi][q + 4].y);
        mma16816_bf16(e[gi][1], A.c0, A.c1, A.c2, A.c3, bx[gi][q + 4].z, bx[gi][q + 4].w);
      }
    }
  }
#pragma unroll
  for (int gi = 0; gi < NV; ++gi) {
    acc[0] = fmaf(slo[gi], (e[gi][0][0] + e[gi][1][0]) - cx[gi][0], acc[0]);
    acc[1] = fmaf(slo[gi], (e[gi][0][1] + e[gi][1][1]) - cx[gi][1], acc[1]);
    acc[2] = fmaf(shi[gi], (e[gi][0][2] + e[gi][1][2]) - cx[gi][0], acc[2]);
    acc[3] = fmaf(shi[gi], (e[gi][0][3] + e[gi][1][3]) - cx[gi][1], acc[3]);
  }
}

template <bool GATEUP, int GPW>
__global__ void __launch_bounds__(Roles<GATEUP>::kThreads, 1) stream_kernel(Args a) {
  constexpr int kMaxParts = PartsCap<GATEUP>::value;
  constexpr int kConsumerWarps = Roles<GATEUP>::kConsumerWarps, kProducerWarp = Roles<GATEUP>::kProducerWarp,
                kEpilogueWarp = Roles<GATEUP>::kEpilogueWarp, kEpilogueWarps = Roles<GATEUP>::kEpilogueWarps,
                kThreads = Roles<GATEUP>::kThreads;
  extern __shared__ __align__(128) unsigned char smem[];
  const int K = a.p0.k, N = a.p0.n;
  const int nG = K / 128;
  const int P = a.parts, S = a.stages, R = a.rows;
  const Smem L = smem_layout<GATEUP>(K, a.max_active);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  const uint32_t bar0 = ac::smem_u32(&bars[0]);
  auto bar = [bar0](int i) { return bar0 + 8u * static_cast<uint32_t>(i); };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 8 * kNumBars);
  int* tab = reinterpret_cast<int*>(smem + L.tab);
  const unsigned char* raw = smem + L.raw;  // [kTok][K] activation rows of the current chunk
  float* red = reinterpret_cast<float*>(smem + L.red);
  unsigned char* stages = smem + L.stage;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const unsigned long long t_entry = ac::global_ns();
  if (threadIdx.x == 0) STREAM_TRACE(0, t_entry);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ac::mbar_init(bar(kBarFull + s), 1);
      ac::mbar_init(bar(kBarEmpty + s), kConsumerWarps);
    }
    for (int b = 0; b < kRedBufs; ++b) {
      ac::mbar_init(bar(kBarRedFull + b), kConsumerWarps);
      ac::mbar_init(bar(kBarRedEmpty + b), kEpilogueWarps);
    }
    ac::mbar_init(bar(kBarXEmpty), kConsumerWarps);
    ac::mbar_init(bar(kBarRaw), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // chunk table: exclusive prefix of ceil(count / 8) over the active experts,
  // every thread loading one entry (warp totals meet in the first red buffer)
  const int n_act = min(*a.n_active, a.max_active);
  const int cap = a.max_active + 1;
  {
    int* wtot = reinterpret_cast<int*>(smem + L.red);
    int run = 0;
    for (int base = 0; base < n_act; base += kThreads) {
      const int i = base + threadIdx.x;
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
      if (lane == 31) wtot[warp] = inc;
      __syncthreads();
      int before = run, all = run;
      for (int w = 0; w < kThreads / 32; ++w) {
        const int v = wtot[w];
        if (w < warp) before += v;
        all += v;
      }
      if (i < n_act) {
        tab[i] = before + inc - c;
        tab[cap + i] = e;
        tab[2 * cap + i] = off;
        tab[3 * cap + i] = cnt;
      }
      run = all;
      __syncthreads();
    }
    if (threadIdx.x == 0) tab[n_act] = run;
  }
  __syncthreads();
  if (threadIdx.x == 0) STREAM_TRACE(1, t_entry);

  const int total_chunks = tab[n_act];
  const int blocks = N / R;
  const long long total = static_cast<long long>(total_chunks) * blocks;
  const int lo = static_cast<int>(total * blockIdx.x / gridDim.x);
  const int hi = static_cast<int>(total * (blockIdx.x + 1) / gridDim.x);
  const size_t rowb = static_cast<size_t>(K) / 2;
  const int sstride = a.p0.sstride;

  if (warp == kProducerWarp) {
    // ---------------- producer ----------------
    if (lane == 0 && hi > lo) {
      Cursor cur{tab, cap};
      int gc = lo / blocks, rbk = lo - gc * blocks;
      ChunkRef c = cur.at(gc);
      int s = 0, ph = 0, issued = 0;
      bool failed = false;
      const uint32_t cpp = static_cast<uint32_t>(R * rowb), spp = static_cast<uint32_t>(R * sstride * 2);
      for (int it = lo; it < hi; ++it) {
        if (!wait_phase(bar(kBarEmpty + s), ph ^ 1, abort_flag)) {
          failed = true;
          break;
        }
        const size_t row0 = static_cast<size_t>(c.e) * N + static_cast<size_t>(rbk) * R;
        const uint32_t dst = ac::smem_u32(stages + static_cast<size_t>(s) * a.stage_bytes);
        const uint32_t fb = bar(kBarFull + s);
        ac::mbar_arrive_expect_tx(fb, a.code_bytes + a.scale_bytes);
        ac::bulk_g2s(dst, a.p0.q + row0 * rowb, cpp, fb);
        if constexpr (GATEUP) {
          ac::bulk_g2s(dst + cpp, a.p1.q + row0 * rowb, cpp, fb);
          ac::bulk_g2s(dst + 2 * cpp, a.p0.s + row0 * sstride, spp, fb);
          ac::bulk_g2s(dst + 2 * cpp + spp, a.p1.s + row0 * sstride, spp, fb);
        } else {
          ac::bulk_g2s(dst + cpp, a.p0.s + row0 * sstride, spp, fb);
        }
        ++issued;
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
        if (++rbk == blocks && it + 1 < hi) {
          rbk = 0;
          c = cur.at(++gc);
        }
      }
      // the copies still in flight land before the CTA may exit: the last
      // min(S, issued) stages, walking back from the next slot
      for (int j = 0; j < min(S, issued); ++j) {
        if (--s < 0) {
          s = S - 1;
          ph ^= 1;
        }
        wait_landed(bar(kBarFull + s), ph);
      }
      STREAM_TRACE(4, t_entry);
      if (a.trace != nullptr) a.trace[blockIdx.x * 16 + 6] = static_cast<unsigned long long>(hi - lo);
      if (failed) atomicOr(a.status, kStatusTimeout);
    }
    return;
  }

  if (warp >= kEpilogueWarp) {
    // ---------------- operand rows (first epilogue warp) + epilogue ----------------
    if (hi <= lo) return;
    const int ew = warp - kEpilogueWarp;
    const uint32_t rowsz = row_bytes<GATEUP>(K);
    // the activation rows of chunk gc into the raw area, one bulk copy per token
    auto stage_rows = [&](const ChunkRef& ch) {
      if (lane == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the consumers' reads before the copies
        ac::mbar_arrive_expect_tx(bar(kBarRaw), static_cast<uint32_t>(ch.cnt) * rowsz);
      }
      __syncwarp();
      if (lane < ch.cnt) {
        const void* src = GATEUP
            ? static_cast<const void*>(a.x + static_cast<size_t>(a.sorted_pair[ch.s0 + lane] / a.top_k) * K)
            : static_cast<const void*>(a.h + static_cast<size_t>(ch.s0 + lane) * K);
        ac::bulk_g2s(ac::smem_u32(raw + static_cast<size_t>(lane) * rowsz), src, rowsz, bar(kBarRaw));
      }
    };
    // lanes per token in an epilogue pass: R is 16 or a multiple of 32 ... (16 | R)
    const int lsh = R < 32 ? 4 : 5, lpt = 1 << lsh, tpp = 32 / lpt;
    Cursor cur{tab, cap}, ahead{tab, cap};
    int gc = lo / blocks, rbk = lo - gc * blocks;
    const int gc_last = (hi - 1) / blocks;
    ChunkRef c = cur.at(gc);
    if (ew == 0) stage_rows(c);
    int staged = 1, xph = 1;  // chunks whose rows were requested; phase of the next xempty wait
    bool failed = false;
    int b = 0, ph = 0;
    for (int it = lo; it < hi; ++it) {
      if (!wait_phase(bar(kBarRedFull + b), ph, abort_flag)) {
        failed = true;
        break;
      }
      // once the consumers have taken a chunk's operands, the next chunk's rows
      if (ew == 0 && gc + 1 <= gc_last && staged == gc + 1 - lo / blocks) {
        if (!wait_phase(bar(kBarXEmpty), xph ^ 1, abort_flag)) {
          failed = true;
          break;
        }
        xph ^= 1;
        stage_rows(ahead.at(gc + 1));
        ++staged;
      }
      // outputs (token n, row r) of this item: a pass of the warp covers tpp
      // tokens (lane >> lsh) and rows r = lane & (lpt - 1) (+ lpt ...); the
      // warps take passes in turn.  All P partials of an output are loaded before
      // they are added in part order (independent shared loads, one dependent
      // add chain); consecutive lanes read consecutive rows (no bank conflicts).
      const float* rp = red + b * kRedFloats;
      float* ob = a.out + static_cast<size_t>(c.s0) * N + rbk * R;
      const int rows = GATEUP ? 2 * R : R;  // item rows in the partial-sum buffer
      for (int n0 = ew * tpp; n0 < kTok; n0 += kEpilogueWarps * tpp) {
        const int n = n0 + (lane >> lsh);
        if (n >= c.cnt) continue;
        for (int r = lane & (lpt - 1); r < R; r += lpt) {
          const float* pg = rp + n * P * rows + r;
          float pv[kMaxParts], pu[GATEUP ? kMaxParts : 1];
#pragma unroll
          for (int q = 0; q < kMaxParts; ++q) {
            pv[q] = q < P ? pg[q * rows] : 0.0f;
            if constexpr (GATEUP) pu[q] = q < P ? pg[q * rows + R] : 0.0f;
          }
          float gs = 0.0f, us = 0.0f;
#pragma unroll
          for (int q = 0; q < kMaxParts; ++q) {
            if (q < P) {
              gs += pv[q];
              if constexpr (GATEUP) us += pu[q];
            }
          }
          const float v = GATEUP ? silu_f32(gs) * us : gs;
          ob[static_cast<size_t>(n) * N + r] = v;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kBarRedEmpty + b));
      if (++b == kRedBufs) {
        b = 0;
        ph ^= 1;
      }
      if (++rbk == blocks && it + 1 < hi) {
        rbk = 0;
        c = cur.at(++gc);
      }
    }
    // the last requested rows land before the CTA may exit
    if (ew == 0 && lane == 0) wait_landed(bar(kBarRaw), (staged - 1) & 1);
    if (lane == 0) STREAM_TRACE(5, t_entry);
    if (failed && lane == 0) atomicOr(a.status, kStatusTimeout);
    return;
  }

  // ---------------- consumers ----------------
  const int part = warp % P, tl = warp / P;
  const int g = lane >> 2, t = lane & 3;
  // stage row of this warp's tile row g: gate/up [gate R rows][up R rows]; down [R rows]
  const int r0 = GATEUP ? (tl & 1) * R + (tl >> 1) * 16 : tl * 16;
  // per group of this warp: byte offset of the lane's 16 code bytes of row g
  // within a stage, and the scale element of row g (row g + 8: + 8 rows)
  uint32_t woff[GPW], soff[GPW];
  bool gon[GPW];
  int nv = 0;  // valid groups of this warp: they come first (G = part + gi * P ascending)
#pragma unroll
  for (int gi = 0; gi < GPW; ++gi) {
    const int G = part + gi * P;
    gon[gi] = G < nG;
    nv += gon[gi] ? 1 : 0;
    woff[gi] = static_cast<uint32_t>((r0 + g) * rowb + G * 64 + 16 * t);
    soff[gi] = static_cast<uint32_t>((r0 + g) * sstride + (G * 128) / a.p0.group);
  }
  const uint32_t w8 = static_cast<uint32_t>(8 * rowb), s8 = static_cast<uint32_t>(8 * sstride);
  Cursor cur{tab, cap};
  uint4 bx[GPW][GATEUP ? 4 : 8];
  float cx[GPW][2];
  bool failed = false;
  int gc = lo / blocks, chunk_end = lo;  // items [.., chunk_end) use the operands in registers
  int k = 0, s = 0, ph = 0, b = 0, rph = 0, xph = 0;
  for (int it = lo; it < hi; ++it, ++k) {
    if (it == chunk_end) {  // first item of a chunk: its operands into registers
      if (it > lo) ++gc;
      chunk_end = min(hi, (gc + 1) * blocks);
      const ChunkRef c = cur.at(gc);
      if (!wait_phase(bar(kBarRaw), xph, abort_flag)) {
        failed = true;
        break;
      }
      xph ^= 1;
      if (threadIdx.x == 0 && it == lo) STREAM_TRACE(2, t_entry);
      // lane (g, t) takes token g's 32 activations [32t, 32t + 32) of each of its
      // groups: operand words in the mma order, and the token's group sum for
      // the 136 * sum(x) correction (tokens past the chunk's count are zero)
      const unsigned char* row = raw + static_cast<size_t>(g) * row_bytes<GATEUP>(K);
      const bool live = g < c.cnt;
#pragma unroll
      for (int gi = 0; gi < GPW; ++gi) {
        const int G = part + gi * P;
        float sum = 0.0f;
        if (gon[gi]) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int k0 = G * 128 + 32 * t + 8 * j;  // first of this word's 8 activations
            if constexpr (GATEUP) {
              uint4 v = make_uint4(0, 0, 0, 0);
              if (live) v = lds128(row + 2 * k0);
              bx[gi][j] = w4_pack_x(v, sum);
            } else {
              uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0;
              if (live) {
                v0 = lds128(row + 4 * k0);
                v1 = lds128(row + 4 * k0 + 16);
              }
              const float f[8] = {__uint_as_float(v0.x), __uint_as_float(v0.y), __uint_as_float(v0.z),
                                  __uint_as_float(v0.w), __uint_as_float(v1.x), __uint_as_float(v1.y),
                                  __uint_as_float(v1.z), __uint_as_float(v1.w)};
              uint16_t hb[8], lb[8];
              float sh = 0.0f, sl = 0.0f;
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                split_bf16(f[i], hb[i], lb[i]);
                sh += bf16_to_f32(hb[i]);
                sl += bf16_to_f32(lb[i]);
              }
              sum += 136.0f * (sh + sl);
              bx[gi][j] = pack_pairs(pack_bf16x2(hb[0], hb[1]), pack_bf16x2(hb[2], hb[3]),
                                     pack_bf16x2(hb[4], hb[5]), pack_bf16x2(hb[6], hb[7]));
              bx[gi][j + 4] = pack_pairs(pack_bf16x2(lb[0], lb[1]), pack_bf16x2(lb[2], lb[3]),
                                         pack_bf16x2(lb[4], lb[5]), pack_bf16x2(lb[6], lb[7]));
            }
          }
        }
        // the 4 lanes of token g hold the group's 4 quarters; the C fragment
        // columns of lane (g, t) are tokens 2t and 2t + 1
        sum += __shfl_xor_sync(kFullMask, sum, 1);
        sum += __shfl_xor_sync(kFullMask, sum, 2);
        cx[gi][0] = __shfl_sync(kFullMask, sum, (2 * t) * 4);
        cx[gi][1] = __shfl_sync(kFullMask, sum, (2 * t + 1) * 4);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kBarXEmpty));
    }
    if (!wait_phase(bar(kBarFull + s), ph, abort_flag)) {
      failed = true;
      break;
    }
    const unsigned char* st = stages + static_cast<size_t>(s) * a.stage_bytes;
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(st + a.code_bytes);
    const uint32_t eb = bar(kBarEmpty + s);
    auto release = [eb, lane]() {
      __syncwarp();
      if (lane == 0) mbar_arrive(eb);  // the stage is in registers now
    };
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (nv == GPW)
      item_compute<GATEUP, GPW>(st, sc, woff, soff, w8, s8, bx, cx, release, acc);
    else if (nv > 0)
      item_compute<GATEUP, 1>(st, sc, woff, soff, w8, s8, bx, cx, release, acc);
    else
      release();
    if (++s == S) {
      s = 0;
      ph ^= 1;
    }
    // partial sums of this warp: red[buf][warp][token][row]
    if (!wait_phase(bar(kBarRedEmpty + b), rph ^ 1, abort_flag)) {
      failed = true;
      break;
    }
    // this warp's partials: red[token][part][item row], item rows of the tile = stage rows r0 + g (+ 8)
    const int rows = GATEUP ? 2 * R : R;
    float* rp = red + b * kRedFloats + part * rows + r0 + g;
    rp[(2 * t) * P * rows] = acc[0];
    rp[(2 * t + 1) * P * rows] = acc[1];
    rp[(2 * t) * P * rows + 8] = acc[2];
    rp[(2 * t + 1) * P * rows + 8] = acc[3];
    warp_arrive(bar(kBarRedFull + b));
    if (++b == kRedBufs) {
      b = 0;
      rph ^= 1;
    }
  }
  if (threadIdx.x == 0) STREAM_TRACE(3, t_entry);
  if (failed && lane == 0) atomicOr(a.status, kStatusTimeout);
}

template <bool GATEUP, int GPW>
static void* kernel_ptr() {
  return reinterpret_cast<void*>(stream_kernel<GATEUP, GPW>);
}

// P (K-parts) of a projection; P divides the consumer warp count and the
// item's rows R = 16 * tiles (gate/up: tiles alternate gate and up rows, so
// R = 8 * tiles) must divide N.  Gate/up: P = 8, at most 2 groups per warp.
// Down: one group per warp (its two-term operand holds twice the registers),
// the smallest P covering the groups.
template <bool GATEUP>
static int pick_parts(int nG, int N) {
  constexpr int C = Roles<GATEUP>::kConsumerWarps;
  if (GATEUP) return nG <= 16 ? 8 : 0;
  for (int p = 1; p <= C; ++p)
    if (C % p == 0 && nG <= p && N % (16 * (C / p)) == 0) return p;
  return 0;
}

struct Plan {
  Args a{};  // every pointer null until the launcher sets it (trace stays null for down)
  void* kern = nullptr;
  size_t smem = 0;
  int threads = 0;
};

template <bool GATEUP>
static bool plan(const QuantProj& p0, int max_active, Plan& pl) {
  const int K = p0.k, N = p0.n;
  if (K % 128 || p0.group % 128 || K % p0.group) return false;
  const int nG = K / 128;
  const int P = pick_parts<GATEUP>(nG, N);
  if (P == 0 || P > PartsCap<GATEUP>::value) return false;
  const int gpw = (nG + P - 1) / P;
  if (gpw > 2) return false;
  const int tiles = Roles<GATEUP>::kConsumerWarps / P;
  const int R = GATEUP ? 16 * tiles / 2 : 16 * tiles;
  if (R < 16 || N % R || (R > 16 && R % 32)) return false;  // the epilogue's lane split: R = 16 or 32j
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
  pl.threads = Roles<GATEUP>::kThreads;
  if constexpr (GATEUP)
    pl.kern = gpw == 1 ? kernel_ptr<true, 1>() : kernel_ptr<true, 2>();
  else
    pl.kern = kernel_ptr<false, 1>();
  return true;
}

static int launch(Plan& pl, int num_sms, cudaStream_t st) {
  if (!ensure_dynamic_smem(pl.kern, pl.smem, pl.threads)) return -1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(num_sms);
  cfg.blockDim = dim3(pl.threads);
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
                         const QuantProj& up, float* h, int* status, unsigned long long* trace, int num_sms,
                         cudaStream_t st) {
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
  a.trace = trace;
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
