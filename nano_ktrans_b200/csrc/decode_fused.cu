// decode_fused.cu — the whole routed-expert step in one launch, for decode-
// sized batches (at most 32 (token, expert) pairs, at most 256 experts).
//
// Replaces, for small T, the chain route -> permute -> gate/up -> down ->
// combine (nano_ktrans/layers/hybrid_moe.py:3321-3329 routing,
// nano_ktrans/kernels/cpu_moe.py:491-539 expert loop and index_add_
// combine, quantized_ops.py:86-124 grouped matvec arithmetic).
//
// One CTA per SM, launched cooperatively (all CTAs co-resident):
//  1. Every CTA routes all T tokens itself (route_warp.cuh, one warp per
//     token) and warp 0 sorts the <= 32 (token, expert) pairs by expert with
//     ballot-radix ranks — no extra launch, no grid barrier.
//  2. Phase B (gate/up): the active experts' gate/up rows form one flat row
//     space split evenly over the CTAs.  A CTA walks its range in stages of up
//     to 16 rows of one expert: one thread issues TMA bulk copies
//     (cp.async.bulk global -> shared, completion counted on an mbarrier) of
//     the gate codes, up codes and both scale rows into a 3-slot ring; warp w
//     computes row w with 16-byte shared loads, the exact unpack of
//     common.cuh and a warp-shuffle reduction, and writes SiLU(gate)*up (fp32)
//     to global h.
//  3. One grid barrier.  Phase-C weight stages are already in flight: their
//     copies are issued as ring slots free up, before the barrier.
//  4. Phase C (down + combine): CTA c owns output rows [c*H/G, (c+1)*H/G).
//     h of every pair is staged in shared memory.  For each stage (a run of
//     consecutive active experts) all 16 warps compute y[expert][row][token]
//     in parallel (8 lanes per row), then one thread per (token, row) adds
//     w * y expert by expert in ascending expert order into an fp32
//     accumulator — the reference's index_add_ order — and the result is
//     written as bf16 once.
// Every wait is bounded: on expiry the kernel records kStatusTimeout in the
// status word, stops computing, drains its outstanding copies (bounded) and
// still arrives at the grid barrier, so no other CTA waits on it.

#include <algorithm>

#include "async_copy.cuh"
#include "common.cuh"
#include "kernels.h"
#include "route_warp.cuh"

namespace moe {

constexpr int kFThreads = 512;
constexpr int kFWarps = kFThreads / 32;
constexpr int kFStages = 3;
constexpr int kFSlotBytes = 34816;  // 16 rows x 2 projections x (1024 + 32) bytes
constexpr int kFMaxStages = 96;     // stage descriptors per CTA
constexpr int kFRowsC = 64;         // phase-C rows per CTA (16 warps x 4 rows)
constexpr int kFMaxPairs = 32;      // (token, expert) pairs per launch
constexpr int kFMaxExpC = 8;        // experts per phase-C stage

struct FusedArgs {
  const uint16_t* x;
  const uint16_t* logits;
  const int64_t* ids_in;
  const uint16_t* w_in;
  const uint8_t* mask;
  int64_t* ids_out;
  uint16_t* w_out;
  QuantProj gate, up, down;
  int T, E, top_k, use_softmax, renorm;
  float* hbuf;
  uint16_t* out;
  unsigned long long* bar;    // grid-barrier arrival counter (monotonic)
  unsigned long long* trace;  // [G][16] %globaltimer stamps, or null
  int* status;
  int rows_b;  // phase-B rows per stage
  int exp_c;   // phase-C experts per stage
  int pc_mode; // 1: every phase-C weight block is copied once, right after routing, into its own region
  // dynamic shared-memory carve-up (byte offsets)
  int off_bar, off_tab, off_stage, off_act, off_acc, off_ys, off_pc;
};

struct StageDesc {
  int kind;  // 0 = gate/up rows of one expert, 1 = down rows of consecutive experts
  int n;     // rows (kind 0) or experts (kind 1)
  int a;     // index into the active-expert table
  int row0;  // first row
};

// Per-launch tables in shared memory.
struct Tables {
  int pair_e[kFMaxPairs];  // expert of pair p = t*k + j, -1 if excluded
  float pair_w[kFMaxPairs];
  int stok[kFMaxPairs];    // token of sorted pair s
  float sw[kFMaxPairs];    // routing weight of sorted pair s
  int act_e[kFMaxPairs];   // active experts, ascending
  int act_s0[kFMaxPairs];  // first sorted pair of active expert a
  int act_n[kFMaxPairs];   // pairs of active expert a
  int pa[kFMaxPairs];      // active-expert index of sorted pair s
  int tok_pairs[kFMaxPairs];  // token t's sorted pairs in ascending expert order, at [t*k, t*k + tok_cnt[t])
  int tok_cnt[kFMaxPairs];
  int n_act, n_pairs, n_stages, n_ring, abort;
};

// mbarrier, bulk-copy and grid-barrier primitives: async_copy.cuh
using ac::bulk_g2s;
using ac::global_ns;
using ac::mbar_init;
using ac::mbar_try_wait;
using ac::mbar_wait_bounded;
using ac::smem_u32;
MOE_DEV void mbar_expect_tx(uint32_t bar, uint32_t bytes) { ac::mbar_arrive_expect_tx(bar, bytes); }

// Phase timestamps (thread 0 of each CTA), when tracing is on: 0 entry,
// 1 routing and stage list done, 2 phase B done, 3 grid barrier passed,
// 4 h staged, 5 exit.
#define MOE_TRACE(i)                                                                              \
  do {                                                                                            \
    if (a.trace != nullptr && threadIdx.x == 0) a.trace[blockIdx.x * 16 + (i)] = global_ns(); \
  } while (0)

// --------------------------------------------------------------------------

// BITS: 4 or 8.  EPL: experts per lane in routing (E <= 32 * EPL).  TOK: max
// tokens per expert handled per pass (1 when T == 1, else 4).
template <int BITS, int EPL, int TOK>
__global__ void __launch_bounds__(kFThreads, 1) moe_decode_fused_kernel(FusedArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int kCodes = ChunkTraits<BITS>::kCodes;
  constexpr int kQ = ChunkTraits<BITS>::kQ;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = a.T, E = a.E, k = a.top_k, P = T * k;
  const int H = a.gate.k, I = a.gate.n;
  const int G = gridDim.x, cta = blockIdx.x;

  unsigned char* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  Tables& tb = *reinterpret_cast<Tables*>(smem + a.off_tab);
  StageDesc* stages = reinterpret_cast<StageDesc*>(smem + a.off_stage);
  float4* act4 = reinterpret_cast<float4*>(smem + a.off_act);
  float* out_acc = reinterpret_cast<float*>(smem + a.off_acc);  // [T][kFRowsC]
  float* ys = reinterpret_cast<float*>(smem + a.off_ys);         // [exp_c][kFRowsC][TOK]
  __shared__ int grid_ok;

  MOE_TRACE(0);
  unsigned long long bar_seen = 0;  // thread 0: the grid-barrier counter before this CTA arrives
  if (tid == 0) {
    for (int s = 0; s <= kFStages; ++s) mbar_init(smem_u32(&bars[s]), 1);  // ring slots + phase-C region
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tb.abort = 0;
    bar_seen = ac::grid_epoch_read(a.bar);
  }
  for (int i = tid; i < T * kFRowsC; i += kFThreads) out_acc[i] = 0.0f;

  // ---- 1. routing: warp t routes token t --------------------------------------
  if (warp < T) {
    const int t = warp;
    int id = -1;
    float w = 0.0f;
    if (a.ids_in != nullptr) {
      if (lane < k) {
        const int64_t v = a.ids_in[t * k + lane];
        id = (v >= 0 && v < E) ? static_cast<int>(v) : -1;
        w = bf16_to_f32(a.w_in[t * k + lane]);
        if (id < 0 && cta == 0) atomicOr(a.status, kStatusBadExpertId);
      }
    } else {
      route_token_warp<EPL>(a.logits + static_cast<size_t>(t) * E, E, k, a.use_softmax != 0, a.renorm != 0, id, w);
      if (cta == 0 && lane < k) {
        a.ids_out[t * k + lane] = id;
        a.w_out[t * k + lane] = f32_to_bf16(w);
      }
    }
    if (lane < k) {
      const bool inc = id >= 0 && (a.mask == nullptr || a.mask[id] != 0);
      tb.pair_e[t * k + lane] = inc ? id : -1;
      tb.pair_w[t * k + lane] = w;
    }
  }
  __syncthreads();

  // ---- warp 0: sort the pairs by expert (stable), build the expert table ----
  if (warp == 0) {
    const int p = lane;
    const int e = p < P ? tb.pair_e[p] : -1;
    const bool valid = e >= 0;
    const uint32_t ek = valid ? static_cast<uint32_t>(e) : 0x7ffu;  // excluded pairs sort last
    uint32_t lt = 0, eq = kFullMask;
#pragma unroll
    for (int b = 10; b >= 0; --b) {
      const uint32_t bit = (ek >> b) & 1u;
      const uint32_t bal = __ballot_sync(kFullMask, bit);
      if (bit) lt |= eq & ~bal;
      eq &= bit ? bal : ~bal;
    }
    const uint32_t below = (1u << lane) - 1u;
    const int rank = __popc(lt) + __popc(eq & below);
    const bool first = valid && (eq & below) == 0;
    const uint32_t firsts = __ballot_sync(kFullMask, first);
    const uint32_t valids = __ballot_sync(kFullMask, valid);
    // this pair's position among its token's valid pairs, by ascending expert
    const int t0 = (p / k) * k;
    const int myrank = valid ? rank : 0x7fffffff;
    int pos = 0;
    for (int jj = 0; jj < k; ++jj) {
      const int r = __shfl_sync(kFullMask, myrank, min(t0 + jj, 31));
      pos += (t0 + jj < P && r < myrank) ? 1 : 0;
    }
    if (valid) {
      tb.stok[rank] = p / k;
      tb.sw[rank] = tb.pair_w[p];
      tb.pa[rank] = __popc(firsts & lt);
      tb.tok_pairs[t0 + pos] = rank;
    }
    if (first) {
      const int ai = __popc(firsts & lt);
      tb.act_e[ai] = e;
      tb.act_s0[ai] = rank;
      tb.act_n[ai] = __popc(eq);
    }
    if (p < T) {
      const uint32_t tok_lanes = (k >= 32 ? kFullMask : ((1u << k) - 1u)) << (p * k);
      tb.tok_cnt[p] = __popc(valids & tok_lanes);
    }
    if (lane == 0) {
      tb.n_act = __popc(firsts);
      tb.n_pairs = __popc(valids);
    }
  }
  __syncthreads();

  // ---- 2. stage list ------------------------------------------------------------
  const int n_act = tb.n_act;
  const int n0 = (cta * H) / G;
  const int nrc = ((cta + 1) * H) / G - n0;
  if (tid == 0) {
    int ns = 0;
    const int total = n_act * I;
    int r = static_cast<int>((static_cast<long long>(total) * cta) / G);
    const int r1 = static_cast<int>((static_cast<long long>(total) * (cta + 1)) / G);
    int ai = r / I, row = r - ai * I;
    while (r < r1 && ns < kFMaxStages) {
      const int n = min(a.rows_b, min(I - row, r1 - r));
      stages[ns++] = StageDesc{0, n, ai, row};
      r += n;
      row += n;
      if (row == I) {
        row = 0;
        ++ai;
      }
    }
    tb.n_ring = ns;  // in pc_mode only the gate/up stages go through the ring
    for (int a0 = 0; nrc > 0 && a0 < n_act && ns < kFMaxStages; a0 += a.exp_c)
      stages[ns++] = StageDesc{1, min(a.exp_c, n_act - a0), a0, n0};
    tb.n_stages = ns;
    if (!a.pc_mode) tb.n_ring = ns;
    if (r < r1) atomicOr(a.status, kStatusTimeout);  // stage table overflow (cannot happen within limits)
  }
  __syncthreads();
  const int nst = tb.n_stages;
  MOE_TRACE(1);

  const size_t rb_b = static_cast<size_t>(H) * BITS / 8, sb_b = static_cast<size_t>(a.gate.sstride) * 2;
  const size_t rb_c = static_cast<size_t>(I) * BITS / 8, sb_c = static_cast<size_t>(a.down.sstride) * 2;
  const size_t per_c = static_cast<size_t>(nrc) * (rb_c + sb_c);

  auto issue = [&](int j) {  // thread 0 only
    const StageDesc d = stages[j];
    const int slot = j % kFStages;
    const uint32_t dst = smem_u32(ring + static_cast<size_t>(slot) * kFSlotBytes);
    const uint32_t bar = smem_u32(&bars[slot]);
    if (d.kind == 0) {
      const size_t rix = static_cast<size_t>(tb.act_e[d.a]) * I + d.row0;
      const uint32_t cb = static_cast<uint32_t>(d.n * rb_b), sbt = static_cast<uint32_t>(d.n * sb_b);
      mbar_expect_tx(bar, 2 * cb + 2 * sbt);
      bulk_g2s(dst, a.gate.q + rix * rb_b, cb, bar);
      bulk_g2s(dst + cb, a.up.q + rix * rb_b, cb, bar);
      bulk_g2s(dst + 2 * cb, a.gate.s + rix * a.gate.sstride, sbt, bar);
      bulk_g2s(dst + 2 * cb + sbt, a.up.s + rix * a.up.sstride, sbt, bar);
    } else {
      mbar_expect_tx(bar, static_cast<uint32_t>(d.n * per_c));
      for (int i = 0; i < d.n; ++i) {
        const size_t rix = static_cast<size_t>(tb.act_e[d.a + i]) * H + d.row0;
        const uint32_t o = dst + static_cast<uint32_t>(i * per_c);
        bulk_g2s(o, a.down.q + rix * rb_c, static_cast<uint32_t>(nrc * rb_c), bar);
        bulk_g2s(o + static_cast<uint32_t>(nrc * rb_c), a.down.s + rix * a.down.sstride,
                 static_cast<uint32_t>(nrc * sb_c), bar);
      }
    }
  };

  const int nring = tb.n_ring;
  unsigned char* pc = smem + a.off_pc;
  int issued = 0;   // thread 0: ring stages whose copies were issued
  int drained = 0;  // thread 0: ring stages whose full barrier it has passed
  bool pc_pending = false;  // thread 0: phase-C region copies issued, not yet waited on
  if (tid == 0) {
    if (a.pc_mode && nrc > 0 && n_act > 0) {
      // every down-projection block this CTA will need, issued before any gate/up stage
      const uint32_t bar = smem_u32(&bars[kFStages]);
      mbar_expect_tx(bar, static_cast<uint32_t>(n_act * per_c));
      for (int i = 0; i < n_act; ++i) {
        const size_t rix = static_cast<size_t>(tb.act_e[i]) * H + n0;
        const uint32_t o = smem_u32(pc + i * per_c);
        bulk_g2s(o, a.down.q + rix * rb_c, static_cast<uint32_t>(nrc * rb_c), bar);
        bulk_g2s(o + static_cast<uint32_t>(nrc * rb_c), a.down.s + rix * a.down.sstride,
                 static_cast<uint32_t>(nrc * sb_c), bar);
      }
      pc_pending = true;
    }
    for (; issued < min(kFStages, nring); ++issued) issue(issued);
  }

  // ---- 3. stage loop ---------------------------------------------------------------
  const int nch_b = H / kCodes, it_b = (nch_b + 31) / 32, k4p_b = it_b * 32 * kQ;
  const int nch_c = I / kCodes, it_c = (nch_c + 7) / 8, k4p_c = it_c * 8 * kQ;
  const int H4 = H / 4, I4 = I / 4;
  // W4 phase-B operands: [TOK][it_b*32 chunks][4 words] uint4, then [TOK][it_b*32] corrections
  const int kw_b = it_b * 32 * 4, cw_b = it_b * 32;
  uint4* xq_b = reinterpret_cast<uint4*>(smem + a.off_act);
  float* corr_b = reinterpret_cast<float*>(xq_b + TOK * kw_b);
  int staged_a = -1;  // active expert whose tokens' x is staged (CTA-uniform)
  bool synced = false;

  for (int j = 0; j < nst; ++j) {
    const StageDesc d = stages[j];
    if (d.kind == 1 && !synced) {
      // phase B -> C: grid barrier, then stage every pair's h (pre-scaled)
      MOE_TRACE(2);
      const bool passed = ac::grid_sync_epoch(a.bar, bar_seen, &grid_ok);
      MOE_TRACE(3);
      if (!passed && tid == 0) {
        atomicOr(a.status, kStatusTimeout);
        tb.abort = 1;
      }
      synced = true;
      const int np = tb.n_pairs;
      for (int idx = tid; idx < np * I4; idx += kFThreads) {
        const int s = idx / I4, f = idx - s * I4;
        const int c = f / kQ, q = f - c * kQ;
        float4 v = __ldcg(reinterpret_cast<const float4*>(a.hbuf + static_cast<size_t>(s) * I) + f);
        v.x *= act_prescale<BITS>(4 * f);
        v.y *= act_prescale<BITS>(4 * f + 1);
        v.z *= act_prescale<BITS>(4 * f + 2);
        v.w *= act_prescale<BITS>(4 * f + 3);
        act4[s * k4p_c + ((c >> 3) * kQ + q) * 8 + (c & 7)] = v;
      }
      __syncthreads();
      MOE_TRACE(4);
    }
    if (d.kind == 0 && d.a != staged_a && !(TOK == 1 && staged_a >= 0)) {
      // stage the tokens of this expert (pre-scaled fp32, interleaved for 32 lanes)
      const int s0 = tb.act_s0[d.a], nt = tb.act_n[d.a];
      if constexpr (BITS == 4) {
        // bf16 operand words + one correction per chunk (common.cuh, W4 with
        // bf16 operands); the 4 words of a chunk sit in 4 adjacent lanes
        const int H8 = H / 8, nw = nt * H8;
        for (int base = 0; base < nw; base += kFThreads) {
          const int idx = base + tid;
          const bool ok = idx < nw;
          const int tt = ok ? idx / H8 : 0, wi = ok ? idx - tt * H8 : 0;
          const int c = wi >> 2, q = wi & 3;
          float corr = 0.0f;
          if (ok) {
            const uint4 raw = *reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(tb.stok[s0 + tt]) * H + 8 * wi);
            xq_b[tt * kw_b + ((c >> 5) * 4 + q) * 32 + (c & 31)] = w4_pack_x(raw, corr);
          }
          corr += __shfl_xor_sync(kFullMask, corr, 1);
          corr += __shfl_xor_sync(kFullMask, corr, 2);
          if (ok && q == 0) corr_b[tt * cw_b + c] = corr;
        }
      } else {
        for (int idx = tid; idx < nt * H4; idx += kFThreads) {
          const int tt = idx / H4, f = idx - tt * H4;
          const int c = f / kQ, q = f - c * kQ;
          const uint2 raw = *reinterpret_cast<const uint2*>(a.x + static_cast<size_t>(tb.stok[s0 + tt]) * H + 4 * f);
          float4 v = make_float4(__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u),
                                 __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xffff0000u));
          act4[tt * k4p_b + ((c >> 5) * kQ + q) * 32 + (c & 31)] = v;
        }
      }
      staged_a = d.a;
      __syncthreads();
    }

    // wait for this stage's bytes (a ring slot, or the phase-C region)
    const int slot = j % kFStages;
    const bool in_ring = j < nring;
    if (!tb.abort) {
      const uint32_t bar = smem_u32(&bars[in_ring ? slot : kFStages]);
      if (mbar_wait_bounded(bar, in_ring ? static_cast<uint32_t>((j / kFStages) & 1) : 0u)) {
        if (tid == 0) {
          if (in_ring) drained = j + 1;
          else pc_pending = false;
        }
      } else {
        atomicOr(a.status, kStatusTimeout);
        tb.abort = 1;
      }
    }
    const unsigned char* sl = in_ring ? ring + static_cast<size_t>(slot) * kFSlotBytes : pc + d.a * per_c;
    if (j < 5) MOE_TRACE(6 + 2 * j);  // stage j: bytes landed

    if (d.kind == 0) {
      if (!tb.abort && warp < d.n) {
        // gate/up row `warp` of this stage for every token of the expert
        const int s0 = tb.act_s0[d.a], nt = tb.act_n[d.a];
        const unsigned char* wg = sl + warp * rb_b;
        const unsigned char* wu = sl + d.n * rb_b + warp * rb_b;
        const uint16_t* sg = reinterpret_cast<const uint16_t*>(sl + 2 * d.n * rb_b + warp * sb_b);
        const uint16_t* su = reinterpret_cast<const uint16_t*>(sl + 2 * d.n * rb_b + d.n * sb_b + warp * sb_b);
        float ag[TOK], au[TOK];
#pragma unroll
        for (int t = 0; t < TOK; ++t) ag[t] = au[t] = 0.0f;
#pragma unroll 2
        for (int it = 0; it < it_b; ++it) {
          const int c = it * 32 + lane;
          if (c < nch_b) {
            const uint4 vg = *reinterpret_cast<const uint4*>(wg + 16 * c);
            const uint4 vu = *reinterpret_cast<const uint4*>(wu + 16 * c);
            const float scg = bf16_to_f32(sg[(c * kCodes) / a.gate.group]);
            const float scu = bf16_to_f32(su[(c * kCodes) / a.up.group]);
            if constexpr (BITS == 4) {
              const uint4* xb = xq_b + (it * 4) * 32 + lane;
#pragma unroll
              for (int t = 0; t < TOK; ++t) {
                if (t < nt) {
                  const float cr = corr_b[t * cw_b + c];
                  ag[t] = fmaf(scg, w4_chunk_dot_bf16(vg, xb + t * kw_b, 32, cr), ag[t]);
                  au[t] = fmaf(scu, w4_chunk_dot_bf16(vu, xb + t * kw_b, 32, cr), au[t]);
                }
              }
            } else {
              const float4* xb = act4 + (it * kQ) * 32 + lane;
#pragma unroll
              for (int t = 0; t < TOK; ++t) {
                if (t < nt) {
                  ag[t] = fmaf(scg, chunk_dot<BITS>(vg, xb + t * k4p_b, 32), ag[t]);
                  au[t] = fmaf(scu, chunk_dot<BITS>(vu, xb + t * k4p_b, 32), au[t]);
                }
              }
            }
          }
        }
#pragma unroll
        for (int t = 0; t < TOK; ++t) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            ag[t] += __shfl_xor_sync(kFullMask, ag[t], o);
            au[t] += __shfl_xor_sync(kFullMask, au[t], o);
          }
        }
        if (lane == 0) {
#pragma unroll
          for (int t = 0; t < TOK; ++t)
            if (t < nt) a.hbuf[static_cast<size_t>(s0 + t) * I + d.row0 + warp] = silu_f32(ag[t]) * au[t];
        }
      }
    } else if (!tb.abort) {
      // down rows of this stage's experts: (expert, row) items over all warps
      const int items = d.n * nrc;
      const int sl8 = lane & 7;
      for (int item0 = warp * 4; item0 < items; item0 += kFWarps * 4) {
        const int item = item0 + (lane >> 3);
        const bool live = item < items;
        const int i = live ? item / nrc : 0, rs = live ? item - i * nrc : 0;
        const int ai = d.a + i;
        const int s0 = tb.act_s0[ai], nt = live ? tb.act_n[ai] : 0;
        const unsigned char* wd = sl + i * per_c + static_cast<size_t>(rs) * rb_c;
        const uint16_t* sd = reinterpret_cast<const uint16_t*>(sl + i * per_c + nrc * rb_c + rs * sb_c);
        float ay[TOK];
#pragma unroll
        for (int t = 0; t < TOK; ++t) ay[t] = 0.0f;
        if (live) {
#pragma unroll 3
          for (int it = 0; it < it_c; ++it) {
            const int c = it * 8 + sl8;
            if (c < nch_c) {
              const uint4 v = *reinterpret_cast<const uint4*>(wd + 16 * c);
              const float sc = bf16_to_f32(sd[(c * kCodes) / a.down.group]);
              const float4* hb = act4 + (it * kQ) * 8 + sl8;
#pragma unroll
              for (int t = 0; t < TOK; ++t)
                if (t < nt) ay[t] = fmaf(sc, chunk_dot<BITS>(v, hb + (s0 + t) * k4p_c, 8), ay[t]);
            }
          }
        }
#pragma unroll
        for (int t = 0; t < TOK; ++t) {
#pragma unroll
          for (int o = 4; o > 0; o >>= 1) ay[t] += __shfl_xor_sync(kFullMask, ay[t], o);
        }
        if (live && sl8 == 0) {
#pragma unroll
          for (int t = 0; t < TOK; ++t)
            if (t < nt) ys[(s0 + t) * kFRowsC + rs] = ay[t];
        }
      }
      __syncthreads();
      // ordered combine: per (token, row), the token's pairs of this stage in
      // ascending expert order (tok_pairs is sorted by expert)
      for (int idx = tid; idx < T * nrc; idx += kFThreads) {
        const int t = idx / nrc, rs = idx - t * nrc;
        float acc = out_acc[t * kFRowsC + rs];
        const int cnt = tb.tok_cnt[t];
        for (int jj = 0; jj < cnt; ++jj) {
          const int s = tb.tok_pairs[t * k + jj];
          const int ai = tb.pa[s];
          if (ai >= d.a && ai < d.a + d.n) acc = __fadd_rn(acc, __fmul_rn(ys[s * kFRowsC + rs], tb.sw[s]));
        }
        out_acc[t * kFRowsC + rs] = acc;
      }
    }
    __syncthreads();  // slot and ys consumed by every thread
    if (j < 5) MOE_TRACE(7 + 2 * j);  // stage j: consumed by every warp
    if (tid == 0 && !tb.abort && issued < nring && issued == j + kFStages) issue(issued++);
  }
  if (!synced) {
    if (!ac::grid_sync_epoch(a.bar, bar_seen, &grid_ok) && tid == 0) atomicOr(a.status, kStatusTimeout);
  }
  // abort path: let copies that were issued but never waited on land before
  // the CTA's shared memory is released (bounded)
  if (tid == 0) {
    for (int j = drained; j < issued; ++j) mbar_wait_bounded(smem_u32(&bars[j % kFStages]), (j / kFStages) & 1);
    if (pc_pending) mbar_wait_bounded(smem_u32(&bars[kFStages]), 0u);
  }
  __syncthreads();
  if (tb.abort) return;
  for (int idx = tid; idx < T * nrc; idx += kFThreads) {
    const int t = idx / nrc, r = idx - t * nrc;
    a.out[static_cast<size_t>(t) * H + n0 + r] = f32_to_bf16(out_acc[t * kFRowsC + r]);
  }
  MOE_TRACE(5);
}

// --------------------------------------------------------------------------
// host side
// --------------------------------------------------------------------------

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static int rows_c_of(int H, int num_sms) { return (H + num_sms - 1) / num_sms; }

bool decode_fused_eligible(int bits, int T, int E, int top_k, const QuantProj& gate, const QuantProj& down,
                           int num_sms) {
  const int H = gate.k, I = gate.n;
  if (T < 1 || T > 4 || T * top_k > kFMaxPairs || E > 256 || E < 1) return false;
  if (bits != 4 && bits != 8) return false;
  const size_t rb_b = static_cast<size_t>(H) * bits / 8, sb_b = static_cast<size_t>(gate.sstride) * 2;
  if (2 * (rb_b + sb_b) > static_cast<size_t>(kFSlotBytes)) return false;  // one gate/up row pair per stage
  const int rows_c = rows_c_of(H, num_sms);
  if (rows_c > kFRowsC) return false;
  const size_t per_c = static_cast<size_t>(rows_c) * (static_cast<size_t>(I) * bits / 8 + down.sstride * 2);
  if (per_c > static_cast<size_t>(kFSlotBytes)) return false;
  const size_t h_bytes = static_cast<size_t>(T) * top_k * I * sizeof(float);
  return h_bytes <= 96 * 1024;
}

template <int BITS, int EPL, int TOK>
static void* kernel_ptr() {
  return reinterpret_cast<void*>(moe_decode_fused_kernel<BITS, EPL, TOK>);
}

template <int BITS, int TOK>
static void* pick_epl(int E) {
  if (E <= 32) return kernel_ptr<BITS, 1, TOK>();
  if (E <= 64) return kernel_ptr<BITS, 2, TOK>();
  if (E <= 128) return kernel_ptr<BITS, 4, TOK>();
  return kernel_ptr<BITS, 8, TOK>();
}

int launch_decode_fused(int bits, const DecodeFusedParams& p, cudaStream_t st) {
  const int H = p.gate.k, I = p.gate.n;
  const int P = p.T * p.top_k;
  const int tok = p.T == 1 ? 1 : 4;
  FusedArgs a{};
  a.x = p.x;
  a.logits = p.logits;
  a.ids_in = p.ids_in;
  a.w_in = p.w_in;
  a.mask = p.mask;
  a.ids_out = p.ids_out;
  a.w_out = p.w_out;
  a.gate = p.gate;
  a.up = p.up;
  a.down = p.down;
  a.T = p.T;
  a.E = p.E;
  a.top_k = p.top_k;
  a.use_softmax = p.use_softmax;
  a.renorm = p.renorm;
  a.hbuf = p.hbuf;
  a.out = p.out;
  a.bar = p.bar;
  a.trace = p.trace;
  a.status = p.status;
  const size_t rb_b = static_cast<size_t>(H) * bits / 8, sb_b = static_cast<size_t>(p.gate.sstride) * 2;
  a.rows_b = static_cast<int>(std::min<size_t>(kFWarps, kFSlotBytes / (2 * (rb_b + sb_b))));
  const int G = p.num_sms;
  const size_t per_c =
      static_cast<size_t>(rows_c_of(H, G)) * (static_cast<size_t>(I) * bits / 8 + p.down.sstride * 2);
  a.exp_c = static_cast<int>(std::min<size_t>(kFMaxExpC, std::max<size_t>(1, kFSlotBytes / per_c)));

  const int kQ = bits == 4 ? 8 : 4, kCodes = bits == 4 ? 32 : 16;
  const int it_b = (H / kCodes + 31) / 32, it_c = (I / kCodes + 7) / 8;
  const size_t xs_bytes = static_cast<size_t>(tok) * it_b * 32 * kQ * 16;
  const size_t hs_bytes = static_cast<size_t>(P) * it_c * 8 * kQ * 16;
  size_t off = static_cast<size_t>(kFStages) * kFSlotBytes;
  a.off_bar = static_cast<int>(off);
  off += (kFStages + 1) * 8;
  off = align_up(off, 16);
  a.off_tab = static_cast<int>(off);
  off += sizeof(Tables);
  off = align_up(off, 16);
  a.off_stage = static_cast<int>(off);
  off += sizeof(StageDesc) * kFMaxStages;
  off = align_up(off, 16);
  a.off_act = static_cast<int>(off);
  off += std::max(xs_bytes, hs_bytes);
  a.off_acc = static_cast<int>(off);
  off += sizeof(float) * static_cast<size_t>(p.T) * kFRowsC;
  a.off_ys = static_cast<int>(off);
  off += sizeof(float) * static_cast<size_t>(kFMaxPairs) * kFRowsC;  // ys[sorted pair][row]
  off = align_up(off, 128);
  // phase-C region: room for the down blocks of every expert a launch can route
  const size_t pc_bytes = static_cast<size_t>(std::min(P, p.E)) * per_c;
  const size_t smem_limit = 227 * 1024;
  a.pc_mode = off + pc_bytes <= smem_limit ? 1 : 0;
  a.off_pc = static_cast<int>(off);
  if (a.pc_mode) {
    off += pc_bytes;
    a.exp_c = kFMaxPairs;  // the region holds every active expert: one phase-C stage
  }
  const size_t smem = off;
  if (smem > smem_limit) return -1;

  void* kern = bits == 4 ? (tok == 1 ? pick_epl<4, 1>(p.E) : pick_epl<4, 4>(p.E))
                         : (tok == 1 ? pick_epl<8, 1>(p.E) : pick_epl<8, 4>(p.E));
  if (!ensure_dynamic_smem(kern, smem, kFThreads)) return -1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {&a};
  return cudaLaunchKernelExC(&cfg, kern, args) == cudaSuccess ? 1 : -2;
}

}  // namespace moe
