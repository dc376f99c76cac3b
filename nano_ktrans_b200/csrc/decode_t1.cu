// decode_t1.cu — the routed-expert step of a single decode token in one
// launch (W4 weights), built to keep HBM busy from the first microsecond.
//
// Replaces, for T == 1, the chain route -> permute -> gate/up -> down ->
// combine (nano_ktrans/layers/hybrid_moe.py:3321-3329 routing,
// nano_ktrans/kernels/cpu_moe.py:491-539 expert loop and index_add_
// combine, quantized_ops.py:86-124 grouped matvec arithmetic).
//
// One CTA of 1024 threads per SM, launched cooperatively:
//  1. Thread 0 bulk-copies the token's logits and activations into shared
//     memory at entry.  Warp 0 routes the token (route_warp.cuh) and orders
//     its experts ascending; the other warps pack x into bf16 operand words.
//  2. The routed experts' gate/up rows form one flat row space split evenly
//     over the CTAs.  Each CTA's whole share (about 42 row pairs, 88 KB at
//     Qwen3 shapes) is requested at once, in chunks of up to 8 rows with one
//     mbarrier each, followed by every down-projection block the CTA will
//     need in phase 4.  Nothing waits for shared memory to be recycled.
//  3. Warp w computes rows w, w+32, ... as soon as each row's chunk lands:
//     gate and up dot products with the exact bf16-operand W4 arithmetic of
//     common.cuh, warp-shuffle reduced, SiLU(gate)*up written to global h.
//  4. One grid barrier; h of every routed expert is staged in shared memory.
//  5. CTA c owns output rows [c*H/G, (c+1)*H/G): 8 lanes per (expert, row)
//     compute the down projection from the blocks already in shared memory,
//     then one thread per row adds w * y over the experts in ascending
//     expert order in fp32 (the reference's index_add_ order) and writes bf16.
// Every wait is bounded; on expiry the kernel records kStatusTimeout, stops
// computing, still arrives at the grid barrier and lets its issued copies
// land before exiting.
#include <algorithm>

#include "async_copy.cuh"
#include "common.cuh"
#include "kernels.h"
#include "route_warp.cuh"

namespace moe {
namespace t1 {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxK = 32;        // routed experts of the token
constexpr int kChunkRows = 8;    // phase-2 rows per bulk-copy chunk
constexpr int kMaxChunks = 40;
constexpr int kRowsC = 64;       // phase-5 rows per CTA

struct Args {
  const uint16_t* x;
  const uint16_t* logits;  // routing computed in-kernel when ids_in == nullptr
  const int64_t* ids_in;
  const uint16_t* w_in;
  const uint8_t* mask;
  int64_t* ids_out;
  uint16_t* w_out;
  QuantProj gate, up, down;
  int E, top_k, use_softmax, renorm;
  float* hbuf;  // [k][I]
  uint16_t* out;
  unsigned long long* bar;
  unsigned long long* trace;  // [G][16] %globaltimer stamps, or null
  int* status;
  // dynamic shared-memory carve-up (byte offsets)
  int off_lg, off_x, off_xq, off_corr, off_b, off_c, off_sb, off_sc, off_act, off_ys, off_tab, off_bar;
};

struct Chunk {
  int a;     // active-expert index
  int row0;  // first row within the expert
  int n;     // rows
  int lr0;   // first local row of the CTA's range
  int off;   // byte offset in the phase-2 region
};

struct Tab {
  int act_e[kMaxK];    // routed experts, ascending
  float act_w[kMaxK];  // their routing weights
  Chunk ch[kMaxChunks];
  int n_act, n_chunks, n_rows, r0, abort;
};

#define T1_TRACE(i)                                                                                 \
  do {                                                                                              \
    if (a.trace != nullptr && threadIdx.x == 0) a.trace[blockIdx.x * 16 + (i)] = ac::global_ns(); \
  } while (0)

template <int EPL>
__global__ void __launch_bounds__(kThreads, 1) moe_decode_t1_kernel(Args a) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int kCodes = ChunkTraits<4>::kCodes;  // 32
  constexpr int kQ = ChunkTraits<4>::kQ;          // 8
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = a.E, k = a.top_k;
  const int H = a.gate.k, I = a.gate.n;
  const int G = gridDim.x, cta = blockIdx.x;

  uint16_t* lg = reinterpret_cast<uint16_t*>(smem + a.off_lg);
  const uint16_t* xs = reinterpret_cast<const uint16_t*>(smem + a.off_x);
  uint4* xq = reinterpret_cast<uint4*>(smem + a.off_xq);
  float* corr = reinterpret_cast<float*>(smem + a.off_corr);
  unsigned char* reg_b = smem + a.off_b;
  unsigned char* reg_c = smem + a.off_c;
  uint16_t* sc_b = reinterpret_cast<uint16_t*>(smem + a.off_sb);  // [row][gate, up][gate.sstride] scales
  uint16_t* sc_c = reinterpret_cast<uint16_t*>(smem + a.off_sc);  // [expert][row][down.sstride] scales
  float4* act4 = reinterpret_cast<float4*>(smem + a.off_act);
  float* ys = reinterpret_cast<float*>(smem + a.off_ys);  // [k][kRowsC]
  Tab& tb = *reinterpret_cast<Tab*>(smem + a.off_tab);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_bar);  // [0] inputs, [1] phase-5 blocks, [2+i] chunk i
  __shared__ int grid_ok;
  volatile int* abort_flag = &tb.abort;
  auto fail = [&]() {
    *abort_flag = 1;
    atomicOr(a.status, kStatusTimeout);
  };

  const bool route_here = a.ids_in == nullptr;
  T1_TRACE(0);
  if (tid == 0) {
    for (int i = 0; i < 2 + kMaxChunks; ++i) ac::mbar_init(ac::smem_u32(&bars[i]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint32_t b0 = ac::smem_u32(&bars[0]);
    const uint32_t xb = static_cast<uint32_t>(H) * 2, lb = route_here ? static_cast<uint32_t>(E) * 2 : 0u;
    ac::mbar_arrive_expect_tx(b0, xb + lb);
    ac::bulk_g2s(ac::smem_u32(smem + a.off_x), a.x, xb, b0);
    if (route_here) ac::bulk_g2s(ac::smem_u32(lg), a.logits, lb, b0);
    tb.abort = 0;
  }
  __syncthreads();
  const bool in_ok = __all_sync(kFullMask, ac::mbar_wait_bounded(ac::smem_u32(&bars[0]), 0u));
  if (!in_ok && lane == 0) fail();

  // ---- 1. routing (warp 0) and x packing (the other warps) --------------------------
  const int nch_b = H / kCodes, it_b = (nch_b + 31) / 32;
  if (warp == 0) {
    int id = -1;
    float w = 0.0f;
    if (!route_here) {
      if (lane < k) {
        const int64_t v = a.ids_in[lane];
        id = (v >= 0 && v < E) ? static_cast<int>(v) : -1;
        w = bf16_to_f32(a.w_in[lane]);
        if (id < 0 && cta == 0) atomicOr(a.status, kStatusBadExpertId);
      }
    } else if (in_ok) {
      route_token_warp<EPL>(lg, E, k, a.use_softmax != 0, a.renorm != 0, id, w);
      if (cta == 0 && lane < k) {
        a.ids_out[lane] = id;
        a.w_out[lane] = f32_to_bf16(w);
      }
    }
    const bool valid = lane < k && id >= 0 && (a.mask == nullptr || a.mask[id] != 0);
    // rank among the valid pairs by (expert, slot)
    int rank = 0;
    for (int m = 0; m < k; ++m) {
      const int em = __shfl_sync(kFullMask, valid ? id : -1, m);
      rank += (em >= 0 && (em < id || (em == id && m < lane))) ? 1 : 0;
    }
    if (valid) {
      tb.act_e[rank] = id;
      tb.act_w[rank] = w;
    }
    const int n_act = __popc(__ballot_sync(kFullMask, valid));
    // this CTA's share [r0, r1) of the flat (expert, row) space, cut at multiples
    // of kChunkRows (I is a multiple of it, so no chunk spans two experts):
    // lane j builds chunk j
    const int total = n_act * I;
    const int r0 = static_cast<int>((static_cast<long long>(total) * cta) / G);
    const int r1 = static_cast<int>((static_cast<long long>(total) * (cta + 1)) / G);
    const int c0 = r0 / kChunkRows;
    const int nc = r1 > r0 ? (r1 + kChunkRows - 1) / kChunkRows - c0 : 0;
    const int rowpair = H;  // gate + up codes of one row: 2 x H/2 bytes
    for (int j = lane; j < nc && j < kMaxChunks; j += 32) {
      const int b = max(r0, (c0 + j) * kChunkRows), e = min(r1, (c0 + j + 1) * kChunkRows);
      const int ai = b / I;
      tb.ch[j] = Chunk{ai, b - ai * I, e - b, b - r0, (b - r0) * rowpair};
    }
    if (lane == 0) {
      tb.n_act = n_act;
      tb.n_chunks = min(nc, kMaxChunks);
      tb.n_rows = r1 - r0;
      tb.r0 = r0;
      if (nc > kMaxChunks) fail();  // chunk table overflow: excluded by the launch limits
    }
  } else if (in_ok) {
    // bf16 operand words + one correction per 32-code chunk (w4_pack_x)
    const int H8 = H / 8;
    for (int base = 0; base < H8; base += kThreads - 32) {
      const int wi = base + tid - 32;
      const bool ok = wi < H8;
      const int c = ok ? wi >> 2 : 0, q = wi & 3;
      float cr = 0.0f;
      if (ok) {
        const uint4 raw = *reinterpret_cast<const uint4*>(xs + 8 * wi);
        xq[((c >> 5) * 4 + q) * 32 + (c & 31)] = w4_pack_x(raw, cr);
      }
      cr += __shfl_xor_sync(kFullMask, cr, 1);
      cr += __shfl_xor_sync(kFullMask, cr, 2);
      if (ok && q == 0) corr[c] = cr;
    }
  }
  __syncthreads();
  T1_TRACE(1);

  // ---- 2. request every byte this CTA will read -----------------------------------------
  const int n_act = tb.n_act, nchunks = tb.n_chunks;
  const size_t rb_b = static_cast<size_t>(H) / 2, rb_c = static_cast<size_t>(I) / 2;
  const int ssb = a.gate.sstride, ssc = a.down.sstride;  // bf16 per scale row (multiples of 8)
  const int n0 = (cta * H) / G;
  const int nrc = ((cta + 1) * H) / G - n0;
  const size_t per_c = static_cast<size_t>(nrc) * rb_c;
  const int nrows = tb.n_rows, r0 = tb.r0;
  const bool issued = !*abort_flag;  // CTA-uniform: nothing writes the flag between the barrier above and here
  if (issued && warp == 0) {
    // bulk copies of the codes only (the TMA unit takes one request at a time,
    // so chunk 0 goes first, then the other gate/up chunks, then the down blocks)
    auto issue_chunk = [&](int j) {
      const Chunk c = tb.ch[j];
      const uint32_t bar = ac::smem_u32(&bars[2 + j]);
      const uint32_t dst = ac::smem_u32(reg_b + c.off);
      const size_t rix = static_cast<size_t>(tb.act_e[c.a]) * I + c.row0;
      const uint32_t cb = static_cast<uint32_t>(c.n * rb_b);
      ac::mbar_arrive_expect_tx(bar, 2 * cb);
      ac::bulk_g2s(dst, a.gate.q + rix * rb_b, cb, bar);
      ac::bulk_g2s(dst + cb, a.up.q + rix * rb_b, cb, bar);
    };
    if (lane == 0 && nchunks > 0) issue_chunk(0);
    __syncwarp();
    for (int j = 1 + lane; j < nchunks; j += 32) issue_chunk(j);
    __syncwarp();
    if (nrc > 0 && n_act > 0) {
      const uint32_t bar = ac::smem_u32(&bars[1]);
      if (lane == 0) ac::mbar_arrive_expect_tx(bar, static_cast<uint32_t>(n_act * per_c));
      __syncwarp();
      for (int i = lane; i < n_act; i += 32) {
        const size_t rix = static_cast<size_t>(tb.act_e[i]) * H + n0;
        ac::bulk_g2s(ac::smem_u32(reg_c + i * per_c), a.down.q + rix * rb_c, static_cast<uint32_t>(per_c), bar);
      }
    }
  } else if (issued) {
    // the other warps fetch the scale rows with plain 16-byte loads meanwhile
    const int vb = ssb / 8, vc = ssc / 8;  // 16-byte vectors per scale row
    const int nb = nrows * 2 * vb, ncv = n_act * nrc * vc;
    for (int v = tid - 32; v < nb + ncv; v += kThreads - 32) {
      const uint4* src;
      uint4* dst;
      if (v < nb) {
        const int lr = v / (2 * vb), rem = v - lr * 2 * vb, pj = rem / vb, q = rem - pj * vb;
        const int gr = r0 + lr, ai = gr / I;
        const size_t srow = static_cast<size_t>(tb.act_e[ai]) * I + (gr - ai * I);
        src = reinterpret_cast<const uint4*>((pj == 0 ? a.gate.s : a.up.s) + srow * ssb) + q;
        dst = reinterpret_cast<uint4*>(sc_b + (lr * 2 + pj) * ssb) + q;
      } else {
        const int u = v - nb, ir = u / vc, q = u - ir * vc;
        const int i = ir / nrc, rs = ir - i * nrc;
        src = reinterpret_cast<const uint4*>(a.down.s + (static_cast<size_t>(tb.act_e[i]) * H + n0 + rs) * ssc) + q;
        dst = reinterpret_cast<uint4*>(sc_c + ir * ssc) + q;
      }
      *dst = __ldg(src);
    }
  }
  __syncthreads();  // scales in shared memory; the code copies are still in flight
  T1_TRACE(2);

  // ---- 3. gate/up rows as their chunks land -----------------------------------------------
  for (int lr = warp; lr < nrows; lr += kWarps) {
    if (__any_sync(kFullMask, *abort_flag)) break;
    int ci = 0;
    while (ci + 1 < nchunks && tb.ch[ci + 1].lr0 <= lr) ++ci;
    const Chunk c = tb.ch[ci];
    if (!__all_sync(kFullMask, ac::mbar_wait_bounded(ac::smem_u32(&bars[2 + ci]), 0u))) {
      if (lane == 0) fail();
      break;
    }
    const int rr = lr - c.lr0;  // row within the chunk
    const unsigned char* base = reg_b + c.off;
    const unsigned char* wg = base + rr * rb_b;
    const unsigned char* wu = base + c.n * rb_b + rr * rb_b;
    const uint16_t* sg = sc_b + (lr * 2) * ssb;
    const uint16_t* su = sc_b + (lr * 2 + 1) * ssb;
    const int gsh = 31 - __clz(a.gate.group / kCodes);  // chunks per scale group, a power of two
    float ag = 0.0f, au = 0.0f;
#pragma unroll 2
    for (int it = 0; it < it_b; ++it) {
      const int ch = it * 32 + lane;
      if (ch < nch_b) {
        const uint4 vg = *reinterpret_cast<const uint4*>(wg + 16 * ch);
        const uint4 vu = *reinterpret_cast<const uint4*>(wu + 16 * ch);
        const float scg = bf16_to_f32(sg[ch >> gsh]);
        const float scu = bf16_to_f32(su[ch >> gsh]);
        const uint4* xb = xq + (it * 4) * 32 + lane;
        const float cr = corr[ch];
        ag = fmaf(scg, w4_chunk_dot_bf16(vg, xb, 32, cr), ag);
        au = fmaf(scu, w4_chunk_dot_bf16(vu, xb, 32, cr), au);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ag += __shfl_xor_sync(kFullMask, ag, o);
      au += __shfl_xor_sync(kFullMask, au, o);
    }
    if (lane == 0) a.hbuf[static_cast<size_t>(c.a) * I + c.row0 + rr] = silu_f32(ag) * au;
  }
  T1_TRACE(3);

  // ---- 4. grid barrier, stage h ----------------------------------------------------------------
  const bool passed = ac::grid_sync_bounded(a.bar, &grid_ok);
  if (!passed && tid == 0) fail();
  T1_TRACE(4);
  const int nch_c = I / kCodes, it_c = (nch_c + 7) / 8, k4p_c = it_c * 8 * kQ;
  const int I4 = I / 4;
  for (int idx = tid; idx < n_act * I4; idx += kThreads) {
    const int s = idx / I4, f = idx - s * I4;
    const int c = f / kQ, q = f - c * kQ;
    float4 v = __ldcg(reinterpret_cast<const float4*>(a.hbuf + static_cast<size_t>(s) * I) + f);
    v.x *= act_prescale<4>(4 * f);
    v.y *= act_prescale<4>(4 * f + 1);
    v.z *= act_prescale<4>(4 * f + 2);
    v.w *= act_prescale<4>(4 * f + 3);
    act4[s * k4p_c + ((c >> 3) * kQ + q) * 8 + (c & 7)] = v;
  }
  __syncthreads();
  T1_TRACE(5);

  // ---- 5. down rows + ordered combine ---------------------------------------------------------------
  const bool c_ok = !issued || nrc == 0 || n_act == 0 || ac::mbar_wait_bounded(ac::smem_u32(&bars[1]), 0u);
  if (!c_ok) fail();
  __syncthreads();
  T1_TRACE(6);
  const bool ok5 = !*abort_flag;  // CTA-uniform after the barrier above
  if (ok5) {
    const int items = n_act * nrc;
    const int sl8 = lane & 7;
    const int gshc = 31 - __clz(a.down.group / kCodes);
    for (int item0 = warp * 4; item0 < items; item0 += kWarps * 4) {
      const int item = item0 + (lane >> 3);
      const bool live = item < items;
      const int i = live ? item / nrc : 0, rs = live ? item - i * nrc : 0;
      const unsigned char* wd = reg_c + i * per_c + static_cast<size_t>(rs) * rb_c;
      const uint16_t* sd = sc_c + (i * nrc + rs) * ssc;
      float ay = 0.0f;
      if (live) {
#pragma unroll 3
        for (int it = 0; it < it_c; ++it) {
          const int ch = it * 8 + sl8;
          if (ch < nch_c) {
            const uint4 v = *reinterpret_cast<const uint4*>(wd + 16 * ch);
            const float sc = bf16_to_f32(sd[ch >> gshc]);
            ay = fmaf(sc, chunk_dot<4>(v, act4 + i * k4p_c + (it * kQ) * 8 + sl8, 8), ay);
          }
        }
      }
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) ay += __shfl_xor_sync(kFullMask, ay, o);
      if (live && sl8 == 0) ys[i * kRowsC + rs] = ay;
    }
  }
  __syncthreads();
  T1_TRACE(7);
  if (ok5 && tid < nrc) {
    float acc = 0.0f;
    for (int i = 0; i < n_act; ++i) acc = __fadd_rn(acc, __fmul_rn(ys[i * kRowsC + tid], tb.act_w[i]));
    a.out[n0 + tid] = f32_to_bf16(acc);
  }
  // copies issued but never waited on (abort path) must land before exit
  if (issued && !ok5 && tid == 0) {
    for (int i = 0; i < nchunks; ++i) ac::mbar_wait_bounded(ac::smem_u32(&bars[2 + i]), 0u);
    if (nrc > 0 && n_act > 0) ac::mbar_wait_bounded(ac::smem_u32(&bars[1]), 0u);
  }
  T1_TRACE(8);
}

}  // namespace t1

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static size_t t1_align(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct T1Plan {
  t1::Args a{};
  size_t smem = 0;
};

// Shared-memory plan of the single-token kernel; smem == 0 when it does not fit.
static T1Plan t1_plan(const DecodeT1Params& p) {
  T1Plan pl;
  const int H = p.gate.k, I = p.gate.n, k = p.top_k, G = p.num_sms;
  const size_t rowpair = static_cast<size_t>(H);  // gate + up codes of one row
  const size_t rows_b = (static_cast<size_t>(k) * I + G - 1) / G;
  const int nrc = (H + G - 1) / G;
  const size_t per_c = static_cast<size_t>(nrc) * (static_cast<size_t>(I) / 2);
  const int it_b = (H / 32 + 31) / 32, it_c = (I / 32 + 7) / 8;
  size_t off = 0;
  auto take = [&](size_t bytes, size_t align) {
    off = t1_align(off, align);
    const size_t o = off;
    off += bytes;
    return static_cast<int>(o);
  };
  pl.a.off_b = take(rows_b * rowpair, 128);
  pl.a.off_c = take(static_cast<size_t>(k) * per_c, 128);
  pl.a.off_sb = take(rows_b * 2 * p.gate.sstride * 2, 16);
  pl.a.off_sc = take(static_cast<size_t>(k) * nrc * p.down.sstride * 2, 16);
  pl.a.off_x = take(static_cast<size_t>(H) * 2, 128);
  pl.a.off_lg = take(static_cast<size_t>(p.E) * 2, 128);
  pl.a.off_xq = take(static_cast<size_t>(it_b) * 32 * 4 * 16, 16);
  pl.a.off_corr = take(static_cast<size_t>(it_b) * 32 * 4, 16);
  pl.a.off_act = take(static_cast<size_t>(k) * it_c * 8 * 8 * 16, 16);
  pl.a.off_ys = take(static_cast<size_t>(k) * t1::kRowsC * 4, 16);
  pl.a.off_tab = take(sizeof(t1::Tab), 16);
  pl.a.off_bar = take(8 * (2 + t1::kMaxChunks), 8);
  pl.smem = off;
  const size_t chunks = (rows_b + t1::kChunkRows - 1) / t1::kChunkRows + 1;  // aligned chunks over the share
  if (off > 227 * 1024 || nrc > t1::kRowsC || chunks > static_cast<size_t>(t1::kMaxChunks)) pl.smem = 0;
  return pl;
}

bool decode_t1_eligible(const DecodeT1Params& p) {
  const int H = p.gate.k, I = p.gate.n;
  if (p.bits != 4 || p.top_k < 1 || p.top_k > t1::kMaxK || p.E < 1 || p.E > 256) return false;
  if (H % 256 || I % 256) return false;  // whole 8-lane and 32-lane chunk rounds
  // scale groups: powers of two that are multiples of the 32-code chunk
  for (int g : {p.gate.group, p.down.group})
    if (g < 32 || (g & (g - 1)) || g % 32) return false;
  if (p.up.group != p.gate.group || p.up.sstride != p.gate.sstride) return false;
  if (reinterpret_cast<uintptr_t>(p.x) % 16) return false;
  if (p.logits != nullptr && (reinterpret_cast<uintptr_t>(p.logits) % 16 || (p.E * 2) % 16)) return false;
  return t1_plan(p).smem > 0;
}

template <int EPL>
static void* t1_kernel() {
  return reinterpret_cast<void*>(t1::moe_decode_t1_kernel<EPL>);
}

int launch_decode_t1(const DecodeT1Params& p, cudaStream_t st) {
  T1Plan pl = t1_plan(p);
  if (pl.smem == 0) return -1;
  t1::Args& a = pl.a;
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
  a.E = p.E;
  a.top_k = p.top_k;
  a.use_softmax = p.use_softmax;
  a.renorm = p.renorm;
  a.hbuf = p.hbuf;
  a.out = p.out;
  a.bar = p.bar;
  a.trace = p.trace;
  a.status = p.status;
  void* kern = p.E <= 32 ? t1_kernel<1>() : p.E <= 64 ? t1_kernel<2>() : p.E <= 128 ? t1_kernel<4>() : t1_kernel<8>();
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(pl.smem)) !=
      cudaSuccess)
    return -1;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, t1::kThreads, pl.smem) != cudaSuccess ||
      per_sm < 1)
    return -1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.num_sms);
  cfg.blockDim = dim3(t1::kThreads);
  cfg.dynamicSmemBytes = pl.smem;
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
