// decode_t1.cu — the routed-expert step of a single decode token in one
// launch (W4 weights), built to keep HBM busy from the first microsecond.
//
// Replaces, for T == 1, the chain route -> permute -> gate/up -> down ->
// combine (nano_ktrans/layers/hybrid_moe.py:3321-3329 routing,
// nano_ktrans/kernels/cpu_moe.py:491-539 expert loop and index_add_
// combine, quantized_ops.py:86-124 grouped matvec arithmetic).
//
// One CTA of 1024 threads per SM, launched cooperatively and as a
// programmatic dependent of the previous kernel on the stream (its launch
// overlaps that kernel's tail; griddepcontrol.wait precedes every global
// access):
//  1. Thread 0 bulk-copies the token's logits and activations into shared
//     memory at entry.  Warp 0 routes the token (route_warp.cuh) and orders
//     its experts ascending; the other warps pack x into bf16 operand words.
//  2. The routed experts' gate/up rows form one flat row space split evenly
//     over the CTAs.  Each CTA's whole share (about 42 row pairs, 88 KB at
//     Qwen3 shapes) is requested at once, in chunks of up to 4 rows with one
//     mbarrier each, followed by every down-projection block the CTA will
//     need in phase 5.  Nothing waits for shared memory to be recycled.
//  3. Warp w computes rows w, w+32, ... as soon as each row's chunk lands:
//     gate and up dot products with the exact bf16-operand W4 arithmetic of
//     common.cuh, warp-shuffle reduced, SiLU(gate)*up written to global h.
//  4. One grid barrier; every CTA stages h of all routed experts in shared
//     memory as bf16 (high, low) operand pairs.
//  5. CTA c owns output rows [c*H/G, (c+1)*H/G): 16-row tiles of each routed
//     expert's down block (already in shared memory) against h on the
//     warp-level tensor-core path (mma_gemv.cuh), B's column halves carrying
//     the high and low parts of h; then one warp per row adds w * y over the
//     experts in ascending expert order in fp32 (the reference's index_add_
//     order) and writes bf16.
// Every wait is bounded; on expiry the kernel records kStatusTimeout, stops
// computing, still arrives at the grid barrier and lets its issued copies
// land before exiting.
#include <algorithm>

#include "async_copy.cuh"
#include "common.cuh"
#include "kernels.h"
#include "mma_gemv.cuh"
#include "route_warp.cuh"

namespace moe {
namespace t1 {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxK = 32;        // routed experts of the token
constexpr int kChunkRows = 4;    // phase-2 rows per bulk-copy chunk (4 measured fastest of 2, 4, 8, 16)
constexpr int kMaxChunks = 40;
constexpr int kRowsC = 64;       // most phase-5 output rows per CTA

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
  unsigned long long* trace;  // [G][16] phase stamps (see T1_TRACE), or null
  int* status;
  // dynamic shared-memory carve-up (byte offsets)
  int off_lg, off_x, off_xq, off_corr, off_b, off_c, off_sb, off_sc, off_act, off_cc, off_tt, off_ys, off_tab, off_bar;
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

// Phase stamps (MOE_OPT_TRACE), thread 0 of each CTA: slot 0 holds %globaltimer
// at entry (ns), slots 1-12 SM clock cycles since entry.
#define T1_TRACE(i)                                                                      \
  do {                                                                                   \
    if (a.trace != nullptr && threadIdx.x == 0)                                          \
      a.trace[blockIdx.x * 16 + (i)] = (i) == 0 ? ac::global_ns() : clock64() - t_entry; \
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
  Tab& tb = *reinterpret_cast<Tab*>(smem + a.off_tab);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_bar);  // [0] inputs, [1] phase-5 blocks, [2+i] chunk i
  __shared__ int grid_ok;
  volatile int* abort_flag = &tb.abort;
  auto fail = [&]() {
    *abort_flag = 1;
    atomicOr(a.status, kStatusTimeout);
  };

  const bool route_here = a.ids_in == nullptr;
  // Programmatic dependent launch: this grid may start while the previous
  // kernel on the stream finishes; nothing in global memory is touched before
  // that kernel has completed and its writes are visible.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const long long t_entry = clock64();
  T1_TRACE(0);
  unsigned long long bar_seen = 0;  // thread 0: the grid-barrier counter before this CTA arrives
  if (tid == 0) {
    // the input barrier first, so the input copies leave before the other inits
    const uint32_t b0 = ac::smem_u32(&bars[0]);
    ac::mbar_init(b0, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint32_t xb = static_cast<uint32_t>(H) * 2, lb = route_here ? static_cast<uint32_t>(E) * 2 : 0u;
    ac::mbar_arrive_expect_tx(b0, xb + lb);
    ac::bulk_g2s(ac::smem_u32(smem + a.off_x), a.x, xb, b0);
    if (route_here) ac::bulk_g2s(ac::smem_u32(lg), a.logits, lb, b0);
    for (int i = 1; i < 2 + kMaxChunks; ++i) ac::mbar_init(ac::smem_u32(&bars[i]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tb.abort = 0;
    bar_seen = ac::grid_epoch_read(a.bar);
  }
  __syncthreads();
  const bool in_ok = __all_sync(kFullMask, ac::mbar_wait_bounded(ac::smem_u32(&bars[0]), 0u));
  if (!in_ok && lane == 0) fail();
  T1_TRACE(1);

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
      T1_TRACE(2);
      if (cta == 0 && lane < k) {
        a.ids_out[lane] = id;
        a.w_out[lane] = f32_to_bf16(w);
      }
    }
    const bool valid = lane < k && id >= 0 && (a.mask == nullptr || a.mask[id] != 0);
    // rank among the valid pairs by (expert, slot)
    int rank = 0;
    const int vid = valid ? id : -1;
#pragma unroll 8
    for (int m = 0; m < k; ++m) {
      const int em = __shfl_sync(kFullMask, vid, m);
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
    const int r0 = static_cast<int>(static_cast<uint32_t>(total) * cta / static_cast<uint32_t>(G));
    const int r1 = static_cast<int>(static_cast<uint32_t>(total) * (cta + 1) / static_cast<uint32_t>(G));
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
    T1_TRACE(3);
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
  T1_TRACE(4);

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
    // phase-5 task table: (expert slot, 16-row tile, 128-code group, scale index)
    const int ts = (nrc + 15) / 16, ngc = I / 128, gpg = a.down.group / 128;
    int2* ttab = reinterpret_cast<int2*>(smem + a.off_tt);
    for (int t = tid - 32; t < n_act * ts * ngc; t += kThreads - 32) {
      const int G = t % ngc, tile = t / ngc, i = tile / ts, m = tile - i * ts;
      ttab[t] = make_int2((i << 8) | m, G | ((G / gpg) << 16));
    }
  }
  __syncthreads();  // scales in shared memory; the code copies are still in flight
  T1_TRACE(5);

  // ---- 3. gate/up rows as their chunks land -----------------------------------------------
  for (int lr = warp; lr < nrows; lr += kWarps) {
    if (__any_sync(kFullMask, *abort_flag)) break;
    const int ci = (tb.r0 + lr) / kChunkRows - tb.r0 / kChunkRows;
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
  T1_TRACE(6);  // (stamp 7 marks the same point: h is written by the rows themselves)
  T1_TRACE(7);

  // ---- 4. grid barrier, stage h ----------------------------------------------------------------
  const bool passed = ac::grid_sync_epoch(a.bar, bar_seen, &grid_ok);
  if (!passed && tid == 0) fail();
  T1_TRACE(8);
  // Stage h as bf16 (hi, lo) operand words: word w = 4c + q (8 activations,
  // 32-code chunk c) of expert slot s goes to hq[s * I/8 + q * I/32 + c] (high
  // parts) and the same index past lo_off (low parts) in the w4_pack_x pair
  // order; one correction 136 * sum(hi + lo) per 128-code group.
  const int w8 = I / 8, w32 = I / 32, ngc = I / 128, ts = (nrc + 15) / 16;
  const int lo_off = k * w8 + 4;  // the low plane sits 64 bytes off the high plane's bank alignment
  uint4* hq = reinterpret_cast<uint4*>(smem + a.off_act);
  float* corr_c = reinterpret_cast<float*>(smem + a.off_cc);  // [slot][group]
  {
    const float4* h4 = reinterpret_cast<const float4*>(a.hbuf);
    const int nw = n_act * w8;
    for (int base = 0; base < nw; base += kThreads) {
      const int wd = base + tid;
      const bool ok = wd < nw;
      float cs = 0.0f;
      if (ok) {
        const int sl = wd / w8, wi = wd - sl * w8;
        const int dst = sl * w8 + (wi & 3) * w32 + (wi >> 2);
        const float4 v0 = __ldcg(h4 + 2 * wd), v1 = __ldcg(h4 + 2 * wd + 1);
        const float hv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        uint16_t hi[8], lo[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) split_bf16(hv[e], hi[e], lo[e]);
        hq[dst] = make_uint4(pack_bf16x2(hi[0], hi[4]), pack_bf16x2(hi[1], hi[5]), pack_bf16x2(hi[2], hi[6]),
                             pack_bf16x2(hi[3], hi[7]));
        hq[lo_off + dst] = make_uint4(pack_bf16x2(lo[0], lo[4]), pack_bf16x2(lo[1], lo[5]),
                                      pack_bf16x2(lo[2], lo[6]), pack_bf16x2(lo[3], lo[7]));
        float sv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) sv[e] = bf16_to_f32(hi[e]) + bf16_to_f32(lo[e]);  // exact
        cs = ((sv[0] + sv[1]) + (sv[2] + sv[3])) + ((sv[4] + sv[5]) + (sv[6] + sv[7]));
      }
      // a 128-code group is 16 consecutive words: aligned 16-lane segments
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) cs += __shfl_xor_sync(kFullMask, cs, o);
      if (ok && (wd & 15) == 0) corr_c[wd >> 4] = 136.0f * cs;
    }
  }
  __syncthreads();
  T1_TRACE(9);

  // ---- 5. down tiles + ordered combine ---------------------------------------------------------------
  const bool c_ok = !issued || nrc == 0 || n_act == 0 || ac::mbar_wait_bounded(ac::smem_u32(&bars[1]), 0u);
  if (!c_ok) fail();
  __syncthreads();
  T1_TRACE(10);
  const bool ok5 = !*abort_flag;  // CTA-uniform after the barrier above
  // Tile = 16 of the CTA's output rows of one expert slot (rows past nrc repeat
  // the last one).  B's columns 0-3 carry the high bf16 parts of h, columns 4-7
  // the low parts, so lanes t and t ^ 2 hold the two halves of each row sum.
  // Task (tile, group): one warp, 8 mma; lanes t == 0 store s * (sum - corr).
  float* part_c = reinterpret_cast<float*>(smem + a.off_ys);  // [slot][tile][16 rows][group]
  const int g4 = lane >> 2, t4 = lane & 3;
  if (ok5) {
    const int ntask = n_act * ts * ngc;
    const int2* ttab = reinterpret_cast<const int2*>(smem + a.off_tt);
    for (int task = warp; task < ntask; task += kWarps) {
      const int2 te = ttab[task];
      const int i = te.x >> 8, m = te.x & 255, G = te.y & 0xffff, si = te.y >> 16;
      const int ch = G * 4 + t4;
      const uint4* hp = hq + (g4 < 4 ? 0 : lo_off) + i * w8 + ch;
      const uint4 src[4] = {hp[0], hp[w32], hp[2 * w32], hp[3 * w32]};
      const int rl = min(m * 16 + g4, nrc - 1), rh = min(m * 16 + 8 + g4, nrc - 1);
      const unsigned char* wb = reg_c + i * per_c + 16 * ch;
      const uint4 wl = *reinterpret_cast<const uint4*>(wb + static_cast<size_t>(rl) * rb_c);
      const uint4 wh = *reinterpret_cast<const uint4*>(wb + static_cast<size_t>(rh) * rb_c);
      float d[4];
      w4_group_mma(wl, wh, src, d);
      const float sl = d[0] + __shfl_xor_sync(kFullMask, d[0], 2);
      const float sh = d[2] + __shfl_xor_sync(kFullMask, d[2], 2);
      if (t4 == 0) {
        const float cg = corr_c[i * ngc + G];
        float* p = part_c + (i * ts + m) * 16 * ngc + G;  // [slot][tile][row][group]
        p[g4 * ngc] = bf16_to_f32(sc_c[(i * nrc + rl) * ssc + si]) * (sl - cg);
        p[(8 + g4) * ngc] = bf16_to_f32(sc_c[(i * nrc + rh) * ssc + si]) * (sh - cg);
      }
    }
  }
  __syncthreads();
  T1_TRACE(11);
  // one warp per output row: lane i forms w_i * y_i, the products are added in
  // slot (ascending expert) order in fp32
  if (ok5) {
    for (int rs = warp; rs < nrc; rs += kWarps) {
      const int m = rs >> 4, r = rs & 15;
      float yw = 0.0f;
      if (lane < n_act) {
        const float* p = part_c + ((lane * ts + m) * 16 + r) * ngc;
        float yv = 0.0f;
#pragma unroll 4
        for (int G = 0; G < ngc; ++G) yv += p[G];
        yw = __fmul_rn(yv, tb.act_w[lane]);
      }
      float acc = 0.0f;
#pragma unroll 8
      for (int i = 0; i < n_act; ++i) acc = __fadd_rn(acc, __shfl_sync(kFullMask, yw, i));
      if (lane == 0) a.out[n0 + rs] = f32_to_bf16(acc);
    }
  }
  // copies issued but never waited on (abort path) must land before exit
  if (issued && !ok5 && tid == 0) {
    for (int i = 0; i < nchunks; ++i) ac::mbar_wait_bounded(ac::smem_u32(&bars[2 + i]), 0u);
    if (nrc > 0 && n_act > 0) ac::mbar_wait_bounded(ac::smem_u32(&bars[1]), 0u);
  }
  T1_TRACE(12);
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
  const size_t ngc = I / 128, ts = (nrc + 15) / 16;
  pl.a.off_act = take(static_cast<size_t>(k) * I * 4 + 64, 16);  // h as bf16 (hi, lo) operand words
  pl.a.off_cc = take(static_cast<size_t>(k) * ngc * 4, 16);
  pl.a.off_tt = take(static_cast<size_t>(k) * ts * ngc * 8, 16);
  pl.a.off_ys = take(static_cast<size_t>(k) * ts * ngc * 16 * 4, 16);
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
  if (p.down.group % 128) return false;  // one scale per 128-code tensor-core group
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
  if (!ensure_dynamic_smem(kern, pl.smem, t1::kThreads)) return -1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.num_sms);
  cfg.blockDim = dim3(t1::kThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  void* args[] = {&a};
  return cudaLaunchKernelExC(&cfg, kern, args) == cudaSuccess ? 1 : -2;
}

}  // namespace moe
