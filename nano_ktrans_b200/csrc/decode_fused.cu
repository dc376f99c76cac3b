// decode_fused.cu — the whole routed-expert step in one launch, for decode-
// sized batches (T * top_k * inter small enough that every pair's SiLU*up
// intermediate fits in shared memory).
//
// Replaces, for small T, the chain route -> permute -> gate/up -> down ->
// combine (nano_ktrans/layers/hybrid_moe.py:3321-3329 routing,
// nano_ktrans/kernels/cpu_moe.py:491-539 expert loop and index_add_
// combine, quantized_ops.py:86-124 grouped matvec arithmetic).
//
// One CTA per SM, launched cooperatively (all CTAs co-resident):
//  1. Every CTA routes all T tokens itself (route_warp.cuh) and builds the
//     expert-sorted pair table in shared memory — no launch, no barrier.
//  2. Phase B (gate/up): the active experts' gate/up rows form one flat row
//     space split evenly over the CTAs.  A CTA walks its range in stages of up
//     to 16 rows of one expert: one thread issues TMA bulk copies
//     (cp.async.bulk, global -> shared, completion on an mbarrier) of the gate
//     codes, up codes and both scale rows into a 3-slot ring; warp w computes
//     row w: 16-byte shared loads, exact unpack (common.cuh), warp-shuffle
//     reduction, SiLU(gate)*up written to global h (fp32).
//  3. One grid barrier (bounded spin).  Phase-C weight stages are already in
//     flight: their copies are issued as ring slots free up, before the
//     barrier.
//  4. Phase C (down + combine): CTA c owns output rows [c*H/G, (c+1)*H/G).
//     h of every pair is staged in shared memory; for each active expert in
//     ascending order the CTA multiplies its rows of W_down with the expert's
//     tokens' h and adds w * y into an fp32 accumulator per (token, row) —
//     the reference's combine order — then writes bf16 once.
// Every wait is bounded: on expiry the kernel records kStatusTimeout in the
// status word, stops computing, drains its outstanding copies (bounded) and
// still arrives at the grid barrier so no other CTA waits on it.
#include <cuda/atomic>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "route_warp.cuh"

namespace moe {

constexpr int kFThreads = 512;
constexpr int kFWarps = kFThreads / 32;
constexpr int kFStages = 3;
constexpr int kFSlotBytes = 34816;   // 16 rows x 2 projections x (1024 + 32) bytes
constexpr int kFMaxStages = 96;      // stage descriptors per CTA
constexpr int kFRowsC = 64;          // phase-C rows per CTA (16 warps x 4 rows)
constexpr int kFMaxTok = 4;          // tokens per launch
constexpr uint32_t kSpinLimit = 1u << 22;

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
  unsigned* bar;
  int* status;
  int rows_b;  // phase-B rows per stage
  int exp_c;   // phase-C experts per stage
  // shared-memory carve-up (bytes from the start of dynamic smem)
  int off_bar, off_tab, off_stage, off_act, off_acc, act_bytes;
};

struct StageDesc {
  int kind;  // 0 = gate/up rows, 1 = down rows of consecutive experts
  int n;     // rows (kind 0) or experts (kind 1)
  int a;     // index into the active-expert list
  int row0;  // first row
};

// --------------------------------------------------------------------------
// TMA / mbarrier primitives
// --------------------------------------------------------------------------

MOE_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

MOE_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

MOE_DEV void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

MOE_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

MOE_DEV bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

MOE_DEV void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// Grid-wide barrier for a cooperative launch: arrival counter + generation.
// Returns false if the wait hit its iteration limit.
MOE_DEV bool grid_sync_bounded(unsigned* bar) {
  __threadfence();
  __syncthreads();
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    cuda::atomic_ref<unsigned, cuda::thread_scope_device> count(bar[0]), gen(bar[1]);
    const unsigned g = gen.load(cuda::memory_order_relaxed);
    const unsigned prev = count.fetch_add(1u, cuda::memory_order_acq_rel);
    int ok = 1;
    if (prev == gridDim.x - 1) {
      count.store(0u, cuda::memory_order_relaxed);
      gen.fetch_add(1u, cuda::memory_order_release);
    } else {
      uint32_t i = 0;
      while (gen.load(cuda::memory_order_acquire) == g) {
        if (++i > kSpinLimit) {
          ok = 0;
          break;
        }
        __nanosleep(32);
      }
    }
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

// --------------------------------------------------------------------------

template <int BITS>
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
  int* cnt = reinterpret_cast<int*>(smem + a.off_tab);  // [E]
  int* off = cnt + E;                                   // [E+1]
  int* act = off + E + 1;                               // [E]
  int* fill = act + E;                                  // [E]
  int* misc = fill + E;                                 // [4]: n_act, n_stages, first_c, abort
  int* pair_e = misc + 4;                               // [P]
  float* pair_w = reinterpret_cast<float*>(pair_e + P); // [P]
  int* stok = reinterpret_cast<int*>(pair_w + P);       // [P] token of sorted pair
  float* sw = reinterpret_cast<float*>(stok + P);       // [P] weight of sorted pair
  StageDesc* stages = reinterpret_cast<StageDesc*>(smem + a.off_stage);
  float4* act4 = reinterpret_cast<float4*>(smem + a.off_act);
  float* out_acc = reinterpret_cast<float*>(smem + a.off_acc);  // [T][kFRowsC]

  // ---- 0. barriers, accumulators -----------------------------------------
  if (tid == 0) {
    for (int s = 0; s < kFStages; ++s) mbar_init(smem_u32(&bars[s]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    misc[3] = 0;
  }
  for (int i = tid; i < T * kFRowsC; i += kFThreads) out_acc[i] = 0.0f;
  for (int e = tid; e < E; e += kFThreads) {
    cnt[e] = 0;
    fill[e] = 0;
  }

  // ---- 1. routing (every CTA, redundantly) ---------------------------------
  for (int t = warp; t < T; t += kFWarps) {
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
      with_epl(E, [&](auto c) {
        route_token_warp<decltype(c)::value>(a.logits + static_cast<size_t>(t) * E, E, k, a.use_softmax != 0,
                                             a.renorm != 0, id, w);
      });
      if (cta == 0 && lane < k) {
        a.ids_out[t * k + lane] = id;
        a.w_out[t * k + lane] = f32_to_bf16(w);
      }
    }
    if (lane < k) {
      const bool inc = id >= 0 && (a.mask == nullptr || a.mask[id] != 0);
      pair_e[t * k + lane] = inc ? id : -1;
      pair_w[t * k + lane] = w;
    }
  }
  __syncthreads();
  for (int p = tid; p < P; p += kFThreads)
    if (pair_e[p] >= 0) atomicAdd(&cnt[pair_e[p]], 1);
  __syncthreads();
  if (warp == 0) {  // exclusive scan of counts + ascending active list
    const int per = (E + 31) / 32, e0 = lane * per, e1 = min(E, e0 + per);
    int sum = 0, nz = 0;
    for (int e = e0; e < e1; ++e) {
      sum += cnt[e];
      nz += cnt[e] > 0;
    }
    int isum = sum, inz = nz;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int a1 = __shfl_up_sync(kFullMask, isum, o), a2 = __shfl_up_sync(kFullMask, inz, o);
      if (lane >= o) {
        isum += a1;
        inz += a2;
      }
    }
    int run = isum - sum, ra = inz - nz;
    for (int e = e0; e < e1; ++e) {
      off[e] = run;
      run += cnt[e];
      if (cnt[e] > 0) act[ra++] = e;
    }
    if (lane == 31) {
      off[E] = isum;
      misc[0] = inz;
    }
  }
  __syncthreads();
  for (int p = tid; p < P; p += kFThreads) {
    const int e = pair_e[p];
    if (e >= 0) {
      const int s = off[e] + atomicAdd(&fill[e], 1);
      stok[s] = p / k;
      sw[s] = pair_w[p];
    }
  }

  // ---- 2. stage list ------------------------------------------------------
  const int n_act = misc[0];
  const int n0 = static_cast<int>((static_cast<long long>(cta) * H) / G);
  const int nrc = static_cast<int>((static_cast<long long>(cta + 1) * H) / G) - n0;
  if (tid == 0) {
    int ns = 0;
    const long long total = static_cast<long long>(n_act) * I;
    long long r = total * cta / G;
    const long long r1 = total * (cta + 1) / G;
    while (r < r1 && ns < kFMaxStages) {
      const int ai = static_cast<int>(r / I), row = static_cast<int>(r - static_cast<long long>(ai) * I);
      const int n = static_cast<int>(min(static_cast<long long>(min(a.rows_b, I - row)), r1 - r));
      stages[ns++] = StageDesc{0, n, ai, row};
      r += n;
    }
    misc[2] = ns;
    for (int a0 = 0; nrc > 0 && a0 < n_act && ns < kFMaxStages; a0 += a.exp_c)
      stages[ns++] = StageDesc{1, min(a.exp_c, n_act - a0), a0, n0};
    misc[1] = ns;
    if (r < r1) atomicOr(a.status, kStatusTimeout);  // stage table overflow (cannot happen within limits)
  }
  __syncthreads();
  const int nst = misc[1], first_c = misc[2];

  const size_t rb_b = static_cast<size_t>(H) * BITS / 8, sb_b = static_cast<size_t>(a.gate.sstride) * 2;
  const size_t rb_c = static_cast<size_t>(I) * BITS / 8, sb_c = static_cast<size_t>(a.down.sstride) * 2;
  const size_t per_c = static_cast<size_t>(nrc) * (rb_c + sb_c);

  auto issue = [&](int j) {  // thread 0 only
    const StageDesc d = stages[j];
    const int slot = j % kFStages;
    const uint32_t dst = smem_u32(ring + static_cast<size_t>(slot) * kFSlotBytes);
    const uint32_t bar = smem_u32(&bars[slot]);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (d.kind == 0) {
      const int e = act[d.a];
      const size_t rix = static_cast<size_t>(e) * I + d.row0;
      const uint32_t cb = static_cast<uint32_t>(d.n * rb_b), sbt = static_cast<uint32_t>(d.n * sb_b);
      mbar_expect_tx(bar, 2 * cb + 2 * sbt);
      bulk_g2s(dst, a.gate.q + rix * rb_b, cb, bar);
      bulk_g2s(dst + cb, a.up.q + rix * rb_b, cb, bar);
      bulk_g2s(dst + 2 * cb, a.gate.s + rix * a.gate.sstride, sbt, bar);
      bulk_g2s(dst + 2 * cb + sbt, a.up.s + rix * a.up.sstride, sbt, bar);
    } else {
      mbar_expect_tx(bar, static_cast<uint32_t>(d.n * per_c));
      for (int i = 0; i < d.n; ++i) {
        const size_t rix = static_cast<size_t>(act[d.a + i]) * H + d.row0;
        const uint32_t o = dst + static_cast<uint32_t>(i * per_c);
        bulk_g2s(o, a.down.q + rix * rb_c, static_cast<uint32_t>(nrc * rb_c), bar);
        bulk_g2s(o + static_cast<uint32_t>(nrc * rb_c), a.down.s + rix * a.down.sstride,
                 static_cast<uint32_t>(nrc * sb_c), bar);
      }
    }
  };

  int issued = 0;   // thread 0: stages whose copies were issued
  int drained = 0;  // thread 0: stages whose full barrier it has passed
  if (tid == 0)
    for (; issued < min(kFStages, nst); ++issued) issue(issued);

  // ---- 3. stage loop --------------------------------------------------------
  const int nch_b = H / kCodes, it_b = (nch_b + 31) / 32, k4p_b = it_b * 32 * kQ;
  const int nch_c = I / kCodes, it_c = (nch_c + 7) / 8, k4p_c = it_c * 8 * kQ;
  const int H4 = H / 4, I4 = I / 4;
  int staged_e = -1;  // expert whose tokens' activations are staged (CTA-uniform)
  bool synced = false;

  for (int j = 0; j < nst; ++j) {
    const StageDesc d = stages[j];
    if (d.kind == 1 && !synced) {
      // phase B -> C: grid barrier, then stage every pair's h (pre-scaled)
      if (!grid_sync_bounded(a.bar) && tid == 0) {
        atomicOr(a.status, kStatusTimeout);
        misc[3] = 1;
      }
      synced = true;
      for (int idx = tid; idx < P * I4; idx += kFThreads) {
        const int s = idx / I4, f = idx - s * I4;
        if (s >= off[E]) continue;
        const int c = f / kQ, q = f - c * kQ;
        float4 v = __ldcg(reinterpret_cast<const float4*>(a.hbuf + static_cast<size_t>(s) * I) + f);
        v.x *= act_prescale<BITS>(4 * f);
        v.y *= act_prescale<BITS>(4 * f + 1);
        v.z *= act_prescale<BITS>(4 * f + 2);
        v.w *= act_prescale<BITS>(4 * f + 3);
        act4[s * k4p_c + ((c >> 3) * kQ + q) * 8 + (c & 7)] = v;
      }
      __syncthreads();
    }
    if (d.kind == 0) {
      const int e = act[d.a];
      if (e != staged_e && !(T == 1 && staged_e >= 0)) {  // stage the expert's tokens' x (pre-scaled)
        const int s0 = off[e], nt = off[e + 1] - s0;
        for (int idx = tid; idx < nt * H4; idx += kFThreads) {
          const int tt = idx / H4, f = idx - tt * H4;
          const int c = f / kQ, q = f - c * kQ;
          const uint2 raw =
              *reinterpret_cast<const uint2*>(a.x + static_cast<size_t>(stok[s0 + tt]) * H + 4 * f);
          float4 v = make_float4(__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u),
                                 __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xffff0000u));
          v.x *= act_prescale<BITS>(4 * f);
          v.y *= act_prescale<BITS>(4 * f + 1);
          v.z *= act_prescale<BITS>(4 * f + 2);
          v.w *= act_prescale<BITS>(4 * f + 3);
          act4[tt * k4p_b + ((c >> 5) * kQ + q) * 32 + (c & 31)] = v;
        }
        staged_e = e;
        __syncthreads();
      }
    }

    // wait for this stage's bytes
    const int slot = j % kFStages;
    if (!misc[3]) {
      if (mbar_wait_bounded(smem_u32(&bars[slot]), static_cast<uint32_t>((j / kFStages) & 1))) {
        if (tid == 0) drained = j + 1;
      } else {
        atomicOr(a.status, kStatusTimeout);
        misc[3] = 1;
      }
    }
    const unsigned char* sl = ring + static_cast<size_t>(slot) * kFSlotBytes;

    if (!misc[3] && d.kind == 0 && warp < d.n) {
      // ---- gate/up row `warp` of this stage, every token of the expert
      const int e = act[d.a];
      const int s0 = off[e], nt = off[e + 1] - s0;
      const unsigned char* wg = sl + warp * rb_b;
      const unsigned char* wu = sl + d.n * rb_b + warp * rb_b;
      const uint16_t* sg = reinterpret_cast<const uint16_t*>(sl + 2 * d.n * rb_b + warp * sb_b);
      const uint16_t* su = reinterpret_cast<const uint16_t*>(sl + 2 * d.n * rb_b + d.n * sb_b + warp * sb_b);
      float ag[kFMaxTok], au[kFMaxTok];
#pragma unroll
      for (int t = 0; t < kFMaxTok; ++t) ag[t] = au[t] = 0.0f;
      for (int it = 0; it < it_b; ++it) {
        const int c = it * 32 + lane;
        if (c < nch_b) {
          const uint4 vg = *reinterpret_cast<const uint4*>(wg + 16 * c);
          const uint4 vu = *reinterpret_cast<const uint4*>(wu + 16 * c);
          const float scg = bf16_to_f32(sg[(c * kCodes) / a.gate.group]);
          const float scu = bf16_to_f32(su[(c * kCodes) / a.up.group]);
          const float4* xb = act4 + (it * kQ) * 32 + lane;
#pragma unroll
          for (int t = 0; t < kFMaxTok; ++t) {
            if (t < nt) {
              ag[t] = fmaf(scg, chunk_dot<BITS>(vg, xb + t * k4p_b, 32), ag[t]);
              au[t] = fmaf(scu, chunk_dot<BITS>(vu, xb + t * k4p_b, 32), au[t]);
            }
          }
        }
      }
#pragma unroll
      for (int t = 0; t < kFMaxTok; ++t) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          ag[t] += __shfl_xor_sync(kFullMask, ag[t], o);
          au[t] += __shfl_xor_sync(kFullMask, au[t], o);
        }
      }
      if (lane == 0) {
#pragma unroll
        for (int t = 0; t < kFMaxTok; ++t)
          if (t < nt) a.hbuf[static_cast<size_t>(s0 + t) * I + d.row0 + warp] = silu_f32(ag[t]) * au[t];
      }
    } else if (!misc[3] && d.kind == 1) {
      // ---- down rows of consecutive experts, combined in ascending expert order
      const int rs = warp * 4 + (lane >> 3), sl8 = lane & 7;
      for (int i = 0; i < d.n; ++i) {
        const int e = act[d.a + i];
        const int s0 = off[e], nt = off[e + 1] - s0;
        const unsigned char* wd = sl + i * per_c + static_cast<size_t>(rs) * rb_c;
        const uint16_t* sd = reinterpret_cast<const uint16_t*>(sl + i * per_c + nrc * rb_c + rs * sb_c);
        float ay[kFMaxTok];
#pragma unroll
        for (int t = 0; t < kFMaxTok; ++t) ay[t] = 0.0f;
        if (rs < nrc) {
          for (int it = 0; it < it_c; ++it) {
            const int c = it * 8 + sl8;
            if (c < nch_c) {
              const uint4 v = *reinterpret_cast<const uint4*>(wd + 16 * c);
              const float sc = bf16_to_f32(sd[(c * kCodes) / a.down.group]);
              const float4* hb = act4 + (it * kQ) * 8 + sl8;
#pragma unroll
              for (int t = 0; t < kFMaxTok; ++t)
                if (t < nt) ay[t] = fmaf(sc, chunk_dot<BITS>(v, hb + (s0 + t) * k4p_c, 8), ay[t]);
            }
          }
        }
#pragma unroll
        for (int t = 0; t < kFMaxTok; ++t) {
#pragma unroll
          for (int o = 4; o > 0; o >>= 1) ay[t] += __shfl_xor_sync(kFullMask, ay[t], o);
        }
        if (rs < nrc && sl8 == 0) {
#pragma unroll
          for (int t = 0; t < kFMaxTok; ++t) {
            if (t < nt) {
              float* o = out_acc + stok[s0 + t] * kFRowsC + rs;
              *o = __fadd_rn(*o, __fmul_rn(ay[t], sw[s0 + t]));
            }
          }
        }
      }
    }
    __syncthreads();  // slot consumed by every warp
    if (tid == 0 && !misc[3] && issued < nst && issued == j + kFStages) issue(issued++);
  }
  if (!synced) {
    if (!grid_sync_bounded(a.bar) && tid == 0) atomicOr(a.status, kStatusTimeout);
  }
  // abort path: let copies that were issued but never waited on land before
  // the CTA's shared memory is released (bounded)
  if (tid == 0)
    for (int j = drained; j < issued; ++j) mbar_wait_bounded(smem_u32(&bars[j % kFStages]), (j / kFStages) & 1);
  __syncthreads();
  if (misc[3]) return;
  for (int idx = tid; idx < T * nrc; idx += kFThreads) {
    const int t = idx / nrc, r = idx - t * nrc;
    a.out[static_cast<size_t>(t) * H + n0 + r] = f32_to_bf16(out_acc[t * kFRowsC + r]);
  }
}

// --------------------------------------------------------------------------
// host side
// --------------------------------------------------------------------------

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool decode_fused_eligible(int bits, int T, int E, int top_k, const QuantProj& gate, const QuantProj& down,
                           int num_sms) {
  const int H = gate.k, I = gate.n;
  if (T < 1 || T > kFMaxTok || top_k > 32) return false;
  if (bits != 4 && bits != 8) return false;
  const size_t rb_b = static_cast<size_t>(H) * bits / 8, sb_b = static_cast<size_t>(gate.sstride) * 2;
  if (2 * (rb_b + sb_b) > static_cast<size_t>(kFSlotBytes)) return false;  // one gate/up row pair per stage
  const int rows_c = (H + num_sms - 1) / num_sms;
  if (rows_c > kFRowsC) return false;
  const size_t per_c = static_cast<size_t>(rows_c) * (static_cast<size_t>(I) * bits / 8 + down.sstride * 2);
  if (per_c > static_cast<size_t>(kFSlotBytes)) return false;
  const size_t h_bytes = static_cast<size_t>(T) * top_k * I * sizeof(float);
  return h_bytes <= 96 * 1024 && E <= 1024;
}

int launch_decode_fused(int bits, const DecodeFusedParams& p, cudaStream_t st) {
  const int H = p.gate.k, I = p.gate.n;
  const int P = p.T * p.top_k;
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
  a.status = p.status;
  const size_t rb_b = static_cast<size_t>(H) * bits / 8, sb_b = static_cast<size_t>(p.gate.sstride) * 2;
  a.rows_b = static_cast<int>(std::min<size_t>(kFWarps, kFSlotBytes / (2 * (rb_b + sb_b))));
  const int G = p.num_sms;
  const int rows_c = (H + G - 1) / G;
  const size_t per_c = static_cast<size_t>(rows_c) * (static_cast<size_t>(I) * bits / 8 + p.down.sstride * 2);
  a.exp_c = static_cast<int>(std::max<size_t>(1, kFSlotBytes / per_c));

  const int kQ = bits == 4 ? 8 : 4, kCodes = bits == 4 ? 32 : 16;
  const int it_b = (H / kCodes + 31) / 32, it_c = (I / kCodes + 7) / 8;
  const size_t xs_bytes = static_cast<size_t>(std::min(p.T, kFMaxTok)) * it_b * 32 * kQ * 16;
  const size_t hs_bytes = static_cast<size_t>(P) * it_c * 8 * kQ * 16;
  size_t off = static_cast<size_t>(kFStages) * kFSlotBytes;
  a.off_bar = static_cast<int>(off);
  off += kFStages * 8;
  a.off_tab = static_cast<int>(off);
  off += sizeof(int) * (4 * static_cast<size_t>(p.E) + 1 + 4 + 4 * static_cast<size_t>(P));
  off = align_up(off, 16);
  a.off_stage = static_cast<int>(off);
  off += sizeof(StageDesc) * kFMaxStages;
  off = align_up(off, 16);
  a.off_act = static_cast<int>(off);
  a.act_bytes = static_cast<int>(std::max(xs_bytes, hs_bytes));
  off += a.act_bytes;
  a.off_acc = static_cast<int>(off);
  off += sizeof(float) * static_cast<size_t>(p.T) * kFRowsC;
  const size_t smem = off;
  if (smem > 227 * 1024) return -1;

  void (*kern)(FusedArgs) = bits == 4 ? moe_decode_fused_kernel<4> : moe_decode_fused_kernel<8>;
  // opt in to exactly the dynamic shared memory this launch needs (the
  // kernel's static shared memory counts against the same per-block limit)
  static size_t configured[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  size_t& have = configured[bits == 4 ? 0 : 1][dev & 63];
  if (smem > have) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return -1;
    have = smem;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kFThreads, smem) != cudaSuccess || per_sm < 1)
    return -1;
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
  return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? 1 : -2;
}

}  // namespace moe
