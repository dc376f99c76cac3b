// expert_matvec.cu — dequant-fused grouped matvec for the routed experts.
//
// Replaces, per routed (token, expert) pair, the reference's
//   gate = cpu_w4a32_matvec(x, W_gate); up = cpu_w4a32_matvec(x, W_up)
//   h = silu(gate) * up;                 down = cpu_w4a32_matvec(h, W_down)
// (nano_ktrans/kernels/cpu_moe.py:419-450 over quantized_ops.py:86-124) and
// the weighted index_add_ combine (cpu_moe.py:528-538).
//
// Work decomposition.  A tile is (active expert, block of output rows).  Each
// warp owns 32/LPR rows; LPR lanes share one row and walk its 16-byte chunks
// (lane sl takes chunks sl, sl+LPR, ...), so a warp's loads of one row are
// contiguous 16-byte vectors.  The activations of up to `tch` tokens of the
// expert are staged once per tile in shared memory as fp32 (pre-scaled for
// the W4 unpack), interleaved so the LPR lanes of a row read consecutive
// 16-byte words (bank-conflict free).  Per chunk a lane accumulates
// (q - z) * x exactly-multiplied in fp32 (common.cuh), scales the chunk sum
// by its group scale, and the LPR partial sums are combined with shuffles.
//
// Tiles are scheduled by a grid-stride loop over n_active * tiles_per_expert
// (n_active is read on the device, so launch shapes never depend on routing).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace moe {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxTch = 8;

struct MatvecArgs {
  const uint16_t* x;  // gate/up: bf16 [T][K]
  const float* h;     // down: fp32 [rows][K], rows indexed like the output
  const int32_t* sorted_pair;
  const int32_t* offsets;
  const int32_t* active;
  const int32_t* n_active;
  int top_k;
  int identity_tokens;
  QuantProj p0, p1;
  float* out;  // [rows][N]
  int tch;
};

template <int BITS, int LPR, bool GATEUP>
__global__ void __launch_bounds__(kThreads) expert_matvec_kernel(MatvecArgs a) {
  extern __shared__ float4 xs4[];
  constexpr int kCodes = ChunkTraits<BITS>::kCodes;
  constexpr int kQ = ChunkTraits<BITS>::kQ;
  constexpr int kRowsPerWarp = 32 / LPR;
  constexpr int kRowsPerTile = kWarps * kRowsPerWarp;

  const int K = a.p0.k, N = a.p0.n;
  const int K4 = K / 4;
  const int nchunks = K / kCodes;
  const int chunk_iters = (nchunks + LPR - 1) / LPR;
  // per-token stride of the interleaved activation layout, padded to whole
  // LPR-chunk groups so the last partial group stays inside its token's slot
  const int K4p = chunk_iters * LPR * kQ;
  // W4 gate/up operands: [tch][Kw] uint4 words, then [tch][CW] chunk corrections
  const int Kw = chunk_iters * LPR * 4, CW = chunk_iters * LPR;
  uint4* xq = reinterpret_cast<uint4*>(xs4);
  float* cq = reinterpret_cast<float*>(xq + a.tch * Kw);
  const size_t row_bytes = static_cast<size_t>(K) * BITS / 8;
  const int G = a.p0.sstride;
  const int tiles_per_expert = (N + kRowsPerTile - 1) / kRowsPerTile;
  const int n_act = a.identity_tokens > 0 ? 1 : *a.n_active;
  const int total = n_act * tiles_per_expert;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sl = lane % LPR;

  for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
    const int ai = tile / tiles_per_expert, rb = tile - ai * tiles_per_expert;
    int e, s0, s1;
    if (a.identity_tokens > 0) {
      e = 0;
      s0 = 0;
      s1 = a.identity_tokens;
    } else {
      e = a.active[ai];
      s0 = a.offsets[e];
      s1 = a.offsets[e + 1];
    }
    const int row = rb * kRowsPerTile + warp * kRowsPerWarp + lane / LPR;
    const bool row_ok = row < N;
    const size_t rix = static_cast<size_t>(e) * N + (row_ok ? row : 0);
    const uint8_t* w0 = a.p0.q + rix * row_bytes;
    const uint16_t* sc0 = a.p0.s + rix * G;
    const uint8_t* w1 = nullptr;
    const uint16_t* sc1 = nullptr;
    if constexpr (GATEUP) {
      w1 = a.p1.q + rix * row_bytes;
      sc1 = a.p1.s + rix * G;
    }

    for (int tb = s0; tb < s1; tb += a.tch) {
      const int nt = min(a.tch, s1 - tb);
      __syncthreads();  // previous pass finished reading xs4
      if constexpr (GATEUP && BITS == 4) {
        // bf16 operand words + one correction per chunk (common.cuh, W4 with
        // bf16 operands); the 4 words of a chunk sit in 4 adjacent lanes
        const int K8 = K / 8, nw = nt * K8;
        for (int base = 0; base < nw; base += kThreads) {
          const int idx = base + threadIdx.x;
          const bool ok = idx < nw;
          const int tt = ok ? idx / K8 : 0, wi = ok ? idx - tt * K8 : 0;
          const int c = wi >> 2, q = wi & 3;
          float corr = 0.0f;
          if (ok) {
            const int s = tb + tt;
            const int tok = a.identity_tokens > 0 ? s : a.sorted_pair[s] / a.top_k;
            const uint4 raw = *reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(tok) * K + 8 * wi);
            xq[tt * Kw + ((c / LPR) * 4 + q) * LPR + (c % LPR)] = w4_pack_x(raw, corr);
          }
          corr += __shfl_xor_sync(kFullMask, corr, 1);
          corr += __shfl_xor_sync(kFullMask, corr, 2);
          if (ok && q == 0) cq[tt * CW + c] = corr;
        }
      } else {
        for (int idx = threadIdx.x; idx < nt * K4; idx += kThreads) {
          const int tt = idx / K4, f = idx - tt * K4;
          const int c = f / kQ, q = f - c * kQ;
          float4 v;
          if constexpr (GATEUP) {
            const int s = tb + tt;
            const int tok = a.identity_tokens > 0 ? s : a.sorted_pair[s] / a.top_k;
            const uint2 raw = *reinterpret_cast<const uint2*>(a.x + static_cast<size_t>(tok) * K + 4 * f);
            v = make_float4(__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u),
                            __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xffff0000u));
          } else {
            v = *reinterpret_cast<const float4*>(a.h + static_cast<size_t>(tb + tt) * K + 4 * f);
          }
          const int k0 = 4 * f;
          v.x *= act_prescale<BITS>(k0);
          v.y *= act_prescale<BITS>(k0 + 1);
          v.z *= act_prescale<BITS>(k0 + 2);
          v.w *= act_prescale<BITS>(k0 + 3);
          xs4[tt * K4p + ((c / LPR) * kQ + q) * LPR + (c % LPR)] = v;
        }
      }
      __syncthreads();

      float acc0[kMaxTch], acc1[kMaxTch];
#pragma unroll
      for (int t = 0; t < kMaxTch; ++t) acc0[t] = acc1[t] = 0.0f;
      if (row_ok) {
        for (int it = 0; it < chunk_iters; ++it) {
          const int c = it * LPR + sl;
          if (c < nchunks) {
            const uint4 wv0 = ld_stream16(w0 + static_cast<size_t>(c) * 16);
            const float s0v = bf16_to_f32(__ldg(sc0 + (c * kCodes) / a.p0.group));
            uint4 wv1 = make_uint4(0, 0, 0, 0);
            float s1v = 0.0f;
            if constexpr (GATEUP) {
              wv1 = ld_stream16(w1 + static_cast<size_t>(c) * 16);
              s1v = bf16_to_f32(__ldg(sc1 + (c * kCodes) / a.p1.group));
            }
            if constexpr (GATEUP && BITS == 4) {
              const uint4* xb = xq + (it * 4) * LPR + sl;
#pragma unroll
              for (int t = 0; t < kMaxTch; ++t) {
                if (t < nt) {
                  const float cr = cq[t * CW + c];
                  acc0[t] = fmaf(s0v, w4_chunk_dot_bf16(wv0, xb + t * Kw, LPR, cr), acc0[t]);
                  acc1[t] = fmaf(s1v, w4_chunk_dot_bf16(wv1, xb + t * Kw, LPR, cr), acc1[t]);
                }
              }
            } else {
              const float4* xb = xs4 + (it * kQ) * LPR + sl;
#pragma unroll
              for (int t = 0; t < kMaxTch; ++t) {
                if (t < nt) {
                  const float4* xt = xb + t * K4p;
                  acc0[t] = fmaf(s0v, chunk_dot<BITS>(wv0, xt, LPR), acc0[t]);
                  if constexpr (GATEUP) acc1[t] = fmaf(s1v, chunk_dot<BITS>(wv1, xt, LPR), acc1[t]);
                }
              }
            }
          }
        }
      }
#pragma unroll
      for (int t = 0; t < kMaxTch; ++t) {
#pragma unroll
        for (int off = LPR / 2; off > 0; off >>= 1) {
          acc0[t] += __shfl_xor_sync(kFullMask, acc0[t], off);
          if constexpr (GATEUP) acc1[t] += __shfl_xor_sync(kFullMask, acc1[t], off);
        }
      }
      if (row_ok && sl == 0) {
#pragma unroll
        for (int t = 0; t < kMaxTch; ++t) {
          if (t < nt) {
            float r = acc0[t];
            if constexpr (GATEUP) r = silu_f32(acc0[t]) * acc1[t];
            a.out[static_cast<size_t>(tb + t) * N + row] = r;
          }
        }
      }
    }
  }
}

constexpr int kSmemLimit = 227 * 1024;

// Shared-memory bytes per staged token: K fp32 activations, padded to whole
// groups of LPR chunks.
template <int BITS, int LPR>
static size_t token_smem_bytes(int K) {
  constexpr int kCodes = ChunkTraits<BITS>::kCodes;
  const int nchunks = K / kCodes;
  const int chunk_iters = (nchunks + LPR - 1) / LPR;
  return static_cast<size_t>(chunk_iters) * LPR * kCodes * sizeof(float);
}

template <int BITS, int LPR>
static int pick_tch(int K) {
  const size_t per = token_smem_bytes<BITS, LPR>(K);
  return static_cast<int>(std::max<size_t>(1, std::min<size_t>(kMaxTch, kSmemLimit / per)));
}

template <int BITS, int LPR, bool GATEUP>
static int launch_mv(MatvecArgs a, int max_active, int num_sms, cudaStream_t st) {
  constexpr int kRowsPerTile = kWarps * (32 / LPR);
  const int K = a.p0.k;
  a.tch = std::max(1, std::min(pick_tch<BITS, LPR>(K), a.tch));  // caller set a.tch = tokens per expert bound
  const size_t smem = static_cast<size_t>(a.tch) * token_smem_bytes<BITS, LPR>(K);
  static int configured_mask = 0;  // per device bit
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured_mask & (1 << dev))) {
    cudaFuncSetAttribute(expert_matvec_kernel<BITS, LPR, GATEUP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmemLimit);
    configured_mask |= 1 << dev;
  }
  const int tiles = max_active * ((a.p0.n + kRowsPerTile - 1) / kRowsPerTile);
  const int grid = std::max(1, std::min(tiles, num_sms * 4));
  expert_matvec_kernel<BITS, LPR, GATEUP><<<grid, kThreads, smem, st>>>(a);
  return 1;
}

template <bool GATEUP>
static int dispatch(int bits, MatvecArgs& a, int max_active, int num_sms, cudaStream_t st) {
  const int chunks = a.p0.k * bits / 128;
  const bool wide = chunks >= 64;
  if (bits == 4) {
    return wide ? launch_mv<4, 32, GATEUP>(a, max_active, num_sms, st)
                : launch_mv<4, 8, GATEUP>(a, max_active, num_sms, st);
  }
  return wide ? launch_mv<8, 32, GATEUP>(a, max_active, num_sms, st)
              : launch_mv<8, 8, GATEUP>(a, max_active, num_sms, st);
}

int launch_gateup(int bits, const uint16_t* x, const RouteTables& rt, int top_k, int max_active, int num_tokens,
                  int identity_tokens,
                  const QuantProj& gate, const QuantProj& up, float* h, int num_sms, cudaStream_t st) {
  MatvecArgs a{};
  a.x = x;
  a.sorted_pair = rt.sorted_pair;
  a.offsets = rt.offsets;
  a.active = rt.active;
  a.n_active = rt.n_active;
  a.top_k = top_k;
  a.identity_tokens = identity_tokens;
  a.p0 = gate;
  a.p1 = up;
  a.out = h;
  a.tch = num_tokens;
  return dispatch<true>(bits, a, identity_tokens > 0 ? 1 : max_active, num_sms, st);
}

int launch_down(int bits, const float* h, const RouteTables& rt, int max_active, int num_tokens, int identity_tokens,
                const QuantProj& down, float* y, int num_sms, cudaStream_t st) {
  MatvecArgs a{};
  a.h = h;
  a.sorted_pair = rt.sorted_pair;
  a.offsets = rt.offsets;
  a.active = rt.active;
  a.n_active = rt.n_active;
  a.top_k = 1;
  a.identity_tokens = identity_tokens;
  a.p0 = down;
  a.out = y;
  a.tch = num_tokens;
  return dispatch<false>(bits, a, identity_tokens > 0 ? 1 : max_active, num_sms, st);
}

// ---------------------------------------------------------------------------
// Combine: out[t] = bf16( sum over the token's slots, in ascending expert
// order, of fp32(w) * y  (+ sg[t] * ys[t]) ).  The product and the sum are
// rounded separately, as `index_add_(out, tok, y * w)` does
// (cpu_moe.py:528-536); experts are visited in ascending order as in the
// reference's expert loop (:515).
// ---------------------------------------------------------------------------

constexpr int kMaxTopK = 16;

__global__ void __launch_bounds__(256) combine_kernel(const int64_t* __restrict__ ids,
                                                      const uint16_t* __restrict__ weights,
                                                      const int32_t* __restrict__ pair_pos, int T, int top_k, int H,
                                                      const float* __restrict__ y, const float* __restrict__ sg,
                                                      const float* __restrict__ ys, uint16_t* __restrict__ out) {
  const int cols4 = H / 4;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= T * cols4) return;
  const int t = idx / cols4, c4 = idx - t * cols4;
  int ex[kMaxTopK], ps[kMaxTopK];
  float wt[kMaxTopK];
  int n = 0;
  for (int j = 0; j < top_k; ++j) {
    const int p = t * top_k + j;
    const int pos = pair_pos[p];
    if (pos < 0) continue;
    const int e = static_cast<int>(ids[p]);
    const float w = bf16_to_f32(weights[p]);
    int i = n++;
    while (i > 0 && ex[i - 1] > e) {
      ex[i] = ex[i - 1];
      ps[i] = ps[i - 1];
      wt[i] = wt[i - 1];
      --i;
    }
    ex[i] = e;
    ps[i] = pos;
    wt[i] = w;
  }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i = 0; i < n; ++i) {
    const float4 v = reinterpret_cast<const float4*>(y + static_cast<size_t>(ps[i]) * H)[c4];
    acc.x = __fadd_rn(acc.x, __fmul_rn(v.x, wt[i]));
    acc.y = __fadd_rn(acc.y, __fmul_rn(v.y, wt[i]));
    acc.z = __fadd_rn(acc.z, __fmul_rn(v.z, wt[i]));
    acc.w = __fadd_rn(acc.w, __fmul_rn(v.w, wt[i]));
  }
  if (ys != nullptr) {
    const float g = sg[t];
    const float4 v = reinterpret_cast<const float4*>(ys + static_cast<size_t>(t) * H)[c4];
    acc.x = __fadd_rn(acc.x, __fmul_rn(g, v.x));
    acc.y = __fadd_rn(acc.y, __fmul_rn(g, v.y));
    acc.z = __fadd_rn(acc.z, __fmul_rn(g, v.z));
    acc.w = __fadd_rn(acc.w, __fmul_rn(g, v.w));
  }
  uint2 o;
  o.x = static_cast<uint32_t>(f32_to_bf16(acc.x)) | (static_cast<uint32_t>(f32_to_bf16(acc.y)) << 16);
  o.y = static_cast<uint32_t>(f32_to_bf16(acc.z)) | (static_cast<uint32_t>(f32_to_bf16(acc.w)) << 16);
  reinterpret_cast<uint2*>(out + static_cast<size_t>(t) * H)[c4] = o;
}

void launch_combine(const int64_t* ids, const uint16_t* weights, const RouteTables& rt, int T, int top_k, int H,
                    const float* y, const float* shared_gate, const float* shared_y, uint16_t* out, cudaStream_t st) {
  const int n = T * (H / 4);
  if (n <= 0) return;
  combine_kernel<<<(n + 255) / 256, 256, 0, st>>>(ids, weights, rt.pair_pos, T, top_k, H, y, shared_gate, shared_y,
                                                  out);
}

// sg[t] = sigmoid(sum_k x[t][k] * g[k]) in fp32 (models/mixtral.py:216-217
// `torch.sigmoid(self.shared_expert_gate(mlp_input))`).
__global__ void __launch_bounds__(256) shared_gate_kernel(const uint16_t* __restrict__ x,
                                                          const uint16_t* __restrict__ g, int T, int H,
                                                          float* __restrict__ sg) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float acc = 0.0f;
  for (int k = lane; k < H; k += 32) acc = fmaf(bf16_to_f32(x[static_cast<size_t>(t) * H + k]), bf16_to_f32(g[k]), acc);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(kFullMask, acc, off);
  if (lane == 0) sg[t] = sigmoid_f32(acc);
}

void launch_shared_gate(const uint16_t* x, const uint16_t* g, int T, int H, float* sg, cudaStream_t st) {
  if (T <= 0) return;
  shared_gate_kernel<<<(T + 7) / 8, 256, 0, st>>>(x, g, T, H, sg);
}

// ---------------------------------------------------------------------------
// Dequantization dump: the unpack of common.cuh, rescaled to (q - z) * s.
// ---------------------------------------------------------------------------

template <int BITS>
__global__ void dequant_rows_kernel(QuantProj p, int expert, int row0, int nrows, float* __restrict__ out) {
  constexpr int kVpw = 32 / BITS;
  const int words = p.k / kVpw;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= nrows * words) return;
  const int r = idx / words, wi = idx - r * words;
  const size_t rix = static_cast<size_t>(expert) * p.n + row0 + r;
  const uint32_t w = reinterpret_cast<const uint32_t*>(p.q + rix * (static_cast<size_t>(p.k) * BITS / 8))[wi];
  const float s = bf16_to_f32(p.s[rix * p.sstride + (wi * kVpw) / p.group]);
  float* o = out + static_cast<size_t>(r) * p.k + wi * kVpw;
  if constexpr (BITS == 4) {
    float2 d[4];
    w4_unpack(w, d[0], d[1], d[2], d[3]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = (j & 1) ? d[j >> 1].y : d[j >> 1].x;
      o[j] = (v * w4_prescale(j)) * s;
    }
  } else {
    float2 d[2];
    w8_unpack(w, d[0], d[1]);
    o[0] = d[0].x * s;
    o[1] = d[0].y * s;
    o[2] = d[1].x * s;
    o[3] = d[1].y * s;
  }
}

void launch_dequant_rows(int bits, const QuantProj& p, int expert, int row0, int nrows, float* out, cudaStream_t st) {
  const int words = p.k * bits / 32;
  const int n = nrows * words;
  if (n <= 0) return;
  if (bits == 4)
    dequant_rows_kernel<4><<<(n + 255) / 256, 256, 0, st>>>(p, expert, row0, nrows, out);
  else
    dequant_rows_kernel<8><<<(n + 255) / 256, 256, 0, st>>>(p, expert, row0, nrows, out);
}

}  // namespace moe
