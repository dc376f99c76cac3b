// kernels.h — host-side launchers for the routed-expert kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace moe {

// Routing tables produced by the permute kernel (all device memory).
struct RouteTables {
  int32_t* counts;       // [E]     pairs per expert (after the offload mask)
  int32_t* offsets;      // [E+1]   exclusive prefix of counts
  int32_t* active;       // [E]     experts with counts > 0, ascending
  int32_t* n_active;     // [1]
  int32_t* sorted_pair;  // [P]     pair index p = t*k + j, grouped by expert, p ascending
  int32_t* pair_pos;     // [P]     position of pair p in sorted_pair, -1 if excluded
  int32_t* status;       // [1]     error bits (kStatusBadExpertId)
};

// Expert-projection operand: stacked [E][N][K*bits/8] codes + [E][N][G] scales.
struct QuantProj {
  const uint8_t* q;
  const uint16_t* s;
  int n;           // output rows
  int k;           // input dim
  int group;       // group size along K (== k for per-channel)
  int sstride;     // bf16 elements per scale row: K/group rounded up to 8 (16 bytes)
};

void launch_route(const uint16_t* logits, int T, int E, int top_k, bool use_softmax, bool renorm,
                  int64_t* ids, uint16_t* weights, cudaStream_t st);

// logits[t][e] = bf16(sum_h x[t][h] * wr[e][h]), fp32 accumulation; x [T][H]
// and wr [E][H] bf16, 16-byte aligned, H a multiple of 32.
bool router_shape_ok(int E, int H, const void* x, const void* wr);
void launch_router_logits(const uint16_t* x, const uint16_t* wr, int T, int E, int H, uint16_t* logits,
                          cudaStream_t st);

// Stable counting sort of the T*top_k pairs by expert (route tables).  Ids
// outside [0, E) are excluded and flagged in the status word, except negative
// ids when skip_negative (pairs that belong to no local expert).
void launch_permute(const int64_t* ids, int T, int top_k, int E, const uint8_t* offload_mask,
                    const RouteTables& rt, cudaStream_t st, bool skip_negative = false);

// gate/up projection + SiLU(gate)*up for every (expert, token) pair:
// h[s][n] for sorted positions s.  When identity_tokens > 0 the routing
// tables are ignored and a single expert serves tokens 0..identity_tokens-1
// (the shared expert), h indexed by token.
int launch_gateup(int bits, const uint16_t* x, const RouteTables& rt, int top_k, int max_active, int num_tokens,
                  int identity_tokens, const QuantProj& gate, const QuantProj& up, float* h,
                  int num_sms, cudaStream_t st);

// down projection: y[s][n] = down_e(h[s]).
int launch_down(int bits, const float* h, const RouteTables& rt, int max_active, int num_tokens, int identity_tokens,
                const QuantProj& down, float* y, int num_sms, cudaStream_t st);

// Weight-streaming tensor-core projections (stream.cu) for batches that give
// each active expert a few tokens: same inputs and outputs as launch_gateup /
// launch_down over the routing tables.  W4 with group sizes that are multiples
// of 128; stream_eligible says whether this layer's shapes fit.  Launchers
// return 1 when launched, negative when not.
bool stream_eligible(int bits, const QuantProj& gate, const QuantProj& up, const QuantProj& down, int max_active);
int launch_stream_gateup(const uint16_t* x, const RouteTables& rt, int top_k, int max_active, const QuantProj& gate,
                         const QuantProj& up, float* h, int* status, unsigned long long* trace, int num_sms,
                         cudaStream_t st);
int launch_stream_down(const float* h, const RouteTables& rt, int max_active, const QuantProj& down, float* y,
                       int* status, int num_sms, cudaStream_t st);

// out[t][n] = bf16( sum_{slots by expert asc} w * y[pos] + sg[t] * ys[t][n] )
void launch_combine(const int64_t* ids, const uint16_t* weights, const RouteTables& rt, int T, int top_k,
                    int H, const float* y, const float* shared_gate, const float* shared_y, uint16_t* out,
                    cudaStream_t st);

// sg[t] = sigmoid(x[t] . g) for the shared expert's gate.
void launch_shared_gate(const uint16_t* x, const uint16_t* g, int T, int H, float* sg, cudaStream_t st);

// Single-launch decode step (decode_fused.cu).
struct DecodeFusedParams {
  const uint16_t* x;
  const uint16_t* logits;   // routing computed in-kernel when ids_in == nullptr
  const int64_t* ids_in;
  const uint16_t* w_in;
  const uint8_t* mask;
  int64_t* ids_out;
  uint16_t* w_out;
  QuantProj gate, up, down;
  int T, E, top_k, use_softmax, renorm;
  float* hbuf;
  uint16_t* out;
  unsigned long long* bar;  // grid-barrier arrival counter, zero-initialised, never reset
  unsigned long long* trace;  // optional [num_sms][16] phase timestamps (ns)
  int* status;
  int num_sms;
};
bool decode_fused_eligible(int bits, int T, int E, int top_k, const QuantProj& gate, const QuantProj& down,
                           int num_sms);
// 1 = launched; negative = not launched (caller uses the multi-kernel path).
int launch_decode_fused(int bits, const DecodeFusedParams& p, cudaStream_t st);

// Single-launch decode step for one token (decode_t1.cu).
struct DecodeT1Params {
  const uint16_t* x;
  const uint16_t* logits;  // routing computed in-kernel when ids_in == nullptr
  const int64_t* ids_in;
  const uint16_t* w_in;
  const uint8_t* mask;
  int64_t* ids_out;
  uint16_t* w_out;
  QuantProj gate, up, down;
  int bits, E, top_k, use_softmax, renorm;
  float* hbuf;                // [top_k][I]
  uint16_t* out;
  unsigned long long* bar;    // grid-barrier arrival counter, zero-initialised, never reset
  unsigned long long* trace;  // optional [num_sms][16] phase timestamps (ns)
  int* status;
  int num_sms;
};
// Dynamic shared-memory opt-in + one-CTA-per-SM check, done once per (kernel,
// device) and new maximum size (launch_util.cu).
bool ensure_dynamic_smem(const void* kern, size_t smem, int threads);
// Page-locked, device-mapped host memory (readable by kernels through the same pointer).
bool host_mapped(const void* p);
// xd <- x, ld <- l (byte counts multiples of 16) by a kernel reading mapped host memory.
void launch_stage_in(const void* x, size_t xbytes, const void* l, size_t lbytes, void* xd, void* ld,
                     cudaStream_t st);

bool decode_t1_eligible(const DecodeT1Params& p);
// 1 = launched; negative = not launched.
int launch_decode_t1(const DecodeT1Params& p, cudaStream_t st);

void launch_dequant_rows(int bits, const QuantProj& p, int expert, int row0, int nrows, float* out,
                         cudaStream_t st);

// ---- prefill path: tcgen05 grouped GEMM (grouped_gemm.cu) ----

// 2-D tensor map (CUtensorMap, 128 bytes, 64-byte aligned storage at out_map)
// over a row-major [rows][inner] fp16 or uint8 array; false if the driver
// entry point is unavailable or the encode fails.
bool make_tmap_2d(void* out_map, const void* base, bool fp16, uint64_t inner, uint64_t rows, uint32_t box_inner,
                  uint32_t box_rows, bool swizzle128);
// Shape rules of the GEMM path for one projection (N % 128, K % 64, W4 group
// % 64, W8 per-channel).
bool gemm_shape_ok(int bits, const QuantProj& p);
// Box sizes the tensor maps must be encoded with: codes {64*bits/8, kGemmBM},
// activations {kGemmBK, bn} for the launch's token-tile width bn.
constexpr int kGemmBM = 128, kGemmBK = 64;
constexpr int kGemmTileWidths = 4;  // bn = 16 << i, i < kGemmTileWidths
inline int gemm_tile_index(int bn) { return bn == 16 ? 0 : bn == 32 ? 1 : bn == 64 ? 2 : 3; }

struct GemmLaunch {
  RouteTables rt;
  const int32_t* tile_off;  // [E+1] from launch_tile_table
  QuantProj p0, p1;         // gate, up (gate/up GEMM) or down, unused
  const void* tmap_x;       // activations fp16 [rows][K], box {64, bn}, 128-byte swizzle
  const void* tmap_w0;      // codes of p0 as uint8 [E*N][K*bits/8], box {64*bits/8, 128}
  const void* tmap_w1;      // codes of p1 (gate/up only)
  void* hout;               // gate/up: fp16 SiLU(g)*u [pairs][N], K-permuted for the down GEMM
  float* yout;              // down: fp32 [pairs][N]
  int* status;
  int max_pairs;            // upper bound of the pair count of this call
  int max_active;           // upper bound of the active expert count of this call
  int bn;                   // token-tile width: 16, 32, 64 or 128 (tile_off and tmap_x built for it)
};
// tile_off over the active experts; with shared_tables != nullptr also the
// int32[6] one-expert tables of the shared expert over T tokens: offsets[2],
// active[1], n_active[1], tile_off[2].
void launch_tile_table(const RouteTables& rt, int32_t* tile_off, int32_t* shared_tables, int T, int bn, int sbn,
                       cudaStream_t st);
// x16[s] = fp16(x[token of sorted pair s]) with K permuted to the dequant order.
void launch_pack_x(int bits, const uint16_t* x, const RouteTables& rt, int E, int top_k, int identity_tokens, int H,
                   int max_pairs, void* x16, int num_sms, cudaStream_t st);
// 1 = launched, negative = refused (shared-memory opt-in failed).
int launch_grouped_gemm(int bits, bool gateup, const GemmLaunch& g, cudaStream_t st);

// ---- expert parallelism (ep.cu) ----
// g[p] = slot_of_expert[ids[p]] (ids outside [0, E) -> num_slots).
void launch_ep_remap(const int64_t* ids, int P, const int32_t* slot_of_expert, int E, int num_slots, int64_t* g,
                     cudaStream_t st);
// send_rows[s] = x[token of sorted pair s], send_local[s] = g % experts_per_rank.
void launch_ep_gather(const uint16_t* x, const RouteTables& rt, int num_slots, const int64_t* g, int top_k, int H,
                      int experts_per_rank, int max_pairs, uint16_t* send_rows, int64_t* send_local, int num_sms,
                      cudaStream_t st);
// rows[r] = y[pos[r]] (zero where pos[r] < 0).
void launch_scatter_rows(const int32_t* pos, int n, int H, const float* y, float* rows, int num_sms,
                         cudaStream_t st);

}  // namespace moe
