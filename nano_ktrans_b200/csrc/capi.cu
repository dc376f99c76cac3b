// capi.cu — extern "C" entry points declared in include/moe_b200.h.
//
// Handle lifecycle and error convention follow the reference's native bridge
// (nano_ktrans/kernels/pim_native/host_quantized_bridge.c: opaque handle from
// an init call :233, int status return, caller-provided error buffer filled by
// set_error :157, explicit shutdown :1306).  Unlike that bridge, every compute
// entry point only enqueues work on the caller's CUDA stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/moe_b200.h"
#include "common.cuh"
#include "ep_peer.h"
#include "kernels.h"

namespace {

using moe::QuantProj;
using moe::RouteTables;

struct Handle {
  moe_layer_desc d{};
  int device = 0;
  int num_sms = 148;
  moe_weights w{};
  bool has_weights = false;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  RouteTables rt{};
  float* hbuf = nullptr;   // [max_pairs][I]
  float* ybuf = nullptr;   // [max_pairs][H]
  float* sh_h = nullptr;   // [max_tokens][I_s]
  float* sh_y = nullptr;   // [max_tokens][H]
  float* sh_g = nullptr;   // [max_tokens]
  uint16_t* logits_tmp = nullptr;  // [max_tokens][E] router logits of moe_forward_x / moe_forward_host
  uint16_t* x_stage = nullptr;     // [max_tokens][H] moe_forward_host input
  uint16_t* out_stage = nullptr;   // [max_tokens][H] moe_forward_host output
  int64_t* ids_tmp = nullptr;
  uint16_t* w_tmp = nullptr;
  unsigned long long* grid_bar = nullptr;  // grid-barrier arrival counter of the fused decode kernel
  int decode_fused = 1;  // 0 off, 1 single-token kernel for T == 1 else multi-token, 2 multi-token only
  unsigned long long* trace = nullptr;  // [num_sms][16] phase timestamps when tracing
  // prefill GEMM path: tensor maps over the activation buffers and the codes
  int32_t* tile_off = nullptr;  // [E+1]
  int gemm_mode = 1;            // 0 never, 1 by batch size, 2 whenever the shape allows
  int gemm_tile = 0;            // token-tile width of the GEMM launches: 0 by batch, else 16/32/64/128
  int stream_mode = 1;          // 1: weight-streaming kernels where eligible, 0: matvec kernels
  int host_io = 2;              // moe_forward_host: 0 copies, 1 device reads the inputs, 2 also stores the output
  bool gemm_maps = false;       // tensor maps encoded (shape supported, driver entry point found)
  // activation maps, one per token-tile width 16 << i
  alignas(64) unsigned char tm_x[moe::kGemmTileWidths][128];  // fp16 [max_pairs][H] over ybuf (x in pair order)
  alignas(64) unsigned char tm_h[moe::kGemmTileWidths][128];  // fp16 [max_pairs][I] over hbuf (SiLU(g)*u)
  alignas(64) unsigned char tm_gate[128];  // uint8 [E*I][H*bits/8]
  alignas(64) unsigned char tm_up[128];
  alignas(64) unsigned char tm_down[128];  // uint8 [E*H][I*bits/8]
  // shared expert on the GEMM path
  bool shared_gemm_maps = false;
  int32_t* sh_tables = nullptr;             // int32[6]: one-expert tables over T tokens
  int64_t* slot_ids = nullptr;              // [max_pairs] expert-parallel slot of each pair (moe_ep_dispatch)
  alignas(64) unsigned char tm_sx[moe::kGemmTileWidths][128];  // fp16 [max_tokens][H] over sh_y
  alignas(64) unsigned char tm_sh[moe::kGemmTileWidths][128];  // fp16 [max_tokens][S] over sh_h
  alignas(64) unsigned char tm_sgate[128];  // uint8 [S][H*bits/8]
  alignas(64) unsigned char tm_sup[128];
  alignas(64) unsigned char tm_sdown[128];  // uint8 [H][S*bits/8]
  std::string err;
  int last_launches = 0;
  // profiling: events bracketing one kernel class
  int prof_class = 0;
  int prof_max = 0;
  int prof_n = 0;
  std::vector<cudaEvent_t> prof_ev;
};

// Under stream capture a plain event record only becomes a dependency marker;
// the external flag makes it a real event-record node of the graph, so the
// bracketed kernel can be timed on every replay.
void prof_mark(Handle* h, int cls, bool after, cudaStream_t st) {
  if (h->prof_class != cls || h->prof_n >= h->prof_max) return;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cap);
  cudaEvent_t ev = h->prof_ev[2 * h->prof_n + (after ? 1 : 0)];
  if (cap == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(ev, st, cudaEventRecordExternal);
  else
    cudaEventRecord(ev, st);
  if (after) ++h->prof_n;
}

void fmt_err(char* buf, size_t len, const char* f, ...) {
  if (buf == nullptr || len == 0) return;
  va_list ap;
  va_start(ap, f);
  vsnprintf(buf, len, f, ap);
  va_end(ap);
}

int fail(Handle* h, int code, const char* f, ...) {
  char tmp[512];
  va_list ap;
  va_start(ap, f);
  vsnprintf(tmp, sizeof(tmp), f, ap);
  va_end(ap);
  if (h) h->err = tmp;
  return code;
}

int check_launch(Handle* h, const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(h, MOE_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return MOE_OK;
}

int proj_group(const moe_layer_desc& d, int k) { return d.group_size > 0 ? d.group_size : k; }

QuantProj make_proj(const Handle* h, const void* q, const void* s, int n, int k) {
  QuantProj p;
  p.q = static_cast<const uint8_t*>(q);
  p.s = static_cast<const uint16_t*>(s);
  p.n = n;
  p.k = k;
  p.group = proj_group(h->d, k);
  p.sstride = (k / p.group + 7) / 8 * 8;
  return p;
}

const char* validate_desc(const moe_layer_desc& d) {
  if (d.num_experts < 1 || d.num_experts > 1024) return "num_experts must be in [1, 1024]";
  if (d.top_k < 1 || d.top_k > 16 || d.top_k > d.num_experts) return "top_k must be in [1, min(16, num_experts)]";
  if (d.bits != 4 && d.bits != 8) return "bits must be 4 or 8";
  const int align = d.bits == 4 ? 32 : 16;  // codes per 16-byte chunk
  if (d.hidden_size <= 0 || d.hidden_size % align) return "hidden_size must be a positive multiple of 32 (W4) / 16 (W8)";
  if (d.inter_size <= 0 || d.inter_size % align) return "inter_size must be a positive multiple of 32 (W4) / 16 (W8)";
  if (d.shared_inter < 0 || d.shared_inter % align) return "shared_inter must be a multiple of 32 (W4) / 16 (W8)";
  if (d.group_size < 0) return "group_size must be >= 0";
  if (d.group_size > 0) {
    if (d.group_size % align) return "group_size must be a multiple of 32 (W4) / 16 (W8)";
    if (d.hidden_size % d.group_size || d.inter_size % d.group_size) return "group_size must divide hidden and inter";
    if (d.shared_inter % d.group_size) return "group_size must divide shared_inter";
  }
  if (d.max_tokens < 1) return "max_tokens must be >= 1";
  return nullptr;
}

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

// Tensor maps of the prefill GEMM path.  The activation maps cover the
// workspace buffers at their full max_pairs extent: x (fp16) aliases ybuf,
// which the down GEMM writes only after the gate/up GEMM has read x, and
// SiLU(g)*u (fp16) aliases hbuf.  False when a projection's shape is outside
// the GEMM rules; the multi-kernel matvec path then serves every batch.
bool encode_gemm_maps(Handle* h) {
  const moe_layer_desc& d = h->d;
  const int H = d.hidden_size, I = d.inter_size, E = d.num_experts, bits = d.bits;
  const uint64_t P = static_cast<uint64_t>(d.max_tokens) * d.top_k;
  const QuantProj gate = make_proj(h, h->w.gate_q_dev, h->w.gate_s_dev, I, H);
  const QuantProj down = make_proj(h, h->w.down_q_dev, h->w.down_s_dev, H, I);
  if (!moe::gemm_shape_ok(bits, gate) || !moe::gemm_shape_ok(bits, down)) return false;
  const uint32_t code_box = moe::kGemmBK * bits / 8;
  bool ok = true;
  for (int i = 0; i < moe::kGemmTileWidths; ++i) {
    ok = ok && moe::make_tmap_2d(h->tm_x[i], h->ybuf, true, H, P, moe::kGemmBK, 16u << i, true);
    ok = ok && moe::make_tmap_2d(h->tm_h[i], h->hbuf, true, I, P, moe::kGemmBK, 16u << i, true);
  }
  ok = ok && moe::make_tmap_2d(h->tm_gate, h->w.gate_q_dev, false, static_cast<uint64_t>(H) * bits / 8,
                               static_cast<uint64_t>(E) * I, code_box, moe::kGemmBM, false);
  ok = ok && moe::make_tmap_2d(h->tm_up, h->w.up_q_dev, false, static_cast<uint64_t>(H) * bits / 8,
                               static_cast<uint64_t>(E) * I, code_box, moe::kGemmBM, false);
  ok = ok && moe::make_tmap_2d(h->tm_down, h->w.down_q_dev, false, static_cast<uint64_t>(I) * bits / 8,
                               static_cast<uint64_t>(E) * H, code_box, moe::kGemmBM, false);
  h->shared_gemm_maps = false;
  const int S = d.shared_inter;
  if (ok && S > 0) {
    const QuantProj sg = make_proj(h, h->w.shared_gate_q_dev, h->w.shared_gate_s_dev, S, H);
    const QuantProj sd = make_proj(h, h->w.shared_down_q_dev, h->w.shared_down_s_dev, H, S);
    const uint64_t T = static_cast<uint64_t>(d.max_tokens);
    bool sok = moe::gemm_shape_ok(bits, sg) && moe::gemm_shape_ok(bits, sd);
    for (int i = 0; i < moe::kGemmTileWidths; ++i) {
      sok = sok && moe::make_tmap_2d(h->tm_sx[i], h->sh_y, true, H, T, moe::kGemmBK, 16u << i, true);
      sok = sok && moe::make_tmap_2d(h->tm_sh[i], h->sh_h, true, S, T, moe::kGemmBK, 16u << i, true);
    }
    sok = sok && moe::make_tmap_2d(h->tm_sgate, h->w.shared_gate_q_dev, false, static_cast<uint64_t>(H) * bits / 8,
                                   S, code_box, moe::kGemmBM, false);
    sok = sok && moe::make_tmap_2d(h->tm_sup, h->w.shared_up_q_dev, false, static_cast<uint64_t>(H) * bits / 8, S,
                                   code_box, moe::kGemmBM, false);
    sok = sok && moe::make_tmap_2d(h->tm_sdown, h->w.shared_down_q_dev, false, static_cast<uint64_t>(S) * bits / 8,
                                   H, code_box, moe::kGemmBM, false);
    h->shared_gemm_maps = sok;
  }
  return ok;
}

// The GEMM path pays off once experts see several tokens each; below that
// the matvec kernels stream the same weight bytes with less fixed cost.
// Token-tile width of a grouped-GEMM launch: the smallest of 16/32/64/128
// covering the mean token count of an active expert.
int pick_bn(int pairs, int experts) {
  const int active = std::max(1, std::min(experts, pairs));
  const int mean = (pairs + active - 1) / active;
  return mean <= 16 ? 16 : mean <= 32 ? 32 : mean <= 64 ? 64 : 128;
}

// With the weight-streaming kernels available the GEMM takes over once the
// mean expert sees two full 8-token chunks; without them, at half that.
bool use_gemm(const Handle* h, int pairs, bool stream_ok) {
  if (!h->gemm_maps || h->gemm_mode == 0) return false;
  if (h->gemm_mode == 2) return true;
  return pairs >= (stream_ok ? 16 : 4) * h->d.num_experts;
}

}  // namespace

extern "C" {

int moe_abi_version(void) { return MOE_B200_ABI_VERSION; }

int moe_create(const moe_layer_desc* desc, void** handle, char* err, size_t err_len) {
  if (desc == nullptr || handle == nullptr) {
    fmt_err(err, err_len, "moe_create: null argument");
    return MOE_EINVAL;
  }
  if (const char* why = validate_desc(*desc)) {
    fmt_err(err, err_len, "moe_create: %s", why);
    return MOE_EINVAL;
  }
  Handle* h = new Handle();
  h->d = *desc;
  cudaGetDevice(&h->device);
  cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, h->device);
  const moe_layer_desc& d = h->d;
  const size_t E = d.num_experts, T = d.max_tokens, P = T * d.top_k;
  const size_t H = d.hidden_size, I = d.inter_size, S = d.shared_inter;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  const size_t o_status = take(4), o_counts = take(4 * E), o_offsets = take(4 * (E + 1)), o_active = take(4 * E),
               o_nact = take(4), o_sorted = take(4 * P), o_pos = take(4 * P), o_h = take(4 * P * I),
               o_y = take(4 * P * H), o_shh = take(S ? 4 * T * S : 0), o_shy = take(S ? 4 * T * H : 0),
               o_shg = take(S ? 4 * T : 0), o_ids = take(8 * P), o_w = take(2 * P), o_bar = take(8),
               o_tiles = take(4 * (E + 1)), o_shtab = take(4 * 8), o_gids = take(8 * P), o_lg = take(2 * T * E),
               o_xs = take(2 * T * H), o_os = take(2 * T * H);
  h->ws_bytes = off;
  cudaError_t e = cudaMalloc(&h->ws, h->ws_bytes);
  if (e != cudaSuccess) {
    fmt_err(err, err_len, "moe_create: cudaMalloc(%zu) failed: %s", h->ws_bytes, cudaGetErrorString(e));
    delete h;
    return MOE_ECUDA;
  }
  char* b = static_cast<char*>(h->ws);
  h->rt.status = reinterpret_cast<int32_t*>(b + o_status);
  h->rt.counts = reinterpret_cast<int32_t*>(b + o_counts);
  h->rt.offsets = reinterpret_cast<int32_t*>(b + o_offsets);
  h->rt.active = reinterpret_cast<int32_t*>(b + o_active);
  h->rt.n_active = reinterpret_cast<int32_t*>(b + o_nact);
  h->rt.sorted_pair = reinterpret_cast<int32_t*>(b + o_sorted);
  h->rt.pair_pos = reinterpret_cast<int32_t*>(b + o_pos);
  h->hbuf = reinterpret_cast<float*>(b + o_h);
  h->ybuf = reinterpret_cast<float*>(b + o_y);
  if (S) {
    h->sh_h = reinterpret_cast<float*>(b + o_shh);
    h->sh_y = reinterpret_cast<float*>(b + o_shy);
    h->sh_g = reinterpret_cast<float*>(b + o_shg);
  }
  h->ids_tmp = reinterpret_cast<int64_t*>(b + o_ids);
  h->w_tmp = reinterpret_cast<uint16_t*>(b + o_w);
  h->grid_bar = reinterpret_cast<unsigned long long*>(b + o_bar);
  h->tile_off = reinterpret_cast<int32_t*>(b + o_tiles);
  h->sh_tables = reinterpret_cast<int32_t*>(b + o_shtab);
  h->slot_ids = reinterpret_cast<int64_t*>(b + o_gids);
  h->logits_tmp = reinterpret_cast<uint16_t*>(b + o_lg);
  h->x_stage = reinterpret_cast<uint16_t*>(b + o_xs);
  h->out_stage = reinterpret_cast<uint16_t*>(b + o_os);
  e = cudaMemset(h->ws, 0, h->ws_bytes);
  if (e != cudaSuccess) {
    fmt_err(err, err_len, "moe_create: cudaMemset failed: %s", cudaGetErrorString(e));
    cudaFree(h->ws);
    delete h;
    return MOE_ECUDA;
  }
  *handle = h;
  return MOE_OK;
}

int moe_set_weights(void* handle, const moe_weights* w, char* err, size_t err_len) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr || w == nullptr) {
    fmt_err(err, err_len, "moe_set_weights: null argument");
    return MOE_EINVAL;
  }
  const void* need[] = {w->gate_q_dev, w->gate_s_dev, w->up_q_dev, w->up_s_dev, w->down_q_dev, w->down_s_dev};
  for (const void* p : need) {
    if (p == nullptr) {
      fmt_err(err, err_len, "moe_set_weights: routed-expert weight pointer is NULL");
      return MOE_EINVAL;
    }
    if (reinterpret_cast<uintptr_t>(p) % 16) {
      fmt_err(err, err_len, "moe_set_weights: weight pointers must be 16-byte aligned");
      return MOE_EINVAL;
    }
  }
  if (h->d.shared_inter > 0) {
    const void* sh[] = {w->shared_gate_q_dev, w->shared_gate_s_dev, w->shared_up_q_dev, w->shared_up_s_dev,
                        w->shared_down_q_dev, w->shared_down_s_dev, w->shared_gate_vec_dev};
    for (const void* p : sh) {
      if (p == nullptr) {
        fmt_err(err, err_len, "moe_set_weights: shared-expert weight pointer is NULL");
        return MOE_EINVAL;
      }
    }
  }
  h->w = *w;
  h->has_weights = true;
  h->gemm_maps = encode_gemm_maps(h);
  return MOE_OK;
}

int moe_route(void* handle, const uint16_t* logits_dev, int32_t T, int64_t* ids_dev, uint16_t* w_dev, void* stream) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return MOE_EINVAL;
  if (T < 0) return fail(h, MOE_EINVAL, "moe_route: negative token count");
  if (T > 0 && (logits_dev == nullptr || ids_dev == nullptr || w_dev == nullptr))
    return fail(h, MOE_EINVAL, "moe_route: null device pointer");
  moe::launch_route(logits_dev, T, h->d.num_experts, h->d.top_k, h->d.router_use_softmax != 0,
                    h->d.normalize_topk_prob != 0, ids_dev, w_dev, static_cast<cudaStream_t>(stream));
  return check_launch(h, "moe_route");
}

// The single-launch decode kernel, when the batch is small enough and no
// shared expert is requested.  `logits` set: route in-kernel, writing
// ids_out/w_out; otherwise ids/wts are the given routing.  Returns true when
// launched.
static bool try_decode_fused(Handle* h, const uint16_t* x, const uint16_t* logits, const int64_t* ids,
                             const uint16_t* wts, int64_t* ids_out, uint16_t* w_out, int T, const uint8_t* mask,
                             bool add_shared, uint16_t* out, cudaStream_t st) {
  const moe_layer_desc& d = h->d;
  if (!h->decode_fused || (add_shared && d.shared_inter > 0)) return false;
  const int H = d.hidden_size, I = d.inter_size;
  if (T == 1 && h->decode_fused == 1) {
    moe::DecodeT1Params q{};
    q.gate = make_proj(h, h->w.gate_q_dev, h->w.gate_s_dev, I, H);
    q.up = make_proj(h, h->w.up_q_dev, h->w.up_s_dev, I, H);
    q.down = make_proj(h, h->w.down_q_dev, h->w.down_s_dev, H, I);
    q.x = x;
    q.logits = logits;
    q.ids_in = logits ? nullptr : ids;
    q.w_in = logits ? nullptr : wts;
    q.mask = mask;
    q.ids_out = ids_out;
    q.w_out = w_out;
    q.bits = d.bits;
    q.E = d.num_experts;
    q.top_k = d.top_k;
    q.use_softmax = d.router_use_softmax;
    q.renorm = d.normalize_topk_prob;
    q.hbuf = h->hbuf;
    q.out = out;
    q.bar = h->grid_bar;
    q.trace = h->trace;
    q.status = h->rt.status;
    q.num_sms = h->num_sms;
    if (moe::decode_t1_eligible(q)) {
      prof_mark(h, MOE_K_DECODE_FUSED, false, st);
      const int rc = moe::launch_decode_t1(q, st);
      prof_mark(h, MOE_K_DECODE_FUSED, true, st);
      if (rc > 0) {
        h->last_launches = 1;
        return true;
      }
      cudaGetLastError();  // a refused launch configuration is not sticky; fall through
    }
  }
  moe::DecodeFusedParams p{};
  p.gate = make_proj(h, h->w.gate_q_dev, h->w.gate_s_dev, I, H);
  p.up = make_proj(h, h->w.up_q_dev, h->w.up_s_dev, I, H);
  p.down = make_proj(h, h->w.down_q_dev, h->w.down_s_dev, H, I);
  if (!moe::decode_fused_eligible(d.bits, T, d.num_experts, d.top_k, p.gate, p.down, h->num_sms)) return false;
  p.x = x;
  p.logits = logits;
  p.ids_in = logits ? nullptr : ids;
  p.w_in = logits ? nullptr : wts;
  p.mask = mask;
  p.ids_out = ids_out;
  p.w_out = w_out;
  p.T = T;
  p.E = d.num_experts;
  p.top_k = d.top_k;
  p.use_softmax = d.router_use_softmax;
  p.renorm = d.normalize_topk_prob;
  p.hbuf = h->hbuf;
  p.out = out;
  p.bar = h->grid_bar;
  p.trace = h->trace;
  p.status = h->rt.status;
  p.num_sms = h->num_sms;
  prof_mark(h, MOE_K_DECODE_FUSED, false, st);
  const int rc = moe::launch_decode_fused(d.bits, p, st);
  prof_mark(h, MOE_K_DECODE_FUSED, true, st);
  if (rc < 0) {
    cudaGetLastError();  // a refused launch configuration is not sticky; use the multi-kernel path
    return false;
  }
  h->last_launches = 1;
  return true;
}

// Routed experts for T tokens with `ids` [T][k].  Normally ends with the
// weighted combine into `out`; with rows_out set, k is 1 (each "token" is one
// (token, expert) row), the shared expert is skipped and the unweighted fp32
// expert output of row r goes to rows_out[r].
// Output of the expert-parallel peer step (moe_ep_peer_experts): each pair's
// fp32 row goes to its token's rank's region instead of a local combine.
struct PeerScatter {
  const moe::PeerView* view;
  const unsigned long long* epoch;
  unsigned int* counter;
  int bound;       // tokens per rank in the step: T = world * bound
  int pairs_hint;  // pairs expected among the T*k slots: picks the kernels
};

static int experts_forward(Handle* h, const uint16_t* x, const int64_t* ids, const uint16_t* wts, int T,
                           const uint8_t* mask, bool add_shared, uint16_t* out, cudaStream_t st, int launches,
                           float* rows_out = nullptr, const PeerScatter* peer = nullptr) {
  const moe_layer_desc& d = h->d;
  const int E = d.num_experts, H = d.hidden_size, I = d.inter_size;
  const int k = rows_out ? 1 : d.top_k;
  if (rows_out || peer) add_shared = false;
  if (launches == 0 && !rows_out && !peer &&
      try_decode_fused(h, x, nullptr, ids, wts, nullptr, nullptr, T, mask, add_shared, out, st))
    return check_launch(h, "moe_experts_forward");
  prof_mark(h, MOE_K_PERMUTE, false, st);
  moe::launch_permute(ids, T, k, E, mask, h->rt, st, peer != nullptr);
  prof_mark(h, MOE_K_PERMUTE, true, st);
  ++launches;
  const int max_active = std::min(E, T * k);
  const int pairs = peer ? std::max(1, std::min(peer->pairs_hint, T * k)) : T * k;  // for the kernel choice
  const QuantProj gate = make_proj(h, h->w.gate_q_dev, h->w.gate_s_dev, I, H);
  const QuantProj up = make_proj(h, h->w.up_q_dev, h->w.up_s_dev, I, H);
  const QuantProj down = make_proj(h, h->w.down_q_dev, h->w.down_s_dev, H, I);
  if (h->gemm_mode == 2 && !h->gemm_maps)
    return fail(h, MOE_EINVAL, "GEMM path forced but this layer's shape is outside its rules");
  const bool shared_gemm = add_shared && d.shared_inter > 0 && h->shared_gemm_maps && h->gemm_mode != 0 &&
                           (h->gemm_mode == 2 || T >= 16);
  const bool stream_ok = h->stream_mode && moe::stream_eligible(d.bits, gate, up, down, max_active);
  const bool routed_gemm = use_gemm(h, pairs, stream_ok);
  const int bn = h->gemm_tile ? h->gemm_tile : pick_bn(pairs, E);
  const int sbn = h->gemm_tile ? h->gemm_tile : pick_bn(T, 1);
  if (routed_gemm || shared_gemm) {
    moe::launch_tile_table(h->rt, h->tile_off, shared_gemm ? h->sh_tables : nullptr, T, bn, sbn, st);
    ++launches;
  }
  if (routed_gemm) {
    moe::launch_pack_x(d.bits, x, h->rt, E, k, 0, H, T * k, h->ybuf, h->num_sms, st);
    ++launches;
    moe::GemmLaunch g{};
    g.rt = h->rt;
    g.tile_off = h->tile_off;
    g.status = h->rt.status;
    g.max_pairs = T * k;
    g.max_active = max_active;
    g.bn = bn;
    g.p0 = gate;
    g.p1 = up;
    g.tmap_x = h->tm_x[moe::gemm_tile_index(bn)];
    g.tmap_w0 = h->tm_gate;
    g.tmap_w1 = h->tm_up;
    g.hout = h->hbuf;
    prof_mark(h, MOE_K_GATEUP, false, st);
    int rc = moe::launch_grouped_gemm(d.bits, true, g, st);
    prof_mark(h, MOE_K_GATEUP, true, st);
    if (rc < 0) return fail(h, MOE_ECUDA, "grouped GEMM (gate/up): shared-memory opt-in refused");
    g.p0 = down;
    g.p1 = down;
    g.tmap_x = h->tm_h[moe::gemm_tile_index(bn)];
    g.tmap_w0 = h->tm_down;
    g.tmap_w1 = h->tm_down;
    g.hout = nullptr;
    g.yout = h->ybuf;
    prof_mark(h, MOE_K_DOWN, false, st);
    rc = moe::launch_grouped_gemm(d.bits, false, g, st);
    prof_mark(h, MOE_K_DOWN, true, st);
    if (rc < 0) return fail(h, MOE_ECUDA, "grouped GEMM (down): shared-memory opt-in refused");
    launches += 2;
  } else if (stream_ok) {
    prof_mark(h, MOE_K_GATEUP, false, st);
    int rc = moe::launch_stream_gateup(x, h->rt, k, max_active, gate, up, h->hbuf, h->rt.status, h->trace,
                                       h->num_sms, st);
    prof_mark(h, MOE_K_GATEUP, true, st);
    if (rc < 0) return fail(h, MOE_ECUDA, "streaming gate/up: launch refused");
    prof_mark(h, MOE_K_DOWN, false, st);
    rc = moe::launch_stream_down(h->hbuf, h->rt, max_active, down, h->ybuf, h->rt.status, h->num_sms, st);
    prof_mark(h, MOE_K_DOWN, true, st);
    if (rc < 0) return fail(h, MOE_ECUDA, "streaming down: launch refused");
    launches += 2;
  } else {
    prof_mark(h, MOE_K_GATEUP, false, st);
    launches += moe::launch_gateup(d.bits, x, h->rt, k, max_active, T, 0, gate, up, h->hbuf, h->num_sms, st);
    prof_mark(h, MOE_K_GATEUP, true, st);
    prof_mark(h, MOE_K_DOWN, false, st);
    launches += moe::launch_down(d.bits, h->hbuf, h->rt, max_active, T, 0, down, h->ybuf, h->num_sms, st);
    prof_mark(h, MOE_K_DOWN, true, st);
  }
  const float* sg = nullptr;
  const float* sy = nullptr;
  if (add_shared && d.shared_inter > 0) {
    const int S = d.shared_inter;
    const QuantProj sgp = make_proj(h, h->w.shared_gate_q_dev, h->w.shared_gate_s_dev, S, H);
    const QuantProj sup = make_proj(h, h->w.shared_up_q_dev, h->w.shared_up_s_dev, S, H);
    const QuantProj sdp = make_proj(h, h->w.shared_down_q_dev, h->w.shared_down_s_dev, H, S);
    moe::launch_shared_gate(x, static_cast<const uint16_t*>(h->w.shared_gate_vec_dev), T, H, h->sh_g, st);
    ++launches;
    if (shared_gemm) {
      // one expert over tokens 0..T-1; x (fp16) staged in sh_y, which the down GEMM overwrites afterwards
      moe::launch_pack_x(d.bits, x, h->rt, E, k, T, H, T, h->sh_y, h->num_sms, st);
      moe::GemmLaunch g{};
      g.rt.offsets = h->sh_tables;
      g.rt.active = h->sh_tables + 2;
      g.rt.n_active = h->sh_tables + 3;
      g.tile_off = h->sh_tables + 4;
      g.status = h->rt.status;
      g.max_pairs = T;
      g.max_active = 1;
      g.bn = sbn;
      g.p0 = sgp;
      g.p1 = sup;
      g.tmap_x = h->tm_sx[moe::gemm_tile_index(sbn)];
      g.tmap_w0 = h->tm_sgate;
      g.tmap_w1 = h->tm_sup;
      g.hout = h->sh_h;
      int rc = moe::launch_grouped_gemm(d.bits, true, g, st);
      if (rc < 0) return fail(h, MOE_ECUDA, "grouped GEMM (shared gate/up): shared-memory opt-in refused");
      g.p0 = sdp;
      g.p1 = sdp;
      g.tmap_x = h->tm_sh[moe::gemm_tile_index(sbn)];
      g.tmap_w0 = h->tm_sdown;
      g.tmap_w1 = h->tm_sdown;
      g.hout = nullptr;
      g.yout = h->sh_y;
      rc = moe::launch_grouped_gemm(d.bits, false, g, st);
      if (rc < 0) return fail(h, MOE_ECUDA, "grouped GEMM (shared down): shared-memory opt-in refused");
      launches += 3;
    } else {
      launches += moe::launch_gateup(d.bits, x, h->rt, 1, 1, T, T, sgp, sup, h->sh_h, h->num_sms, st);
      launches += moe::launch_down(d.bits, h->sh_h, h->rt, 1, T, T, sdp, h->sh_y, h->num_sms, st);
    }
    sg = h->sh_g;
    sy = h->sh_y;
  }
  prof_mark(h, MOE_K_COMBINE, false, st);
  if (peer)
    moe::launch_ep_peer_scatter(*peer->view, h->rt.pair_pos, T * k, peer->bound, h->ybuf, peer->epoch,
                                peer->counter, h->num_sms, st);
  else if (rows_out)
    moe::launch_scatter_rows(h->rt.pair_pos, T, H, h->ybuf, rows_out, h->num_sms, st);
  else
    moe::launch_combine(ids, wts, h->rt, T, k, H, h->ybuf, sg, sy, out, st);
  prof_mark(h, MOE_K_COMBINE, true, st);
  ++launches;
  h->last_launches = launches;
  return check_launch(h, peer ? "moe_ep_peer_experts" : rows_out ? "moe_rows_forward" : "moe_experts_forward");
}

static int check_forward_args(Handle* h, const void* x, const void* out, int T) {
  if (!h->has_weights) return fail(h, MOE_ENOWEIGHTS, "weights not set (call moe_set_weights first)");
  if (T < 0) return fail(h, MOE_EINVAL, "negative token count");
  if (T > h->d.max_tokens) return fail(h, MOE_ERANGE, "token count %d above max_tokens %d", T, h->d.max_tokens);
  if (T > 0 && (x == nullptr || out == nullptr)) return fail(h, MOE_EINVAL, "null device pointer");
  return MOE_OK;
}

int moe_experts_forward(void* handle, const uint16_t* x_dev, const int64_t* ids_dev, const uint16_t* w_dev, int32_t T,
                        const uint8_t* mask_dev, int32_t add_shared, uint16_t* out_dev, void* stream) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return MOE_EINVAL;
  if (int rc = check_forward_args(h, x_dev, out_dev, T)) return rc;
  if (T > 0 && (ids_dev == nullptr || w_dev == nullptr)) return fail(h, MOE_EINVAL, "null routing pointer");
  h->last_launches = 0;
  if (T == 0) return MOE_OK;
  return experts_forward(h, x_dev, ids_dev, w_dev, T, mask_dev, add_shared != 0, out_dev,
                         static_cast<cudaStream_t>(stream), 0);
}

int moe_forward(void* handle, const uint16_t* x_dev, const uint16_t* logits_dev, int32_t T, uint16_t* out_dev,
                int64_t* ids_dev, uint16_t* w_dev, void* stream) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return MOE_EINVAL;
  if (int rc = check_forward_args(h, x_dev, out_dev, T)) return rc;
  if (T > 0 && logits_dev == nullptr) return fail(h, MOE_EINVAL, "null logits pointer");
  h->last_launches = 0;
  if (T == 0) return MOE_OK;
  int64_t* ids = ids_dev ? ids_dev : h->ids_tmp;
  uint16_t* wts = w_dev ? w_dev : h->w_tmp;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (try_decode_fused(h, x_dev, logits_dev, nullptr, nullptr, ids, wts, T, nullptr, true, out_dev, st))
    return check_launch(h, "moe_forward");
  prof_mark(h, MOE_K_ROUTE, false, st);
  moe::launch_route(logits_dev, T, h->d.num_experts, h->d.top_k, h->d.router_use_softmax != 0,
                    h->d.normalize_topk_prob != 0, ids, wts, st);
  prof_mark(h, MOE_K_ROUTE, true, st);
  return experts_forward(h, x_dev, ids, wts, T, nullptr, true, out_dev, st, 1);
}

int moe_forward_host(void* handle, const uint16_t* x_host, const uint16_t* logits_host, int32_t T,
                     uint16_t* out_host, void* stream) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return MOE_EINVAL;
  if (int rc = check_forward_args(h, x_host, out_host, T)) return rc;
  if (T > 0 && logits_host == nullptr) return fail(h, MOE_EINVAL, "null logits pointer");
  h->last_launches = 0;
  if (T == 0) return MOE_OK;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t xb = sizeof(uint16_t) * static_cast<size_t>(T) * h->d.hidden_size;
  const size_t lb = sizeof(uint16_t) * static_cast<size_t>(T) * h->d.num_experts;
  // Page-locked host buffers are mapped into the device's address space: the
  // inputs are then read by one small kernel (no copy-engine round trips) and,
  // with host_io 2, the output is stored straight into host memory by the
  // step's last kernel.  Pageable buffers always take the copy engine.
  // every call asks the driver what each pointer is: a kernel may only touch
  // memory that is page-locked and mapped right now
  const bool in_mapped = h->host_io > 0 && xb % 16 == 0 && lb % 16 == 0 && moe::host_mapped(x_host) &&
                         moe::host_mapped(logits_host);
  const bool out_mapped = h->host_io > 1 && moe::host_mapped(out_host);
  int launches = 0;
  if (in_mapped) {
    moe::launch_stage_in(x_host, xb, logits_host, lb, h->x_stage, h->logits_tmp, st);
    launches = 1;
  } else if (cudaMemcpyAsync(h->x_stage, x_host, xb, cudaMemcpyHostToDevice, st) != cudaSuccess ||
             cudaMemcpyAsync(h->logits_tmp, logits_host, lb, cudaMemcpyHostToDevice, st) != cudaSuccess) {
    return fail(h, MOE_ECUDA, "moe_forward_host: input copy failed: %s", cudaGetErrorString(cudaGetLastError()));
  }
  uint16_t* dst = out_mapped ? out_host : h->out_stage;
  if (int rc = moe_forward(handle, h->x_stage, h->logits_tmp, T, dst, nullptr, nullptr, stream)) return rc;
  h->last_launches += launches;
  if (!out_mapped && cudaMemcpyAsync(out_host, h->out_stage, xb, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return fail(h, MOE_ECUDA, "moe_forward_host: output copy failed: %s", cudaGetErrorString(cudaGetLastError()));
  return check_launch(h, "moe_forward_host");
}

int moe_router_logits(void* handle, const uint16_t* x_dev, const uint16_t* router_w_dev, int32_t T,
                      uint16_t* logits_dev, void* stream) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return MOE_EINVAL;
  if (T < 0) return fail(h, MOE_EINVAL, "moe_router_logits: negative token count");
  if (T == 0) return MOE_OK;
  if (x_dev == nullptr || router_w_dev == nullptr || logits_dev == nullptr)
    return fail(h, MOE_EINVAL, "moe_router_logits: null device pointer");
  if (!moe::router_shape_ok(h->d.num_experts, h->d.hidden_size, x_dev, router_w_dev))
    return fail(h, MOE_EINVAL, "moe_router_logits: x and the router weight must be 16-byte aligned");
  moe::launch_router_logits(x_dev, router_w_dev, T, h->d.num_experts, h->d.hidden_size, logits_dev,
                            static_cast<cudaStream_t>(stream));
  return check_launch(h, "moe_router_logits");
}

int moe_forward_x(void* handle, const uint16_t* x_dev, const uint16_t* router_w_dev, int32_t T, uint16_t* out_dev,
                  int64_t* ids_dev, uint16_t* w_dev, uint16_t* logits_dev, void* stream) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return MOE_EINVAL;
  if (int rc = check_forward_args(h, x_dev, out_dev, T)) return rc;
  if (T == 0) {
    h->last_launches = 0;
    return MOE_OK;
  }
  uint16_t* lg = logits_dev ? logits_dev : h->logits_tmp;
  if (int rc = moe_router_logits(handle, x_dev, router_w_dev, T, lg, stream)) return rc;
  if (int rc = moe_forward(handle, x_dev, lg, T, out_dev, ids_dev, w_dev, stream)) return rc;
  h->last_launches += 1;
  return MOE_OK;
}

int moe_ep_dispatch(void* handle, const uint16_t* x_dev, const int64_t* ids_dev, int32_t T,
                    const int32_t* slot_of_expert_dev, int32_t experts_per_rank, int32_t world,
                    uint16_t* send_rows_dev, int64_t* send_local_dev, int32_t* slot_counts_dev, void* stream) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return MOE_EINVAL;
  const moe_layer_desc& d = h->d;
  if (T < 0) return fail(h, MOE_EINVAL, "moe_ep_dispatch: negative token count");
  if (T > d.max_tokens) return fail(h, MOE_ERANGE, "moe_ep_dispatch: token count %d above max_tokens %d", T,
                                    d.max_tokens);
  if (world < 1 || experts_per_rank < 1 || static_cast<int64_t>(world) * experts_per_rank != d.num_experts)
    return fail(h, MOE_EINVAL, "moe_ep_dispatch: world * experts_per_rank must equal num_experts");
  if (slot_counts_dev == nullptr || slot_of_expert_dev == nullptr)
    return fail(h, MOE_EINVAL, "moe_ep_dispatch: null table pointer");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int E = d.num_experts, k = d.top_k, P = T * d.top_k;
  if (T > 0) {
    if (x_dev == nullptr || ids_dev == nullptr || send_rows_dev == nullptr || send_local_dev == nullptr)
      return fail(h, MOE_EINVAL, "moe_ep_dispatch: null device pointer");
    moe::launch_ep_remap(ids_dev, P, slot_of_expert_dev, E, E, h->slot_ids, st);
    moe::launch_permute(h->slot_ids, T, k, E, nullptr, h->rt, st);
    moe::launch_ep_gather(x_dev, h->rt, E, h->slot_ids, k, d.hidden_size, experts_per_rank, P, send_rows_dev,
                          send_local_dev, h->num_sms, st);
    if (cudaMemcpyAsync(slot_counts_dev, h->rt.counts, sizeof(int32_t) * E, cudaMemcpyDeviceToDevice, st) !=
        cudaSuccess)
      return fail(h, MOE_ECUDA, "moe_ep_dispatch: counts copy failed");
  } else if (cudaMemsetAsync(slot_counts_dev, 0, sizeof(int32_t) * E, st) != cudaSuccess) {
    return fail(h, MOE_ECUDA, "moe_ep_dispatch: counts reset failed");
  }
  h->last_launches = T > 0 ? 3 : 0;
  return check_launch(h, "moe_ep_dispatch");
}

int moe_rows_forward(void* handle, const uint16_t* x_rows_dev, const int64_t* row_expert_dev, int32_t n,
                     float* y_rows_dev, void* stream) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return MOE_EINVAL;
  if (!h->has_weights) return fail(h, MOE_ENOWEIGHTS, "weights not set (call moe_set_weights first)");
  if (n < 0) return fail(h, MOE_EINVAL, "moe_rows_forward: negative row count");
  if (static_cast<int64_t>(n) > static_cast<int64_t>(h->d.max_tokens) * h->d.top_k)
    return fail(h, MOE_ERANGE, "moe_rows_forward: %d rows above max_tokens * top_k = %d", n,
                h->d.max_tokens * h->d.top_k);
  h->last_launches = 0;
  if (n == 0) return MOE_OK;
  if (x_rows_dev == nullptr || row_expert_dev == nullptr || y_rows_dev == nullptr)
    return fail(h, MOE_EINVAL, "moe_rows_forward: null device pointer");
  return experts_forward(h, x_rows_dev, row_expert_dev, nullptr, n, nullptr, false, nullptr,
                         static_cast<cudaStream_t>(stream), 0, y_rows_dev);
}

int moe_ep_peer_experts(void* group, void* expert_handle, int32_t tokens_per_rank, int32_t pairs_hint,
                        void* stream) {
  auto* g = static_cast<moe::PeerGroup*>(group);
  Handle* h = static_cast<Handle*>(expert_handle);
  if (g == nullptr || h == nullptr) return MOE_EINVAL;
  const moe::PeerView& v = g->v;
  auto gerr = [&](int code, const char* msg) {
    g->err = std::string("moe_ep_peer_experts: ") + msg;
    return code;
  };
  if (g->phase != 1) return gerr(MOE_EINVAL, "moe_ep_peer_publish has not run for this step");
  if (!h->has_weights) return gerr(MOE_ENOWEIGHTS, "the expert handle has no weights");
  if (h->device != g->device) return gerr(MOE_EINVAL, "the expert handle lives on another device");
  if (h->d.num_experts != v.experts_per_rank || h->d.top_k != v.top_k || h->d.hidden_size != v.hidden)
    return gerr(MOE_EINVAL, "the expert handle must hold num_experts / world experts with the group's top_k and hidden");
  const int bound = tokens_per_rank > 0 ? tokens_per_rank : v.max_tokens;
  if (bound > v.max_tokens) return gerr(MOE_ERANGE, "tokens_per_rank above the group's max_tokens");
  if (bound < g->published_tokens) return gerr(MOE_ERANGE, "tokens_per_rank below this rank's published tokens");
  const int T_all = v.world * bound;
  if (h->d.max_tokens < T_all) return gerr(MOE_ERANGE, "the expert handle's max_tokens is below world * tokens_per_rank");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaGetLastError();
  moe::launch_ep_peer_collect(v, g->epoch, bound, g->x_all, g->ids_all, g->num_sms, st);
  const PeerScatter ps{&g->v, g->epoch, g->counters + 1, bound, pairs_hint};
  if (int rc = experts_forward(h, g->x_all, g->ids_all, nullptr, T_all, nullptr, false, nullptr, st, 1, nullptr, &ps)) {
    g->err = "moe_ep_peer_experts: " + h->err;
    return rc;
  }
  g->phase = 2;
  return MOE_OK;
}

int moe_ep_combine(void* handle, const int64_t* ids_dev, const uint16_t* w_dev, int32_t T, const float* rows_dev,
                   uint16_t* out_dev, void* stream) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return MOE_EINVAL;
  if (T < 0 || T > h->d.max_tokens) return fail(h, MOE_ERANGE, "moe_ep_combine: bad token count %d", T);
  h->last_launches = 0;
  if (T == 0) return MOE_OK;
  if (ids_dev == nullptr || w_dev == nullptr || rows_dev == nullptr || out_dev == nullptr)
    return fail(h, MOE_EINVAL, "moe_ep_combine: null device pointer");
  moe::launch_combine(ids_dev, w_dev, h->rt, T, h->d.top_k, h->d.hidden_size, rows_dev, nullptr, nullptr, out_dev,
                      static_cast<cudaStream_t>(stream));
  h->last_launches = 1;
  return check_launch(h, "moe_ep_combine");
}

int moe_dequant_rows(void* handle, int32_t proj, int32_t expert, int32_t row0, int32_t nrows, float* out_dev,
                     void* stream) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return MOE_EINVAL;
  if (!h->has_weights) return fail(h, MOE_ENOWEIGHTS, "weights not set");
  const moe_layer_desc& d = h->d;
  const int H = d.hidden_size, I = d.inter_size, S = d.shared_inter;
  QuantProj p;
  int E = d.num_experts;
  switch (proj) {
    case 0: p = make_proj(h, h->w.gate_q_dev, h->w.gate_s_dev, I, H); break;
    case 1: p = make_proj(h, h->w.up_q_dev, h->w.up_s_dev, I, H); break;
    case 2: p = make_proj(h, h->w.down_q_dev, h->w.down_s_dev, H, I); break;
    case 3: case 4: case 5:
      if (S == 0) return fail(h, MOE_EINVAL, "layer has no shared expert");
      E = 1;
      p = proj == 3 ? make_proj(h, h->w.shared_gate_q_dev, h->w.shared_gate_s_dev, S, H)
        : proj == 4 ? make_proj(h, h->w.shared_up_q_dev, h->w.shared_up_s_dev, S, H)
                    : make_proj(h, h->w.shared_down_q_dev, h->w.shared_down_s_dev, H, S);
      break;
    default: return fail(h, MOE_EINVAL, "proj must be 0..5");
  }
  if (expert < 0 || expert >= E) return fail(h, MOE_EINVAL, "expert out of range");
  if (row0 < 0 || nrows < 0 || row0 + nrows > p.n) return fail(h, MOE_EINVAL, "row range out of bounds");
  if (nrows > 0 && out_dev == nullptr) return fail(h, MOE_EINVAL, "null output");
  moe::launch_dequant_rows(d.bits, p, expert, row0, nrows, out_dev, static_cast<cudaStream_t>(stream));
  return check_launch(h, "moe_dequant_rows");
}

int moe_read_status(void* handle, int32_t* status, void* stream) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr || status == nullptr) return MOE_EINVAL;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(status, h->rt.status, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaMemsetAsync(h->rt.status, 0, sizeof(int32_t), st);
  // a timed-out grid barrier may have left its arrival count behind: reset it
  if (e == cudaSuccess && (*status & moe::kStatusTimeout)) e = cudaMemsetAsync(h->grid_bar, 0, 8, st);
  if (e != cudaSuccess) return fail(h, MOE_ECUDA, "moe_read_status: %s", cudaGetErrorString(e));
  return MOE_OK;
}

int moe_set_option(void* handle, int32_t option, int32_t value) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return MOE_EINVAL;
  switch (option) {
    case MOE_OPT_DECODE_FUSED:
      if (value < 0 || value > 2) return fail(h, MOE_EINVAL, "moe_set_option(decode fused): value must be 0, 1 or 2");
      h->decode_fused = value;
      return MOE_OK;
    case MOE_OPT_GEMM:
      if (value < 0 || value > 2) return fail(h, MOE_EINVAL, "moe_set_option(gemm): value must be 0, 1 or 2");
      if (value == 2 && h->has_weights && !h->gemm_maps)
        return fail(h, MOE_EINVAL, "moe_set_option(gemm): this layer's shape is outside the GEMM path's rules");
      h->gemm_mode = value;
      return MOE_OK;
    case MOE_OPT_GEMM_TILE:
      if (value != 0 && value != 16 && value != 32 && value != 64 && value != 128)
        return fail(h, MOE_EINVAL, "moe_set_option(gemm tile): value must be 0, 16, 32, 64 or 128");
      h->gemm_tile = value;
      return MOE_OK;
    case MOE_OPT_HOST_IO:
      if (value < 0 || value > 2) return fail(h, MOE_EINVAL, "moe_set_option(host io): value must be 0, 1 or 2");
      h->host_io = value;
      return MOE_OK;
    case MOE_OPT_STREAM:
      if (value < 0 || value > 1) return fail(h, MOE_EINVAL, "moe_set_option(stream): value must be 0 or 1");
      h->stream_mode = value;
      return MOE_OK;
    case MOE_OPT_TRACE:
      if (value && h->trace == nullptr) {
        const size_t bytes = static_cast<size_t>(h->num_sms) * 16 * sizeof(unsigned long long);
        cudaError_t e = cudaMalloc(&h->trace, bytes);
        if (e == cudaSuccess) e = cudaMemset(h->trace, 0, bytes);
        if (e != cudaSuccess) return fail(h, MOE_ECUDA, "moe_set_option(trace): %s", cudaGetErrorString(e));
      } else if (!value && h->trace != nullptr) {
        cudaFree(h->trace);
        h->trace = nullptr;
      }
      return MOE_OK;
    default: return fail(h, MOE_EINVAL, "moe_set_option: unknown option %d", option);
  }
}

int moe_read_trace(void* handle, uint64_t* out, int32_t max_entries, int32_t* n, void* stream) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr || out == nullptr || n == nullptr) return MOE_EINVAL;
  if (h->trace == nullptr) return fail(h, MOE_EINVAL, "moe_read_trace: tracing is off");
  const int entries = std::min(max_entries, h->num_sms * 16);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(out, h->trace, sizeof(uint64_t) * entries, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(h, MOE_ECUDA, "moe_read_trace: %s", cudaGetErrorString(e));
  *n = h->num_sms;
  return MOE_OK;
}

int moe_last_launch_count(void* handle) {
  Handle* h = static_cast<Handle*>(handle);
  return h ? h->last_launches : 0;
}

int moe_profile_begin(void* handle, int32_t kernel_class, int32_t max_samples) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return MOE_EINVAL;
  if (kernel_class < MOE_K_ROUTE || kernel_class > MOE_K_DECODE_FUSED || max_samples < 1)
    return fail(h, MOE_EINVAL, "moe_profile_begin: bad kernel class or sample count");
  for (cudaEvent_t e : h->prof_ev) cudaEventDestroy(e);
  h->prof_ev.assign(2 * static_cast<size_t>(max_samples), nullptr);
  for (auto& e : h->prof_ev) {
    if (cudaEventCreate(&e) != cudaSuccess) return fail(h, MOE_ECUDA, "moe_profile_begin: cudaEventCreate failed");
  }
  h->prof_class = kernel_class;
  h->prof_max = max_samples;
  h->prof_n = 0;
  return MOE_OK;
}

int moe_profile_end(void* handle, float* total_ms, int32_t* samples) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr || total_ms == nullptr || samples == nullptr) return MOE_EINVAL;
  double sum = 0.0;
  for (int i = 0; i < h->prof_n; ++i) {
    cudaError_t e = cudaEventSynchronize(h->prof_ev[2 * i + 1]);
    if (e != cudaSuccess) return fail(h, MOE_ECUDA, "moe_profile_end: event sync: %s", cudaGetErrorString(e));
    float ms = 0.f;
    e = cudaEventElapsedTime(&ms, h->prof_ev[2 * i], h->prof_ev[2 * i + 1]);
    if (e != cudaSuccess) return fail(h, MOE_ECUDA, "moe_profile_end: elapsed time: %s", cudaGetErrorString(e));
    sum += ms;
  }
  *total_ms = static_cast<float>(sum);
  *samples = h->prof_n;
  h->prof_class = 0;
  for (cudaEvent_t e : h->prof_ev) cudaEventDestroy(e);
  h->prof_ev.clear();
  h->prof_n = h->prof_max = 0;
  return MOE_OK;
}

int moe_last_error(void* handle, char* buf, size_t len) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return MOE_EINVAL;
  fmt_err(buf, len, "%s", h->err.c_str());
  return MOE_OK;
}

void moe_destroy(void* handle) {
  Handle* h = static_cast<Handle*>(handle);
  if (h == nullptr) return;
  for (cudaEvent_t e : h->prof_ev) cudaEventDestroy(e);
  if (h->trace) cudaFree(h->trace);
  if (h->ws) cudaFree(h->ws);
  delete h;
}

}  // extern "C"
