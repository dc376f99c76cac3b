/*
 * moe_b200.h — C ABI of the B200 (sm_100a) routed-expert MoE path.
 *
 * This library is the device backend for nano-ktrans's HybridMoE routed
 * experts.  Each entry point replaces one step of the reference's Python
 * path (paths are relative to the nano-ktrans project root):
 *
 *   moe_route            nano_ktrans/layers/hybrid_moe.py:3321-3329
 *                        (softmax -> top-k -> renormalise, or Mixtral's
 *                         top-k -> softmax)
 *   moe_experts_forward  nano_ktrans/kernels/offload_backend.py:40-52
 *                        ExpertOffloadBackend.submit_forward, as implemented
 *                        by CPUMoEBackend's GPTQ branch
 *                        nano_ktrans/kernels/cpu_moe.py:491-539 (per-expert
 *                        grouped W4A32 matvec quantized_ops.py:86-124,
 *                        SiLU(gate)*up cpu_moe.py:419-450, weighted
 *                        index_add_ combine cpu_moe.py:528-538)
 *   moe_forward          HybridMoE.forward with every expert offloaded
 *                        (hybrid_moe.py:3310-3570): route + experts
 *   moe_forward_host     moe_forward on host buffers: the step the reference's
 *                        CPU backend serves from host copies of the hidden
 *                        states (hybrid_moe.py:3373-3378, cpu_moe.py:491-539),
 *                        here copied to the device and back on the stream
 *   moe_router_logits    the router projection `self.gate(hidden_states)`
 *                        nano_ktrans/models/mixtral.py:127, :212 (bf16
 *                        nn.Linear, no bias)
 *   moe_forward_x        router projection + moe_forward: the MoE block of
 *                        models/mixtral.py:212-218 from hidden states
 *   moe_dequant_rows     GPTQLinearWeight.dequantize
 *                        nano_ktrans/kernels/weight_loader.py:57-69, for the
 *                        bit-exact dequantization check
 *   moe_create / moe_set_weights / moe_last_error / moe_destroy
 *                        the handle / int-status / caller-error-buffer
 *                        convention of the reference's native bridge
 *                        nano_ktrans/kernels/pim_native/host_quantized_bridge.c
 *                        (pim_quantized_init :233, load_weights :589,
 *                        set_error :157, shutdown :1306)
 *
 * Conventions
 *   - Every pointer argument named *_dev is device memory on the handle's
 *     device; nothing in this ABI takes a torch type.
 *   - Every call that takes a `stream` (a cudaStream_t passed as void*) only
 *     enqueues work on that stream and returns; results are stream-ordered.
 *   - Return value 0 = success; otherwise an MOE_E* code, and the message is
 *     available from moe_last_error().
 *   - bf16 tensors are passed as raw 16-bit patterns (uint16_t storage).
 *
 * Weight layout (device, borrowed by the handle, never copied):
 *   q[e][n][K*bits/8] uint8  — exactly the little-endian bytes of the
 *                              reference GPTQLinearWeight.qweight int32 words
 *                              [N, K*bits/32] (codes LSB-first along K,
 *                              offset-binary, zero point 2^(bits-1));
 *   s[e][n][SS] bf16         — per-group scales, SS = K/group rounded up to
 *                              a multiple of 8 (each scale row is 16-byte
 *                              aligned so it can be bulk-copied; the padding
 *                              is never read).
 *   gate/up: N = inter, K = hidden.  down: N = hidden, K = inter.
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_B200_ABI_VERSION 1

enum moe_status {
  MOE_OK = 0,
  MOE_EINVAL = 1,     /* bad argument or unsupported shape */
  MOE_ECUDA = 2,      /* a CUDA runtime call failed */
  MOE_ENOWEIGHTS = 3, /* moe_set_weights was not called */
  MOE_ERANGE = 4,     /* token count above the handle's max_tokens */
  MOE_EDEVICE = 5     /* a kernel recorded a bad input (see moe_read_status) */
};

/* Layer description.  group_size == 0 means one group per output channel
 * (group = K of each projection). */
typedef struct moe_layer_desc {
  int32_t num_experts;
  int32_t top_k;
  int32_t hidden_size;
  int32_t inter_size;
  int32_t bits;                /* 4 or 8 */
  int32_t group_size;          /* 0 (per-channel) or a multiple of 32 (W4) / 16 (W8) */
  int32_t router_use_softmax;  /* 1: Qwen softmax->topk; 0: Mixtral topk->softmax */
  int32_t normalize_topk_prob; /* renormalise top-k weights (softmax routing only) */
  int32_t max_tokens;          /* largest T any call will pass */
  int32_t shared_inter;        /* shared-expert intermediate size, 0 = none */
} moe_layer_desc;

/* Device pointers to the stacked expert weights (see layout above). */
typedef struct moe_weights {
  const void* gate_q_dev;
  const void* gate_s_dev;
  const void* up_q_dev;
  const void* up_s_dev;
  const void* down_q_dev;
  const void* down_s_dev;
  /* shared expert (only read when shared_inter > 0): same per-projection
   * layout with E = 1, plus the bf16 [hidden] sigmoid-gate vector */
  const void* shared_gate_q_dev;
  const void* shared_gate_s_dev;
  const void* shared_up_q_dev;
  const void* shared_up_s_dev;
  const void* shared_down_q_dev;
  const void* shared_down_s_dev;
  const void* shared_gate_vec_dev;
} moe_weights;

int moe_abi_version(void);

/* Create a handle on the current CUDA device; allocates the handle's
 * workspace (sized by desc->max_tokens). */
int moe_create(const moe_layer_desc* desc, void** handle, char* err, size_t err_len);

/* Register (borrow) the device weight pointers. */
int moe_set_weights(void* handle, const moe_weights* w, char* err, size_t err_len);

/* Routing: logits [T, E] bf16 -> topk_ids [T, k] int64, topk_weights [T, k]
 * bf16.  Ties are broken by (value desc, expert index asc). */
int moe_route(void* handle, const uint16_t* logits_dev, int32_t num_tokens,
              int64_t* topk_ids_dev, uint16_t* topk_weights_dev, void* stream);

/* Routed experts + weighted combine:
 *   out[t] = bf16( sum over slots j, expert e = ids[t][j] ascending, with
 *                  offload_mask[e] != 0 (or all when the mask is NULL):
 *                  w[t][j] * down(silu(gate(x[t])) * up(x[t])) )
 * accumulated in fp32.  When the layer has a shared expert and
 * `add_shared` is nonzero, sigmoid(x . g_s) * shared(x) is added before the
 * single bf16 rounding. */
int moe_experts_forward(void* handle, const uint16_t* x_dev, const int64_t* topk_ids_dev,
                        const uint16_t* topk_weights_dev, int32_t num_tokens,
                        const uint8_t* offload_mask_dev, int32_t add_shared,
                        uint16_t* out_dev, void* stream);

/* moe_route followed by moe_experts_forward (all experts, shared expert
 * added when present).  topk_ids_dev / topk_weights_dev may be NULL. */
int moe_forward(void* handle, const uint16_t* x_dev, const uint16_t* logits_dev,
                int32_t num_tokens, uint16_t* out_dev, int64_t* topk_ids_dev,
                uint16_t* topk_weights_dev, void* stream);

/* moe_forward with HOST buffers: x_host [T, H] and logits_host [T, E] bf16
 * are moved into the handle's workspace, the step runs, and the bf16 output
 * lands in out_host [T, H] — all enqueued on `stream`; the output is valid
 * once the stream reaches that point.  Page-locked buffers are read (and, with
 * MOE_OPT_HOST_IO 2, written) by the kernels through their mapped addresses;
 * pageable buffers go through copy-engine copies (synchronous ones). */
int moe_forward_host(void* handle, const uint16_t* x_host, const uint16_t* logits_host,
                     int32_t num_tokens, uint16_t* out_host, void* stream);

/* Router logits [T, E] bf16 = bf16(x [T, H] . router_w [E, H]^T), fp32
 * accumulation (the reference's bf16 nn.Linear gate).  x_dev and
 * router_w_dev 16-byte aligned; hidden_size a multiple of 32. */
int moe_router_logits(void* handle, const uint16_t* x_dev, const uint16_t* router_w_dev,
                      int32_t num_tokens, uint16_t* logits_dev, void* stream);

/* moe_router_logits followed by moe_forward.  logits_dev (may be NULL: the
 * handle's workspace is used) receives the logits, as the reference's MoE
 * block also returns them.  topk_ids_dev / topk_weights_dev may be NULL. */
int moe_forward_x(void* handle, const uint16_t* x_dev, const uint16_t* router_w_dev,
                  int32_t num_tokens, uint16_t* out_dev, int64_t* topk_ids_dev,
                  uint16_t* topk_weights_dev, uint16_t* logits_dev, void* stream);

/* ---- Expert parallelism (no counterpart in the reference, whose offload
 * backends are single-device) ----
 * The routed experts are split over `world` ranks; expert e lives on rank
 * slot_of_expert[e] / experts_per_rank as local expert
 * slot_of_expert[e] % experts_per_rank (slot_of_expert is a permutation of
 * 0..num_experts-1, world * experts_per_rank == num_experts).  The three
 * calls below are the device steps; the exchanges between them are two
 * all-to-alls the caller runs (NCCL all_to_all_single):
 *   1. moe_ep_dispatch on the token's rank (handle with the layer's
 *      num_experts / top_k): sorts the T*k (token, slot) pairs by slot
 *      (= by destination rank, then local expert; stable in pair index),
 *      writes send_rows [T*k][H] (bf16 token rows in that order),
 *      send_local [T*k] (int64 local expert of each row) and slot_counts
 *      [num_experts] (rows per slot; rows for rank r are the slots
 *      r*experts_per_rank .. (r+1)*experts_per_rank-1).  The pair order is
 *      kept in the handle for step 3.
 *   2. moe_rows_forward on the expert's rank (handle whose weights are that
 *      rank's experts_per_rank experts): y_rows[i] = fp32
 *      down(silu(gate(x_i)) * up(x_i)) of local expert row_expert[i], for the
 *      rows received from every rank, returned in the order received.
 *   3. moe_ep_combine on the token's rank, same handle as step 1, after the
 *      returned rows arrived in send order: out[t] = bf16(sum over slots j in
 *      ascending expert order of w[t][j] * rows[pos(t, j)]), accumulated in
 *      fp32 (nano_ktrans/kernels/cpu_moe.py:515-538 order).
 * Expert ids outside [0, num_experts) are flagged in the status word and
 * dropped, as in moe_experts_forward. */
int moe_ep_dispatch(void* handle, const uint16_t* x_dev, const int64_t* topk_ids_dev, int32_t num_tokens,
                    const int32_t* slot_of_expert_dev, int32_t experts_per_rank, int32_t world,
                    uint16_t* send_rows_dev, int64_t* send_local_dev, int32_t* slot_counts_dev, void* stream);
/* num_rows <= max_tokens * top_k of the handle. */
int moe_rows_forward(void* handle, const uint16_t* x_rows_dev, const int64_t* row_expert_dev, int32_t num_rows,
                     float* y_rows_dev, void* stream);
int moe_ep_combine(void* handle, const int64_t* topk_ids_dev, const uint16_t* topk_weights_dev, int32_t num_tokens,
                   const float* returned_rows_dev, uint16_t* out_dev, void* stream);

/* ---- Expert parallelism over peer memory (no counterpart in the reference) ----
 * The same split of the routed experts over `world` ranks (one process per
 * GPU, every GPU reachable from every other over NVLink / NVSwitch), with
 * the exchanges done by this library's kernels through each rank's
 * "region": one device allocation of the same layout on every rank, opened
 * by the others through CUDA IPC.  Nothing in a step reads device memory
 * back to the host, so a whole multi-layer step can be captured in a CUDA
 * graph; ranks hand over with epoch flags in the regions (bounded waits:
 * a wait that runs out sets MOE_EP_STATUS_TIMEOUT in the group's status word
 * and every later wait of the group returns at once until the word is read).
 *
 * Region of a rank: flags, its published token count, slots [max_tokens][top_k]
 * (int32 expert slot of each routed pair), x [max_tokens][hidden] (bf16 token
 * rows) and y [max_tokens][top_k][hidden] (fp32 expert output of each pair,
 * written by the pair's owner).
 *
 * One step on every rank, in this order on one stream:
 *   1. moe_ep_peer_publish: copies x and the slots of the routed ids
 *      (slot_of_expert as in moe_ep_dispatch) into the region; signals
 *      "ready" to every rank.
 *   2. moe_ep_peer_experts (expert_handle: the rank's experts_per_rank experts,
 *      top_k = the layer's, max_tokens >= world * group max_tokens): waits for
 *      every rank's "ready"; gathers every rank's token rows, selects the
 *      pairs whose slot this rank owns, runs them through its experts and
 *      stores each fp32 output row into the token's rank's y at (token, slot
 *      index); signals "done" to every rank.  tokens_per_rank (0: the group's
 *      max_tokens) bounds every rank's token count in this step and sizes the
 *      work (a rank above it is clamped and MOE_EP_STATUS_OVERFLOW set);
 *      pairs_hint (the pairs this rank expects, e.g. its own T * top_k) only
 *      picks the kernels.
 *   3. moe_ep_peer_combine: waits for every rank's "done"; out[t] =
 *      bf16(sum over slots j in ascending expert order of w[t][j] * y[t][j]),
 *      fp32, the single-GPU combine's arithmetic and order.
 * A pair's output does not depend on which other pairs share its kernels, so
 * the result is bit-identical to moe_experts_forward on one GPU whenever the
 * expert kernels chosen are the same.
 * Lifetime: a rank may destroy its group only after every rank has finished
 * its last step (synchronise, then a host barrier). */
#define MOE_EP_STATUS_BAD_ID 1
#define MOE_EP_STATUS_TIMEOUT 2
#define MOE_EP_STATUS_OVERFLOW 4
#define MOE_EP_IPC_HANDLE_BYTES 64
int moe_ep_group_create(int32_t rank, int32_t world, int32_t max_tokens, int32_t top_k, int32_t hidden_size,
                        int32_t num_experts, void** group, char* err, size_t err_len);
/* Unmap the other ranks' regions (every rank first finishes its last step and
 * meets the others at a host barrier), then free this rank's region once every
 * rank has unmapped it (a second barrier). */
int moe_ep_group_close_peers(void* group);
int moe_ep_group_destroy(void* group);
/* CUDA IPC handle of this rank's region (MOE_EP_IPC_HANDLE_BYTES bytes). */
int moe_ep_group_ipc_handle(void* group, void* handle_out);
/* Open `peer`'s region from its IPC handle (peer != own rank). */
int moe_ep_group_open_peer(void* group, int32_t peer, const void* ipc_handle);
/* Emulated ranks in one process on one device: this rank's region pointer,
 * and another group's region given directly. */
int moe_ep_group_region(void* group, void** region_dev);
int moe_ep_group_set_peer(void* group, int32_t peer, void* region_dev);
int moe_ep_peer_publish(void* group, const uint16_t* x_dev, const int64_t* topk_ids_dev, int32_t num_tokens,
                        const int32_t* slot_of_expert_dev, void* stream);
int moe_ep_peer_experts(void* group, void* expert_handle, int32_t tokens_per_rank, int32_t pairs_hint,
                        void* stream);
int moe_ep_peer_combine(void* group, const int64_t* topk_ids_dev, const uint16_t* topk_weights_dev,
                        int32_t num_tokens, uint16_t* out_dev, void* stream);
/* Copy the group's status word to *status and clear it (synchronises `stream`). */
int moe_ep_group_read_status(void* group, int32_t* status, void* stream);
/* Last error message of the group's calls, as moe_last_error. */
int moe_ep_group_last_error(void* group, char* buf, size_t len);

/* Dequantize rows [row0, row0+nrows) of projection `proj` (0 gate, 1 up,
 * 2 down, 3..5 shared gate/up/down) of expert `expert` into fp32 [nrows, K],
 * with the same unpack code the matvec kernels use. */
int moe_dequant_rows(void* handle, int32_t proj, int32_t expert, int32_t row0, int32_t nrows,
                     float* out_dev, void* stream);

/* Copy the device status word to *status (synchronises `stream`).  Nonzero
 * means a kernel saw an expert id outside [0, E) since the last reset; the
 * word is cleared by this call. */
int moe_read_status(void* handle, int32_t* status, void* stream);

/* Kernels launched by the last moe_experts_forward / moe_forward call. */
int moe_last_launch_count(void* handle);

/* Kernel classes for moe_profile_begin. */
enum moe_kernel_class {
  MOE_K_ROUTE = 1,
  MOE_K_PERMUTE = 2,
  MOE_K_GATEUP = 3,
  MOE_K_DOWN = 4,
  MOE_K_COMBINE = 5,
  MOE_K_DECODE_FUSED = 6 /* single-launch decode step (route + experts + combine) */
};

/* Handle options for moe_set_option. */
enum moe_option {
  /* 1 (default): batches small enough run as one cooperative launch (a
   * single-token kernel for T == 1 with W4 weights, else the multi-token
   * kernel); 2: the multi-token kernel also for T == 1; 0: always use the
   * multi-kernel path. */
  MOE_OPT_DECODE_FUSED = 1,
  /* 1: the single-launch decode kernels record per-CTA phase stamps
   * (allocates num_SMs * 16 * 8 bytes); read them with moe_read_trace. */
  MOE_OPT_TRACE = 2,
  /* Expert projections of the multi-kernel path: 0 = no GEMM (streaming or
   * matvec kernels, see MOE_OPT_STREAM); 1 (default) = tensor-core grouped
   * GEMM once T * top_k >= 16 * num_experts where the streaming kernels apply
   * (>= 4 * num_experts elsewhere);
   * 2 = grouped GEMM for every batch the single-launch kernel does not take.
   * The GEMM path needs inter and hidden multiples of 128 and, for W4,
   * group_size a multiple of 64 (W8: per-channel); value 2 on another shape
   * is refused. */
  MOE_OPT_GEMM = 3,
  /* Token-tile width of the grouped GEMM: 0 (default) = the smallest of
   * 16/32/64/128 covering the mean tokens per routed expert; or one of those
   * four values. */
  MOE_OPT_GEMM_TILE = 4,
  /* Expert projections of batches the single-launch kernels and the GEMM do
   * not take: 1 (default) = weight-streaming tensor-core kernels (each active
   * expert's rows read once per call, applied to up to 8 of its tokens at a
   * time) when the layer is W4 with inter, hidden and group_size multiples of
   * 128; 0 = the CUDA-core matvec kernels. */
  MOE_OPT_STREAM = 5,
  /* How moe_forward_host moves page-locked host buffers: 0 = copy-engine
   * copies in and out; 1 = a kernel reads the inputs from mapped host memory,
   * the output is copied back; 2 (default) = as 1, and the step's last kernel
   * stores the output straight into host memory.  Pageable buffers always take
   * the copy engine (each call asks the driver which kind every pointer is). */
  MOE_OPT_HOST_IO = 6
};

/* Copy the phase stamps of the last traced single-launch decode step, 16 per
 * CTA: out[c * 16 + i].  Single-token kernel (T == 1): slot 0 = %globaltimer
 * (ns) at CTA entry, slots 1-12 = SM clock cycles since entry at: inputs
 * landed, routing done, chunk table built, prologue done, copies queued, own
 * gate/up rows done, h written, grid barrier passed, h staged, down blocks
 * landed, down tiles done, exit.  Multi-token kernel: slots 0-5 =
 * %globaltimer (ns) at entry, routing done, gate/up done, grid barrier
 * passed, intermediate staged, exit.  *n receives the CTA count.
 * Synchronises `stream`.  (No counterpart in the reference: tracing support.) */
int moe_read_trace(void* handle, uint64_t* out, int32_t max_entries, int32_t* n, void* stream);

/* Set a handle option (no counterpart in the reference: selects between two
 * device implementations of the same step). */
int moe_set_option(void* handle, int32_t option, int32_t value);

/* Bracket the launch of one kernel class with CUDA events on the launching
 * stream in each of the next `max_samples` forward calls (no counterpart in
 * the reference: measurement support, allocates the events). */
int moe_profile_begin(void* handle, int32_t kernel_class, int32_t max_samples);

/* Wait for the recorded events and return the summed kernel time and the
 * number of bracketed launches; stops profiling. */
int moe_profile_end(void* handle, float* total_ms, int32_t* samples);

int moe_last_error(void* handle, char* buf, size_t len);
void moe_destroy(void* handle);

/* Single-launch decode step (route + experts + combine, as moe_forward)
 * that allocates nothing: no handle, no cudaMalloc/cudaFree.  For callers
 * that cannot allocate device memory when they run a layer (a memory budget
 * fixed up front, an embedding that only hands out pre-registered buffers, a
 * caller that must not enter the allocator while other work is in flight).
 * No counterpart in the reference.
 *   - The caller passes the layer description, the device weight pointers
 *     (layout as for moe_set_weights), x [T, H] and logits [T, E] (bf16), and
 *     the outputs out [T, H] (bf16), topk_ids [T, k] (int64), topk_weights
 *     [T, k] (bf16).  status_dev receives the device status bits (see
 *     moe_read_status): pass a zeroed int32, the bits accumulate until the
 *     caller clears them; NULL discards them (timeouts and bad ids then go
 *     unreported).
 *   - Scratch is one file-scope device array per GPU that loads the library:
 *     T * top_k * inter_size must be <= 24576 floats (96 KiB), and the batch
 *     must fit the single-launch kernel (T <= 4, T * top_k <= 32, E <= 256);
 *     larger calls return MOE_ERANGE with a message and launch nothing.
 *   - Every call on a device shares that array: calls whose kernels overlap
 *     on the GPU race and give wrong results; serialise them.
 *   - The first call on a device looks up the array's address
 *     (cudaGetSymbolAddress); make it outside any stream capture.  The
 *     address is kept for the life of the process, so the entry point must
 *     not be used after cudaDeviceReset.
 * err/err_len receive a message on failure. */
int moe_decode_noalloc(const moe_layer_desc* desc, const moe_weights* w, const uint16_t* x_dev,
                       const uint16_t* logits_dev, int32_t num_tokens, uint16_t* out_dev,
                       int64_t* topk_ids_dev, uint16_t* topk_weights_dev, int32_t* status_dev,
                       void* stream, char* err, size_t err_len);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H */
