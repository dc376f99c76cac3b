// ep_peer.h — the peer-memory exchange of an expert-parallel step: every
// rank's region (one device allocation of the same layout on every rank,
// mapped into the others through CUDA IPC) and the kernels that move token
// rows and expert outputs through those mappings.
//
// Region layout (byte offsets; identical on every rank of a group):
//   0           ready[kEpMaxWorld]  u64 epoch flags, slot s written by rank s
//   64          done[kEpMaxWorld]   u64 epoch flags, slot s written by rank s
//   256         T                   int32, tokens the owner published
//   off_slots   slots[max_tokens][top_k]        int32 expert slot of each pair (-1: bad id)
//   off_x       x[max_tokens][hidden]           bf16 token rows
//   off_y       y[max_tokens][top_k][hidden]    fp32 output row of each pair,
//                                               written by the pair's owner
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

namespace moe {

constexpr int kEpMaxWorld = 8;        // one NVLink / NVSwitch domain
constexpr int kEpFlagReady = 0;
constexpr int kEpFlagDone = 1;
constexpr size_t kEpOffHdr = 256;
constexpr size_t kEpOffSlots = 512;
constexpr int kEpStatusOverflow = 4;  // a rank published more tokens than the step's bound (clamped)

// What the kernels of one rank see of the group (passed by value).
struct PeerView {
  unsigned char* region[kEpMaxWorld];  // every rank's region, addressable from this device
  int32_t* status;                     // this rank's group status word (MOE_EP_STATUS_*)
  int rank, world;
  int max_tokens, top_k, hidden;
  int experts_per_rank, num_experts;
  size_t off_slots, off_x, off_y;
};

struct PeerGroup {
  PeerView v{};
  int device = 0;
  int num_sms = 148;
  unsigned char* region = nullptr;  // this rank's region (cudaMalloc)
  size_t region_bytes = 0;
  bool opened[kEpMaxWorld] = {};    // regions mapped through cudaIpcOpenMemHandle
  bool have[kEpMaxWorld] = {};      // regions known (own, opened or given)
  void* local = nullptr;            // this rank's private buffers (cudaMalloc)
  uint16_t* x_all = nullptr;        // [world][max_tokens][hidden] every rank's token rows
  int64_t* ids_all = nullptr;       // [world][max_tokens][top_k] local expert of each pair, -1 elsewhere
  unsigned long long* epoch = nullptr;  // [1] epoch of the step in flight
  unsigned int* counters = nullptr;     // [2] last-block counters of publish / scatter
  int phase = 0;                        // host-side order check: 0 publish next, 1 experts, 2 combine
  int published_tokens = 0;
  std::string err;
};

// Region layout for a group shape.
void ep_region_layout(int max_tokens, int top_k, int hidden, size_t& off_slots, size_t& off_x, size_t& off_y,
                      size_t& total);

// x and the slots of the routed ids into this rank's region, T into its
// header; the last block to finish advances the epoch and signals "ready" to
// every rank.
void launch_ep_peer_publish(const PeerView& v, const uint16_t* x, const int64_t* ids, int T,
                            const int32_t* slot_of_expert, unsigned long long* epoch, unsigned int* counter,
                            int num_sms, cudaStream_t st);
// Wait for every rank's "ready"; x_all [world][bound][hidden] / ids_all
// [world][bound][top_k] from every rank's region (bound: tokens per rank in
// this step, <= max_tokens).
void launch_ep_peer_collect(const PeerView& v, const unsigned long long* epoch, int bound, uint16_t* x_all,
                            int64_t* ids_all, int num_sms, cudaStream_t st);
// Output rows y[pos] of the pairs p with pair_pos[p] >= 0 into their token's
// rank's region; the last block signals "done" to every rank.
void launch_ep_peer_scatter(const PeerView& v, const int32_t* pair_pos, int P, int bound, const float* y,
                            const unsigned long long* epoch, unsigned int* counter, int num_sms, cudaStream_t st);
// Wait for every rank's "done"; out[t] = bf16(sum, experts ascending, of w * y[t][j]).
void launch_ep_peer_combine(const PeerView& v, const unsigned long long* epoch, const int64_t* ids,
                            const uint16_t* weights, int T, uint16_t* out, cudaStream_t st);

}  // namespace moe
