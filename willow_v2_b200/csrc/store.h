// Host-side state behind the opaque wmoe_ctx / wmoe_store handles of include/wmoe.h.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>
#include <list>
#include <string>
#include <vector>

#include "kernels.cuh"

struct wmoe_ctx {
  int device = 0;
  int sm_count = 0;
  std::string error;
  uint64_t launches = 0;
  int* d_status = nullptr;  // device status word (see wmoe::DeviceStatus)
  void* scratch = nullptr;  // grown on demand
  size_t scratch_bytes = 0;
  void* stack_xn = nullptr;  // wmoe_prefill_stack: the normalised input rows passed from layer to layer
  size_t stack_xn_bytes = 0;
  // wmoe_batched_decode_experts: the host pointer and order arrays go to the GPU through a ring of pinned slots; a
  // slot is rewritten only after the event recorded behind the kernels that read it has completed
  static constexpr int kStageSlots = 16, kStageWords = 3 * 256;
  int64_t* stage_host = nullptr;
  int64_t* stage_dev = nullptr;
  cudaEvent_t stage_ev[kStageSlots] = {};
  bool stage_used[kStageSlots] = {};
  int stage_next = 0;
  int decode_ctas = 0;      // CTAs of the persistent decode kernel (all co-resident)
  bool use_decode_kernel = true;
  int prefill_threshold = 16;  // token count from which wmoe_moe_forward uses the tcgen05 grouped GEMMs
  float min_expert_weight = 0.f;  // willow's --min-expert-weight (wmoe_set_min_expert_weight); 0: off
  uint64_t* trace = nullptr;  // decode phase timestamps (device), or null
  size_t trace_entries = 0;
  // expert parallelism over the library's own NCCL communicator (wmoe_ep_init)
  void* nccl_comm = nullptr;  // ncclComm_t
  int ep_rank = 0, ep_world = 0;
  void* ep_buf = nullptr;     // received rows, pair lists, result rows and the expert stage's scratch (grown)
  size_t ep_buf_bytes = 0;
  cudaStream_t ep_stream = nullptr;     // the exchanges (overlapping the expert stage on the caller's stream)
  std::vector<cudaEvent_t> ep_events;   // ordering between the two streams
  int ep_chunks = 1;                    // token chunks per layer (wmoe_ep_set_chunks), the same on every rank
  int ep_timeout_ms = 30000;            // bound of every host wait on the communicator (wmoe_ep_set_timeout)
  bool ep_dead = false;                 // the communicator was aborted after a failure; wmoe_ep_finalize, then init
  // exchange windows: this rank's device buffer, written by the peers' copy engines through CUDA IPC
  bool ep_ipc = false;                  // windows mapped on every rank (else the rows go through NCCL send/recv)
  void* ep_win = nullptr;
  size_t ep_win_bytes = 0;              // the same on every rank
  std::vector<void*> ep_peer_win;       // [world]: every rank's window in this process (own one included)
  std::vector<cudaStream_t> ep_peer_streams;  // one per destination rank: copies to different ranks run together
  std::vector<cudaEvent_t> ep_peer_events;
  int* ep_flag = nullptr;               // one int: the all-reduce that serves as the exchanges' barrier
  void* ep_handles = nullptr;           // [world][sizeof(cudaIpcMemHandle_t)] device staging of the handle all-gather
  // pinned host copies of the all-gathered counts and handles: a device-to-host copy into pageable memory would
  // block the host behind the communicator's kernels, outside the bounded waits
  int32_t* ep_host_counts = nullptr;    // [kMaxRanks][kMaxRanks][kCountWords]
  void* ep_host_handles = nullptr;      // [kMaxRanks][sizeof(cudaIpcMemHandle_t)]
  // per-phase CUDA events of the last profile_calls multi-token MoE calls (opt-in): [profile_calls][kProfMarks]
  static constexpr int kProfMarks = 7;
  std::vector<cudaEvent_t> prof_events;
  int profile_calls = 0;
  uint64_t profile_seq = 0;  // calls recorded so far
};

struct wmoe_store {
  static constexpr int kRing = 256;
  wmoe_ctx* ctx = nullptr;
  int layers = 0, experts = 0, hidden = 0, ffn = 0;
  int expert_begin = 0, expert_end = 0;  // the experts of each layer this store holds (expert parallelism)
  bool owns(int e) const { return e >= expert_begin && e < expert_end; }
  size_t owned() const { return size_t(expert_end - expert_begin); }
  // index of an owned blob among the store's blobs (layer-major), e.g. into the pinned host copy
  size_t blob_index(int layer, int e) const { return size_t(layer) * owned() + size_t(e - expert_begin); }
  size_t gate_up_bytes = 0, down_bytes = 0, blob_bytes = 0, slot_stride = 0;
  // ggml type of each layer's down matrices (Q6_K, or Q4_K as some layers of llama.cpp's Q4_K_M files), and the
  // layer's blob size (gate_up then down; a Q4_K layer's blob is shorter than blob_bytes, the slot stride)
  std::vector<int> down_type;
  size_t layer_blob_bytes(int layer) const {
    return down_type[size_t(layer)] == 12 ? gate_up_bytes + size_t(hidden) * ffn / 256 * 144 : blob_bytes;
  }
  bool capped = false;
  int n_slots = 0;
  uint8_t* d_slab = nullptr;
  int32_t* d_slot_of = nullptr;   // [layers * experts] slot or -1
  std::vector<int32_t> slot_of;   // host mirror
  uint8_t* h_master = nullptr;    // pinned host copy of every blob (capped stores)
  std::vector<int64_t> slot_key;  // (layer * experts + expert) held by each slot, -1 free
  std::vector<uint64_t> slot_use; // sequence number of the last call that read the slot
  std::vector<uint64_t> slot_batch;       // side-stream copy batch that filled the slot (0: none)
  std::vector<char> slot_prefetched;      // filled by a prefetch whose layer has not run yet (not evictable)
  std::vector<char> slot_from_prefetch;   // filled by a prefetch and not yet read by a call (counter only)
  std::list<int> lru;             // slots, least recently used first
  std::vector<std::list<int>::iterator> lru_pos;
  std::vector<uint64_t> usage;    // [layers * experts] tokens routed to each expert (store.py:482-484)
  std::vector<char> hot;          // [layers * experts] the hot set: evicted only when no other slot can go
  cudaStream_t side = nullptr;
  cudaEvent_t ring[kRing] = {};       // compute-stream event of call seq at [seq % kRing]
  cudaEvent_t batch_ev[kRing] = {};   // side-stream event of copy batch b at [b % kRing]
  uint64_t seq = 0;
  uint64_t batches = 0, waited = 0;   // copy batches issued; the last one the compute stream has waited for
  uint64_t hits = 0, misses = 0, bytes_in = 0, evictions = 0, prefetched = 0, prefetch_used = 0;
};

int ctx_fail(wmoe_ctx* ctx, int code, const std::string& msg);
void ctx_count_launch(wmoe_ctx* ctx, int n = 1);

int store_create(wmoe_ctx* ctx, int layers, int experts, int expert_begin, int expert_end, int hidden, int ffn,
                 size_t cap_bytes, wmoe_store** out);
void store_destroy(wmoe_store* s);
int store_upload(wmoe_store* s, int layer, int expert, const void* host_src, cudaStream_t st);
int store_fill_synthetic(wmoe_store* s, uint64_t seed, int layer_begin, int layer_end, cudaStream_t st);
int store_prepare(wmoe_store* s, int layer, const int32_t* experts, int n, cudaStream_t st);
int store_prefetch(wmoe_store* s, int layer, const int32_t* experts, int n, cudaStream_t st);
int store_mark_used(wmoe_store* s, int layer, const int32_t* experts, int n, cudaStream_t st);
void store_record_usage(wmoe_store* s, int layer, const int32_t* experts, size_t n);
int store_choose_hot(wmoe_store* s, double share);
// the source of one layer: its down type comes with it
wmoe::ExpertSource store_source(const wmoe_store* s, int layer, const uint8_t* shared_gate_up,
                                const uint8_t* shared_down);
int store_set_down_type(wmoe_store* s, int layer, int ggml_type);
