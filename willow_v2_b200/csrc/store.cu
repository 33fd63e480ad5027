// The HBM expert store (replaces gguf/store.py ExpertStore and gguf/mps_shared.{py,mm}).
//
// willow reads experts from an SSD pack into slab slots on a thread pool, keeping an LRU plus a usage-driven hot
// set (store.py:41-536), with slabs in memory the GPU shares (mps_shared.mm:10-20). On a B200 the whole
// 40-layer store (~21 GB) fits in HBM, so the default is every (layer, expert) blob resident in one slab and an
// identity slot table. With a cap, the slab holds cap/blob slots; every blob lives in pinned host memory and a
// miss is one cudaMemcpyAsync on a side stream, ordered against the compute stream by events, least recently
// used slot evicted first, slots of the usage-driven hot set only when nothing else can go. A prefetch starts the
// copies of a coming layer without making the compute stream wait; the call that uses them waits for that batch
// of copies only. Kernels find a blob through the device slot table [layers, experts] (-1: absent).
#include <algorithm>
#include <cstring>
#include <list>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"
#include "store.h"
#include "synth.cuh"

namespace wmoe {

// ---------------------------------------------------------------- synthetic weights on the device

// One thread per super-block. Blob i of the list gets (layer, expert) = layer_expert[2i], [2i+1].
__global__ void __launch_bounds__(256) fill_synthetic_kernel(uint8_t* __restrict__ dst, uint64_t seed,
                                                             const int32_t* __restrict__ layer_expert, int n,
                                                             uint64_t stride, int hidden, int ffn) {
  const uint64_t q4_blocks = uint64_t(2 * ffn) * hidden / QK, q6_blocks = uint64_t(hidden) * ffn / QK;
  const uint64_t per_blob = q4_blocks + q6_blocks;
  const uint64_t gid = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x;
  if (gid >= per_blob * uint64_t(n)) return;
  const int i = int(gid / per_blob);
  const uint64_t b = gid % per_blob;
  const uint64_t layer = uint64_t(layer_expert[2 * i]), expert = uint64_t(layer_expert[2 * i + 1]);
  uint8_t* blob = dst + uint64_t(i) * stride;
  if (b < q4_blocks) {
    const uint64_t key = synth::tensor_key(seed, layer, expert, synth::kTensorGateUp);
    uint64_t w[18];
#pragma unroll
    for (int k = 0; k < 18; ++k) w[k] = synth::word(key, b, k);
    const uint64_t d = synth::scale_f16(synth::word(key, b, 18)), dmin = synth::scale_f16(synth::word(key, b, 19));
    w[0] = (w[0] & ~0xFFFFFFFFull) | d | (dmin << 16);
    uint4* o = reinterpret_cast<uint4*>(blob + b * Q4K_BYTES);
#pragma unroll
    for (int k = 0; k < 9; ++k)
      o[k] = make_uint4(uint32_t(w[2 * k]), uint32_t(w[2 * k] >> 32), uint32_t(w[2 * k + 1]),
                        uint32_t(w[2 * k + 1] >> 32));
  } else {
    const uint64_t bb = b - q4_blocks;
    const uint64_t key = synth::tensor_key(seed, layer, expert, synth::kTensorDown);
    uint16_t* o = reinterpret_cast<uint16_t*>(blob + uint64_t(2 * ffn) * hidden / QK * Q4K_BYTES + bb * Q6K_BYTES);
    for (int k = 0; k < 24; ++k) {  // ql, qh: bytes 0..191
      const uint64_t w = synth::word(key, bb, k);
#pragma unroll
      for (int j = 0; j < 4; ++j) o[4 * k + j] = uint16_t(w >> (16 * j));
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {  // 16 int8 scales in [-32, 31]: bytes 192..207
      const uint64_t w = synth::word(key, bb, 24 + k);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t b0 = uint32_t((w >> (16 * j)) & 63) - 32u, b1 = uint32_t((w >> (16 * j + 8)) & 63) - 32u;
        o[96 + 4 * k + j] = uint16_t((b0 & 0xFF) | ((b1 & 0xFF) << 8));
      }
    }
    o[104] = synth::scale_f16(synth::word(key, bb, 26));
  }
}

cudaError_t fill_synthetic(uint8_t* dst, uint64_t seed, const int32_t* layer_expert, int n, uint64_t stride,
                           int hidden, int ffn, cudaStream_t st) {
  const uint64_t per_blob = uint64_t(2 * ffn) * hidden / QK + uint64_t(hidden) * ffn / QK;
  const uint64_t threads = per_blob * uint64_t(n);
  if (threads == 0) return cudaSuccess;
  fill_synthetic_kernel<<<unsigned((threads + 255) / 256), 256, 0, st>>>(dst, seed, layer_expert, n, stride, hidden,
                                                                         ffn);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- slot table updates

struct SlotUpdates {
  int n;
  int32_t index[64];
  int32_t value[64];
};

__global__ void set_slots_kernel(int32_t* table, SlotUpdates u) {
  const int i = threadIdx.x;
  if (i < u.n) table[u.index[i]] = u.value[i];
}

}  // namespace wmoe

using namespace wmoe;

static int store_fail(wmoe_store* s, int code, const std::string& msg) { return ctx_fail(s->ctx, code, msg); }

static int flush_updates(wmoe_store* s, SlotUpdates& u, cudaStream_t st) {
  if (u.n == 0) return 0;
  set_slots_kernel<<<1, 64, 0, st>>>(s->d_slot_of, u);
  ctx_count_launch(s->ctx);
  u.n = 0;
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : store_fail(s, -2, std::string("slot table update: ") + cudaGetErrorString(e));
}

static void push_update(wmoe_store* s, SlotUpdates& u, int index, int value, cudaStream_t st) {
  if (u.n == 64) flush_updates(s, u, st);
  u.index[u.n] = index;
  u.value[u.n] = value;
  ++u.n;
}

int store_create(wmoe_ctx* ctx, int layers, int experts, int expert_begin, int expert_end, int hidden, int ffn,
                 size_t cap_bytes, wmoe_store** out) {
  auto* s = new wmoe_store();
  s->ctx = ctx;
  s->layers = layers;
  s->experts = experts;
  s->expert_begin = expert_begin;
  s->expert_end = expert_end;
  s->hidden = hidden;
  s->ffn = ffn;
  s->gate_up_bytes = size_t(2 * ffn) * hidden / QK * Q4K_BYTES;
  s->down_bytes = size_t(hidden) * ffn / QK * Q6K_BYTES;
  s->blob_bytes = s->gate_up_bytes + s->down_bytes;
  s->slot_stride = (s->blob_bytes + 255) / 256 * 256;
  const size_t total = size_t(layers) * experts;          // slot table entries (every expert id)
  const size_t held = size_t(layers) * s->owned();         // blobs this store holds
  s->capped = cap_bytes != 0 && cap_bytes < held * s->slot_stride;
  s->n_slots = s->capped ? int(std::min(cap_bytes / s->slot_stride, held)) : int(held);
  if (s->n_slots <= 0) {
    delete s;
    return ctx_fail(ctx, -3, "expert store cap is smaller than one expert");
  }
  cudaError_t e = cudaMalloc(&s->d_slab, size_t(s->n_slots) * s->slot_stride);
  if (e == cudaSuccess) e = cudaMalloc(&s->d_slot_of, total * sizeof(int32_t));
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s->side, cudaStreamNonBlocking);
  for (int i = 0; i < wmoe_store::kRing && e == cudaSuccess; ++i) {
    e = cudaEventCreateWithFlags(&s->ring[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->batch_ev[i], cudaEventDisableTiming);
  }
  s->slot_of.assign(total, -1);
  s->usage.assign(total, 0);
  s->down_type.assign(size_t(layers), kGgmlQ6K);
  if (e == cudaSuccess && s->capped) e = cudaHostAlloc(&s->h_master, held * s->blob_bytes, cudaHostAllocDefault);
  if (e != cudaSuccess) {
    const std::string msg = std::string("expert store allocation: ") + cudaGetErrorString(e);
    store_destroy(s);
    return ctx_fail(ctx, -2, msg);
  }
  if (!s->capped) {
    for (int l = 0; l < layers; ++l)
      for (int x = expert_begin; x < expert_end; ++x) s->slot_of[size_t(l) * experts + x] = int32_t(s->blob_index(l, x));
  } else {
    s->slot_key.assign(size_t(s->n_slots), -1);
    s->slot_use.assign(size_t(s->n_slots), 0);
    s->slot_batch.assign(size_t(s->n_slots), 0);
    s->slot_prefetched.assign(size_t(s->n_slots), 0);
    s->slot_from_prefetch.assign(size_t(s->n_slots), 0);
    s->hot.assign(total, 0);
    s->lru_pos.resize(size_t(s->n_slots));
    for (int i = 0; i < s->n_slots; ++i) s->lru_pos[size_t(i)] = s->lru.insert(s->lru.end(), i);
  }
  e = cudaMemcpy(s->d_slot_of, s->slot_of.data(), total * sizeof(int32_t), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    store_destroy(s);
    return ctx_fail(ctx, -2, std::string("slot table upload: ") + cudaGetErrorString(e));
  }
  *out = s;
  return 0;
}

void store_destroy(wmoe_store* s) {
  if (!s) return;
  if (s->side) cudaStreamSynchronize(s->side);
  cudaFree(s->d_slab);
  cudaFree(s->d_slot_of);
  if (s->h_master) cudaFreeHost(s->h_master);
  for (auto& ev : s->ring)
    if (ev) cudaEventDestroy(ev);
  for (auto& ev : s->batch_ev)
    if (ev) cudaEventDestroy(ev);
  if (s->side) cudaStreamDestroy(s->side);
  delete s;
}

int store_upload(wmoe_store* s, int layer, int expert, const void* host_src, cudaStream_t st) {
  if (layer < 0 || layer >= s->layers || expert < 0 || expert >= s->experts || !host_src)
    return store_fail(s, -1, "wmoe_store_upload: bad layer/expert/source");
  if (!s->owns(expert)) return store_fail(s, -1, "wmoe_store_upload: expert outside the store's range");
  const size_t key = size_t(layer) * s->experts + expert;
  cudaError_t e;
  if (s->capped) {
    // the host copy is the master; drop any resident copy so the next prepare reloads it
    e = cudaStreamSynchronize(st);
    if (e == cudaSuccess) {
      memcpy(s->h_master + s->blob_index(layer, expert) * s->blob_bytes, host_src, s->layer_blob_bytes(layer));
      const int slot = s->slot_of[key];
      if (slot >= 0) {
        SlotUpdates u{};
        push_update(s, u, int(key), -1, st);
        if (flush_updates(s, u, st)) return -2;
        s->slot_of[key] = -1;
        s->slot_key[size_t(slot)] = -1;
      }
    }
  } else {
    e = cudaMemcpyAsync(s->d_slab + size_t(s->slot_of[key]) * s->slot_stride, host_src, s->layer_blob_bytes(layer),
                        cudaMemcpyHostToDevice, st);
  }
  if (e != cudaSuccess) return store_fail(s, -6, std::string("wmoe_store_upload: ") + cudaGetErrorString(e));
  return 0;
}

int store_fill_synthetic(wmoe_store* s, uint64_t seed, int layer_begin, int layer_end, cudaStream_t st) {
  if (layer_begin < 0 || layer_end > s->layers || layer_begin > layer_end)
    return store_fail(s, -1, "wmoe_store_fill_synthetic: bad layer range");
  for (int l = layer_begin; l < layer_end; ++l)
    if (s->down_type[size_t(l)] != kGgmlQ6K)
      return store_fail(s, -1, "wmoe_store_fill_synthetic: the generator makes Q6_K down matrices only");
  const int E = s->experts, n = int(s->owned());
  std::vector<int32_t> le(size_t(2) * n);
  int32_t* d_le = nullptr;
  uint8_t* staging = nullptr;
  cudaError_t e = cudaMalloc(&d_le, le.size() * sizeof(int32_t));
  if (e == cudaSuccess && s->capped) e = cudaMalloc(&staging, size_t(n) * s->blob_bytes);
  for (int layer = layer_begin; layer < layer_end && e == cudaSuccess; ++layer) {
    for (int i = 0; i < n; ++i) {
      le[size_t(2) * i] = layer;
      le[size_t(2) * i + 1] = s->expert_begin + i;
    }
    e = cudaMemcpyAsync(d_le, le.data(), le.size() * sizeof(int32_t), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) break;
    if (!s->capped) {
      // uncapped slots hold the owned experts layer-major in id order: one launch covers the layer
      e = fill_synthetic(s->d_slab + s->blob_index(layer, s->expert_begin) * s->slot_stride, seed, d_le, n,
                         s->slot_stride, s->hidden, s->ffn, st);
      ctx_count_launch(s->ctx);
    } else {
      e = fill_synthetic(staging, seed, d_le, n, s->blob_bytes, s->hidden, s->ffn, st);
      ctx_count_launch(s->ctx);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(s->h_master + s->blob_index(layer, s->expert_begin) * s->blob_bytes, staging,
                            size_t(n) * s->blob_bytes, cudaMemcpyDeviceToHost, st);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);  // le is reused for the next layer
  }
  if (e == cudaSuccess && s->capped) {
    // every resident copy is stale now
    SlotUpdates u{};
    for (int slot = 0; slot < s->n_slots; ++slot) {
      const int64_t key = s->slot_key[size_t(slot)];
      if (key >= 0 && key / E >= layer_begin && key / E < layer_end) {
        push_update(s, u, int(key), -1, st);
        s->slot_of[size_t(key)] = -1;
        s->slot_key[size_t(slot)] = -1;
      }
    }
    flush_updates(s, u, st);
    e = cudaStreamSynchronize(st);
  }
  cudaFree(d_le);
  cudaFree(staging);
  if (e != cudaSuccess)
    return store_fail(s, -2, std::string("wmoe_store_fill_synthetic: ") + cudaGetErrorString(e));
  return 0;
}

// Copies the listed missing experts of a layer into slots on the side stream, as one batch with its own event
// (returned in *batch). Victims are the least recently used slots that this request does not need and that hold
// no pending prefetch, slots of hot experts only when no other slot can go (store.py:348). Before overwriting a
// slot, the side stream waits for the compute work that last read it; the slot table entries are published on
// the compute stream.
static int copy_in(wmoe_store* s, int layer, const std::vector<int>& misses, std::vector<char>& needed, bool prefetch,
                   cudaStream_t st, uint64_t* batch) {
  const size_t E = size_t(s->experts);
  std::vector<int> victims;
  victims.reserve(misses.size());
  for (int pass = 0; pass < 2 && victims.size() < misses.size(); ++pass) {
    for (auto it = s->lru.begin(); it != s->lru.end() && victims.size() < misses.size(); ++it) {
      const int slot = *it;
      if (needed[size_t(slot)] || s->slot_prefetched[size_t(slot)]) continue;
      const int64_t key = s->slot_key[size_t(slot)];
      const bool is_hot = key >= 0 && s->hot[size_t(key)];
      if (is_hot != (pass == 1)) continue;
      needed[size_t(slot)] = 1;
      victims.push_back(slot);
    }
  }
  if (victims.size() < misses.size()) return store_fail(s, -3, "expert store: no evictable slot");
  const uint64_t b = ++s->batches;
  cudaError_t e = cudaSuccess;
  SlotUpdates u{};
  for (size_t i = 0; i < misses.size() && e == cudaSuccess; ++i) {
    const int slot = victims[i], x = misses[i];
    const int64_t old = s->slot_key[size_t(slot)];
    if (old >= 0) {
      ++s->evictions;
      s->slot_of[size_t(old)] = -1;
      push_update(s, u, int(old), -1, st);
    }
    const uint64_t last = s->slot_use[size_t(slot)];
    // the compute event of the call that last read the slot orders the overwrite. When the ring has wrapped past
    // that call, its entry holds a later call's event: a context issues its calls on one compute stream (it is
    // single-stream), so that later call's completion implies the earlier one's, and waiting on it is still safe.
    if (last > 0) e = cudaStreamWaitEvent(s->side, s->ring[last % wmoe_store::kRing], 0);
    if (e != cudaSuccess) break;
    const size_t key = size_t(layer) * E + size_t(x);
    e = cudaMemcpyAsync(s->d_slab + size_t(slot) * s->slot_stride, s->h_master + s->blob_index(layer, x) * s->blob_bytes,
                        s->blob_bytes, cudaMemcpyHostToDevice, s->side);
    if (e != cudaSuccess) break;
    ++s->misses;
    s->bytes_in += s->blob_bytes;
    if (prefetch) ++s->prefetched;
    s->slot_key[size_t(slot)] = int64_t(key);
    s->slot_of[key] = slot;
    s->slot_batch[size_t(slot)] = b;
    s->slot_prefetched[size_t(slot)] = prefetch ? 1 : 0;
    s->slot_from_prefetch[size_t(slot)] = prefetch ? 1 : 0;
    push_update(s, u, int(key), slot, st);
    s->lru.splice(s->lru.end(), s->lru, s->lru_pos[size_t(slot)]);
  }
  if (e == cudaSuccess) e = cudaEventRecord(s->batch_ev[b % wmoe_store::kRing], s->side);
  if (e != cudaSuccess) return store_fail(s, -6, std::string("expert copy: ") + cudaGetErrorString(e));
  *batch = b;
  return flush_updates(s, u, st);
}

static int check_request(wmoe_store* s, int layer, const int32_t* experts, int n, const char* fn) {
  if (layer < 0 || layer >= s->layers || n < 0) return store_fail(s, -1, std::string(fn) + ": bad layer");
  for (int i = 0; i < n; ++i) {
    if (experts[i] < 0 || experts[i] >= s->experts) return store_fail(s, -1, std::string(fn) + ": bad expert id");
    if (!s->owns(experts[i])) return store_fail(s, -1, std::string(fn) + ": expert outside the store's range");
  }
  return 0;
}

int store_prepare(wmoe_store* s, int layer, const int32_t* experts, int n, cudaStream_t st) {
  if (int rc = check_request(s, layer, experts, n, "wmoe_store_prepare")) return rc;
  if (!s->capped) {
    s->hits += uint64_t(n);
    return 0;
  }
  if (n > s->n_slots) return store_fail(s, -3, "expert store cap holds fewer experts than one layer call needs");
  const size_t E = size_t(s->experts);
  // this layer's prefetches that the call does not use become ordinary cached slots (store.py:221-232)
  for (int slot = 0; slot < s->n_slots; ++slot)
    if (s->slot_prefetched[size_t(slot)] && s->slot_key[size_t(slot)] / int64_t(E) == layer)
      s->slot_prefetched[size_t(slot)] = 0;
  std::vector<int> wanted(experts, experts + n);
  std::sort(wanted.begin(), wanted.end());
  wanted.erase(std::unique(wanted.begin(), wanted.end()), wanted.end());
  std::vector<char> needed(size_t(s->n_slots), 0);
  std::vector<int> misses;
  uint64_t wait_for = 0;  // the latest copy batch this call's slots came from
  for (int x : wanted) {
    const size_t key = size_t(layer) * E + size_t(x);
    const int slot = s->slot_of[key];
    if (slot >= 0) {
      ++s->hits;
      needed[size_t(slot)] = 1;
      if (s->slot_from_prefetch[size_t(slot)]) {
        ++s->prefetch_used;
        s->slot_from_prefetch[size_t(slot)] = 0;
      }
      wait_for = std::max(wait_for, s->slot_batch[size_t(slot)]);
      s->lru.splice(s->lru.end(), s->lru, s->lru_pos[size_t(slot)]);  // most recently used at the back
    } else {
      misses.push_back(x);
    }
  }
  if (!misses.empty()) {
    uint64_t b = 0;
    if (int rc = copy_in(s, layer, misses, needed, false, st, &b)) return rc;
    wait_for = b;
  }
  // the compute stream waits for the copies (side-stream batches complete in order); once is enough
  if (wait_for > s->waited) {
    const cudaError_t e = cudaStreamWaitEvent(st, s->batch_ev[wait_for % wmoe_store::kRing], 0);
    if (e != cudaSuccess) return store_fail(s, -2, std::string("expert copy ordering: ") + cudaGetErrorString(e));
    s->waited = wait_for;
  }
  return 0;
}

int store_prefetch(wmoe_store* s, int layer, const int32_t* experts, int n, cudaStream_t st) {
  if (int rc = check_request(s, layer, experts, n, "wmoe_store_prefetch")) return rc;
  if (!s->capped) return 0;
  const size_t E = size_t(s->experts);
  // in the order given (the first ones get the room when it runs out), each expert once
  std::vector<int> wanted;
  std::vector<char> seen(E, 0);
  for (int i = 0; i < n; ++i)
    if (!seen[size_t(experts[i])]) {
      seen[size_t(experts[i])] = 1;
      wanted.push_back(experts[i]);
    }
  std::vector<char> needed(size_t(s->n_slots), 0);
  std::vector<int> misses;
  for (int x : wanted) {
    const int slot = s->slot_of[size_t(layer) * E + size_t(x)];
    if (slot >= 0)
      needed[size_t(slot)] = 1;
    else
      misses.push_back(x);
  }
  // a prefetch never takes the slots the last call read or pending prefetches: it fills at most the slots left
  for (int slot = 0; slot < s->n_slots; ++slot)
    if (s->seq > 0 && s->slot_use[size_t(slot)] == s->seq) needed[size_t(slot)] = 1;
  size_t room = 0;
  for (int slot = 0; slot < s->n_slots; ++slot) room += !needed[size_t(slot)] && !s->slot_prefetched[size_t(slot)];
  if (misses.size() > room) misses.resize(room);
  if (misses.empty()) return 0;
  uint64_t b = 0;
  return copy_in(s, layer, misses, needed, true, st, &b);
}

void store_record_usage(wmoe_store* s, int layer, const int32_t* experts, size_t n) {
  const size_t base = size_t(layer) * size_t(s->experts);
  for (size_t i = 0; i < n; ++i)
    if (experts[i] >= 0 && experts[i] < s->experts) ++s->usage[base + size_t(experts[i])];
}

int store_choose_hot(wmoe_store* s, double share) {
  if (!s->capped) return 0;
  if (!(share >= 0.0 && share <= 1.0)) return store_fail(s, -1, "wmoe_store_choose_hot: share outside [0, 1]");
  std::fill(s->hot.begin(), s->hot.end(), 0);
  const size_t room = size_t(double(s->n_slots) * share);
  std::vector<uint32_t> keys;
  for (size_t k = 0; k < s->usage.size(); ++k)
    if (s->usage[k] > 0) keys.push_back(uint32_t(k));
  // most used first; ties in (layer, expert) order
  std::stable_sort(keys.begin(), keys.end(), [&](uint32_t a, uint32_t b) { return s->usage[a] > s->usage[b]; });
  for (size_t i = 0; i < keys.size() && i < room; ++i) s->hot[keys[i]] = 1;
  return 0;
}

int store_mark_used(wmoe_store* s, int layer, const int32_t* experts, int n, cudaStream_t st) {
  if (!s->capped) return 0;
  const uint64_t seq = ++s->seq;
  const cudaError_t e = cudaEventRecord(s->ring[seq % wmoe_store::kRing], st);
  if (e != cudaSuccess) return store_fail(s, -2, std::string("store event: ") + cudaGetErrorString(e));
  for (int i = 0; i < n; ++i) {
    const int slot = s->slot_of[size_t(layer) * s->experts + size_t(experts[i])];
    if (slot >= 0) s->slot_use[size_t(slot)] = seq;
  }
  return 0;
}

int store_set_down_type(wmoe_store* s, int layer, int ggml_type) {
  if (layer < 0 || layer >= s->layers) return store_fail(s, -1, "wmoe_store_set_down_type: bad layer");
  if (ggml_type != kGgmlQ6K && ggml_type != kGgmlQ4K)
    return store_fail(s, -1, "wmoe_store_set_down_type: down matrices run as Q6_K (14) or Q4_K (12)");
  s->down_type[size_t(layer)] = ggml_type;
  return 0;
}

ExpertSource store_source(const wmoe_store* s, int layer, const uint8_t* shared_gate_up, const uint8_t* shared_down) {
  ExpertSource src;
  src.down_type = s->down_type[size_t(layer >= 0 && layer < s->layers ? layer : 0)];
  src.slab = s->d_slab;
  src.slot_of = s->d_slot_of;
  src.slot_bytes = s->slot_stride;
  src.gate_up_bytes = s->gate_up_bytes;
  src.experts = s->experts;
  src.n_slots = s->n_slots;
  src.shared_gate_up = shared_gate_up;
  src.shared_down = shared_down;
  return src;
}
