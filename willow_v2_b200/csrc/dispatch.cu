// Dispatch: groups the T*k (token, slot) picks by expert, stably in token order, with no sort library and no
// atomics whose order matters (so the result is the same on every run). Replaces engines/base.py:456-467 and
// 555-566 (selected.cpu(), unique(), a nonzero() per expert) and store.py:482-484 (record_usage).
//   pass 1  per tile of 256 tokens: per-expert counts (shared-memory histogram)
//   pass 2  one CTA: per-expert totals, exclusive scan -> offsets, per-(tile, expert) bases, used-expert list
//   pass 3  per tile: each pick's rank among earlier tokens of the tile that picked the same expert, from a
//           [expert][256-bit] token mask and popcounts; position = base + rank
// Up to 256 tokens (one tile) the three passes run in one CTA (dispatch_small_kernel).
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace wmoe {

constexpr int kTile = 256;

size_t dispatch_scratch_bytes(int T, int E) {
  const size_t ntiles = (size_t(T) + kTile - 1) / kTile;
  return 2 * ntiles * size_t(E) * sizeof(int32_t);
}

__global__ void __launch_bounds__(kTile) tile_hist_kernel(const int32_t* __restrict__ idx, int T, int k, int E,
                                                          int32_t* __restrict__ tile_counts, int* status) {
  extern __shared__ int32_t hist[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int t = blockIdx.x * kTile + threadIdx.x;
  if (t < T) {
    for (int s = 0; s < k; ++s) {
      const int e = idx[size_t(t) * k + s];
      if (e < 0 || e >= E) {
        set_status(status, kStatusBadExpert);
        continue;
      }
      atomicAdd(&hist[e], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) tile_counts[size_t(blockIdx.x) * E + e] = hist[e];
}

// Exclusive scan of one value per thread over the block (blockDim.x <= 1024, a multiple of 32).
__device__ int block_exclusive_scan(int v, int* total) {
  __shared__ int warp_tot[32];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32, nwarps = blockDim.x / 32;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nwarps ? warp_tot[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    if (lane < nwarps) warp_tot[lane] = wi - w;  // exclusive prefix of warp totals
    if (lane == nwarps - 1) warp_tot[31] = wi;    // grand total (nwarps <= 31 when blockDim < 1024)
  }
  __syncthreads();
  const int result = warp_tot[warp] + incl - v;
  if (total) *total = warp_tot[31];
  __syncthreads();
  return result;
}

__global__ void scan_kernel(const int32_t* __restrict__ tile_counts, int ntiles, int T, int k, int E, int shared_rows,
                            int32_t* __restrict__ tile_base, int32_t* __restrict__ counts,
                            int32_t* __restrict__ offsets, int32_t* __restrict__ used, int32_t* __restrict__ seg,
                            int32_t* __restrict__ n_used, int64_t* __restrict__ usage) {
  const int e = threadIdx.x;
  int total = 0;
  if (e < E)
    for (int tl = 0; tl < ntiles; ++tl) total += tile_counts[size_t(tl) * E + e];
  int grand = 0;
  const int off = block_exclusive_scan(e < E ? total : 0, &grand);
  int nflag = 0;
  const int slot = block_exclusive_scan(e < E && total > 0 ? 1 : 0, &nflag);
  if (e < E) {
    counts[e] = total;
    offsets[e] = off;
    if (usage) usage[e] += total;
    int run = off;
    for (int tl = 0; tl < ntiles; ++tl) {
      tile_base[size_t(tl) * E + e] = run;
      run += tile_counts[size_t(tl) * E + e];
    }
    if (total > 0) {
      used[slot] = e;
      seg[slot] = off;
    }
  }
  if (e == 0) {
    offsets[E] = T * k;
    used[nflag] = E;  // the shared expert's segment: shared_rows rows (one per token)
    seg[nflag] = T * k;
    seg[nflag + 1] = T * k + shared_rows;
    *n_used = nflag + 1;
  }
}

__global__ void __launch_bounds__(kTile) scatter_kernel(const int32_t* __restrict__ idx, int T, int k, int E,
                                                        const int32_t* __restrict__ tile_base,
                                                        int32_t* __restrict__ perm, int32_t* __restrict__ pos) {
  extern __shared__ uint32_t mask[];  // [E][kTile / 32]
  constexpr int W = kTile / 32;
  for (int i = threadIdx.x; i < E * W; i += blockDim.x) mask[i] = 0;
  __syncthreads();
  const int lt = threadIdx.x, t = blockIdx.x * kTile + lt;
  if (t < T)
    for (int s = 0; s < k; ++s) {
      const int e = idx[size_t(t) * k + s];
      if (e >= 0 && e < E) atomicOr(&mask[e * W + lt / 32], 1u << (lt % 32));
    }
  __syncthreads();
  if (t >= T) return;
  for (int s = 0; s < k; ++s) {
    const int e = idx[size_t(t) * k + s];
    if (e < 0 || e >= E) continue;
    const uint32_t* m = mask + e * W;
    int rank = __popc(m[lt / 32] & ((1u << (lt % 32)) - 1u));
    for (int w = 0; w < lt / 32; ++w) rank += __popc(m[w]);
    const int p = tile_base[size_t(blockIdx.x) * E + e] + rank;
    perm[p] = t * k + s;
    pos[size_t(t) * k + s] = p;
  }
}

// One tile (T <= kTile): the three passes in one CTA of max(kTile, E) threads, the per-expert counts and token masks
// in shared memory. Same ranks, offsets and used-expert list as the three launches, for two launches fewer.
__global__ void __launch_bounds__(992) dispatch_small_kernel(const int32_t* __restrict__ idx, int T, int k, int E,
                                                              int shared_rows, int32_t* __restrict__ counts,
                                                              int32_t* __restrict__ offsets, int32_t* __restrict__ perm,
                                                              int32_t* __restrict__ pos, int32_t* __restrict__ used,
                                                              int32_t* __restrict__ seg, int32_t* __restrict__ n_used,
                                                              int64_t* __restrict__ usage, int* status) {
  constexpr int W = kTile / 32;
  extern __shared__ int32_t sm[];
  int32_t* hist = sm;                                         // [E]
  int32_t* base = sm + E;                                     // [E] offsets
  uint32_t* mask = reinterpret_cast<uint32_t*>(sm + 2 * E);  // [E][W]
  const int tid = threadIdx.x;
  for (int i = tid; i < E; i += blockDim.x) hist[i] = 0;
  for (int i = tid; i < E * W; i += blockDim.x) mask[i] = 0;
  __syncthreads();
  if (tid < T)
    for (int s = 0; s < k; ++s) {
      const int e = idx[size_t(tid) * k + s];
      if (e < 0 || e >= E) {
        set_status(status, kStatusBadExpert);
        continue;
      }
      atomicAdd(&hist[e], 1);
      atomicOr(&mask[e * W + tid / 32], 1u << (tid % 32));
    }
  __syncthreads();
  const int e = tid;
  const int total = e < E ? hist[e] : 0;
  int grand = 0;
  const int off = block_exclusive_scan(total, &grand);
  int nflag = 0;
  const int slot = block_exclusive_scan(e < E && total > 0 ? 1 : 0, &nflag);
  if (e < E) {
    counts[e] = total;
    offsets[e] = off;
    base[e] = off;
    if (usage) usage[e] += total;
    if (total > 0) {
      used[slot] = e;
      seg[slot] = off;
    }
  }
  if (e == 0) {
    offsets[E] = T * k;
    used[nflag] = E;  // the shared expert's segment: shared_rows rows (one per token)
    seg[nflag] = T * k;
    seg[nflag + 1] = T * k + shared_rows;
    *n_used = nflag + 1;
  }
  __syncthreads();
  if (tid >= T) return;
  for (int s = 0; s < k; ++s) {
    const int x = idx[size_t(tid) * k + s];
    if (x < 0 || x >= E) continue;
    const uint32_t* m = mask + x * W;
    int rank = __popc(m[tid / 32] & ((1u << (tid % 32)) - 1u));
    for (int w = 0; w < tid / 32; ++w) rank += __popc(m[w]);
    const int p = base[x] + rank;
    perm[p] = tid * k + s;
    pos[size_t(tid) * k + s] = p;
  }
}

cudaError_t dispatch(const int32_t* topk_idx, int T, int k, int E, void* scratch, int32_t* counts,
                     int32_t* offsets, int32_t* perm, int32_t* pos, int32_t* used, int32_t* seg, int32_t* n_used,
                     int64_t* usage, int* status, cudaStream_t st, int* launches) {
  return dispatch_rows(topk_idx, T, k, E, T, scratch, counts, offsets, perm, pos, used, seg, n_used, usage, status,
                       st, launches);
}

cudaError_t dispatch_rows(const int32_t* topk_idx, int T, int k, int E, int shared_rows, void* scratch,
                          int32_t* counts, int32_t* offsets, int32_t* perm, int32_t* pos, int32_t* used,
                          int32_t* seg, int32_t* n_used, int64_t* usage, int* status, cudaStream_t st,
                          int* launches) {
  const int ntiles = (T + kTile - 1) / kTile;
  if (ntiles <= 1 && (E + 31) / 32 * 32 <= 992) {  // block_exclusive_scan: at most 31 warps
    const int threads = std::max(kTile, (E + 31) / 32 * 32);
    dispatch_small_kernel<<<1, threads, size_t(E) * (2 + kTile / 32) * sizeof(int32_t), st>>>(
        topk_idx, T, k, E, shared_rows, counts, offsets, perm, pos, used, seg, n_used, usage, status);
    ++*launches;
    return cudaGetLastError();
  }
  int32_t* tile_counts = static_cast<int32_t*>(scratch);
  int32_t* tile_base = tile_counts + size_t(ntiles) * E;
  if (T > 0) {
    tile_hist_kernel<<<ntiles, kTile, E * sizeof(int32_t), st>>>(topk_idx, T, k, E, tile_counts, status);
    ++*launches;
  }
  const int threads = ((E + 31) / 32) * 32;
  scan_kernel<<<1, threads < 64 ? 64 : threads, 0, st>>>(tile_counts, ntiles, T, k, E, shared_rows, tile_base, counts,
                                                         offsets, used, seg, n_used, usage);
  ++*launches;
  if (T > 0) {
    scatter_kernel<<<ntiles, kTile, size_t(E) * (kTile / 32) * sizeof(uint32_t), st>>>(topk_idx, T, k, E, tile_base,
                                                                                      perm, pos);
    ++*launches;
  }
  return cudaGetLastError();
}

}  // namespace wmoe
