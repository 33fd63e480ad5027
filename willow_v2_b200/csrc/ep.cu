// Expert parallelism: `world` ranks own the experts in contiguous blocks of E / world; every rank routes its own
// tokens, sends each token once to every rank that owns one of its picks (an fp16 row in the GEMM operand format plus
// one (row, expert) entry per pick), runs its experts on what it received (and the shared expert on its own tokens),
// and returns one fp16 result row per pick; the token's home rank then combines in ascending expert id, exactly as
// on one GPU, so the result does not depend on the number of ranks. willow runs on one device and has no
// counterpart; the exchange is the dispatch/combine all-to-all of the expert-parallel configurations.
//
// Home side:  ep_plan (counts, send order, pair lists, where each pick's result row comes back) and ep_pack (rows).
// Expert side: ep_fixup (received pair lists -> global row numbers), dispatch by expert, ep_gather, the GEMMs with
// the down output written in the order the pairs arrived.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace wmoe {

namespace {

constexpr int kPlanThreads = 512;

// Exclusive scan of one value per thread over a block of kPlanThreads threads (16 warps).
__device__ int plan_scan(int v, int* total) {
  __shared__ int warp_tot[32];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  constexpr int nwarps = kPlanThreads / 32;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = lane < nwarps ? warp_tot[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    if (lane < nwarps) warp_tot[lane] = wi - w;
    if (lane == nwarps - 1) warp_tot[31] = wi;
  }
  __syncthreads();
  const int r = warp_tot[warp] + incl - v;
  *total = warp_tot[31];
  __syncthreads();
  return r;
}

// One CTA. Thread i takes tokens [i * chunk, (i + 1) * chunk). Rows to rank d are its tokens with a pick on d, in
// token order; pairs to d are those picks in (token, slot) order, which is also the order of the result rows d
// sends back. ret_index[t][j]: position of pick (t, j)'s result row among all result rows this rank receives
// (blocks of send_pairs[d] in rank order).
__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(const int32_t* __restrict__ idx, int T, int k, int E,
                                                               int world, int32_t* __restrict__ send_rows,
                                                               int32_t* __restrict__ send_pairs,
                                                               int32_t* __restrict__ send_tok,
                                                               int2* __restrict__ pair_list,
                                                               int32_t* __restrict__ ret_index, int* status) {
  __shared__ int base_r[kMaxRanks], base_p[kMaxRanks];
  const int per = E / world;
  const int chunk = (T + kPlanThreads - 1) / kPlanThreads;
  const int t0 = min(T, int(threadIdx.x) * chunk), t1 = min(T, t0 + chunk);
  int rows[kMaxRanks], pairs[kMaxRanks];
#pragma unroll
  for (int d = 0; d < kMaxRanks; ++d) rows[d] = pairs[d] = 0;
  for (int t = t0; t < t1; ++t) {
    unsigned mask = 0;
    for (int j = 0; j < k; ++j) {
      const int e = idx[size_t(t) * k + j];
      if (e < 0 || e >= E) continue;
      mask |= 1u << (e / per);
    }
#pragma unroll
    for (int d = 0; d < kMaxRanks; ++d) rows[d] += (mask >> d) & 1u;
    for (int j = 0; j < k; ++j) {
      const int e = idx[size_t(t) * k + j];
      if (e < 0 || e >= E) continue;
#pragma unroll
      for (int d = 0; d < kMaxRanks; ++d) pairs[d] += e / per == d;
    }
  }
  int rb[kMaxRanks], pb[kMaxRanks];
#pragma unroll
  for (int d = 0; d < kMaxRanks; ++d) {
    int tr, tp;
    rb[d] = plan_scan(rows[d], &tr);
    pb[d] = plan_scan(pairs[d], &tp);
    if (threadIdx.x == 0) {
      base_r[d] = tr;
      base_p[d] = tp;
      if (d < world) {
        send_rows[d] = tr;
        send_pairs[d] = tp;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int r = 0, p = 0;
    for (int d = 0; d < kMaxRanks; ++d) {
      const int nr = base_r[d], np = base_p[d];
      base_r[d] = r;
      base_p[d] = p;
      r += nr;
      p += np;
    }
  }
  __syncthreads();
  for (int t = t0; t < t1; ++t) {
    unsigned mask = 0;
    for (int j = 0; j < k; ++j) {
      const int e = idx[size_t(t) * k + j];
      if (e < 0 || e >= E) {
        set_status(status, kStatusBadExpert);
        ret_index[size_t(t) * k + j] = 0;
        continue;
      }
      mask |= 1u << (e / per);
    }
#pragma unroll
    for (int d = 0; d < kMaxRanks; ++d) {
      if (!((mask >> d) & 1u)) continue;
      const int local_row = rb[d]++;
      send_tok[base_r[d] + local_row] = t;
      for (int j = 0; j < k; ++j) {
        const int e = idx[size_t(t) * k + j];
        if (e < 0 || e >= E || e / per != d) continue;
        const int q = base_p[d] + pb[d]++;
        pair_list[q] = make_int2(local_row, e);
        ret_index[size_t(t) * k + j] = q;
      }
    }
  }
}

// send_buf[r] = x[send_tok[r]] as an fp16 row in run-of-8 order; blocks past the total row count return.
template <typename XT>
__global__ void __launch_bounds__(256) ep_pack_kernel(const XT* __restrict__ x, int H, const int32_t* __restrict__ send_tok,
                                                      const int32_t* __restrict__ send_rows, int world,
                                                      __half* __restrict__ send_buf) {
  int total = 0;
  for (int d = 0; d < world; ++d) total += send_rows[d];
  const int r = blockIdx.x;
  if (r >= total) return;
  const XT* src = x + size_t(send_tok[r]) * H;
  __half* dst = send_buf + size_t(r) * H;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    float v[8];
    load8(src + i, v);
    *reinterpret_cast<uint4*>(dst + i) = pack8_perm(v);
  }
}

struct RankBlocks {
  int pair_base[kMaxRanks + 1];  // received pairs of source s: [pair_base[s], pair_base[s + 1])
  int row_base[kMaxRanks];       // received rows of source s start at row_base[s]
};

// Received pair lists (source blocks in rank order, rows numbered within each source) -> global row and expert.
__global__ void ep_fixup_kernel(const int2* __restrict__ pairs, int P, int world, RankBlocks blocks,
                                int32_t* __restrict__ pair_row, int32_t* __restrict__ pair_expert) {
  for (int q = blockIdx.x * blockDim.x + threadIdx.x; q < P; q += gridDim.x * blockDim.x) {
    int s = 0;
    while (s + 1 < world && q >= blocks.pair_base[s + 1]) ++s;
    const int2 v = pairs[q];
    pair_row[q] = blocks.row_base[s] + v.x;
    pair_expert[q] = v.y;
  }
}

// GEMM operand rows: position p < P_r (routed, sorted by expert) copies its received row; the shared segment
// p = P_r + t converts the rank's own token t.
template <typename XT>
__global__ void __launch_bounds__(256) ep_gather_kernel(const int32_t* __restrict__ perm, const int32_t* __restrict__ pair_row,
                                                        int P_r, const __half* __restrict__ recv, const XT* __restrict__ x,
                                                        int H, __half* __restrict__ xg) {
  const int p = blockIdx.x;
  __half* dst = xg + size_t(p) * H;
  if (p < P_r) {
    const uint4* src = reinterpret_cast<const uint4*>(recv + size_t(pair_row[perm[p]]) * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) reinterpret_cast<uint4*>(dst)[i] = src[i];
  } else {
    const XT* src = x + size_t(p - P_r) * H;
    for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
      float v[8];
      load8(src + i, v);
      *reinterpret_cast<uint4*>(dst + i) = pack8_perm(v);
    }
  }
}

}  // namespace

cudaError_t ep_plan(const int32_t* topk_idx, int T, int k, int E, int world, int32_t* send_rows, int32_t* send_pairs,
                    int32_t* send_tok, int32_t* pair_list, int32_t* ret_index, int* status, cudaStream_t st,
                    int* launches) {
  if (world < 1 || world > kMaxRanks || E % world) return cudaErrorInvalidValue;
  ep_plan_kernel<<<1, kPlanThreads, 0, st>>>(topk_idx, T, k, E, world, send_rows, send_pairs, send_tok,
                                             reinterpret_cast<int2*>(pair_list), ret_index, status);
  ++*launches;
  return cudaGetLastError();
}

cudaError_t ep_pack(const void* x, int x_dtype, int H, const int32_t* send_tok, const int32_t* send_rows, int world,
                    int max_rows, void* send_buf, cudaStream_t st, int* launches) {
  if (H % 8 || reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(send_buf) % 16)
    return cudaErrorInvalidValue;
  if (max_rows <= 0) return cudaSuccess;
  if (x_dtype == kF32)
    ep_pack_kernel<float><<<unsigned(max_rows), 256, 0, st>>>(static_cast<const float*>(x), H, send_tok, send_rows,
                                                              world, static_cast<__half*>(send_buf));
  else
    ep_pack_kernel<__nv_bfloat16><<<unsigned(max_rows), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), H, send_tok, send_rows, world, static_cast<__half*>(send_buf));
  ++*launches;
  return cudaGetLastError();
}

cudaError_t ep_fixup(const int32_t* pair_list, int P, int world, const int32_t* recv_rows, const int32_t* recv_pairs,
                     int32_t* pair_row, int32_t* pair_expert, cudaStream_t st, int* launches) {
  if (world < 1 || world > kMaxRanks) return cudaErrorInvalidValue;
  RankBlocks b{};
  int r = 0, p = 0;
  for (int s = 0; s < world; ++s) {
    b.pair_base[s] = p;
    b.row_base[s] = r;
    p += recv_pairs[s];
    r += recv_rows[s];
  }
  b.pair_base[world] = p;
  if (p != P) return cudaErrorInvalidValue;
  if (P > 0) {
    ep_fixup_kernel<<<unsigned(std::min((P + 255) / 256, 1024)), 256, 0, st>>>(
        reinterpret_cast<const int2*>(pair_list), P, world, b, pair_row, pair_expert);
    ++*launches;
  }
  return cudaGetLastError();
}

cudaError_t ep_gather(const int32_t* perm, const int32_t* pair_row, int P_r, const void* recv, const void* x,
                      int x_dtype, int T, int H, void* xg, cudaStream_t st, int* launches) {
  if (H % 8 || reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(recv) % 16) return cudaErrorInvalidValue;
  const unsigned rows = unsigned(P_r + T);
  if (rows == 0) return cudaSuccess;
  if (x_dtype == kF32)
    ep_gather_kernel<float><<<rows, 256, 0, st>>>(perm, pair_row, P_r, static_cast<const __half*>(recv),
                                                  static_cast<const float*>(x), H, static_cast<__half*>(xg));
  else
    ep_gather_kernel<__nv_bfloat16><<<rows, 256, 0, st>>>(perm, pair_row, P_r, static_cast<const __half*>(recv),
                                                          static_cast<const __nv_bfloat16*>(x), H,
                                                          static_cast<__half*>(xg));
  ++*launches;
  return cudaGetLastError();
}

}  // namespace wmoe
