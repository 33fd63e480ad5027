// Expert parallelism: `world` ranks own the experts in contiguous blocks of E / world; every rank routes its own
// tokens, sends each token once to every rank that owns one of its picks (an fp16 row in the GEMM operand format plus
// one (row, expert) entry per pick), runs its experts on what it received (and the shared expert on its own tokens),
// and returns one fp16 result row per pick; the token's home rank then combines in ascending expert id, exactly as
// on one GPU, so the result does not depend on the number of ranks. willow runs on one device and has no
// counterpart; the exchange is the dispatch/combine all-to-all of the expert-parallel configurations.
//
// Home side:  ep_plan (three passes over tiles of 256 tokens: counts, a scan over tiles, placement) and ep_pack.
// Expert side: ep_fixup (received pair lists -> global row numbers), dispatch by expert, ep_gather, the GEMMs with
// the down output written in the order the pairs arrived.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace wmoe {

namespace {

constexpr int kPlanTile = 256;  // tokens per CTA of the plan's counting and placing passes

// Inclusive scan of one value per thread over a block of kPlanTile threads (8 warps); *total = block sum.
__device__ int tile_scan_incl(int v, int* total) {
  __shared__ int warp_tot[kPlanTile / 32];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  int before = 0, sum = 0;
#pragma unroll
  for (int w = 0; w < kPlanTile / 32; ++w) {
    before += w < warp ? warp_tot[w] : 0;
    sum += warp_tot[w];
  }
  __syncthreads();
  *total = sum;
  return before + incl;
}

// Pass 1: per tile of 256 tokens and destination rank d, the tokens with a pick on d (rows) and those picks
// (pairs): tile_counts[tile][d] = rows | pairs << 12 (a tile has <= 256 rows and <= 2048 pairs per rank).
__global__ void __launch_bounds__(kPlanTile) ep_count_kernel(const int32_t* __restrict__ idx, int T, int k, int E,
                                                             int world, int32_t* __restrict__ tile_counts,
                                                             int* status) {
  const int t = blockIdx.x * kPlanTile + threadIdx.x, per = E / world;
  int packed[kMaxRanks];
#pragma unroll
  for (int d = 0; d < kMaxRanks; ++d) packed[d] = 0;
  if (t < T) {
    unsigned mask = 0;
    for (int j = 0; j < k; ++j) {
      const int e = idx[size_t(t) * k + j];
      if (e < 0 || e >= E) {
        set_status(status, kStatusBadExpert);
        continue;
      }
      const int d = e / per;
      mask |= 1u << d;
#pragma unroll
      for (int dd = 0; dd < kMaxRanks; ++dd) packed[dd] += dd == d ? 1 << 12 : 0;
    }
#pragma unroll
    for (int d = 0; d < kMaxRanks; ++d) packed[d] += (mask >> d) & 1u;
  }
#pragma unroll
  for (int d = 0; d < kMaxRanks; ++d) {
    if (d >= world) break;
    int total;
    tile_scan_incl(packed[d], &total);
    if (threadIdx.x == 0) tile_counts[size_t(blockIdx.x) * world + d] = total;
  }
}

// Pass 2 (one warp per rank d): exclusive scan over tiles -> per-tile bases; totals -> send_rows / send_pairs; the
// bases include the offsets of the earlier ranks' blocks.
__global__ void ep_scan_kernel(const int32_t* __restrict__ tile_counts, int ntiles, int world,
                               int32_t* __restrict__ tile_base, int32_t* __restrict__ send_rows,
                               int32_t* __restrict__ send_pairs, int count_stride) {
  __shared__ int tot_r[kMaxRanks], tot_p[kMaxRanks];
  const int d = threadIdx.x / 32, lane = threadIdx.x % 32;
  int run_r = 0, run_p = 0;
  if (d < world) {
    for (int t0 = 0; t0 < ntiles; t0 += 32) {
      const int t = t0 + lane;
      const int v = t < ntiles ? tile_counts[size_t(t) * world + d] : 0;
      int r = v & 0xFFF, p = v >> 12;
      int ir = r, ip = p;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int nr = __shfl_up_sync(0xffffffffu, ir, o), np = __shfl_up_sync(0xffffffffu, ip, o);
        if (lane >= o) ir += nr, ip += np;
      }
      if (t < ntiles) tile_base[size_t(t) * world * 2 + 2 * d] = run_r + ir - r;
      if (t < ntiles) tile_base[size_t(t) * world * 2 + 2 * d + 1] = run_p + ip - p;
      run_r += __shfl_sync(0xffffffffu, ir, 31);
      run_p += __shfl_sync(0xffffffffu, ip, 31);
    }
    if (lane == 0) {
      tot_r[d] = run_r;
      tot_p[d] = run_p;
      send_rows[d * count_stride] = run_r;
      send_pairs[d * count_stride] = run_p;
    }
  }
  __syncthreads();
  if (d < world) {  // add the start of rank d's block (earlier ranks' totals)
    int br = 0, bp = 0;
    for (int q = 0; q < d; ++q) br += tot_r[q], bp += tot_p[q];
    for (int t = lane; t < ntiles; t += 32) {
      tile_base[size_t(t) * world * 2 + 2 * d] += br;
      tile_base[size_t(t) * world * 2 + 2 * d + 1] += bp;
    }
    if (lane == 0) {
      // per-rank block starts for pass 3's row numbers within a block (stored after the tile bases)
      tile_base[size_t(ntiles) * world * 2 + 2 * d] = br;
      tile_base[size_t(ntiles) * world * 2 + 2 * d + 1] = bp;
    }
  }
}

// Pass 3: each token's place. Rows to rank d: tokens with a pick on d, in token order; pairs to d: those picks in
// (token, slot) order, which is also the order of the result rows d sends back. ret_index[t][j]: position of pick
// (t, j)'s result row among all result rows this rank receives (blocks of send_pairs[d] in rank order).
__global__ void __launch_bounds__(kPlanTile) ep_place_kernel(const int32_t* __restrict__ idx, int T, int k, int E,
                                                             int world, const int32_t* __restrict__ tile_base,
                                                             int32_t* __restrict__ send_tok, int2* __restrict__ pair_list,
                                                             int32_t* __restrict__ ret_index) {
  const int t = blockIdx.x * kPlanTile + threadIdx.x, per = E / world;
  const int ntiles = gridDim.x;
  int packed[kMaxRanks];
  unsigned mask = 0;
#pragma unroll
  for (int d = 0; d < kMaxRanks; ++d) packed[d] = 0;
  if (t < T) {
    for (int j = 0; j < k; ++j) {
      const int e = idx[size_t(t) * k + j];
      if (e < 0 || e >= E) {
        ret_index[size_t(t) * k + j] = 0;
        continue;
      }
      const int d = e / per;
      mask |= 1u << d;
#pragma unroll
      for (int dd = 0; dd < kMaxRanks; ++dd) packed[dd] += dd == d ? 1 << 12 : 0;
    }
#pragma unroll
    for (int d = 0; d < kMaxRanks; ++d) packed[d] += (mask >> d) & 1u;
  }
#pragma unroll
  for (int d = 0; d < kMaxRanks; ++d) {
    if (d >= world) break;
    int total;
    const int incl = tile_scan_incl(packed[d], &total);
    if (t >= T || !((mask >> d) & 1u)) continue;
    const int excl = incl - packed[d];
    const int row = tile_base[size_t(blockIdx.x) * world * 2 + 2 * d] + (excl & 0xFFF);
    int q = tile_base[size_t(blockIdx.x) * world * 2 + 2 * d + 1] + (excl >> 12);
    const int local_row = row - tile_base[size_t(ntiles) * world * 2 + 2 * d];
    send_tok[row] = t;
    for (int j = 0; j < k; ++j) {
      const int e = idx[size_t(t) * k + j];
      if (e < 0 || e >= E || e / per != d) continue;
      pair_list[q] = make_int2(local_row, e);
      ret_index[size_t(t) * k + j] = q;
      ++q;
    }
  }
}

// send_buf[r] = x[send_tok[r]] as an fp16 row in run-of-8 order; blocks past the total row count return.
template <typename XT>
__global__ void __launch_bounds__(256) ep_pack_kernel(const XT* __restrict__ x, int H, const int32_t* __restrict__ send_tok,
                                                      const int32_t* __restrict__ send_rows, int count_stride,
                                                      int world, __half* __restrict__ send_buf) {
  int total = 0;
  for (int d = 0; d < world; ++d) total += send_rows[d * count_stride];
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

// The send side of the EP count exchange: per rank `words` ints, the chunk count first, zeros after.
__global__ void ep_count_header_kernel(int32_t* __restrict__ cnt, int world, int words, int chunks) {
  for (int i = threadIdx.x; i < world * words; i += blockDim.x) cnt[i] = i % words == 0 ? chunks : 0;
}

}  // namespace

cudaError_t ep_count_header(int32_t* cnt, int world, int words, int chunks, cudaStream_t st, int* launches) {
  ep_count_header_kernel<<<1, 256, 0, st>>>(cnt, world, words, chunks);
  ++*launches;
  return cudaGetLastError();
}

size_t ep_plan_scratch_bytes(int T, int world) {
  const size_t ntiles = (size_t(T) + kPlanTile - 1) / kPlanTile;
  return (ntiles * world + (ntiles + 1) * world * 2) * sizeof(int32_t);
}

cudaError_t ep_plan(const int32_t* topk_idx, int T, int k, int E, int world, int32_t* send_rows, int32_t* send_pairs,
                    int count_stride, int32_t* send_tok, int32_t* pair_list, int32_t* ret_index, void* scratch,
                    int* status, cudaStream_t st, int* launches) {
  if (world < 1 || world > kMaxRanks || E % world || k > 8 || T < 1) return cudaErrorInvalidValue;
  const int ntiles = (T + kPlanTile - 1) / kPlanTile;
  int32_t* tile_counts = static_cast<int32_t*>(scratch);
  int32_t* tile_base = tile_counts + size_t(ntiles) * world;
  ep_count_kernel<<<ntiles, kPlanTile, 0, st>>>(topk_idx, T, k, E, world, tile_counts, status);
  ep_scan_kernel<<<1, 32 * kMaxRanks, 0, st>>>(tile_counts, ntiles, world, tile_base, send_rows, send_pairs,
                                               count_stride);
  ep_place_kernel<<<ntiles, kPlanTile, 0, st>>>(topk_idx, T, k, E, world, tile_base, send_tok,
                                                reinterpret_cast<int2*>(pair_list), ret_index);
  *launches += 3;
  return cudaGetLastError();
}

cudaError_t ep_pack(const void* x, int x_dtype, int H, const int32_t* send_tok, const int32_t* send_rows,
                    int count_stride, int world, int max_rows, void* send_buf, cudaStream_t st, int* launches) {
  if (H % 8 || reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(send_buf) % 16)
    return cudaErrorInvalidValue;
  if (max_rows <= 0) return cudaSuccess;
  if (x_dtype == kF32)
    ep_pack_kernel<float><<<unsigned(max_rows), 256, 0, st>>>(static_cast<const float*>(x), H, send_tok, send_rows,
                                                              count_stride, world, static_cast<__half*>(send_buf));
  else
    ep_pack_kernel<__nv_bfloat16><<<unsigned(max_rows), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), H, send_tok, send_rows, count_stride, world, static_cast<__half*>(send_buf));
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
