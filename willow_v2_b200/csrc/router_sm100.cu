// Router logits for many bf16 tokens on the tensor cores: logits = x . R^T with the float32 router R carried as three
// bf16 terms R = R1 + R2 + R3 (R1 = bf16(R), R2 = bf16(R - R1), R3 = bf16(R - R1 - R2); together ~24 mantissa bits).
// bf16 x times each term is exact in the fp32 accumulator, so the logits match a float32 GEMM to ~1e-7 relative,
// well inside the 1e-5 tie rule of the routing parity (engines/base.py:91-97 computes them in float32).
//
// One CTA: 128 tokens x E = 256 experts over one quarter of the hidden size (K split 4 ways for SM coverage; the
// top-k kernel adds the four partial logits in a fixed order). Warp 0 lane 0 loads the token tile (128 x 64 bf16)
// and the three router terms (3 x 256 x 64) of each K block by TMA into a 2-stage ring; warp 1 lane 0 issues
// 4 x 3 tcgen05.mma (M 128, N 256, K 16) per K block into a 256-column TMEM accumulator; then all four warps read
// their 32 token rows back and store the partial logits. Every wait is bounded (1 s), as in the grouped GEMM.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace wmoe {

namespace {

using namespace sm100;

constexpr int kRT = 128, kRE = 256, kRK = 64, kRStages = 2;
constexpr int kRTileX = kRT * kRK * 2;       // 16 KB
constexpr int kRTileW = kRE * kRK * 2;       // 32 KB per term
constexpr int kRStage = kRTileX + 3 * kRTileW;
constexpr int kRSmem = kRStages * kRStage + 1024;
static_assert(kRSmem <= 232448 - 256, "shared memory");

struct RouterBars {
  uint64_t full[kRStages], empty[kRStages], done;
  uint32_t tmem;
  int fail;
};

__global__ void __launch_bounds__(128, 1) router_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                           const __grid_constant__ CUtensorMap tmap_w, int T, int H,
                                                           float* __restrict__ partial, int* status) {
  extern __shared__ __align__(1024) uint8_t dyn[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn) + 1023) & ~uintptr_t(1023));
  __shared__ RouterBars bars;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int t0 = blockIdx.x * kRT, split = blockIdx.y, nsplit = gridDim.y;
  const int nkb = H / kRK / nsplit, kb0 = split * nkb;

  if (tid == 0) {
    bars.fail = 0;
    for (int s = 0; s < kRStages; ++s) {
      mbar_init(&bars.full[s], 1);
      mbar_init(&bars.empty[s], 1);
    }
    mbar_init(&bars.done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&bars.tmem)),
                 "r"(kRE)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = bars.tmem;
  volatile int* fail = &bars.fail;
  int issued = 0;

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < nkb; ++i) {
      const int s = i % kRStages;
      if (i >= kRStages && !mbar_wait(&bars.empty[s], unsigned((i / kRStages - 1) & 1), fail)) break;
      uint8_t* st = base + s * kRStage;
      const int k = (kb0 + i) * kRK;
      mbar_arrive_expect_tx(&bars.full[s], unsigned(kRStage));
      tma_load_2d(st, &tmap_x, k, t0, &bars.full[s]);
      for (int p = 0; p < 3; ++p) tma_load_2d(st + kRTileX + p * kRTileW, &tmap_w, k, p * kRE, &bars.full[s]);
      issued = i + 1;
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = idesc_f16(kRT, kRE, true);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % kRStages;
      if (!mbar_wait(&bars.full[s], unsigned((i / kRStages) & 1), fail)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint8_t* st = base + s * kRStage;
      const uint64_t da = smem_desc(st);
#pragma unroll
      for (int k = 0; k < kRK / 16; ++k)
#pragma unroll
        for (int p = 0; p < 3; ++p)
          mma_f16_ss(tmem, da + 2 * k, smem_desc(st + kRTileX + p * kRTileW) + 2 * k, idesc, (i | k | p) != 0);
      mma_commit(&bars.empty[s]);
    }
    mma_commit(&bars.done);
  }
  __syncwarp();
  // epilogue: thread = token row 32 warp + lane, 256 columns of its TMEM lane
  const bool ok = mbar_wait(&bars.done, 0, fail) && !*fail;
  if (__all_sync(0xffffffffu, ok)) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int t = t0 + 32 * warp + lane;
    float* row = partial + (size_t(split) * T + t) * kRE;
    for (int c0 = 0; c0 < kRE; c0 += 32) {
      float v[32];
      tmem_ld32(tmem + (uint32_t(32 * warp) << 16) + uint32_t(c0), v);
      if (t < T) {
#pragma unroll
        for (int c = 0; c < 32; c += 4)
          *reinterpret_cast<float4*>(row + c0 + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
      }
    }
  }
  if (tid == 0 && *fail) set_status(status, kStatusBarrierTimeout);
  if (*fail) {  // bounded waits for the copies and MMAs this CTA issued before it frees shared memory and TMEM
    volatile int never = 0;
    if (warp == 1) mbar_wait(&bars.done, 0, &never);
    if (warp == 0 && lane == 0)
      for (int i = max(0, issued - kRStages); i < issued; ++i)
        mbar_wait(&bars.full[i % kRStages], unsigned((i / kRStages) & 1), &never);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kRE) : "memory");
}

cudaError_t make_tmap_bf16(CUtensorMap* map, const void* ptr, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  EncodeFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {uint32_t(kRK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// R (f32 [E][H]) -> three bf16 terms [3][E][H]: R1 = bf16(R), R2 = bf16(R - R1), R3 = bf16(R - R1 - R2). The
// differences are exact in float32.
__global__ void router_split_kernel(const float* __restrict__ R, size_t n, __nv_bfloat16* __restrict__ out) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    const float w = R[i];
    const __nv_bfloat16 a = __float2bfloat16_rn(w);
    const float r1 = w - __bfloat162float(a);
    const __nv_bfloat16 b = __float2bfloat16_rn(r1);
    const float r2 = r1 - __bfloat162float(b);
    out[i] = a;
    out[n + i] = b;
    out[2 * n + i] = __float2bfloat16_rn(r2);
  }
}

}  // namespace

bool router_tc_supported(int T, int H, int E) {
  return E == kRE && H % (kRK * kRouterKSplit) == 0 && T >= 1;
}

cudaError_t router_split(const float* router_w, int E, int H, void* out, cudaStream_t st) {
  const size_t n = size_t(E) * H;
  router_split_kernel<<<unsigned(std::min<size_t>((n + 255) / 256, 4096)), 256, 0, st>>>(
      router_w, n, static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

cudaError_t router_logits_tc(const void* x_bf16, int T, int H, int E, const void* router_split3, float* partial,
                             int* status, cudaStream_t st, int* launches) {
  if (!router_tc_supported(T, H, E)) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_done{0};  // the kernel's shared memory limit, once per device
  cudaError_t e = once_per_device(attr_done, []() {
    return cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRSmem);
  });
  if (e != cudaSuccess) return e;
  CUtensorMap mx, mw;
  if ((e = make_tmap_bf16(&mx, x_bf16, uint64_t(T), uint64_t(H), kRT)) != cudaSuccess) return e;
  if ((e = make_tmap_bf16(&mw, router_split3, uint64_t(3) * E, uint64_t(H), kRE)) != cudaSuccess) return e;
  router_tc_kernel<<<dim3(unsigned((T + kRT - 1) / kRT), unsigned(kRouterKSplit)), 128, kRSmem, st>>>(mx, mw, T, H,
                                                                                                      partial, status);
  ++*launches;
  return cudaGetLastError();
}

}  // namespace wmoe
