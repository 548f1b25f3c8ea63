// Covariance pass of the rotation builder on the 5th-generation tensor cores.
//
// For every matrix m = (b, h) of visual Keys K [S x 128] (bf16 / fp16):
//   cov[m]  = sum_s k_s k_s^T   (fp32, 128 x 128, uncentred)
//   ksum[m] = sum_s k_s          (fp32, 128)
// -- the raw sums behind kv_pruning_utils.py:112-115 (the eigensolver prologue
// centres them).
//
// A cluster of Z CTAs (Z in {1, 2, 4, 8}) owns one matrix; CTA z of the
// cluster takes the z-th contiguous share of its 64-token tiles.  Per CTA:
//   warp 0  TMA producer: 4-D tensor-map loads of a tile as two 64 x 64 boxes
//           (128B swizzle) into a 6-stage ring (no multicast)
//   warp 1  allocates 128 TMEM columns; one lane issues, per tile, four
//           tcgen05.mma kind::f16 M=128 N=128 K=16: A = K^T and B = K are the
//           same shared-memory tile read MN-major (channels contiguous), fp32
//           accumulation in TMEM; tcgen05.commit releases the stage
//   warps 2-5  sum the tile's channels (CUDA cores) for ksum, then read the
//           TMEM accumulator (warp w reads lanes 32 (w % 4) ...) into shared
//           memory
// Then the cluster reduces: CTA z sums rows [z 128/Z, (z+1) 128/Z) of every
// peer's partial through distributed shared memory and writes them; CTA 0 does
// the same for ksum.  Only the reduced 64 KB per matrix reaches HBM.
#include <type_traits>

#include "builder.h"
#include "tcgen05.cuh"

namespace rtk {
namespace {

constexpr int kTile = 64;              // tokens per stage
constexpr int kBox = kTile * 128;      // one {64 channels x 64 tokens} box, bytes
constexpr int kStageBytes = 2 * kBox;  // channels 0-63 | 64-127
constexpr int kStages = 6;
constexpr int kThreads = 192;
constexpr int kDumpStride = 132;       // fp32 row stride of the accumulator dump

struct CovSmem {
  static constexpr int kRing = 0;
  static constexpr int kBar = kRing + kStages * kStageBytes;   // full[6], empty[6], acc
  static constexpr int kTmemSlot = kBar + (2 * kStages + 1) * 8;
  static constexpr int kSums = (kTmemSlot + 16 + 15) & ~15;     // fp32 [4 warps][128]
  static constexpr int kColSum = kSums + 4 * 128 * 4;           // fp32 [128] this CTA's ksum
  static constexpr int kBytes = kColSum + 128 * 4;
  static_assert(kStages * kStageBytes >= 128 * kDumpStride * 4, "dump must fit in the ring");
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    cov_tc_kernel(const __grid_constant__ CUtensorMap keys_map, const CovParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem + CovSmem::kBar);
  uint64_t *empty_bar = full_bar + kStages;
  uint64_t *acc_bar = empty_bar + kStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + CovSmem::kTmemSlot);
  float *sums = reinterpret_cast<float *>(smem + CovSmem::kSums);
  float *colsum = reinterpret_cast<float *>(smem + CovSmem::kColSum);
  float *dump = reinterpret_cast<float *>(smem + CovSmem::kRing);
  __shared__ int abort_flag;
  __shared__ unsigned int dummy_status;

  const int Z = p.splits;
  const int m = blockIdx.x / Z;
  const int z = static_cast<int>(cluster_rank());
  const int b = m / p.heads, h = m % p.heads;
  const int tiles = (p.seq + kTile - 1) / kTile;
  const int t0 = static_cast<int>((long long)z * tiles / Z);
  const int t1 = static_cast<int>((long long)(z + 1) * tiles / Z);
  const int nt = t1 - t0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned int *status = &dummy_status;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1 + 4);
    }
    mbar_init(acc_bar, 1);
    abort_flag = 0;
    dummy_status = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&keys_map);
      for (int i = 0; i < nt; ++i) {
        const int st = i % kStages;
        if (!mbar_wait_bounded(&empty_bar[st], ((i / kStages) & 1) ^ 1, &abort_flag, status)) break;
        unsigned char *dst = smem + CovSmem::kRing + st * kStageBytes;
        mbar_arrive_expect_tx(&full_bar[st], kStageBytes);
        tma_load_4d(dst, &keys_map, 0, (t0 + i) * kTile, h, b, &full_bar[st]);
        tma_load_4d(dst + kBox, &keys_map, 64, (t0 + i) * kTile, h, b, &full_bar[st]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_f16(std::is_same<T, __nv_bfloat16>::value ? 1u : 0u, 1u, 1u, 128u, 128u);
      for (int i = 0; i < nt; ++i) {
        const int st = i % kStages;
        mbar_wait_bounded(&full_bar[st], (i / kStages) & 1, &abort_flag, status);
        tc_fence_after();
        const uint32_t base = smem_u32(smem + CovSmem::kRing + st * kStageBytes);
#pragma unroll
        for (int ks = 0; ks < kTile / 16; ++ks) {
          const uint64_t d = smem_desc_sw128(base + ks * 2048, kBox, 1024);
          umma_f16(tmem, d, d, kIdesc, (i > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(&empty_bar[st]);   // stage free once these MMAs have read it
      }
      umma_commit(acc_bar);            // accumulator complete
    }
  } else {
    // ---------------- channel sums, then the accumulator
    const int et = threadIdx.x - 64;         // 0..127
    const int chunk = et & 15, rg = et >> 4; // 8 channels x 8 rows per thread
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
    for (int i = 0; i < nt; ++i) {
      const int st = i % kStages;
      mbar_wait_bounded(&full_bar[st], (i / kStages) & 1, &abort_flag, status);
      const unsigned char *tile = smem + CovSmem::kRing + st * kStageBytes + (chunk >> 3) * kBox;
#pragma unroll
      for (int rr = 0; rr < 8; ++rr) {
        const int r = rg * 8 + rr;
        const uint4 v = *reinterpret_cast<const uint4 *>(tile + swizzled_offset<128>(r, (chunk & 7) * 8));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float lo, hi;
          unpack2<T>(w[k], lo, hi);
          acc[2 * k] += lo;
          acc[2 * k + 1] += hi;
        }
      }
      // the generic-proxy reads above must be ordered before the TMA write
      // that refills this stage (async proxy): without the proxy fence a
      // refill overwrote tiles still being read when two CTAs shared an SM
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[st]);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], 16);
    if ((lane & 16) == 0) {
#pragma unroll
      for (int k = 0; k < 8; ++k) sums[(warp - 2) * 128 + chunk * 8 + k] = acc[k];
    }
    named_barrier_sync(1, 128);
    colsum[et] = sums[et] + sums[128 + et] + sums[256 + et] + sums[384 + et];
    // accumulator -> shared memory (fp32 rows, stride 132); reuses the ring
    mbar_wait_bounded(acc_bar, 0, &abort_flag, status);
    tc_fence_after();
    const int lane_base = 32 * (warp & 3);
    const int row = lane_base + lane;
#pragma unroll
    for (int c0 = 0; c0 < 128; c0 += 32) {
      float v[32];
      if (nt > 0) {
        tmem_ld32(tmem + ((uint32_t)lane_base << 16) + (uint32_t)c0, v);
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < 32; k += 4)
        *reinterpret_cast<float4 *>(dump + row * kDumpStride + c0 + k) =
            make_float4(v[k], v[k + 1], v[k + 2], v[k + 3]);
    }
    tc_fence_before();
  }
  __syncthreads();
  cluster_sync();  // every CTA of the cluster has its partial in shared memory

  // ---------------- cluster reduction: this CTA's share of rows, every peer summed
  {
    const int rows = 128 / Z;
    const int r0 = z * rows;
    float *out = p.cov + (long long)m * 128 * 128;
    for (int e = threadIdx.x; e < rows * 32; e += kThreads) {
      const int row = r0 + e / 32, c4 = (e % 32) * 4;
      const uint32_t local = smem_u32(dump + row * kDumpStride + c4);
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < Z; ++q) {
        const float4 v = ld_cluster_f4(map_to_cta(local, q));
        a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
      }
      *reinterpret_cast<float4 *>(out + row * 128 + c4) = a;
    }
    if (z == 0 && threadIdx.x < 128) {
      const uint32_t local = smem_u32(colsum + threadIdx.x);
      float a = 0.f;
      for (int q = 0; q < Z; ++q) a += ld_cluster_f32(map_to_cta(local, q));
      p.ksum[(long long)m * 128 + threadIdx.x] = a;
    }
  }
  cluster_sync();  // peers are done reading this CTA's shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

}  // namespace

cudaError_t launch_cov_tc(int dtype_is_bf16, const CUtensorMap &keys_map, const CovParams &p,
                          cudaStream_t stream) {
  const int smem = CovSmem::kBytes + 1024;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.batch * p.heads * p.splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (dtype_is_bf16) {
    cudaError_t err = cudaFuncSetAttribute(cov_tc_kernel<__nv_bfloat16>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    err = cudaLaunchKernelEx(&cfg, cov_tc_kernel<__nv_bfloat16>, keys_map, p);
    if (err != cudaSuccess) return err;
  } else {
    cudaError_t err = cudaFuncSetAttribute(cov_tc_kernel<__half>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    err = cudaLaunchKernelEx(&cfg, cov_tc_kernel<__half>, keys_map, p);
    if (err != cudaSuccess) return err;
  }
  return cudaGetLastError();
}

}  // namespace rtk
