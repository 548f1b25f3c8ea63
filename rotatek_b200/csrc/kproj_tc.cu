// Fused Key projection + RoPE + covariance sums on the 5th-generation tensor cores.
//
// The attention adapters compute the prefill Keys as k_proj(X) -> RoPE
// (llava_next/llama_visionzip.py:144-153, qwen/qwen2_5vl_visionzip.py:932-942),
// and ChannelPruner.update_rotatek then reads the visual Keys again for their
// mean and covariance (kv_pruning_utils.py:112-115).  This kernel produces the
// post-RoPE Keys and, in the same pass, the raw sums sum_s k k^T and sum_s k of
// the visual span -- the inputs of the Jacobi prologue -- so the covariance
// pass over K disappears.
//
// Work: a cluster of Z CTAs owns one (b, h); its 128-token tiles (prompt tiles,
// then visual, then text, each span tiled from its own start) are split into Z
// contiguous ranges.  Per CTA (192 threads, one CTA per SM):
//   warp 0     TMA producer: per tile and per 64-wide hidden chunk, an X box
//              {64 hidden x 128 tokens} and a W box {64 hidden x 128 channels}
//              (128B swizzle) into a 5-stage ring
//   warp 1     TMEM owner (512 columns) and MMA issuer: per chunk four
//              tcgen05.mma kind::f16 M=128 N=128 K=16, both operands K-major,
//              into one of two fp32 projection accumulators (columns 0 / 128);
//              after a visual tile has been staged, eight more MMAs add
//              K_tile^T K_tile into the covariance accumulator (columns 256..383)
//              from the staged tile read MN-major
//   warps 2-5  epilogue, one token row per thread: TMEM -> registers, + bias,
//              round, RoPE with torch's roundings, -> a 128B-swizzled staging
//              tile that is at once the TMA-store source and the covariance
//              MMA operand; channel sums of visual tiles from the staging tile
// Rows past the end of their span are zeroed (no covariance contribution) and
// clipped by the span's output tensor map.  At the end the cluster reduces the
// Z partial sums through distributed shared memory (as the covariance kernel
// does) and writes cov / ksum.
#include <type_traits>

#include "builder.h"
#include "tcgen05.cuh"

namespace rtk {
namespace {

constexpr int kRows = 128;              // tokens per tile
constexpr int kBox = 128 * 128;         // bytes of a {64 x 128} 16-bit box
constexpr int kStages = 5;
constexpr int kThreads = 192;
constexpr int kDumpStride = 132;        // fp32 row stride of the covariance dump
constexpr uint32_t kAccCols = 128;      // one projection accumulator
constexpr uint32_t kCovCol = 256;       // covariance accumulator
constexpr uint32_t kTmemCols = 512;

struct KpSmem {
  static constexpr int kRing = 0;                                 // stage: X box | W box
  static constexpr int kStage = kRing + kStages * 2 * kBox;       // channels 0-63 | 64-127
  static constexpr int kBar = kStage + 2 * kBox;
  // full[kStages], empty[kStages], acc_full[2], acc_empty[2], staged, staging_free, cov_done
  static constexpr int kNumBars = 2 * kStages + 7;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kBias = (kTmemSlot + 16 + 15) & ~15;       // fp32 [128]
  static constexpr int kSums = kBias + 128 * 4;                   // fp32 [4 warps][128]
  static constexpr int kColSum = kSums + 4 * 128 * 4;             // fp32 [128]
  static constexpr int kBytes = kColSum + 128 * 4;
  static_assert(kStages * 2 * kBox >= 128 * kDumpStride * 4, "dump must fit in the ring");
  static_assert(kStage % 1024 == 0, "swizzled boxes need 1024-byte alignment");
};

// The three spans of a (b, h) row of tokens and their 128-token tiles.
struct Spans {
  int start[3], end[3], first_tile[4];

  __device__ void init(int seq, int vs, int vl) {
    start[0] = 0;       end[0] = vs;
    start[1] = vs;      end[1] = vs + vl;
    start[2] = vs + vl; end[2] = seq;
    first_tile[0] = 0;
#pragma unroll
    for (int i = 0; i < 3; ++i) first_tile[i + 1] = first_tile[i] + (end[i] - start[i] + kRows - 1) / kRows;
  }
  __device__ int total() const { return first_tile[3]; }
  __device__ int span_of(int tile) const {
    return tile < first_tile[1] ? 0 : tile < first_tile[2] ? 1 : 2;
  }
  __device__ int row0(int tile, int span) const { return start[span] + (tile - first_tile[span]) * kRows; }
};

template <typename T>
__device__ __forceinline__ float round_to(float x) {
  return to_f32<T>(from_f32<T>(x));
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4 &v, float (&f)[8]) {
  unpack2<T>(v.x, f[0], f[1]);
  unpack2<T>(v.y, f[2], f[3]);
  unpack2<T>(v.z, f[4], f[5]);
  unpack2<T>(v.w, f[6], f[7]);
}

// One token row of the epilogue: 128 fp32 projection values from TMEM ->
// bias, rounding, RoPE -> 64 packed 16-bit pairs (channels 2j, 2j+1 in out[j]).
//   k      = round(acc + bias)                     (the projection's output)
//   out_lo = round(round(k_lo cos_lo) - round(k_hi sin_lo))   channels d < 64
//   out_hi = round(round(k_hi cos_hi) + round(k_lo sin_hi))   channels d + 64
// which is torch's  k * cos + rotate_half(k) * sin  in the Keys' dtype.
template <typename T>
__device__ __forceinline__ void rope_row(uint32_t tmem_row, const float *bias, const T *crow,
                                         const T *srow, bool valid, uint32_t (&out)[64]) {
#pragma unroll
  for (int h2 = 0; h2 < 4; ++h2) {
    uint32_t rlo[16], rhi[16];
    tmem_ld16_nowait(tmem_row + 16 * h2, rlo);
    tmem_ld16_nowait(tmem_row + 64 + 16 * h2, rhi);
    tmem_wait_ld();
    float lo[16], hi[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      lo[e] = __uint_as_float(rlo[e]);
      hi[e] = __uint_as_float(rhi[e]);
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int d = 16 * h2 + 8 * q;
      float cl[8], ch[8], sl[8], sh[8];
      if (valid) {
        unpack8<T>(__ldg(reinterpret_cast<const uint4 *>(crow + d)), cl);
        unpack8<T>(__ldg(reinterpret_cast<const uint4 *>(crow + d + 64)), ch);
        unpack8<T>(__ldg(reinterpret_cast<const uint4 *>(srow + d)), sl);
        unpack8<T>(__ldg(reinterpret_cast<const uint4 *>(srow + d + 64)), sh);
      }
      float olo[8], ohi[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (valid) {
          const float klo = round_to<T>(__fadd_rn(lo[8 * q + e], bias[d + e]));
          const float khi = round_to<T>(__fadd_rn(hi[8 * q + e], bias[d + 64 + e]));
          olo[e] = round_to<T>(__fsub_rn(round_to<T>(__fmul_rn(klo, cl[e])),
                                         round_to<T>(__fmul_rn(khi, sl[e]))));
          ohi[e] = round_to<T>(__fadd_rn(round_to<T>(__fmul_rn(khi, ch[e])),
                                         round_to<T>(__fmul_rn(klo, sh[e]))));
        } else {
          olo[e] = 0.f;
          ohi[e] = 0.f;
        }
      }
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        out[(d + e) >> 1] = pack2<T>(olo[e], olo[e + 1]);
        out[(d + 64 + e) >> 1] = pack2<T>(ohi[e], ohi[e + 1]);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    kproj_tc_kernel(const __grid_constant__ KProjMaps maps, const KProjParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem + KpSmem::kBar);
  uint64_t *empty_bar = full_bar + kStages;
  uint64_t *acc_full = empty_bar + kStages;    // [2] accumulator ready for the epilogue
  uint64_t *acc_empty = acc_full + 2;          // [2] accumulator drained (4 warp arrivals)
  uint64_t *staged_bar = acc_empty + 2;        // a visual tile is in the staging buffer
  uint64_t *free_bar = staged_bar + 1;         // its covariance MMAs have read it
  uint64_t *cov_bar = free_bar + 1;            // every MMA of this CTA has completed
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + KpSmem::kTmemSlot);
  float *bias_s = reinterpret_cast<float *>(smem + KpSmem::kBias);
  float *sums = reinterpret_cast<float *>(smem + KpSmem::kSums);
  float *colsum = reinterpret_cast<float *>(smem + KpSmem::kColSum);
  float *dump = reinterpret_cast<float *>(smem + KpSmem::kRing);
  unsigned char *stage = smem + KpSmem::kStage;
  __shared__ int abort_flag;

  const int Z = p.splits;
  const int m = blockIdx.x / Z;
  const int z = static_cast<int>(cluster_rank());
  const int b = m / p.heads, h = m % p.heads;
  Spans sp;
  sp.init(p.seq, p.vis_start, p.vis_len);
  const int tiles = sp.total();
  const int t0 = static_cast<int>((long long)z * tiles / Z);
  const int nt = static_cast<int>((long long)(z + 1) * tiles / Z) - t0;
  const int nk = p.hidden / 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned int *status = p.status;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    mbar_init(staged_bar, 1);
    mbar_init(free_bar, 1);
    mbar_init(cov_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  if (threadIdx.x >= 64) {
    const int c = threadIdx.x - 64;
    bias_s[c] = p.bias != nullptr ? to_f32<T>(static_cast<const T *>(p.bias)[h * 128 + c]) : 0.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&maps.x);
      tma_prefetch_desc(&maps.w);
      int it = 0;
      bool ok = true;
      for (int i = 0; i < nt && ok; ++i) {
        const int tile = t0 + i, span = sp.span_of(tile), r0 = sp.row0(tile, span);
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int st = it % kStages;
          if (!mbar_wait_bounded(&empty_bar[st], ((it / kStages) & 1) ^ 1, &abort_flag, status)) {
            ok = false;
            break;
          }
          unsigned char *dst = smem + KpSmem::kRing + st * 2 * kBox;
          mbar_arrive_expect_tx(&full_bar[st], 2 * kBox);
          tma_load_3d(dst, &maps.x, kc * 64, r0, b, &full_bar[st]);
          tma_load_2d(dst + kBox, &maps.w, kc * 64, h * 128, &full_bar[st]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t kIdProj = idesc_f16(kFmt, 0u, 0u, 128u, 128u);   // X, W K-major
      constexpr uint32_t kIdCov = idesc_f16(kFmt, 1u, 1u, 128u, 128u);    // K^T, K MN-major
      const uint32_t stage_addr = smem_u32(stage);
      int it = 0, ncov = 0;
      auto issue_cov = [&]() {
        mbar_wait_bounded(staged_bar, ncov & 1, &abort_flag, status);
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kRows / 16; ++ks) {
          const uint64_t d = smem_desc_sw128(stage_addr + ks * 2048, kBox, 1024);
          umma_f16(tmem + kCovCol, d, d, kIdCov, (ncov > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(free_bar);
        ++ncov;
      };
      for (int i = 0; i < nt; ++i) {
        const int a = i & 1;
        mbar_wait_bounded(&acc_empty[a], ((i >> 1) & 1) ^ 1, &abort_flag, status);
        tc_fence_after();
        const uint32_t d_acc = tmem + a * kAccCols;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int st = it % kStages;
          mbar_wait_bounded(&full_bar[st], (it / kStages) & 1, &abort_flag, status);
          tc_fence_after();
          const uint32_t base = smem_u32(smem + KpSmem::kRing + st * 2 * kBox);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t da = smem_desc_sw128(base + ks * 32, 16, 1024);
            const uint64_t db = smem_desc_sw128(base + kBox + ks * 32, 16, 1024);
            umma_f16(d_acc, da, db, kIdProj, (kc > 0 || ks > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[st]);   // stage free once these MMAs have read it
        }
        // the previous tile's covariance update runs behind this tile's projection
        if (i > 0 && sp.span_of(t0 + i - 1) == 1) issue_cov();
        umma_commit(&acc_full[a]);
      }
      if (nt > 0 && sp.span_of(t0 + nt - 1) == 1) issue_cov();
      umma_commit(cov_bar);
    }
  } else {
    // ---------------- epilogue: one token row per thread
    const int et = threadIdx.x - 64;
    const int quarter = warp & 3;                  // TMEM lanes this warp may read
    const int row = 32 * quarter + lane;
    const uint32_t tmem_lane = tmem + ((uint32_t)(32 * quarter) << 16);
    const int chunk = et & 15, rg = et >> 4;       // channel sums: 8 channels x 16 rows
    float ks_acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) ks_acc[k] = 0.f;
    const T *cos_b = static_cast<const T *>(p.cos) + (long long)b * p.cs_sb;
    const T *sin_b = static_cast<const T *>(p.sin) + (long long)b * p.cs_sb;
    int nvis = 0;
    bool pending = false, stored = false;
    for (int i = 0; i < nt; ++i) {
      const int tile = t0 + i, span = sp.span_of(tile), r0 = sp.row0(tile, span);
      const int a = i & 1;
      const int t = r0 + row;
      const bool valid = t < sp.end[span];
      mbar_wait_bounded(&acc_full[a], (i >> 1) & 1, &abort_flag, status);
      tc_fence_after();
      uint32_t out[64];
      rope_row<T>(tmem_lane + a * kAccCols, bias_s, cos_b + (long long)t * p.cs_ss,
                  sin_b + (long long)t * p.cs_ss, valid, out);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
      // the staging tile is reusable once the previous visual tile's MMAs and
      // the previous TMA store have read it
      if (pending) {
        mbar_wait_bounded(free_bar, (nvis - 1) & 1, &abort_flag, status);
        pending = false;
      }
      if (et == 0 && stored) bulk_wait_read_all();
      named_barrier_sync(1, 128);
#pragma unroll
      for (int c8 = 0; c8 < 16; ++c8)
        *reinterpret_cast<uint4 *>(stage + (c8 >> 3) * kBox + swizzled_offset<128>(row, (c8 & 7) * 8)) =
            make_uint4(out[4 * c8], out[4 * c8 + 1], out[4 * c8 + 2], out[4 * c8 + 3]);
      fence_proxy_async_smem();
      named_barrier_sync(1, 128);
      if (et == 0) {
        tma_store_4d(&maps.k_out[span], stage, 0, r0 - sp.start[span], h, b);
        tma_store_4d(&maps.k_out[span], stage + kBox, 64, r0 - sp.start[span], h, b);
        bulk_commit_group();
        if (span == 1) mbar_arrive(staged_bar);
      }
      stored = true;
      if (span == 1) {
        pending = true;
        ++nvis;
        const unsigned char *box = stage + (chunk >> 3) * kBox;
#pragma unroll 4
        for (int rr = 0; rr < 16; ++rr) {
          const uint4 v = *reinterpret_cast<const uint4 *>(box + swizzled_offset<128>(rg * 16 + rr, (chunk & 7) * 8));
          float f[8];
          unpack8<T>(v, f);
#pragma unroll
          for (int k = 0; k < 8; ++k) ks_acc[k] += f[k];
        }
      }
    }
    if (et == 0 && stored) bulk_wait_all();
#pragma unroll
    for (int k = 0; k < 8; ++k) ks_acc[k] += __shfl_xor_sync(0xffffffffu, ks_acc[k], 16);
    if ((lane & 16) == 0) {
#pragma unroll
      for (int k = 0; k < 8; ++k) sums[(warp - 2) * 128 + chunk * 8 + k] = ks_acc[k];
    }
    named_barrier_sync(1, 128);
    colsum[et] = sums[et] + sums[128 + et] + sums[256 + et] + sums[384 + et];
    // covariance accumulator -> shared memory (fp32 rows, stride 132); reuses the ring
    mbar_wait_bounded(cov_bar, 0, &abort_flag, status);
    tc_fence_after();
#pragma unroll
    for (int c0 = 0; c0 < 128; c0 += 32) {
      float v[32];
      if (nvis > 0) {
        tmem_ld32(tmem_lane + kCovCol + (uint32_t)c0, v);
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
    const int q0 = z * rows;
    float *out = p.cov + (long long)m * 128 * 128;
    for (int e = threadIdx.x; e < rows * 32; e += kThreads) {
      const int r = q0 + e / 32, c4 = (e % 32) * 4;
      const uint32_t local = smem_u32(dump + r * kDumpStride + c4);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < Z; ++q) {
        const float4 v = ld_cluster_f4(map_to_cta(local, q));
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      *reinterpret_cast<float4 *>(out + r * 128 + c4) = acc;
    }
    if (z == 0 && threadIdx.x < 128) {
      const uint32_t local = smem_u32(colsum + threadIdx.x);
      float acc = 0.f;
      for (int q = 0; q < Z; ++q) acc += ld_cluster_f32(map_to_cta(local, q));
      p.ksum[(long long)m * 128 + threadIdx.x] = acc;
    }
  }
  cluster_sync();  // peers are done reading this CTA's shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

cudaError_t launch_kproj_tc(int dtype_is_bf16, const KProjMaps &maps, const KProjParams &p,
                            cudaStream_t stream) {
  const int smem = KpSmem::kBytes + 1024;
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
    cudaError_t err = cudaFuncSetAttribute(kproj_tc_kernel<__nv_bfloat16>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    err = cudaLaunchKernelEx(&cfg, kproj_tc_kernel<__nv_bfloat16>, maps, p);
    if (err != cudaSuccess) return err;
  } else {
    cudaError_t err = cudaFuncSetAttribute(kproj_tc_kernel<__half>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    err = cudaLaunchKernelEx(&cfg, kproj_tc_kernel<__half>, maps, p);
    if (err != cudaSuccess) return err;
  }
  return cudaGetLastError();
}

}  // namespace rtk

