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
// Work: the 128-token tiles of a sequence run over the prompt, visual and
// text spans, each span tiled from its own start.  The grid (one CTA per SM,
// 320 threads) is groups x P CTAs, P = ceil(H / 2) head pairs: the B x T
// (b, tile) items are split into contiguous ranges over the groups, and the P
// CTAs of a group walk the same range in step, CTA p producing head pair p --
// so a hidden-state tile comes from HBM once and from L2 for the other pairs.
// A unit is (b, head pair): its sums are flushed when a range leaves a b.
//   warp 0     TMA producer: per tile and 64-wide hidden chunk an X box
//              {64 x 128 tokens} and a W box {64 x 256 channels} (128B
//              swizzle) into a 4-stage ring; W rows past H * 128 read as zero
//   warp 1     TMEM owner (512 columns) and MMA issuer: per chunk four
//              tcgen05.mma kind::f16 M=128 N=256 K=16 (both operands K-major)
//              into the projection accumulator (columns 0-255, head h of the
//              pair in 128 h ...); each staged visual (tile, head) then gets
//              eight M=128 N=128 K=16 MMAs adding K^T K into that head's
//              covariance accumulator (columns 256 + 128 h) from the staging
//              tile read MN-major, interleaved with the next tile's chunks
//   warps 2-9  epilogue, one (token row, head) per thread: drain TMEM (+ bias,
//              round) into registers and free the accumulator, then RoPE with
//              torch's roundings, a 128B-swizzled staging tile (TMA-store
//              source and covariance operand, used by the two heads in turn),
//              channel sums of visual tiles; at the end of each unit in the
//              range, the covariance and channel-sum partials go to the
//              workspace
// A second kernel sums each unit's partials in a fixed order (deterministic).
// Rows past the end of their span are zeroed (no covariance contribution) and
// clipped by the span's output tensor map.
#include <type_traits>

#include "builder.h"
#include "tcgen05.cuh"

namespace rtk {
namespace {

constexpr int kRows = 128;                   // tokens per tile
constexpr int kXBox = 128 * 128;             // {64 hidden x 128 tokens}, 16-bit
constexpr int kWBox = 256 * 128;             // {64 hidden x 256 channels}
constexpr int kStageBytes = kXBox + kWBox;   // 48 KB
constexpr int kStages = 4;
constexpr int kOutBox = 128 * 128;           // {64 channels x 128 tokens}
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t kCovCol = 256;            // head h: columns 256 + 128 h
constexpr uint32_t kTmemCols = 512;

struct KpSmem {
  static constexpr int kRing = 0;
  static constexpr int kStage = kRing + kStages * kStageBytes;   // channels 0-63 | 64-127
  static constexpr int kBar = kStage + 2 * kOutBox;
  // full[kStages], empty[kStages], acc_full, acc_empty, staged, staging_free, cov_done, cov_flushed
  static constexpr int kNumBars = 2 * kStages + 6;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kAbort = kTmemSlot + 4;                     // bounded-wait abort flag
  static constexpr int kBias = (kAbort + 4 + 15) & ~15;           // fp32 [256]
  static constexpr int kBytes = kBias + 256 * 4;
  static_assert(kStage % 1024 == 0 && kStageBytes % 1024 == 0, "swizzled boxes need 1024-byte alignment");
  // + 1024 alignment slack; no static shared memory in the kernel (it would
  // sit in front of the 1024-aligned dynamic array)
  static_assert(kBytes + 1024 <= 232448, "shared memory budget");
};

// The three spans of a unit's tokens and their 128-token tiles.
struct Spans {
  int start0, start1, start2, end0, end1, end2, first1, first2, total;

  __device__ void init(int seq, int vs, int vl) {
    start0 = 0; end0 = vs;
    start1 = vs; end1 = vs + vl;
    start2 = vs + vl; end2 = seq;
    first1 = (vs + kRows - 1) / kRows;
    first2 = first1 + (vl + kRows - 1) / kRows;
    total = first2 + (seq - vs - vl + kRows - 1) / kRows;
  }
  // span index, first token of the tile, end of its span, first token of its span
  __device__ void locate(int tile, int &span, int &row0, int &end, int &start) const {
    if (tile < first1) { span = 0; start = start0; end = end0; row0 = tile * kRows; }
    else if (tile < first2) { span = 1; start = start1; end = end1; row0 = start1 + (tile - first1) * kRows; }
    else { span = 2; start = start2; end = end2; row0 = start2 + (tile - first2) * kRows; }
  }
  __device__ bool visual(int tile) const { return tile >= first1 && tile < first2; }
};

// A group's share of the B * T (b, tile) items, and the b / tile behind an index.
struct Range {
  int begin, end, tiles_per_unit;
  __device__ int unit(int j) const { return j / tiles_per_unit; }
  __device__ int tile(int j) const { return j % tiles_per_unit; }
  // last index of the range that belongs to unit(j)
  __device__ int unit_last(int j) const {
    const int u_end = (unit(j) + 1) * tiles_per_unit;
    return (u_end < end ? u_end : end) - 1;
  }
};

__host__ __device__ inline long long range_begin(int c, long long total, int grid) {
  return (long long)c * total / grid;
}

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

// Drain one head's 128 accumulator columns of this thread's row:
// k = round(acc + bias), packed in pairs (channels 2j, 2j+1 in k[j]).
template <typename T>
__device__ __forceinline__ void drain_row(uint32_t tmem_row, const float *bias, uint32_t (&k)[64]) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint32_t r[16];
    tmem_ld16_nowait(tmem_row + 16 * c, r);
    tmem_wait_ld();
#pragma unroll
    for (int e = 0; e < 16; e += 2)
      k[8 * c + e / 2] = pack2<T>(__fadd_rn(__uint_as_float(r[e]), bias[16 * c + e]),
                                  __fadd_rn(__uint_as_float(r[e + 1]), bias[16 * c + e + 1]));
  }
}

// RoPE on a drained row, in place:
//   out_lo = round(round(k_lo cos_lo) - round(k_hi sin_lo))   channels d < 64
//   out_hi = round(round(k_hi cos_hi) + round(k_lo sin_hi))   channels d + 64
// which is torch's  k * cos + rotate_half(k) * sin  in the Keys' dtype.
// Rows past the end of their span become zero.
template <typename T>
__device__ __forceinline__ void rope_row(const T *crow, const T *srow, bool valid, uint32_t (&k)[64]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int d = 8 * q;
    if (!valid) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        k[d / 2 + e] = 0u;
        k[(d + 64) / 2 + e] = 0u;
      }
      continue;
    }
    float cl[8], ch[8], sl[8], sh[8], lo[8], hi[8];
    unpack8<T>(__ldg(reinterpret_cast<const uint4 *>(crow + d)), cl);
    unpack8<T>(__ldg(reinterpret_cast<const uint4 *>(crow + d + 64)), ch);
    unpack8<T>(__ldg(reinterpret_cast<const uint4 *>(srow + d)), sl);
    unpack8<T>(__ldg(reinterpret_cast<const uint4 *>(srow + d + 64)), sh);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      unpack2<T>(k[(d + e) / 2], lo[e], lo[e + 1]);
      unpack2<T>(k[(d + 64 + e) / 2], hi[e], hi[e + 1]);
    }
    float olo[8], ohi[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      olo[e] = __fsub_rn(round_to<T>(__fmul_rn(lo[e], cl[e])), round_to<T>(__fmul_rn(hi[e], sl[e])));
      ohi[e] = __fadd_rn(round_to<T>(__fmul_rn(hi[e], ch[e])), round_to<T>(__fmul_rn(lo[e], sh[e])));
    }
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      k[(d + e) / 2] = pack2<T>(olo[e], olo[e + 1]);
      k[(d + 64 + e) / 2] = pack2<T>(ohi[e], ohi[e + 1]);
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
  uint64_t *acc_full = empty_bar + kStages;   // projection accumulator ready
  uint64_t *acc_empty = acc_full + 1;         // drained (one arrival per epilogue warp)
  uint64_t *staged_bar = acc_empty + 1;       // staging use n written (phase n)
  uint64_t *free_bar = staged_bar + 1;        // use n read by its TMA store and its MMAs
  uint64_t *cov_done = free_bar + 1;          // a unit's covariance MMAs completed
  uint64_t *cov_flushed = cov_done + 1;       // ... and its accumulators read out
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + KpSmem::kTmemSlot);
  float *bias_s = reinterpret_cast<float *>(smem + KpSmem::kBias);
  unsigned char *stage = smem + KpSmem::kStage;
  int &abort_flag = *reinterpret_cast<int *>(smem + KpSmem::kAbort);

  const int pairs = (p.heads + 1) / 2;
  const int groups = gridDim.x / pairs;
  const int grp = blockIdx.x / pairs, hp = blockIdx.x % pairs;   // this CTA's group and head pair
  const int nh = p.heads - 2 * hp < 2 ? p.heads - 2 * hp : 2;     // heads of the pair (2, or 1 if H is odd)
  Spans sp;
  sp.init(p.seq, p.vis_start, p.vis_len);
  const long long total = (long long)p.batch * sp.total;
  Range rg;
  rg.tiles_per_unit = sp.total;
  rg.begin = static_cast<int>(range_begin(grp, total, groups));
  rg.end = static_cast<int>(range_begin(grp + 1, total, groups));
  const int nt = rg.end - rg.begin;
  const int nk = p.hidden / 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned int *status = p.status;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kEpiWarps);
    mbar_init(staged_bar, 1);
    mbar_init(free_bar, 2);            // the use's TMA store + its MMA side
    mbar_init(cov_done, 1);
    mbar_init(cov_flushed, kEpiWarps);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
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
      for (int j = rg.begin; j < rg.end && ok; ++j) {
        const int b = rg.unit(j);
        int span, row0, end, start;
        sp.locate(rg.tile(j), span, row0, end, start);
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int st = it % kStages;
          if (!mbar_wait_bounded(&empty_bar[st], ((it / kStages) & 1) ^ 1, &abort_flag, status)) {
            ok = false;
            break;
          }
          unsigned char *dst = smem + KpSmem::kRing + st * kStageBytes;
          mbar_arrive_expect_tx(&full_bar[st], kStageBytes);
          tma_load_3d(dst, &maps.x, kc * 64, row0, b, &full_bar[st]);
          tma_load_2d(dst + kXBox, &maps.w, kc * 64, hp * 256, &full_bar[st]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t kIdProj = idesc_f16(kFmt, 0u, 0u, 128u, 256u);   // X, W K-major
      constexpr uint32_t kIdCov = idesc_f16(kFmt, 1u, 1u, 128u, 128u);    // K^T, K MN-major
      const uint32_t stage_addr = smem_u32(stage);
      // staging uses in order: tile uj, head uh; un uses done, nflush units done
      int uj = rg.begin, uh = 0, un = 0, nflush = 0, cur_unit = -1;
      bool started[2] = {false, false};
      auto take_use = [&](bool block) -> bool {
        if (block) {
          mbar_wait_bounded(staged_bar, un & 1, &abort_flag, status);
        } else if (!mbar_try_wait(staged_bar, un & 1)) {
          return false;
        }
        const int u = rg.unit(uj), tile = rg.tile(uj);
        if (u != cur_unit) {
          // the previous unit's accumulators must have been read out
          if (cur_unit >= 0) mbar_wait_bounded(cov_flushed, (nflush - 1) & 1, &abort_flag, status);
          cur_unit = u;
          started[0] = started[1] = false;
        }
        if (sp.visual(tile)) {
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < kRows / 16; ++ks) {
            const uint64_t d = smem_desc_sw128(stage_addr + ks * 2048, kOutBox, 1024);
            umma_f16(tmem + kCovCol + 128 * uh, d, d, kIdCov, (started[uh] || ks > 0) ? 1u : 0u);
          }
          started[uh] = true;
          umma_commit(free_bar);
        } else {
          mbar_arrive(free_bar);
        }
        ++un;
        if (uh + 1 >= nh) {
          if (uj == rg.unit_last(uj)) {
            umma_commit(cov_done);   // the unit's last use: its sums are complete
            ++nflush;
          }
          ++uj;
          uh = 0;
        } else {
          ++uh;
        }
        return true;
      };
      int it = 0;
      for (int i = 0; i < nt; ++i) {
        mbar_wait_bounded(acc_empty, (i & 1) ^ 1, &abort_flag, status);
        tc_fence_after();
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int st = it % kStages;
          mbar_wait_bounded(&full_bar[st], (it / kStages) & 1, &abort_flag, status);
          tc_fence_after();
          const uint32_t base = smem_u32(smem + KpSmem::kRing + st * kStageBytes);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t da = smem_desc_sw128(base + ks * 32, 16, 1024);
            const uint64_t db = smem_desc_sw128(base + kXBox + ks * 32, 16, 1024);
            umma_f16(tmem, da, db, kIdProj, (kc > 0 || ks > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[st]);   // stage free once these MMAs have read it
          // covariance updates of earlier tiles, as their uses get staged
          while (uj < rg.begin + i && take_use(false)) {
          }
        }
        // the previous tile's uses go before this accumulator is handed over
        while (uj < rg.begin + i) take_use(true);
        umma_commit(acc_full);
      }
      while (uj < rg.end) take_use(true);
    }
  } else {
    // ---------------- epilogue: warp group hh handles head hh of the pair
    const int e = warp - 2;
    const int hh = e >> 2;
    const int quarter = warp & 3;                  // TMEM lanes this warp may read
    const int row = 32 * quarter + lane;           // token row (projection) / channel (covariance)
    const int gt = (e & 3) * 32 + lane;            // thread index inside the group
    const uint32_t tmem_lane = tmem + ((uint32_t)(32 * quarter) << 16);
    const int chunk = gt & 15, rgp = gt >> 4;      // channel sums: 8 channels x 16 rows
    float ks_acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) ks_acc[k] = 0.f;
    const T *bias_g = static_cast<const T *>(p.bias);
    int un = 0, nflush = 0, cur_unit = -1;
    bool stored = false, unit_vis = false;
    for (int i = 0; i < nt; ++i) {
      const int j = rg.begin + i;
      const int u = rg.unit(j), tile = rg.tile(j);
      const int b = u;
      const bool has = hh < nh;
      const int head = 2 * hp + hh;
      int span, row0, end, start;
      sp.locate(tile, span, row0, end, start);
      if (u != cur_unit) {   // this head's bias
        named_barrier_sync(1 + hh, 128);
        bias_s[128 * hh + gt] = (has && bias_g != nullptr) ? to_f32<T>(bias_g[head * 128 + gt]) : 0.f;
        named_barrier_sync(1 + hh, 128);
        cur_unit = u;
        unit_vis = false;
      }
      mbar_wait_bounded(acc_full, i & 1, &abort_flag, status);
      tc_fence_after();
      uint32_t kv[64];
      if (has) drain_row<T>(tmem_lane + 128 * hh, bias_s + 128 * hh, kv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);       // the accumulator may be overwritten
      const int use = un + hh;
      if (has) {
        const int t = row0 + row;
        const bool valid = t < end;
        const long long cs = (long long)b * p.cs_sb + (long long)t * p.cs_ss;
        rope_row<T>(static_cast<const T *>(p.cos) + cs, static_cast<const T *>(p.sin) + cs, valid, kv);
        // the staging tile is free once the previous use's store and MMAs have read it
        if (use > 0) mbar_wait_bounded(free_bar, (use - 1) & 1, &abort_flag, status);
#pragma unroll
        for (int c8 = 0; c8 < 16; ++c8)
          *reinterpret_cast<uint4 *>(stage + (c8 >> 3) * kOutBox + swizzled_offset<128>(row, (c8 & 7) * 8)) =
              make_uint4(kv[4 * c8], kv[4 * c8 + 1], kv[4 * c8 + 2], kv[4 * c8 + 3]);
        fence_proxy_async_smem();
        named_barrier_sync(1 + hh, 128);
        if (gt == 0) {
          tma_store_4d(&maps.k_out[span], stage, 0, row0 - start, head, b);
          tma_store_4d(&maps.k_out[span], stage + kOutBox, 64, row0 - start, head, b);
          bulk_commit_group();
          stored = true;
          mbar_arrive(staged_bar);
        }
        if (span == 1) {
          unit_vis = true;
          const unsigned char *box = stage + (chunk >> 3) * kOutBox;
#pragma unroll 4
          for (int rr = 0; rr < 16; ++rr) {
            const uint4 v = *reinterpret_cast<const uint4 *>(box + swizzled_offset<128>(rgp * 16 + rr, (chunk & 7) * 8));
            float f[8];
            unpack8<T>(v, f);
#pragma unroll
            for (int k = 0; k < 8; ++k) ks_acc[k] += f[k];
          }
        }
        named_barrier_sync(1 + hh, 128);           // every thread is done reading the staging tile
        if (gt == 0) {
          bulk_wait_read_all();
          mbar_arrive(free_bar);
        }
      }
      un += nh;
      if (j == rg.unit_last(j)) {
        // end of this unit in the range: covariance and channel-sum partials out
        mbar_wait_bounded(cov_done, nflush & 1, &abort_flag, status);
        tc_fence_after();
        if (has) {
          float *part = p.part + (((long long)(grp + b) * pairs + hp) * 2 + hh) * kKProjPartFloats;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t r[16];
            if (unit_vis) {
              tmem_ld16_nowait(tmem_lane + kCovCol + 128 * hh + 16 * c, r);
              tmem_wait_ld();
            } else {
#pragma unroll
              for (int k = 0; k < 16; ++k) r[k] = 0u;
            }
#pragma unroll
            for (int k = 0; k < 16; k += 4)
              *reinterpret_cast<float4 *>(part + row * 128 + 16 * c + k) =
                  make_float4(__uint_as_float(r[k]), __uint_as_float(r[k + 1]), __uint_as_float(r[k + 2]),
                              __uint_as_float(r[k + 3]));
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            ks_acc[k] += __shfl_xor_sync(0xffffffffu, ks_acc[k], 16);
            if ((lane & 16) == 0) part[128 * 128 + (e & 3) * 128 + chunk * 8 + k] = ks_acc[k];
            ks_acc[k] = 0.f;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(cov_flushed);
        ++nflush;
      }
    }
    if (gt == 0 && stored) bulk_wait_all();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// cov / ksum of (b, h): the sum, in group order, of the partials of the
// groups whose range meets b's items.  Block (m, y) sums the 1024 floats
// [1024 y, 1024 y + 1024) of matrix m; y == 0 also the channel sums.
constexpr int kReduceSplit = 128 * 128 / 1024;

__global__ void __launch_bounds__(256)
    kproj_reduce_kernel(const KProjParams p, int tiles_per_unit) {
  const int pairs = (p.heads + 1) / 2;
  const int groups = p.grid / pairs;
  const int m = blockIdx.x;                 // b * heads + head
  const int b = m / p.heads, head = m % p.heads;
  const int hp = head / 2, hh = head & 1;
  const long long total = (long long)p.batch * tiles_per_unit;
  const long long lo = (long long)b * tiles_per_unit, hi = lo + tiles_per_unit;
  // groups g with range_begin(g) <= lo ... range_begin(g) < hi
  const int c0 = static_cast<int>(((lo + 1) * groups + total - 1) / total) - 1;
  const int c1 = static_cast<int>((hi * groups + total - 1) / total) - 1;
  const int off = (blockIdx.y * 256 + threadIdx.x) * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float ks = 0.f;
  for (int c = c0 < 0 ? 0 : c0; c <= c1 && c < groups; ++c) {
    if (range_begin(c + 1, total, groups) <= lo || range_begin(c, total, groups) >= hi) continue;
    const float *part = p.part + (((long long)(c + b) * pairs + hp) * 2 + hh) * kKProjPartFloats;
    const float4 v = *reinterpret_cast<const float4 *>(part + off);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    if (blockIdx.y == 0 && threadIdx.x < 128) {
#pragma unroll
      for (int w = 0; w < 4; ++w) ks += part[128 * 128 + w * 128 + threadIdx.x];
    }
  }
  *reinterpret_cast<float4 *>(p.cov + (long long)m * 128 * 128 + off) = acc;
  if (blockIdx.y == 0 && threadIdx.x < 128) p.ksum[(long long)m * 128 + threadIdx.x] = ks;
}

}  // namespace

cudaError_t launch_kproj_tc(int dtype_is_bf16, const KProjMaps &maps, const KProjParams &p,
                            cudaStream_t stream) {
  const int smem = KpSmem::kBytes + 1024;
  auto kernel = dtype_is_bf16 ? kproj_tc_kernel<__nv_bfloat16> : kproj_tc_kernel<__half>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  kernel<<<p.grid, kThreads, smem, stream>>>(maps, p);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  const int tiles_per_unit = (p.vis_start + kRows - 1) / kRows + (p.vis_len + kRows - 1) / kRows +
                             (p.seq - p.vis_start - p.vis_len + kRows - 1) / kRows;
  kproj_reduce_kernel<<<dim3(p.batch * p.heads, kReduceSplit), 256, 0, stream>>>(p, tiles_per_unit);
  return cudaGetLastError();
}

}  // namespace rtk

