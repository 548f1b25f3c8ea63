// Fused Key projection + RoPE + covariance sums on the 5th-generation tensor cores.
//
// The attention adapters compute the prefill Keys as k_proj(X) -> RoPE
// (llava_next/llama_visionzip.py:144-153, qwen/qwen2_5vl_visionzip.py:932-942),
// and ChannelPruner.update_rotatek then reads the visual Keys again for their
// mean and covariance (kv_pruning_utils.py:112-115).  This kernel produces the
// post-RoPE Keys and, in the same pass, the raw sums sum_s k k^T and sum_s k of
// the visual span -- the inputs of the eigensolver prologue -- so the covariance
// pass over K disappears.
//
// CTA pairs.  A cluster of two CTAs computes a {256 tokens x 256 channels}
// tile -- a pair of KV heads -- with tcgen05.mma.cta_group::2 (M = 256, N = 256,
// K = 16): CTA r loads its 128 token rows of X and W's rows of head r of the
// pair, so each CTA moves half the operand bytes of a 1-CTA 128 x 256 tile for
// the same flops (shared memory is what bounds this GEMM on one SM).  Rank 0
// issues the MMAs; D's rows of CTA r are its own tokens, both heads.
//
// Per CTA (320 threads, one CTA per SM):
//   warp 0     TMA producer: X box {64 hidden x 128 tokens} and W box {64 x 128
//              channels} per 64-wide hidden chunk into a 5-stage ring; both
//              CTAs' bytes complete on rank 0's full barrier
//   warp 1     TMEM (512 columns, allocated for the pair); on rank 0 the MMA
//              issuer: projection into columns 0-255, and per staged tile the
//              covariance MMAs (M = N = 256, K = 256 tokens, both operands the
//              staging tiles read MN-major) into columns 256-511 -- issued
//              right after the next tile's projection, while its accumulator
//              drains
//   warps 2-9  epilogue, group h = head h of the pair, one token row per
//              thread: drain TMEM (+ bias, round) into registers, free the
//              accumulator, RoPE with torch's roundings, then write the row
//              into head h's staging tile -- in CTA h, through DSMEM when that
//              is the other CTA.  CTA h's staging thus holds head h for all
//              256 tokens: the TMA-store source, the covariance operand (D's
//              rows in CTA h are head h's channels, and its columns 128 h ...
//              hold cov(head h); the other 128 columns get cross terms that are
//              never read), and the source of head h's channel sums.
//
// Work split: each span (prompt, visual, text) is tiled from its own start in
// 128-token tiles, and its tiles are taken two at a time (CTA 0, CTA 1) -- a
// pair step never mixes spans.  The B x steps items are cut into contiguous
// ranges over groups of ceil(H / 2) pairs; the pairs of a group (one per head
// pair) walk the same range in step, so an X tile comes from HBM once.  When a
// range leaves a b, its covariance and channel-sum partials go to the
// workspace; a second kernel sums them in a fixed order (deterministic).
// Rows past the end of their span are zeroed (no covariance contribution) and
// clipped by the span's output tensor map.  No multicast loads.
#include <type_traits>

#include "builder.h"
#include "tcgen05.cuh"

namespace rtk {
namespace {

constexpr int kRows = 128;                   // tokens per CTA tile
constexpr int kXBox = 128 * 128;             // {64 hidden x 128 tokens}, 16-bit
constexpr int kWBox = 128 * 128;             // {64 hidden x 128 channels}
constexpr int kStageBytes = kXBox + kWBox;   // 32 KB
constexpr int kStages = 5;
constexpr int kStageTile = 256 * 128;        // {64 channels x 256 tokens} staging box
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t kCovCol = 256;            // covariance accumulator columns 256-511
constexpr uint32_t kTmemCols = 512;
constexpr uint16_t kPairMask = 0x3;          // both CTAs of the (two-CTA) cluster

struct KpSmem {
  static constexpr int kRing = 0;
  static constexpr int kStage = kRing + kStages * kStageBytes;   // channels 0-63 | 64-127, 256 rows each
  static constexpr int kBar = kStage + 2 * kStageTile;
  // full[S], empty[S], acc_full, acc_empty, staged, filled, free[2], cov_done, cov_flushed
  static constexpr int kNumBars = 2 * kStages + 8;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kAbort = kTmemSlot + 4;                     // bounded-wait abort flag
  static constexpr int kBias = (kAbort + 4 + 15) & ~15;           // fp32 [2][128]
  static constexpr int kBytes = kBias + 256 * 4;
  static_assert(kStage % 1024 == 0 && kStageBytes % 1024 == 0, "swizzled boxes need 1024-byte alignment");
  // + 1024 alignment slack; no static shared memory in the kernel (it would
  // sit in front of the 1024-aligned dynamic array)
  static_assert(kBytes + 1024 <= 232448, "shared memory budget");
};

// The three spans of a sequence, their 128-token tiles and pair steps (two
// tiles of one span per step).
struct Spans {
  int start[3], end[3], tiles[3], first[4];   // first: first pair step of each span

  __device__ void init(int seq, int vs, int vl) {
    start[0] = 0; end[0] = vs;
    start[1] = vs; end[1] = vs + vl;
    start[2] = vs + vl; end[2] = seq;
    first[0] = 0;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      tiles[i] = (end[i] - start[i] + kRows - 1) / kRows;
      first[i + 1] = first[i] + (tiles[i] + 1) / 2;
    }
  }
  __device__ int steps() const { return first[3]; }
  __device__ int span_of(int step) const { return step < first[1] ? 0 : step < first[2] ? 1 : 2; }
};

// Where CTA r's tile of a pair step lies.
struct StepTile {
  int span, start, end, row0;   // span, its first / end token, the tile's first token
  bool exists;                  // the span has this tile (the last step of a span may have one)
};

__device__ __forceinline__ StepTile step_tile(const Spans &sp, int step, int r) {
  StepTile t;
  t.span = sp.span_of(step);
  t.start = t.end = t.row0 = 0;
  t.exists = false;
#pragma unroll
  for (int i = 0; i < 3; ++i)
    if (i == t.span) {
      const int tile = 2 * (step - sp.first[i]) + r;
      t.start = sp.start[i];
      t.end = sp.end[i];
      t.row0 = sp.start[i] + tile * kRows;
      t.exists = tile < sp.tiles[i];
    }
  return t;
}

// A group's share of the B x steps items, and the b / step behind an index.
struct Range {
  int begin, end, steps_per_b;
  __device__ int unit(int j) const { return j / steps_per_b; }
  __device__ int step(int j) const { return j % steps_per_b; }
  // last index of the range that belongs to unit(j)
  __device__ int unit_last(int j) const {
    const int u_end = (unit(j) + 1) * steps_per_b;
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
  // two batches of four loads per wait: the accumulator is released sooner
#pragma unroll
  for (int c4 = 0; c4 < 8; c4 += 4) {
    uint32_t r[4][16];
#pragma unroll
    for (int c = 0; c < 4; ++c) tmem_ld16_nowait(tmem_row + 16 * (c4 + c), r[c]);
    tmem_wait_ld();
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int e = 0; e < 16; e += 2)
        k[8 * (c4 + c) + e / 2] = pack2<T>(__fadd_rn(__uint_as_float(r[c][e]), bias[16 * (c4 + c) + e]),
                                           __fadd_rn(__uint_as_float(r[c][e + 1]), bias[16 * (c4 + c) + e + 1]));
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
    kproj_pair_kernel(const __grid_constant__ KProjMaps maps, const KProjParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem + KpSmem::kBar);   // rank 0's is used
  uint64_t *empty_bar = full_bar + kStages;
  uint64_t *acc_full = empty_bar + kStages;   // projection accumulator ready (both CTAs)
  uint64_t *acc_empty = acc_full + 1;         // rank 0: drained, one arrival per epilogue warp of the pair
  uint64_t *staged_bar = acc_empty + 1;       // rank 0: both staging tiles written (4 group arrivals)
  uint64_t *filled_bar = staged_bar + 1;      // this CTA's staging tile written by both CTAs
  uint64_t *free_bar = filled_bar + 1;        // [2]: staging tile of head h read by its store and MMAs
  uint64_t *cov_done = free_bar + 2;          // a unit's covariance MMAs completed (both CTAs)
  uint64_t *cov_flushed = cov_done + 1;       // rank 0: ... and read out by both CTAs
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + KpSmem::kTmemSlot);
  float *bias_s = reinterpret_cast<float *>(smem + KpSmem::kBias);
  unsigned char *stage = smem + KpSmem::kStage;
  int &abort_flag = *reinterpret_cast<int *>(smem + KpSmem::kAbort);

  const uint32_t r = cluster_rank();                 // 0: issues the MMAs
  const int pairs = (p.heads + 1) / 2;
  const int clusters = gridDim.x / 2;
  const int groups = clusters / pairs;
  const int cl = blockIdx.x / 2;
  const int grp = cl / pairs, hp = cl % pairs;       // this pair's group and head pair
  const int nh = p.heads - 2 * hp < 2 ? p.heads - 2 * hp : 2;
  Spans sp;
  sp.init(p.seq, p.vis_start, p.vis_len);
  const long long total = (long long)p.batch * sp.steps();
  Range rg;
  rg.steps_per_b = sp.steps();
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
    mbar_init(acc_empty, 2 * kEpiWarps);
    mbar_init(staged_bar, 4);
    mbar_init(filled_bar, 2);
    mbar_init(&free_bar[0], 2);    // the tile's MMA side + its store
    mbar_init(&free_bar[1], 2);
    mbar_init(cov_done, 1);
    mbar_init(cov_flushed, 2 * kEpiWarps);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  cluster_sync();   // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs): bytes complete on rank 0's full barrier
    if (lane == 0) {
      tma_prefetch_desc(&maps.x);
      tma_prefetch_desc(&maps.w);
      const uint32_t full0 = map_to_cta(smem_u32(full_bar), 0);
      int it = 0;
      bool ok = true;
      for (int j = rg.begin; j < rg.end && ok; ++j) {
        const int b = rg.unit(j);
        const StepTile mine = step_tile(sp, rg.step(j), static_cast<int>(r));
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int st = it % kStages;
          if (!mbar_wait_cluster_bounded(&empty_bar[st], ((it / kStages) & 1) ^ 1, &abort_flag, status)) {
            ok = false;
            break;
          }
          unsigned char *dst = smem + KpSmem::kRing + st * kStageBytes;
          if (r == 0) mbar_arrive_expect_tx(&full_bar[st], 2 * kStageBytes);
          tma_load_3d_pair(dst, &maps.x, kc * 64, mine.row0, b, full0 + st * 8);
          tma_load_2d_pair(dst + kXBox, &maps.w, kc * 64, hp * 256 + 128 * static_cast<int>(r), full0 + st * 8);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (rank 0)
    if (lane == 0 && r == 0) {
      constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t kIdProj = idesc_f16(kFmt, 0u, 0u, 256u, 256u);   // X, W K-major
      constexpr uint32_t kIdCov = idesc_f16(kFmt, 1u, 1u, 256u, 256u);    // staging MN-major
      const uint32_t stage_addr = smem_u32(stage);
      uint32_t free_at[2][2];                        // [head][cta]
      for (int h = 0; h < 2; ++h)
        for (int c = 0; c < 2; ++c) free_at[h][c] = map_to_cta(smem_u32(&free_bar[h]), c);
      // staging uses (one per pair step) in order
      int uj = rg.begin, un = 0, nflush = 0, cur_unit = -1;
      bool started = false;
      auto take_use = [&]() {
        mbar_wait_cluster_bounded(staged_bar, un & 1, &abort_flag, status);
        const int u = rg.unit(uj);
        if (u != cur_unit) {
          // the previous unit's accumulators must have been read out
          if (cur_unit >= 0) mbar_wait_cluster_bounded(cov_flushed, (nflush - 1) & 1, &abort_flag, status);
          cur_unit = u;
          started = false;
        }
        if (sp.span_of(rg.step(uj)) == 1) {
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < 2 * kRows / 16; ++ks) {
            const uint64_t d = smem_desc_sw128(stage_addr + ks * 2048, kStageTile, 1024);
            umma_pair_f16(tmem + kCovCol, d, d, kIdCov, (started || ks > 0) ? 1u : 0u);
          }
          started = true;
          umma_pair_commit(&free_bar[0], kPairMask);
          umma_pair_commit(&free_bar[1], kPairMask);
        } else {
          for (int h = 0; h < 2; ++h)
            for (int c = 0; c < 2; ++c) mbar_arrive_cluster(free_at[h][c]);
        }
        ++un;
        if (uj == rg.unit_last(uj)) {
          umma_pair_commit(cov_done, kPairMask);   // the unit's last use: its sums are complete
          ++nflush;
        }
        ++uj;
      };
      int it = 0;
      for (int i = 0; i < nt; ++i) {
        mbar_wait_cluster_bounded(acc_empty, (i & 1) ^ 1, &abort_flag, status);
        tc_fence_after();
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int st = it % kStages;
          mbar_wait_cluster_bounded(&full_bar[st], (it / kStages) & 1, &abort_flag, status);
          tc_fence_after();
          const uint32_t base = smem_u32(smem + KpSmem::kRing + st * kStageBytes);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t da = smem_desc_sw128(base + ks * 32, 16, 1024);
            const uint64_t db = smem_desc_sw128(base + kXBox + ks * 32, 16, 1024);
            umma_pair_f16(tmem, da, db, kIdProj, (kc > 0 || ks > 0) ? 1u : 0u);
          }
          umma_pair_commit(&empty_bar[st], kPairMask);   // both CTAs' stages free once read
        }
        umma_pair_commit(acc_full, kPairMask);
        // the previous step's covariance MMAs keep the tensor pipe busy while
        // the epilogue drains this accumulator
        while (uj < rg.begin + i) take_use();
      }
      while (uj < rg.end) take_use();
    }
  } else {
    // ---------------- epilogue: warp group hh handles head hh of the pair
    const int e = warp - 2;
    const int hh = e >> 2;
    const int quarter = warp & 3;                  // TMEM lanes this warp may read
    const int row = 32 * quarter + lane;           // token row (projection) / channel (covariance)
    const int gt = (e & 3) * 32 + lane;            // thread index inside the group
    const uint32_t tmem_lane = tmem + ((uint32_t)(32 * quarter) << 16);
    const bool owner = hh == static_cast<int>(r);   // head hh's staging tile lives in this CTA
    const bool has = hh < nh;
    const int head = 2 * hp + hh;
    const uint32_t stage_hh = map_to_cta(smem_u32(stage), hh);
    const uint32_t filled_hh = map_to_cta(smem_u32(filled_bar), hh);
    const uint32_t staged0 = map_to_cta(smem_u32(staged_bar), 0);
    const uint32_t acc_empty0 = map_to_cta(smem_u32(acc_empty), 0);
    const uint32_t cov_flushed0 = map_to_cta(smem_u32(cov_flushed), 0);
    const uint32_t free_mine = map_to_cta(smem_u32(&free_bar[hh]), r);
    const uint32_t free_peer = map_to_cta(smem_u32(&free_bar[hh]), r ^ 1u);
    const int chunk = gt & 15, rgp = gt >> 4;      // channel sums: 8 channels x 32 rows
    float ks_acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) ks_acc[k] = 0.f;
    const T *bias_g = static_cast<const T *>(p.bias);
    int nflush = 0, cur_unit = -1;
    bool stored = false, unit_vis = false;
    for (int i = 0; i < nt; ++i) {
      const int j = rg.begin + i;
      const int b = rg.unit(j), step = rg.step(j);
      const StepTile mine = step_tile(sp, step, static_cast<int>(r));
      if (b != cur_unit) {   // this head's bias
        named_barrier_sync(1 + hh, 128);
        bias_s[128 * hh + gt] = (has && bias_g != nullptr) ? to_f32<T>(bias_g[head * 128 + gt]) : 0.f;
        named_barrier_sync(1 + hh, 128);
        cur_unit = b;
        unit_vis = false;
      }
      mbar_wait_cluster_bounded(acc_full, i & 1, &abort_flag, status);
      tc_fence_after();
      uint32_t kv[64];
      if (has) drain_row<T>(tmem_lane + 128 * hh, bias_s + 128 * hh, kv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0);   // the accumulator may be overwritten
      if (has) {
        const int t = mine.row0 + row;
        const bool valid = mine.exists && t < mine.end;
        const long long cs = (long long)b * p.cs_sb + (long long)t * p.cs_ss;
        rope_row<T>(static_cast<const T *>(p.cos) + cs, static_cast<const T *>(p.sin) + cs, valid, kv);
      }
      // head hh's staging tile is free once the previous step's store and MMAs have read it
      if (i > 0) mbar_wait_cluster_bounded(&free_bar[hh], (i - 1) & 1, &abort_flag, status);
      if (has) {
        const int srow = static_cast<int>(r) * kRows + row;
#pragma unroll
        for (int c8 = 0; c8 < 16; ++c8)
          st_cluster_v4(stage_hh + (c8 >> 3) * kStageTile + swizzled_offset<128>(srow, (c8 & 7) * 8),
                        make_uint4(kv[4 * c8], kv[4 * c8 + 1], kv[4 * c8 + 2], kv[4 * c8 + 3]));
      }
      fence_proxy_async_cluster();
      named_barrier_sync(1 + hh, 128);
      if (gt == 0) {
        mbar_arrive_cluster(staged0);
        mbar_arrive_cluster(filled_hh);
      }
      if (owner) {
        // both CTAs' rows of head hh are in this CTA's staging tile
        mbar_wait_cluster_bounded(filled_bar, i & 1, &abort_flag, status);
        fence_proxy_async_smem();
        if (gt == 0 && has) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const StepTile tl = step_tile(sp, step, half);
            if (!tl.exists) continue;
            for (int c = 0; c < 2; ++c)
              tma_store_4d(&maps.k_out[tl.span], stage + c * kStageTile + half * kRows * 128, 64 * c,
                           tl.row0 - tl.start, head, b);
          }
          bulk_commit_group();
          stored = true;
        }
        if (has && mine.span == 1) {
          unit_vis = true;
          const unsigned char *box = stage + (chunk >> 3) * kStageTile;
#pragma unroll 4
          for (int rr = 0; rr < 32; ++rr) {
            const uint4 v = *reinterpret_cast<const uint4 *>(box + swizzled_offset<128>(rgp * 32 + rr, (chunk & 7) * 8));
            float f[8];
            unpack8<T>(v, f);
#pragma unroll
            for (int k = 0; k < 8; ++k) ks_acc[k] += f[k];
          }
        }
        named_barrier_sync(1 + hh, 128);           // every thread is done reading the staging tile
        if (gt == 0) {
          if (stored) bulk_wait_read_all();
          mbar_arrive_cluster(free_mine);
          mbar_arrive_cluster(free_peer);
        }
      }
      if (j == rg.unit_last(j)) {
        // end of this b in the range: head hh's covariance and channel-sum partials out
        mbar_wait_cluster_bounded(cov_done, nflush & 1, &abort_flag, status);
        tc_fence_after();
        if (owner && has) {
          float *part = p.part + (((long long)(grp + b) * pairs + hp) * 2 + hh) * kKProjPartFloats;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t v[16];
            if (unit_vis) {
              tmem_ld16_nowait(tmem_lane + kCovCol + 128 * hh + 16 * c, v);
              tmem_wait_ld();
            } else {
#pragma unroll
              for (int k = 0; k < 16; ++k) v[k] = 0u;
            }
#pragma unroll
            for (int k = 0; k < 16; k += 4)
              *reinterpret_cast<float4 *>(part + row * 128 + 16 * c + k) =
                  make_float4(__uint_as_float(v[k]), __uint_as_float(v[k + 1]), __uint_as_float(v[k + 2]),
                              __uint_as_float(v[k + 3]));
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
        if (lane == 0) mbar_arrive_cluster(cov_flushed0);
        ++nflush;
      }
    }
    if (gt == 0 && stored) bulk_wait_all();
  }
  __syncthreads();
  cluster_sync();   // the peer is done with this CTA's shared and tensor memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

// cov / ksum of (b, h): the sum, in group order, of the partials of the
// groups whose range meets b's items.  Block (m, y) sums the 1024 floats
// [1024 y, 1024 y + 1024) of matrix m; y == 0 also the channel sums.
constexpr int kReduceSplit = 128 * 128 / 1024;

__global__ void __launch_bounds__(256)
    kproj_reduce_kernel(const KProjParams p, int steps_per_b) {
  const int pairs = (p.heads + 1) / 2;
  const int groups = p.grid / (2 * pairs);
  const int m = blockIdx.x;                 // b * heads + head
  const int b = m / p.heads, head = m % p.heads;
  const int hp = head / 2, hh = head & 1;
  const long long total = (long long)p.batch * steps_per_b;
  const long long lo = (long long)b * steps_per_b, hi = lo + steps_per_b;
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

int kproj_steps_per_b(int seq, int vis_start, int vis_len) {
  const int t0 = (vis_start + kRows - 1) / kRows, t1 = (vis_len + kRows - 1) / kRows,
            t2 = (seq - vis_start - vis_len + kRows - 1) / kRows;
  return (t0 + 1) / 2 + (t1 + 1) / 2 + (t2 + 1) / 2;
}

int kproj_max_clusters(int dtype_is_bf16) {
  const int smem = KpSmem::kBytes + 1024;
  auto kernel = dtype_is_bf16 ? kproj_pair_kernel<__nv_bfloat16> : kproj_pair_kernel<__half>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) return 0;
  return n;
}

cudaError_t launch_kproj_tc(int dtype_is_bf16, const KProjMaps &maps, const KProjParams &p,
                            cudaStream_t stream) {
  const int smem = KpSmem::kBytes + 1024;
  auto kernel = dtype_is_bf16 ? kproj_pair_kernel<__nv_bfloat16> : kproj_pair_kernel<__half>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, kernel, maps, p);
  if (err != cudaSuccess) return err;
  kproj_reduce_kernel<<<dim3(p.batch * p.heads, kReduceSplit), 256, 0, stream>>>(
      p, kproj_steps_per_b(p.seq, p.vis_start, p.vis_len));
  return cudaGetLastError();
}

}  // namespace rtk


