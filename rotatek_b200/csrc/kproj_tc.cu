// Key projection + bias + RoPE on the 5th-generation tensor cores.
//
// The attention adapters compute the prefill Keys as k_proj(X) -> RoPE
// (llava_next/llama_visionzip.py:144-153, qwen/qwen2_5vl_visionzip.py:932-942).
// This kernel writes the post-RoPE Keys of every token straight from the
// hidden states, so neither the projection's output nor a RoPE pass goes
// through HBM; the visual span's sums (kv_pruning_utils.py:112-115) are taken
// afterwards from the Keys written, by the builder's covariance kernel.
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
//   warp 1     TMEM (512 columns: two accumulators of 256); on rank 0 the MMA
//              issuer, tile i into accumulator i mod 2, so the tensor pipe
//              never waits for a drain
//   warps 2-9  epilogue, one token row per thread; warp group c (warps 2-5,
//              6-9) takes channel half c of BOTH heads: the channels
//              [32 c, 32 c + 32) and their RoPE partners + 64.  Per tile:
//              thread 0 loads the tile's cos rows into head 0's staging boxes
//              and its sin rows into head 1's (TMA); every thread drains its
//              accumulator columns (+ bias, round) into registers and frees
//              the accumulator, then applies RoPE with torch's roundings,
//              reading cos / sin from the staging boxes and writing its Keys
//              over exactly the values it read; thread 0 stores the boxes
//              with TMA (per-span tensor maps clip rows past a span).
//
//              The epilogue shares the SM's L1 / shared-memory data path with
//              the tensor core's operand reads and the TMA writes, so what it
//              costs there is what it takes from the GEMM: cos / sin come in
//              by TMA once per tile (not once per head, not per thread) and
//              the Keys leave by TMA.
//
// Work split: each span (prompt, visual, text) is tiled from its own start in
// 128-token tiles, and its tiles are taken two at a time (CTA 0, CTA 1) -- a
// pair step never mixes spans.  The B x steps items are cut into contiguous
// ranges over groups of ceil(H / 2) pairs; the pairs of a group (one per head
// pair) walk the same range in step, so an X tile comes from HBM once.  Rows
// past the end of their span are zeroed and clipped by the span's output
// tensor map.  No multicast loads.
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
constexpr int kBox = 128 * 128;              // {64 channels x 128 tokens} staging / store box
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t kAccCols = 256;           // one accumulator: 128 tokens x (2 heads x 128 channels)
constexpr uint32_t kTmemCols = 2 * kAccCols; // double-buffered
constexpr uint16_t kPairMask = 0x3;          // both CTAs of the (two-CTA) cluster

struct KpSmem {
  static constexpr int kRing = 0;
  // this CTA's 128 tokens of both heads: boxes [head][channels 0-63 | 64-127]
  static constexpr int kStage = kRing + kStages * kStageBytes;
  static constexpr int kBar = kStage + 4 * kBox;
  // full[S], empty[S], acc_full[2], acc_empty[2], cos / sin landed
  static constexpr int kNumBars = 2 * kStages + 5;
  static constexpr int kTmemSlot = kBar + kNumBars * 8;
  static constexpr int kAbort = kTmemSlot + 4;                     // bounded-wait abort flag
  static constexpr int kBytes = kAbort + 4;
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

// An epilogue thread owns one token row and one half of the channel pairs
// that RoPE couples: channels [32 c, 32 c + 32) and [64 + 32 c, 96 + 32 c) of
// BOTH heads of the pair (c = 0, 1 for the two warp groups).  Per head it
// keeps 64 values packed in 32 words: k[0..15] the low channels, k[16..31]
// the high ones.  The row's cos / sin for those channels (256 bytes) are
// fetched once and serve both heads.

// Drain one head's 64 accumulator columns of this thread's row:
// k = round(acc + bias).  `cols` addresses channel 32 c of the head, `bias`
// the same channel of the head's bias in global memory (NULL: none).  The
// bias is read with warp-uniform 16-byte loads (one L1 wavefront each; a
// broadcast 16-byte shared-memory load takes four).
template <typename T>
__device__ __forceinline__ void drain_half(uint32_t cols, const T *bias, uint32_t (&k)[32]) {
#pragma unroll
  for (int c2 = 0; c2 < 4; c2 += 2) {        // low channels, then their partners + 64
    uint32_t r[2][16];
    tmem_ld16_nowait(cols + 32 * c2, r[0]);
    tmem_ld16_nowait(cols + 32 * c2 + 16, r[1]);
    float bf[32];
    if (bias != nullptr) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float f[8];
        unpack8<T>(__ldg(reinterpret_cast<const uint4 *>(bias + 32 * c2 + 8 * q)), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) bf[8 * q + e] = f[e];
      }
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) bf[e] = 0.f;
    }
    tmem_wait_ld();
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int e = 0; e < 16; e += 2)
        k[8 * (c2 + c) + e / 2] = pack2<T>(__fadd_rn(__uint_as_float(r[c][e]), bf[16 * c + e]),
                                           __fadd_rn(__uint_as_float(r[c][e + 1]), bf[16 * c + e + 1]));
  }
}

// RoPE on 8 channel pairs of a half row (group u: low channels k[4u .. 4u+3],
// their partners + 64 in k[16 + 4u ...]), in place, for both heads (the
// second only when `both`):
//   out_lo = round(round(k_lo cos_lo) - round(k_hi sin_lo))   channels d < 64
//   out_hi = round(round(k_hi cos_hi) + round(k_lo sin_hi))   channels d + 64
// which is torch's  k * cos + rotate_half(k) * sin  in the Keys' dtype.
// Computed two channels at a time with the packed 16-bit instructions, each
// one rounding (.rn) of the exact result.  That equals torch's fp32 compute
// then round: the product of two 16-bit values is exact in fp32, and a sum
// of two 16-bit values is either exact in fp32 or so lopsided that both
// roundings return the larger operand.  .rn also keeps the compiler from
// fusing a product into the sum.
template <typename T>
__device__ __forceinline__ uint32_t mul2_rn(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <typename T>
__device__ __forceinline__ uint32_t add2_rn(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
template <typename T>
__device__ __forceinline__ uint32_t sub2_rn(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

template <typename T>
__device__ __forceinline__ void rope_pair(uint32_t cl, uint32_t ch, uint32_t sl, uint32_t sh, uint32_t &klo,
                                          uint32_t &khi) {
  const uint32_t lo = klo, hi = khi;
  klo = sub2_rn<T>(mul2_rn<T>(lo, cl), mul2_rn<T>(hi, sl));
  khi = add2_rn<T>(mul2_rn<T>(hi, ch), mul2_rn<T>(lo, sh));
}

template <typename T>
__device__ __forceinline__ void rope_group(const uint4 &clo, const uint4 &chi, const uint4 &slo, const uint4 &shi,
                                           int u, bool both, uint32_t (&k0)[32], uint32_t (&k1)[32]) {
  const uint32_t c[4] = {clo.x, clo.y, clo.z, clo.w}, d[4] = {chi.x, chi.y, chi.z, chi.w};
  const uint32_t s[4] = {slo.x, slo.y, slo.z, slo.w}, t[4] = {shi.x, shi.y, shi.z, shi.w};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    rope_pair<T>(c[w], d[w], s[w], t[w], k0[4 * u + w], k0[16 + 4 * u + w]);
    if (both) rope_pair<T>(c[w], d[w], s[w], t[w], k1[4 * u + w], k1[16 + 4 * u + w]);
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
  uint64_t *acc_full = empty_bar + kStages;   // [2] accumulator ready (both CTAs)
  uint64_t *acc_empty = acc_full + 2;         // [2] rank 0: drained, one arrival per epilogue warp of the pair
  uint64_t *cs_bar = acc_empty + 2;           // this CTA's cos / sin rows in the staging boxes
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + KpSmem::kTmemSlot);
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
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * kEpiWarps);
    }
    mbar_init(cs_bar, 1);
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
    // ---------------- MMA issuer (rank 0): tile i accumulates into buffer i & 1
    if (lane == 0 && r == 0) {
      constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t kIdProj = idesc_f16(kFmt, 0u, 0u, 256u, 256u);   // X, W K-major
      int it = 0;
      for (int i = 0; i < nt; ++i) {
        const int a = i & 1;
        if (!mbar_wait_cluster_bounded(&acc_empty[a], ((i >> 1) & 1) ^ 1, &abort_flag, status)) break;
        tc_fence_after();
        const uint32_t acc = tmem + kAccCols * a;
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int st = it % kStages;
          mbar_wait_cluster_bounded(&full_bar[st], (it / kStages) & 1, &abort_flag, status);
          tc_fence_after();
          const uint32_t base = smem_u32(smem + KpSmem::kRing + st * kStageBytes);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t da = smem_desc_sw128(base + ks * 32, 16, 1024);
            const uint64_t db = smem_desc_sw128(base + kXBox + ks * 32, 16, 1024);
            umma_pair_f16(acc, da, db, kIdProj, (kc > 0 || ks > 0) ? 1u : 0u);
          }
          umma_pair_commit(&empty_bar[st], kPairMask);   // both CTAs' stages free once read
        }
        umma_pair_commit(&acc_full[a], kPairMask);
      }
    }
  } else {
    // ---------------- epilogue: warp group c handles channel half c of both heads
    const int e = warp - 2;                        // 0..7
    const int ch = e >> 2;                         // channel half
    const int quarter = warp & 3;                  // TMEM lanes this warp may read
    const int row = 32 * quarter + lane;           // token row of this CTA's tile
    const int tid = e * 32 + lane;                 // 0..255
    const uint32_t tmem_lane = tmem + ((uint32_t)(32 * quarter) << 16);
    const bool has1 = nh > 1;
    const uint32_t acc_empty0 = map_to_cta(smem_u32(acc_empty), 0);
    const uint32_t stage_u32 = smem_u32(stage);
    const T *bias_g = static_cast<const T *>(p.bias);
    bool stored = false;
    int ncs = 0;   // cos / sin loads so far (phase of cs_bar)
    for (int i = 0; i < nt; ++i) {
      const int j = rg.begin + i;
      const int b = rg.unit(j), step = rg.step(j);
      const int a = i & 1;
      const StepTile mine = step_tile(sp, step, static_cast<int>(r));
      // the staging boxes are free once the previous step's stores have read
      // them; this step's cos rows then go into head 0's boxes and its sin rows
      // into head 1's, where each thread's Keys will overwrite exactly the
      // values it has read
      if (tid == 0 && stored) bulk_wait_read_all();
      named_barrier_sync(1, 256);
      if (tid == 0 && mine.exists) {
        mbar_arrive_expect_tx(cs_bar, 4 * kBox);
        const int bc = p.cs_sb == 0 ? 0 : b;
        for (int c = 0; c < 2; ++c) {
          tma_load_3d(stage + c * kBox, &maps.cs[0], 64 * c, mine.row0, bc, cs_bar);
          tma_load_3d(stage + (2 + c) * kBox, &maps.cs[1], 64 * c, mine.row0, bc, cs_bar);
        }
      }
      mbar_wait_cluster_bounded(&acc_full[a], (i >> 1) & 1, &abort_flag, status);
      tc_fence_after();
      uint32_t kv[2][32];
      const uint32_t acc = tmem_lane + kAccCols * a;
      drain_half<T>(acc + 32 * ch, bias_g == nullptr ? nullptr : bias_g + 2 * hp * 128 + 32 * ch, kv[0]);
      if (has1)
        drain_half<T>(acc + 128 + 32 * ch, bias_g == nullptr ? nullptr : bias_g + (2 * hp + 1) * 128 + 32 * ch, kv[1]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0 + 8 * a);   // this buffer may be overwritten
      if (mine.exists) {
        mbar_wait_bounded(cs_bar, ncs & 1, &abort_flag, status);
        ++ncs;
        const bool valid = mine.row0 + row < mine.end;   // rows past the span's end become zero
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t off = stage_u32 + swizzled_offset<128>(row, (4 * ch + u) * 8);
          const uint4 clo = ld_shared_u4(off), chi = ld_shared_u4(off + kBox);
          const uint4 slo = ld_shared_u4(off + 2 * kBox), shi = ld_shared_u4(off + 3 * kBox);
          if (valid) {
            rope_group<T>(clo, chi, slo, shi, u, has1, kv[0], kv[1]);
          } else {
#pragma unroll
            for (int k = 0; k < 4; ++k)
              kv[0][4 * u + k] = kv[0][16 + 4 * u + k] = kv[1][4 * u + k] = kv[1][16 + 4 * u + k] = 0u;
          }
          st_shared_v4(off, kv[0][4 * u], kv[0][4 * u + 1], kv[0][4 * u + 2], kv[0][4 * u + 3]);
          st_shared_v4(off + kBox, kv[0][16 + 4 * u], kv[0][17 + 4 * u], kv[0][18 + 4 * u], kv[0][19 + 4 * u]);
          if (has1) {
            st_shared_v4(off + 2 * kBox, kv[1][4 * u], kv[1][4 * u + 1], kv[1][4 * u + 2], kv[1][4 * u + 3]);
            st_shared_v4(off + 3 * kBox, kv[1][16 + 4 * u], kv[1][17 + 4 * u], kv[1][18 + 4 * u], kv[1][19 + 4 * u]);
          }
        }
      }
      fence_proxy_async_smem();   // generic-proxy writes -> the TMA store
      named_barrier_sync(1, 256);
      if (tid == 0 && mine.exists) {
        for (int h = 0; h < nh; ++h)
          for (int c = 0; c < 2; ++c)
            tma_store_4d(&maps.k_out[mine.span], stage + (2 * h + c) * kBox, 64 * c, mine.row0 - mine.start,
                         2 * hp + h, b);
        bulk_commit_group();
        stored = true;
      }
    }
    if (tid == 0 && stored) bulk_wait_all();
  }
  __syncthreads();
  cluster_sync();   // the peer is done with this CTA's shared and tensor memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

}  // namespace

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
  return cudaGetLastError();
}

}  // namespace rtk


