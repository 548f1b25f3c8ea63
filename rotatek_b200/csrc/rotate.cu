// Rotation of the visual Keys, kept = K_vis . R (kv_pruning_utils.py:152: the
// Keys are rotated uncentred and stored in their own dtype), plus the generic
// CUDA-core covariance used for fp32 Keys.
//
// Tensor-core path (bf16 / fp16): grid (chunks, matrices); a CTA owns a run of
// 64-token tiles of one matrix.  Tiles arrive by cp.async (16 B per thread,
// any row stride that keeps rows 16-B aligned) into a 2-stage ring laid out
// like a 128B-swizzled TMA box, so ldmatrix reads are conflict-free.  Each of
// the 4 warps multiplies 16 tokens x 128 channels by R [128 x keep]
// (mma.m16n8k16, fp32 accumulate), rounds to the Keys' dtype and stages the
// tile in shared memory; the CTA then writes it with 16-byte stores.
//
// The bytes that matter: read K (128 channels) once, write kept (keep
// channels) once -- 4.9 MB per (b, h) at S_v = 15 360, keep = 32.
#include "builder.h"
#include "common.cuh"

namespace rtk {
namespace {

constexpr int kTile = 64;
constexpr int kBox = kTile * 128;        // one 64-channel half of a tile, bytes
constexpr int kTileBytes = 2 * kBox;
constexpr int kRotThreads = 128;

template <typename T>
__device__ __forceinline__ void load_tile_async(unsigned char *dst, const RotateParams &p, int b, int h,
                                                int tok0, int tid) {
  const T *base = reinterpret_cast<const T *>(p.keys) + (long long)b * p.k_s[0] + (long long)h * p.k_s[1];
#pragma unroll
  for (int u = 0; u < (kTile * 16) / kRotThreads; ++u) {
    const int e = tid + u * kRotThreads;
    const int row = e >> 4, chunk = e & 15;
    unsigned char *d = dst + (chunk >> 3) * kBox + swizzled_offset<128>(row, (chunk & 7) * 8);
    const int tok = tok0 + row;
    if (tok < p.seq) {
      cp_async_16(d, base + (long long)tok * p.k_s[2] + chunk * 8);
    } else {
      *reinterpret_cast<uint4 *>(d) = make_uint4(0, 0, 0, 0);
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <typename T, int KEEP>
__global__ void __launch_bounds__(kRotThreads) rotate_tc_kernel(const RotateParams p, int tiles_per_cta) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *ring = smem;                                  // 2 x 16 KB
  T *rs = reinterpret_cast<T *>(smem + 2 * kTileBytes);       // R [128][KEEP]
  T *os = rs + 128 * KEEP;                                     // out tile [64][KEEP]

  const int m = blockIdx.y;
  const int b = m / p.heads, h = m % p.heads;
  const int tiles = (p.seq + kTile - 1) / kTile;
  const int first = blockIdx.x * tiles_per_cta;
  const int last = min(tiles, first + tiles_per_cta);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (first >= last) return;

  // R of this matrix into shared memory
  const T *Rb = reinterpret_cast<const T *>(p.R) + (long long)b * p.R_s[0] + (long long)h * p.R_s[1];
  for (int e = tid; e < 128 * KEEP; e += kRotThreads) rs[e] = Rb[(long long)(e / KEEP) * p.R_s[2] + (e % KEEP) * p.R_s[3]];
  load_tile_async<T>(ring, p, b, h, first * kTile, tid);

  const int g8 = lane >> 2, t4 = lane & 3;
  const int arow = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int acol = (lane >> 4) * 8;
  const int brow = (lane & 7) + ((lane >> 3) & 1) * 8;
  const int bcol = (lane >> 4) * 8;
  T *ob = reinterpret_cast<T *>(p.out) + (long long)b * p.o_s[0] + (long long)h * p.o_s[1];

  for (int t = first; t < last; ++t) {
    const int cur = (t - first) & 1;
    if (t + 1 < last) {
      load_tile_async<T>(ring + (cur ^ 1) * kTileBytes, p, b, h, (t + 1) * kTile, tid);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const uint32_t tile = smem_u32(ring + cur * kTileBytes);
    float acc[KEEP / 8][4];
#pragma unroll
    for (int n = 0; n < KEEP / 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t a[4];
      ldmatrix_x4(tile + (ks >= 4 ? kBox : 0) + swizzled_offset<128>(arow, (ks & 3) * 16 + acol), a[0],
                  a[1], a[2], a[3]);
#pragma unroll
      for (int n = 0; n < KEEP / 16; ++n) {
        uint32_t bfr[4];
        ldmatrix_x4_trans(smem_u32(rs + (ks * 16 + brow) * KEEP + n * 16 + bcol), bfr[0], bfr[1],
                          bfr[2], bfr[3]);
        mma_16816<T>(acc[2 * n], a, bfr[0], bfr[1]);
        mma_16816<T>(acc[2 * n + 1], a, bfr[2], bfr[3]);
      }
    }
    // round to the Keys' dtype and stage the 64 x KEEP tile
#pragma unroll
    for (int n = 0; n < KEEP / 8; ++n) {
      const int ch = n * 8 + 2 * t4;
      *reinterpret_cast<uint32_t *>(os + (warp * 16 + g8) * KEEP + ch) = pack2<T>(acc[n][0], acc[n][1]);
      *reinterpret_cast<uint32_t *>(os + (warp * 16 + g8 + 8) * KEEP + ch) = pack2<T>(acc[n][2], acc[n][3]);
    }
    __syncthreads();
    constexpr int kChunks = kTile * KEEP * 2 / 16;   // 16-byte chunks of the output tile
    for (int e = tid; e < kChunks; e += kRotThreads) {
      const int row = e / (KEEP / 8), c = e % (KEEP / 8);
      const int tok = t * kTile + row;
      if (tok < p.seq)
        *reinterpret_cast<uint4 *>(ob + (long long)tok * p.o_s[2] + c * 8) =
            *reinterpret_cast<const uint4 *>(os + row * KEEP + c * 8);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------- TMA kernel
// keep <= 64.  One persistent CTA per SM takes a contiguous range of the
// linear (matrix, 64-token tile) units; unit i of the range goes to warp i % 4.
// Each warp owns kStages / 4 ring stages and refills a stage itself, by TMA
// (two 64-channel x 64-token boxes, 128B swizzle), as soon as it has read the
// tile in it, so up to kStages tiles (~190 KB) per SM are in flight.  R's MMA
// B-fragments live in registers and are reloaded only when the matrix
// changes (R rows must be 16-byte aligned).  A warp stages its rounded 64 x
// keep output tile in its own shared buffer and writes it with 16-byte stores.
template <int KEEP>
struct RotCfg {
  static constexpr int kWarps = 4;
  static constexpr int kOutStride = KEEP + 8;                   // staged row, elements
  static constexpr int kOutBytes = kTile * kOutStride * 2;      // per warp
  // two 16 KB tiles per warp (128 KB per SM) keep HBM busy; deeper rings
  // measured slower
  static constexpr int kStages = 2 * kWarps;
  static constexpr int kPerWarp = kStages / kWarps;
  static constexpr int kRSlot = 128 * kOutStride * 2;            // one matrix's R, padded rows
  static constexpr int kRSlots = 2;                              // preloaded at kernel start
  static_assert(kStages * kTileBytes + kWarps * kOutBytes + kRSlots * kRSlot + 2048 <= 227 * 1024,
                "shared memory");
  static constexpr int kSmem = kStages * kTileBytes + kWarps * kOutBytes + kRSlots * kRSlot + kStages * 8 + 1024;
  static_assert(kStages >= kWarps, "at least one stage per warp");
};

template <typename T, int KEEP>
__global__ void __launch_bounds__(128, 1)
    rotate_tma_kernel(const __grid_constant__ CUtensorMap kmap, const RotateParams p) {
  using C = RotCfg<KEEP>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *ring = smem;
  T *outs = reinterpret_cast<T *>(smem + C::kStages * kTileBytes);
  T *rslot = reinterpret_cast<T *>(smem + C::kStages * kTileBytes + C::kWarps * C::kOutBytes);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::kStages * kTileBytes + C::kWarps * C::kOutBytes +
                                                C::kRSlots * C::kRSlot);
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // units (< 2^31, checked by the launcher) are walked with (matrix, tile)
  // cursors; no division on the per-tile path
  const int tiles = (p.seq + kTile - 1) / kTile;
  const long long total = (long long)p.batch * p.heads * tiles;
  const int u0 = static_cast<int>(blockIdx.x * total / gridDim.x);
  const int n = static_cast<int>((blockIdx.x + 1) * total / gridDim.x) - u0;
  if (tid < C::kStages) mbar_init(&full[tid], 1);
  if (tid == 0) {
    abort_flag = 0;
    tma_prefetch_desc(&kmap);
  }
  fence_barrier_init();
  __syncthreads();

  // unit i -> warp i % 4, ring stage warp + 4 * ((i / 4) % kPerWarp), used for
  // the ((i / 4) / kPerWarp)-th time.  A cursor is (unit i, matrix m, tile t).
  struct Cursor {
    int i, m, t;
  };
  auto advance = [&](Cursor &c, int step) {
    c.i += step;
    c.t += step;
    while (c.t >= tiles) {
      c.t -= tiles;
      ++c.m;
    }
  };
  auto issue = [&](const Cursor &c) {
    const int b = c.m / p.heads, h = c.m - b * p.heads;
    const int stage = warp + C::kWarps * ((c.i / C::kWarps) % C::kPerWarp);
    unsigned char *dst = ring + stage * kTileBytes;
    mbar_arrive_expect_tx(&full[stage], kTileBytes);
    tma_load_4d(dst, &kmap, 0, c.t * kTile, h, b, &full[stage]);
    tma_load_4d(dst + kBox, &kmap, 64, c.t * kTile, h, b, &full[stage]);
  };
  Cursor cc = {0, (u0 + warp) / tiles, (u0 + warp) % tiles};   // the unit being computed
  cc.i = warp;
  Cursor ic = cc;                                                // the next unit to load
  for (int j = 0; j < C::kPerWarp && ic.i < n; ++j) {
    if (lane == 0) issue(ic);
    advance(ic, C::kWarps);
  }
  // R of the range's first kRSlots matrices -> shared memory (all threads,
  // cp.async, while the first tiles are in flight); a range that reaches
  // further loads the rest per warp when it gets there
  const int m_first = n > 0 ? u0 / tiles : 0;
  const int nslot = n > 0 ? min(C::kRSlots, (u0 + n - 1) / tiles - m_first + 1) : 0;
  for (int e = tid; e < nslot * 128 * (KEEP / 8); e += blockDim.x) {
    const int sl = e / (128 * (KEEP / 8)), rem = e % (128 * (KEEP / 8));
    const int row = rem / (KEEP / 8), c = rem % (KEEP / 8);
    const int mm = m_first + sl, bb = mm / p.heads, hh = mm - bb * p.heads;
    cp_async_16(rslot + sl * (C::kRSlot / 2) + row * C::kOutStride + c * 8,
                reinterpret_cast<const T *>(p.R) + (long long)bb * p.R_s[0] + (long long)hh * p.R_s[1] +
                    (long long)row * p.R_s[2] + c * 8);
  }
  cp_async_wait_all();
  __syncthreads();

  const int g8 = lane >> 2, t4 = lane & 3;
  const int arow = (lane & 7) + ((lane >> 3) & 1) * 8, acol = (lane >> 4) * 8;
  T *ob = outs + warp * (C::kOutBytes / 2);
  int cur_m = -1, b = 0, h = 0;
  uint32_t rf[8][KEEP / 8][2];
  for (; cc.i < n; advance(cc, C::kWarps)) {
    const int i = cc.i, m = cc.m, t = cc.t;
    if (m != cur_m) {
      b = m / p.heads;
      h = m - b * p.heads;
      // R of the new matrix -> B fragments, through this warp's (idle) output
      // buffer in two 64-row halves: 16-byte loads, then ldmatrix.trans
      const T *R = reinterpret_cast<const T *>(p.R) + (long long)b * p.R_s[0] + (long long)h * p.R_s[1];
      const int brow = (lane & 7) + ((lane >> 3) & 1) * 8, bcol = (lane >> 4) * 8;
      const bool preloaded = m - m_first < nslot;
      const T *src = rslot + (m - m_first) * (C::kRSlot / 2);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const T *rows = src + 64 * half * C::kOutStride;
        if (!preloaded) {
          constexpr int kVec = 64 * KEEP / 8;               // 16-byte pieces per half
#pragma unroll
          for (int e = lane; e < kVec; e += 32) {
            const int row = e / (KEEP / 8), c = e % (KEEP / 8);
            *reinterpret_cast<uint4 *>(ob + row * C::kOutStride + c * 8) =
                *reinterpret_cast<const uint4 *>(R + (long long)(64 * half + row) * p.R_s[2] + c * 8);
          }
          __syncwarp();
          rows = ob;
        }
#pragma unroll
        for (int kq = 0; kq < 4; ++kq)
#pragma unroll
          for (int g = 0; g < KEEP / 16; ++g) {
            uint32_t f[4];
            ldmatrix_x4_trans(smem_u32(rows + (kq * 16 + brow) * C::kOutStride + g * 16 + bcol), f[0], f[1], f[2], f[3]);
            rf[4 * half + kq][2 * g][0] = f[0];
            rf[4 * half + kq][2 * g][1] = f[1];
            rf[4 * half + kq][2 * g + 1][0] = f[2];
            rf[4 * half + kq][2 * g + 1][1] = f[3];
          }
        __syncwarp();
      }
      cur_m = m;
    }
    const int stage = warp + C::kWarps * ((i / C::kWarps) % C::kPerWarp);
    const uint32_t parity = static_cast<uint32_t>((i / C::kWarps) / C::kPerWarp) & 1u;
    if (!mbar_wait_bounded(&full[stage], parity, &abort_flag, p.status)) break;
    const uint32_t tile = smem_u32(ring + stage * kTileBytes);
    // MBP m-blocks of 16 rows at once: each k-step issues MBP x keep/8
    // independent MMAs (one warp per SM sub-partition has no other latency cover)
    constexpr int MBP = KEEP <= 32 ? 4 : 2;
#pragma unroll 1
    for (int mb0 = 0; mb0 < 4; mb0 += MBP) {
      float acc[MBP][KEEP / 8][4];
#pragma unroll
      for (int j = 0; j < MBP; ++j)
#pragma unroll
        for (int nn = 0; nn < KEEP / 8; ++nn) acc[j][nn][0] = acc[j][nn][1] = acc[j][nn][2] = acc[j][nn][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t a[MBP][4];
#pragma unroll
        for (int j = 0; j < MBP; ++j)
          ldmatrix_x4(tile + (ks >= 4 ? kBox : 0) + swizzled_offset<128>((mb0 + j) * 16 + arow, (ks & 3) * 16 + acol),
                      a[j][0], a[j][1], a[j][2], a[j][3]);
#pragma unroll
        for (int j = 0; j < MBP; ++j)
#pragma unroll
          for (int nn = 0; nn < KEEP / 8; ++nn) mma_16816<T>(acc[j][nn], a[j], rf[ks][nn][0], rf[ks][nn][1]);
      }
#pragma unroll
      for (int j = 0; j < MBP; ++j)
#pragma unroll
        for (int nn = 0; nn < KEEP / 8; ++nn) {
          const int ch = nn * 8 + 2 * t4, row = (mb0 + j) * 16 + g8;
          *reinterpret_cast<uint32_t *>(ob + row * C::kOutStride + ch) = pack2<T>(acc[j][nn][0], acc[j][nn][1]);
          *reinterpret_cast<uint32_t *>(ob + (row + 8) * C::kOutStride + ch) = pack2<T>(acc[j][nn][2], acc[j][nn][3]);
        }
    }
    // the tile has been read: every lane orders its reads before the TMA
    // write (async proxy) that refills the stage with this warp's unit
    // kStages ahead
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0 && ic.i < n) issue(ic);
    advance(ic, C::kWarps);
    T *og = reinterpret_cast<T *>(p.out) + (long long)b * p.o_s[0] + (long long)h * p.o_s[1];
    constexpr int kChunks = kTile * KEEP / 8;                   // 16-byte chunks of the tile
#pragma unroll 4
    for (int e = lane; e < kChunks; e += 32) {
      const int row = e / (KEEP / 8), c = e % (KEEP / 8);
      const int tok = t * kTile + row;
      if (tok < p.seq)
        *reinterpret_cast<uint4 *>(og + (long long)tok * p.o_s[2] + c * 8) =
            *reinterpret_cast<const uint4 *>(ob + row * C::kOutStride + c * 8);
    }
    __syncwarp();
  }
}

template <typename T, int KEEP>
cudaError_t launch_rot_tma(const CUtensorMap &kmap, const RotateParams &p, cudaStream_t stream) {
  using C = RotCfg<KEEP>;
  const long long units = (long long)p.batch * p.heads * ((p.seq + kTile - 1) / kTile);
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (units >= (1ll << 31)) return cudaErrorInvalidValue;
  if (p.max_ctas > 0 && p.max_ctas < sms) sms = p.max_ctas;
  const int grid = static_cast<int>(units < sms ? units : sms);
  if (grid == 0) return cudaSuccess;
  cudaError_t err = cudaFuncSetAttribute(rotate_tma_kernel<T, KEEP>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  if (err != cudaSuccess) return err;
  rotate_tma_kernel<T, KEEP><<<grid, 128, C::kSmem, stream>>>(kmap, p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch_rot_tma(const CUtensorMap &kmap, const RotateParams &p, cudaStream_t stream) {
  switch (p.keep) {
    case 16: return launch_rot_tma<T, 16>(kmap, p, stream);
    case 32: return launch_rot_tma<T, 32>(kmap, p, stream);
    case 48: return launch_rot_tma<T, 48>(kmap, p, stream);
    case 64: return launch_rot_tma<T, 64>(kmap, p, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
__device__ __forceinline__ float ldf(const void *p, long long i) {
  return to_f32(reinterpret_cast<const T *>(p)[i]);
}

// Generic rotation: one CTA per (64-token tile, matrix), fp32 arithmetic.
template <typename T>
__global__ void __launch_bounds__(256) rotate_simt_kernel(const RotateParams p) {
  extern __shared__ float rf[];                       // R [128][keep] fp32
  const int m = blockIdx.y, b = m / p.heads, h = m % p.heads;
  const int tok0 = blockIdx.x * kTile;
  for (int e = threadIdx.x; e < 128 * p.keep; e += blockDim.x)
    rf[e] = ldf<T>(p.R, (long long)b * p.R_s[0] + (long long)h * p.R_s[1] +
                            (long long)(e / p.keep) * p.R_s[2] + (e % p.keep) * p.R_s[3]);
  __syncthreads();
  for (int e = threadIdx.x; e < kTile * p.keep; e += blockDim.x) {
    const int r = e / p.keep, c = e % p.keep, tok = tok0 + r;
    if (tok >= p.seq) continue;
    const long long kb = (long long)b * p.k_s[0] + (long long)h * p.k_s[1] + (long long)tok * p.k_s[2];
    float acc = 0.f;
    for (int d = 0; d < 128; ++d) acc = fmaf(ldf<T>(p.keys, kb + d * p.k_s[3]), rf[d * p.keep + c], acc);
    reinterpret_cast<T *>(p.out)[(long long)b * p.o_s[0] + (long long)h * p.o_s[1] +
                                 (long long)tok * p.o_s[2] + c * p.o_s[3]] = from_f32<T>(acc);
  }
}

// Generic covariance: one CTA per matrix, 256 threads, each an 8 x 8 block of
// sum k k^T; tokens staged 32 at a time in shared memory (fp32).
template <typename T>
__global__ void __launch_bounds__(256) cov_simt_kernel(const CovParams p) {
  __shared__ float ks[32][128];
  const int m = blockIdx.x, b = m / p.heads, h = m % p.heads;
  const int tid = threadIdx.x;
  const int i0 = (tid >> 4) * 8, j0 = (tid & 15) * 8;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  float colsum = 0.f;
  const long long base = (long long)b * p.k_s[0] + (long long)h * p.k_s[1];
  for (int s0 = 0; s0 < p.seq; s0 += 32) {
    __syncthreads();
    for (int e = tid; e < 32 * 128; e += 256) {
      const int r = e >> 7, d = e & 127;
      ks[r][d] = s0 + r < p.seq ? ldf<T>(p.keys, base + (long long)(s0 + r) * p.k_s[2] + d * p.k_s[3]) : 0.f;
    }
    __syncthreads();
    for (int r = 0; r < 32; ++r) {
      float ki[8], kj[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) { ki[i] = ks[r][i0 + i]; kj[i] = ks[r][j0 + i]; }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(ki[i], kj[j], acc[i][j]);
      if (tid < 128) colsum += ks[r][tid];
    }
  }
  float *out = p.cov + (long long)m * 128 * 128;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) out[(i0 + i) * 128 + j0 + j] = acc[i][j];
  if (tid < 128) p.ksum[(long long)m * 128 + tid] = colsum;
}

template <typename T, int KEEP>
cudaError_t launch_rot(const RotateParams &p, cudaStream_t stream) {
  const int tiles = (p.seq + kTile - 1) / kTile;
  const int nmat = p.batch * p.heads;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int want_chunks = (8 * sms + nmat - 1) / nmat;
  const int chunks = max(1, min(tiles, want_chunks));
  const int per = (tiles + chunks - 1) / chunks;
  const int grid_x = (tiles + per - 1) / per;
  const int smem = 2 * kTileBytes + 128 * KEEP * 2 + kTile * KEEP * 2 + 1024;
  cudaError_t err = cudaFuncSetAttribute(rotate_tc_kernel<T, KEEP>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  rotate_tc_kernel<T, KEEP><<<dim3(grid_x, nmat), kRotThreads, smem, stream>>>(p, per);
  return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch_rot(const RotateParams &p, cudaStream_t stream) {
  switch (p.keep) {
    case 16: return launch_rot<T, 16>(p, stream);
    case 32: return launch_rot<T, 32>(p, stream);
    case 48: return launch_rot<T, 48>(p, stream);
    case 64: return launch_rot<T, 64>(p, stream);
    case 96: return launch_rot<T, 96>(p, stream);
    case 128: return launch_rot<T, 128>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_rotate_tc(int dtype_is_bf16, const RotateParams &p, cudaStream_t stream) {
  return dtype_is_bf16 ? dispatch_rot<__nv_bfloat16>(p, stream) : dispatch_rot<__half>(p, stream);
}

cudaError_t launch_rotate_tma(int dtype_is_bf16, const CUtensorMap &keys_map, const RotateParams &p,
                              cudaStream_t stream) {
  return dtype_is_bf16 ? dispatch_rot_tma<__nv_bfloat16>(keys_map, p, stream)
                       : dispatch_rot_tma<__half>(keys_map, p, stream);
}

cudaError_t launch_rotate_simt(const RotateParams &p, cudaStream_t stream) {
  const int tiles = (p.seq + kTile - 1) / kTile;
  const dim3 grid(max(tiles, 1), p.batch * p.heads);
  const int smem = 128 * p.keep * 4;
  switch (p.dtype) {
    case 0:
      cudaFuncSetAttribute(rotate_simt_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      rotate_simt_kernel<float><<<grid, 256, smem, stream>>>(p);
      break;
    case 1:
      cudaFuncSetAttribute(rotate_simt_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      rotate_simt_kernel<__nv_bfloat16><<<grid, 256, smem, stream>>>(p);
      break;
    case 2:
      cudaFuncSetAttribute(rotate_simt_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      rotate_simt_kernel<__half><<<grid, 256, smem, stream>>>(p);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_cov_simt(const CovParams &p, cudaStream_t stream) {
  const dim3 grid(p.batch * p.heads);
  switch (p.dtype) {
    case 0: cov_simt_kernel<float><<<grid, 256, 0, stream>>>(p); break;
    case 1: cov_simt_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(p); break;
    case 2: cov_simt_kernel<__half><<<grid, 256, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace rtk
