// Fused GQA flash-decode for RotateK on sm_100a (bf16 / fp16, head_dim 128).
//
// Computes, for one query token per (batch, query head),
//   out = softmax([q.k_f * s ; (q R . k_s + q . delta_mu) * s]) . [v_f ; v_s] / (l + 1e-6)
// -- the arithmetic of rotatek/kernels/fused_decode.py:131-296 (full-width
// prompt/text span `f`, rotated-truncated visual span `s`), and with an empty
// visual span the dense decode of full_channel_flash_decoding.py:34-155.
//
// Work decomposition (persistent, stream-K):
//   unit   = (batch, KV head, head chunk of <= 8*NT query heads); every query
//            head of a GQA group shares each K/V tile, so K/V bytes are read
//            once per group, not once per query head.
//   block  = 64 tokens of one unit: first the ceil(S_f/64) full-width blocks,
//            then the ceil(S_v/64) visual blocks.
//   The U * blocks_per_unit blocks are cut into `grid` equal contiguous ranges,
//   one per CTA (one CTA per SM).  A CTA walks its range as segments (maximal
//   runs inside one unit); a segment that covers a whole unit writes the
//   output directly, otherwise it writes a partial (m, l, acc) to slot
//   unit + cta of the workspace and takes a ticket; the last CTA of a unit
//   merges that unit's partials and writes the output.  No CTA ever waits on
//   another.
//
// Inside a CTA: warp 4*NGROUP is the producer -- it streams each block's K and
// V tiles with 4-D TMA tensor copies (128B/64B/32B swizzle) into an NSTAGE
// ring.  Consumer warps come in NGROUP groups of 4; group g takes the blocks
// i = g (mod NGROUP) and each of its warps owns 16 of the 64 tokens.  Scores
// are S^T[16 tokens x 8 heads] = K[16 x d] . Q^T on mma.m16n8k16 (bf16 in,
// fp32 accumulate); the rotated query q~ = q.R is built in fp32 once per
// segment and fed to the tensor cores as a bf16 hi/lo pair, so visual scores
// keep ~16 mantissa bits of q~.  Probabilities go to bf16 (fp16) through
// movmatrix and accumulate O^T[128 d x 8 heads] += V^T . P^T in fp32 registers.
#include "common.cuh"
#include "decode.h"

namespace rtk {
namespace {

constexpr int kBlockTokens = 64;
constexpr int kHeadDim = 128;
constexpr int kStages = 5;
constexpr int kStageBytes = 32768;        // K region 16 KB + V region 16 KB
constexpr int kKRegion = 16384;
constexpr int kWarpsPerGroup = 4;
constexpr float kNegBig = -1e30f;         // running-max floor (fused_decode.py:151)

template <int NT, int NGROUP>
struct SmemLayout {
  static constexpr int kHeads = 8 * NT;
  static constexpr int kConsumerWarps = kWarpsPerGroup * NGROUP;
  static constexpr int kAccStride = kHeadDim + 4;  // padding keeps red.shared conflict-free
  static constexpr int kStagesOff = 0;
  static constexpr int kQOff = kStages * kStageBytes;                        // fp32 [H][128]
  static constexpr int kQRotOff = kQOff + kHeads * kHeadDim * 4;             // fp32 [H][64]
  static constexpr int kBiasOff = kQRotOff + kHeads * 64 * 4;                // fp32 [H]
  static constexpr int kAccOff = kBiasOff + kHeads * 4;                      // fp32 [H][132]
  static constexpr int kMwOff = kAccOff + kHeads * kAccStride * 4;           // fp32 [W][H]
  static constexpr int kLwOff = kMwOff + kConsumerWarps * kHeads * 4;        // fp32 [W][H]
  static constexpr int kBarOff = (kLwOff + kConsumerWarps * kHeads * 4 + 15) & ~15;
  static constexpr int kFlagOff = kBarOff + 2 * kStages * 8;
  static constexpr int kBytes = kFlagOff + 16;
};

struct Seg {
  int unit, b, kvh, hc, head0, nheads;
};

__device__ __forceinline__ long long cta_of_block(long long blk, long long total, int grid) {
  // the CTA whose range [floor(c*T/P), floor((c+1)*T/P)) holds block `blk`
  return ((blk + 1) * grid - 1) / total;
}

template <typename T, int NT, int DK, int NGROUP>
__global__ void __launch_bounds__((kWarpsPerGroup * NGROUP + 1) * 32, 1)
    rotatek_decode_tc_kernel(const __grid_constant__ CUtensorMap tm_kf,
                             const __grid_constant__ CUtensorMap tm_vf,
                             const __grid_constant__ CUtensorMap tm_ks,
                             const __grid_constant__ CUtensorMap tm_vs, const DecodeParams p) {
  using L = SmemLayout<NT, NGROUP>;
  constexpr int kHeads = L::kHeads;
  constexpr int kConsumers = L::kConsumerWarps * 32;
  constexpr int kKsRowBytes = DK * 2;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float *q_s = reinterpret_cast<float *>(smem + L::kQOff);
  float *qrot_s = reinterpret_cast<float *>(smem + L::kQRotOff);
  float *bias_s = reinterpret_cast<float *>(smem + L::kBiasOff);
  float *acc_s = reinterpret_cast<float *>(smem + L::kAccOff);
  float *mw_s = reinterpret_cast<float *>(smem + L::kMwOff);
  float *lw_s = reinterpret_cast<float *>(smem + L::kLwOff);
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem + L::kBarOff);
  uint64_t *empty_bar = full_bar + kStages;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::kFlagOff);
  volatile int *last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long total = p.total_blocks;
  const long long lo = (long long)blockIdx.x * total / gridDim.x;
  const long long hi = (long long)(blockIdx.x + 1) * total / gridDim.x;
  const int nblk = static_cast<int>(hi - lo);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kWarpsPerGroup);
    }
    *abort_flag = 0;
    *last_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // ======================================================== producer warp
  if (warp == L::kConsumerWarps) {
    if (lane == 0) {
      if (p.blocks_full > 0) { tma_prefetch_desc(&tm_kf); tma_prefetch_desc(&tm_vf); }
      if (p.blocks_sparse > 0) { tma_prefetch_desc(&tm_ks); tma_prefetch_desc(&tm_vs); }
      int issued = 0;
      for (int i = 0; i < nblk; ++i) {
        const int stage = i % kStages;
        const uint32_t parity = ((i / kStages) & 1) ^ 1;
        if (!mbar_wait_bounded(&empty_bar[stage], parity, abort_flag, p.status)) break;
        const long long g = lo + i;
        const int unit = static_cast<int>(g / p.blocks_per_unit);
        const int j = static_cast<int>(g - (long long)unit * p.blocks_per_unit);
        const int bk = unit / (p.kv_heads * p.head_chunks);
        const int kvh = (unit / p.head_chunks) % p.kv_heads;
        unsigned char *st = smem + stage * kStageBytes;
        if (j < p.blocks_full) {
          const int tok = j * kBlockTokens;
          mbar_arrive_expect_tx(&full_bar[stage], 4 * 8192);
          tma_load_4d(st, &tm_kf, 0, tok, kvh, bk, &full_bar[stage]);
          tma_load_4d(st + 8192, &tm_kf, 64, tok, kvh, bk, &full_bar[stage]);
          tma_load_4d(st + kKRegion, &tm_vf, 0, tok, kvh, bk, &full_bar[stage]);
          tma_load_4d(st + kKRegion + 8192, &tm_vf, 64, tok, kvh, bk, &full_bar[stage]);
        } else {
          const int tok = (j - p.blocks_full) * kBlockTokens;
          mbar_arrive_expect_tx(&full_bar[stage], kBlockTokens * DK * 2 + 2 * 8192);
          tma_load_4d(st, &tm_ks, 0, tok, kvh, bk, &full_bar[stage]);
          tma_load_4d(st + kKRegion, &tm_vs, 0, tok, kvh, bk, &full_bar[stage]);
          tma_load_4d(st + kKRegion + 8192, &tm_vs, 64, tok, kvh, bk, &full_bar[stage]);
        }
        ++issued;
      }
      if (*abort_flag) {
        // leave no copy in flight: wait (bounded) for the stages still loading
        const int first = issued > kStages ? issued - kStages : 0;
        for (int i = first; i < issued; ++i) {
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&full_bar[i % kStages], (i / kStages) & 1)) {
            if (globaltimer_ns() - t0 > kWaitLimitNs / 4) break;
          }
        }
      }
    }
    return;
  }

  // ======================================================== consumer warps
  const int cw = warp;                         // consumer warp 0 .. 4*NGROUP-1
  const int group = cw / kWarpsPerGroup;
  const int wig = cw % kWarpsPerGroup;         // warp in group: owns tokens [16*wig, +16)
  const int g8 = lane >> 2;                    // fragment row
  const int t4 = lane & 3;                     // fragment column pair
  const int ctid = threadIdx.x;                // 0 .. kConsumers-1

  int it = 0;
  while (it < nblk) {
    Seg sg;
    sg.unit = static_cast<int>((lo + it) / p.blocks_per_unit);
    const long long unit_end = (long long)(sg.unit + 1) * p.blocks_per_unit;
    const int seg_end = static_cast<int>((hi < unit_end ? hi : unit_end) - lo);
    sg.hc = sg.unit % p.head_chunks;
    sg.kvh = (sg.unit / p.head_chunks) % p.kv_heads;
    sg.b = sg.unit / (p.kv_heads * p.head_chunks);
    sg.head0 = sg.kvh * p.groups + sg.hc * kHeads;
    sg.nheads = min(kHeads, p.groups - sg.hc * kHeads);

    // ---- segment set-up: q tile, q~ = q R, bias = q . delta_mu, zero the accumulator
    named_barrier_sync(1, kConsumers);
    {
      const T *qb = reinterpret_cast<const T *>(p.q) + (long long)sg.b * p.q_sb;
      for (int e = ctid; e < kHeads * kHeadDim; e += kConsumers) {
        const int h = e / kHeadDim, d = e % kHeadDim;
        q_s[e] = h < sg.nheads ? to_f32(qb[(long long)(sg.head0 + h) * p.q_sh + d]) : 0.f;
      }
      for (int e = ctid; e < kHeads * L::kAccStride; e += kConsumers) acc_s[e] = 0.f;
    }
    named_barrier_sync(1, kConsumers);
    {
      const T *Rb = reinterpret_cast<const T *>(p.R) + (long long)sg.b * p.R_sb +
                    (long long)sg.kvh * p.R_sh;
      for (int e = ctid; e < kHeads * DK; e += kConsumers) {
        const int h = e / DK, jj = e % DK;
        const float *qh = q_s + h * kHeadDim;
        float acc = 0.f;
        if (p.R != nullptr) {  // NULL for the dense (full-channel) decode
#pragma unroll 8
          for (int d = 0; d < kHeadDim; ++d) acc = fmaf(qh[d], to_f32(Rb[(long long)d * p.R_sd + jj]), acc);
        }
        qrot_s[h * 64 + jj] = acc;
      }
      if (ctid < kHeads) {
        float acc = 0.f;
        if (p.dm != nullptr) {
          const T *db = reinterpret_cast<const T *>(p.dm) + (long long)sg.b * p.dm_sb +
                        (long long)sg.kvh * p.dm_sh;
          const float *qh = q_s + ctid * kHeadDim;
          for (int d = 0; d < kHeadDim; ++d) acc = fmaf(qh[d], to_f32(db[d]), acc);
        }
        bias_s[ctid] = acc;
      }
    }
    named_barrier_sync(1, kConsumers);

    // ---- per-warp fragments of the queries (B operands: k = channel, n = head)
    uint32_t qhi[DK / 16][NT][2], qlo[DK / 16][NT][2];
    float bias2[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int h = nt * 8 + g8;
#pragma unroll
      for (int ks = 0; ks < DK / 16; ++ks) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int c = ks * 16 + half * 8 + 2 * t4;
          const float v0 = qrot_s[h * 64 + c], v1 = qrot_s[h * 64 + c + 1];
          const uint32_t hpk = pack2<T>(v0, v1);
          float h0, h1;
          unpack2<T>(hpk, h0, h1);
          qhi[ks][nt][half] = hpk;
          qlo[ks][nt][half] = pack2<T>(v0 - h0, v1 - h1);
        }
      }
      bias2[nt][0] = bias_s[nt * 8 + 2 * t4];
      bias2[nt][1] = bias_s[nt * 8 + 2 * t4 + 1];
    }

    float o[8][NT][4];
    float m_run[NT][2], l_run[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m_run[nt][0] = m_run[nt][1] = kNegBig;
      l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
    }

    // ---- stream this segment's blocks
    for (int i = it; i < seg_end; ++i) {
      if ((i % NGROUP) != group) continue;
      const int stage = i % kStages;
      const bool ready = mbar_wait_bounded(&full_bar[stage], (i / kStages) & 1, abort_flag, p.status);
      const int j = static_cast<int>(lo + i - (long long)sg.unit * p.blocks_per_unit);
      const bool is_full = j < p.blocks_full;
      const int tok0 = (is_full ? j : j - p.blocks_full) * kBlockTokens + wig * 16;
      const int seq = is_full ? p.seq_full : p.seq_sparse;
      const uint32_t kbase = smem_u32(smem + stage * kStageBytes);
      const uint32_t vbase = kbase + kKRegion;
      const int r0 = wig * 16;                    // first box row of this warp

      if (ready) {
        float s[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
        // A-operand row/col for this lane (non-transposed ldmatrix.x4)
        const int arow = r0 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int acol = (lane >> 4) * 8;
        if (is_full) {
#pragma unroll
          for (int ks = 0; ks < kHeadDim / 16; ++ks) {
            uint32_t a[4];
            const uint32_t box = kbase + (ks >= 4 ? 8192u : 0u);
            ldmatrix_x4(box + swizzled_offset<128>(arow, (ks & 3) * 16 + acol), a[0], a[1], a[2], a[3]);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const float *qh = q_s + (nt * 8 + g8) * kHeadDim + ks * 16 + 2 * t4;
              const uint32_t b0 = pack2<T>(qh[0], qh[1]);
              const uint32_t b1 = pack2<T>(qh[8], qh[9]);
              mma_16816<T>(s[nt], a, b0, b1);
            }
          }
        } else {
#pragma unroll
          for (int ks = 0; ks < DK / 16; ++ks) {
            uint32_t a[4];
            ldmatrix_x4(kbase + swizzled_offset<kKsRowBytes>(arow, ks * 16 + acol), a[0], a[1], a[2], a[3]);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              mma_16816<T>(s[nt], a, qhi[ks][nt][0], qhi[ks][nt][1]);
              mma_16816<T>(s[nt], a, qlo[ks][nt][0], qlo[ks][nt][1]);
            }
          }
        }
        // ---- scale, bias, masks -> online softmax (rows g8 / g8+8 = tokens, cols = heads)
        const int tokA = tok0 + g8, tokB = tok0 + g8 + 8;
        bool validA = tokA < seq, validB = tokB < seq;
        if (is_full && p.mask != nullptr) {
          const uint8_t *mrow = p.mask + (long long)sg.b * p.mask_sb;
          if (validA) validA = mrow[(long long)tokA * p.mask_ss] != 0;
          if (validB) validB = mrow[(long long)tokB * p.mask_ss] != 0;
        }
        uint32_t pb[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          float sc[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float bias = is_full ? 0.f : bias2[nt][e & 1];
            sc[e] = (s[nt][e] + bias) * p.scale_log2;
          }
          if (!validA) sc[0] = sc[1] = -INFINITY;
          if (!validB) sc[2] = sc[3] = -INFINITY;
          float mx0 = fmaxf(sc[0], sc[2]), mx1 = fmaxf(sc[1], sc[3]);
#pragma unroll
          for (int off = 4; off < 32; off <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
          }
          const float mn0 = fmaxf(m_run[nt][0], mx0), mn1 = fmaxf(m_run[nt][1], mx1);
          const float al0 = fast_exp2(m_run[nt][0] - mn0), al1 = fast_exp2(m_run[nt][1] - mn1);
          m_run[nt][0] = mn0;
          m_run[nt][1] = mn1;
          const float p0 = fast_exp2(sc[0] - mn0), p1 = fast_exp2(sc[1] - mn1);
          const float p2 = fast_exp2(sc[2] - mn0), p3 = fast_exp2(sc[3] - mn1);
          l_run[nt][0] = l_run[nt][0] * al0 + (p0 + p2);
          l_run[nt][1] = l_run[nt][1] * al1 + (p1 + p3);
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            o[mt][nt][0] *= al0;
            o[mt][nt][1] *= al1;
            o[mt][nt][2] *= al0;
            o[mt][nt][3] *= al1;
          }
          pb[nt][0] = movmatrix_trans(pack2<T>(p0, p1));
          pb[nt][1] = movmatrix_trans(pack2<T>(p2, p3));
        }
        // ---- O^T[d, head] += V^T[d, tok] . P^T[tok, head]
        const int vrow = r0 + (lane & 7) + ((lane >> 4) & 1) * 8;
        const int vcol = ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          uint32_t a[4];
          const uint32_t box = vbase + (mt >= 4 ? 8192u : 0u);
          ldmatrix_x4_trans(box + swizzled_offset<128>(vrow, (mt & 3) * 16 + vcol), a[0], a[1], a[2], a[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_16816<T>(o[mt][nt], a, pb[nt][0], pb[nt][1]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[stage]);
    }

    // ---- segment end: merge the consumer warps (red.shared into acc_s)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float l = l_run[nt][c];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        l_run[nt][c] = l;
      }
      if (g8 == 0) {
        mw_s[cw * kHeads + nt * 8 + 2 * t4] = m_run[nt][0];
        mw_s[cw * kHeads + nt * 8 + 2 * t4 + 1] = m_run[nt][1];
        lw_s[cw * kHeads + nt * 8 + 2 * t4] = l_run[nt][0];
        lw_s[cw * kHeads + nt * 8 + 2 * t4 + 1] = l_run[nt][1];
      }
    }
    named_barrier_sync(1, kConsumers);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int h = nt * 8 + 2 * t4 + c;
        float mx = kNegBig;
        for (int w = 0; w < L::kConsumerWarps; ++w) mx = fmaxf(mx, mw_s[w * kHeads + h]);
        const float sc = fast_exp2(m_run[nt][c] - mx);
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int d0 = mt * 16 + g8;
          atomicAdd(&acc_s[h * L::kAccStride + d0], o[mt][nt][c] * sc);
          atomicAdd(&acc_s[h * L::kAccStride + d0 + 8], o[mt][nt][2 + c] * sc);
        }
      }
    }
    named_barrier_sync(1, kConsumers);

    // per-head merged (m, l) of this CTA's segment, recomputed by every thread that needs it
    auto seg_ml = [&](int h, float &m_out, float &l_out) {
      float mx = kNegBig;
      for (int w = 0; w < L::kConsumerWarps; ++w) mx = fmaxf(mx, mw_s[w * kHeads + h]);
      float l = 0.f;
      for (int w = 0; w < L::kConsumerWarps; ++w)
        l += lw_s[w * kHeads + h] * fast_exp2(mw_s[w * kHeads + h] - mx);
      m_out = mx;
      l_out = l;
    };

    const long long ublk0 = (long long)sg.unit * p.blocks_per_unit;
    const int c_first = static_cast<int>(cta_of_block(ublk0, total, gridDim.x));
    const int c_last = static_cast<int>(cta_of_block(ublk0 + p.blocks_per_unit - 1, total, gridDim.x));
    T *outb = reinterpret_cast<T *>(p.out) + (long long)sg.b * p.o_sb;

    if (c_first == c_last) {
      // the whole unit lives in this CTA: normalise and store
      for (int e = ctid; e < kHeads * kHeadDim; e += kConsumers) {
        const int h = e / kHeadDim, d = e % kHeadDim;
        if (h >= sg.nheads) continue;
        float m, l;
        seg_ml(h, m, l);
        outb[(long long)(sg.head0 + h) * p.o_sh + d] = from_f32<T>(acc_s[h * L::kAccStride + d] / (l + 1e-6f));
      }
    } else {
      float *slot = p.partials + (long long)(sg.unit + blockIdx.x) * p.slot_floats;
      for (int e = ctid; e < kHeads * kHeadDim; e += kConsumers) {
        const int h = e / kHeadDim, d = e % kHeadDim;
        slot[32 + e] = acc_s[h * L::kAccStride + d];
      }
      if (ctid < kHeads) {
        float m, l;
        seg_ml(ctid, m, l);
        slot[ctid] = m;
        slot[16 + ctid] = l;
      }
      __threadfence();
      named_barrier_sync(1, kConsumers);
      if (ctid == 0) {
        const int count = c_last - c_first + 1;
        const int prev = atomicAdd(&p.tickets[sg.unit], 1);
        const int last = prev == count - 1;
        if (last) p.tickets[sg.unit] = 0;  // ready for the next call
        *last_flag = last;
      }
      named_barrier_sync(1, kConsumers);
      if (*last_flag) {
        __threadfence();
        for (int e = ctid; e < kHeads * kHeadDim; e += kConsumers) {
          const int h = e / kHeadDim, d = e % kHeadDim;
          if (h >= sg.nheads) continue;
          float mx = kNegBig;
          for (int c = c_first; c <= c_last; ++c) {
            const float *sl = p.partials + (long long)(sg.unit + c) * p.slot_floats;
            mx = fmaxf(mx, __ldcg(sl + h));
          }
          float l = 0.f, a = 0.f;
          for (int c = c_first; c <= c_last; ++c) {
            const float *sl = p.partials + (long long)(sg.unit + c) * p.slot_floats;
            const float w = fast_exp2(__ldcg(sl + h) - mx);
            l += __ldcg(sl + 16 + h) * w;
            a += __ldcg(sl + 32 + e) * w;
          }
          outb[(long long)(sg.head0 + h) * p.o_sh + d] = from_f32<T>(a / (l + 1e-6f));
        }
      }
    }
    it = seg_end;
  }
}

template <typename T, int NT, int DK, int NGROUP>
cudaError_t launch_tc(const DecodeTensorMaps &maps, const DecodeParams &p, int grid,
                      cudaStream_t stream) {
  using L = SmemLayout<NT, NGROUP>;
  const int smem = L::kBytes + 1024;
  auto kern = rotatek_decode_tc_kernel<T, NT, DK, NGROUP>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  kern<<<grid, (kWarpsPerGroup * NGROUP + 1) * 32, smem, stream>>>(maps.kf, maps.vf, maps.ks,
                                                                    maps.vs, p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch_nt_dk(const DecodeTensorMaps &maps, const DecodeParams &p, int nt, int dk,
                           int grid, cudaStream_t stream) {
  constexpr int NG = 2;
  if (nt == 1) {
    if (dk == 16) return launch_tc<T, 1, 16, NG>(maps, p, grid, stream);
    if (dk == 32) return launch_tc<T, 1, 32, NG>(maps, p, grid, stream);
    if (dk == 64) return launch_tc<T, 1, 64, NG>(maps, p, grid, stream);
  } else {
    if (dk == 16) return launch_tc<T, 2, 16, NG>(maps, p, grid, stream);
    if (dk == 32) return launch_tc<T, 2, 32, NG>(maps, p, grid, stream);
    if (dk == 64) return launch_tc<T, 2, 64, NG>(maps, p, grid, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_decode_tc(int dtype_is_bf16, const DecodeTensorMaps &maps, const DecodeParams &p,
                             int heads_tile, int dk, int grid, cudaStream_t stream) {
  const int nt = heads_tile / 8;
  if (dtype_is_bf16) return dispatch_nt_dk<__nv_bfloat16>(maps, p, nt, dk, grid, stream);
  return dispatch_nt_dk<__half>(maps, p, nt, dk, grid, stream);
}

}  // namespace rtk
