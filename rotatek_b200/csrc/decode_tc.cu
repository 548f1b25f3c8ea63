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
//   block  = 32 prompt/text tokens or 64 visual tokens (128 in fp8, two halves
//            of 64) of one unit: first the ceil(S_f/32) full-width blocks, then
//            the visual ones.
//   The U * blocks_per_unit blocks are cut into `grid` contiguous ranges, one
//   per CTA (one CTA per SM), equal except that a range holding a unit start
//   gives up a few blocks for the switch (`Split`).  Inside a CTA, block i goes
//   to consumer warp i % W and ring stage i % S (S a multiple of W: every stage
//   belongs to one warp, so its parity waits are exact).
//
// Warps: one producer, W consumers, no CTA-wide barrier after the prologue.
//   producer  streams each block's K and V tiles with 4-D TMA tensor copies
//             (128B/64B/32B swizzle, no multicast, L2 evict-first: read once)
//             into a ring of ~20 KB stages sized to fill shared memory (10
//             stages = 200 KB in flight per SM at D_keep <= 32); at every unit
//             change its lanes also start cp.async copies of the unit's query
//             rows, R, delta_mu and mask row into a double-buffered header,
//             which arrive on the header's barrier as they land.
//   consumer  builds its own query fragments from the header -- q~^T = R^T q^T
//             on the tensor cores, split into a 16-bit hi + lo pair -- then for
//             each of its blocks
//               S^T[tokens x 8 heads] = K[tokens x d] . Q^T      (mma.m16n8k16)
//               O^T[128 d x 8 heads] += V^T . P^T               (fp32 registers)
//             with P split hi + lo and moved into B fragments by movmatrix, and
//             the running-max rescale only when a max grows.  At the end of a
//             unit it stores its partial (m, l, acc) to its own workspace slot
//             and takes a ticket; the warp that completes the unit's count
//             merges all of the unit's partials in slot order (deterministic)
//             and writes the output.  No warp waits on another warp's merge,
//             except at the end of the CTA's range: the unit of its last
//             segment is merged by all consumer warps together, each taking a
//             share of the heads, after one named barrier among them.
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "decode.h"

namespace rtk {
namespace {

constexpr int kVisTokens = 64;           // tokens per visual block
constexpr int kFullTokens = 32;          // tokens per prompt/text block
constexpr int kHeadDim = 128;
constexpr int kFullBoxBytes = kFullTokens * 128;  // one {64 d x 32 tokens} box
constexpr int kVisBoxBytes = kVisTokens * 128;    // one {64 d x 64 tokens} box
constexpr int kSmemBudget = 232448;      // 227 KB opt-in per CTA
constexpr float kNegBig = -1e30f;        // running-max floor (fused_decode.py:151)

// What the visual span holds:
//   kModeRotK   rotated-truncated Keys k~ [S_v, D_keep] and Values, 16-bit
//   kModeFp8    the same in e4m3 with per-channel Key / per-token Value scales;
//               the Values stored transposed (V^T rows of tokens), so that the
//               e4m3 bytes load straight into f16 A fragments (see fp8_afrag)
//   kModeSpark  SparK's per-token channel pruning: the kept channels' values
//               [S_v, D_keep] (channel order), their channel indices [S_v, D_keep]
//               (uint8, ascending) and the pruned channels' mean per token; the
//               dense Keys are rebuilt in shared memory, 32 tokens at a time, in
//               an area of each consumer warp's own (64-token blocks, two halves)
enum : int { kModeRotK = 0, kModeFp8 = 1, kModeSpark = 2 };

template <int NT, int DK, int MODE = kModeRotK>
struct Cfg {
  static constexpr int kHeads = 8 * NT;
  // consumer warps (SparK: fewer, so that its per-warp rebuild areas and a ring
  // of 22 KB stages fit)
  static constexpr int kWarps = MODE == kModeSpark ? (DK <= 32 ? 4 : 3) : (NT == 1 && DK <= 32) ? 5 : 4;
  static constexpr int kThreads = (kWarps + 1) * 32;             // + producer warp
  static_assert(kWarps <= 5, "the host sizes the workspace for at most 5 partial slots per CTA");
  // visual tokens per block: 64, or in fp8 128 (two halves of 64).  A ring
  // stage's round trip (TMA issue, data in, consumer release, producer refill)
  // takes a few microseconds whatever its size, so the bytes a stage carries
  // set the stream's rate: 128 e4m3 tokens are 20 KB, as many as 64 16-bit ones
  static constexpr int kVisBlk = MODE == kModeFp8 ? 2 * kVisTokens : MODE == kModeSpark ? 2 * kFullTokens
                                                                                        : kVisTokens;
  static_assert(kVisBlk % kVisTokens == 0, "whole 64-token halves");
  static constexpr int kKsBytes = kVisTokens * DK * 2;           // visual Keys of a block
  // SparK visual block (64 tokens): the Values of each 32-token half in two
  // 64-channel boxes | kept values [64][DK] | kept channel indices [64][DK]
  static constexpr int kSpValOff = 4 * kFullBoxBytes;
  static constexpr int kSpIdxOff = kSpValOff + 2 * kFullTokens * DK * 2;
  // fp8 visual block: e4m3 Keys [128 tokens][DK] | e4m3 V^T [128 channels][64
  // tokens] for each half
  static constexpr int kFp8VOff = 2 * kVisTokens * DK;
  static constexpr int kFp8Raw = kFp8VOff + 2 * kVisBoxBytes > 4 * kFullBoxBytes ? kFp8VOff + 2 * kVisBoxBytes
                                                                                 : 4 * kFullBoxBytes;
  static constexpr int kStageRaw = MODE == kModeSpark ? kSpIdxOff + 2 * kFullTokens * DK
                                   : MODE == kModeFp8 ? kFp8Raw
                                                      : kKsBytes + 2 * kVisBoxBytes;
  static constexpr int kStageBytes = (kStageRaw + 1023) / 1024 * 1024;
  static_assert(kStageBytes >= 4 * kFullBoxBytes, "a stage must hold a prompt/text block");
  // per-unit header: q rows [H][128], R [128][DK], delta_mu [128] (16-bit), mask bytes
  static constexpr int kHdrQ = 0;
  static constexpr int kHdrR = kHdrQ + kHeads * kHeadDim * 2;
  static constexpr int kHdrDm = kHdrR + (MODE == kModeSpark ? 0 : kHeadDim * DK * 2);   // SparK: no R
  static constexpr int kHdrMask = kHdrDm + kHeadDim * 2;
  static constexpr int kHdrMaskBytes = 1024;  // prompt/text masks up to this length live here
  static constexpr int kHdrKsc = kHdrMask + kHdrMaskBytes;   // fp8 visual span: Key scales, fp32 [DK]
  static constexpr int kHdrBytes = (kHdrKsc + DK * 4 + 127) / 128 * 128;
  static constexpr int kHdrBufs = DK == 64 ? 1 : 2;
  static constexpr int kMaxStages = 16;
  // barriers: full[16], empty[16], hdr_full[2], hdr_empty[2]; then flags
  static constexpr int kBarOff = 0;
  static constexpr int kFlagOff = kBarOff + (2 * kMaxStages + 4) * 8;
  static constexpr int kHdrOff = 1024;
  static constexpr int kRingOff = (kHdrOff + kHdrBufs * kHdrBytes + 1023) / 1024 * 1024;
  // as many stages as fit, rounded down to a multiple of the consumer warps so
  // that every stage belongs to exactly one warp (its parity waits are exact)
  // SparK: each consumer warp's rebuilt Keys of a 32-token half, after the ring
  static constexpr int kWarpKBytes = MODE == kModeSpark ? 2 * kFullBoxBytes : 0;
  static constexpr int kStages0 = (kSmemBudget - 1024 - kRingOff - kWarps * kWarpKBytes) / kStageBytes;
  static constexpr int kStages = (kStages0 < kMaxStages ? kStages0 : kMaxStages) / kWarps * kWarps;
  static_assert(kStages >= 2 * kWarps, "ring too small: two stages per consumer warp");
  static constexpr int kWarpKOff = kRingOff + kStages * kStageBytes;
  static constexpr int kBytes = kWarpKOff + kWarps * kWarpKBytes;
};

// The split of the U * bpu blocks among the CTAs.  A CTA whose range crosses
// from one unit into the next pays for the switch (partial store and ticket,
// new query fragments, the new unit's first tiles), so each unit counts `ph`
// phantom blocks at its start: CTA c takes the virtual blocks
// [floor(c*Tv/P), floor((c+1)*Tv/P)) of Tv = U * (bpu + ph), and a virtual
// block maps to the real one at or after it.  ph = 0 is the even split.
struct Split {
  long long vtotal;
  int bpu, ph;
  __device__ __forceinline__ long long real_of(long long v) const {
    const long long u = v / (bpu + ph);
    const long long off = v - u * (bpu + ph) - ph;
    return u * bpu + (off > 0 ? off : 0);
  }
  // [lo, hi) of CTA c
  __device__ __forceinline__ long long lo(int c, int grid) const { return real_of((long long)c * vtotal / grid); }
  // the CTA whose range holds real block `blk`
  __device__ __forceinline__ int cta_of(long long blk) const {
    const long long u = blk / bpu;
    const long long v = u * (bpu + ph) + ph + (blk - u * bpu);
    return static_cast<int>(((v + 1) * gridDim.x - 1) / vtotal);
  }
};

// ---- fp8 (e4m3) operands, converted in registers.
// ldmatrix of e4m3 bytes as 16-bit elements gives lane (g, j) = (lane / 4,
// lane % 4) bytes 4j .. 4j+3 of row g of each 8-row x 16-byte matrix.  An
// m16n8k16 A fragment wants row g at k = 2j, 2j+1 (a0, a1 for row g+8) and at
// k = 8+2j, 9+2j (a2, a3), so bytes 4j, 4j+1 serve as k = 2j, 2j+1 and bytes
// 4j+2, 4j+3 as k = 8+2j, 9+2j: the MMA's k index runs over the 16 bytes of a
// row in the order kperm(k) below, and its other operand follows that order.
//   Keys [tokens][channels]: k = channel; the query's B fragments are permuted
//     to channel order kperm once per unit (fp8_query_order).
//   V^T [channels][tokens]: k = token; the probabilities' B fragments hold the
//     logits tile's rows 2j, 2j+1 and 8+2j, 9+2j, so row rho of the logits tile
//     is made token kperm(rho) of its 16 (the Keys' ldmatrix row addresses).
__device__ __forceinline__ int kperm(int k) {   // 0..15 -> 0,1,4,5,8,9,12,13, 2,3,6,7,10,11,14,15
  return ((k & 7) >> 1) * 4 + (k & 1) + ((k >> 3) << 1);
}
// two e4m3 (low byte first) -> two f16 (exact)
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(static_cast<uint16_t>(two)));
  return r;
}
// the A fragment from the two ldmatrix registers of its rows 0-7 and 8-15
__device__ __forceinline__ void fp8_afrag(uint32_t rows0, uint32_t rows8, uint32_t (&a)[4]) {
  a[0] = e4m3x2_to_f16x2(rows0);
  a[1] = e4m3x2_to_f16x2(rows8);
  a[2] = e4m3x2_to_f16x2(rows0 >> 16);
  a[3] = e4m3x2_to_f16x2(rows8 >> 16);
}
// B fragments (k = channel 2j, 2j+1 | 8+2j, 9+2j of head g) -> the same
// channels in kperm order (channels 4j, 4j+1 | 4j+2, 4j+3): from lane
// (g, 2j mod 4) and (g, 2j+1 mod 4), first or second register as 4j < 8
__device__ __forceinline__ void fp8_query_order(uint32_t (&b)[2], int lane) {
  const int s0 = (lane & ~3) | ((2 * lane) & 3);
  const bool first = (lane & 3) < 2;
  const uint32_t x0 = __shfl_sync(0xffffffffu, b[0], s0), y0 = __shfl_sync(0xffffffffu, b[1], s0);
  const uint32_t x1 = __shfl_sync(0xffffffffu, b[0], s0 | 1), y1 = __shfl_sync(0xffffffffu, b[1], s0 | 1);
  b[0] = first ? x0 : y0;
  b[1] = first ? x1 : y1;
}

// Online softmax over MT 16-token tiles of scores already in log2 units,
// then O^T += V^T . P^T with P split hi + lo.  `valid[mt][r]` masks row g8 + 8r
// of tile mt.  V tile: rows = tokens, two 64-d boxes `vbox` bytes apart.
// With `vscale` the probabilities of row g8 + 8r of tile mt are multiplied by
// vscale[mt][r] after the normaliser has taken them (per-token Value scales of
// an fp8 visual span: sum_t p_t (s_t v8_t)).  PLO = false drops the low half of
// P's split (11 bits of P are plenty against e4m3 Values' 4).  V8T: the Values
// are e4m3 V^T rows (channel rows of 64 token bytes, 64-byte swizzle, at vbase)
// and row rho of each score tile is token kperm(rho) of its 16.
template <typename T, int NT, int MT, bool PLO = true, bool V8T = false>
__device__ __forceinline__ void softmax_pv(float (&s)[MT][NT][4], const bool (&valid)[MT][2],
                                           float (&m_run)[NT][2], float (&l_run)[NT][2],
                                           float (&o)[8][NT][4], uint32_t vbase, uint32_t vbox,
                                           int lane, const float (*vscale)[2] = nullptr) {
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if (!valid[mt][0]) s[mt][nt][0] = s[mt][nt][1] = -INFINITY;
      if (!valid[mt][1]) s[mt][nt][2] = s[mt][nt][3] = -INFINITY;
    }
  }
  bool grow = false;
  float mnew[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float mx = fmaxf(s[0][nt][c], s[0][nt][c + 2]);
#pragma unroll
      for (int mt = 1; mt < MT; ++mt) mx = fmaxf(mx, fmaxf(s[mt][nt][c], s[mt][nt][c + 2]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      mnew[nt][c] = fmaxf(m_run[nt][c], mx);
      grow |= mnew[nt][c] > m_run[nt][c];
    }
  }
  if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float a0 = fast_exp2(m_run[nt][0] - mnew[nt][0]);
      const float a1 = fast_exp2(m_run[nt][1] - mnew[nt][1]);
      l_run[nt][0] *= a0;
      l_run[nt][1] *= a1;
#pragma unroll
      for (int d = 0; d < 8; ++d) {
        o[d][nt][0] *= a0;
        o[d][nt][1] *= a1;
        o[d][nt][2] *= a0;
        o[d][nt][3] *= a1;
      }
      m_run[nt][0] = mnew[nt][0];
      m_run[nt][1] = mnew[nt][1];
    }
  }
  // probabilities -> hi/lo B fragments (k = token, n = head) per 16-token tile
  uint32_t pb[MT][NT][2], pl[MT][NT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float p0 = fast_exp2(s[mt][nt][0] - m_run[nt][0]);
      float p1 = fast_exp2(s[mt][nt][1] - m_run[nt][1]);
      float p2 = fast_exp2(s[mt][nt][2] - m_run[nt][0]);
      float p3 = fast_exp2(s[mt][nt][3] - m_run[nt][1]);
      l_run[nt][0] += p0 + p2;
      l_run[nt][1] += p1 + p3;
      if (vscale != nullptr) {
        p0 *= vscale[mt][0];
        p1 *= vscale[mt][0];
        p2 *= vscale[mt][1];
        p3 *= vscale[mt][1];
      }
      float r0, r1, r2, r3;
      const uint32_t h01 = pack2<T>(p0, p1), h23 = pack2<T>(p2, p3);
      unpack2<T>(h01, r0, r1);
      unpack2<T>(h23, r2, r3);
      pb[mt][nt][0] = movmatrix_trans(h01);
      pb[mt][nt][1] = movmatrix_trans(h23);
      if constexpr (PLO) {
        pl[mt][nt][0] = movmatrix_trans(pack2<T>(p0 - r0, p1 - r1));
        pl[mt][nt][1] = movmatrix_trans(pack2<T>(p2 - r2, p3 - r3));
      }
    }
  }
  if constexpr (V8T) {
    // O^T[d, head] += V^T[d, tok] . P^T[tok, head]: e4m3 V^T rows d*16 + 0..15,
    // tokens 16 kk + 0..15 and 16 (kk+1) + 0..15 per ldmatrix
    static_assert(MT % 2 == 0 && !PLO, "token tiles in pairs, P without a low half");
    const int vr = (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
    for (int d = 0; d < 8; ++d) {
#pragma unroll
      for (int kk = 0; kk < MT; kk += 2) {
        uint32_t r[4], a0[4], a1[4];
        ldmatrix_x4(vbase + swizzled_offset<64>(d * 16 + vr, (kk + (lane >> 4)) * 8), r[0], r[1], r[2], r[3]);
        fp8_afrag(r[0], r[1], a0);
        fp8_afrag(r[2], r[3], a1);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_16816<T>(o[d][nt], a0, pb[kk][nt][0], pb[kk][nt][1]);
          mma_16816<T>(o[d][nt], a1, pb[kk + 1][nt][0], pb[kk + 1][nt][1]);
        }
      }
    }
    return;
  }
  // O^T[d, head] += V^T[d, tok] . P^T[tok, head]   (ldmatrix.trans of V rows)
  const int vrow = (lane & 7) + ((lane >> 4) & 1) * 8;
  const int vcol = ((lane >> 3) & 1) * 8;
#pragma unroll
  for (int d = 0; d < 8; ++d) {
    const uint32_t box = vbase + (d >= 4 ? vbox : 0u);
#pragma unroll
    for (int kk = 0; kk < MT; ++kk) {
      uint32_t a[4];
      ldmatrix_x4_trans(box + swizzled_offset<128>(kk * 16 + vrow, (d & 3) * 16 + vcol), a[0], a[1],
                        a[2], a[3]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        mma_16816<T>(o[d][nt], a, pb[kk][nt][0], pb[kk][nt][1]);
        if constexpr (PLO) mma_16816<T>(o[d][nt], a, pl[kk][nt][0], pl[kk][nt][1]);
      }
    }
  }
}

// Copy one unit's small operands into a header buffer (producer warp, all
// lanes): the unit's query rows, R[b, kvh], delta_mu[b, kvh], mask row and (fp8)
// Key scales.  16-byte aligned rows go by cp.async and are not waited for here:
// the caller has each lane arrive on the header's barrier when its copies land,
// so the producer goes back to issuing tiles at once.  The rest is staged
// through registers (every load issued first) and stored before returning.
template <typename T, int NT, int DK, int MODE>
__device__ __forceinline__ void load_header(unsigned char *hdr, const DecodeParams &p, int b,
                                            int kvh, int head0, int nheads, int lane,
                                            const float *ksc = nullptr) {
  using C = Cfg<NT, DK, MODE>;
  constexpr int kHeads = C::kHeads;
  constexpr int kRowChunks = kHeadDim / 8;  // 16-byte chunks of a 128-wide row
  unsigned char *hq = hdr + C::kHdrQ;
  unsigned char *hr = hdr + C::kHdrR;
  T *hd = reinterpret_cast<T *>(hdr + C::kHdrDm);
  uint8_t *hm = hdr + C::kHdrMask;
  const T *q = reinterpret_cast<const T *>(p.q) + (long long)b * p.q_sb;
  const bool q_vec = (p.q_sh * (long long)sizeof(T)) % 16 == 0 &&
                     (reinterpret_cast<uintptr_t>(q + (long long)head0 * p.q_sh) & 15) == 0;
  // query rows (zero rows pad the head tile)
#pragma unroll
  for (int e = lane; e < kHeads * kRowChunks; e += 32) {
    const int h = e / kRowChunks, c = e % kRowChunks;
    unsigned char *dst = hq + e * 16;
    const T *src = q + (long long)(head0 + h) * p.q_sh + c * 8;
    if (h >= nheads) {
      *reinterpret_cast<uint4 *>(dst) = make_uint4(0, 0, 0, 0);
    } else if (q_vec) {
      cp_async_16(dst, src);
    } else {
      T tmp[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) tmp[k] = src[k];
      *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<uint4 *>(tmp);
    }
  }
  if (p.R != nullptr) {
    const T *Rb = reinterpret_cast<const T *>(p.R) + (long long)b * p.R_sb + (long long)kvh * p.R_sh;
    if (p.R_sd == DK && (reinterpret_cast<uintptr_t>(Rb) & 15) == 0) {
#pragma unroll
      for (int e = lane; e < kHeadDim * DK / 8; e += 32) cp_async_16(hr + e * 16, Rb + e * 8);
    } else {
      T *hrt = reinterpret_cast<T *>(hr);
      for (int e = lane; e < kHeadDim * DK; e += 32) hrt[e] = Rb[(long long)(e / DK) * p.R_sd + e % DK];
    }
  }
  const T *dmr = p.dm != nullptr
                     ? reinterpret_cast<const T *>(p.dm) + (long long)b * p.dm_sb + (long long)kvh * p.dm_sh
                     : nullptr;
  if (dmr != nullptr && (reinterpret_cast<uintptr_t>(dmr) & 15) == 0) {
    if (lane < kHeadDim / 8) cp_async_16(hd + lane * 8, dmr + lane * 8);
  } else {
    T dv[kHeadDim / 32];
#pragma unroll
    for (int k = 0; k < kHeadDim / 32; ++k) dv[k] = dmr != nullptr ? dmr[lane + 32 * k] : from_f32<T>(0.f);
#pragma unroll
    for (int k = 0; k < kHeadDim / 32; ++k) hd[lane + 32 * k] = dv[k];
  }
  if (ksc != nullptr) {   // fp8 visual span: this unit's Key scales
    float *hk = reinterpret_cast<float *>(hdr + C::kHdrKsc);
    if ((reinterpret_cast<uintptr_t>(ksc) & 15) == 0) {
      for (int c = lane; c < DK / 4; c += 32) cp_async_16(hk + 4 * c, ksc + 4 * c);
    } else {
      for (int c = lane; c < DK; c += 32) hk[c] = ksc[c];
    }
  }
  const uint8_t *mrow = p.mask != nullptr ? p.mask + (long long)b * p.mask_sb : nullptr;
  if (mrow != nullptr && p.seq_full <= C::kHdrMaskBytes && p.mask_ss == 1 &&
      (reinterpret_cast<uintptr_t>(mrow) & 15) == 0) {
    // the row's bytes only: the last chunk's tail is zero-filled, not read
    for (int c = lane; c * 16 < p.seq_full; c += 32)
      cp_async_16_zfill(hm + 16 * c, mrow + 16 * c, min(16, p.seq_full - 16 * c));
  } else if (mrow != nullptr && p.seq_full <= C::kHdrMaskBytes) {
    uint8_t mv[C::kHdrMaskBytes / 32];
#pragma unroll
    for (int k = 0; k < C::kHdrMaskBytes / 32; ++k) {
      const int t = lane + 32 * k;
      mv[k] = t < p.seq_full ? mrow[(long long)t * p.mask_ss] : 0;
    }
#pragma unroll
    for (int k = 0; k < C::kHdrMaskBytes / 32; ++k) hm[lane + 32 * k] = mv[k];
  }
}

// Merge of one unit's partials (one per consumer warp of CTAs c_first..c_last),
// in slot order (deterministic): per-head max, weights 2^(m_k - max), weighted
// sums; output in the query dtype.  KH = heads merged: the slot's heads
// hb .. hb+KH-1 (a single-head unit -- G = 1 -- reads one head per slot).  Each
// head's sums run in slot order whatever KH, so warps that split a unit's
// heads among them write the same bits as one warp merging them all.
template <typename T, int KH, int kWarps>
__device__ __forceinline__ void merge_unit(const DecodeParams &p, int unit, int c_first, int c_last,
                                           int bk, int head0, int nheads, int lane, int hb = 0,
                                           bool acquire = true) {

  // every partial of the unit is in place: merge them in slot order.
  // Pass 1: lane k holds slot k0 + k; per-head max and normaliser by shuffles.
  if (acquire) __threadfence();
  const float *s0 = p.partials + (long long)(unit + c_first) * kWarps * p.slot_floats;
  const int nslots = kWarps * (c_last - c_first + 1);
  float mx[KH];
#pragma unroll
  for (int h = 0; h < KH; ++h) mx[h] = kNegBig;
  for (int k0 = 0; k0 < nslots; k0 += 32) {
    const bool on = k0 + lane < nslots;
    const float *sl = s0 + (long long)(k0 + lane) * p.slot_floats;
#pragma unroll
    for (int h = 0; h < KH; ++h) {
      float v = on ? __ldcg(sl + hb + h) : kNegBig;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
      mx[h] = fmaxf(mx[h], v);
    }
  }
  // Pass 2: weights w[k][h] = 2^(m_k - max) (lane k), then acc over slots;
  // lane owns channels 4*lane .. 4*lane+3 of every head.
  float lsum[KH];
  float4 acc[KH];
#pragma unroll
  for (int h = 0; h < KH; ++h) {
    lsum[h] = 0.f;
    acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int k0 = 0; k0 < nslots; k0 += 32) {
    const bool on = k0 + lane < nslots;
    const float *sl = s0 + (long long)(k0 + lane) * p.slot_floats;
    float w[KH];
#pragma unroll
    for (int h = 0; h < KH; ++h) {
      w[h] = on ? fast_exp2(__ldcg(sl + hb + h) - mx[h]) : 0.f;
      float lw = on ? __ldcg(sl + 16 + hb + h) * w[h] : 0.f;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, off);
      lsum[h] += lw;
    }
    // kU slots per step with all their loads issued first: the L2 round
    // trips overlap instead of running one slot at a time
    constexpr int kU = KH == 1 ? 32 : KH == 2 ? 16 : KH == 4 ? 8 : KH == 8 ? 4 : 1;
    const int nk = min(32, nslots - k0);
    for (int k = 0; k < nk; k += kU) {
      float4 v[kU][KH];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const float4 *ok =
            reinterpret_cast<const float4 *>(s0 + (long long)(k0 + k + u) * p.slot_floats + 32) + lane;
#pragma unroll
        for (int h = 0; h < KH; ++h)
          v[u][h] = k + u < nk ? __ldcg(ok + (hb + h) * (kHeadDim / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
#pragma unroll
        for (int h = 0; h < KH; ++h) {
          const float wk = __shfl_sync(0xffffffffu, w[h], (k + u) & 31);
          acc[h].x += v[u][h].x * wk;
          acc[h].y += v[u][h].y * wk;
          acc[h].z += v[u][h].z * wk;
          acc[h].w += v[u][h].w * wk;
        }
      }
    }
  }
  T *outb = reinterpret_cast<T *>(p.out) + (long long)bk * p.o_sb;
#pragma unroll
  for (int h = 0; h < KH; ++h) {
    if (hb + h < nheads) {
      const float inv = 1.f / (lsum[h] + 1e-6f);
      T *orow = outb + (long long)(head0 + hb + h) * p.o_sh + lane * 4;
      orow[0] = from_f32<T>(acc[h].x * inv);
      orow[1] = from_f32<T>(acc[h].y * inv);
      orow[2] = from_f32<T>(acc[h].z * inv);
      orow[3] = from_f32<T>(acc[h].w * inv);
    }
  }
}

// byte offset of 16-byte chunk c of row t in a TMA box of DK-byte rows
template <int DK>
__device__ __forceinline__ uint32_t k8_offset(int t, int c) {
  if constexpr (DK == 16) return static_cast<uint32_t>(t) * 16;
  else return swizzled_offset<DK>(t, c * 8);
}

// SparK visual block: rebuild one 32-token half's full-width Keys in `kdst` as
// the two 128B-swizzled {64 channels x 32 tokens} boxes a prompt/text block
// has, from the kept values and channel indices (rows 32 half + 0..31) the TMA
// put at kSpValOff / kSpIdxOff of stage `st` --
// the adapters' recovery (llama_visionzip.py:226-230): every channel first
// takes the token's pruned-channel mean, then the kept channels their values.
// Lane t owns token row t (its fill, its scatter), so only the caller's
// __syncwarp before the MMAs orders lanes.  `mean2` is the token's mean (16-bit
// bits) in both halves.  Indices are taken mod 128, so no write leaves the row.
// The area is this warp's own (no TMA writes it), so its 16-byte chunks are
// swizzled by (row & 7) ^ ((row >> 3) & 3) rather than the TMA's row & 7: each
// 8-row ldmatrix group still sees 8 distinct chunks, and rows t, t+8, t+16,
// t+24 -- which under row & 7 put a channel that all four keep in one bank --
// now differ.  spark_key_xor gives the reader the extra term.
template <int DK>
__device__ __forceinline__ void rebuild_spark_keys(unsigned char *kdst, const unsigned char *st, int half,
                                                   int lane, uint32_t mean2) {
  constexpr int kValOff = Cfg<1, DK, kModeSpark>::kSpValOff;
  constexpr int kIdxOff = Cfg<1, DK, kModeSpark>::kSpIdxOff;
  const int t = half * kFullTokens + lane;   // this lane's row of the kept values / indices
  const uint32_t row = smem_u32(kdst) + static_cast<uint32_t>(lane) * 128;
  const uint32_t x = static_cast<uint32_t>((lane & 7) ^ ((lane >> 3) & 3)) << 4;   // the row's chunk pattern
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    st_shared_v4(row + ((c << 4) ^ x), mean2, mean2, mean2, mean2);
    st_shared_v4(row + kFullBoxBytes + ((c << 4) ^ x), mean2, mean2, mean2, mean2);
  }
  uint32_t val[DK / 2], idx[DK / 4];
#pragma unroll
  for (int c = 0; c < DK / 8; ++c) {
    const uint4 v = *reinterpret_cast<const uint4 *>(st + kValOff + swizzled_offset<DK * 2>(t, c * 8));
    val[4 * c] = v.x; val[4 * c + 1] = v.y; val[4 * c + 2] = v.z; val[4 * c + 3] = v.w;
  }
#pragma unroll
  for (int c = 0; c < DK / 16; ++c) {
    const uint4 v = *reinterpret_cast<const uint4 *>(st + kIdxOff + k8_offset<DK>(t, c));
    idx[4 * c] = v.x; idx[4 * c + 1] = v.y; idx[4 * c + 2] = v.z; idx[4 * c + 3] = v.w;
  }
#pragma unroll
  for (int k = 0; k < DK; ++k) {
    const uint32_t b2 = ((idx[k >> 2] >> (8 * (k & 3))) & 127u) << 1;   // byte offset in a 256-byte row
    const uint32_t addr = row + ((b2 & 128u) << 5) + ((b2 & 127u) ^ x);  // box 1 holds channels 64-127
    st_shared_u16(addr, static_cast<uint16_t>(val[k >> 1] >> (16 * (k & 1))));
  }
}

// The rebuilt Keys' extra chunk XOR for row `row` (see rebuild_spark_keys), as
// a byte mask to XOR into a 128B-swizzled offset.
__device__ __forceinline__ uint32_t spark_key_xor(int row) { return static_cast<uint32_t>((row >> 3) & 3) << 4; }

template <typename T, int NT, int DK, int MODE>
__global__ void __launch_bounds__(Cfg<NT, DK, MODE>::kThreads, 1)
    rotatek_decode_tc_kernel(const __grid_constant__ CUtensorMap tm_kf,
                             const __grid_constant__ CUtensorMap tm_vf,
                             const __grid_constant__ CUtensorMap tm_ks,
                             const __grid_constant__ CUtensorMap tm_vs,
                             const __grid_constant__ CUtensorMap tm_ki, const DecodeParams p,
                             const DecodeFp8 f8, const DecodeSpark sp) {
  constexpr bool FP8 = MODE == kModeFp8;
  constexpr bool SPARK = MODE == kModeSpark;
  // the visual span's MMAs run in f16 when it is stored in fp8 (e4m3 -> f16 is exact)
  using TV = typename std::conditional<FP8, __half, T>::type;
  using C = Cfg<NT, DK, MODE>;
  constexpr int kHeads = C::kHeads;
  constexpr int kStages = C::kStages;
  constexpr int kWarps = C::kWarps;
  constexpr int kNB = C::kHdrBufs;
  constexpr int kKsRowBytes = DK * 2;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *full_bar = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
  uint64_t *empty_bar = full_bar + C::kMaxStages;
  uint64_t *hdr_full = empty_bar + C::kMaxStages;
  uint64_t *hdr_empty = hdr_full + 2;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::kFlagOff);
  // the unit whose merge the consumer warps share at the end (unit, c_first,
  // c_last, whether the CTA released its partials; unit -1 = none)
  volatile int *pending = abort_flag + 1;
  unsigned char *ring = smem + C::kRingOff;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bpu = p.blocks_per_unit;
  const Split split{p.total_blocks / bpu * (bpu + p.phantom), bpu, p.phantom};
  const long long lo = split.lo(blockIdx.x, gridDim.x);
  const long long hi = split.lo(blockIdx.x + 1, gridDim.x);
  const int nblk = static_cast<int>(hi - lo);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < kNB; ++b) {
      mbar_init(&hdr_full[b], 1);
      mbar_init(&hdr_empty[b], kWarps);
    }
    *abort_flag = 0;
    pending[0] = -1;
    fence_barrier_init();
  }
  __syncthreads();

  // ======================================================== producer warp
  if (warp == kWarps) {
    if (lane == 0) {
      if (p.blocks_full > 0) { tma_prefetch_desc(&tm_kf); tma_prefetch_desc(&tm_vf); }
      if (p.blocks_sparse > 0) { tma_prefetch_desc(&tm_ks); tma_prefetch_desc(&tm_vs); }
      if (SPARK && p.blocks_sparse > 0) tma_prefetch_desc(&tm_ki);
    }
    int unit = static_cast<int>(lo / bpu);
    int j = static_cast<int>(lo - (long long)unit * bpu);
    int seg = -1, bk = 0, kvh = 0, issued = 0;
    // K/V tiles are read once: let them leave L2 first, so that the split
    // partials (written early, merged at the end) stay there
    const uint64_t stream_pol = l2_evict_first_policy();
    for (int i = 0; i < nblk; ++i) {
      if (i == 0 || j == 0) {
        // a new unit: its header goes into buffer seg % kNB once the consumers
        // are done with the unit that used the buffer before
        ++seg;
        const int buf = seg % kNB;
        const int hc = unit % p.head_chunks;
        kvh = (unit / p.head_chunks) % p.kv_heads;
        bk = unit / (p.kv_heads * p.head_chunks);
        int ok = 1;
        if (lane == 0) ok = mbar_wait_bounded(&hdr_empty[buf], ((seg / kNB) & 1) ^ 1, abort_flag, p.status);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (ok)
          load_header<T, NT, DK, MODE>(smem + C::kHdrOff + buf * C::kHdrBytes, p, bk, kvh,
                                 kvh * p.groups + hc * kHeads, min(kHeads, p.groups - hc * kHeads), lane,
                                 FP8 ? f8.k_scale + (long long)bk * f8.ksc_sb + (long long)kvh * f8.ksc_sh
                                     : nullptr);
        // not waited for: tiles keep streaming while it lands (a wait here left
        // a ~5 us gap in the tile stream at each unit switch)
        cp_async_mbar_arrive(&hdr_full[buf]);   // this lane's copies, when they land
        __syncwarp();
        if (lane == 0) mbar_arrive(&hdr_full[buf]);   // the staged stores
      }
      if (lane == 0) {
        const int stage = i % kStages;
        if (mbar_wait_bounded(&empty_bar[stage], ((i / kStages) & 1) ^ 1, abort_flag, p.status)) {
          unsigned char *st = ring + stage * C::kStageBytes;
          if (j < p.blocks_full) {
            const int tok = j * kFullTokens;
            mbar_arrive_expect_tx(&full_bar[stage], 4 * kFullBoxBytes);
            tma_load_4d_hint(st, &tm_kf, 0, tok, kvh, bk, &full_bar[stage], stream_pol);
            tma_load_4d_hint(st + kFullBoxBytes, &tm_kf, 64, tok, kvh, bk, &full_bar[stage], stream_pol);
            tma_load_4d_hint(st + 2 * kFullBoxBytes, &tm_vf, 0, tok, kvh, bk, &full_bar[stage], stream_pol);
            tma_load_4d_hint(st + 3 * kFullBoxBytes, &tm_vf, 64, tok, kvh, bk, &full_bar[stage], stream_pol);
          } else if constexpr (SPARK) {
            // the Values of both 32-token halves, the kept values and the kept
            // channel indices of all 64 tokens; the consumer rebuilds the Keys
            const int tok = (j - p.blocks_full) * C::kVisBlk;
            mbar_arrive_expect_tx(&full_bar[stage], 4 * kFullBoxBytes + C::kVisBlk * DK * 3);
            tma_load_4d_hint(st, &tm_vs, 0, tok, kvh, bk, &full_bar[stage], stream_pol);
            tma_load_4d_hint(st + kFullBoxBytes, &tm_vs, 64, tok, kvh, bk, &full_bar[stage], stream_pol);
            tma_load_4d_hint(st + 2 * kFullBoxBytes, &tm_vs, 0, tok + kFullTokens, kvh, bk, &full_bar[stage],
                             stream_pol);
            tma_load_4d_hint(st + 3 * kFullBoxBytes, &tm_vs, 64, tok + kFullTokens, kvh, bk, &full_bar[stage],
                             stream_pol);
            tma_load_4d_hint(st + C::kSpValOff, &tm_ks, 0, tok, kvh, bk, &full_bar[stage], stream_pol);
            tma_load_4d_hint(st + C::kSpIdxOff, &tm_ki, 0, tok, kvh, bk, &full_bar[stage], stream_pol);
          } else {
            const int tok = (j - p.blocks_full) * kVisTokens;
            if constexpr (FP8) {
              // 128 e4m3 Key rows, then the 128 V^T rows of each 64-token half
              const int tok2 = (j - p.blocks_full) * C::kVisBlk;
              mbar_arrive_expect_tx(&full_bar[stage], C::kVisBlk * DK + 2 * kVisBoxBytes);
              tma_load_4d_hint(st, &tm_ks, 0, tok2, kvh, bk, &full_bar[stage], stream_pol);
              tma_load_4d_hint(st + C::kFp8VOff, &tm_vs, tok2, 0, kvh, bk, &full_bar[stage], stream_pol);
              tma_load_4d_hint(st + C::kFp8VOff + kVisBoxBytes, &tm_vs, tok2 + kVisTokens, 0, kvh, bk,
                               &full_bar[stage], stream_pol);
            } else {
              mbar_arrive_expect_tx(&full_bar[stage], C::kKsBytes + 2 * kVisBoxBytes);
              tma_load_4d_hint(st, &tm_ks, 0, tok, kvh, bk, &full_bar[stage], stream_pol);
              tma_load_4d_hint(st + C::kKsBytes, &tm_vs, 0, tok, kvh, bk, &full_bar[stage], stream_pol);
              tma_load_4d_hint(st + C::kKsBytes + kVisBoxBytes, &tm_vs, 64, tok, kvh, bk, &full_bar[stage], stream_pol);
            }
          }
          ++issued;
        }
      }
      if (++j == bpu) {
        j = 0;
        ++unit;
      }
    }
    cp_async_wait_all();   // no header copy in flight when the warp exits
    if (lane == 0 && *abort_flag) {
      // leave no copy in flight: wait (bounded) for the stages still loading
      const int first = issued > kStages ? issued - kStages : 0;
      for (int i = first; i < issued; ++i) {
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(&full_bar[i % kStages], (i / kStages) & 1)) {
          if (globaltimer_ns() - t0 > kWaitLimitNs / 4) break;
        }
      }
    }
    return;
  }

  // ======================================================== consumer warps
  const int cw = warp;                // consumer warp: owns blocks i = cw (mod kWarps)
  const int g8 = lane >> 2;           // fragment row
  const int t4 = lane & 3;            // fragment column pair
  const int arow = (lane & 7) + ((lane >> 3) & 1) * 8;   // A-operand (ldmatrix) row
  const int acol = (lane >> 4) * 8;                      // A-operand column offset

  int it = 0;
  int seg = -1;
  int unit = static_cast<int>(lo / bpu);
  while (it < nblk) {
    ++seg;
    const int buf = seg % kNB;
    const long long unit_end = (long long)(unit + 1) * bpu;
    const int seg_end = static_cast<int>((hi < unit_end ? hi : unit_end) - lo);
    const int j0 = static_cast<int>(lo + it - (long long)unit * bpu);  // first block of the unit here
    const int hc = unit % p.head_chunks;
    const int bk = unit / (p.kv_heads * p.head_chunks);
    const int kvh = (unit / p.head_chunks) % p.kv_heads;
    const int head0 = kvh * p.groups + hc * kHeads;
    const int nheads = min(kHeads, p.groups - hc * kHeads);

    // ---- unit header -> this warp's query fragments (no CTA-wide barrier)
    mbar_wait_bounded(&hdr_full[buf], (seg / kNB) & 1, abort_flag, p.status);
    const unsigned char *hdr = smem + C::kHdrOff + buf * C::kHdrBytes;
    const uint32_t hq = smem_u32(hdr + C::kHdrQ);
    const uint32_t hr = smem_u32(hdr + C::kHdrR);
    const T *hdm = reinterpret_cast<const T *>(hdr + C::kHdrDm);
    const uint8_t *hmask = hdr + C::kHdrMask;
    // full-width query B fragments (k = d, n = head): ldmatrix of the query rows
    uint32_t qf[kHeadDim / 16][NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int ks = 0; ks < kHeadDim / 16; ks += 2) {
        const int row = nt * 8 + (lane & 7);
        const int col = (ks + (lane >> 4)) * 16 + ((lane >> 3) & 1) * 8;
        ldmatrix_x4(hq + row * (kHeadDim * 2) + col * 2, qf[ks][nt][0], qf[ks][nt][1],
                    qf[ks + 1][nt][0], qf[ks + 1][nt][1]);
      }
    }
    // q~^T[ch, head] = R^T . q^T on the tensor cores (fp32 accumulate), then the
    // fp32 result -> 16-bit hi + lo B fragments (k = channel, n = head)
    uint32_t qhi[DK / 16][NT][2], qlo[DK / 16][NT][2];
#pragma unroll
    for (int mt = 0; mt < (SPARK ? 0 : DK / 16); ++mt) {
      float c[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) c[nt][0] = c[nt][1] = c[nt][2] = c[nt][3] = 0.f;
      if (p.R != nullptr) {
#pragma unroll
        for (int ks = 0; ks < kHeadDim / 16; ++ks) {
          uint32_t a[4];
          const int d = ks * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
          const int ch = mt * 16 + ((lane >> 3) & 1) * 8;
          ldmatrix_x4_trans(hr + d * kKsRowBytes + ch * 2, a[0], a[1], a[2], a[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_16816<T>(c[nt], a, qf[ks][nt][0], qf[ks][nt][1]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          float v0 = c[nt][2 * half], v1 = c[nt][2 * half + 1];
          if constexpr (FP8) {   // channel mt*16 + g8 + 8 half: fold its Key scale in
            const float sc = reinterpret_cast<const float *>(hdr + C::kHdrKsc)[mt * 16 + (lane >> 2) + 8 * half];
            v0 *= sc;
            v1 *= sc;
          }
          const uint32_t h = pack2<TV>(v0, v1);
          float h0, h1;
          unpack2<TV>(h, h0, h1);
          qhi[mt][nt][half] = movmatrix_trans(h);
          qlo[mt][nt][half] = movmatrix_trans(pack2<TV>(v0 - h0, v1 - h1));
        }
        if constexpr (FP8) {   // the e4m3 Key fragments' channel order
          fp8_query_order(qhi[mt][nt], lane);
          fp8_query_order(qlo[mt][nt], lane);
        }
      }
    }
    // bias = q . delta_mu per head: lane sums 4 channels, butterfly over the warp
    float bias2[NT][2];
    if constexpr (SPARK) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) bias2[nt][0] = bias2[nt][1] = 0.f;
    } else {
      float dmv[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) dmv[k] = to_f32(hdm[lane * 4 + k]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        bias2[nt][0] = bias2[nt][1] = 0.f;
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const T *qrow = reinterpret_cast<const T *>(hdr + C::kHdrQ) + (nt * 8 + h) * kHeadDim + lane * 4;
          float part = 0.f;
#pragma unroll
          for (int k = 0; k < 4; ++k) part = fmaf(to_f32(qrow[k]), dmv[k], part);
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
          if (h == 2 * t4) bias2[nt][0] = part;
          if (h == 2 * t4 + 1) bias2[nt][1] = part;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&hdr_empty[buf]);

    float o[8][NT][4];
    float m_run[NT][2], l_run[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m_run[nt][0] = m_run[nt][1] = kNegBig;
      l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
      for (int d = 0; d < 8; ++d) o[d][nt][0] = o[d][nt][1] = o[d][nt][2] = o[d][nt][3] = 0.f;
    }

    // ---- this warp's blocks of the segment
    const int first = it + ((cw - it) % kWarps + kWarps) % kWarps;
    for (int i = first; i < seg_end; i += kWarps) {
      const int stage = i % kStages;
      const int j = j0 + (i - it);
      // fp8 span: this block's per-token Value scales (rows g8, g8 + 8 of each
      // score tile: tokens kperm(g8), kperm(g8) + 2), requested before the
      // stage wait so that their L2 latency hides behind it
      float vs[2][4][2];
      if constexpr (FP8) {
        if (j >= p.blocks_full) {
          const float *vsc = f8.v_scale + (long long)bk * f8.vsc_sb + (long long)kvh * f8.vsc_sh;
          const int tv = (j - p.blocks_full) * C::kVisBlk + kperm(g8);
#pragma unroll
          for (int hf = 0; hf < 2; ++hf)
#pragma unroll
            for (int mt = 0; mt < 4; ++mt)
#pragma unroll
              for (int r = 0; r < 2; ++r) {
                const int tok = tv + hf * kVisTokens + mt * 16 + 2 * r;
                vs[hf][mt][r] = tok < p.seq_sparse ? __ldg(vsc + (long long)tok * f8.vsc_ss) : 0.f;
              }
        }
      }
      // SparK span: this lane's tokens' pruned-channel means (one per half),
      // requested before the stage wait
      uint32_t mean2[2] = {0u, 0u};
      if constexpr (SPARK) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int tok = (j - p.blocks_full) * C::kVisBlk + hf * kFullTokens + lane;
          if (j >= p.blocks_full && tok < p.seq_sparse) {
            const uint32_t m = __ldg(reinterpret_cast<const unsigned short *>(sp.mean) + (long long)bk * sp.mean_sb +
                                     (long long)kvh * sp.mean_sh + (long long)tok * sp.mean_ss);
            mean2[hf] = m | (m << 16);
          }
        }
      }
      const bool ready = mbar_wait_bounded(&full_bar[stage], (i / kStages) & 1, abort_flag, p.status);
      const uint32_t sbase = smem_u32(ring + stage * C::kStageBytes);
      const bool spark_vis = SPARK && j >= p.blocks_full;
      if (ready) {
        if (j < p.blocks_full || spark_vis) {
          // ---- 32 tokens at full width, q . k: a prompt/text block, or each
          //      32-token half of a SparK visual block once its Keys are rebuilt
          //      in this warp's area
          unsigned char *wk = smem + C::kWarpKOff + cw * C::kWarpKBytes;
#pragma unroll 1
          for (int hf = 0; hf < (spark_vis ? 2 : 1); ++hf) {
          const int tok0 = spark_vis ? (j - p.blocks_full) * C::kVisBlk + hf * kFullTokens : j * kFullTokens;
          if (spark_vis && tok0 >= p.seq_sparse) break;   // a SparK block's second half past the span
          uint32_t kb = sbase, vb = sbase + 2 * kFullBoxBytes;
          bool rebuilt = false;   // Keys in this warp's area (their own chunk pattern)
          if constexpr (SPARK) {
            if (spark_vis) {
              __syncwarp();   // every lane is done with the previous half's Keys
              rebuild_spark_keys<DK>(wk, ring + stage * C::kStageBytes, hf, lane, hf == 0 ? mean2[0] : mean2[1]);
              __syncwarp();
              kb = smem_u32(wk);
              vb = sbase + hf * 2 * kFullBoxBytes;
              rebuilt = true;
            }
          }
          float s[2][NT][4];
#pragma unroll
          for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) s[mt][nt][0] = s[mt][nt][1] = s[mt][nt][2] = s[mt][nt][3] = 0.f;
#pragma unroll
          for (int ks = 0; ks < kHeadDim / 16; ++ks) {
            const uint32_t box = kb + (ks >= 4 ? (uint32_t)kFullBoxBytes : 0u);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
              uint32_t a[4];
              const uint32_t kx = rebuilt ? spark_key_xor(mt * 16 + arow) : 0u;
              ldmatrix_x4(box + (swizzled_offset<128>(mt * 16 + arow, (ks & 3) * 16 + acol) ^ kx), a[0],
                          a[1], a[2], a[3]);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) mma_16816<T>(s[mt][nt], a, qf[ks][nt][0], qf[ks][nt][1]);
            }
          }
          bool valid[2][2];
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
              const int tok = tok0 + mt * 16 + g8 + 8 * r;
              bool v = tok < (spark_vis ? p.seq_sparse : p.seq_full);
              if (v && !spark_vis && p.mask != nullptr)
                v = (p.seq_full <= C::kHdrMaskBytes ? hmask[tok]
                                                    : p.mask[(long long)bk * p.mask_sb +
                                                             (long long)tok * p.mask_ss]) != 0;
              valid[mt][r] = v;
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int e = 0; e < 4; ++e) s[mt][nt][e] *= p.scale_log2;
          }
          softmax_pv<T, NT, 2>(s, valid, m_run, l_run, o, vb, kFullBoxBytes, lane);
          }
        } else if constexpr (!SPARK) {
          // ---- visual block: 64 tokens (fp8: two halves of 64), rotated-truncated
          //      Keys, (q~ . k~ + bias)
#pragma unroll
          for (int hf = 0; hf < C::kVisBlk / kVisTokens; ++hf) {
          const int tok0 = (j - p.blocks_full) * C::kVisBlk + hf * kVisTokens;
          if (tok0 >= p.seq_sparse) break;   // only an fp8 block's second half lies past the span
          const uint32_t kbase = sbase + hf * kVisTokens * DK;   // this half's e4m3 Key rows
          float s[4][NT][4];
#pragma unroll
          for (int mt = 0; mt < 4; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) s[mt][nt][0] = s[mt][nt][1] = s[mt][nt][2] = s[mt][nt][3] = 0.f;
          if constexpr (FP8) {
            // e4m3 Key rows straight into f16 A fragments; lane l addresses
            // token kperm(l % 16) of the tile (and its next 16-byte chunk, or
            // for D_keep 16 the next tile, in lanes 16-31)
            const int krow = kperm(lane & 15);
            auto kmma = [&](int mt, int ks, const uint32_t (&a)[4]) {
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                mma_16816<TV>(s[mt][nt], a, qhi[ks][nt][0], qhi[ks][nt][1]);
                mma_16816<TV>(s[mt][nt], a, qlo[ks][nt][0], qlo[ks][nt][1]);
              }
            };
#pragma unroll
            for (int mt = 0; mt < 4; mt += (DK == 16 ? 2 : 1)) {
#pragma unroll
              for (int kc = 0; kc < (DK == 16 ? 1 : DK / 32); ++kc) {
                uint32_t r[4], a0[4], a1[4];
                const int t = DK == 16 ? (mt + (lane >> 4)) * 16 + krow : mt * 16 + krow;
                const int c = DK == 16 ? 0 : 2 * kc + (lane >> 4);
                ldmatrix_x4(kbase + k8_offset<DK>(t, c), r[0], r[1], r[2], r[3]);
                fp8_afrag(r[0], r[1], a0);
                fp8_afrag(r[2], r[3], a1);
                if constexpr (DK == 16) {
                  kmma(mt, 0, a0);
                  kmma(mt + 1, 0, a1);
                } else {
                  kmma(mt, 2 * kc, a0);
                  kmma(mt, 2 * kc + 1, a1);
                }
              }
            }
          } else {
#pragma unroll
            for (int ks = 0; ks < DK / 16; ++ks) {
#pragma unroll
              for (int mt = 0; mt < 4; ++mt) {
                uint32_t a[4];
                ldmatrix_x4(sbase + swizzled_offset<kKsRowBytes>(mt * 16 + arow, ks * 16 + acol), a[0],
                            a[1], a[2], a[3]);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                  mma_16816<TV>(s[mt][nt], a, qhi[ks][nt][0], qhi[ks][nt][1]);
                  mma_16816<TV>(s[mt][nt], a, qlo[ks][nt][0], qlo[ks][nt][1]);
                }
              }
            }
          }
          // rows g8 and g8 + 8 of tile mt: tokens g8, g8 + 8, or for fp8
          // kperm(g8), kperm(g8) + 2
          const int row0 = FP8 ? kperm(g8) : g8, row1 = FP8 ? row0 + 2 : g8 + 8;
          bool valid[4][2];
#pragma unroll
          for (int mt = 0; mt < 4; ++mt) {
            valid[mt][0] = tok0 + mt * 16 + row0 < p.seq_sparse;
            valid[mt][1] = tok0 + mt * 16 + row1 < p.seq_sparse;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              s[mt][nt][0] = (s[mt][nt][0] + bias2[nt][0]) * p.scale_log2;
              s[mt][nt][1] = (s[mt][nt][1] + bias2[nt][1]) * p.scale_log2;
              s[mt][nt][2] = (s[mt][nt][2] + bias2[nt][0]) * p.scale_log2;
              s[mt][nt][3] = (s[mt][nt][3] + bias2[nt][1]) * p.scale_log2;
            }
          }
          if constexpr (FP8) {
            // per-token Value scales of the fp8 span fold into the probabilities
            softmax_pv<TV, NT, 4, false, true>(s, valid, m_run, l_run, o,
                                               sbase + C::kFp8VOff + hf * kVisBoxBytes, 0u, lane, vs[hf]);
          } else {
            softmax_pv<T, NT, 4>(s, valid, m_run, l_run, o, sbase + C::kKsBytes, kVisBoxBytes, lane);
          }
          }
        }
      }
      // this warp's reads (and, for SparK, in-place writes) of the stage
      // are ordered before the TMA write that refills it (async proxy)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[stage]);
    }

    // ---- segment end: this warp's partial (m, l, acc) -> its workspace slot
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
    }
    const long long ublk0 = (long long)unit * bpu;
    const int c_first = split.cta_of(ublk0);
    const int c_last = split.cta_of(ublk0 + bpu - 1);
    float *slot = p.partials + ((long long)(unit + blockIdx.x) * kWarps + cw) * p.slot_floats;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int h = nt * 8 + 2 * t4 + c;
        if (h >= nheads) continue;  // padding heads: never merged
        if (g8 == 0) {
          slot[h] = m_run[nt][c];
          slot[16 + h] = l_run[nt][c];
        }
#pragma unroll
        for (int d = 0; d < 8; ++d) {
          slot[32 + h * kHeadDim + d * 16 + g8] = o[d][nt][c];
          slot[32 + h * kHeadDim + d * 16 + g8 + 8] = o[d][nt][2 + c];
        }
      }
    }
    if (seg_end == nblk) break;   // the CTA's last segment: one ticket for all warps, below
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      const int count = kWarps * (c_last - c_first + 1);
      const int prev = atomicAdd(&p.tickets[unit], 1);
      last = prev == count - 1;
      if (last) p.tickets[unit] = 0;  // ready for the next call
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      if (nheads == 1)
        merge_unit<T, 1, kWarps>(p, unit, c_first, c_last, bk, head0, nheads, lane);
      else
        merge_unit<T, kHeads, kWarps>(p, unit, c_first, c_last, bk, head0, nheads, lane);
    }
    it = seg_end;
    ++unit;
  }

  // ---- the CTA's last segment (unit `unit`): every consumer warp has stored
  //      its partial (the barrier: no warp returns early and every wait above
  //      is bounded).  One ticket for the CTA: when the unit's other CTAs have
  //      all taken theirs -- the usual case, their pieces came at the start of
  //      their ranges -- this CTA merges without releasing its own partials to
  //      the GPU (its warps see them through the barrier), so no warp waits for
  //      its stores to drain.  Otherwise one fence and one add of W.  The merge
  //      is shared: warp cw takes heads cw*KS .. cw*KS+KS-1.
  named_barrier_sync(1, kWarps * 32);
  if (cw == 0 && lane == 0) {
    const long long ublk0 = (long long)unit * bpu;
    const int c_first = split.cta_of(ublk0);
    const int c_last = split.cta_of(ublk0 + bpu - 1);
    const int others = kWarps * (c_last - c_first);
    bool last = ld_acquire_gpu(&p.tickets[unit]) == others;
    const bool released = !last;
    if (!last) {
      __threadfence();
      last = atomicAdd(&p.tickets[unit], kWarps) == others;
    }
    if (last) p.tickets[unit] = 0;  // ready for the next call
    pending[1] = c_first;
    pending[2] = c_last;
    pending[3] = released;
    pending[0] = last ? unit : -1;
  }
  named_barrier_sync(1, kWarps * 32);
  const int pu = pending[0];
  if (pu >= 0) {
    constexpr int KS = (kHeads + kWarps - 1) / kWarps;
    const int hc = pu % p.head_chunks;
    const int kvh = (pu / p.head_chunks) % p.kv_heads;
    const int bk = pu / (p.kv_heads * p.head_chunks);
    const int nheads = min(kHeads, p.groups - hc * kHeads);
    const int head0 = kvh * p.groups + hc * kHeads;
    // the acquiring fence only after the CTA's own add; after the acquire load
    // above the barrier orders every warp's loads
    const bool acq = pending[3] != 0;
    if (nheads == 1) {
      if (cw == 0) merge_unit<T, 1, kWarps>(p, pu, pending[1], pending[2], bk, head0, nheads, lane, 0, acq);
    } else if (cw * KS < nheads) {
      merge_unit<T, KS, kWarps>(p, pu, pending[1], pending[2], bk, head0, nheads, lane, cw * KS, acq);
    }
  }
}

template <typename T, int NT, int DK, int MODE>
cudaError_t launch_tc(const DecodeTensorMaps &maps, const DecodeParams &p, const DecodeFp8 &f8,
                      const DecodeSpark &sp, int grid, cudaStream_t stream) {
  using C = Cfg<NT, DK, MODE>;
  const int smem = C::kBytes + 1024;
  auto kern = rotatek_decode_tc_kernel<T, NT, DK, MODE>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  kern<<<grid, C::kThreads, smem, stream>>>(maps.kf, maps.vf, maps.ks, maps.vs, maps.ki, p, f8, sp);
  return cudaGetLastError();
}

template <typename T, int MODE>
cudaError_t dispatch_nt_dk(const DecodeTensorMaps &maps, const DecodeParams &p, const DecodeFp8 &f8,
                           const DecodeSpark &sp, int nt, int dk, int grid, cudaStream_t stream) {
  if (nt == 1) {
    if (dk == 16) return launch_tc<T, 1, 16, MODE>(maps, p, f8, sp, grid, stream);
    if (dk == 32) return launch_tc<T, 1, 32, MODE>(maps, p, f8, sp, grid, stream);
    if (dk == 64) return launch_tc<T, 1, 64, MODE>(maps, p, f8, sp, grid, stream);
  } else {
    if (dk == 16) return launch_tc<T, 2, 16, MODE>(maps, p, f8, sp, grid, stream);
    if (dk == 32) return launch_tc<T, 2, 32, MODE>(maps, p, f8, sp, grid, stream);
    if (dk == 64) return launch_tc<T, 2, 64, MODE>(maps, p, f8, sp, grid, stream);
  }
  return cudaErrorInvalidValue;
}

template <int MODE>
cudaError_t dispatch(int dtype_is_bf16, const DecodeTensorMaps &maps, const DecodeParams &p,
                     const DecodeFp8 &f8, const DecodeSpark &sp, int heads_tile, int dk, int grid,
                     cudaStream_t stream) {
  const int nt = heads_tile / 8;
  if (dtype_is_bf16) return dispatch_nt_dk<__nv_bfloat16, MODE>(maps, p, f8, sp, nt, dk, grid, stream);
  return dispatch_nt_dk<__half, MODE>(maps, p, f8, sp, nt, dk, grid, stream);
}

}  // namespace

cudaError_t launch_decode_tc(int dtype_is_bf16, const DecodeTensorMaps &maps, const DecodeParams &p,
                             int heads_tile, int dk, int grid, cudaStream_t stream) {
  DecodeFp8 f8;
  DecodeSpark sp;
  std::memset(&f8, 0, sizeof(f8));
  std::memset(&sp, 0, sizeof(sp));
  return dispatch<kModeRotK>(dtype_is_bf16, maps, p, f8, sp, heads_tile, dk, grid, stream);
}

cudaError_t launch_decode_tc_fp8(int dtype_is_bf16, const DecodeTensorMaps &maps, const DecodeParams &p,
                                 const DecodeFp8 &f, int heads_tile, int dk, int grid, cudaStream_t stream) {
  DecodeSpark sp;
  std::memset(&sp, 0, sizeof(sp));
  return dispatch<kModeFp8>(dtype_is_bf16, maps, p, f, sp, heads_tile, dk, grid, stream);
}

cudaError_t launch_decode_tc_spark(int dtype_is_bf16, const DecodeTensorMaps &maps, const DecodeParams &p,
                                   const DecodeSpark &sp, int heads_tile, int dk, int grid, cudaStream_t stream) {
  DecodeFp8 f8;
  std::memset(&f8, 0, sizeof(f8));
  return dispatch<kModeSpark>(dtype_is_bf16, maps, p, f8, sp, heads_tile, dk, grid, stream);
}

}  // namespace rtk
