// Batched 128x128 symmetric eigensolver (cyclic Jacobi in shared memory) with
// the RotateK prologue and epilogue fused around it:
//
//   prologue  C = S_kk - mu^ s^T - s mu^^T + n mu^ mu^^T     (centring,
//             kv_pruning_utils.py:112-115, with the reference's mean rounded to
//             the Keys' dtype), then the query weighting of kv_pruning_utils.py:
//             117-140: per channel q_norm = ||group-mean(q)||_2 over the query
//             window, floored at 1e-3 * lower median; C *= q_norm q_norm^T;
//             C += 1e-4 * max(mean|diag C|, 1e-6) I
//   solve     cyclic Jacobi, parallel ordering: round r = 1..127 pairs every
//             index i with i XOR r (each round is a perfect matching, and the
//             127 rounds meet every pair once); a sweep is 127 rounds; stop when
//             off(A) <= tol * ||diag A|| or after max_sweeps sweeps
//   epilogue  eigenvalues descending; the top `keep` eigenvectors (largest
//             component made positive) rounded to the output dtype are R
//             (kv_pruning_utils.py:142-150 takes eigh's columns in descending
//             order); delta_mu = mu - (mu R) R^T with that rounded R in fp32
//             (kv_pruning_utils.py:153-156).
//
// One CTA of 512 threads per matrix, two CTAs per SM.  A (fp32, row stride
// 129) lives in shared memory and only its upper triangle is kept current:
// element (x, y) is read and written at (min, max), whose bank (x + y) mod 32 is
// the same either way.  Per round: 64 threads compute the rotations (symmetric
// Schur 2x2, Golub & Van Loan 8.4.2), apply them to their own 2x2 diagonal block
// and append them to a per-matrix log in global memory; then every thread
// updates its fixed set of off-diagonal 2x2 blocks (a < b) -- one load and one
// store per element, loads issued before stores.
//
// The eigenvector matrix V = J_1 J_2 ... J_n is never formed.  Once the
// eigenvalues are known, only the `keep` columns that are needed, V e_i for the
// selected i, are computed by applying the logged rounds in reverse to those
// unit vectors (X <- J_t X, t = n..1).  X (128 x keep) stays in registers: each
// warp owns whole columns, lane l holds rows l, l+32, l+64, l+96, so the round-r
// partner row j ^ r is one __shfl_xor away (in register u ^ (r >> 5)); the log is
// streamed through shared memory with cp.async, 16 rounds per stage.
#include "builder.h"
#include "common.cuh"

namespace rtk {
namespace {

constexpr int kN = 128;
constexpr int kPairs = kN / 2;
constexpr int kRounds = kN - 1;        // rounds per sweep
constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kAS = kN + 1;            // A row stride: bank of (x, y) = (x + y) mod 32
constexpr int kXS = kN;                // row stride of X^T (selected eigenvectors, one per row)
constexpr int kOffBlocks = kPairs * (kPairs - 1) / 2;             // 2x2 blocks with a < b
constexpr int kItems = (kOffBlocks + kThreads - 1) / kThreads;    // blocks per thread
constexpr int kChunk = 16;             // logged rounds per shared-memory stage
static_assert(kJacobiLogBytes == sizeof(float2) * kJacobiMaxSweeps * kRounds * kPairs, "log size");

// The matrix, then the staged log, then X^T: each is dead before the next.
// (With keep > 64 the pass for columns 64.. writes X^T rows 64.. before the
// pass for columns 0..63 stages again: staging must stay below row 64.)
struct BackStage {
  float2 raw[2][kChunk][kPairs];       // logged (c, s), double-buffered
  float2 coef[kChunk][kN];             // per-row coefficients of the current chunk
};
union JWork {
  float A[kN * kAS];
  BackStage bt;
  float XT[kN * kXS];
};
static_assert(sizeof(BackStage) <= sizeof(float) * 64 * kXS, "staging must stay below X^T row 64");

struct JSmem {
  JWork w;
  float2 cs[kPairs];                   // (c, s) of this round's rotations
  float vec[kN];                       // fp32 mean
  float vec2[kN];                      // query norms, then eigenvalues, then mu . R[:, c]
  int rank[kN];                        // descending rank of eigenvalue i
  int sel[kN];                         // sel[c]: the eigenvalue of rank c
  float red[2][kWarps];
};

// k with a 0 bit inserted at position h: the smaller index of pair k in a round
// whose highest set bit is h.
__device__ __forceinline__ int insert0(int k, int h) {
  return ((k >> h) << (h + 1)) | (k & ((1 << h) - 1));
}

// Offset of A(x, y), x != y, in upper-triangle storage.
__device__ __forceinline__ int upper(int x, int y) { return x < y ? x * kAS + y : y * kAS + x; }

// Pair index of row/column j in round r (h = msb(r)): j or j ^ r, whichever has
// bit h clear, with bit h removed.  `qside` tells which of the two j is.
__device__ __forceinline__ int pair_of(int j, int r, int h, bool &qside) {
  qside = (j >> h) & 1;
  const int pj = qside ? (j ^ r) : j;
  return ((pj >> (h + 1)) << h) | (pj & ((1 << h) - 1));
}

// Per-thread state of the sweep loop.
struct Sweep {
  int blk[kItems];           // this thread's off-diagonal blocks a | b << 8 (-1: none)
  int pab[kItems];           // their smaller indices pa | pb << 8 for the current h
  int pp;                    // rotation threads: smaller index of pair `tid`
};

// Start of a run of rounds sharing h = msb(r): the smaller pair indices.
__device__ __forceinline__ void segment(Sweep &w, int h, int tid) {
#pragma unroll
  for (int u = 0; u < kItems; ++u)
    w.pab[u] = insert0(w.blk[u] & 0xff, h) | (insert0((w.blk[u] >> 8) & 0xff, h) << 8);
  w.pp = insert0(tid & (kPairs - 1), h);
}

// One round r: rotation threads compute (c, s), log them to `log` [64] and
// finish their diagonal block; then all threads update their off-diagonal blocks.
__device__ __forceinline__ void round_step(float *A, float2 *cs, float2 *log, const Sweep &w, int r,
                                           int tid) {
  if (tid < kPairs) {
    const int pp = w.pp, qq = pp ^ r;
    const float app = A[pp * kAS + pp], aqq = A[qq * kAS + qq], apq = A[pp * kAS + qq];
    float c = 1.f, s = 0.f, t = 0.f;
    if (apq != 0.f && fabsf(apq) > 1e-12f * (fabsf(app) + fabsf(aqq))) {
      // t = sign(theta) / (|theta| + sqrt(theta^2 + 1)), theta = (aqq - app) / (2 apq);
      // |t| <= 1.  c = 1 / sqrt(1 + t^2) from rsqrt plus one Newton step.
      const float theta = __fdividef(aqq - app, 2.f * apq);
      t = copysignf(__fdividef(1.f, fabsf(theta) + sqrtf(fmaf(theta, theta, 1.f))), theta);
      const float x = fmaf(t, t, 1.f);
      const float c0 = rsqrtf(x);
      c = c0 * fmaf(-0.5f * x * c0, c0, 1.5f);
      s = t * c;
    }
    const float2 j = make_float2(c, s);
    cs[tid] = j;
    log[tid] = j;
    A[pp * kAS + pp] = app - t * apq;
    A[qq * kAS + qq] = aqq + t * apq;
    A[pp * kAS + qq] = 0.f;
  }
  __syncthreads();
  // ---- A <- J^T A J on this thread's off-diagonal blocks (pa < pb < qb always),
  // two blocks at a time with their loads issued before their stores
#pragma unroll
  for (int u0 = 0; u0 < kItems; u0 += 2) {
    int off[2][4];
    float x[2][4];
    float2 ja[2], jb[2];
#pragma unroll
    for (int d = 0; d < 2; ++d) {
      const int u = u0 + d;
      if (w.blk[u] < 0) continue;
      const int pa = w.pab[u] & 0xff, pb = w.pab[u] >> 8, qa = pa ^ r, qb = pb ^ r;
      off[d][0] = pa * kAS + pb;
      off[d][1] = pa * kAS + qb;
      off[d][2] = upper(qa, pb);
      off[d][3] = upper(qa, qb);
#pragma unroll
      for (int e = 0; e < 4; ++e) x[d][e] = A[off[d][e]];
      ja[d] = cs[w.blk[u] & 0xff];
      jb[d] = cs[w.blk[u] >> 8];
    }
#pragma unroll
    for (int d = 0; d < 2; ++d) {
      if (w.blk[u0 + d] < 0) continue;
      const float ca = ja[d].x, sa = ja[d].y, cb = jb[d].x, sb = jb[d].y;
      // rows (J_a^T): p' = c p - s q, q' = s p + c q
      const float y00 = ca * x[d][0] - sa * x[d][2], y01 = ca * x[d][1] - sa * x[d][3];
      const float y10 = sa * x[d][0] + ca * x[d][2], y11 = sa * x[d][1] + ca * x[d][3];
      // columns (J_b)
      A[off[d][0]] = y00 * cb - y01 * sb;
      A[off[d][1]] = y00 * sb + y01 * cb;
      A[off[d][2]] = y10 * cb - y11 * sb;
      A[off[d][3]] = y10 * sb + y11 * cb;
    }
  }
  __syncthreads();
}

// One sweep (rounds 1..127 in runs of equal h = msb(r)); round r logs to
// log[(r - 1) * 64 ...].
__device__ __forceinline__ void sweep_rounds(float *A, float2 *cs, float2 *log, Sweep &w, int tid) {
#pragma unroll 1
  for (int h = 0; h < 7; ++h) {
    segment(w, h, tid);
#pragma unroll 1
    for (int r = 1 << h; r < (2 << h); ++r) round_step(A, cs, log + (r - 1) * kPairs, w, r, tid);
  }
}

// X <- J X for one round (RH = r >> 5, rl = r & 31): row j mixes with row j ^ r,
// p-side j' = c j + s (j ^ r), q-side j' = c j - s (j ^ r) (J[p][q] = s).
template <int RH, int CPW>
__device__ __forceinline__ void back_round(float (&x)[4][CPW], const float (&cu)[4], const float (&su)[4],
                                           int rl) {
#pragma unroll
  for (int t = 0; t < CPW; ++t) {
    float part[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) part[u] = __shfl_xor_sync(0xffffffffu, x[u ^ RH][t], rl);
#pragma unroll
    for (int u = 0; u < 4; ++u) x[u][t] = fmaf(su[u], part[u], cu[u] * x[u][t]);
  }
}

// Columns c0 .. c0 + 16 CPW - 1 (those below keep) of X = J_1 ... J_n
// [e_sel[0] ... e_sel[keep-1]] from the n logged rounds, written to X^T (row c =
// selected eigenvector c, unnormalised).  CPW = columns per warp.  The log is
// staged kChunk rounds at a time (cp.async, double-buffered) and expanded once
// per CTA into per-row coefficients (c, +-s), so that the per-warp loop is
// loads, shuffles and FMAs only.
template <int CPW>
__device__ __forceinline__ void back_transform(JSmem &sm, const float2 *log, int nrounds, int c0,
                                               int keep, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  const int cw = c0 + warp * CPW;            // this warp's first column
  const bool active = cw < keep;
  float x[4][CPW];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int t = 0; t < CPW; ++t) {
      const int c = cw + t;
      x[u][t] = (c < keep && sm.sel[c] == lane + 32 * u) ? 1.f : 0.f;
    }
  // chunk ci: rounds [lo, hi), hi = nrounds - ci * kChunk, into raw[ci & 1]
  const int nchunks = (nrounds + kChunk - 1) / kChunk;
  auto issue = [&](int ci) {
    const int hi = nrounds - ci * kChunk, lo = hi > kChunk ? hi - kChunk : 0;
    const char *src = reinterpret_cast<const char *>(log + (long long)lo * kPairs);
    char *dst = reinterpret_cast<char *>(&sm.w.bt.raw[ci & 1][0][0]);
    const int n16 = (hi - lo) * kPairs * static_cast<int>(sizeof(float2)) / 16;
    for (int e = tid; e < n16; e += kThreads) cp_async_16(dst + 16 * e, src + 16 * e);
    cp_async_commit();
  };
  if (nchunks > 0) issue(0);
#pragma unroll 1
  for (int ci = 0; ci < nchunks; ++ci) {
    if (ci + 1 < nchunks) {
      issue(ci + 1);
      cp_async_wait_group<1>();
    } else {
      cp_async_wait_group<0>();
    }
    __syncthreads();
    const int hi = nrounds - ci * kChunk, lo = hi > kChunk ? hi - kChunk : 0;
    // expand: coef[n - lo][j] = (c, s) of row j's pair, s negated on the q side
    // (X <- J X: p' = c p + s q, q' = c q - s p)
    for (int e = tid; e < (hi - lo) * kN; e += kThreads) {
      const int nl = e / kN, j = e % kN;
      const int r = (lo + nl) % kRounds + 1, h = 31 - __clz(r);
      bool qside;
      const float2 cs = sm.w.bt.raw[ci & 1][nl][pair_of(j, r, h, qside)];
      sm.w.bt.coef[nl][j] = make_float2(cs.x, qside ? -cs.y : cs.y);
    }
    __syncthreads();
    if (active) {
#pragma unroll 1
      for (int n = hi - 1; n >= lo; --n) {
        const int r = n % kRounds + 1;
        const float2 *cf = sm.w.bt.coef[n - lo];
        float cu[4], su[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 j = cf[lane + 32 * u];
          cu[u] = j.x;
          su[u] = j.y;
        }
        switch (r >> 5) {
          case 0: back_round<0, CPW>(x, cu, su, r & 31); break;
          case 1: back_round<1, CPW>(x, cu, su, r & 31); break;
          case 2: back_round<2, CPW>(x, cu, su, r & 31); break;
          default: back_round<3, CPW>(x, cu, su, r & 31); break;
        }
      }
    }
  }
  __syncthreads();
  if (active) {
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int t = 0; t < CPW; ++t)
        if (cw + t < keep) sm.w.XT[(cw + t) * kXS + lane + 32 * u] = x[u][t];
  }
  __syncthreads();
}

__device__ __forceinline__ float load_any(const void *p, int dtype, long long i) {
  if (dtype == 1) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
  if (dtype == 2) return __half2float(reinterpret_cast<const __half *>(p)[i]);
  return reinterpret_cast<const float *>(p)[i];
}

__device__ __forceinline__ void store_any(void *p, int dtype, long long i, float v) {
  if (dtype == 1) reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
  else if (dtype == 2) reinterpret_cast<__half *>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<float *>(p)[i] = v;
}

__device__ __forceinline__ float round_to(float v, int dtype) {
  if (dtype == 1) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == 2) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ float block_sum(float v, float *red, int tid) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  __syncthreads();
  if ((tid & 31) == 0) red[tid >> 5] = v;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) tot += red[w];
  return tot;
}

__global__ void __launch_bounds__(kThreads, 2) jacobi_kernel(const JacobiParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  JSmem &sm = *reinterpret_cast<JSmem *>(smem_raw);
  const int tid = threadIdx.x;
  const int m = blockIdx.x;
  const int b = m / p.heads, h = m % p.heads;
  float *A = sm.w.A;

  // ---------------------------------------------------------------- prologue
  const float *C0 = p.cov + (long long)m * kN * kN;
  if (tid < kN) {
    float mu = 0.f;
    if (p.ksum != nullptr) mu = p.ksum[(long long)m * kN + tid] / static_cast<float>(p.count);
    sm.vec[tid] = mu;                                  // fp32 mean
    sm.vec2[tid] = round_to(mu, p.center_dtype);       // the mean the reference centres with
  }
  __syncthreads();
  for (int e = tid; e < kN * kN; e += kThreads) {
    const int i = e / kN, j = e % kN;
    float v = C0[e];
    if (p.ksum != nullptr) {
      const float si = p.ksum[(long long)m * kN + i], sj = p.ksum[(long long)m * kN + j];
      const float mi = sm.vec2[i], mj = sm.vec2[j];
      v = v - mi * sj - si * mj + static_cast<float>(p.count) * mi * mj;
    }
    A[i * kAS + j] = v;
  }
  __syncthreads();
  for (int e = tid; e < kN * kN; e += kThreads) {  // symmetrise: (C + C^T) / 2
    const int i = e / kN, j = e % kN;
    if (i < j) {
      const float v = 0.5f * (A[i * kAS + j] + A[j * kAS + i]);
      A[i * kAS + j] = v;
      A[j * kAS + i] = v;
    }
  }
  __syncthreads();
  if (p.q != nullptr) {
    // q_norm[d] = || mean_g q[b, h*G + g, w, d] ||_2 over the window (mean rounded
    // to the query dtype when G > 1, as torch's bf16 mean does)
    if (tid < kN) {
      float acc = 0.f;
      const float inv_g = 1.f / static_cast<float>(p.groups);
      for (int w = 0; w < p.window; ++w) {
        float v;
        if (p.groups > 1) {
          float sgrp = 0.f;
          for (int g = 0; g < p.groups; ++g)
            sgrp += load_any(p.q, p.q_dtype,
                             b * p.q_s[0] + (long long)(h * p.groups + g) * p.q_s[1] +
                                 (long long)w * p.q_s[2] + tid * p.q_s[3]);
          v = round_to(sgrp * inv_g, p.q_dtype);
        } else {
          v = load_any(p.q, p.q_dtype,
                       b * p.q_s[0] + (long long)h * p.q_s[1] + (long long)w * p.q_s[2] + tid * p.q_s[3]);
        }
        acc = fmaf(v, v, acc);
      }
      sm.vec2[tid] = sqrtf(acc);
    }
    __syncthreads();
    if (tid < kN) {  // lower median: the element of rank 63
      const float x = sm.vec2[tid];
      int r = 0;
      for (int e = 0; e < kN; ++e) {
        const float y = sm.vec2[e];
        r += (y < x) || (y == x && e < tid);
      }
      sm.rank[tid] = r;
      if (r == (kN - 1) / 2) sm.red[1][0] = x;
    }
    __syncthreads();
    const float qfloor = 1e-3f * sm.red[1][0];
    __syncthreads();
    if (tid < kN) sm.vec2[tid] = fmaxf(sm.vec2[tid], qfloor);
    __syncthreads();
    for (int e = tid; e < kN * kN; e += kThreads) {
      const int i = e / kN, j = e % kN;
      A[i * kAS + j] *= sm.vec2[i] * sm.vec2[j];
    }
    __syncthreads();
    float dsum = 0.f;
    if (tid < kN) dsum = fabsf(A[tid * kAS + tid]);
    const float ridge = 1e-4f * fmaxf(block_sum(dsum, sm.red[0], tid) / kN, 1e-6f);
    if (tid < kN) A[tid * kAS + tid] += ridge;
  }
  __syncthreads();

  // ---------------------------------------------------------------- sweeps
  // This thread's off-diagonal blocks: items i = tid + 512 u of the strict upper
  // triangle of the 64 x 64 block grid, folded so rows g and 62 - g share 64
  // items (consecutive lanes take consecutive b).
  Sweep w;
#pragma unroll
  for (int u = 0; u < kItems; ++u) {
    const int i = tid + kThreads * u;
    const int g = i >> 6, o = i & 63;
    const int a = (o < 63 - g) ? g : 62 - g;
    const int bb = (o < 63 - g) ? g + 1 + o : o;
    w.blk[u] = (i < kOffBlocks) ? (a | (bb << 8)) : -1;
  }
  float2 *log = p.rot_log + (long long)m * (kJacobiMaxSweeps * kRounds * kPairs);
  const int max_sweeps = p.max_sweeps < kJacobiMaxSweeps ? p.max_sweeps : kJacobiMaxSweeps;
  int sweep = 0;
  for (; sweep < max_sweeps; ++sweep) {
    float off = 0.f, dia = 0.f;
    for (int e = tid; e < kN * kN; e += kThreads) {
      const int i = e / kN, j = e % kN;
      const float x = A[i * kAS + j];
      if (i == j) dia = fmaf(x, x, dia);
      else if (i < j) off = fmaf(x, x, off);
    }
    off = 2.f * block_sum(off, sm.red[0], tid);
    dia = block_sum(dia, sm.red[1], tid);
    if (off <= p.tol * p.tol * dia) break;
    sweep_rounds(A, sm.cs, log + (long long)sweep * kRounds * kPairs, w, tid);
  }
  if (tid == 0 && p.sweeps != nullptr) p.sweeps[m] = sweep;

  // ---------------------------------------------------------------- epilogue
  // eigenvalues, their descending ranks and the selected indices
  if (tid < kN) sm.vec2[tid] = A[tid * kAS + tid];
  __syncthreads();
  if (tid < kN) {
    const float x = sm.vec2[tid];
    int r = 0;
    for (int e = 0; e < kN; ++e) {
      const float y = sm.vec2[e];
      r += (y > x) || (y == x && e < tid);
    }
    sm.rank[tid] = r;
    sm.sel[r] = tid;
    if (p.evals != nullptr) p.evals[(long long)m * kN + r] = x;
  }
  __syncthreads();
  // the selected eigenvectors (A is dead from here on)
  const int nrounds = sweep * kRounds;
  if (p.keep <= kWarps) {
    back_transform<1>(sm, log, nrounds, 0, p.keep, tid);
  } else if (p.keep <= 2 * kWarps) {
    back_transform<2>(sm, log, nrounds, 0, p.keep, tid);
  } else {
    // at most 64 columns per pass (8 per warp would not fit two CTAs' registers
    // per SM); columns 64.. first, since their X^T rows lie above the staging
    if (p.keep > 4 * kWarps) back_transform<4>(sm, log, nrounds, 4 * kWarps, p.keep, tid);
    back_transform<4>(sm, log, nrounds, 0, p.keep, tid);
  }
  // unit length (rounding drift over ~10^3 rotations), largest component
  // positive, rounded to the output dtype; then mu . R[:, c] with that R
  const int warp = tid >> 5, lane = tid & 31;
  for (int c = warp; c < p.keep; c += kWarps) {
    float *xr = sm.w.XT + c * kXS;
    float vals[4], best = 0.f, nrm = 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float v = xr[lane + 32 * u];
      vals[u] = v;
      nrm = fmaf(v, v, nrm);
      if (fabsf(v) > fabsf(best)) best = v;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float o = __shfl_xor_sync(0xffffffffu, best, off);
      if (fabsf(o) > fabsf(best) || (fabsf(o) == fabsf(best) && o > best)) best = o;
      nrm += __shfl_xor_sync(0xffffffffu, nrm, off);
    }
    const float scale = (best < 0.f ? -1.f : 1.f) / sqrtf(nrm);
    float pr = 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int d = lane + 32 * u;
      const float v = round_to(scale * vals[u], p.R_dtype);
      xr[d] = v;
      store_any(p.R, p.R_dtype,
                b * p.R_s[0] + (long long)h * p.R_s[1] + (long long)d * p.R_s[2] + (long long)c * p.R_s[3], v);
      pr = fmaf(sm.vec[d], v, pr);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) pr += __shfl_xor_sync(0xffffffffu, pr, off);
    if (lane == 0) sm.vec2[c] = pr;
  }
  __syncthreads();
  if (p.dm != nullptr && tid < kN) {
    // delta_mu = mu - sum_c (mu . R[:, c]) R[:, c]
    float acc = 0.f;
    for (int c = 0; c < p.keep; ++c) acc = fmaf(sm.vec2[c], sm.w.XT[c * kXS + tid], acc);
    store_any(p.dm, p.R_dtype, b * p.dm_s[0] + (long long)h * p.dm_s[1] + tid * p.dm_s[2], sm.vec[tid] - acc);
  }
}

}  // namespace

cudaError_t launch_jacobi(const JacobiParams &p, cudaStream_t stream) {
  if (p.rot_log == nullptr) return cudaErrorInvalidValue;
  const int smem = static_cast<int>(sizeof(JSmem));
  cudaError_t err = cudaFuncSetAttribute(jacobi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  jacobi_kernel<<<p.nmat, kThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace rtk
