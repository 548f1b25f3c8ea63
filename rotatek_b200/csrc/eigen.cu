// Batched 128x128 symmetric eigensolver with the RotateK prologue and epilogue
// fused around it, one CTA of 512 threads per matrix:
//
//   prologue  C = S_kk - mu^ s^T - s mu^^T + n mu^ mu^^T     (centring,
//             kv_pruning_utils.py:112-115, with the reference's mean rounded to
//             the Keys' dtype), then the query weighting of kv_pruning_utils.py:
//             117-140: per channel q_norm = ||group-mean(q)||_2 over the query
//             window, floored at 1e-3 * lower median; C *= q_norm q_norm^T;
//             C += 1e-4 * max(mean|diag C|, 1e-6) I.  The matrix is then scaled
//             by 1 / max|C_ij| (eigenvalues are scaled back on output).
//   solve     1. Householder tridiagonalisation Q^T C Q = T (Golub & Van Loan,
//                Matrix Computations, 4th ed., Alg. 8.3.1): step k reflects
//                column k below the diagonal onto e_1 with H_k = I - tau v v^T,
//                then updates the trailing block by the symmetric rank-2 form
//                A <- A - v w^T - w v^T, p = tau A v, w = p - (tau/2)(p.v) v.
//                The matrix lives in registers (thread (c, q) holds rows
//                32q .. 32q+31 of column c); v_k is kept in shared memory.
//             2. the eigenvalues of T that are needed (all 128 when they are
//                returned, else the top `keep`) by multisection on Sturm counts
//                (GVL 8.4.1): P threads per eigenvalue evaluate the count of
//                negative pivots of T - x I at P interior points of its
//                bracket, which shrinks (P + 1)-fold per pass, down to
//                2^-22 * ||T||.
//             3. eigenvectors of T for the top `keep` eigenvalues by inverse
//                iteration (GVL 8.2.2), one thread per vector: two solves of
//                (T - lambda I) y = x from a fixed pseudo-random start, with the
//                pivots D_i = (d_i - lambda) - e_{i-1}^2 / D_{i-1} kept away from
//                zero like the Sturm pivots.
//             4. Gram-Schmidt (twice) of each vector against the earlier ones
//                of its cluster -- consecutive eigenvalues closer than
//                1e-3 * ||T||, the criterion of LAPACK's xSTEIN -- so that
//                (near-)repeated eigenvalues still give orthonormal vectors.
//             5. the reflectors applied back, y = H_0 H_1 ... H_125 x (each warp
//                owns whole columns in registers; one warp-wide dot product per
//                reflector and column).
//   epilogue  eigenvalues descending; the top `keep` eigenvectors (unit length,
//             largest component made positive) rounded to the output dtype are
//             R (kv_pruning_utils.py:142-150 takes eigh's columns in descending
//             order); delta_mu = mu - (mu R) R^T with that rounded R in fp32
//             (kv_pruning_utils.py:153-156).
//
// Shared memory: the matrix as the prologue builds it (fp32, row stride 129:
// element (j, i) sits in bank (j + i) mod 32, so a warp reading a row reads 32
// banks), whose rows then hold the reflectors; the vectors of T (column-major,
// stride 129) and the inverse-iteration pivots.  keep <= 32 needs ~105 KB, two
// CTAs per SM; keep <= 64 and <= 128 one CTA per SM.  No global scratch.
#include "builder.h"
#include "common.cuh"

namespace rtk {
namespace {

constexpr int kN = 128;
constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kAS = kN + 1;            // row stride of the matrix
constexpr int kXS = kN + 1;            // stride between the vectors of X and D

template <int KMAX>
struct ESmem {
  float A[kN * kAS];     // the matrix; during the reduction row k receives v_k
  float X[KMAX * kXS];   // vector c of T (then of the matrix) at X[c * kXS + row]
  float D[KMAX * kXS];   // inverse-iteration pivots of vector c
  float d[kN], e[kN], e2[kN], tau[kN];   // T = tridiag(e, d, e); tau of each reflector
  float lam[kN];         // eigenvalues of T ascending (the wanted ones)
  float pbuf[kN];        // p = tau A v of the current step
  float xbuf[2][kN];     // tail of column k (rows >= k+2), zero elsewhere
  float rowbuf[2][kN];   // row k+1
  float part[4][kN];     // matrix-vector partial sums per row quarter
  float ssbuf[2][4];     // partial sums of squares of the tail, per row quarter
  float vec[kN];         // fp32 mean
  float vec2[kN];        // query norms, then mu . R[:, c]
  int first[kN];         // first vector of vector c's eigenvalue cluster
  float red[2][kWarps];
  float scale;           // max |C_ij| before scaling
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__device__ __forceinline__ float block_sum(float v, float *red, int tid) {
  v = warp_sum(v);
  __syncthreads();
  if ((tid & 31) == 0) red[tid >> 5] = v;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) tot += red[w];
  return tot;
}

__device__ __forceinline__ float block_max(float v, float *red, int tid) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  __syncthreads();
  if ((tid & 31) == 0) red[tid >> 5] = v;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) m = fmaxf(m, red[w]);
  return m;
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

// a[i] for a runtime i < 32 by a tree of selects on the bits of i (5 levels,
// 31 selects).  The bits come through inline asm, which the compiler cannot
// see through: a select by comparing each register's index with i would be
// turned back into dynamic indexing, which moves the array to local memory.
__device__ __forceinline__ float pick32(const float2 (&a)[16], int i) {
  uint32_t bits;
  asm volatile("mov.b32 %0, %1;" : "=r"(bits) : "r"(i));
  float t16[16], t8[8], t4[4], t2[2];
#pragma unroll
  for (int u = 0; u < 16; ++u) t16[u] = (bits & 1u) ? a[u].y : a[u].x;
#pragma unroll
  for (int u = 0; u < 8; ++u) t8[u] = (bits & 2u) ? t16[2 * u + 1] : t16[2 * u];
#pragma unroll
  for (int u = 0; u < 4; ++u) t4[u] = (bits & 4u) ? t8[2 * u + 1] : t8[2 * u];
#pragma unroll
  for (int u = 0; u < 2; ++u) t2[u] = (bits & 8u) ? t4[2 * u + 1] : t4[2 * u];
  return (bits & 16u) ? t2[1] : t2[0];
}

// Negative pivots of T - x I (= eigenvalues of T below x).  A pivot of
// magnitude below `pivmin` is replaced by -pivmin, which keeps every quotient
// finite (|e^2 / q| <= ||T||^2 / pivmin).
__device__ __forceinline__ int sturm_count(const float *d, const float *e2, float x, float pivmin) {
  int cnt = 0;
  float q = 1.f, e2p = 0.f;
#pragma unroll 4
  for (int i = 0; i < kN; i += 4) {
    const float4 dv = *reinterpret_cast<const float4 *>(d + i);
    const float4 ev = *reinterpret_cast<const float4 *>(e2 + i);
    const float dd[4] = {dv.x, dv.y, dv.z, dv.w};
    const float ee[4] = {ev.x, ev.y, ev.z, ev.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      q = (dd[u] - x) - __fdividef(e2p, q);
      if (fabsf(q) < pivmin) q = -pivmin;
      cnt += q < 0.f;
      e2p = ee[u];
    }
  }
  return cnt;
}

// Fixed pseudo-random start of inverse iteration: uniform in [-1, 1) from (vector, row).
__device__ __forceinline__ float start_value(int c, int i) {
  uint32_t h = static_cast<uint32_t>(c) * 0x9E3779B1u + static_cast<uint32_t>(i) * 0x85EBCA77u + 0x165667B1u;
  h ^= h >> 15;
  h *= 0x2C1B3C6Du;
  h ^= h >> 12;
  h *= 0x297A2D39u;
  h ^= h >> 15;
  return static_cast<float>(h >> 8) * (1.f / 8388608.f) - 1.f;
}

// Apply the reflectors to the CPW vectors of this warp (rows lane + 32 u in registers):
// x <- H_0 H_1 ... H_125 x, i.e. H_125 first.
template <int KMAX, int CPW>
__device__ __forceinline__ void back_transform(ESmem<KMAX> &sm, int keep, int warp, int lane) {
  const int c0 = warp * CPW;
  if (c0 >= keep) return;
  float x[CPW][4];
#pragma unroll
  for (int t = 0; t < CPW; ++t)
#pragma unroll
    for (int u = 0; u < 4; ++u) x[t][u] = sm.X[(c0 + t) * kXS + lane + 32 * u];
#pragma unroll 1
  for (int k = kN - 3; k >= 0; --k) {
    const float tk = sm.tau[k];
    if (tk == 0.f) continue;
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int row = lane + 32 * u;
      v[u] = row > k ? sm.A[k * kAS + row] : 0.f;
    }
    float dot[CPW];
#pragma unroll
    for (int t = 0; t < CPW; ++t) dot[t] = v[0] * x[t][0] + v[1] * x[t][1] + v[2] * x[t][2] + v[3] * x[t][3];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int t = 0; t < CPW; ++t) dot[t] += __shfl_xor_sync(0xffffffffu, dot[t], off);
#pragma unroll
    for (int t = 0; t < CPW; ++t) {
      const float s = tk * dot[t];
#pragma unroll
      for (int u = 0; u < 4; ++u) x[t][u] = fmaf(-s, v[u], x[t][u]);
    }
  }
#pragma unroll
  for (int t = 0; t < CPW; ++t)
    if (c0 + t < keep)
#pragma unroll
      for (int u = 0; u < 4; ++u) sm.X[(c0 + t) * kXS + lane + 32 * u] = x[t][u];
}

template <int KMAX>
__global__ void __launch_bounds__(kThreads, KMAX <= 32 ? 2 : 1) eigh_kernel(const EighParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  ESmem<KMAX> &sm = *reinterpret_cast<ESmem<KMAX> *>(smem_raw);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int m = p.m0 + blockIdx.x;
  const int b = m / p.heads, h = m % p.heads;
  float *A = sm.A;
  const int keep = p.keep;

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
  // scale to max |A_ij| = 1 (eigenvectors unchanged; eigenvalues scaled back)
  {
    float mx = 0.f;
    for (int e = tid; e < kN * kN; e += kThreads) mx = fmaxf(mx, fabsf(A[(e / kN) * kAS + e % kN]));
    mx = block_max(mx, sm.red[0], tid);
    const float s = (mx > 0.f && mx < INFINITY) ? mx : 1.f;
    const float inv = 1.f / s;
    for (int e = tid; e < kN * kN; e += kThreads) A[(e / kN) * kAS + e % kN] *= inv;
    if (tid == 0) sm.scale = s;
  }
  __syncthreads();

  // ------------------------------------------- 1. tridiagonalisation Q^T A Q = T
  // Thread (c, q) holds A[32 q + r][c], r < 32, in registers for the whole
  // reduction; shared memory carries what every thread needs each step: the
  // tail of column k (rows >= k+2; zero elsewhere), row k+1, p = tau A v and the
  // partial sums, double-buffered by step parity where one step writes what
  // the next reads.  The Householder vectors go to the matrix's shared-memory
  // rows (row k = v_k), which the registers have freed.
  const int col = tid & (kN - 1), qtr = tid >> 7, r0 = 32 * qtr;
  // rows r0 + 2u, r0 + 2u + 1 in a2[u]: register pairs for the packed fp32
  // FMAs (fma.rn.f32x2, one rounding per lane as fmaf) of the two hot loops
  float2 a2[16];
#define AR(r) (((r) & 1) ? a2[(r) >> 1].y : a2[(r) >> 1].x)
#pragma unroll
  for (int u = 0; u < 16; ++u) a2[u] = make_float2(A[(r0 + 2 * u) * kAS + col], A[(r0 + 2 * u + 1) * kAS + col]);
  __syncthreads();
  // column 0 and row 1 for step 0
  if (col == 0) {
    float ss = 0.f;
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      const int j = r0 + r;
      const float t = j >= 2 ? AR(r) : 0.f;
      sm.xbuf[0][j] = t;
      ss = fmaf(t, t, ss);
    }
    sm.ssbuf[0][qtr] = ss;
  }
  if (qtr == 0) sm.rowbuf[0][col] = a2[0].y;
  __syncthreads();
#pragma unroll 1
  for (int k = 0; k < kN - 2; ++k) {
    const int cur = k & 1, nxt = cur ^ 1;
    // the reflector of column k: x = A[k+1:, k], H x = alpha e_1, needed when
    // the tail of x (its sum of squares ss) is not zero
    const float ss = sm.ssbuf[cur][0] + sm.ssbuf[cur][1] + sm.ssbuf[cur][2] + sm.ssbuf[cur][3];
    const int k1 = k + 1;
    const bool live_rows = r0 + 31 >= k1;          // this quarter holds rows of the trailing block
    if (ss > 0.f) {                                 // uniform across the CTA
      // only warps 0-3, which form p below, need the reflector's scalars
      float tk = 0.f, v0 = 0.f;
      if (warp < 4) {
        const float x0 = sm.rowbuf[cur][k];         // A[k+1][k]
        const float nrm = sqrtf(fmaf(x0, x0, ss));
        const float alpha = x0 >= 0.f ? -nrm : nrm;
        v0 = x0 - alpha;
        tk = 2.f / fmaf(v0, v0, ss);
        if (tid == 0) {
          sm.e[k] = alpha;
          sm.tau[k] = tk;
        }
        // v_k -> row k of the shared matrix (for the back-transform)
        A[k * kAS + tid] = tid == k1 ? v0 : sm.xbuf[cur][tid];
      }
      // p = tau A22 v: this thread's rows; row k+1 (v = v0) is added from rowbuf below
      float acc = 0.f;
      if (live_rows && col > k) {
        // four partial sums (rows = 0, 1, 2, 3 mod 4), combined as (0 + 1) + (2 + 3)
        float2 s01 = make_float2(0.f, 0.f), s23 = make_float2(0.f, 0.f);
#pragma unroll
        for (int r = 0; r < 32; r += 4) {
          const float4 xv = *reinterpret_cast<const float4 *>(&sm.xbuf[cur][r0 + r]);
          s01 = __ffma2_rn(a2[r >> 1], make_float2(xv.x, xv.y), s01);
          s23 = __ffma2_rn(a2[(r >> 1) + 1], make_float2(xv.z, xv.w), s23);
        }
        acc = (s01.x + s01.y) + (s23.x + s23.y);
      }
      sm.part[qtr][col] = acc;
      __syncthreads();
      float pv = 0.f;
      if (tid < kN) {
        float pi = 0.f;
        if (tid > k)
          pi = tk * (sm.part[0][tid] + sm.part[1][tid] + sm.part[2][tid] + sm.part[3][tid] +
                     sm.rowbuf[cur][tid] * v0);
        sm.pbuf[tid] = pi;
        const float vi = tid == k1 ? v0 : sm.xbuf[cur][tid];
        pv = pi * vi;
        // from here on the tail buffer holds all of v: row k+1 gets v0
        if (tid == k1) sm.xbuf[cur][k1] = v0;
      }
      if (warp < 4) {
        pv = warp_sum(pv);
        if (lane == 0) sm.red[0][warp] = pv;
      }
      __syncthreads();
      // A22 <- A22 - v w^T - w v^T, w = p - K v, K = (tau / 2) p.v:
      // A_jc -= v_j (p_c - 2 K v_c) + p_j v_c
      if (live_rows && col > k) {
        const float K = 0.5f * sm.tau[k] * (sm.red[0][0] + sm.red[0][1] + sm.red[0][2] + sm.red[0][3]);
        const float vc = sm.xbuf[cur][col];
        const float cc = fmaf(-2.f * K, vc, sm.pbuf[col]);
        const float2 ncc = make_float2(-cc, -cc), nvc = make_float2(-vc, -vc);
#pragma unroll
        for (int r = 0; r < 32; r += 4) {
          const float4 xv = *reinterpret_cast<const float4 *>(&sm.xbuf[cur][r0 + r]);
          const float4 pv4 = *reinterpret_cast<const float4 *>(&sm.pbuf[r0 + r]);
          // a -= x cc + p vc, as fmaf(-x, cc, fmaf(-p, vc, a)) lane by lane
          a2[r >> 1] = __ffma2_rn(make_float2(xv.x, xv.y), ncc,
                                  __ffma2_rn(make_float2(pv4.x, pv4.y), nvc, a2[r >> 1]));
          a2[(r >> 1) + 1] = __ffma2_rn(make_float2(xv.z, xv.w), ncc,
                                        __ffma2_rn(make_float2(pv4.z, pv4.w), nvc, a2[(r >> 1) + 1]));
        }
      }
    } else if (tid == 0) {                          // column k is already reduced
      sm.e[k] = sm.rowbuf[cur][k];
      sm.tau[k] = 0.f;
    }
    // column k+1 and row k+2 for the next step
    const int k2 = k + 2;
    if (col == k1) {
      float ssn = 0.f;
#pragma unroll
      for (int r = 0; r < 32; r += 4) {
        float4 t;
        t.x = r0 + r > k2 ? a2[r >> 1].x : 0.f;
        t.y = r0 + r + 1 > k2 ? a2[r >> 1].y : 0.f;
        t.z = r0 + r + 2 > k2 ? a2[(r >> 1) + 1].x : 0.f;
        t.w = r0 + r + 3 > k2 ? a2[(r >> 1) + 1].y : 0.f;
        *reinterpret_cast<float4 *>(&sm.xbuf[nxt][r0 + r]) = t;
        ssn = fmaf(t.x, t.x, fmaf(t.y, t.y, fmaf(t.z, t.z, fmaf(t.w, t.w, ssn))));
      }
      sm.ssbuf[nxt][qtr] = ssn;
    }
    if (qtr == (k2 >> 5)) sm.rowbuf[nxt][col] = pick32(a2, k2 & 31);
    __syncthreads();
  }
  // the diagonal (column c leaves the trailing block after step c - 1 and is
  // not touched again) and the last off-diagonal element
  if (qtr == (col >> 5)) sm.d[col] = pick32(a2, col & 31);
  if (qtr == 3 && col == kN - 2) sm.e[kN - 2] = a2[15].y;
#undef AR
  if (tid == 0) {
    sm.e[kN - 1] = 0.f;
    sm.tau[kN - 2] = sm.tau[kN - 1] = 0.f;
  }
  __syncthreads();

  // ------------------------------------------- 2. eigenvalues (Sturm multisection)
  float lo = INFINITY, hi = -INFINITY;
  if (tid < kN) {
    const float el = tid > 0 ? fabsf(sm.e[tid - 1]) : 0.f, er = fabsf(sm.e[tid]);
    lo = sm.d[tid] - el - er;
    hi = sm.d[tid] + el + er;
    sm.e2[tid] = sm.e[tid] * sm.e[tid];
  }
  lo = -block_max(-lo, sm.red[0], tid);
  hi = block_max(hi, sm.red[1], tid);
  const float tnorm = fmaxf(fmaxf(fabsf(lo), fabsf(hi)), 1e-30f);
  const float pivmin = tnorm * 0x1p-40f;
  lo -= tnorm * 0x1p-20f;
  hi += tnorm * 0x1p-20f;
  const int nwant = p.evals != nullptr ? kN : keep;
  // P threads per eigenvalue (a power of two, at most a warp)
  int P = 32;
  if (nwant > 16) P = nwant <= 32 ? 16 : nwant <= 64 ? 8 : 4;
  const int g = tid / P, s = tid % P;          // descending rank g, point s of its bracket
  const int j = kN - 1 - g;                    // its ascending index
  float blo = lo, bhi = hi;
  const float tol = tnorm * 0x1p-22f;
#pragma unroll 1
  for (int it = 0; it < 48; ++it) {
    if (!__any_sync(0xffffffffu, g < nwant && bhi - blo > tol)) break;
    const float x = blo + (bhi - blo) * (static_cast<float>(s + 1) / static_cast<float>(P + 1));
    const int cnt = sturm_count(sm.d, sm.e2, x, pivmin);
    float na = cnt <= j ? x : blo, nb = cnt > j ? x : bhi;
    for (int off = 1; off < P; off <<= 1) {
      na = fmaxf(na, __shfl_xor_sync(0xffffffffu, na, off));
      nb = fminf(nb, __shfl_xor_sync(0xffffffffu, nb, off));
    }
    blo = na;
    bhi = nb;
  }
  if (g < nwant && s == 0) sm.lam[j] = 0.5f * (blo + bhi);
  __syncthreads();

  // ------------------------------------------- 3. vectors of T by inverse iteration
  if (tid < keep) {
    const int c = tid;
    const float lambda = sm.lam[kN - 1 - c];
    float *xc = sm.X + c * kXS;
    float *dc = sm.D + c * kXS;
    for (int i = 0; i < kN; ++i) xc[i] = start_value(c, i);
#pragma unroll 1
    for (int iter = 0; iter < 2; ++iter) {
      // forward: pivots of T - lambda I and L^{-1} x
      float q = sm.d[0] - lambda;
      if (fabsf(q) < pivmin) q = -pivmin;
      dc[0] = q;
      float z = xc[0];
      for (int i = 1; i < kN; ++i) {
        const float ep = sm.e[i - 1];
        const float mlt = __fdividef(ep, q);
        q = fmaf(-mlt, ep, sm.d[i] - lambda);
        if (fabsf(q) < pivmin) q = -pivmin;
        dc[i] = q;
        z = fmaf(-mlt, z, xc[i]);
        xc[i] = z;
      }
      // back: y = U^{-1} z, U = D + e (superdiagonal)
      float y = __fdividef(z, q);
      xc[kN - 1] = y;
      float nrm = y * y;
      for (int i = kN - 2; i >= 0; --i) {
        y = __fdividef(fmaf(-sm.e[i], y, xc[i]), dc[i]);
        xc[i] = y;
        nrm = fmaf(y, y, nrm);
      }
      const float inv = (nrm > 0.f && nrm < INFINITY) ? rsqrtf(nrm) : 0.f;
      for (int i = 0; i < kN; ++i) xc[i] *= inv;
    }
  }
  // clusters: consecutive selected eigenvalues closer than 1e-3 ||T||
  if (tid == 0) {
    int f = 0;
    for (int c = 0; c < keep; ++c) {
      if (c > 0 && sm.lam[kN - c] - sm.lam[kN - 1 - c] > 1e-3f * tnorm) f = c;
      sm.first[c] = f;
    }
  }
  __syncthreads();

  // ------------------------------------------- 4. Gram-Schmidt inside clusters
#pragma unroll 1
  for (int c = 1; c < keep; ++c) {
    const int f = sm.first[c];
    if (f == c) continue;                      // uniform
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
      for (int jj = f + warp; jj < c; jj += kWarps) {
        float dot = 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) dot = fmaf(sm.X[jj * kXS + lane + 32 * u], sm.X[c * kXS + lane + 32 * u], dot);
        dot = warp_sum(dot);
        if (lane == 0) sm.pbuf[jj] = dot;
      }
      __syncthreads();
      if (tid < kN) {
        float v = sm.X[c * kXS + tid];
        for (int jj = f; jj < c; ++jj) v = fmaf(-sm.pbuf[jj], sm.X[jj * kXS + tid], v);
        sm.X[c * kXS + tid] = v;
      }
      __syncthreads();
    }
    const float sq = tid < kN ? sm.X[c * kXS + tid] * sm.X[c * kXS + tid] : 0.f;
    const float tot = block_sum(sq, sm.red[0], tid);
    if (tid < kN) sm.X[c * kXS + tid] *= tot > 0.f ? rsqrtf(tot) : 0.f;
    __syncthreads();
  }

  // ------------------------------------------- 5. back to the matrix's basis
  back_transform<KMAX, KMAX / kWarps>(sm, keep, warp, lane);
  __syncthreads();

  // ---------------------------------------------------------------- epilogue
  const float scale = sm.scale;
  if (p.evals != nullptr && tid < kN) p.evals[(long long)m * kN + tid] = sm.lam[kN - 1 - tid] * scale;
  // unit length, largest component positive, rounded to the output dtype; then
  // mu . R[:, c] with that R
  for (int c = warp; c < keep; c += kWarps) {
    float *xr = sm.X + c * kXS;
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
    const float sc = nrm > 0.f ? (best < 0.f ? -1.f : 1.f) / sqrtf(nrm) : 0.f;
    float pr = 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int d = lane + 32 * u;
      const float v = round_to(sc * vals[u], p.R_dtype);
      xr[d] = v;
      store_any(p.R, p.R_dtype,
                b * p.R_s[0] + (long long)h * p.R_s[1] + (long long)d * p.R_s[2] + (long long)c * p.R_s[3], v);
      pr = fmaf(sm.vec[d], v, pr);
    }
    pr = warp_sum(pr);
    if (lane == 0) sm.vec2[c] = pr;
  }
  __syncthreads();
  if (p.dm != nullptr && tid < kN) {
    // delta_mu = mu - sum_c (mu . R[:, c]) R[:, c]
    float acc = 0.f;
    for (int c = 0; c < keep; ++c) acc = fmaf(sm.vec2[c], sm.X[c * kXS + tid], acc);
    store_any(p.dm, p.R_dtype, b * p.dm_s[0] + (long long)h * p.dm_s[1] + tid * p.dm_s[2], sm.vec[tid] - acc);
  }
}

template <int KMAX>
cudaError_t launch(const EighParams &p, cudaStream_t stream) {
  const int smem = static_cast<int>(sizeof(ESmem<KMAX>));
  cudaError_t err = cudaFuncSetAttribute(eigh_kernel<KMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  eigh_kernel<KMAX><<<p.nmat, kThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_eigh(const EighParams &p, cudaStream_t stream) {
  if (p.keep < 1 || p.keep > kN) return cudaErrorInvalidValue;
  if (p.keep <= 32) return launch<32>(p, stream);
  if (p.keep <= 64) return launch<64>(p, stream);
  return launch<128>(p, stream);
}

}  // namespace rtk
