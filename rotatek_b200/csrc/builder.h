// Parameters of the prefill rotation-builder kernels (covariance, eigensolver
// + top-k + delta_mu, rotation of the visual Keys).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace rtk {

constexpr int kBuildDim = 128;  // head_dim the builder kernels are written for

// Covariance pass: per matrix m = (b, h), S_m = sum_s k k^T (fp32) and the
// channel sums sum_s k (fp32), written to `cov` [nmat][128][128] / `ksum` [nmat][128].
struct CovParams {
  int dtype;                    // rtk_dtype of the Keys
  int batch, heads, seq;        // matrices = batch * heads
  const void *keys; long long k_s[4];   // [B, H, S, 128] element strides (generic kernel)
  float *cov;                   // [nmat][128][128]
  float *ksum;                  // [nmat][128]
  int splits;                   // token splits per matrix (cluster size on the tensor-core path)
};

cudaError_t launch_cov_tc(int dtype_is_bf16, const CUtensorMap &keys_map, const CovParams &p,
                          cudaStream_t stream);
cudaError_t launch_cov_simt(const CovParams &p, cudaStream_t stream);

// Key projection (the prefill K path of the attention adapters): for every
// (b, h) and every token s,
//   K[b, h, s, :] = RoPE(X[b, s, :] W[h*128 : h*128 + 128, :]^T + bias)
// in the Keys' dtype, rounded like torch's bf16 / fp16 ops (projection output,
// k * cos, rotate_half(k) * sin, their sum).  The visual span's sums of
// CovParams are taken afterwards from the K values written (L2-warm).
struct KProjParams {
  int batch, heads, seq, hidden;  // hidden % 64 == 0
  int vis_start, vis_len;
  const void *bias;                       // [heads * 128] or NULL
  long long cs_sb;                        // cos / sin batch stride (0 = one table for every b)
  unsigned int *status;                   // device status word (bounded-wait timeouts)
  int grid;                               // CTAs: groups * ceil(H / 2) clusters of 2
};

inline long long kproj_pairs(long long heads) { return (heads + 1) / 2; }

// x: [B, S, hidden] 3-D map, box {64, 128, 1}; w: [H*128, hidden] 2-D map, box
// {64, 128}; k_out[i]: the output [B, H, len_i, 128] of span i (prompt, visual,
// text) as 4-D maps with box {64, 128, 1, 1}; cs[0] / cs[1]: cos / sin
// [B | 1, S, 128] as 3-D maps with box {64, 128, 1}; all 128B-swizzled.
struct KProjMaps {
  CUtensorMap x, w, k_out[3], cs[2];
};

// Two-CTA clusters of the projection kernel that fit the current device at once (0 if unknown).
int kproj_max_clusters(int dtype_is_bf16);

// The projection kernel (grid = p.grid).
cudaError_t launch_kproj_tc(int dtype_is_bf16, const KProjMaps &maps, const KProjParams &p,
                            cudaStream_t stream);

// Eigensolver: per matrix, the covariance (centred if ksum is given), optionally
// weighted by the query norms, reduced to tridiagonal form by Householder
// reflections; the top `keep` eigenvectors (descending eigenvalue) go out as R,
// plus delta_mu.  No global scratch.
struct EighParams {
  int nmat, heads;              // matrices m0 .. m0 + nmat - 1 of this launch; m = b * heads + h
  int m0;
  const float *cov;             // [nmat][128][128]
  const float *ksum;            // [nmat][128] or NULL: `cov` is already the matrix to solve
  int count;                    // tokens behind cov / ksum
  int center_dtype;             // dtype the reference rounds the mean to before centring
  // query weighting (kv_pruning_utils.py:117-140); q == NULL disables it
  const void *q; int q_dtype; long long q_s[4];  // [B, H_q, W, 128]
  int window, groups;
  // outputs
  int keep;                                       // 1..128
  void *R; int R_dtype; long long R_s[4];        // [B, H, 128, keep]
  void *dm; long long dm_s[3];                    // [B, H, 128] (R's dtype), nullable
  float *evals;                                   // [nmat][128] descending, nullable
};

cudaError_t launch_eigh(const EighParams &p, cudaStream_t stream);

// Rotation: kept = K_vis . R (uncentred), stored in the Keys' dtype.
struct RotateParams {
  int dtype;
  int batch, heads, seq, keep;
  const void *keys; long long k_s[4];             // [B, H, S, 128]
  const void *R; long long R_s[4];                // [B, H, 128, keep]
  void *out; long long o_s[4];                    // [B, H, S, keep]
  unsigned int *status;                           // device status word (bounded-wait timeouts)
  int max_ctas;                                   // TMA kernel: CTAs at most (0: one per SM)
};

// keep in {16, 32, 48, 64}; keys_map: [B, H, S, 128] bf16/f16, box 64 x 64, 128B swizzle
cudaError_t launch_rotate_tma(int dtype_is_bf16, const CUtensorMap &keys_map, const RotateParams &p,
                              cudaStream_t stream);
// keep in {16, 32, 48, 64, 96, 128}
cudaError_t launch_rotate_tc(int dtype_is_bf16, const RotateParams &p, cudaStream_t stream);
cudaError_t launch_rotate_simt(const RotateParams &p, cudaStream_t stream);

}  // namespace rtk
