// Parameters shared by the decode kernels and their host-side launchers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rtk {

// Tensor-core path (decode_tc.cu).  All strides in elements; the head_dim
// stride of every tensor is 1 and the D_keep stride of R is 1.
struct DecodeParams {
  int batch, q_heads, kv_heads, groups;   // groups = H_q / H_kv
  int head_dim_keep;
  int seq_full, seq_sparse;
  int head_chunks;                        // ceil(groups / heads_tile)
  int blocks_full, blocks_sparse, blocks_per_unit;
  long long total_blocks;                 // units * blocks_per_unit
  int phantom;                            // blocks each unit counts extra when the
                                          // units are split among CTAs (0 = even split)
  float scale_log2;                       // log2(e) / sqrt(head_dim)
  const void *q;  long long q_sb, q_sh;
  const void *R;  long long R_sb, R_sh, R_sd;
  const void *dm; long long dm_sb, dm_sh;                // nullable
  const uint8_t *mask; long long mask_sb, mask_ss;       // nullable
  void *out; long long o_sb, o_sh;
  float *partials; int slot_floats;       // (units + grid) slots
  int *tickets;                           // one per unit, zero between calls
  unsigned int *status;                   // RTK_DEVICE_TIMEOUT bits
};

struct DecodeTensorMaps {
  CUtensorMap kf, vf, ks, vs;             // [D|Dk, S, H_kv, B] views, 64-token boxes
  CUtensorMap ki;                         // SparK: kept channel indices [Dk, S, H_kv, B] (uint8)
};

// heads_tile: 8 or 16 query heads per unit; dk: 16, 32 or 64.
cudaError_t launch_decode_tc(int dtype_is_bf16, const DecodeTensorMaps &maps,
                             const DecodeParams &p, int heads_tile, int dk, int grid,
                             cudaStream_t stream);

// fp8 visual span (decode_tc.cu with the fp8 flag): K~8 [B, H_kv, S_v, D_keep]
// and the Values transposed, V8t [B, H_kv, 128, S_v] (token stride 1), e4m3,
// dequantised as k_scale[b, h, c] * K~8[.., t, c] and v_scale[b, h, t] *
// V8t[.., d, t] (quant_fp8.cu).
struct DecodeFp8 {
  const float *k_scale; long long ksc_sb, ksc_sh;               // [B, H_kv, D_keep]
  const float *v_scale; long long vsc_sb, vsc_sh, vsc_ss;       // [B, H_kv, S_v]
};

// heads_tile 8 or 16, dk 16 / 32 / 64; maps.ks / maps.vs are uint8 maps (maps.vs
// over V8t: 64-token x 128-channel boxes, 64-byte swizzle).
cudaError_t launch_decode_tc_fp8(int dtype_is_bf16, const DecodeTensorMaps &maps,
                                 const DecodeParams &p, const DecodeFp8 &f, int heads_tile, int dk,
                                 int grid, cudaStream_t stream);

// SparK visual span (decode_tc.cu with the SparK flag): per token the kept
// channels' values [B, H_kv, S_v, D_keep] (maps.ks, 32-token boxes), their
// channel indices [B, H_kv, S_v, D_keep] uint8 ascending (maps.ki) and the
// pruned channels' mean [B, H_kv, S_v] (16-bit, below); Values in maps.vs with
// 32-token boxes.  The dense Keys are the adapters' recovery of those.
struct DecodeSpark {
  const void *mean; long long mean_sb, mean_sh, mean_ss;
};

cudaError_t launch_decode_tc_spark(int dtype_is_bf16, const DecodeTensorMaps &maps, const DecodeParams &p,
                                   const DecodeSpark &sp, int heads_tile, int dk, int grid,
                                   cudaStream_t stream);

// Kept-channel indices of a SparK keep mask (spark_pack.cu): keep [B, H, S, 128]
// bytes (nonzero = kept) -> idx [B, H, S, keep] uint8, ascending.  A token with
// a kept count other than `keep` sets bit RTK_DEVICE_BAD_INPUT of *status.
struct SparkPackParams {
  int batch, heads, seq, keep;
  const uint8_t *mask; long long m_s[3];     // channel stride 1
  uint8_t *idx;                              // contiguous
  unsigned int *status;
};

cudaError_t launch_spark_pack(const SparkPackParams &p, cudaStream_t stream);

// Quantisation of a visual span to the layout above (quant_fp8.cu).
struct QuantParams {
  int batch, heads, seq, keep;
  const void *keys; long long k_s[4];        // [B, H, S, keep], 16-bit, channel stride 1
  const void *values; long long v_s[4];      // [B, H, S, 128], 16-bit, channel stride 1
  uint8_t *keys8;                            // [B, H, S, keep] contiguous
  float *k_scale;                            // [B, H, keep]
  uint8_t *values8t;                         // [B, H, 128, S] token stride 1; rows of
  long long v8_s[3];                         //   >= S rounded up to 16 bytes, strides in
                                             //   bytes, multiples of 16
  float *v_scale;                            // [B, H, S]
};

cudaError_t launch_quantize_fp8(int dtype_is_bf16, const QuantParams &p, cudaStream_t stream);

// Generic path (decode_simt.cu): any dtype, any strides, head_dim <= 256.
struct SimtParams {
  int dtype;                              // rtk_dtype of q / K / V / out
  int batch, q_heads, kv_heads, groups, head_dim, head_dim_keep;
  int seq_full, seq_sparse, splits, tokens_per_split;
  float scale_log2;
  const void *q;  long long q_s[3];
  const void *R;  long long R_s[4];
  const void *dm; long long dm_s[3];      // nullable
  const uint8_t *mask; long long mask_s[2];  // nullable
  const void *kf; long long kf_s[4];
  const void *vf; long long vf_s[4];
  const void *ks; long long ks_s[4];
  const void *vs; long long vs_s[4];
  void *out; long long o_s[3];
  float *partials; int slot_floats;       // (B * H_q * splits) slots
  int *tickets;                           // one per (b, query head)
  unsigned int *status;
};

cudaError_t launch_decode_simt(const SimtParams &p, cudaStream_t stream);

// Leading bytes of a decode workspace that must be zero before a call (the
// status word and the ticket counters); the rest is scratch the kernels overwrite.
size_t decode_counter_bytes(int64_t batch, int64_t q_heads);

// Set the calling thread's rtk_last_error() message; returns `code`.
int report_error(int code, const char *msg);

}  // namespace rtk
