// Generic decode kernel (CUDA cores, fp32 arithmetic) for what the tensor-core
// path does not cover: fp32 tensors (reference config 1), head_dim other than
// 128, D_keep outside {16, 32, 64}, strides TMA cannot describe, G > 16 heads
// per KV head.  Same arithmetic as rotatek/kernels/fused_decode.py:131-296:
//   q~ = q . R (fp32), bias = q . delta_mu, visual logit = (q~ . k~ + bias) * s,
//   prompt/text logit = q . k * s masked to -inf where mask == 0, running max
//   floored at -1e30, out = acc / (l + 1e-6).
//
// Grid (splits, B * H_q): CTA (s, b*H_q + h) owns one query head and the s-th
// slice of the token sequence [prompt/text tokens | visual tokens].  Its four
// warps take every fourth token; a warp computes one logit per step with a
// shuffle reduction over head_dim and keeps an fp32 online-softmax state.  The
// CTA merges its warps in shared memory and, when the sequence is split,
// writes a partial; the last CTA of a query head (ticket counter) merges the
// partials and stores the output.
#include "common.cuh"
#include "decode.h"

namespace rtk {
namespace {

constexpr int kWarps = 4;
constexpr int kMaxD = 256;
constexpr float kNegBig = -1e30f;

template <typename T>
__device__ __forceinline__ float ld(const void *base, long long off) {
  return to_f32(reinterpret_cast<const T *>(base)[off]);
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) rotatek_decode_simt_kernel(const SimtParams p) {
  __shared__ float q_s[kMaxD];
  __shared__ float qrot_s[kMaxD];
  __shared__ float red_s[kWarps];
  __shared__ float m_s[kWarps], l_s[kWarps];
  __shared__ float acc_s[kWarps][kMaxD];
  __shared__ int last_s;

  const int split = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / p.q_heads, h = bh % p.q_heads;
  const int kvh = h / p.groups;
  const int D = p.head_dim, DK = p.head_dim_keep;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  for (int d = threadIdx.x; d < D; d += blockDim.x)
    q_s[d] = ld<T>(p.q, b * p.q_s[0] + h * p.q_s[1] + d * p.q_s[2]);
  __syncthreads();
  const long long rb = b * p.R_s[0] + kvh * p.R_s[1];
  for (int j = threadIdx.x; j < DK; j += blockDim.x) {
    float a = 0.f;
    for (int d = 0; d < D; ++d) a = fmaf(q_s[d], ld<T>(p.R, rb + d * p.R_s[2] + j * p.R_s[3]), a);
    qrot_s[j] = a;
  }
  {
    float part = 0.f;
    if (p.dm != nullptr) {
      const long long db = b * p.dm_s[0] + kvh * p.dm_s[1];
      for (int d = threadIdx.x; d < D; d += blockDim.x)
        part = fmaf(q_s[d], ld<T>(p.dm, db + d * p.dm_s[2]), part);
    }
    for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
    if (lane == 0) red_s[warp] = part;
  }
  __syncthreads();
  float bias = 0.f;
  for (int w = 0; w < kWarps; ++w) bias += red_s[w];

  float m = kNegBig, l = 0.f;
  float acc[kMaxD / 32];
#pragma unroll
  for (int k = 0; k < kMaxD / 32; ++k) acc[k] = 0.f;

  const int seq = p.seq_full + p.seq_sparse;
  const int t_begin = split * p.tokens_per_split;
  const int t_end = min(seq, t_begin + p.tokens_per_split);
  for (int t = t_begin + warp; t < t_end; t += kWarps) {
    const bool full = t < p.seq_full;
    float dot = 0.f;
    const void *vbase;
    long long voff;
    bool valid = true;
    if (full) {
      const long long kb = b * p.kf_s[0] + kvh * p.kf_s[1] + (long long)t * p.kf_s[2];
      for (int d = lane; d < D; d += 32) dot = fmaf(q_s[d], ld<T>(p.kf, kb + d * p.kf_s[3]), dot);
      if (p.mask != nullptr) valid = p.mask[b * p.mask_s[0] + (long long)t * p.mask_s[1]] != 0;
      vbase = p.vf;
      voff = b * p.vf_s[0] + kvh * p.vf_s[1] + (long long)t * p.vf_s[2];
    } else {
      const int tv = t - p.seq_full;
      const long long kb = b * p.ks_s[0] + kvh * p.ks_s[1] + (long long)tv * p.ks_s[2];
      for (int j = lane; j < DK; j += 32) dot = fmaf(qrot_s[j], ld<T>(p.ks, kb + j * p.ks_s[3]), dot);
      vbase = p.vs;
      voff = b * p.vs_s[0] + kvh * p.vs_s[1] + (long long)tv * p.vs_s[2];
    }
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    if (!full) dot += bias;
    const float s = valid ? dot * p.scale_log2 : -INFINITY;
    const float mn = fmaxf(m, s);
    const float alpha = fast_exp2(m - mn);
    const float pr = fast_exp2(s - mn);
    m = mn;
    l = l * alpha + pr;
    const long long vstride = full ? p.vf_s[3] : p.vs_s[3];
#pragma unroll
    for (int k = 0; k < kMaxD / 32; ++k) {
      const int d = lane + 32 * k;
      if (d < D) acc[k] = acc[k] * alpha + pr * ld<T>(vbase, voff + d * vstride);
    }
  }

  // merge the four warps
  if (lane == 0) {
    m_s[warp] = m;
    l_s[warp] = l;
  }
  __syncthreads();
  float mx = kNegBig;
  for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, m_s[w]);
  const float sc = fast_exp2(m - mx);
#pragma unroll
  for (int k = 0; k < kMaxD / 32; ++k) {
    const int d = lane + 32 * k;
    if (d < D) acc_s[warp][d] = acc[k] * sc;
  }
  __syncthreads();
  float lt = 0.f;
  for (int w = 0; w < kWarps; ++w) lt += l_s[w] * fast_exp2(m_s[w] - mx);

  const long long ob = b * p.o_s[0] + h * p.o_s[1];
  T *out = reinterpret_cast<T *>(p.out);
  if (p.splits == 1) {
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float a = 0.f;
      for (int w = 0; w < kWarps; ++w) a += acc_s[w][d];
      out[ob + d * p.o_s[2]] = from_f32<T>(a / (lt + 1e-6f));
    }
    return;
  }
  float *slot = p.partials + ((long long)bh * p.splits + split) * p.slot_floats;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float a = 0.f;
    for (int w = 0; w < kWarps; ++w) a += acc_s[w][d];
    slot[4 + d] = a;
  }
  if (threadIdx.x == 0) {
    slot[0] = mx;
    slot[1] = lt;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&p.tickets[bh], 1);
    last_s = prev == p.splits - 1;
    if (last_s) p.tickets[bh] = 0;
  }
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  const float *base = p.partials + (long long)bh * p.splits * p.slot_floats;
  float gm = kNegBig;
  for (int s = 0; s < p.splits; ++s) gm = fmaxf(gm, __ldcg(base + (long long)s * p.slot_floats));
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float a = 0.f, lsum = 0.f;
    for (int s = 0; s < p.splits; ++s) {
      const float *sl = base + (long long)s * p.slot_floats;
      const float w = fast_exp2(__ldcg(sl) - gm);
      lsum += __ldcg(sl + 1) * w;
      a += __ldcg(sl + 4 + d) * w;
    }
    out[ob + d * p.o_s[2]] = from_f32<T>(a / (lsum + 1e-6f));
  }
}

}  // namespace

cudaError_t launch_decode_simt(const SimtParams &p, cudaStream_t stream) {
  dim3 grid(p.splits, p.batch * p.q_heads);
  switch (p.dtype) {
    case 0: rotatek_decode_simt_kernel<float><<<grid, kWarps * 32, 0, stream>>>(p); break;
    case 1: rotatek_decode_simt_kernel<__nv_bfloat16><<<grid, kWarps * 32, 0, stream>>>(p); break;
    case 2: rotatek_decode_simt_kernel<__half><<<grid, kWarps * 32, 0, stream>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace rtk
