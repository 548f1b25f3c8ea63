// fp8 (e4m3) storage of the visual span for the decode kernel.
//
// Rotated-truncated Keys K~ [B, H, S_v, D_keep]: one scale per (b, h, channel)
// -- the rotated channels have very different spreads (top eigen-directions
// first), so a per-channel scale keeps the small channels' resolution.  At
// decode the scale folds into the rotated query: q~ . k~ = sum_c (q~_c s_c) k8_c.
// Visual Values [B, H, S_v, 128]: one scale per (b, h, token); at decode it
// folds into that token's softmax weight: sum_t p_t (s_t v8_t).  The e4m3
// Values are stored transposed, V8t [B, H, 128, S_v] (each channel a row of
// token bytes, padded to 16 bytes), the operand layout of the decode's P.V
// product.
//
//   amax  = max |x| over the group (channel over tokens, or token over channels)
//   scale = amax / 448 (e4m3's largest finite value), 1 for an all-zero group
//   x8    = e4m3(x / scale), division and conversion rounded to nearest even,
//           saturating at +-448
#include "common.cuh"
#include "decode.h"

namespace rtk {
namespace {

constexpr float kE4m3Max = 448.f;

// two fp32 -> two e4m3 (lo in the low byte), round to nearest even, saturating
__device__ __forceinline__ uint16_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

template <typename T>
__device__ __forceinline__ void load8(const T *src, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4 *>(src);
  unpack2<T>(v.x, f[0], f[1]);
  unpack2<T>(v.y, f[2], f[3]);
  unpack2<T>(v.z, f[4], f[5]);
  unpack2<T>(v.w, f[6], f[7]);
}

// One CTA per (b, h): per-channel amax over the tokens, then quantize.
// Thread t covers channels 8 (t % (DK / 8)) ... of rows t / (DK / 8) + k * rows_per_pass.
template <typename T, int DK>
__global__ void __launch_bounds__(256) quant_keys_kernel(const QuantParams p) {
  constexpr int kChunks = DK / 8;
  constexpr int kRowsPerPass = 256 / kChunks;
  __shared__ unsigned int amax_bits[DK];
  __shared__ float scale_s[DK];
  const int m = blockIdx.x, b = m / p.heads, h = m % p.heads;
  const int chunk = threadIdx.x % kChunks, r0 = threadIdx.x / kChunks;
  const T *src = static_cast<const T *>(p.keys) + (long long)b * p.k_s[0] + (long long)h * p.k_s[1] + chunk * 8;
  if (threadIdx.x < DK) amax_bits[threadIdx.x] = 0u;
  __syncthreads();
  float mx[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) mx[k] = 0.f;
  for (int s = r0; s < p.seq; s += kRowsPerPass) {
    float f[8];
    load8<T>(src + (long long)s * p.k_s[2], f);
#pragma unroll
    for (int k = 0; k < 8; ++k) mx[k] = fmaxf(mx[k], fabsf(f[k]));
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) atomicMax(&amax_bits[chunk * 8 + k], __float_as_uint(mx[k]));
  __syncthreads();
  if (threadIdx.x < DK) {
    const float a = __uint_as_float(amax_bits[threadIdx.x]);
    const float sc = a > 0.f ? __fdiv_rn(a, kE4m3Max) : 1.f;
    scale_s[threadIdx.x] = sc;
    p.k_scale[(long long)m * DK + threadIdx.x] = sc;
  }
  __syncthreads();
  float sc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) sc[k] = scale_s[chunk * 8 + k];
  uint8_t *dst = p.keys8 + (long long)m * p.seq * DK + chunk * 8;
  for (int s = r0; s < p.seq; s += kRowsPerPass) {
    float f[8];
    load8<T>(src + (long long)s * p.k_s[2], f);
    uint2 o;
    o.x = (uint32_t)e4m3x2(__fdiv_rn(f[0], sc[0]), __fdiv_rn(f[1], sc[1])) |
          ((uint32_t)e4m3x2(__fdiv_rn(f[2], sc[2]), __fdiv_rn(f[3], sc[3])) << 16);
    o.y = (uint32_t)e4m3x2(__fdiv_rn(f[4], sc[4]), __fdiv_rn(f[5], sc[5])) |
          ((uint32_t)e4m3x2(__fdiv_rn(f[6], sc[6]), __fdiv_rn(f[7], sc[7])) << 16);
    *reinterpret_cast<uint2 *>(dst + (long long)s * DK) = o;
  }
}

// One CTA per (b, h, 64-token tile): warp w quantises tokens 8w .. 8w+7 of the
// tile (lane: channels 4 lane .. 4 lane + 3) into a shared [128 channels][64
// tokens] byte tile, then the CTA writes the tile's channel rows in 16-byte
// chunks up to the span's end rounded up to 16 tokens (tokens past it are 0).
constexpr int kVTile = 64;
constexpr int kVTileRow = kVTile + 4;   // shared row bytes: word-aligned, rows spread over the banks

template <typename T>
__global__ void __launch_bounds__(256) quant_values_t_kernel(const QuantParams p) {
  __shared__ __align__(16) uint8_t tile[128 * kVTileRow];
  const int tiles = (p.seq + kVTile - 1) / kVTile;
  const long long bh = blockIdx.x / tiles;
  const int t0 = static_cast<int>(blockIdx.x % tiles) * kVTile;
  const int b = static_cast<int>(bh / p.heads), h = static_cast<int>(bh % p.heads);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T *src = static_cast<const T *>(p.values) + (long long)b * p.v_s[0] + (long long)h * p.v_s[1] + lane * 4;
  uint2 raw[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int s = t0 + warp * 8 + i;
    raw[i] = s < p.seq ? *reinterpret_cast<const uint2 *>(src + (long long)s * p.v_s[2]) : make_uint2(0u, 0u);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int tt = warp * 8 + i, s = t0 + tt;
    float f[4];
    unpack2<T>(raw[i].x, f[0], f[1]);
    unpack2<T>(raw[i].y, f[2], f[3]);
    float mx = fmaxf(fmaxf(fabsf(f[0]), fabsf(f[1])), fmaxf(fabsf(f[2]), fabsf(f[3])));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float sc = mx > 0.f ? __fdiv_rn(mx, kE4m3Max) : 1.f;
    const uint32_t o = s < p.seq ? (uint32_t)e4m3x2(__fdiv_rn(f[0], sc), __fdiv_rn(f[1], sc)) |
                                       ((uint32_t)e4m3x2(__fdiv_rn(f[2], sc), __fdiv_rn(f[3], sc)) << 16)
                                 : 0u;
#pragma unroll
    for (int c = 0; c < 4; ++c) tile[(4 * lane + c) * kVTileRow + tt] = static_cast<uint8_t>(o >> (8 * c));
    if (lane == 0 && s < p.seq) p.v_scale[bh * p.seq + s] = sc;
  }
  __syncthreads();
  const int s16 = (p.seq + 15) / 16 * 16;
  uint8_t *dst = p.values8t + (long long)b * p.v8_s[0] + (long long)h * p.v8_s[1] + t0;
#pragma unroll
  for (int e = threadIdx.x; e < 128 * 4; e += 256) {
    const int row = e >> 2, c = e & 3;
    if (t0 + 16 * c >= s16) continue;
    const uint32_t *w = reinterpret_cast<const uint32_t *>(tile + row * kVTileRow + 16 * c);
    *reinterpret_cast<uint4 *>(dst + (long long)row * p.v8_s[2] + 16 * c) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <typename T>
cudaError_t launch_quant(const QuantParams &p, cudaStream_t stream) {
  const int nmat = p.batch * p.heads;
  if (nmat == 0) return cudaSuccess;
  // (with no tokens the Key scales come out 1 and there is no Value row)
  if (p.keep == 16) quant_keys_kernel<T, 16><<<nmat, 256, 0, stream>>>(p);
  else if (p.keep == 32) quant_keys_kernel<T, 32><<<nmat, 256, 0, stream>>>(p);
  else if (p.keep == 64) quant_keys_kernel<T, 64><<<nmat, 256, 0, stream>>>(p);
  else return cudaErrorInvalidValue;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const long long tiles = (long long)nmat * ((p.seq + kVTile - 1) / kVTile);
  if (tiles > 0) quant_values_t_kernel<T><<<(unsigned)tiles, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_quantize_fp8(int dtype_is_bf16, const QuantParams &p, cudaStream_t stream) {
  return dtype_is_bf16 ? launch_quant<__nv_bfloat16>(p, stream) : launch_quant<__half>(p, stream);
}

}  // namespace rtk
