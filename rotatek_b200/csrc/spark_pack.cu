// SparK keep mask -> kept channel indices (once per layer, after prefill).
//
// The SparK baseline stores, per visual token, a bool mask over the 128 Key
// channels (keep_mask [B, H, S, D], rotatek/baselines/spark.py:15-58) and the
// kept values in channel order.  The decode rebuilds dense Keys from the kept
// values; it wants the channel of each kept value, so this kernel turns each
// token's mask into its ascending kept-channel list [keep] (uint8): what the
// reference's boolean-index assignment (llama_visionzip.py:230) walks.
//
// One warp per token: lane l looks at channels 4l .. 4l+3; an exclusive scan of
// the per-lane counts gives each kept channel its slot.  A token whose kept
// count is not `keep` sets RTK_DEVICE_BAD_INPUT in *status (its slots past the
// count keep whatever the buffer held).
#include "common.cuh"
#include "decode.h"
#include "rotatek_b200.h"

namespace rtk {
namespace {

constexpr int kWarpsPerBlock = 8;

__global__ void __launch_bounds__(kWarpsPerBlock * 32)
    spark_pack_kernel(const SparkPackParams p) {
  const long long token = (long long)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5);
  const long long tokens = (long long)p.batch * p.heads * p.seq;
  if (token >= tokens) return;
  const int lane = threadIdx.x & 31;
  const int s = static_cast<int>(token % p.seq);
  const long long bh = token / p.seq;
  const int h = static_cast<int>(bh % p.heads);
  const int b = static_cast<int>(bh / p.heads);
  const uint8_t *row = p.mask + (long long)b * p.m_s[0] + (long long)h * p.m_s[1] + (long long)s * p.m_s[2];
  bool kept[4];
  int cnt = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    kept[k] = row[lane * 4 + k] != 0;
    cnt += kept[k];
  }
  int incl = cnt;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += v;
  }
  const int total = __shfl_sync(0xffffffffu, incl, 31);
  if (total != p.keep) {
    if (lane == 0 && p.status != nullptr) atomicOr(p.status, RTK_DEVICE_BAD_INPUT);
  }
  uint8_t *out = p.idx + token * p.keep;
  int slot = incl - cnt;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (kept[k]) {
      if (slot < p.keep) out[slot] = static_cast<uint8_t>(lane * 4 + k);
      ++slot;
    }
  }
}

}  // namespace

cudaError_t launch_spark_pack(const SparkPackParams &p, cudaStream_t stream) {
  const long long tokens = (long long)p.batch * p.heads * p.seq;
  if (tokens == 0) return cudaSuccess;
  const long long blocks = (tokens + kWarpsPerBlock - 1) / kWarpsPerBlock;
  spark_pack_kernel<<<static_cast<unsigned int>(blocks), kWarpsPerBlock * 32, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace rtk
