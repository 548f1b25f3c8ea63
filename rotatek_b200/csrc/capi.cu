// extern "C" entry points of librotatek_b200.so (declared in include/rotatek_b200.h).
//
// Host-side work per call: validate shapes and dtypes (messages follow the
// reference's ValueErrors, rotatek/kernels/fused_decode.py:323-338 and
// full_channel_flash_decoding.py:173-178), choose the kernel, encode the TMA
// tensor maps, carve the caller's workspace, launch on the caller's stream.
// Nothing allocates device memory and nothing synchronises the stream.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>

#include "../../include/rotatek_b200.h"
#include "builder.h"
#include "decode.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  return fail(RTK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

constexpr size_t kAlign = 256;
constexpr size_t kStatusBytes = 256;   // device-status word at the head of a workspace
constexpr int kBlockTokens = 64;      // generic-kernel split granularity
constexpr int kVisBlockTokens = 64;   // tensor-core kernel: visual block
constexpr int kFullBlockTokens = 32;  // tensor-core kernel: prompt/text block

size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

int sm_count(int device) {
  static std::mutex mu;
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    cache[device] = n;
  }
  return cache[device];
}

// SMs the tensor-core decode kernels leave free (rtk_decode_set_sm_reserve).
std::atomic<int> g_decode_sm_reserve{0};

// CTAs of a persistent decode launch on `device`: one per SM not reserved.
int decode_ctas(int device) {
  const int n = sm_count(device) - g_decode_sm_reserve.load(std::memory_order_relaxed);
  return n > 1 ? n : 1;
}

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ------------------------------------------------------------------ shapes
struct View4 {  // a tensor seen as [B, H, S, D] with element strides
  const void *data;
  int64_t n[4], s[4];
};

bool as4(const rtk_tensor *t, View4 &v) {
  if (t == nullptr || t->ndim != 4) return false;
  v.data = t->data;
  for (int i = 0; i < 4; ++i) {
    v.n[i] = t->shape[i];
    v.s[i] = t->stride[i];
  }
  return true;
}

// out may be [B, H_q, D] or [B, 1, H_q, D] (the reference returns the latter).
bool out_view(const rtk_tensor *o, int64_t B, int64_t Hq, int64_t D, int64_t s[3]) {
  if (o == nullptr || o->data == nullptr) return false;
  if (o->ndim == 3 && o->shape[0] == B && o->shape[1] == Hq && o->shape[2] == D) {
    s[0] = o->stride[0]; s[1] = o->stride[1]; s[2] = o->stride[2];
    return true;
  }
  if (o->ndim == 4 && o->shape[0] == B && o->shape[1] == 1 && o->shape[2] == Hq && o->shape[3] == D) {
    s[0] = o->stride[0]; s[1] = o->stride[2]; s[2] = o->stride[3];
    return true;
  }
  return false;
}

// ------------------------------------------------------------------ TMA maps
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// [B, H, S, inner] 16-bit tensor -> 4-D map with a {box_inner, box_rows, 1, 1} box.
// Returns false when TMA cannot describe the layout (the caller then uses the
// generic kernel).  Size-1 dimensions get a canonical stride.
bool encode_map(CUtensorMap *map, const View4 &v, CUtensorMapDataType dt, int box_inner,
                int box_rows, CUtensorMapSwizzle sw, int esize = 2) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  if (v.s[3] != 1) return false;
  if (reinterpret_cast<uintptr_t>(v.data) % 16 != 0) return false;
  cuuint64_t dims[4] = {(cuuint64_t)v.n[3], (cuuint64_t)v.n[2], (cuuint64_t)v.n[1],
                        (cuuint64_t)v.n[0]};
  cuuint64_t strides[3];
  int64_t natural = v.n[3] * esize;
  for (int i = 0; i < 3; ++i) {
    const int dim = 2 - i;  // S, H, B
    int64_t sb = v.s[dim] * esize;
    if (v.n[dim] == 1) sb = (natural + 15) / 16 * 16;
    if (sb <= 0 || sb % 16 != 0) return false;
    strides[i] = (cuuint64_t)sb;
    natural = sb * v.n[dim];
  }
  for (int i = 0; i < 4; ++i)
    if (dims[i] == 0 || dims[i] > (1ull << 31)) return false;
  cuuint32_t box[4] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estride[4] = {1, 1, 1, 1};
  return fn(map, dt, 4, const_cast<void *>(v.data), dims, strides, box, estride,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

CUtensorMapSwizzle swizzle_for_row_bytes(int bytes) {
  if (bytes == 32) return CU_TENSOR_MAP_SWIZZLE_32B;
  if (bytes == 64) return CU_TENSOR_MAP_SWIZZLE_64B;
  return CU_TENSOR_MAP_SWIZZLE_128B;
}

// ------------------------------------------------------------------ workspace
// Layout of a decode workspace (every offset a multiple of 256 bytes):
//   [0, 256)                   device-status word
//   [256, counter_end)         one ticket counter per unit; units <= B * H_q for
//                              every kernel, so counter_end depends on B * H_q only
//   [counter_end, bytes)       split partials (scratch, overwritten by each call)
// The counters must read zero before a call and every call leaves them zero,
// so for a fixed B * H_q the workspace needs zeroing once, whatever the
// sequence lengths; a call with a larger B * H_q needs the larger counter
// region zeroed first (rtk_decode_workspace_counter_bytes).
struct WorkspacePlan {
  size_t ticket_off, partial_off, bytes;
};

size_t counter_end(int64_t batch, int64_t q_heads) {
  return kAlign + align_up((size_t)(batch * q_heads) * sizeof(int));
}

WorkspacePlan plan_workspace(int64_t batch, int64_t q_heads, int64_t slots, int64_t slot_floats) {
  WorkspacePlan w;
  w.ticket_off = kAlign;
  w.partial_off = counter_end(batch, q_heads);
  w.bytes = w.partial_off + align_up((size_t)slots * slot_floats * sizeof(float));
  return w;
}

struct TcShape {
  int heads_tile, head_chunks;
  int64_t units, blocks_full, blocks_sparse, blocks_per_unit, total;
  int grid;
  int slot_floats;
  int64_t slots;  // one per (unit + cta, consumer warp); <= 5 consumer warps per CTA
  int phantom;    // blocks each unit counts extra in the split among CTAs
};

// What a CTA's switch from one unit to the next costs, in blocks of streaming
// (measured at config 2: ranges that cross a unit start finished ~5 us, about
// 12 blocks, after those that do not).  Used only where every CTA has at least
// 16 times as many blocks, so that no range is left without real blocks.
constexpr int kUnitSwitchBlocks = 12;

TcShape tc_shape(int64_t B, int64_t Hkv, int64_t G, int64_t Sf, int64_t Sv, int device,
                 int64_t vis_tokens = kVisBlockTokens) {
  TcShape t;
  t.heads_tile = G <= 8 ? 8 : 16;
  t.head_chunks = (int)cdiv(G, t.heads_tile);
  t.units = B * Hkv * t.head_chunks;
  t.blocks_full = cdiv(Sf, kFullBlockTokens);
  t.blocks_sparse = cdiv(Sv, vis_tokens);
  t.blocks_per_unit = t.blocks_full + t.blocks_sparse;
  t.total = t.units * t.blocks_per_unit;
  t.grid = (int)std::max<int64_t>(1, std::min<int64_t>(t.total, decode_ctas(device)));
  t.slot_floats = 32 + 16 * 128;
  t.slots = (t.units + t.grid) * 5;
  t.phantom = t.total / t.grid >= 16 * kUnitSwitchBlocks ? kUnitSwitchBlocks : 0;
  return t;
}

struct SimtShape {
  int splits, tokens_per_split, slot_floats;
  int64_t units;
};

SimtShape simt_shape(int64_t B, int64_t Hq, int64_t D, int64_t seq, int device) {
  SimtShape s;
  s.units = B * Hq;
  const int64_t want = cdiv(4 * (int64_t)sm_count(device), std::max<int64_t>(1, s.units));
  const int64_t max_splits = std::max<int64_t>(1, std::min<int64_t>(256, cdiv(seq, kBlockTokens)));
  s.splits = (int)std::max<int64_t>(1, std::min(want, max_splits));
  s.tokens_per_split = (int)std::max<int64_t>(1, cdiv(seq, s.splits));
  s.slot_floats = (int)(4 + (D + 3) / 4 * 4);
  return s;
}

size_t decode_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t Sf,
                              int64_t Sv, int device) {
  const int64_t G = Hkv > 0 ? Hq / Hkv : 1;
  const TcShape t = tc_shape(B, Hkv, std::max<int64_t>(G, 1), Sf, Sv, device);
  const size_t tc = plan_workspace(B, Hq, t.slots, t.slot_floats).bytes;
  const SimtShape s = simt_shape(B, Hq, D, Sf + Sv, device);
  const size_t simt = plan_workspace(B, Hq, s.units * s.splits, s.slot_floats).bytes;
  return std::max(tc, simt);
}

bool is_half_type(int dt) { return dt == RTK_BF16 || dt == RTK_F16; }

}  // namespace

namespace rtk {
// Bytes at the start of a decode workspace that must read zero before a call:
// the device-status word and one ticket counter per unit (at most B * H_q).
size_t decode_counter_bytes(int64_t batch, int64_t q_heads) { return counter_end(batch, q_heads); }

// Record `msg` as this thread's rtk_last_error() and return `code`.
int report_error(int code, const char *msg) { return fail(code, "%s", msg); }
}  // namespace rtk

namespace {

// ------------------------------------------------------------------ decode core
struct DecodeArgs {
  const rtk_tensor *q, *R, *dm, *kf, *vf, *mask, *ks, *vs, *out;
  int64_t groups;
  bool dense;  // full_channel_decode: no visual span, no mask
  const rtk_tensor *ksc = nullptr, *vsc = nullptr;   // fp8 visual span: ks / vs are e4m3 (uint8)
  // SparK visual span: ks = kept values [B, H_kv, S_v, D_keep], kidx = their
  // channels (uint8), kmean = pruned-channel means [B, H_kv, S_v, 1]; R unused
  const rtk_tensor *kidx = nullptr, *kmean = nullptr;
};

int run_decode(const DecodeArgs &a, void *workspace, size_t workspace_bytes, cudaStream_t stream) {
  View4 kf{}, vf{}, ks{}, vs{}, R{}, ki{}, km{};
  as4(a.kf, kf);
  as4(a.vf, vf);
  const int64_t B = a.q->shape[0], Hq = a.q->shape[1], D = a.q->shape[2];
  const int64_t Hkv = kf.n[1];
  const int64_t G = a.groups;
  const int64_t Sf = kf.n[2];
  const bool spark = a.kidx != nullptr;
  int64_t Sv = 0, DK = 0;
  if (!a.dense) {
    as4(a.ks, ks);
    as4(a.vs, vs);
    Sv = ks.n[2];
    if (spark) {
      as4(a.kidx, ki);
      as4(a.kmean, km);
      DK = ks.n[3];
    } else {
      as4(a.R, R);
      DK = R.n[3];
    }
  }
  int64_t os[3] = {0, 0, 0};
  out_view(a.out, B, Hq, D, os);
  const int dt = a.q->dtype;
  const int device = current_device();

  if (workspace == nullptr)
    return fail(RTK_ERR_WORKSPACE, "workspace is NULL (size it with *_workspace_size)");
  const size_t need = decode_workspace_bytes(B, Hq, Hkv, D, Sf, Sv, device);
  if (workspace_bytes < need)
    return fail(RTK_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes, need);
  unsigned char *ws = static_cast<unsigned char *>(workspace);
  unsigned int *status = reinterpret_cast<unsigned int *>(ws);
  const double scale_log2 = 1.4426950408889634 / std::sqrt((double)D);

  const bool fp8 = a.ksc != nullptr;
  // ---------------- tensor-core path
  bool tc = is_half_type(dt) && D == 128 && (Sf + Sv) > 0 && a.q->stride[2] == 1 &&
            os[2] == 1 && (a.dense || ((DK == 16 || DK == 32 || DK == 64) && (spark || R.s[3] == 1) &&
                                       (a.dm == nullptr || a.dm->stride[2] == 1)));
  rtk::DecodeTensorMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  if (tc) {
    const CUtensorMapDataType et =
        dt == RTK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (Sf > 0)
      tc = encode_map(&maps.kf, kf, et, 64, kFullBlockTokens, CU_TENSOR_MAP_SWIZZLE_128B) &&
           encode_map(&maps.vf, vf, et, 64, kFullBlockTokens, CU_TENSOR_MAP_SWIZZLE_128B);
    if (tc && Sv > 0 && spark)   // 64-row kept values / index boxes (DK-byte index rows); 32-token Value boxes
      tc = encode_map(&maps.ks, ks, et, (int)DK, 2 * kFullBlockTokens, swizzle_for_row_bytes((int)DK * 2)) &&
           encode_map(&maps.vs, vs, et, 64, kFullBlockTokens, CU_TENSOR_MAP_SWIZZLE_128B) &&
           encode_map(&maps.ki, ki, CU_TENSOR_MAP_DATA_TYPE_UINT8, (int)DK, 2 * kFullBlockTokens,
                      DK == 16 ? CU_TENSOR_MAP_SWIZZLE_NONE : swizzle_for_row_bytes((int)DK), 1);
    if (tc && Sv > 0 && !fp8 && !spark)
      tc = encode_map(&maps.ks, ks, et, (int)DK, kVisBlockTokens, swizzle_for_row_bytes((int)DK * 2)) &&
           encode_map(&maps.vs, vs, et, 64, kVisBlockTokens, CU_TENSOR_MAP_SWIZZLE_128B);
    if (tc && Sv > 0 && fp8)   // 128 e4m3 Key rows of DK bytes; V^T: 128 channel rows of 64 token bytes
      tc = encode_map(&maps.ks, ks, CU_TENSOR_MAP_DATA_TYPE_UINT8, (int)DK, 2 * kVisBlockTokens,
                      DK == 16 ? CU_TENSOR_MAP_SWIZZLE_NONE : swizzle_for_row_bytes((int)DK), 1) &&
           encode_map(&maps.vs, vs, CU_TENSOR_MAP_DATA_TYPE_UINT8, kVisBlockTokens, 128,
                      CU_TENSOR_MAP_SWIZZLE_64B, 1);
  }
  if (fp8 && !tc)
    return fail(RTK_ERR_UNSUPPORTED, "the fp8 visual span needs bf16 / fp16 queries, head_dim 128, D_keep 16, "
                                     "32 or 64 and 16-byte aligned e4m3 rows (Keys) and channel rows (V^T)");
  if (spark && !tc)
    return fail(RTK_ERR_UNSUPPORTED, "the SparK decode needs bf16 / fp16 tensors, head_dim 128, D_keep 16, 32 "
                                     "or 64, and channel-contiguous, 16-byte aligned rows");
  if (tc) {
    // visual block tokens: 64 for SparK (two halves of 32), 128 for fp8 (two
    // halves of 64), else 64
    const TcShape t = tc_shape(B, Hkv, G, Sf, Sv, device,
                               spark ? 2 * kFullBlockTokens : fp8 ? 2 * kVisBlockTokens : kVisBlockTokens);
    const WorkspacePlan w = plan_workspace(B, Hq, t.slots, t.slot_floats);
    rtk::DecodeParams p;
    std::memset(&p, 0, sizeof(p));
    p.batch = (int)B; p.q_heads = (int)Hq; p.kv_heads = (int)Hkv; p.groups = (int)G;
    p.head_dim_keep = (int)DK;
    p.seq_full = (int)Sf; p.seq_sparse = (int)Sv;
    p.head_chunks = t.head_chunks;
    p.blocks_full = (int)t.blocks_full; p.blocks_sparse = (int)t.blocks_sparse;
    p.blocks_per_unit = (int)t.blocks_per_unit;
    p.total_blocks = t.total;
    p.phantom = t.phantom;
    p.scale_log2 = (float)scale_log2;
    p.q = a.q->data; p.q_sb = a.q->stride[0]; p.q_sh = a.q->stride[1];
    if (!a.dense) {
      if (!spark) { p.R = R.data; p.R_sb = R.s[0]; p.R_sh = R.s[1]; p.R_sd = R.s[2]; }
      if (a.dm != nullptr) { p.dm = a.dm->data; p.dm_sb = a.dm->stride[0]; p.dm_sh = a.dm->stride[1]; }
      if (a.mask != nullptr) { p.mask = static_cast<const uint8_t *>(a.mask->data); p.mask_sb = a.mask->stride[0]; p.mask_ss = a.mask->stride[1]; }
    }
    p.out = a.out->data; p.o_sb = os[0]; p.o_sh = os[1];
    p.partials = reinterpret_cast<float *>(ws + w.partial_off);
    p.slot_floats = t.slot_floats;
    p.tickets = reinterpret_cast<int *>(ws + w.ticket_off);
    p.status = status;
    cudaError_t e;
    if (spark) {
      rtk::DecodeSpark sp;
      sp.mean = km.data; sp.mean_sb = km.s[0]; sp.mean_sh = km.s[1]; sp.mean_ss = km.s[2];
      e = rtk::launch_decode_tc_spark(dt == RTK_BF16, maps, p, sp, t.heads_tile, (int)DK, t.grid, stream);
    } else if (fp8) {
      rtk::DecodeFp8 f;
      f.k_scale = static_cast<const float *>(a.ksc->data);
      f.ksc_sb = a.ksc->stride[0]; f.ksc_sh = a.ksc->stride[1];
      f.v_scale = static_cast<const float *>(a.vsc->data);
      f.vsc_sb = a.vsc->stride[0]; f.vsc_sh = a.vsc->stride[1]; f.vsc_ss = a.vsc->stride[2];
      e = rtk::launch_decode_tc_fp8(dt == RTK_BF16, maps, p, f, t.heads_tile, (int)DK, t.grid, stream);
    } else {
      e = rtk::launch_decode_tc(dt == RTK_BF16, maps, p, t.heads_tile, a.dense ? 32 : (int)DK, t.grid, stream);
    }
    if (e != cudaSuccess) return cuda_fail(e, "rotatek decode (tensor-core kernel) launch");
    return RTK_OK;
  }

  // ---------------- generic path
  if (D > 256) return fail(RTK_ERR_UNSUPPORTED, "head_dim %lld > 256 is not supported", (long long)D);
  const SimtShape s = simt_shape(B, Hq, D, Sf + Sv, device);
  const WorkspacePlan w = plan_workspace(B, Hq, s.units * s.splits, s.slot_floats);
  rtk::SimtParams p;
  std::memset(&p, 0, sizeof(p));
  p.dtype = dt;
  p.batch = (int)B; p.q_heads = (int)Hq; p.kv_heads = (int)Hkv; p.groups = (int)G;
  p.head_dim = (int)D; p.head_dim_keep = (int)DK;
  p.seq_full = (int)Sf; p.seq_sparse = (int)Sv;
  p.splits = s.splits; p.tokens_per_split = s.tokens_per_split;
  p.scale_log2 = (float)scale_log2;
  p.q = a.q->data;
  for (int i = 0; i < 3; ++i) p.q_s[i] = a.q->stride[i];
  p.kf = kf.data; p.vf = vf.data;
  for (int i = 0; i < 4; ++i) { p.kf_s[i] = kf.s[i]; p.vf_s[i] = vf.s[i]; }
  if (!a.dense) {
    p.R = R.data;
    for (int i = 0; i < 4; ++i) { p.R_s[i] = R.s[i]; p.ks_s[i] = ks.s[i]; p.vs_s[i] = vs.s[i]; }
    p.ks = ks.data; p.vs = vs.data;
    if (a.dm != nullptr) { p.dm = a.dm->data; for (int i = 0; i < 3; ++i) p.dm_s[i] = a.dm->stride[i]; }
    if (a.mask != nullptr) { p.mask = static_cast<const uint8_t *>(a.mask->data); p.mask_s[0] = a.mask->stride[0]; p.mask_s[1] = a.mask->stride[1]; }
  }
  p.out = a.out->data;
  for (int i = 0; i < 3; ++i) p.o_s[i] = os[i];
  p.partials = reinterpret_cast<float *>(ws + w.partial_off);
  p.slot_floats = s.slot_floats;
  p.tickets = reinterpret_cast<int *>(ws + w.ticket_off);
  p.status = status;
  const cudaError_t e = rtk::launch_decode_simt(p, stream);
  if (e != cudaSuccess) return cuda_fail(e, "rotatek decode (generic kernel) launch");
  return RTK_OK;
}

bool same_dims(const rtk_tensor *t, int ndim, std::initializer_list<int64_t> want) {
  if (t == nullptr || t->ndim != ndim) return false;
  int i = 0;
  for (int64_t w : want) {
    if (w >= 0 && t->shape[i] != w) return false;
    ++i;
  }
  return true;
}

bool dtype_ok(int dt) { return dt == RTK_F32 || dt == RTK_BF16 || dt == RTK_F16; }

}  // namespace

extern "C" {

int rtk_abi_version(void) { return RTK_ABI_VERSION; }

int rtk_decode_set_sm_reserve(int sms) {
  g_last_error.clear();
  if (sms < 0 || sms > 64) return fail(RTK_ERR_INVALID, "sms must be in [0, 64] (got %d)", sms);
  g_decode_sm_reserve.store(sms, std::memory_order_relaxed);
  return RTK_OK;
}

const char *rtk_last_error(void) { return g_last_error.c_str(); }

size_t rtk_rotatek_decode_workspace_size(int32_t dtype, int64_t batch, int64_t q_heads,
                                         int64_t kv_heads, int64_t head_dim,
                                         int64_t head_dim_keep, int64_t seq_full,
                                         int64_t seq_sparse, int32_t device) {
  (void)dtype;
  (void)head_dim_keep;
  return decode_workspace_bytes(batch, q_heads, kv_heads, head_dim, seq_full, seq_sparse, device);
}

size_t rtk_decode_workspace_counter_bytes(int64_t batch, int64_t q_heads) {
  return counter_end(batch, q_heads);
}

size_t rtk_full_channel_decode_workspace_size(int32_t dtype, int64_t batch, int64_t q_heads,
                                              int64_t kv_heads, int64_t head_dim, int64_t seq,
                                              int32_t device) {
  (void)dtype;
  return decode_workspace_bytes(batch, q_heads, kv_heads, head_dim, seq, 0, device);
}

int rtk_rotatek_decode(const rtk_tensor *q_full, const rtk_tensor *R_partial,
                       const rtk_tensor *delta_mu, const rtk_tensor *k_full,
                       const rtk_tensor *v_full, const rtk_tensor *mask_full,
                       const rtk_tensor *k_sparse, const rtk_tensor *v_sparse,
                       int64_t num_kv_groups, const rtk_tensor *out, void *workspace,
                       size_t workspace_bytes, void *stream) {
  g_last_error.clear();
  if (q_full == nullptr || q_full->ndim != 3) return fail(RTK_ERR_INVALID, "q_full must be [B, H_q, D]");
  if (R_partial == nullptr || R_partial->ndim != 4)
    return fail(RTK_ERR_INVALID, "R_partial must be [B, H_kv, D, D_keep]");
  if (mask_full != nullptr && mask_full->dtype != RTK_U8) return fail(RTK_ERR_INVALID, "mask_full must be uint8");
  const int64_t B = q_full->shape[0], Hq = q_full->shape[1], D = q_full->shape[2];
  const int64_t Hkv = R_partial->shape[1], DK = R_partial->shape[3];
  if (num_kv_groups <= 0 || Hq / num_kv_groups != Hkv)
    return fail(RTK_ERR_INVALID, "R_partial H_kv=%lld but H_q=%lld, num_kv_groups=%lld",
                (long long)Hkv, (long long)Hq, (long long)num_kv_groups);
  if (Hq != Hkv * num_kv_groups)
    return fail(RTK_ERR_INVALID, "H_q=%lld is not H_kv=%lld * num_kv_groups=%lld", (long long)Hq,
                (long long)Hkv, (long long)num_kv_groups);
  if (!dtype_ok(q_full->dtype)) return fail(RTK_ERR_INVALID, "q_full dtype must be float32, bfloat16 or float16");
  if (!same_dims(R_partial, 4, {B, Hkv, D, -1}) || DK < 1 || DK > D)
    return fail(RTK_ERR_INVALID, "R_partial must be [B, H_kv, D, D_keep]");
  if (delta_mu != nullptr && !same_dims(delta_mu, 3, {B, Hkv, D}))
    return fail(RTK_ERR_INVALID, "delta_mu must be [B, H_kv, D]");
  if (!same_dims(k_full, 4, {B, Hkv, -1, D})) return fail(RTK_ERR_INVALID, "k_full must be [B, H_kv, S_full, D]");
  const int64_t Sf = k_full->shape[2];
  if (!same_dims(v_full, 4, {B, Hkv, Sf, D})) return fail(RTK_ERR_INVALID, "v_full must be [B, H_kv, S_full, D]");
  if (mask_full != nullptr && !same_dims(mask_full, 2, {B, Sf})) return fail(RTK_ERR_INVALID, "mask_full must be [B, S_full]");
  if (!same_dims(k_sparse, 4, {B, Hkv, -1, DK})) return fail(RTK_ERR_INVALID, "k_sparse must be [B, H_kv, S_sparse, D_keep]");
  const int64_t Sv = k_sparse->shape[2];
  if (!same_dims(v_sparse, 4, {B, Hkv, Sv, D})) return fail(RTK_ERR_INVALID, "v_sparse must be [B, H_kv, S_sparse, D]");
  for (const rtk_tensor *t : {R_partial, k_full, v_full, k_sparse, v_sparse, out})
    if (t->dtype != q_full->dtype) return fail(RTK_ERR_INVALID, "all tensors but mask_full must share q_full's dtype");
  if (delta_mu != nullptr && delta_mu->dtype != q_full->dtype)
    return fail(RTK_ERR_INVALID, "all tensors but mask_full must share q_full's dtype");
  int64_t os[3] = {0, 0, 0};
  if (!out_view(out, B, Hq, D, os)) return fail(RTK_ERR_INVALID, "out must be [B, H_q, D] or [B, 1, H_q, D]");
  if (B * Hq == 0 || D == 0) return RTK_OK;
  DecodeArgs a{q_full, R_partial, delta_mu, k_full, v_full, mask_full, k_sparse, v_sparse, out, num_kv_groups, false};
  return run_decode(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int rtk_rotatek_decode_fp8(const rtk_tensor *q_full, const rtk_tensor *R_partial,
                           const rtk_tensor *delta_mu, const rtk_tensor *k_full,
                           const rtk_tensor *v_full, const rtk_tensor *mask_full,
                           const rtk_tensor *k8, const rtk_tensor *k_scale, const rtk_tensor *v8,
                           const rtk_tensor *v_scale, int64_t num_kv_groups, const rtk_tensor *out,
                           void *workspace, size_t workspace_bytes, void *stream) {
  g_last_error.clear();
  if (q_full == nullptr || q_full->ndim != 3) return fail(RTK_ERR_INVALID, "q_full must be [B, H_q, D]");
  if (R_partial == nullptr || R_partial->ndim != 4)
    return fail(RTK_ERR_INVALID, "R_partial must be [B, H_kv, D, D_keep]");
  if (mask_full != nullptr && mask_full->dtype != RTK_U8) return fail(RTK_ERR_INVALID, "mask_full must be uint8");
  const int64_t B = q_full->shape[0], Hq = q_full->shape[1], D = q_full->shape[2];
  const int64_t Hkv = R_partial->shape[1], DK = R_partial->shape[3];
  if (num_kv_groups <= 0 || Hq != Hkv * num_kv_groups)
    return fail(RTK_ERR_INVALID, "H_q=%lld is not H_kv=%lld * num_kv_groups=%lld", (long long)Hq,
                (long long)Hkv, (long long)num_kv_groups);
  if (!same_dims(R_partial, 4, {B, Hkv, D, -1}) || DK < 1 || DK > D)
    return fail(RTK_ERR_INVALID, "R_partial must be [B, H_kv, D, D_keep]");
  if (delta_mu != nullptr && !same_dims(delta_mu, 3, {B, Hkv, D}))
    return fail(RTK_ERR_INVALID, "delta_mu must be [B, H_kv, D]");
  if (!same_dims(k_full, 4, {B, Hkv, -1, D})) return fail(RTK_ERR_INVALID, "k_full must be [B, H_kv, S_full, D]");
  const int64_t Sf = k_full->shape[2];
  if (!same_dims(v_full, 4, {B, Hkv, Sf, D})) return fail(RTK_ERR_INVALID, "v_full must be [B, H_kv, S_full, D]");
  if (mask_full != nullptr && !same_dims(mask_full, 2, {B, Sf})) return fail(RTK_ERR_INVALID, "mask_full must be [B, S_full]");
  if (!same_dims(k8, 4, {B, Hkv, -1, DK}) || k8->dtype != RTK_U8)
    return fail(RTK_ERR_INVALID, "k_sparse_fp8 must be a uint8 (e4m3) [B, H_kv, S_sparse, D_keep]");
  const int64_t Sv = k8->shape[2];
  if (!same_dims(v8, 4, {B, Hkv, D, Sv}) || v8->dtype != RTK_U8 || (Sv > 1 && v8->stride[3] != 1))
    return fail(RTK_ERR_INVALID, "v_sparse_fp8 must be a uint8 (e4m3) [B, H_kv, D, S_sparse] with token stride 1 "
                                 "(the Values transposed)");
  if (!same_dims(k_scale, 3, {B, Hkv, DK}) || k_scale->dtype != RTK_F32 || k_scale->stride[2] != 1)
    return fail(RTK_ERR_INVALID, "k_scale must be a float32 [B, H_kv, D_keep] with unit channel stride");
  if (!same_dims(v_scale, 3, {B, Hkv, Sv}) || v_scale->dtype != RTK_F32)
    return fail(RTK_ERR_INVALID, "v_scale must be a float32 [B, H_kv, S_sparse]");
  for (const rtk_tensor *t : {R_partial, k_full, v_full, out})
    if (t->dtype != q_full->dtype) return fail(RTK_ERR_INVALID, "q, R, k_full, v_full and out must share a dtype");
  if (delta_mu != nullptr && delta_mu->dtype != q_full->dtype)
    return fail(RTK_ERR_INVALID, "q, R, k_full, v_full and out must share a dtype");
  int64_t os[3] = {0, 0, 0};
  if (!out_view(out, B, Hq, D, os)) return fail(RTK_ERR_INVALID, "out must be [B, H_q, D] or [B, 1, H_q, D]");
  if (B * Hq == 0 || D == 0) return RTK_OK;
  DecodeArgs a{q_full, R_partial, delta_mu, k_full, v_full, mask_full, k8, v8, out, num_kv_groups, false,
               k_scale, v_scale};
  return run_decode(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int rtk_quantize_visual_fp8(const rtk_tensor *k_sparse, const rtk_tensor *v_sparse, const rtk_tensor *k8_out,
                            const rtk_tensor *k_scale_out, const rtk_tensor *v8_out,
                            const rtk_tensor *v_scale_out, void *stream) {
  g_last_error.clear();
  View4 ks, vs;
  if (!as4(k_sparse, ks) || !as4(v_sparse, vs))
    return fail(RTK_ERR_INVALID, "k_sparse must be [B, H_kv, S, D_keep] and v_sparse [B, H_kv, S, 128]");
  const int64_t B = ks.n[0], H = ks.n[1], S = ks.n[2], DK = ks.n[3];
  if (!is_half_type(k_sparse->dtype) || v_sparse->dtype != k_sparse->dtype)
    return fail(RTK_ERR_UNSUPPORTED, "fp8 quantisation takes bfloat16 or float16 Keys and Values");
  if (vs.n[0] != B || vs.n[1] != H || vs.n[2] != S || vs.n[3] != 128)
    return fail(RTK_ERR_INVALID, "v_sparse must be [B, H_kv, S, 128]");
  if (DK != 16 && DK != 32 && DK != 64) return fail(RTK_ERR_UNSUPPORTED, "D_keep must be 16, 32 or 64");
  auto contiguous = [](const rtk_tensor *t, std::initializer_list<int64_t> dims) {
    if (t == nullptr || t->ndim != (int)dims.size()) return false;
    int64_t st = 1;
    int i = (int)dims.size() - 1;
    for (auto it = dims.end(); it != dims.begin(); --i) {
      --it;
      if (t->shape[i] != *it || (t->stride[i] != st && t->shape[i] != 1)) return false;
      st *= *it;
    }
    return true;
  };
  if (!contiguous(k8_out, {B, H, S, DK}) || k8_out->dtype != RTK_U8)
    return fail(RTK_ERR_INVALID, "k8_out must be a contiguous uint8 [B, H_kv, S, D_keep]");
  // V^T: [B, H, 128, S], token stride 1, channel rows of at least S rounded up
  // to 16 bytes (the quantiser writes whole 16-byte chunks), strides in 16 bytes
  const int64_t s16 = (S + 15) / 16 * 16;
  const bool v8_ok = v8_out != nullptr && v8_out->ndim == 4 && v8_out->dtype == RTK_U8 &&
                     v8_out->shape[0] == B && v8_out->shape[1] == H && v8_out->shape[2] == 128 &&
                     v8_out->shape[3] == S && (S <= 1 || v8_out->stride[3] == 1) &&
                     v8_out->stride[2] >= s16 && v8_out->stride[2] % 16 == 0 &&
                     (H == 1 || (v8_out->stride[1] >= 128 * v8_out->stride[2] && v8_out->stride[1] % 16 == 0)) &&
                     (B == 1 || (v8_out->stride[0] >= H * v8_out->stride[1] && v8_out->stride[0] % 16 == 0)) &&
                     reinterpret_cast<uintptr_t>(v8_out->data) % 16 == 0;
  if (!v8_ok)
    return fail(RTK_ERR_INVALID, "v8_out must be a uint8 [B, H_kv, 128, S] (the Values transposed) with token "
                                 "stride 1, 16-byte aligned rows of at least S rounded up to 16 bytes");
  if (!contiguous(k_scale_out, {B, H, DK}) || k_scale_out->dtype != RTK_F32)
    return fail(RTK_ERR_INVALID, "k_scale_out must be a contiguous float32 [B, H_kv, D_keep]");
  if (!contiguous(v_scale_out, {B, H, S}) || v_scale_out->dtype != RTK_F32)
    return fail(RTK_ERR_INVALID, "v_scale_out must be a contiguous float32 [B, H_kv, S]");
  const bool aligned = ks.s[3] == 1 && vs.s[3] == 1 && reinterpret_cast<uintptr_t>(ks.data) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(vs.data) % 16 == 0 && (ks.s[2] * 2) % 16 == 0 &&
                       (ks.s[1] * 2) % 16 == 0 && (ks.s[0] * 2) % 16 == 0 && (vs.s[2] * 2) % 16 == 0 &&
                       (vs.s[1] * 2) % 16 == 0 && (vs.s[0] * 2) % 16 == 0;
  if (!aligned) return fail(RTK_ERR_UNSUPPORTED, "fp8 quantisation needs channel-contiguous, 16-byte aligned rows");
  if (B * H == 0) return RTK_OK;
  if (B * H * S >= (1ll << 31) / 128) return fail(RTK_ERR_UNSUPPORTED, "tensor too large");
  rtk::QuantParams qp;
  std::memset(&qp, 0, sizeof(qp));
  qp.batch = (int)B; qp.heads = (int)H; qp.seq = (int)S; qp.keep = (int)DK;
  qp.keys = ks.data; qp.values = vs.data;
  for (int i = 0; i < 4; ++i) { qp.k_s[i] = ks.s[i]; qp.v_s[i] = vs.s[i]; }
  qp.keys8 = static_cast<uint8_t *>(k8_out->data);
  qp.k_scale = static_cast<float *>(k_scale_out->data);
  qp.values8t = static_cast<uint8_t *>(v8_out->data);
  for (int i = 0; i < 3; ++i) qp.v8_s[i] = v8_out->stride[i];
  qp.v_scale = static_cast<float *>(v_scale_out->data);
  const cudaError_t e = rtk::launch_quantize_fp8(k_sparse->dtype == RTK_BF16, qp, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fp8 quantisation launch");
  return RTK_OK;
}

int rtk_full_channel_decode(const rtk_tensor *q, const rtk_tensor *k, const rtk_tensor *v,
                            int64_t num_kv_groups, const rtk_tensor *out, void *workspace,
                            size_t workspace_bytes, void *stream) {
  g_last_error.clear();
  if (q == nullptr || q->ndim != 3) return fail(RTK_ERR_INVALID, "q must be [B, H_q, D]");
  const int64_t B = q->shape[0], Hq = q->shape[1], D = q->shape[2];
  if (k == nullptr || v == nullptr || k->ndim != 4 || v->ndim != 4)
    return fail(RTK_ERR_INVALID, "k/v must be [B, H_kv, S, D]");
  if (k->shape[3] != D || v->shape[3] != D) return fail(RTK_ERR_INVALID, "k/v head_dim must match q's");
  const int64_t Hkv = k->shape[1], S = k->shape[2];
  if (!same_dims(k, 4, {B, Hkv, S, D}) || !same_dims(v, 4, {B, Hkv, S, D}))
    return fail(RTK_ERR_INVALID, "k/v must be [B, H_kv, S, D]");
  if (num_kv_groups <= 0 || Hq != Hkv * num_kv_groups)
    return fail(RTK_ERR_INVALID, "H_q=%lld is not H_kv=%lld * num_kv_groups=%lld", (long long)Hq,
                (long long)Hkv, (long long)num_kv_groups);
  if (!dtype_ok(q->dtype) || k->dtype != q->dtype || v->dtype != q->dtype)
    return fail(RTK_ERR_INVALID, "q, k, v and out must share one dtype (float32, bfloat16 or float16)");
  int64_t os[3] = {0, 0, 0};
  if (!out_view(out, B, Hq, D, os) || out->dtype != q->dtype)
    return fail(RTK_ERR_INVALID, "out must be [B, H_q, D] or [B, 1, H_q, D] in q's dtype");
  if (B * Hq == 0 || D == 0) return RTK_OK;
  DecodeArgs a{q, nullptr, nullptr, k, v, nullptr, nullptr, nullptr, out, num_kv_groups, true};
  return run_decode(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int rtk_spark_decode(const rtk_tensor *q_full, const rtk_tensor *k_full, const rtk_tensor *v_full,
                     const rtk_tensor *mask_full, const rtk_tensor *k_kept, const rtk_tensor *keep_idx,
                     const rtk_tensor *pruned_mean, const rtk_tensor *v_sparse, int64_t num_kv_groups,
                     const rtk_tensor *out, void *workspace, size_t workspace_bytes, void *stream) {
  g_last_error.clear();
  if (q_full == nullptr || q_full->ndim != 3) return fail(RTK_ERR_INVALID, "q_full must be [B, H_q, D]");
  if (k_kept == nullptr || k_kept->ndim != 4)
    return fail(RTK_ERR_INVALID, "k_kept must be [B, H_kv, S_sparse, D_keep]");
  if (mask_full != nullptr && mask_full->dtype != RTK_U8) return fail(RTK_ERR_INVALID, "mask_full must be uint8");
  const int64_t B = q_full->shape[0], Hq = q_full->shape[1], D = q_full->shape[2];
  const int64_t Hkv = k_kept->shape[1], Sv = k_kept->shape[2], DK = k_kept->shape[3];
  if (num_kv_groups <= 0 || Hq != Hkv * num_kv_groups)
    return fail(RTK_ERR_INVALID, "H_q=%lld is not H_kv=%lld * num_kv_groups=%lld", (long long)Hq,
                (long long)Hkv, (long long)num_kv_groups);
  if (!same_dims(k_kept, 4, {B, Hkv, Sv, DK}) || DK < 1 || DK > D)
    return fail(RTK_ERR_INVALID, "k_kept must be [B, H_kv, S_sparse, D_keep] with D_keep <= D");
  if (!same_dims(keep_idx, 4, {B, Hkv, Sv, DK}) || keep_idx->dtype != RTK_U8)
    return fail(RTK_ERR_INVALID, "keep_idx must be a uint8 [B, H_kv, S_sparse, D_keep]");
  if (!same_dims(pruned_mean, 4, {B, Hkv, Sv, 1}))
    return fail(RTK_ERR_INVALID, "pruned_mean must be [B, H_kv, S_sparse, 1]");
  if (!same_dims(k_full, 4, {B, Hkv, -1, D})) return fail(RTK_ERR_INVALID, "k_full must be [B, H_kv, S_full, D]");
  const int64_t Sf = k_full->shape[2];
  if (!same_dims(v_full, 4, {B, Hkv, Sf, D})) return fail(RTK_ERR_INVALID, "v_full must be [B, H_kv, S_full, D]");
  if (mask_full != nullptr && !same_dims(mask_full, 2, {B, Sf})) return fail(RTK_ERR_INVALID, "mask_full must be [B, S_full]");
  if (!same_dims(v_sparse, 4, {B, Hkv, Sv, D})) return fail(RTK_ERR_INVALID, "v_sparse must be [B, H_kv, S_sparse, D]");
  if (!dtype_ok(q_full->dtype)) return fail(RTK_ERR_INVALID, "q_full dtype must be float32, bfloat16 or float16");
  for (const rtk_tensor *t : {k_full, v_full, k_kept, pruned_mean, v_sparse, out})
    if (t->dtype != q_full->dtype)
      return fail(RTK_ERR_INVALID, "all tensors but mask_full and keep_idx must share q_full's dtype");
  int64_t os[3] = {0, 0, 0};
  if (!out_view(out, B, Hq, D, os)) return fail(RTK_ERR_INVALID, "out must be [B, H_q, D] or [B, 1, H_q, D]");
  if (B * Hq == 0 || D == 0) return RTK_OK;
  DecodeArgs a{q_full, nullptr, nullptr, k_full, v_full, mask_full, k_kept, v_sparse, out, num_kv_groups, false};
  a.kidx = keep_idx;
  a.kmean = pruned_mean;
  return run_decode(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int rtk_spark_pack(const rtk_tensor *keep_mask, const rtk_tensor *keep_idx_out, void *status, void *stream) {
  g_last_error.clear();
  if (keep_mask == nullptr || keep_mask->ndim != 4 || keep_mask->dtype != RTK_U8)
    return fail(RTK_ERR_INVALID, "keep_mask must be a bool / uint8 [B, H_kv, S, D]");
  const int64_t B = keep_mask->shape[0], H = keep_mask->shape[1], S = keep_mask->shape[2];
  if (keep_mask->shape[3] != 128 || keep_mask->stride[3] != 1)
    return fail(RTK_ERR_UNSUPPORTED, "keep_mask needs D = 128 with a unit channel stride");
  if (keep_idx_out == nullptr || keep_idx_out->ndim != 4 || keep_idx_out->dtype != RTK_U8 ||
      keep_idx_out->shape[0] != B || keep_idx_out->shape[1] != H || keep_idx_out->shape[2] != S)
    return fail(RTK_ERR_INVALID, "keep_idx_out must be a uint8 [B, H_kv, S, D_keep]");
  const int64_t DK = keep_idx_out->shape[3];
  if (DK < 1 || DK > 128) return fail(RTK_ERR_INVALID, "D_keep must be in 1..128");
  if (keep_idx_out->stride[3] != 1 || keep_idx_out->stride[2] != DK || keep_idx_out->stride[1] != S * DK ||
      keep_idx_out->stride[0] != H * S * DK)
    return fail(RTK_ERR_INVALID, "keep_idx_out must be contiguous");
  if (B * H * S == 0) return RTK_OK;
  if (B * H * S >= (1ll << 31) * 8) return fail(RTK_ERR_UNSUPPORTED, "tensor too large");
  rtk::SparkPackParams p;
  p.batch = (int)B; p.heads = (int)H; p.seq = (int)S; p.keep = (int)DK;
  p.mask = static_cast<const uint8_t *>(keep_mask->data);
  for (int i = 0; i < 3; ++i) p.m_s[i] = keep_mask->stride[i];
  p.idx = static_cast<uint8_t *>(keep_idx_out->data);
  p.status = static_cast<unsigned int *>(status);
  const cudaError_t e = rtk::launch_spark_pack(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "SparK index packing launch");
  return RTK_OK;
}

// ------------------------------------------------------------------ rotation builder
}  // extern "C"

namespace {
// sum_s k k^T and sum_s k for every (b, h) of a [B, H, S, 128] Key view:
// tensor-core kernel for bf16 / fp16 layouts TMA can describe, else the
// CUDA-core kernel.
cudaError_t launch_covariance(const View4 &kv, int dt, float *cov, float *ksum, int device,
                              cudaStream_t st) {
  const int64_t B = kv.n[0], H = kv.n[1], S = kv.n[2];
  rtk::CovParams cp;
  std::memset(&cp, 0, sizeof(cp));
  cp.dtype = dt;
  cp.batch = (int)B; cp.heads = (int)H; cp.seq = (int)S;
  cp.keys = kv.data;
  for (int i = 0; i < 4; ++i) cp.k_s[i] = kv.s[i];
  cp.cov = cov; cp.ksum = ksum;
  bool tc = is_half_type(dt) && S > 0;
  CUtensorMap kmap;
  if (tc)
    tc = encode_map(&kmap, kv, dt == RTK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                    64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  if (tc) {
    const int64_t tiles = cdiv(S, 64);
    int z = 8;
    while (z > 1 && (B * H * z > 2 * (int64_t)sm_count(device) || z > tiles)) z >>= 1;
    cp.splits = z;
    return rtk::launch_cov_tc(dt == RTK_BF16, kmap, cp, st);
  }
  cp.splits = 1;
  return rtk::launch_cov_simt(cp, st);
}

// kept = K . R on the tensor cores where the layouts allow (TMA kernel for
// keep <= 64, cp.async kernel for keep in {96, 128}), else the CUDA-core kernel.
cudaError_t launch_rotation(const View4 &kv, int dt, int64_t keep, const rtk_tensor *R_out,
                            const rtk_tensor *kept_out, unsigned int *status, cudaStream_t st,
                            int max_ctas = 0) {
  const int64_t B = kv.n[0], H = kv.n[1], S = kv.n[2];
  if (S == 0) return cudaSuccess;
  rtk::RotateParams rp;
  std::memset(&rp, 0, sizeof(rp));
  rp.dtype = dt;
  rp.batch = (int)B; rp.heads = (int)H; rp.seq = (int)S; rp.keep = (int)keep;
  rp.keys = kv.data;
  for (int i = 0; i < 4; ++i) {
    rp.k_s[i] = kv.s[i];
    rp.R_s[i] = R_out->stride[i];
    rp.o_s[i] = kept_out->stride[i];
  }
  rp.R = R_out->data;
  rp.out = kept_out->data;
  rp.status = status;
  rp.max_ctas = max_ctas;
  const bool rtc = is_half_type(dt) && keep % 16 == 0 && kv.s[3] == 1 && (kv.s[2] * 2) % 16 == 0 &&
                   (kv.s[1] * 2) % 16 == 0 && (kv.s[0] * 2) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(kv.data) % 16 == 0 && kept_out->stride[3] == 1 &&
                   (kept_out->stride[2] * 2) % 16 == 0 && (kept_out->stride[1] * 2) % 16 == 0 &&
                   (kept_out->stride[0] * 2) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(kept_out->data) % 16 == 0;
  const bool r_vec = R_out->stride[3] == 1 && R_out->stride[2] % 8 == 0 && R_out->stride[1] % 8 == 0 &&
                     R_out->stride[0] % 8 == 0 && reinterpret_cast<uintptr_t>(R_out->data) % 16 == 0;
  CUtensorMap kmap;
  const bool tma = rtc && r_vec && keep <= 64 && B * H * cdiv(S, 64) < (1ll << 31) &&
                   encode_map(&kmap, kv, dt == RTK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                              64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
  return tma ? rtk::launch_rotate_tma(dt == RTK_BF16, kmap, rp, st)
             : rtc ? rtk::launch_rotate_tc(dt == RTK_BF16, rp, st) : rtk::launch_rotate_simt(rp, st);
}

// Build workspace: status word (256 B) | cov | ksum.
struct BuildWs {
  unsigned int *status;
  float *cov, *ksum;
};

BuildWs build_ws(void *workspace, int64_t n, int64_t D) {
  unsigned char *ws = static_cast<unsigned char *>(workspace);
  BuildWs w;
  w.status = reinterpret_cast<unsigned int *>(ws);
  w.cov = reinterpret_cast<float *>(ws + kStatusBytes);
  w.ksum = reinterpret_cast<float *>(ws + kStatusBytes + align_up((size_t)n * D * D * sizeof(float)));
  return w;
}

// Shapes and dtypes of the build's query and output arguments for B x H
// matrices of S visual tokens (RTK_OK or a failure already recorded).
int check_build_args(int64_t B, int64_t H, int64_t S, int64_t D, int dt, const rtk_tensor *queries,
                     int64_t num_kv_groups, int64_t keep, const rtk_tensor *kept_out,
                     const rtk_tensor *R_out, const rtk_tensor *delta_mu_out, const rtk_tensor *eigvals_out) {
  if (keep < 1 || keep > D) return fail(RTK_ERR_INVALID, "keep must be in [1, head_dim] (got %lld)", (long long)keep);
  if (queries != nullptr) {
    if (queries->ndim != 4 || queries->shape[0] != B || queries->shape[3] != D ||
        num_kv_groups <= 0 || queries->shape[1] != H * num_kv_groups)
      return fail(RTK_ERR_INVALID, "queries_recent must be [B, H_kv * num_kv_groups, W, D]");
    if (!dtype_ok(queries->dtype)) return fail(RTK_ERR_INVALID, "queries_recent dtype must be float32, bfloat16 or float16");
  }
  if (!same_dims(kept_out, 4, {B, H, S, keep}) || kept_out->dtype != dt)
    return fail(RTK_ERR_INVALID, "kept_out must be [B, H_kv, S_v, keep] in the Keys' dtype");
  if (!same_dims(R_out, 4, {B, H, D, keep}) || R_out->dtype != dt)
    return fail(RTK_ERR_INVALID, "R_out must be [B, H_kv, D, keep] in the Keys' dtype");
  if (delta_mu_out != nullptr && (!same_dims(delta_mu_out, 3, {B, H, D}) || delta_mu_out->dtype != dt))
    return fail(RTK_ERR_INVALID, "delta_mu_out must be [B, H_kv, D] in the Keys' dtype");
  if (eigvals_out != nullptr && (!same_dims(eigvals_out, 3, {B, H, D}) || eigvals_out->dtype != RTK_F32 ||
                                 eigvals_out->stride[2] != 1 || eigvals_out->stride[1] != D ||
                                 eigvals_out->stride[0] != H * D))
    return fail(RTK_ERR_INVALID, "eigvals_out must be a contiguous float32 [B, H_kv, D]");
  return RTK_OK;
}

// The build after the sums are in w.cov / w.ksum: centring, query weighting,
// eigensolver, top-k R and delta_mu, then kept = K_vis . R.
// A private non-blocking stream and two events per device for the build's
// overlap of the eigensolver's last wave with the rotation (created on first
// use, kept for the process).  `mu` is held while a build enqueues its fork
// and join, so that concurrent callers on one device never wait on each
// other's event records.
struct SideStream {
  cudaStream_t stream;
  cudaEvent_t solved, rotated;
  std::mutex mu;
};
SideStream *side_stream(int device, cudaStream_t caller) {
  static std::mutex mu;
  static SideStream cache[64];
  static bool made[64] = {false};
  if (device < 0 || device >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!made[device]) {
    // not created while the caller's stream is being captured into a graph
    // (that call takes the single-stream path; the next eager call creates it)
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(caller, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
      cudaGetLastError();
      return nullptr;
    }
    SideStream &s = cache[device];
    if (cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
    if (cudaEventCreateWithFlags(&s.solved, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&s.rotated, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    made[device] = true;
  }
  return &cache[device];
}

int64_t dtype_size(int dt) { return dt == RTK_F32 ? 4 : 2; }

int finish_build(const View4 &kv, int dt, const rtk_tensor *queries, int64_t num_kv_groups, int64_t keep,
                 const rtk_tensor *kept_out, const rtk_tensor *R_out, const rtk_tensor *delta_mu_out,
                 const rtk_tensor *eigvals_out, const BuildWs &w, cudaStream_t st) {
  const int64_t B = kv.n[0], H = kv.n[1], S = kv.n[2];
  rtk::EighParams jp;
  std::memset(&jp, 0, sizeof(jp));
  jp.nmat = (int)(B * H); jp.heads = (int)H;
  jp.cov = w.cov; jp.ksum = w.ksum; jp.count = (int)std::max<int64_t>(S, 1);
  jp.center_dtype = dt;
  if (queries != nullptr) {
    jp.q = queries->data; jp.q_dtype = queries->dtype;
    for (int i = 0; i < 4; ++i) jp.q_s[i] = queries->stride[i];
    jp.window = (int)queries->shape[2];
    jp.groups = (int)num_kv_groups;
  }
  jp.keep = (int)keep;
  jp.R = R_out->data; jp.R_dtype = dt;
  for (int i = 0; i < 4; ++i) jp.R_s[i] = R_out->stride[i];
  if (delta_mu_out != nullptr) {
    jp.dm = delta_mu_out->data;
    for (int i = 0; i < 3; ++i) jp.dm_s[i] = delta_mu_out->stride[i];
  }
  jp.evals = eigvals_out ? static_cast<float *>(eigvals_out->data) : nullptr;
  // One CTA per matrix.  When the matrices fill whole waves of the device's
  // solver slots but a few, those few would run as a last wave on their own
  // (a lone solve takes ~0.2 ms).  Split them off: the full waves first, then
  // the tail, while the rotation of the solved batch rows streams on the SMs
  // the tail leaves free (a side stream joined by events; capturable).
  const int device = current_device();
  const int64_t nmat = B * H;
  const int64_t sms = sm_count(device);
  const int64_t slots = (keep <= 32 ? 2 : 1) * sms;
  const int64_t tail = nmat % slots;
  const int64_t bt = (nmat > slots && tail > 0 && tail <= slots / 4 && S > 0) ? cdiv(tail, H) : 0;
  SideStream *side = bt > 0 && bt < B ? side_stream(device, st) : nullptr;
  if (side == nullptr) {
    cudaError_t e = rtk::launch_eigh(jp, st);
    if (e != cudaSuccess) return cuda_fail(e, "rotation builder (eigensolver) launch");
    e = launch_rotation(kv, dt, keep, R_out, kept_out, w.status, st);
    if (e != cudaSuccess) return cuda_fail(e, "rotation builder (rotate) launch");
    return RTK_OK;
  }
  std::lock_guard<std::mutex> fork_join(side->mu);
  const int64_t b1 = B - bt;
  jp.m0 = 0;
  jp.nmat = (int)(b1 * H);
  cudaError_t e = rtk::launch_eigh(jp, st);
  if (e == cudaSuccess) e = cudaEventRecord(side->solved, st);
  if (e == cudaSuccess) {
    jp.m0 = (int)(b1 * H);
    jp.nmat = (int)(bt * H);
    e = rtk::launch_eigh(jp, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "rotation builder (eigensolver) launch");
  // batch rows [0, b1) on the side stream, on the SMs the tail's CTAs leave free
  View4 k1 = kv;
  k1.n[0] = b1;
  e = cudaStreamWaitEvent(side->stream, side->solved, 0);
  if (e == cudaSuccess)
    e = launch_rotation(k1, dt, keep, R_out, kept_out, w.status, side->stream,
                        (int)std::max<int64_t>(1, sms - bt * H));   // a tail CTA may hold an SM alone
  if (e == cudaSuccess) e = cudaEventRecord(side->rotated, side->stream);
  // rows [b1, B) behind the tail on the caller's stream, then join
  if (e == cudaSuccess) {
    View4 k2 = kv;
    k2.n[0] = bt;
    k2.data = static_cast<const unsigned char *>(kv.data) + b1 * kv.s[0] * dtype_size(dt);
    rtk_tensor R2 = *R_out, O2 = *kept_out;
    R2.shape[0] = bt;
    R2.data = static_cast<unsigned char *>(R_out->data) + b1 * R_out->stride[0] * dtype_size(R_out->dtype);
    O2.shape[0] = bt;
    O2.data = static_cast<unsigned char *>(kept_out->data) + b1 * kept_out->stride[0] * dtype_size(kept_out->dtype);
    e = launch_rotation(k2, dt, keep, &R2, &O2, w.status, st);
  }
  if (e == cudaSuccess) e = cudaStreamWaitEvent(st, side->rotated, 0);
  if (e != cudaSuccess) return cuda_fail(e, "rotation builder (rotate) launch");
  return RTK_OK;
}

// A 16-bit tensor of rank 2 or 3 (innermost first in dims / box, byte strides
// of the outer dimensions) as a 128B-swizzled TMA map.
bool encode_map_rank(CUtensorMap *map, CUtensorMapDataType dt, int rank, const void *data,
                     const cuuint64_t *dims, const cuuint64_t *strides, const cuuint32_t *box) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr || reinterpret_cast<uintptr_t>(data) % 16 != 0) return false;
  for (int i = 0; i < rank; ++i)
    if (dims[i] == 0 || dims[i] > (1ull << 31)) return false;
  for (int i = 0; i < rank - 1; ++i)
    if (strides[i] % 16 != 0 || strides[i] == 0) return false;
  cuuint32_t estride[3] = {1, 1, 1};
  return fn(map, dt, rank, const_cast<void *>(data), dims, strides, box, estride,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Pair steps (two 128-token tiles of one span) of one sequence.
int64_t kproj_tiles_per_unit(int64_t S, int64_t vis_start, int64_t vis_len) {
  return (cdiv(vis_start, 128) + 1) / 2 + (cdiv(vis_len, 128) + 1) / 2 + (cdiv(S - vis_start - vis_len, 128) + 1) / 2;
}
// Co-resident two-CTA clusters of the projection kernel on `device` (cached;
// one CTA per SM, so at most SMs / 2).
int64_t kproj_cluster_slots(int device) {
  static std::mutex mu;
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return sm_count(device) / 2;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[device] == 0) {
    int n = rtk::kproj_max_clusters(1);
    if (n <= 0) n = sm_count(device) / 2;
    cache[device] = n;
  }
  return cache[device];
}
// groups of ceil(H / 2) two-CTA clusters (one per head pair), as many groups
// as fit the device at once and there are (b, step) items
int64_t kproj_grid(int64_t B, int64_t H, int64_t S, int64_t vis_start, int64_t vis_len, int device) {
  const int64_t pairs = rtk::kproj_pairs(H);
  const int64_t items = B * kproj_tiles_per_unit(S, vis_start, vis_len);
  const int64_t groups = std::max<int64_t>(1, std::min<int64_t>(kproj_cluster_slots(device) / pairs, items));
  return groups * pairs * 2;
}
// Validate and launch the projection, then the visual span's sums from the
// Keys just written; cov / ksum are B*H contiguous fp32 blocks.
// keys_out [B, H, S, 128].
int run_key_projection(const rtk_tensor *x, const rtk_tensor *w, const rtk_tensor *bias,
                       const rtk_tensor *cos, const rtk_tensor *sin, int64_t vis_start, int64_t vis_len,
                       const rtk_tensor *keys_out, float *cov, float *ksum, unsigned int *status, cudaStream_t st) {
  if (x == nullptr || x->ndim != 3) return fail(RTK_ERR_INVALID, "hidden_states must be [B, S, hidden]");
  const int64_t B = x->shape[0], S = x->shape[1], Hd = x->shape[2];
  const int dt = x->dtype;
  if (!is_half_type(dt)) return fail(RTK_ERR_UNSUPPORTED, "the fused Key projection needs bfloat16 or float16 inputs");
  if (w == nullptr || w->ndim != 2 || w->shape[1] != Hd || w->shape[0] % 128 != 0 || w->shape[0] == 0 ||
      w->dtype != dt)
    return fail(RTK_ERR_INVALID, "w_k must be [H_kv * 128, hidden] in the hidden states' dtype");
  const int64_t H = w->shape[0] / 128;
  if (bias != nullptr && (bias->ndim != 1 || bias->shape[0] != H * 128 || bias->dtype != dt || bias->stride[0] != 1))
    return fail(RTK_ERR_INVALID, "bias must be a contiguous [H_kv * 128] vector in the hidden states' dtype");
  for (const rtk_tensor *c : {cos, sin}) {
    if (c == nullptr || c->ndim != 3 || (c->shape[0] != B && c->shape[0] != 1) || c->shape[1] != S ||
        c->shape[2] != 128 || c->dtype != dt)
      return fail(RTK_ERR_INVALID, "cos / sin must be [B or 1, S, 128] in the hidden states' dtype");
  }
  if (cos->stride[0] != sin->stride[0] || cos->stride[1] != sin->stride[1] || cos->shape[0] != sin->shape[0])
    return fail(RTK_ERR_INVALID, "cos and sin must have the same shape and strides");
  if (vis_start < 0 || vis_len < 0 || vis_start + vis_len > S)
    return fail(RTK_ERR_INVALID, "the visual span [%lld, %lld) is not inside [0, %lld)", (long long)vis_start,
                (long long)(vis_start + vis_len), (long long)S);
  if (!same_dims(keys_out, 4, {B, H, S, 128}) || keys_out->dtype != dt)
    return fail(RTK_ERR_INVALID, "keys_out must be [B, H_kv, S, 128] in the hidden states' dtype");
  if (Hd % 64 != 0) return fail(RTK_ERR_UNSUPPORTED, "hidden size must be a multiple of 64 (got %lld)", (long long)Hd);
  if (B * S >= (1ll << 31) || Hd >= (1ll << 31) ||
      B * kproj_tiles_per_unit(S, vis_start, vis_len) >= (1ll << 31) || H >= (1ll << 20))
    return fail(RTK_ERR_UNSUPPORTED, "tensor too large");
  if (B == 0) return RTK_OK;
  if (S == 0) {
    cudaError_t e = cudaMemsetAsync(cov, 0, (size_t)B * H * 128 * 128 * sizeof(float), st);
    if (e == cudaSuccess) e = cudaMemsetAsync(ksum, 0, (size_t)B * H * 128 * sizeof(float), st);
    return e == cudaSuccess ? RTK_OK : cuda_fail(e, "key projection (empty sequence)");
  }
  // layouts: channel stride 1, 16-byte aligned rows for TMA and the cos / sin vector loads
  const int64_t cs_sb = cos->shape[0] == 1 ? 0 : cos->stride[0];
  const bool cs_ok = cos->stride[2] == 1 && sin->stride[2] == 1 && (cos->stride[1] * 2) % 16 == 0 &&
                     (cs_sb * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(cos->data) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(sin->data) % 16 == 0;
  if (!cs_ok || x->stride[2] != 1 || w->stride[1] != 1 || keys_out->stride[3] != 1)
    return fail(RTK_ERR_UNSUPPORTED, "the fused Key projection needs channel-contiguous, 16-byte aligned rows");
  const CUtensorMapDataType tdt = dt == RTK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  rtk::KProjMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  {
    const cuuint64_t dims[3] = {(cuuint64_t)Hd, (cuuint64_t)S, (cuuint64_t)B};
    const cuuint64_t strides[2] = {(cuuint64_t)(S == 1 ? Hd * 2 : x->stride[1] * 2),
                                   (cuuint64_t)(B == 1 ? S * Hd * 2 : x->stride[0] * 2)};
    const cuuint32_t box[3] = {64, 128, 1};
    if (!encode_map_rank(&maps.x, tdt, 3, x->data, dims, strides, box))
      return fail(RTK_ERR_UNSUPPORTED, "hidden_states layout is not describable by TMA (16-byte aligned strides needed)");
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)Hd, (cuuint64_t)(H * 128)};
    const cuuint64_t strides[1] = {(cuuint64_t)(w->stride[0] * 2)};
    const cuuint32_t box[2] = {64, 128};
    if (!encode_map_rank(&maps.w, tdt, 2, w->data, dims, strides, box))
      return fail(RTK_ERR_UNSUPPORTED, "w_k layout is not describable by TMA (16-byte aligned rows needed)");
  }
  {
    // cos / sin rows: one 3-D map each; a table shared by every b has batch extent 1
    const int64_t bc = cs_sb == 0 ? 1 : B;
    const cuuint64_t dims[3] = {128, (cuuint64_t)S, (cuuint64_t)bc};
    const cuuint64_t strides[2] = {(cuuint64_t)(cos->stride[1] * 2),
                                   (cuuint64_t)(bc == 1 ? S * cos->stride[1] * 2 : cs_sb * 2)};
    const cuuint32_t box[3] = {64, 128, 1};
    if (!encode_map_rank(&maps.cs[0], tdt, 3, cos->data, dims, strides, box) ||
        !encode_map_rank(&maps.cs[1], tdt, 3, sin->data, dims, strides, box))
      return fail(RTK_ERR_UNSUPPORTED, "cos / sin layout is not describable by TMA (16-byte aligned rows needed)");
  }
  const int64_t span_start[3] = {0, vis_start, vis_start + vis_len};
  const int64_t span_len[3] = {vis_start, vis_len, S - vis_start - vis_len};
  for (int i = 0; i < 3; ++i) {
    if (span_len[i] == 0) continue;
    View4 v;
    v.data = static_cast<const unsigned char *>(keys_out->data) + span_start[i] * keys_out->stride[2] * 2;
    v.n[0] = B; v.n[1] = H; v.n[2] = span_len[i]; v.n[3] = 128;
    for (int j = 0; j < 4; ++j) v.s[j] = keys_out->stride[j];
    if (!encode_map(&maps.k_out[i], v, tdt, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(RTK_ERR_UNSUPPORTED, "keys_out layout is not describable by TMA (16-byte aligned strides needed)");
  }
  rtk::KProjParams kp;
  std::memset(&kp, 0, sizeof(kp));
  kp.batch = (int)B; kp.heads = (int)H; kp.seq = (int)S; kp.hidden = (int)Hd;
  kp.vis_start = (int)vis_start; kp.vis_len = (int)vis_len;
  kp.bias = bias != nullptr ? bias->data : nullptr;
  kp.cs_sb = cs_sb;
  kp.status = status;
  // persistent: groups x head pairs x 2 CTAs, one CTA per SM; contiguous shares of the B x steps items
  const int device = current_device();
  kp.grid = (int)kproj_grid(B, H, S, vis_start, vis_len, device);
  cudaError_t e = rtk::launch_kproj_tc(dt == RTK_BF16, maps, kp, st);
  if (e != cudaSuccess) return cuda_fail(e, "key projection launch");
  // sum k k^T and sum k over the visual span, read back while the Keys are in L2
  if (vis_len == 0) {
    e = cudaMemsetAsync(cov, 0, (size_t)B * H * 128 * 128 * sizeof(float), st);
    if (e == cudaSuccess) e = cudaMemsetAsync(ksum, 0, (size_t)B * H * 128 * sizeof(float), st);
  } else {
    View4 kv;
    as4(keys_out, kv);
    kv.data = static_cast<const unsigned char *>(keys_out->data) + vis_start * keys_out->stride[2] * 2;
    kv.n[2] = vis_len;
    e = launch_covariance(kv, dt, cov, ksum, device, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "key projection (visual-span sums) launch");
  return RTK_OK;
}
}  // namespace

extern "C" {

int rtk_key_covariance(const rtk_tensor *keys, const rtk_tensor *cov_out, const rtk_tensor *ksum_out,
                       void *stream) {
  g_last_error.clear();
  View4 kv;
  if (!as4(keys, kv) || !dtype_ok(keys->dtype)) return fail(RTK_ERR_INVALID, "keys must be a [B, H, S, 128] float tensor");
  if (kv.n[3] != 128) return fail(RTK_ERR_UNSUPPORTED, "head_dim must be 128 (got %lld)", (long long)kv.n[3]);
  const int64_t B = kv.n[0], H = kv.n[1];
  if (!same_dims(cov_out, 4, {B, H, 128, 128}) || cov_out->dtype != RTK_F32 || cov_out->stride[3] != 1 ||
      cov_out->stride[2] != 128 || cov_out->stride[1] != 128 * 128 || cov_out->stride[0] != H * 128 * 128)
    return fail(RTK_ERR_INVALID, "cov_out must be a contiguous float32 [B, H, 128, 128]");
  if (!same_dims(ksum_out, 3, {B, H, 128}) || ksum_out->dtype != RTK_F32 || ksum_out->stride[2] != 1 ||
      ksum_out->stride[1] != 128 || ksum_out->stride[0] != H * 128)
    return fail(RTK_ERR_INVALID, "ksum_out must be a contiguous float32 [B, H, 128]");
  if (B * H == 0) return RTK_OK;
  const cudaError_t e = launch_covariance(kv, keys->dtype, static_cast<float *>(cov_out->data),
                                          static_cast<float *>(ksum_out->data), current_device(),
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "key covariance launch");
  return RTK_OK;
}

size_t rtk_build_rotation_workspace_size(int64_t batch, int64_t kv_heads, int64_t head_dim) {
  const int64_t n = batch * kv_heads;
  return kStatusBytes + align_up((size_t)n * head_dim * head_dim * sizeof(float)) +
         align_up((size_t)n * head_dim * sizeof(float));
}

// [0, 256) status word, unused by the solver (which needs no global scratch);
// kept so that one buffer can serve every builder entry point
size_t rtk_eigh_topk_workspace_size(int64_t n) {
  (void)n;
  return kStatusBytes;
}

int rtk_build_rotation(const rtk_tensor *keys, const rtk_tensor *queries, int64_t num_kv_groups,
                       int64_t keep, const rtk_tensor *kept_out, const rtk_tensor *R_out,
                       const rtk_tensor *delta_mu_out, const rtk_tensor *eigvals_out,
                       void *workspace, size_t workspace_bytes, void *stream) {
  g_last_error.clear();
  View4 kv;
  if (!as4(keys, kv)) return fail(RTK_ERR_INVALID, "keys_vision must be [B, H_kv, S_v, D]");
  const int64_t B = kv.n[0], H = kv.n[1], S = kv.n[2], D = kv.n[3];
  if (!dtype_ok(keys->dtype)) return fail(RTK_ERR_INVALID, "keys_vision dtype must be float32, bfloat16 or float16");
  if (D != 128) return fail(RTK_ERR_UNSUPPORTED, "the rotation builder supports head_dim 128 (got %lld)", (long long)D);
  const int rc = check_build_args(B, H, S, D, keys->dtype, queries, num_kv_groups, keep, kept_out, R_out,
                                  delta_mu_out, eigvals_out);
  if (rc != RTK_OK) return rc;
  if (B * H == 0) return RTK_OK;
  const size_t need = rtk_build_rotation_workspace_size(B, H, D);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(RTK_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const BuildWs w = build_ws(workspace, B * H, D);
  // ---- covariance + channel sums
  const cudaError_t e = launch_covariance(kv, keys->dtype, w.cov, w.ksum, current_device(), st);
  if (e != cudaSuccess) return cuda_fail(e, "rotation builder (covariance) launch");
  // ---- centring, query weighting, eigensolver, top-k R, delta_mu; kept = K_vis . R
  return finish_build(kv, keys->dtype, queries, num_kv_groups, keep, kept_out, R_out, delta_mu_out,
                      eigvals_out, w, st);
}

int rtk_key_projection(const rtk_tensor *hidden, const rtk_tensor *w_k, const rtk_tensor *bias,
                       const rtk_tensor *cos, const rtk_tensor *sin, int64_t vis_start, int64_t vis_len,
                       const rtk_tensor *keys_out, const rtk_tensor *cov_out, const rtk_tensor *ksum_out,
                       void *workspace, size_t workspace_bytes, void *stream) {
  g_last_error.clear();
  if (keys_out == nullptr || keys_out->ndim != 4) return fail(RTK_ERR_INVALID, "keys_out must be [B, H_kv, S, 128]");
  const int64_t B = keys_out->shape[0], H = keys_out->shape[1];
  if (!same_dims(cov_out, 4, {B, H, 128, 128}) || cov_out->dtype != RTK_F32 || cov_out->stride[3] != 1 ||
      cov_out->stride[2] != 128 || cov_out->stride[1] != 128 * 128 || cov_out->stride[0] != H * 128 * 128)
    return fail(RTK_ERR_INVALID, "cov_out must be a contiguous float32 [B, H_kv, 128, 128]");
  if (!same_dims(ksum_out, 3, {B, H, 128}) || ksum_out->dtype != RTK_F32 || ksum_out->stride[2] != 1 ||
      ksum_out->stride[1] != 128 || ksum_out->stride[0] != H * 128)
    return fail(RTK_ERR_INVALID, "ksum_out must be a contiguous float32 [B, H_kv, 128]");
  if (workspace == nullptr || workspace_bytes < kStatusBytes)
    return fail(RTK_ERR_WORKSPACE, "workspace has %zu bytes, needs at least %zu", workspace_bytes, kStatusBytes);
  return run_key_projection(hidden, w_k, bias, cos, sin, vis_start, vis_len, keys_out,
                            static_cast<float *>(cov_out->data), static_cast<float *>(ksum_out->data),
                            static_cast<unsigned int *>(workspace), static_cast<cudaStream_t>(stream));
}

size_t rtk_key_projection_workspace_size(int64_t batch, int64_t kv_heads, int64_t seq, int64_t vis_start,
                                         int64_t vis_len, int32_t device) {
  // the projection needs no scratch beyond the status word
  (void)batch; (void)kv_heads; (void)seq; (void)vis_start; (void)vis_len; (void)device;
  return kStatusBytes;
}

size_t rtk_build_rotation_projected_workspace_size(int64_t batch, int64_t kv_heads, int64_t seq,
                                                   int64_t vis_start, int64_t vis_len, int32_t device) {
  (void)seq; (void)vis_start; (void)vis_len; (void)device;
  return rtk_build_rotation_workspace_size(batch, kv_heads, 128);
}

int rtk_build_rotation_projected(const rtk_tensor *hidden, const rtk_tensor *w_k, const rtk_tensor *bias,
                                 const rtk_tensor *cos, const rtk_tensor *sin, int64_t vis_start,
                                 int64_t vis_len, const rtk_tensor *queries, int64_t num_kv_groups,
                                 int64_t keep, const rtk_tensor *keys_out, const rtk_tensor *kept_out,
                                 const rtk_tensor *R_out, const rtk_tensor *delta_mu_out,
                                 const rtk_tensor *eigvals_out, void *workspace, size_t workspace_bytes,
                                 void *stream) {
  g_last_error.clear();
  if (keys_out == nullptr || keys_out->ndim != 4 || keys_out->shape[3] != 128)
    return fail(RTK_ERR_INVALID, "keys_out must be [B, H_kv, S, 128]");
  const int64_t B = keys_out->shape[0], H = keys_out->shape[1], S = keys_out->shape[2];
  if (vis_start < 0 || vis_len < 0 || vis_start + vis_len > S)
    return fail(RTK_ERR_INVALID, "the visual span [%lld, %lld) is not inside [0, %lld)", (long long)vis_start,
                (long long)(vis_start + vis_len), (long long)S);
  const int rc = check_build_args(B, H, vis_len, 128, keys_out->dtype, queries, num_kv_groups, keep, kept_out,
                                  R_out, delta_mu_out, eigvals_out);
  if (rc != RTK_OK) return rc;
  if (B * H == 0) return RTK_OK;
  const size_t build_bytes = rtk_build_rotation_workspace_size(B, H, 128);
  if (workspace == nullptr || workspace_bytes < build_bytes)
    return fail(RTK_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes,
                rtk_build_rotation_projected_workspace_size(B, H, S, vis_start, vis_len, current_device()));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const BuildWs w = build_ws(workspace, B * H, 128);
  // ---- K = RoPE(X W^T + b) for every token, with the visual span's sums
  const int prc = run_key_projection(hidden, w_k, bias, cos, sin, vis_start, vis_len, keys_out, w.cov, w.ksum,
                                     w.status, st);
  if (prc != RTK_OK) return prc;
  // ---- the rest of the build on the visual Keys just written
  View4 kv;
  as4(keys_out, kv);
  kv.data = static_cast<const unsigned char *>(keys_out->data) + vis_start * keys_out->stride[2] * 2;
  kv.n[2] = vis_len;
  return finish_build(kv, keys_out->dtype, queries, num_kv_groups, keep, kept_out, R_out, delta_mu_out,
                      eigvals_out, w, st);
}

int rtk_rotate_keys(const rtk_tensor *keys, const rtk_tensor *R, const rtk_tensor *kept_out, void *workspace,
                    size_t workspace_bytes, void *stream) {
  g_last_error.clear();
  View4 kv;
  if (!as4(keys, kv) || !dtype_ok(keys->dtype)) return fail(RTK_ERR_INVALID, "keys must be a [B, H, S, 128] float tensor");
  const int64_t B = kv.n[0], H = kv.n[1], S = kv.n[2], D = kv.n[3];
  if (D != 128) return fail(RTK_ERR_UNSUPPORTED, "head_dim must be 128 (got %lld)", (long long)D);
  if (R == nullptr || R->ndim != 4 || R->shape[0] != B || R->shape[1] != H || R->shape[2] != D ||
      R->dtype != keys->dtype)
    return fail(RTK_ERR_INVALID, "R must be [B, H, D, keep] in the Keys' dtype");
  const int64_t keep = R->shape[3];
  if (keep < 1 || keep > D) return fail(RTK_ERR_INVALID, "keep must be in [1, head_dim] (got %lld)", (long long)keep);
  if (!same_dims(kept_out, 4, {B, H, S, keep}) || kept_out->dtype != keys->dtype)
    return fail(RTK_ERR_INVALID, "kept_out must be [B, H, S, keep] in the Keys' dtype");
  if (workspace == nullptr || workspace_bytes < kStatusBytes)
    return fail(RTK_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes, kStatusBytes);
  if (B * H == 0) return RTK_OK;
  const cudaError_t e = launch_rotation(kv, keys->dtype, keep, R, kept_out, static_cast<unsigned int *>(workspace),
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rotate launch");
  return RTK_OK;
}

int rtk_eigh_topk(const rtk_tensor *cov, int64_t k, const rtk_tensor *vecs_out,
                  const rtk_tensor *vals_out, void *workspace, size_t workspace_bytes, void *stream) {
  g_last_error.clear();
  if (cov == nullptr || cov->ndim != 3 || cov->dtype != RTK_F32)
    return fail(RTK_ERR_INVALID, "cov must be a float32 [N, D, D]");
  const int64_t N = cov->shape[0], D = cov->shape[1];
  if (cov->shape[2] != D) return fail(RTK_ERR_INVALID, "cov must be a float32 [N, D, D]");
  if (D != 128) return fail(RTK_ERR_UNSUPPORTED, "the eigensolver supports D = 128 (got %lld)", (long long)D);
  if (cov->stride[2] != 1 || cov->stride[1] != D || cov->stride[0] != D * D)
    return fail(RTK_ERR_INVALID, "cov must be contiguous");
  if (k < 1 || k > D) return fail(RTK_ERR_INVALID, "k must be in [1, D] (got %lld)", (long long)k);
  if (!same_dims(vecs_out, 3, {N, D, k}) || vecs_out->dtype != RTK_F32)
    return fail(RTK_ERR_INVALID, "vecs_out must be a float32 [N, D, k]");
  if (vals_out != nullptr && (!same_dims(vals_out, 2, {N, D}) || vals_out->dtype != RTK_F32 ||
                              vals_out->stride[1] != 1 || vals_out->stride[0] != D))
    return fail(RTK_ERR_INVALID, "vals_out must be a contiguous float32 [N, D]");
  if (N == 0) return RTK_OK;
  const size_t need = rtk_eigh_topk_workspace_size(N);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(RTK_ERR_WORKSPACE, "workspace has %zu bytes, needs %zu", workspace_bytes, need);
  rtk::EighParams jp;
  std::memset(&jp, 0, sizeof(jp));
  jp.nmat = (int)N; jp.heads = 1;
  jp.cov = static_cast<const float *>(cov->data);
  jp.count = 1;
  jp.keep = (int)k;
  jp.R = vecs_out->data; jp.R_dtype = RTK_F32;
  jp.R_s[0] = vecs_out->stride[0]; jp.R_s[1] = 0; jp.R_s[2] = vecs_out->stride[1]; jp.R_s[3] = vecs_out->stride[2];
  jp.evals = vals_out ? static_cast<float *>(vals_out->data) : nullptr;
  const cudaError_t e = rtk::launch_eigh(jp, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "eigensolver launch");
  return RTK_OK;
}

int rtk_read_status(void *workspace, void *stream, uint32_t *status) {
  g_last_error.clear();
  if (workspace == nullptr || status == nullptr) return fail(RTK_ERR_INVALID, "workspace and status must be non-NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, workspace, sizeof(host), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemsetAsync(workspace, 0, sizeof(host), s);
  if (e != cudaSuccess) return cuda_fail(e, "rtk_read_status");
  *status = host;
  return RTK_OK;
}

}  // extern "C"
