// rtk_rotatek_decode_static: the fused RotateK decode without a caller-owned
// workspace.
//
// Some callers cannot hand this library any scratch memory: a serving runtime
// whose memory pool owns all of HBM and forbids outside cudaMalloc calls, a
// foreign-language binding that only forwards the pointers of tensors it was
// given, or a latency-critical step that must not enter cudaMalloc (which can
// synchronise the device).  For them this entry point keeps its scratch --
// the status word, the per-unit ticket counters and the split partials -- in
// one fixed device array defined below and allocates nothing.
//
// Limits and rules (also stated in include/rotatek_b200.h):
//  * The array holds kStaticScratchBytes (16 MiB).  Every GPU that loads the
//    library reserves it until the process exits.  Shapes whose decode needs
//    more scratch (rtk_rotatek_decode_workspace_size) are rejected with
//    RTK_ERR_WORKSPACE and a message giving both sizes.
//  * The first call on a device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current) and caches it; make that
//    first call before any stream capture.
//  * Every call on a device shares the one array and leaves its contents for
//    the next call; each call first clears the ticket counters, which must
//    start at zero (an async memset on the caller's stream).  Calls that
//    overlap on the GPU -- different streams without ordering -- race on the
//    array.
//  * The array's first 256 bytes are the device-status word of rtk_read_status
//    (RTK_DEVICE_TIMEOUT when a bounded wait gave up).  It is cleared once, by
//    the first call on the device, and then keeps what the calls set until
//    rtk_read_static_status reads and clears it.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/rotatek_b200.h"
#include "decode.h"

namespace {

constexpr size_t kStaticScratchBytes = 16u << 20;
constexpr int kMaxDevices = 64;

// The scratch itself.  In host code `g_static_scratch` only names the symbol;
// its device address comes from cudaGetSymbolAddress (per device).
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// The status word (and the counters after it) start at zero on each device.
constexpr size_t kStatusBytes = 256;

// Device address of the scratch on `device` (the current device), looked up
// once per device and cached.  The first lookup also clears the status word,
// on `stream`.
cudaError_t scratch_address(int device, cudaStream_t stream, void **out) {
  static std::mutex mu;
  static void *addr[kMaxDevices] = {nullptr};
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[device] == nullptr) {
    void *p = nullptr;
    cudaError_t err = cudaGetSymbolAddress(&p, g_static_scratch);
    if (err != cudaSuccess) return err;
    err = cudaMemsetAsync(p, 0, kStatusBytes, stream);
    if (err != cudaSuccess) return err;
    addr[device] = p;
  }
  *out = addr[device];
  return cudaSuccess;
}

int cuda_error(const char *what, cudaError_t err) {
  char buf[256];
  snprintf(buf, sizeof(buf), "rtk_rotatek_decode_static: %s: %s", what, cudaGetErrorString(err));
  return rtk::report_error(RTK_ERR_CUDA, buf);
}

}  // namespace

extern "C" int rtk_rotatek_decode_static(const rtk_tensor *q_full, const rtk_tensor *R_partial,
                                         const rtk_tensor *delta_mu, const rtk_tensor *k_full,
                                         const rtk_tensor *v_full, const rtk_tensor *mask_full,
                                         const rtk_tensor *k_sparse, const rtk_tensor *v_sparse,
                                         int64_t num_kv_groups, const rtk_tensor *out,
                                         void *stream) {
  // Shapes and dtypes are checked by the workspace entry point (no workspace
  // given: it validates, then stops at the workspace check without touching
  // the GPU).  Invalid input returns its error; an empty problem returns OK.
  const int pre = rtk_rotatek_decode(q_full, R_partial, delta_mu, k_full, v_full, mask_full,
                                     k_sparse, v_sparse, num_kv_groups, out, nullptr, 0, stream);
  if (pre != RTK_ERR_WORKSPACE) return pre;

  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return cuda_error("cudaGetDevice", err);
  const size_t need = rtk_rotatek_decode_workspace_size(
      q_full->dtype, q_full->shape[0], q_full->shape[1], R_partial->shape[1], q_full->shape[2],
      R_partial->shape[3], k_full->shape[2], k_sparse->shape[2], device);
  if (need > kStaticScratchBytes) {
    char buf[256];
    snprintf(buf, sizeof(buf),
             "rtk_rotatek_decode_static: these shapes need %zu bytes of scratch, the static "
             "scratch holds %zu; call rtk_rotatek_decode with a workspace instead",
             need, kStaticScratchBytes);
    return rtk::report_error(RTK_ERR_WORKSPACE, buf);
  }
  void *scratch = nullptr;
  err = scratch_address(device, static_cast<cudaStream_t>(stream), &scratch);
  if (err != cudaSuccess) return cuda_error("cudaGetSymbolAddress", err);
  // the ticket counters after the status word must start at zero; the status
  // word keeps what earlier calls set until rtk_read_static_status; the rest
  // is overwritten by the kernels
  size_t zero = rtk::decode_counter_bytes(q_full->shape[0], q_full->shape[1]);
  if (zero > need) zero = need;
  if (zero > kStatusBytes) {
    err = cudaMemsetAsync(static_cast<unsigned char *>(scratch) + kStatusBytes, 0, zero - kStatusBytes,
                          static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_error("clearing the counters", err);
  }
  return rtk_rotatek_decode(q_full, R_partial, delta_mu, k_full, v_full, mask_full, k_sparse,
                            v_sparse, num_kv_groups, out, scratch, kStaticScratchBytes, stream);
}

extern "C" int rtk_read_static_status(void *stream, uint32_t *status) {
  if (status == nullptr) return rtk::report_error(RTK_ERR_INVALID, "status must be non-NULL");
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return cuda_error("cudaGetDevice", err);
  void *scratch = nullptr;
  err = scratch_address(device, static_cast<cudaStream_t>(stream), &scratch);
  if (err != cudaSuccess) return cuda_error("cudaGetSymbolAddress", err);
  return rtk_read_status(scratch, stream, status);
}
