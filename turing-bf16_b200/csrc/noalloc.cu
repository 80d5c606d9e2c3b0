// Allocation-free column quantisation: tbf16_quantize_cols with its scratch in a file-scope device array.
//
// Some callers cannot allocate device memory at the point where they call in: code running inside a
// custom memory arena that owns every device allocation, plugins of a host framework whose allocator
// is not reachable from the call site, or code on a path where a cudaMalloc would synchronise the
// device or break a latency budget. tbf16_quantize_cols needs a K-float workspace for the per-column
// maxima; this entry point takes the same inputs and outputs but keeps that workspace in the array
// below, so the caller passes only tensors it already owns.
//
// The array is a fixed 256 KB per GPU (kMaxCols floats), held by every GPU that loads the library until
// the process exits, and shared by every call on that GPU: calls that overlap on the GPU (different
// streams, no ordering between them) race on it. Each call clears the part it uses before use.
#include <mutex>

#include "common.cuh"

namespace {

constexpr int64_t kMaxCols = TBF16_NOALLOC_MAX_COLS;

// Column-maximum scratch. In host code this name is only a host-side stand-in for the device array, not
// a device address; the address comes from cudaGetSymbolAddress below, once per device.
static __device__ __align__(256) float g_col_amax_scratch[kMaxCols];

constexpr int kMaxDevices = 64;
float* g_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of the scratch array on the current device, resolved on the first call per device
// (with that device current). Returns nullptr if the address cannot be obtained.
float* scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    float* ptr = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_col_amax_scratch) != cudaSuccess || !ptr) {
      cudaGetLastError();
      return nullptr;
    }
    g_scratch_addr[dev] = ptr;
  }
  return g_scratch_addr[dev];
}

}  // namespace

extern "C" int tbf16_quantize_cols_noalloc(const void* x, int64_t rows, int64_t K, int64_t ldx, int target_exp,
                                           const float* row_mul, void* y16, int64_t ldy, float* s_inv, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (K < 0 || K > kMaxCols) return TBF16_ERR_INVALID;  // the fixed scratch holds at most kMaxCols columns
  float* scratch = scratch_for_current_device();
  if (!scratch) return TBF16_ERR_LAUNCH;
  // tbf16_quantize_cols zeroes the first K floats of its workspace (cudaMemsetAsync on the stream) before
  // the column maxima are merged into it, so no state carries over from the previous call.
  return tbf16_quantize_cols(x, rows, K, ldx, target_exp, row_mul, y16, ldy, s_inv, scratch, stream);
}
