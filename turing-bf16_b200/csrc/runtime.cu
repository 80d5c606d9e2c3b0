// Library-level entry points and host helpers: ABI version, status strings, per-device info (SM
// count, compute capability, address of the device error word) and tensor-map encoding through the
// driver entry point (no link-time dependency on libcuda).
#include <mutex>

#include "common.cuh"

__device__ unsigned int g_tbf16_device_error = 0;

namespace tbf16_host {

namespace {
constexpr int kMaxDevices = 64;
DeviceInfo g_info[kMaxDevices];
std::mutex g_mu;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
}  // namespace

const DeviceInfo* device_info() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  DeviceInfo* d = &g_info[dev];
  if (d->device == dev) return d;
  std::lock_guard<std::mutex> lock(g_mu);
  if (d->device == dev) return d;
  DeviceInfo info;
  info.device = dev;
  if (cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&info.cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&info.cc_minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&info.err), g_tbf16_device_error) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  *d = info;
  return d;
}

int require_sm100() {
  const DeviceInfo* d = device_info();
  if (!d) return TBF16_ERR_DEVICE;
  return d->cc_major == 10 && d->cc_minor == 0 ? TBF16_OK : TBF16_ERR_DEVICE;
}

int check_launch() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TBF16_OK : TBF16_ERR_LAUNCH;
}

static EncodeTiledFn encode_fn() {
  if (!g_encode) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_encode) {
      void* fn = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
              cudaSuccess ||
          q != cudaDriverEntryPointSuccess || !fn) {
        cudaGetLastError();
        return nullptr;
      }
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
  }
  return g_encode;
}

int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols,
                 uint32_t box_rows) {
  if (!encode_fn()) return TBF16_ERR_LAUNCH;
  if (!aligned16(base) || (ld * 2) % 16 != 0) return TBF16_ERR_ALIGN;
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TBF16_OK : TBF16_ERR_INVALID;
}

int make_tmap_conv_in(CUtensorMap* map, const void* base, int64_t B, int64_t D, int64_t H, int64_t W, int64_t C,
                      int bx, int by) {
  if (!encode_fn()) return TBF16_ERR_LAUNCH;
  if (!aligned16(base) || C % 8 != 0) return TBF16_ERR_ALIGN;
  cuuint64_t gdim[5] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)D, (cuuint64_t)B};
  cuuint64_t gstride[4] = {(cuuint64_t)(C * 2), (cuuint64_t)(W * C * 2), (cuuint64_t)(H * W * C * 2),
                           (cuuint64_t)(D * H * W * C * 2)};
  cuuint32_t box[5] = {64, (cuuint32_t)bx, (cuuint32_t)by, 1, 1};
  cuuint32_t estride[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, const_cast<void*>(base), gdim, gstride, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TBF16_OK : TBF16_ERR_INVALID;
}

int make_tmap_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                 uint64_t stride2, uint32_t box0, uint32_t box1) {
  if (!encode_fn()) return TBF16_ERR_LAUNCH;
  if (!aligned16(base) || (stride1 * 2) % 16 != 0 || (stride2 * 2) % 16 != 0) return TBF16_ERR_ALIGN;
  cuuint64_t gdim[3] = {d0, d1, d2};
  cuuint64_t gstride[2] = {stride1 * 2, stride2 * 2};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), gdim, gstride, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TBF16_OK : TBF16_ERR_INVALID;
}

int make_tmap_2d_out(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols,
                     uint32_t box_rows) {
  if (!encode_fn()) return TBF16_ERR_LAUNCH;
  if (!aligned16(base) || (ld * 2) % 16 != 0 || box_cols * 2 != 64) return TBF16_ERR_ALIGN;
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TBF16_OK : TBF16_ERR_INVALID;
}

int make_tmap_3d_f32(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                     uint64_t stride2, uint32_t box0, uint32_t box1, int swizzle_bytes) {
  if (!encode_fn()) return TBF16_ERR_LAUNCH;
  if (swizzle_bytes != 64 && swizzle_bytes != 128) return TBF16_ERR_INVALID;
  if (!aligned16(base) || (stride1 * 4) % 16 != 0 || (stride2 * 4) % 16 != 0 || box0 * 4 > (uint32_t)swizzle_bytes)
    return TBF16_ERR_ALIGN;
  cuuint64_t gdim[3] = {d0, d1, d2};
  cuuint64_t gstride[2] = {stride1 * 4, stride2 * 4};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), gdim, gstride, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TBF16_OK : TBF16_ERR_INVALID;
}

}  // namespace tbf16_host

namespace {
using namespace tbf16;

// One warp waits, through the same bounded-wait helper every pipelined kernel uses, on an mbarrier that
// nothing arrives on. The wait gives up after timeout_ns, records kErrWaitTimeout in the device error
// word and the kernel returns: the failure path of a stalled pipeline, exercised without stalling one.
__global__ void bounded_wait_selftest_kernel(unsigned int* err, uint64_t timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  mbar_wait_warp(&bar, 0, &abort, err, timeout_ns);
}

}  // namespace

extern "C" {

int tbf16_abi_version(void) { return 100; }

const char* tbf16_status_string(int status) {
  switch (status) {
    case TBF16_OK: return "ok";
    case TBF16_ERR_INVALID: return "invalid argument (shape, stride or value)";
    case TBF16_ERR_ALIGN: return "pointer or leading dimension not aligned (16-byte rows, multiples of 8 elements)";
    case TBF16_ERR_DTYPE: return "unsupported dtype";
    case TBF16_ERR_LAUNCH: return "CUDA launch or runtime error";
    case TBF16_ERR_DEVICE: return "device is not an sm_100 GPU";
    case TBF16_ERR_UNSUPPORTED: return "not supported by this build";
    case TBF16_ERR_TIMEOUT: return "a kernel gave up on a bounded wait";
    default: return "unknown status";
  }
}

int tbf16_device_check(int device) {
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) { cudaGetLastError(); return TBF16_ERR_DEVICE; }
  if (cudaSetDevice(device) != cudaSuccess) { cudaGetLastError(); return TBF16_ERR_DEVICE; }
  int st = tbf16_host::require_sm100();
  cudaSetDevice(prev);
  return st;
}

int tbf16_selftest_bounded_wait(uint64_t timeout_ns, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (timeout_ns == 0 || timeout_ns > 1000000000ull) return TBF16_ERR_INVALID;
  const tbf16_host::DeviceInfo* d = tbf16_host::device_info();
  bounded_wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(d->err, timeout_ns);
  return tbf16_host::check_launch();
}

int tbf16_device_status(unsigned int* bits, int reset) {
  const tbf16_host::DeviceInfo* d = tbf16_host::device_info();
  if (!d || !bits) return TBF16_ERR_DEVICE;
  if (cudaDeviceSynchronize() != cudaSuccess) return TBF16_ERR_LAUNCH;
  if (cudaMemcpy(bits, d->err, sizeof(unsigned int), cudaMemcpyDeviceToHost) != cudaSuccess) return TBF16_ERR_LAUNCH;
  if (reset && cudaMemset(d->err, 0, sizeof(unsigned int)) != cudaSuccess) return TBF16_ERR_LAUNCH;
  if (reset && cudaDeviceSynchronize() != cudaSuccess) return TBF16_ERR_LAUNCH;
  return TBF16_OK;
}

}  // extern "C"
