// Few-row scaled linear for decode (M <= 8): y[m, n] = bf16((x[m] . w16[n]) * ws[n] + bias[n]), the
// reference's single-row path (tbf16/csrc/small_kernels.cu:107-132, tbf16/ops.py:207-218) with the
// same arithmetic: fp32 products of bf16 x and fp16 w, no activation scaling (fp32 holds any bf16
// product), one rounding to bf16 at the end. Rows 2..8 reuse every weight byte for all rows.
//
// HBM-bound on the weight (2 N K bytes): each warp owns kRows output columns n and streams their
// weight rows in 16-byte vectors (8 halves per lane per step, several steps in flight); x rows are
// small and stay in L1/L2. Grid: enough warps to cover N, 8 warps per block.
#include "common.cuh"

using namespace tbf16;

namespace {

constexpr int kRows = 2;          // weight rows per warp
constexpr int kWarps = 8;         // warps per block
constexpr int kUnroll = 4;        // 16-byte steps per lane in flight per weight row

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <int M>
__global__ void __launch_bounds__(32 * kWarps) gemv_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                          const __half* __restrict__ w, int64_t ldw,
                                                          const float* __restrict__ ws,
                                                          const __nv_bfloat16* __restrict__ bias,
                                                          __nv_bfloat16* __restrict__ y, int64_t ldy, int N, int K) {
  const int lane = threadIdx.x & 31;
  const int n0 = (blockIdx.x * kWarps + (threadIdx.x >> 5)) * kRows;
  if (n0 >= N) return;
  float acc[kRows][M];
#pragma unroll
  for (int r = 0; r < kRows; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.f;
  const int kv = K / 8;  // 16-byte vectors per row
  const __half* wr[kRows];
#pragma unroll
  for (int r = 0; r < kRows; ++r) wr[r] = w + (int64_t)min(n0 + r, N - 1) * ldw;
  for (int i0 = lane; i0 < kv; i0 += 32 * kUnroll) {
    uint4 wv[kRows][kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = i0 + 32 * u;
#pragma unroll
      for (int r = 0; r < kRows; ++r) wv[r][u] = i < kv ? ld_stream(wr[r] + 8 * i) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = i0 + 32 * u;
      if (i >= kv) break;
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + m * ldx) + i);
        const __nv_bfloat162* xb = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          const __half2* wh = reinterpret_cast<const __half2*>(&wv[r][u]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 a = __bfloat1622float2(xb[j]), b = __half22float2(wh[j]);
            acc[r][m] = fmaf(a.x, b.x, fmaf(a.y, b.y, acc[r][m]));
          }
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kRows; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float v = acc[r][m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[r][m] = v;
    }
  if (lane < kRows * M) {
    const int r = lane / M, m = lane % M;
    const int n = n0 + r;
    float v = 0.f;
#pragma unroll
    for (int rr = 0; rr < kRows; ++rr)
#pragma unroll
      for (int mm = 0; mm < M; ++mm)
        if (rr == r && mm == m) v = acc[rr][mm];
    if (n < N) {
      v *= ws[n];
      if (bias) v += __bfloat162float(bias[n]);
      y[m * ldy + n] = __float2bfloat16_rn(v);
    }
  }
}

template <int M>
int launch_gemv(const void* x, int64_t ldx, const void* w16, int64_t ldw, const float* ws, const void* bias, void* y,
                int64_t ldy, int N, int K, cudaStream_t st) {
  const int warps = (N + kRows - 1) / kRows;
  const int blocks = (warps + kWarps - 1) / kWarps;
  gemv_kernel<M><<<blocks, 32 * kWarps, 0, st>>>(static_cast<const __nv_bfloat16*>(x), ldx,
                                                  static_cast<const __half*>(w16), ldw, ws,
                                                  static_cast<const __nv_bfloat16*>(bias),
                                                  static_cast<__nv_bfloat16*>(y), ldy, N, K);
  return tbf16_host::check_launch();
}

}  // namespace

extern "C" int tbf16_gemv(const void* x, int64_t M, int64_t K, int64_t ldx, const void* w16, int64_t N, int64_t ldw,
                          const float* ws, const void* bias, void* y, int64_t ldy, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (M < 0 || K < 0 || N < 0 || !x || !w16 || !ws || !y || ldx < K || ldw < K || ldy < N || N > INT32_MAX ||
      K > INT32_MAX)
    return TBF16_ERR_INVALID;
  if (M > TBF16_GEMV_MAX_ROWS) return TBF16_ERR_UNSUPPORTED;
  if (K % 8 || ldx % 8 || ldw % 8 || !tbf16_host::aligned16(x) || !tbf16_host::aligned16(w16)) return TBF16_ERR_ALIGN;
  if (M == 0 || N == 0) return TBF16_OK;
  auto st = static_cast<cudaStream_t>(stream);
  const int n = (int)N, k = (int)K;
  switch (M) {
    case 1: return launch_gemv<1>(x, ldx, w16, ldw, ws, bias, y, ldy, n, k, st);
    case 2: return launch_gemv<2>(x, ldx, w16, ldw, ws, bias, y, ldy, n, k, st);
    case 3: return launch_gemv<3>(x, ldx, w16, ldw, ws, bias, y, ldy, n, k, st);
    case 4: return launch_gemv<4>(x, ldx, w16, ldw, ws, bias, y, ldy, n, k, st);
    case 5: return launch_gemv<5>(x, ldx, w16, ldw, ws, bias, y, ldy, n, k, st);
    case 6: return launch_gemv<6>(x, ldx, w16, ldw, ws, bias, y, ldy, n, k, st);
    case 7: return launch_gemv<7>(x, ldx, w16, ldw, ws, bias, y, ldy, n, k, st);
    default: return launch_gemv<8>(x, ldx, w16, ldw, ws, bias, y, ldy, n, k, st);
  }
}
