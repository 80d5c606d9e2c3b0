// Few-row scaled linear for decode (M <= 8): y[m, n] = bf16((x[m] . w16[n]) * ws[n] + bias[n]), the
// reference's single-row path (tbf16/csrc/small_kernels.cu:107-132, tbf16/ops.py:207-218) with the
// same arithmetic: fp32 products of bf16 x and fp16 w, no activation scaling (fp32 holds any bf16
// product), one rounding to bf16 at the end. Rows 2..8 reuse every weight byte for all rows.
//
// HBM-bound on the weight (2 N K bytes). A block of 256 threads owns 4 weight rows (2 for M > 4) and
// splits K over all its threads: thread t streams the 16-byte vectors t, t + 256, ... of every row, up
// to 4 vectors per row in flight (8-16 loads per thread, issued before any arithmetic), so one block
// is one or two round trips to HBM. Partial sums (rows x M per thread) are reduced by a halving
// butterfly inside each warp (31 shuffles for 32 values instead of 5 per value), then across the 8
// warps through shared memory. x rows are small and stay in L1/L2.
#include "common.cuh"

using namespace tbf16;

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 4;    // 16-byte vectors per row in flight per thread
// One or two rows of x with K <= 4096 (at most 2 vectors per row per thread): 2 vectors in flight per row
// and three blocks per SM, so that a 4096-square weight (1024 blocks) runs in ~2.3 block rounds instead
// of ~3.5 (8.55 against 9.4 us for one row, 9.3 against 10.0 for two, graph-timed; four rows lose 8 %
// with the extra register pressure, and K = 8192 is unchanged).
constexpr int kShortKV = kThreads * 2;
// Weight rows per block: 4 up to 4 rows of x, 2 above (8 partial sums per thread at most 16 instead of
// 32, so that two blocks of 256 threads fit an SM without spilling).
__host__ __device__ constexpr int rows_for(int M) { return M <= 4 ? 4 : 2; }

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__host__ __device__ constexpr int pow2_at_least(int v) { return v <= 1 ? 1 : 2 * pow2_at_least((v + 1) / 2); }
__host__ __device__ constexpr int log2_exact(int v) { return v <= 1 ? 0 : 1 + log2_exact(v / 2); }

// Sums P values over the 32 lanes of a warp. Each step exchanges half of the remaining values with the
// partner lane (offset 16, 8, ...), so the count halves per step; once one value is left the remaining
// steps are plain xor sums. On return v[0] of lane L is the warp total of value (L >> (5 - log2 P)) & (P-1).
template <int P>
__device__ __forceinline__ void warp_reduce_halving(float (&v)[P], int lane) {
#pragma unroll
  for (int s = 0; s < 5; ++s) {
    const int o = 16 >> s;
    const int n = P >> s;  // values left before this step
    if (n > 1) {
      const int half = n / 2;
      const bool up = (lane & o) != 0;
#pragma unroll
      for (int j = 0; j < half; ++j) {
        const float send = up ? v[j] : v[j + half];
        const float keep = up ? v[j + half] : v[j];
        v[j] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
}

template <int M, int U>
__global__ void __launch_bounds__(kThreads, U == 2 ? 3 : 2) gemv_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                        const __half* __restrict__ w, int64_t ldw,
                                                        const float* __restrict__ ws,
                                                        const __nv_bfloat16* __restrict__ bias,
                                                        __nv_bfloat16* __restrict__ y, int64_t ldy, int N, int K) {
  constexpr int kRowsB = rows_for(M);
  constexpr int V = kRowsB * M;            // partial sums per thread: value r * M + m
  constexpr int P = pow2_at_least(V);      // padded to a power of two for the butterfly
  __shared__ float red[kWarps][P];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int n0 = blockIdx.x * kRowsB;
  float acc[P];
#pragma unroll
  for (int j = 0; j < P; ++j) acc[j] = 0.f;
  const __half* wr[kRowsB];
#pragma unroll
  for (int r = 0; r < kRowsB; ++r) wr[r] = w + (int64_t)min(n0 + r, N - 1) * ldw;
  const int kv = K / 8;  // 16-byte vectors per row
  for (int i0 = t; i0 < kv; i0 += kThreads * U) {
    uint4 wv[kRowsB][U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + kThreads * u;
#pragma unroll
      for (int r = 0; r < kRowsB; ++r) wv[r][u] = i < kv ? ld_stream(wr[r] + 8 * i) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + kThreads * u;
      if (i >= kv) break;
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + m * ldx) + i);
        const __nv_bfloat162* xb = reinterpret_cast<const __nv_bfloat162*>(&xv);
#pragma unroll
        for (int r = 0; r < kRowsB; ++r) {
          const __half2* wh = reinterpret_cast<const __half2*>(&wv[r][u]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 a = __bfloat1622float2(xb[j]), b = __half22float2(wh[j]);
            acc[r * M + m] = fmaf(a.x, b.x, fmaf(a.y, b.y, acc[r * M + m]));
          }
        }
      }
    }
  }
  warp_reduce_halving<P>(acc, lane);
  constexpr int kShift = 5 - log2_exact(P);
  if ((lane & ((1 << kShift) - 1)) == 0) red[warp][(lane >> kShift) & (P - 1)] = acc[0];
  __syncthreads();
  if (t < V) {
    const int r = t / M, m = t % M;
    const int n = n0 + r;
    if (n < N) {
      float v = 0.f;
#pragma unroll
      for (int k = 0; k < kWarps; ++k) v += red[k][t];
      v *= ws[n];
      if (bias) v += __bfloat162float(bias[n]);
      y[m * ldy + n] = __float2bfloat16_rn(v);
    }
  }
}

template <int M>
int launch_gemv(const void* x, int64_t ldx, const void* w16, int64_t ldw, const float* ws, const void* bias, void* y,
                int64_t ldy, int N, int K, cudaStream_t st) {
  const int blocks = (N + rows_for(M) - 1) / rows_for(M);
  auto* kern = gemv_kernel<M, kUnroll>;
  if constexpr (M <= 2)
    if (K / 8 <= kShortKV) kern = gemv_kernel<M, 2>;
  kern<<<blocks, kThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __half*>(w16), ldw,
                                    ws, static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(y), ldy,
                                    N, K);
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
