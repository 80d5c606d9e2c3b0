// HBM-bound scale kernels: row amax -> exponent (+ optional fp16 materialisation), column scales,
// per-head amax / exponents, head scale-cast and the device-side prepare_qkv.
//
// All loads and stores are 128-bit (8 x 16-bit); rows, strides and base pointers are checked on the
// host for 16-byte alignment. Max reductions use fmaxf (NaN ignored, as the reference's kernels do);
// L1 norms accumulate in fp64 so that the exponent does not depend on the reduction order except
// when the sum lies within ~2^-45 (relative) of a power of two.
#include <algorithm>
#include <utility>

#include "common.cuh"

using namespace tbf16;

namespace {

constexpr int kRowWarps = 8;  // rows per 256-thread block (one warp per row)

// Max |x| (or L1 norm) of one bf16 row of K8 16-byte chunks, reduced over the warp.
template <bool L1>
__device__ __forceinline__ float warp_row_reduce(const uint4* __restrict__ xr, int K8, int lane) {
  float m = 0.f;
  double s = 0.0;
  int i = lane;
  for (; i + 96 < K8; i += 128) {  // four independent 16-byte loads in flight per lane
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldg(xr + i + 32 * u);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = fabsf(bf16lo(w[j])), b = fabsf(bf16hi(w[j]));
        if (L1) s += (double)a + (double)b;
        else m = fmaxf(m, fmaxf(a, b));
      }
    }
  }
  for (; i < K8; i += 32) {
    const uint4 v = __ldg(xr + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = fabsf(bf16lo(w[j])), b = fabsf(bf16hi(w[j]));
      if (L1) s += (double)a + (double)b;
      else m = fmaxf(m, fmaxf(a, b));
    }
  }
  if (L1) return (float)warp_sum(s);
  return warp_max(m);
}

// Fused-GEMM row scales (gemm_sm75.cu:27-47): s_inv = 1 / 2^(se - 127), se from the fused rule.
template <bool L1>
__global__ void __launch_bounds__(256) row_scale_kernel(const uint4* __restrict__ x, int64_t rows, int K8, int64_t ldx8,
                                                        int t, float* __restrict__ s_inv, int8_t* __restrict__ exp_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float red = warp_row_reduce<L1>(x + row * ldx8, K8, lane);
  if (lane == 0) {
    const int se = scale_biased_exp_fused(red, t);
    s_inv[row] = inv_pow2_from_biased(se);
    if (exp_out) exp_out[row] = (int8_t)(se - 127);
  }
}

// quantize_rows (small_kernels.cu:35-74) for long rows (two reads of the row): s from the small rule
// (or the fused rule); y = fp16_rn(x * s); s_inv = 1 / s.
template <bool L1, bool FUSED_RULE>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const uint4* __restrict__ x, int64_t rows, int K8,
                                                            int64_t ldx8, int t, uint4* __restrict__ y, int64_t ldy8,
                                                            float* __restrict__ s_inv, int8_t* __restrict__ exp_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint4* xr = x + row * ldx8;
  const float red = warp_row_reduce<L1>(xr, K8, lane);
  const int se = FUSED_RULE ? scale_biased_exp_fused(red, t) : scale_biased_exp_small(red, t);
  const float s = pow2_from_biased(se);
  uint4* yr = y + row * ldy8;
  for (int i = lane; i < K8; i += 32) {
    const uint4 v = __ldg(xr + i);
    uint4 o;
    o.x = pack_f16(bf16lo(v.x) * s, bf16hi(v.x) * s);
    o.y = pack_f16(bf16lo(v.y) * s, bf16hi(v.y) * s);
    o.z = pack_f16(bf16lo(v.z) * s, bf16hi(v.z) * s);
    o.w = pack_f16(bf16lo(v.w) * s, bf16hi(v.w) * s);
    yr[i] = o;
  }
  if (lane == 0) {
    s_inv[row] = inv_pow2_from_biased(se);
    if (exp_out) exp_out[row] = (int8_t)(se - 127);
  }
}

// Single-pass row kernel for rows of up to 32 * NCH 16-byte chunks: one warp per row, the whole row held
// in registers (all loads in flight at once), one HBM read. Computes the row max or L1 norm, the scale
// exponent by the fused rule (gemm_sm75.cu:19-23) or the small-kernel rule (small_kernels.cu:12-18),
// s_inv, optional int8 log2(s), and optionally y = fp16_rn(x * s) from the registers.
template <int NCH, bool L1, bool FUSED_RULE, bool WRITE_Y>
__global__ void __launch_bounds__(256) row_pass_kernel(const uint4* __restrict__ x, int64_t rows, int K8, int64_t ldx8,
                                                       int t, uint4* __restrict__ y, int64_t ldy8,
                                                       float* __restrict__ s_inv, int8_t* __restrict__ exp_out) {
  pdl_launch_dependents();  // the linear's skinny GEMM may start streaming its weight meanwhile
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint4* xr = x + row * ldx8;
  uint4 v[NCH];
#pragma unroll
  for (int u = 0; u < NCH; ++u) {
    const int i = lane + 32 * u;
    v[u] = i < K8 ? __ldg(xr + i) : make_uint4(0, 0, 0, 0);
  }
  float m = 0.f;
  double s4[4] = {0.0, 0.0, 0.0, 0.0};  // four independent fp64 chains (a single one is latency-bound)
#pragma unroll
  for (int u = 0; u < NCH; ++u) {
    const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = fabsf(bf16lo(w[j])), b = fabsf(bf16hi(w[j]));
      if (L1) s4[j] += (double)a + (double)b;
      else m = fmaxf(m, fmaxf(a, b));
    }
  }
  double s = (s4[0] + s4[1]) + (s4[2] + s4[3]);
  const float red = L1 ? (float)warp_sum(s) : warp_max(m);
  const int se = FUSED_RULE ? scale_biased_exp_fused(red, t) : scale_biased_exp_small(red, t);
  if (WRITE_Y) {
    const float sc = pow2_from_biased(se);
    uint4* yr = y + row * ldy8;
#pragma unroll
    for (int u = 0; u < NCH; ++u) {
      const int i = lane + 32 * u;
      if (i < K8) {
        uint4 o;
        o.x = pack_f16(bf16lo(v[u].x) * sc, bf16hi(v[u].x) * sc);
        o.y = pack_f16(bf16lo(v[u].y) * sc, bf16hi(v[u].y) * sc);
        o.z = pack_f16(bf16lo(v[u].z) * sc, bf16hi(v[u].z) * sc);
        o.w = pack_f16(bf16lo(v[u].w) * sc, bf16hi(v[u].w) * sc);
        yr[i] = o;
      }
    }
  }
  if (lane == 0) {
    s_inv[row] = inv_pow2_from_biased(se);
    if (exp_out) exp_out[row] = (int8_t)(se - 127);
  }
}

// The same for few long rows (decode and small batches) and for rows longer than 2048 elements: one
// 256-thread block per row, thread t holding the row's 16-byte chunks t, t + 256, ... in registers, so a
// 16-row linear input spreads over 16 SMs instead of two, each thread waits for at most NCH loads, and
// long rows need no more than 8 vectors a thread. The max (or fp64 L1 sum) is reduced over
// the warp, then over the 8 warps in a fixed order.
template <int NCH, bool L1, bool FUSED_RULE, bool WRITE_Y>
__global__ void __launch_bounds__(256) row_pass_block_kernel(const uint4* __restrict__ x, int K8, int64_t ldx8, int t,
                                                             uint4* __restrict__ y, int64_t ldy8,
                                                             float* __restrict__ s_inv, int8_t* __restrict__ exp_out) {
  pdl_launch_dependents();
  __shared__ float red_m[8];
  __shared__ double red_s[8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x;
  const uint4* xr = x + row * ldx8;
  uint4 v[NCH];
#pragma unroll
  for (int u = 0; u < NCH; ++u) {
    const int i = tid + 256 * u;
    v[u] = i < K8 ? __ldg(xr + i) : make_uint4(0, 0, 0, 0);
  }
  float m = 0.f;
  double s4[4] = {0.0, 0.0, 0.0, 0.0};  // four independent fp64 chains (a single one is latency-bound)
#pragma unroll
  for (int u = 0; u < NCH; ++u) {
    const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = fabsf(bf16lo(w[j])), b = fabsf(bf16hi(w[j]));
      if (L1) s4[j] += (double)a + (double)b;
      else m = fmaxf(m, fmaxf(a, b));
    }
  }
  double s = (s4[0] + s4[1]) + (s4[2] + s4[3]);
  if (L1) s = warp_sum(s);
  else m = warp_max(m);
  if (lane == 0) {
    red_m[warp] = m;
    red_s[warp] = s;
  }
  __syncthreads();
  float red;
  if (L1) {
    double tot = 0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += red_s[k];
    red = (float)tot;
  } else {
    red = red_m[0];
#pragma unroll
    for (int k = 1; k < 8; ++k) red = fmaxf(red, red_m[k]);
  }
  const int se = FUSED_RULE ? scale_biased_exp_fused(red, t) : scale_biased_exp_small(red, t);
  if (WRITE_Y) {
    const float sc = pow2_from_biased(se);
    uint4* yr = y + row * ldy8;
#pragma unroll
    for (int u = 0; u < NCH; ++u) {
      const int i = tid + 256 * u;
      if (i < K8) {
        uint4 o;
        o.x = pack_f16(bf16lo(v[u].x) * sc, bf16hi(v[u].x) * sc);
        o.y = pack_f16(bf16lo(v[u].y) * sc, bf16hi(v[u].y) * sc);
        o.z = pack_f16(bf16lo(v[u].z) * sc, bf16hi(v[u].z) * sc);
        o.w = pack_f16(bf16lo(v[u].w) * sc, bf16hi(v[u].w) * sc);
        yr[i] = o;
      }
    }
  }
  if (tid == 0) {
    s_inv[row] = inv_pow2_from_biased(se);
    if (exp_out) exp_out[row] = (int8_t)(se - 127);
  }
}

// A block per row up to this many rows (8 per block would leave SMs idle), and for every row count when
// the rows are longer than 2048 elements: the warp-per-row form then holds 16 or 32 vectors a lane (153
// to 255 registers, one block per SM, spills at 32) and took, over 8192 rows, 30.7 / 34.8 us at 4096
// columns and 51.2 / 65.5 us at 8192 (max rule with the fp16 copy / L1) against 26.6 / 28.7 and 45.1 /
// 47.1 us for a block per row.
constexpr int64_t kBlockRowsMax = 1024;
constexpr int kBlockRowsAnyK8 = 256;

template <bool L1, bool FUSED_RULE, bool WRITE_Y>
bool launch_row_pass_t(const void* x, int64_t rows, int K8, int64_t ldx8, int t, void* y, int64_t ldy8, float* s_inv,
                       int8_t* exp_out, cudaStream_t st) {
  const unsigned grid = (unsigned)((rows + kRowWarps - 1) / kRowWarps);
  const uint4* xp = static_cast<const uint4*>(x);
  uint4* yp = static_cast<uint4*>(y);
  if ((rows <= kBlockRowsMax || K8 > kBlockRowsAnyK8) && K8 > 256 && K8 <= 2048) {
    const unsigned g = (unsigned)rows;
#define TBF16_ROW_BLOCK(N) row_pass_block_kernel<N, L1, FUSED_RULE, WRITE_Y><<<g, 256, 0, st>>>(xp, K8, ldx8, t, yp, ldy8, s_inv, exp_out)
    if (K8 <= 512) TBF16_ROW_BLOCK(2);
    else if (K8 <= 1024) TBF16_ROW_BLOCK(4);
    else TBF16_ROW_BLOCK(8);
#undef TBF16_ROW_BLOCK
    return true;
  }
#define TBF16_ROW_PASS(N) row_pass_kernel<N, L1, FUSED_RULE, WRITE_Y><<<grid, 256, 0, st>>>(xp, rows, K8, ldx8, t, yp, ldy8, s_inv, exp_out)
  if (K8 <= 32) TBF16_ROW_PASS(1);
  else if (K8 <= 64) TBF16_ROW_PASS(2);
  else if (K8 <= 128) TBF16_ROW_PASS(4);
  else if (K8 <= 256) TBF16_ROW_PASS(8);
  else if (K8 <= 512) TBF16_ROW_PASS(16);
  else if (K8 <= 1024) TBF16_ROW_PASS(32);
  else return false;
#undef TBF16_ROW_PASS
  return true;
}

}  // namespace

namespace tbf16_host {
int row_pass(const void* x, int64_t rows, int64_t K, int64_t ldx, int t, int l1, int fused_rule, void* y, int64_t ldy,
             float* s_inv, int8_t* exp_out, cudaStream_t st) {
  const int K8 = (int)(K / 8);
  const unsigned grid = (unsigned)((rows + kRowWarps - 1) / kRowWarps);
  const uint4* xp = static_cast<const uint4*>(x);
  uint4* yp = static_cast<uint4*>(y);
  bool done;
  if (y) {
    done = l1 ? (fused_rule ? launch_row_pass_t<true, true, true>(x, rows, K8, ldx / 8, t, y, ldy / 8, s_inv, exp_out, st)
                            : launch_row_pass_t<true, false, true>(x, rows, K8, ldx / 8, t, y, ldy / 8, s_inv, exp_out, st))
              : (fused_rule ? launch_row_pass_t<false, true, true>(x, rows, K8, ldx / 8, t, y, ldy / 8, s_inv, exp_out, st)
                            : launch_row_pass_t<false, false, true>(x, rows, K8, ldx / 8, t, y, ldy / 8, s_inv, exp_out, st));
    if (!done) {  // rows longer than 8192 elements: two reads of the row
      const int64_t ldx8 = ldx / 8, ldy8 = ldy / 8;
      if (l1 && fused_rule) quantize_rows_kernel<true, true><<<grid, 256, 0, st>>>(xp, rows, K8, ldx8, t, yp, ldy8, s_inv, exp_out);
      else if (l1) quantize_rows_kernel<true, false><<<grid, 256, 0, st>>>(xp, rows, K8, ldx8, t, yp, ldy8, s_inv, exp_out);
      else if (fused_rule) quantize_rows_kernel<false, true><<<grid, 256, 0, st>>>(xp, rows, K8, ldx8, t, yp, ldy8, s_inv, exp_out);
      else quantize_rows_kernel<false, false><<<grid, 256, 0, st>>>(xp, rows, K8, ldx8, t, yp, ldy8, s_inv, exp_out);
    }
  } else {
    if (!fused_rule) return TBF16_ERR_UNSUPPORTED;
    done = l1 ? launch_row_pass_t<true, true, false>(x, rows, K8, ldx / 8, t, nullptr, 0, s_inv, exp_out, st)
              : launch_row_pass_t<false, true, false>(x, rows, K8, ldx / 8, t, nullptr, 0, s_inv, exp_out, st);
    if (!done) {
      if (l1) row_scale_kernel<true><<<grid, 256, 0, st>>>(xp, rows, K8, ldx / 8, t, s_inv, exp_out);
      else row_scale_kernel<false><<<grid, 256, 0, st>>>(xp, rows, K8, ldx / 8, t, s_inv, exp_out);
    }
  }
  return check_launch();
}
}  // namespace tbf16_host

namespace {

constexpr int kColUnroll = 8;  // rows in flight per thread in the column kernels

// Column amax (small_kernels.cu:136-155): a block owns 32 column vectors (256 columns, 512 contiguous
// bytes of each row per warp) over a chunk of rows; its 8 warps take every 8th row of the chunk with
// kColUnroll rows in flight per thread, reduce their maxima through shared memory, and one atomicMax
// per column and block (on the bits of the non-negative maxima) merges the chunks. Same-address
// atomics are what limits a column reduction, so there are few of them.
__global__ void __launch_bounds__(256) col_amax_kernel(const uint4* __restrict__ x, const float* __restrict__ row_mul,
                                                       float* __restrict__ amax, int64_t R, int K8, int64_t ldx8,
                                                       int64_t rows_per_chunk) {
  __shared__ float red[8][32][9];  // [warp][lane][column of the vector], padded against bank conflicts
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c8 = blockIdx.x * 32 + lane;
  const bool cok = c8 < K8;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_chunk;
  const int64_t r1 = min(R, r0 + rows_per_chunk);
  float m[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  auto fold = [&](const uint4& v, float rm) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      m[2 * j] = fmaxf(m[2 * j], fabsf(bf16lo(w[j])) * rm);
      m[2 * j + 1] = fmaxf(m[2 * j + 1], fabsf(bf16hi(w[j])) * rm);
    }
  };
  if (cok) {
    int64_t r = r0 + warp;
    for (; r + 8 * (kColUnroll - 1) < r1; r += 8 * kColUnroll) {
      uint4 v[kColUnroll];
      float rm[kColUnroll];
#pragma unroll
      for (int u = 0; u < kColUnroll; ++u) {
        v[u] = __ldg(x + (r + 8 * u) * ldx8 + c8);
        rm[u] = row_mul ? fabsf(__ldg(row_mul + r + 8 * u)) : 1.f;
      }
#pragma unroll
      for (int u = 0; u < kColUnroll; ++u) fold(v[u], rm[u]);
    }
    for (; r < r1; r += 8) fold(__ldg(x + r * ldx8 + c8), row_mul ? fabsf(__ldg(row_mul + r)) : 1.f);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[warp][lane][j] = m[j];
  __syncthreads();
  // thread (w, l) reduces column j = w of vector l over the 8 warps
  const int j = warp;
  float v = red[0][lane][j];
#pragma unroll
  for (int k = 1; k < 8; ++k) v = fmaxf(v, red[k][lane][j]);
  if (cok) atomicMax(reinterpret_cast<int*>(amax) + c8 * 8 + j, __float_as_int(v));
}

// Column convert (small_kernels.cu:158-184): y = fp16_rn((x * row_mul[r]) * s[c]). Same layout as
// col_amax_kernel: a thread's 8 column scales are built once, then kColUnroll rows are converted per
// step; the first chunk's threads write s_inv.
__global__ void __launch_bounds__(256) col_convert_kernel(const uint4* __restrict__ x, const float* __restrict__ row_mul,
                                                          const float* __restrict__ amax, uint4* __restrict__ y,
                                                          float* __restrict__ s_inv, int64_t R, int K8, int64_t ldx8,
                                                          int64_t ldy8, int t, int64_t rows_per_chunk) {
  const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
  if (c8 >= K8) return;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_chunk;
  const int64_t r1 = min(R, r0 + rows_per_chunk);
  float s[8];
  int se[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    se[j] = scale_biased_exp_small(__ldg(amax + c8 * 8 + j), t);
    s[j] = pow2_from_biased(se[j]);
  }
  if (blockIdx.y == 0) {
#pragma unroll
    for (int j = 0; j < 8; ++j) s_inv[c8 * 8 + j] = inv_pow2_from_biased(se[j]);
  }
  auto conv = [&](const uint4& v, float rm) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = pack_f16(bf16lo(w[j]) * rm * s[2 * j], bf16hi(w[j]) * rm * s[2 * j + 1]);
    return make_uint4(o[0], o[1], o[2], o[3]);
  };
  int64_t r = r0;
  for (; r + kColUnroll <= r1; r += kColUnroll) {
    uint4 v[kColUnroll];
    float rm[kColUnroll];
#pragma unroll
    for (int u = 0; u < kColUnroll; ++u) {
      v[u] = __ldg(x + (r + u) * ldx8 + c8);
      rm[u] = row_mul ? __ldg(row_mul + r + u) : 1.f;
    }
#pragma unroll
    for (int u = 0; u < kColUnroll; ++u) y[(r + u) * ldy8 + c8] = conv(v[u], rm[u]);
  }
  for (; r < r1; ++r) y[r * ldy8 + c8] = conv(__ldg(x + r * ldx8 + c8), row_mul ? __ldg(row_mul + r) : 1.f);
}

__global__ void fill_kernel(float* p, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = v;
}

// ---------------------------------------------------------------- attention scale helpers

struct Head4 {
  const uint16_t* x;
  int64_t sb, sh, ss;  // element strides
  int H, S, D8;
  float* amax;         // [B*H]
  int is_f16;
  int nbh;             // B*H (set by the launcher)
};

__device__ __forceinline__ void unpack8(const uint4 v, int is_f16, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = is_f16 ? f16lo(w[j]) : bf16lo(w[j]);
    f[2 * j + 1] = is_f16 ? f16hi(w[j]) : bf16hi(w[j]);
  }
}
__device__ __forceinline__ void load8(const uint16_t* p, int is_f16, float (&f)[8]) {
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    f[2 * j] = is_f16 ? f16lo(w[j]) : bf16lo(w[j]);
    f[2 * j + 1] = is_f16 ? f16hi(w[j]) : bf16hi(w[j]);
  }
}

// grid (B*H, chunks, ntensors): amax of each (b, h) slice, merged with atomicMax (small_kernels.cu:221-243).
__global__ void __launch_bounds__(256) head_amax_kernel(Head4 t0, Head4 t1, Head4 t2, int rows_per_chunk) {
  const Head4 t = blockIdx.z == 0 ? t0 : blockIdx.z == 1 ? t1 : t2;
  const int bh = blockIdx.x;
  const int b = bh / t.H, h = bh % t.H;
  const int s0 = blockIdx.y * rows_per_chunk;
  const int s1 = min(t.S, s0 + rows_per_chunk);
  const uint16_t* base = t.x + b * t.sb + h * t.sh;
  float m = 0.f;
  const int n = (s1 - s0) * t.D8;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int s = s0 + i / t.D8, d = (i % t.D8) * 8;
    float f[8];
    load8(base + s * t.ss + d, t.is_f16, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(f[j]));
  }
  __shared__ float red[8];
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) atomicMax(reinterpret_cast<int*>(t.amax) + bh, __float_as_int(v));
  }
}

__global__ void head_exp_kernel(const float* __restrict__ amax, int32_t* __restrict__ e, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) e[i] = frexp_exp(amax[i]);
}

// prepare_qkv exponents (attention.py:41-46), one block: eq, ek = max frexp exponents over (b, h);
// a = clamp(floor((ek - eq) / 2), ek - 14, 14 - eq); ev = frexp(amax_v) - v_exp.
__global__ void __launch_bounds__(256) qkv_exponents_kernel(const float* __restrict__ amax_q, int nq,
                                                            const float* __restrict__ amax_k, int nk,
                                                            const float* __restrict__ amax_v, int v_exp,
                                                            int32_t* __restrict__ a_out, int32_t* __restrict__ ev_out) {
  __shared__ int red[2][8];
  int eq = INT_MIN, ek = INT_MIN;
  for (int i = threadIdx.x; i < nq; i += blockDim.x) eq = max(eq, frexp_exp(amax_q[i]));
  for (int i = threadIdx.x; i < nk; i += blockDim.x) {
    ek = max(ek, frexp_exp(amax_k[i]));
    ev_out[i] = frexp_exp(amax_v[i]) - v_exp;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    eq = max(eq, __shfl_xor_sync(0xffffffffu, eq, o));
    ek = max(ek, __shfl_xor_sync(0xffffffffu, ek, o));
  }
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = eq;
    red[1][threadIdx.x >> 5] = ek;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)blockDim.x / 32; ++w) {
      eq = max(eq, red[0][w]);
      ek = max(ek, red[1][w]);
    }
    eq = max(eq, red[0][0]);
    ek = max(ek, red[1][0]);
    int a = ek - eq;
    a = (a >= 0) ? a / 2 : -((-a + 1) / 2);  // floor division by 2
    a = max(min(a, 14 - eq), ek - 14);
    *a_out = a;
  }
}

// Sharded attention, phase 1: this rank's eq, ek (max frexp exponents of its q and k head maxima).
__global__ void __launch_bounds__(256) qk_max_exponents_kernel(const float* __restrict__ amax_q, int nq,
                                                               const float* __restrict__ amax_k, int nk,
                                                               int32_t* __restrict__ eqk) {
  __shared__ int red[2][8];
  int eq = INT_MIN, ek = INT_MIN;
  for (int i = threadIdx.x; i < nq; i += blockDim.x) eq = max(eq, frexp_exp(amax_q[i]));
  for (int i = threadIdx.x; i < nk; i += blockDim.x) ek = max(ek, frexp_exp(amax_k[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    eq = max(eq, __shfl_xor_sync(0xffffffffu, eq, o));
    ek = max(ek, __shfl_xor_sync(0xffffffffu, ek, o));
  }
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = eq;
    red[1][threadIdx.x >> 5] = ek;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)blockDim.x / 32; ++w) {
      red[0][0] = max(red[0][0], red[0][w]);
      red[1][0] = max(red[1][0], red[1][w]);
    }
    eqk[0] = red[0][0];
    eqk[1] = red[1][0];
  }
}

// Sharded attention, phase 2: a from the all-reduced eq, ek (the rule of qkv_exponents_kernel), and ev
// from this rank's v head maxima.
__global__ void __launch_bounds__(256) qkv_exponents_global_kernel(const int32_t* __restrict__ eqk,
                                                                   const float* __restrict__ amax_v, int nk, int v_exp,
                                                                   int32_t* __restrict__ a_out,
                                                                   int32_t* __restrict__ ev_out) {
  for (int i = threadIdx.x; i < nk; i += blockDim.x) ev_out[i] = frexp_exp(amax_v[i]) - v_exp;
  if (threadIdx.x == 0) {
    const int eq = eqk[0], ek = eqk[1];
    int a = ek - eq;
    a = (a >= 0) ? a / 2 : -((-a + 1) / 2);  // floor division by 2
    a = max(min(a, 14 - eq), ek - 14);
    *a_out = a;
  }
}

struct ScaleCast {
  const uint16_t* x;
  int64_t sb, sh, ss;
  int H, S, D8;
  const int32_t* e;      // exponent source
  int64_t e_sb, e_sh;    // broadcast strides into e
  int e_sign;            // multiply the exponent by this (+1 / -1)
  uint16_t* y;           // contiguous (B, H, S, D)
  int in_f16, out_f16;
  int64_t total8;        // B*H*S*D/8
};

// y = cast(x * 2^(sign * e[b, h])), contiguous output (small_kernels.cu:246-263). grid.z selects the tensor.
__global__ void __launch_bounds__(256) head_scale_cast_kernel(ScaleCast c0, ScaleCast c1, ScaleCast c2) {
  const ScaleCast c = blockIdx.z == 0 ? c0 : blockIdx.z == 1 ? c1 : c2;
  if (c.x == nullptr) return;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < c.total8; i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % c.D8) * 8;
    const int64_t row = i / c.D8;
    const int s = (int)(row % c.S);
    const int64_t bh = row / c.S;
    const int b = (int)(bh / c.H), h = (int)(bh % c.H);
    const float sc = exp2i(c.e_sign * __ldg(c.e + b * c.e_sb + h * c.e_sh));
    float f[8];
    load8(c.x + b * c.sb + h * c.sh + (int64_t)s * c.ss + d, c.in_f16, f);
    uint4 o;
    if (c.out_f16) {
      o.x = pack_f16(f[0] * sc, f[1] * sc); o.y = pack_f16(f[2] * sc, f[3] * sc);
      o.z = pack_f16(f[4] * sc, f[5] * sc); o.w = pack_f16(f[6] * sc, f[7] * sc);
    } else {
      o.x = pack_bf16(f[0] * sc, f[1] * sc); o.y = pack_bf16(f[2] * sc, f[3] * sc);
      o.z = pack_bf16(f[4] * sc, f[5] * sc); o.w = pack_bf16(f[6] * sc, f[7] * sc);
    }
    reinterpret_cast<uint4*>(c.y)[i] = o;
  }
}

// Row-structured forms for head dims of 64, 128 and 256 (D8 = D / 8 sixteen-byte chunks per row, a power of
// two dividing the block): a block owns one (b, h) slice and a range of rows, thread t handles chunk t % D8
// of rows t / D8, t / D8 + 256 / D8, ... -- no 64-bit division per chunk, one exponent per block, and
// consecutive threads touch consecutive 16-byte chunks. grid (row blocks, B*H of the widest tensor, tensors).
template <int D8>
__global__ void __launch_bounds__(256) head_amax_rows_kernel(Head4 t0, Head4 t1, Head4 t2, int rows_per_block) {
  const Head4 t = blockIdx.z == 0 ? t0 : blockIdx.z == 1 ? t1 : t2;
  const int bh = blockIdx.y;
  const int s0 = blockIdx.x * rows_per_block;
  const int s1 = min(t.S, s0 + rows_per_block);
  if (bh >= t.nbh || s0 >= s1) return;  // the grid covers the widest tensor
  const int b = bh / t.H, h = bh % t.H;
  const uint16_t* base = t.x + b * t.sb + h * t.sh + (threadIdx.x % D8) * 8;
  constexpr int RS = 256 / D8;  // rows a block covers per step
  float m = 0.f;
  int s = s0 + (int)threadIdx.x / D8;
  for (; s < s1; s += 8 * RS) {  // up to eight independent 16-byte loads in flight per thread
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      v[u] = s + u * RS < s1 ? __ldg(reinterpret_cast<const uint4*>(base + (int64_t)(s + u * RS) * t.ss))
                             : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      float f[8];
      unpack8(v[u], t.is_f16, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(f[j]));
    }
  }
  __shared__ float red[8];
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) atomicMax(reinterpret_cast<int*>(t.amax) + bh, __float_as_int(v));
  }
}

template <int D8>
__global__ void __launch_bounds__(256) head_scale_cast_rows_kernel(ScaleCast c0, ScaleCast c1, ScaleCast c2,
                                                                   int rows_per_block) {
  const ScaleCast c = blockIdx.z == 0 ? c0 : blockIdx.z == 1 ? c1 : c2;
  const int bh = blockIdx.y;
  if (c.x == nullptr || (int64_t)bh * c.S * D8 >= c.total8) return;  // this tensor has fewer (b, h) slices
  const int b = bh / c.H, h = bh % c.H;
  const int s0 = blockIdx.x * rows_per_block;
  const int s1 = min(c.S, s0 + rows_per_block);
  const float sc = exp2i(c.e_sign * __ldg(c.e + b * c.e_sb + h * c.e_sh));
  const int sub = (int)threadIdx.x % D8;
  const uint16_t* src = c.x + b * c.sb + h * c.sh + sub * 8;
  uint4* dst = reinterpret_cast<uint4*>(c.y) + (int64_t)bh * c.S * D8 + sub;
  auto convert = [&](const uint4 v) -> uint4 {
    float f[8];
    unpack8(v, c.in_f16, f);
    uint4 o;
    if (c.out_f16) {
      o.x = pack_f16(f[0] * sc, f[1] * sc); o.y = pack_f16(f[2] * sc, f[3] * sc);
      o.z = pack_f16(f[4] * sc, f[5] * sc); o.w = pack_f16(f[6] * sc, f[7] * sc);
    } else {
      o.x = pack_bf16(f[0] * sc, f[1] * sc); o.y = pack_bf16(f[2] * sc, f[3] * sc);
      o.z = pack_bf16(f[4] * sc, f[5] * sc); o.w = pack_bf16(f[6] * sc, f[7] * sc);
    }
    return o;
  };
  constexpr int RS = 256 / D8;  // rows a block covers per step
  int s = s0 + (int)threadIdx.x / D8;
  for (; s < s1; s += 8 * RS) {  // up to eight independent 16-byte loads in flight per thread
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (s + u * RS < s1) v[u] = __ldg(reinterpret_cast<const uint4*>(src + (int64_t)(s + u * RS) * c.ss));
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (s + u * RS < s1) dst[(int64_t)(s + u * RS) * D8] = convert(v[u]);
  }
}

bool ok8(int64_t v) { return v % 8 == 0; }

int grid_for(int64_t work, int threads, int waves = 8) {
  const tbf16_host::DeviceInfo* d = tbf16_host::device_info();
  const int64_t cap = (int64_t)(d ? d->sms : 148) * waves;
  const int64_t g = (work + threads - 1) / threads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(g, cap));
}

int check_4d(const void* x, int64_t B, int64_t H, int64_t S, int64_t D, int64_t sb, int64_t sh, int64_t ss) {
  if (B < 0 || H < 0 || S < 0 || D <= 0 || B * H > INT32_MAX || S > INT32_MAX) return TBF16_ERR_INVALID;
  if (!ok8(D) || !ok8(sb) || !ok8(sh) || !ok8(ss) || !tbf16_host::aligned16(x)) return TBF16_ERR_ALIGN;
  return TBF16_OK;
}

Head4 make_head4(const void* x, int64_t H, int64_t S, int64_t D, int64_t sb, int64_t sh, int64_t ss, float* amax,
                 int is_f16) {
  Head4 h;
  h.x = static_cast<const uint16_t*>(x);
  h.sb = sb; h.sh = sh; h.ss = ss;
  h.H = (int)H; h.S = (int)S; h.D8 = (int)(D / 8);
  h.amax = amax;
  h.is_f16 = is_f16;
  return h;
}

int launch_head_amax(Head4 a, Head4 b, Head4 c, int ntensors, int64_t BH, int64_t S, cudaStream_t st) {
  const tbf16_host::DeviceInfo* d = tbf16_host::device_info();
  const int sms = d ? d->sms : 148;
  const int chunks = (int)std::max<int64_t>(1, std::min<int64_t>((sms * 8 + BH - 1) / BH, (S + 63) / 64));
  const int rows = (int)((S + chunks - 1) / chunks);
  a.nbh = b.nbh = c.nbh = (int)BH;
  const int D8 = a.D8;
  if (BH <= 65535 && (D8 == 8 || D8 == 16 || D8 == 32)) {  // row-structured form for head dims 64 / 128 / 256
    const dim3 grid(chunks, (unsigned)BH, ntensors);
    if (D8 == 8) head_amax_rows_kernel<8><<<grid, 256, 0, st>>>(a, b, c, rows);
    else if (D8 == 16) head_amax_rows_kernel<16><<<grid, 256, 0, st>>>(a, b, c, rows);
    else head_amax_rows_kernel<32><<<grid, 256, 0, st>>>(a, b, c, rows);
    return tbf16_host::check_launch();
  }
  head_amax_kernel<<<dim3((unsigned)BH, chunks, ntensors), 256, 0, st>>>(a, b, c, rows);
  return tbf16_host::check_launch();
}

// Head maxima of q (B*Hq slices of Sq rows) and of k and v (B*Hkv slices of Sk rows each): one launch of
// the row-structured kernel over the three when it applies (blocks past a tensor's own slices or rows
// return at once; the maxima are atomicMax over row blocks, so the chunking does not change them), else
// one launch for q and one for k and v.
int launch_head_amax_qkv(Head4 hq, Head4 hk, Head4 hv, int64_t BHq, int64_t Sq, int64_t BHk, int64_t Sk,
                         cudaStream_t st) {
  const int64_t BH = std::max(BHq, BHk), S = std::max(Sq, Sk);
  const int D8 = hq.D8;
  if (Sq > 0 && Sk > 0 && BH <= 65535 && (D8 == 8 || D8 == 16 || D8 == 32)) {
    const tbf16_host::DeviceInfo* d = tbf16_host::device_info();
    const int sms = d ? d->sms : 148;
    const int chunks = (int)std::max<int64_t>(1, std::min<int64_t>((sms * 8 + BH - 1) / BH, (S + 63) / 64));
    const int rows = (int)((S + chunks - 1) / chunks);
    hq.nbh = (int)BHq;
    hk.nbh = hv.nbh = (int)BHk;
    const dim3 grid(chunks, (unsigned)BH, 3);
    if (D8 == 8) head_amax_rows_kernel<8><<<grid, 256, 0, st>>>(hq, hk, hv, rows);
    else if (D8 == 16) head_amax_rows_kernel<16><<<grid, 256, 0, st>>>(hq, hk, hv, rows);
    else head_amax_rows_kernel<32><<<grid, 256, 0, st>>>(hq, hk, hv, rows);
    return tbf16_host::check_launch();
  }
  if (Sq > 0)
    if (int rc = launch_head_amax(hq, hq, hq, 1, BHq, Sq, st)) return rc;
  if (Sk > 0)
    if (int rc = launch_head_amax(hk, hv, hv, 2, BHk, Sk, st)) return rc;
  return TBF16_OK;
}

// Launches the scale-cast of up to three tensors (same head dim): the row-structured form for D8 in
// {8, 16, 32}, the flat form otherwise. max_bh / max_s: the widest tensor's B*H and S.
int launch_scale_cast(const ScaleCast& c0, const ScaleCast& c1, const ScaleCast& c2, int ntensors, int64_t max_bh,
                      int64_t max_s, int64_t max_total8, cudaStream_t st) {
  const int D8 = c0.D8;
  if (max_bh <= 65535 && (D8 == 8 || D8 == 16 || D8 == 32)) {
    const tbf16_host::DeviceInfo* d = tbf16_host::device_info();
    const int sms = d ? d->sms : 148;
    // about 8 blocks per SM over the launch, at least 64 rows a block
    const int64_t chunks = std::max<int64_t>(1, std::min<int64_t>((sms * 8 + max_bh - 1) / max_bh, (max_s + 63) / 64));
    const int rows = (int)((max_s + chunks - 1) / chunks);
    const dim3 grid((unsigned)chunks, (unsigned)max_bh, ntensors);
    if (D8 == 8) head_scale_cast_rows_kernel<8><<<grid, 256, 0, st>>>(c0, c1, c2, rows);
    else if (D8 == 16) head_scale_cast_rows_kernel<16><<<grid, 256, 0, st>>>(c0, c1, c2, rows);
    else head_scale_cast_rows_kernel<32><<<grid, 256, 0, st>>>(c0, c1, c2, rows);
    return tbf16_host::check_launch();
  }
  head_scale_cast_kernel<<<dim3(grid_for(max_total8, 256), 1, ntensors), 256, 0, st>>>(c0, c1, c2);
  return tbf16_host::check_launch();
}

// q16 = fp16(q * 2^a), k16 = fp16(k * 2^-a), v16 = fp16(v * 2^-ev[b, hk]): one launch for the three.
int scale_qkv(const void* q, int64_t qsb, int64_t qsh, int64_t qss, const void* k, int64_t ksb, int64_t ksh,
              int64_t kss, const void* v, int64_t vsb, int64_t vsh, int64_t vss, int64_t B, int64_t Hq, int64_t Hkv,
              int64_t Sq, int64_t Sk, int64_t D, void* q16, void* k16, void* v16, const int32_t* a,
              const int32_t* ev, cudaStream_t st) {
  ScaleCast cq;
  cq.x = static_cast<const uint16_t*>(q); cq.sb = qsb; cq.sh = qsh; cq.ss = qss;
  cq.H = (int)Hq; cq.S = (int)Sq; cq.D8 = (int)(D / 8);
  cq.e = a; cq.e_sb = 0; cq.e_sh = 0; cq.e_sign = 1;
  cq.y = static_cast<uint16_t*>(q16); cq.in_f16 = 0; cq.out_f16 = 1; cq.total8 = B * Hq * Sq * D / 8;
  ScaleCast ck = cq;
  ck.x = static_cast<const uint16_t*>(k); ck.sb = ksb; ck.sh = ksh; ck.ss = kss;
  ck.H = (int)Hkv; ck.S = (int)Sk; ck.e_sign = -1; ck.y = static_cast<uint16_t*>(k16); ck.total8 = B * Hkv * Sk * D / 8;
  ScaleCast cv = ck;
  cv.x = static_cast<const uint16_t*>(v); cv.sb = vsb; cv.sh = vsh; cv.ss = vss;
  cv.e = ev; cv.e_sb = Hkv; cv.e_sh = 1; cv.y = static_cast<uint16_t*>(v16);
  const int64_t work = std::max(cq.total8, ck.total8);
  if (work > 0) return launch_scale_cast(cq, ck, cv, 3, B * Hq, std::max(Sq, Sk), work, st);
  return tbf16_host::check_launch();
}

}  // namespace

extern "C" {

int tbf16_row_scale(const void* x, int64_t rows, int64_t K, int64_t ldx, int target_exp, int l1, float* s_inv,
                    int8_t* exp_out, void* y16, int64_t ldy, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (rows < 0 || K < 0 || ldx < K || target_exp < 0 || target_exp > 64 || !s_inv || (y16 && ldy < K))
    return TBF16_ERR_INVALID;
  if (!ok8(K) || !ok8(ldx) || !tbf16_host::aligned16(x) || (y16 && (!ok8(ldy) || !tbf16_host::aligned16(y16))))
    return TBF16_ERR_ALIGN;
  if (rows == 0) return TBF16_OK;
  return tbf16_host::row_pass(x, rows, K, ldx, target_exp, l1, 1, y16, ldy, s_inv, exp_out,
                              static_cast<cudaStream_t>(stream));
}

int tbf16_quantize_rows(const void* x, int64_t rows, int64_t K, int64_t ldx, int target_exp, int l1, void* y16,
                        int64_t ldy, float* s_inv, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (rows < 0 || K < 0 || ldx < K || ldy < K || target_exp < -126 || target_exp > 126 || !s_inv)
    return TBF16_ERR_INVALID;
  if (!ok8(K) || !ok8(ldx) || !ok8(ldy) || !tbf16_host::aligned16(x) || !tbf16_host::aligned16(y16))
    return TBF16_ERR_ALIGN;
  if (rows == 0) return TBF16_OK;
  return tbf16_host::row_pass(x, rows, K, ldx, target_exp, l1, 0, y16, ldy, s_inv, nullptr,
                              static_cast<cudaStream_t>(stream));
}

int tbf16_quantize_cols(const void* x, int64_t rows, int64_t K, int64_t ldx, int target_exp, const float* row_mul,
                        void* y16, int64_t ldy, float* s_inv, float* amax_ws, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (rows < 0 || K < 0 || ldx < K || ldy < K || target_exp < -126 || target_exp > 126 || !s_inv || !amax_ws)
    return TBF16_ERR_INVALID;
  if (!ok8(K) || !ok8(ldx) || !ok8(ldy) || !tbf16_host::aligned16(x) || !tbf16_host::aligned16(y16))
    return TBF16_ERR_ALIGN;
  auto st = static_cast<cudaStream_t>(stream);
  if (K == 0) return TBF16_OK;
  if (rows == 0) {
    fill_kernel<<<grid_for(K, 256), 256, 0, st>>>(s_inv, K, 1.0f);
    return tbf16_host::check_launch();
  }
  if (cudaMemsetAsync(amax_ws, 0, sizeof(float) * K, st) != cudaSuccess) return TBF16_ERR_LAUNCH;
  const tbf16_host::DeviceInfo* d = tbf16_host::device_info();
  const int sms = d ? d->sms : 148;
  const int K8 = (int)(K / 8);
  // amax: 32 column vectors per block and chunks of at least 128 rows (few same-address atomics);
  // convert: 256 column vectors per block and chunks of at least 16 rows; both up to 16 blocks per SM.
  // blocks per SM, amax / convert minimum rows per chunk (measured on 8192 x 2048, 2048 x 8192 and
  // 8192 x 8192; TBF16_COL_* override them for tuning)
  static const int knobs[3] = {
      getenv("TBF16_COL_BLOCKS_PER_SM") ? atoi(getenv("TBF16_COL_BLOCKS_PER_SM")) : 16,
      getenv("TBF16_COL_AMAX_MINROWS") ? atoi(getenv("TBF16_COL_AMAX_MINROWS")) : 128,
      getenv("TBF16_COL_CONV_MINROWS") ? atoi(getenv("TBF16_COL_CONV_MINROWS")) : 16};
  auto chunking = [&](int col_blocks, int64_t min_rows, int64_t mult) {
    const int64_t chunks = std::max<int64_t>(
        1, std::min<int64_t>((rows + min_rows - 1) / min_rows, ((int64_t)sms * knobs[0] + col_blocks - 1) / col_blocks));
    const int64_t per = ((rows + chunks - 1) / chunks + mult - 1) / mult * mult;
    return std::make_pair(dim3(col_blocks, (unsigned)((rows + per - 1) / per)), per);
  };
  const auto ga = chunking((K8 + 31) / 32, std::max(knobs[1], 8 * kColUnroll), 8 * kColUnroll);
  const auto gc = chunking((K8 + 255) / 256, std::max(knobs[2], kColUnroll), kColUnroll);
  col_amax_kernel<<<ga.first, 256, 0, st>>>(static_cast<const uint4*>(x), row_mul, amax_ws, rows, K8, ldx / 8,
                                            ga.second);
  col_convert_kernel<<<gc.first, 256, 0, st>>>(static_cast<const uint4*>(x), row_mul, amax_ws,
                                               static_cast<uint4*>(y16), s_inv, rows, K8, ldx / 8, ldy / 8, target_exp,
                                               gc.second);
  return tbf16_host::check_launch();
}

int tbf16_head_amax(const void* x, int dtype, int64_t B, int64_t H, int64_t S, int64_t D, int64_t sb, int64_t sh,
                    int64_t ss, float* amax, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (dtype != TBF16_BF16 && dtype != TBF16_F16) return TBF16_ERR_DTYPE;
  if (int st = check_4d(x, B, H, S, D, sb, sh, ss)) return st;
  if (!amax) return TBF16_ERR_INVALID;
  auto st = static_cast<cudaStream_t>(stream);
  if (B * H == 0) return TBF16_OK;
  if (cudaMemsetAsync(amax, 0, sizeof(float) * B * H, st) != cudaSuccess) return TBF16_ERR_LAUNCH;
  if (S == 0) return TBF16_OK;
  Head4 h = make_head4(x, H, S, D, sb, sh, ss, amax, dtype == TBF16_F16);
  return launch_head_amax(h, h, h, 1, B * H, S, st);
}

int tbf16_head_exp(const void* x, int dtype, int64_t B, int64_t H, int64_t S, int64_t D, int64_t sb, int64_t sh,
                   int64_t ss, int32_t* e, float* amax_ws, void* stream) {
  if (!e) return TBF16_ERR_INVALID;
  if (int st = tbf16_head_amax(x, dtype, B, H, S, D, sb, sh, ss, amax_ws, stream)) return st;
  if (B * H == 0) return TBF16_OK;
  head_exp_kernel<<<(unsigned)((B * H + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(amax_ws, e,
                                                                                                  (int)(B * H));
  return tbf16_host::check_launch();
}

int tbf16_head_scale_cast(const void* x, int in_dtype, int64_t B, int64_t H, int64_t S, int64_t D, int64_t sb,
                          int64_t sh, int64_t ss, const int32_t* e, int64_t e_sb, int64_t e_sh, void* y, int out_dtype,
                          void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if ((in_dtype != TBF16_BF16 && in_dtype != TBF16_F16) || (out_dtype != TBF16_BF16 && out_dtype != TBF16_F16))
    return TBF16_ERR_DTYPE;
  if (int st = check_4d(x, B, H, S, D, sb, sh, ss)) return st;
  if (!e || !y) return TBF16_ERR_INVALID;
  if (!tbf16_host::aligned16(y)) return TBF16_ERR_ALIGN;
  const int64_t total8 = B * H * S * D / 8;
  if (total8 == 0) return TBF16_OK;
  ScaleCast c;
  c.x = static_cast<const uint16_t*>(x);
  c.sb = sb; c.sh = sh; c.ss = ss;
  c.H = (int)H; c.S = (int)S; c.D8 = (int)(D / 8);
  c.e = e; c.e_sb = e_sb; c.e_sh = e_sh; c.e_sign = 1;
  c.y = static_cast<uint16_t*>(y);
  c.in_f16 = in_dtype == TBF16_F16; c.out_f16 = out_dtype == TBF16_F16;
  c.total8 = total8;
  ScaleCast none = c;
  none.x = nullptr;
  return launch_scale_cast(c, none, none, 1, B * H, S, total8, static_cast<cudaStream_t>(stream));
}

int tbf16_prepare_qkv(const void* q, int64_t qsb, int64_t qsh, int64_t qss, const void* k, int64_t ksb, int64_t ksh,
                      int64_t kss, const void* v, int64_t vsb, int64_t vsh, int64_t vss, int64_t B, int64_t Hq,
                      int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, int v_exp, void* q16, void* k16, void* v16,
                      int32_t* a_out, int32_t* ev_out, float* ws, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (int st = check_4d(q, B, Hq, Sq, D, qsb, qsh, qss)) return st;
  if (int st = check_4d(k, B, Hkv, Sk, D, ksb, ksh, kss)) return st;
  if (int st = check_4d(v, B, Hkv, Sk, D, vsb, vsh, vss)) return st;
  if (!q16 || !k16 || !v16 || !a_out || !ev_out || !ws || Hkv <= 0 || Hq % Hkv != 0) return TBF16_ERR_INVALID;
  if (!tbf16_host::aligned16(q16) || !tbf16_host::aligned16(k16) || !tbf16_host::aligned16(v16)) return TBF16_ERR_ALIGN;
  auto st = static_cast<cudaStream_t>(stream);
  if (B == 0) return TBF16_OK;
  float* amax_q = ws;
  float* amax_k = ws + B * Hq;
  float* amax_v = amax_k + B * Hkv;
  if (cudaMemsetAsync(ws, 0, sizeof(float) * (B * Hq + 2 * B * Hkv), st) != cudaSuccess) return TBF16_ERR_LAUNCH;
  Head4 hq = make_head4(q, Hq, Sq, D, qsb, qsh, qss, amax_q, 0);
  Head4 hk = make_head4(k, Hkv, Sk, D, ksb, ksh, kss, amax_k, 0);
  Head4 hv = make_head4(v, Hkv, Sk, D, vsb, vsh, vss, amax_v, 0);
  if (int st2 = launch_head_amax_qkv(hq, hk, hv, B * Hq, Sq, B * Hkv, Sk, st)) return st2;
  qkv_exponents_kernel<<<1, 256, 0, st>>>(amax_q, (int)(B * Hq), amax_k, (int)(B * Hkv), amax_v, v_exp, a_out, ev_out);
  return scale_qkv(q, qsb, qsh, qss, k, ksb, ksh, kss, v, vsb, vsh, vss, B, Hq, Hkv, Sq, Sk, D, q16, k16, v16, a_out,
                   ev_out, st);
}

int tbf16_qkv_local_exponents(const void* q, int64_t qsb, int64_t qsh, int64_t qss, const void* k, int64_t ksb,
                              int64_t ksh, int64_t kss, const void* v, int64_t vsb, int64_t vsh, int64_t vss, int64_t B,
                              int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, int32_t* eqk, float* ws,
                              void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (int st = check_4d(q, B, Hq, Sq, D, qsb, qsh, qss)) return st;
  if (int st = check_4d(k, B, Hkv, Sk, D, ksb, ksh, kss)) return st;
  if (int st = check_4d(v, B, Hkv, Sk, D, vsb, vsh, vss)) return st;
  if (!eqk || !ws || Hkv <= 0 || Hq % Hkv != 0 || B < 0) return TBF16_ERR_INVALID;
  auto st = static_cast<cudaStream_t>(stream);
  float* amax_q = ws;
  float* amax_k = ws + B * Hq;
  float* amax_v = amax_k + B * Hkv;
  if (cudaMemsetAsync(ws, 0, sizeof(float) * (B * Hq + 2 * B * Hkv), st) != cudaSuccess) return TBF16_ERR_LAUNCH;
  Head4 hq = make_head4(q, Hq, Sq, D, qsb, qsh, qss, amax_q, 0);
  Head4 hk = make_head4(k, Hkv, Sk, D, ksb, ksh, kss, amax_k, 0);
  Head4 hv = make_head4(v, Hkv, Sk, D, vsb, vsh, vss, amax_v, 0);
  if (B > 0)
    if (int st2 = launch_head_amax_qkv(hq, hk, hv, B * Hq, Sq, B * Hkv, Sk, st)) return st2;
  // with no rows (B = 0) eq = ek = INT_MIN, neutral in the all-reduce (MAX)
  qk_max_exponents_kernel<<<1, 256, 0, st>>>(amax_q, (int)(B * Hq), amax_k, (int)(B * Hkv), eqk);
  return tbf16_host::check_launch();
}

int tbf16_prepare_qkv_global(const void* q, int64_t qsb, int64_t qsh, int64_t qss, const void* k, int64_t ksb,
                             int64_t ksh, int64_t kss, const void* v, int64_t vsb, int64_t vsh, int64_t vss, int64_t B,
                             int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, int v_exp, const int32_t* eqk,
                             const float* ws, void* q16, void* k16, void* v16, int32_t* a_out, int32_t* ev_out,
                             void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (int st = check_4d(q, B, Hq, Sq, D, qsb, qsh, qss)) return st;
  if (int st = check_4d(k, B, Hkv, Sk, D, ksb, ksh, kss)) return st;
  if (int st = check_4d(v, B, Hkv, Sk, D, vsb, vsh, vss)) return st;
  if (!q16 || !k16 || !v16 || !a_out || !ev_out || !eqk || !ws || Hkv <= 0 || Hq % Hkv != 0 || B < 0)
    return TBF16_ERR_INVALID;
  if (!tbf16_host::aligned16(q16) || !tbf16_host::aligned16(k16) || !tbf16_host::aligned16(v16)) return TBF16_ERR_ALIGN;
  auto st = static_cast<cudaStream_t>(stream);
  const float* amax_v = ws + B * Hq + B * Hkv;
  qkv_exponents_global_kernel<<<1, 256, 0, st>>>(eqk, amax_v, (int)(B * Hkv), v_exp, a_out, ev_out);
  return scale_qkv(q, qsb, qsh, qss, k, ksb, ksh, kss, v, vsb, vsh, vss, B, Hq, Hkv, Sq, Sk, D, q16, k16, v16, a_out,
                   ev_out, st);
}

}  // extern "C"
