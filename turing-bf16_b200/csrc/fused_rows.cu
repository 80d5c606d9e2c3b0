// Producer fusion: the kernels that produce a linear's input also compute its row exponents, so the
// linear skips its row pass (one full read of the activation) and the producer writes fp16 operands
// directly. The reference runs these as separate passes (torch's activation / norm, then its
// quantize or row_scale kernel: tbf16/ops.py:74-89, tbf16/csrc/gemm_sm75.cu:27-47).
//
//   glu_rows_kernel      h = bf16(bf16(act(g)) * u) for a gated MLP (act = silu or tanh-gelu),
//                        as torch computes act(g) * u on bf16 tensors (to within one bf16 ulp: fast exp)
//   norm_rows_kernel     r = RMSNorm(x) in the two common roundings (Gemma: bf16(x * rsqrt(ms + eps) *
//                        (w + offset)); Llama: bf16(w * bf16(x * rsqrt(ms + eps)))), optionally after a
//                        first norm and a residual add (x + norm(y), and the next block's norm rows)
// then, for the produced rows: s_inv = the fused rule's power-of-two row scale (row max, target t) and
// y16 = fp16(row / s_inv) -- exactly what tbf16_row_scale with a y16 buffer gives on the bf16 rows.
// Also here, for the attention's operands and for training: norm_rope_kernel (per-head RMSNorm + rotary
// embedding in one pass) and glu_bwd_kernel (the gated activation's backward).
//
// HBM-bound: the threads that own a row keep it in registers, so each input is read once and the fp16
// operand (plus, on request, the bf16 row) written once -- one warp per row for rows up to 1024
// elements (up to 4 x 16 bytes a lane), and for norms of up to 4096 over many rows (8-16 a lane); else
// one block per row with the fewest warps that hold it at one or two 16-byte vectors a thread (rows up
// to 16384 elements), which keeps registers per thread low and several blocks on each SM. Row maxima
// and sums of squares are reduced over the lanes and then over the warps in a fixed order.
#include "common.cuh"

using namespace tbf16;

namespace {

constexpr int kMaxThreads = 1024;
constexpr int kMaxChunks = 2;       // 16-byte vectors per thread and input in the block-per-row kernels
constexpr int kWarpRowsMaxK8 = 128;  // rows up to 1024 elements: one warp per row (up to 4 vectors a lane)
constexpr int kWarpNormMaxK8 = 512;  // many-row norms take a warp per row up to 4096 elements (16 a lane)
constexpr int kWarpRowsPerBlock = 8;

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// The activations use the hardware's fast exp and division (__expf, __fdividef): a few fp32 ulps from
// the correctly rounded expf / division / tanhf that torch's kernels call, so act(g) rounds to the same
// bf16 in all but about 1e-4 of the elements and never lands more than one bf16 ulp away. With the
// accurate library calls these kernels were bound by arithmetic, at about half the HBM rate.
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ float sigmoid_fast(float z) { return __fdividef(1.0f, 1.0f + __expf(-z)); }

constexpr float kGeluBeta = 0.7978845608028654f;  // sqrt(2 / pi)
constexpr float kGeluKappa = 0.044715f;

// tanh(y) for the tanh-GELU's y = sqrt(2 / pi) (x + 0.044715 x^3), as 2 sigmoid(2y) - 1 rounded to fp32:
// within a few fp32 ulps of tanhf(y) for every y (no cancellation near -1, where 1 + tanh(y) takes the
// same 2^-24 steps as torch's 1 + tanhf(y), so tiny negative outputs match too).
__device__ __forceinline__ float gelu_t(float x) {
  const float x3 = x * x * x;
  return 2.0f * sigmoid_fast(2.0f * (kGeluBeta * (x + kGeluKappa * x3))) - 1.0f;
}

// GELU with the tanh approximation: 0.5 x (1 + tanh(y)).
__device__ __forceinline__ float gelu_tanh(float x) { return 0.5f * x * (1.0f + gelu_t(x)); }

// The threads that own one row: a warp (WARP, short rows, 8 rows per block) or the whole block (one row
// per block, up to 1024 threads). Reductions go over the lanes by a shuffle tree and then, for a block,
// over its warps in index order, so a row's result does not depend on scheduling.
template <bool WARP>
struct RowGroup {
  int tid, nthr;
  int64_t row;
  float* red;  // block: one float per warp
  __device__ RowGroup(float* red_) : red(red_) {
    if (WARP) {
      tid = threadIdx.x & 31;
      nthr = 32;
      row = (int64_t)blockIdx.x * kWarpRowsPerBlock + (threadIdx.x >> 5);
    } else {
      tid = threadIdx.x;
      nthr = blockDim.x;
      row = blockIdx.x;
    }
  }
  template <bool MAX>
  __device__ float reduce(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float w = __shfl_xor_sync(0xffffffffu, v, o);
      v = MAX ? fmaxf(v, w) : v + w;
    }
    if (WARP) return v;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();  // red is free (an earlier reduction's readers are done)
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = red[0];
    for (int k = 1; k < nw; ++k) r = MAX ? fmaxf(r, red[k]) : r + red[k];
    return r;
  }
};

// Writes fp16(row / s_inv) from the bf16 row held in registers, s_inv, and the bf16 row if asked.
template <int NCH, bool WARP>
__device__ __forceinline__ void emit_row(const RowGroup<WARP>& rg, const uint4 (&v)[NCH], float amax, int t, int K8,
                                         uint4* __restrict__ y16, int64_t ldy8, float* __restrict__ s_inv,
                                         uint4* __restrict__ out, int64_t ldo8) {
  const int se = scale_biased_exp_fused(amax, t);
  const float sc = pow2_from_biased(se);
#pragma unroll
  for (int u = 0; u < NCH; ++u) {
    const int i = rg.tid + rg.nthr * u;
    if (i < K8) {
      if (y16) {
        uint4 o;
        o.x = pack_f16(bf16lo(v[u].x) * sc, bf16hi(v[u].x) * sc);
        o.y = pack_f16(bf16lo(v[u].y) * sc, bf16hi(v[u].y) * sc);
        o.z = pack_f16(bf16lo(v[u].z) * sc, bf16hi(v[u].z) * sc);
        o.w = pack_f16(bf16lo(v[u].w) * sc, bf16hi(v[u].w) * sc);
        y16[rg.row * ldy8 + i] = o;
      }
      if (out) out[rg.row * ldo8 + i] = v[u];
    }
  }
  if (rg.tid == 0 && y16) s_inv[rg.row] = inv_pow2_from_biased(se);
}

// Block per row: at most 32 registers a thread, so that two blocks of up to 1024 threads (three of the
// 640 a 10240-wide GeGLU row takes) stay on an SM: with 46 the 10240-wide form kept two rows in flight per
// SM and ran 30.9 us at 2048 rows, at 32 (a 20-byte spill) 28.3 us.
template <int NCH, int ACT, bool WARP>
__global__ void __launch_bounds__(WARP ? 32 * kWarpRowsPerBlock : kMaxThreads, WARP ? 1 : 2) glu_rows_kernel(const uint4* __restrict__ g, int64_t ldg8,
                                                               const uint4* __restrict__ u, int64_t ldu8, int64_t M,
                                                               int I8, int t, uint4* __restrict__ y16, int64_t ldy8,
                                                               float* __restrict__ s_inv, uint4* __restrict__ out,
                                                               int64_t ldo8) {
  pdl_launch_dependents();
  __shared__ float red[kMaxThreads / 32];
  RowGroup<WARP> rg(red);
  if (WARP && rg.row >= M) return;
  uint4 gv[NCH], uv[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int i = rg.tid + rg.nthr * c;
    gv[c] = i < I8 ? __ldg(g + rg.row * ldg8 + i) : make_uint4(0, 0, 0, 0);
    uv[c] = i < I8 ? __ldg(u + rg.row * ldu8 + i) : make_uint4(0, 0, 0, 0);
  }
  float m = 0.f;
  uint4 hv[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const uint32_t gw[4] = {gv[c].x, gv[c].y, gv[c].z, gv[c].w};
    const uint32_t uw[4] = {uv[c].x, uv[c].y, uv[c].z, uv[c].w};
    uint32_t hw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a0 = round_bf16(ACT == TBF16_ACT_SILU ? silu(bf16lo(gw[j])) : gelu_tanh(bf16lo(gw[j])));
      const float a1 = round_bf16(ACT == TBF16_ACT_SILU ? silu(bf16hi(gw[j])) : gelu_tanh(bf16hi(gw[j])));
      hw[j] = pack_bf16(a0 * bf16lo(uw[j]), a1 * bf16hi(uw[j]));
      m = fmaxf(m, fmaxf(fabsf(bf16lo(hw[j])), fabsf(bf16hi(hw[j]))));
    }
    hv[c] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  }
  const float amax = rg.template reduce<true>(m);
  emit_row<NCH, WARP>(rg, hv, amax, t, I8, y16, ldy8, s_inv, out, ldo8);
}

// A chain of row operations on one register-resident row (each step optional): a = RMSNorm_a(x) (bf16),
// a = bf16(res + a) (a residual add, the way a model adds two bf16 tensors), a written out; then
// r = RMSNorm_b(a) and the linear's fp16 operand fp16(r / s_inv) with its row scale, and/or r in bf16.
// rmsnorm_rows is the chain with only the second norm; the other uses fold a layer's residual adds into
// the norms around them (x + norm(y), and the next block's norm rows of that sum).
struct NormRows {
  const uint4* x;
  int64_t ldx8;
  const uint4* res;  // nullable
  int64_t ldr8;
  const uint4* wa;   // nullable: the first norm
  const uint4* wb;   // nullable: the second norm
  uint4* a_out;      // nullable
  int64_t lda8;
  uint4* y16;        // nullable (then s_inv is unused)
  int64_t ldy8;
  float* s_inv;
  uint4* r_out;      // nullable
  int64_t ldo8;
  int64_t M;
  int K8, K, t;
  float eps, offset;
};

// v = RMSNorm(v) with weight w, in place: mean of squares in fp32 (per thread, then the group's
// fixed-order reduction), then the style's rounding. WARP: w is the block's shared-memory copy.
template <int NCH, int STYLE, bool WARP>
__device__ __forceinline__ void norm_in_place(RowGroup<WARP>& rg, uint4 (&v)[NCH], const uint4* __restrict__ w, int K8,
                                              int K, float eps, float offset) {
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const uint32_t xw[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = bf16lo(xw[j]), b = bf16hi(xw[j]);
      ss = fmaf(a, a, ss);
      ss = fmaf(b, b, ss);
    }
  }
  const float r = rsqrtf(rg.template reduce<false>(ss) / (float)K + eps);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int i = rg.tid + rg.nthr * c;
    const uint4 wv = i < K8 ? (WARP ? w[i] : __ldg(w + i)) : make_uint4(0, 0, 0, 0);
    const uint32_t xw[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t yw[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float y0, y1;
      if (STYLE == TBF16_NORM_SCALE_FP32) {  // (x * r) * (w + offset) in fp32, one rounding
        y0 = (bf16lo(xw[j]) * r) * (bf16lo(ww[j]) + offset);
        y1 = (bf16hi(xw[j]) * r) * (bf16hi(ww[j]) + offset);
      } else {  // bf16(x * r), then the bf16 weight times it, rounded again
        y0 = bf16lo(ww[j]) * round_bf16(bf16lo(xw[j]) * r);
        y1 = bf16hi(ww[j]) * round_bf16(bf16hi(xw[j]) * r);
      }
      yw[j] = pack_bf16(y0, y1);
    }
    v[c] = make_uint4(yw[0], yw[1], yw[2], yw[3]);
  }
}

// A warp per row: two 256-thread blocks per SM for rows of up to 10 vectors a lane (2560 elements, where
// the 12-vector form took 201 registers and left one block per SM, so 2048 rows ran in two rounds of 148
// blocks; capping it at 128 registers spilled), and the norm
// weights, which every row of the block reads, staged once in shared memory while the rows load (no L2
// round trip after each norm's reduction).
template <int NCH, int STYLE, bool WARP>
__global__ void __launch_bounds__(WARP ? 32 * kWarpRowsPerBlock : kMaxThreads, (WARP && NCH <= 10) ? 2 : 1)
    norm_rows_kernel(const NormRows p) {
  pdl_launch_dependents();
  __shared__ float red[kMaxThreads / 32];
  __shared__ uint4 wsm[WARP ? 2 * kWarpNormMaxK8 : 1];
  RowGroup<WARP> rg(red);
  const bool live = !WARP || rg.row < p.M;
  uint4 v[NCH], rvs[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int i = rg.tid + rg.nthr * c;
    v[c] = live && i < p.K8 ? __ldg(p.x + rg.row * p.ldx8 + i) : make_uint4(0, 0, 0, 0);
  }
  // the residual row's loads go out with x's, not after the first norm's reduction
  if (p.res) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int i = rg.tid + rg.nthr * c;
      rvs[c] = live && i < p.K8 ? __ldg(p.res + rg.row * p.ldr8 + i) : make_uint4(0, 0, 0, 0);
    }
  }
  const uint4* wa = p.wa;
  const uint4* wb = p.wb;
  if (WARP) {
    for (int i = threadIdx.x; i < p.K8; i += blockDim.x) {
      if (p.wa) wsm[i] = __ldg(p.wa + i);
      if (p.wb) wsm[kWarpNormMaxK8 + i] = __ldg(p.wb + i);
    }
    __syncthreads();
    wa = p.wa ? wsm : nullptr;
    wb = p.wb ? wsm + kWarpNormMaxK8 : nullptr;
    if (!live) return;
  }
  if (wa) norm_in_place<NCH, STYLE, WARP>(rg, v, wa, p.K8, p.K, p.eps, p.offset);
  if (p.res) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int i = rg.tid + rg.nthr * c;
      if (i < p.K8) {
        const uint4 rv = rvs[c];
        v[c] = make_uint4(pack_bf16(bf16lo(rv.x) + bf16lo(v[c].x), bf16hi(rv.x) + bf16hi(v[c].x)),
                          pack_bf16(bf16lo(rv.y) + bf16lo(v[c].y), bf16hi(rv.y) + bf16hi(v[c].y)),
                          pack_bf16(bf16lo(rv.z) + bf16lo(v[c].z), bf16hi(rv.z) + bf16hi(v[c].z)),
                          pack_bf16(bf16lo(rv.w) + bf16lo(v[c].w), bf16hi(rv.w) + bf16hi(v[c].w)));
      }
    }
  }
  if (p.a_out) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int i = rg.tid + rg.nthr * c;
      if (i < p.K8) p.a_out[rg.row * p.lda8 + i] = v[c];
    }
  }
  if (wb) norm_in_place<NCH, STYLE, WARP>(rg, v, wb, p.K8, p.K, p.eps, p.offset);
  float amax = 0.f;
  if (p.y16) {
    float m = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const uint32_t yw[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) m = fmaxf(m, fmaxf(fabsf(bf16lo(yw[j])), fabsf(bf16hi(yw[j]))));
    }
    amax = rg.template reduce<true>(m);
  }
  if (p.y16 || p.r_out) emit_row<NCH, WARP>(rg, v, amax, p.t, p.K8, p.y16, p.ldy8, p.s_inv, p.r_out, p.ldo8);
}

// Attention operands: RMSNorm over each head's D values (optional; the QK-norm of Gemma 3 / Qwen 3) and
// rotary embedding with the rotate-half convention, as a model computes them on bf16 tensors:
// y = the norm's bf16 output (rmsnorm_rows' arithmetic), out = bf16(bf16(y cos) + bf16(rot(y) sin)) with
// rot(y) = (-y[D/2:], y[:D/2]) and cos, sin the bf16 rows of the token's position. One warp per row of
// D = 64, 128, 256 or 512 (a lane holds 1 or 2 16-byte vectors); row r is head r % H of token r / H (tokens
// ldtok apart in x, so q and k can be column slices of one fused projection), at position (r / H) % S.
template <int NCH, int STYLE, bool NORM>
__global__ void __launch_bounds__(32 * kWarpRowsPerBlock) norm_rope_kernel(
    const uint4* __restrict__ x, int64_t ldtok8, const uint4* __restrict__ w, int64_t M, int D8, float eps, float offset,
    const uint4* __restrict__ cosv, const uint4* __restrict__ sinv, int64_t ldc8, int64_t S, int64_t H,
    uint4* __restrict__ out, int64_t ldo8) {
  __shared__ float red[1];
  RowGroup<true> rg(red);
  if (rg.row >= M) return;
  const int half = D8 / 2;  // vectors in half a row: the rotation partner of vector c is c ^ half
  const int64_t tok = rg.row / H;
  const uint4* xr = x + tok * ldtok8 + (rg.row - tok * H) * D8;
  uint4 yv[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int i = rg.tid + 32 * c;
    yv[c] = i < D8 ? __ldg(xr + i) : make_uint4(0, 0, 0, 0);
  }
  if (NORM) {
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const uint32_t xw[4] = {yv[c].x, yv[c].y, yv[c].z, yv[c].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = bf16lo(xw[j]), b = bf16hi(xw[j]);
        ss = fmaf(a, a, ss);
        ss = fmaf(b, b, ss);
      }
    }
    const float r = rsqrtf(rg.template reduce<false>(ss) / (float)(D8 * 8) + eps);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int i = rg.tid + 32 * c;
      const uint4 wv = i < D8 ? __ldg(w + i) : make_uint4(0, 0, 0, 0);
      const uint32_t xw[4] = {yv[c].x, yv[c].y, yv[c].z, yv[c].w};
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float y0, y1;
        if (STYLE == TBF16_NORM_SCALE_FP32) {
          y0 = (bf16lo(xw[j]) * r) * (bf16lo(ww[j]) + offset);
          y1 = (bf16hi(xw[j]) * r) * (bf16hi(ww[j]) + offset);
        } else {
          y0 = bf16lo(ww[j]) * round_bf16(bf16lo(xw[j]) * r);
          y1 = bf16hi(ww[j]) * round_bf16(bf16hi(xw[j]) * r);
        }
        o[j] = pack_bf16(y0, y1);
      }
      yv[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  // the partner vectors: another lane's (half < 32) or this lane's other vector (half = 32)
  uint4 pv[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    if (half < 32) {
      pv[c].x = __shfl_xor_sync(0xffffffffu, yv[c].x, half);
      pv[c].y = __shfl_xor_sync(0xffffffffu, yv[c].y, half);
      pv[c].z = __shfl_xor_sync(0xffffffffu, yv[c].z, half);
      pv[c].w = __shfl_xor_sync(0xffffffffu, yv[c].w, half);
    } else {
      pv[c] = yv[c ^ 1];
    }
  }
  const int64_t pos = tok % S;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int i = rg.tid + 32 * c;
    if (i >= D8) continue;
    const float sign = i < half ? -1.f : 1.f;
    const uint4 cv = __ldg(cosv + pos * ldc8 + i), sv = __ldg(sinv + pos * ldc8 + i);
    const uint32_t yw[4] = {yv[c].x, yv[c].y, yv[c].z, yv[c].w}, pw[4] = {pv[c].x, pv[c].y, pv[c].z, pv[c].w};
    const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w}, sw[4] = {sv.x, sv.y, sv.z, sv.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = round_bf16(bf16lo(yw[j]) * bf16lo(cw[j])) + round_bf16(sign * bf16lo(pw[j]) * bf16lo(sw[j]));
      const float hi = round_bf16(bf16hi(yw[j]) * bf16hi(cw[j])) + round_bf16(sign * bf16hi(pw[j]) * bf16hi(sw[j]));
      o[j] = pack_bf16(lo, hi);
    }
    out[rg.row * ldo8 + i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Backward of h = bf16(act(g)) * u as torch's autograd takes it on bf16 tensors: a = bf16(act(g)) again,
// du = bf16(dh a), da = bf16(dh u), dg = bf16(da act'(g)) with act' in fp32, in the order torch's
// silu backward evaluates it (da s (1 + g (1 - s)), s = 1 / (1 + e^-g)); tanh-GELU: da (0.5 (1 + t) +
// 0.5 g (1 - t^2) sqrt(2/pi) (1 + 3 0.044715 g^2)), t = tanh(sqrt(2/pi) (g + 0.044715 g^3)) as the
// forward's gelu_t.
// One block per row, 16-byte vectors.
template <int ACT>
__global__ void __launch_bounds__(256) glu_bwd_kernel(const uint4* __restrict__ dh, int64_t ldh8,
                                                      const uint4* __restrict__ g, int64_t ldg8,
                                                      const uint4* __restrict__ u, int64_t ldu8, int I8,
                                                      uint4* __restrict__ dg, int64_t lddg8, uint4* __restrict__ du,
                                                      int64_t lddu8) {
  const int64_t row = blockIdx.x;
  for (int i = threadIdx.x; i < I8; i += blockDim.x) {
    const uint4 hv = __ldg(dh + row * ldh8 + i), gv = __ldg(g + row * ldg8 + i), uv = __ldg(u + row * ldu8 + i);
    const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t go[4], uo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float dgv[2], duv[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float x = k ? bf16hi(gw[j]) : bf16lo(gw[j]);
        const float d = k ? bf16hi(hw[j]) : bf16lo(hw[j]);
        const float up = k ? bf16hi(uw[j]) : bf16lo(uw[j]);
        const float da = round_bf16(d * up);
        float a;
        if (ACT == TBF16_ACT_SILU) {
          const float e1 = 1.0f + __expf(-x);
          const float sg = __fdividef(1.0f, e1);
          a = __fdividef(x, e1);
          dgv[k] = da * sg * (1.0f + x * (1.0f - sg));
        } else {
          const float t = gelu_t(x);
          a = 0.5f * x * (1.0f + t);
          const float left = 0.5f * x, right = 1.0f + t;
          const float right_d = left * (1.0f - t * t) * (kGeluBeta * (1.0f + 3.0f * kGeluKappa * (x * x)));
          dgv[k] = da * (0.5f * right + right_d);
        }
        duv[k] = d * round_bf16(a);
      }
      go[j] = pack_bf16(dgv[0], dgv[1]);
      uo[j] = pack_bf16(duv[0], duv[1]);
    }
    dg[row * lddg8 + i] = make_uint4(go[0], go[1], go[2], go[3]);
    du[row * lddu8 + i] = make_uint4(uo[0], uo[1], uo[2], uo[3]);
  }
}

// Launch shape for rows of K8 16-byte vectors: short rows one warp each (vectors per lane nch of 1, 2, 4);
// longer rows one block each, nch (1 or 2) vectors per thread and the fewest warps that cover the row (up
// to 512 while two vectors a thread do), so that each thread holds little and many blocks fit an SM.
// nch = 0: the row is too long.
struct RowLaunch {
  bool warp;
  int nch, threads;
};
RowLaunch row_launch(int64_t K8, int64_t M, int64_t warp_max_k8) {
  if (K8 <= kWarpRowsMaxK8) return {true, K8 <= 32 ? 1 : (K8 <= 64 ? 2 : 4), 32 * kWarpRowsPerBlock};
  // enough rows to fill the GPU with warps: a warp per row, 8 or 16 vectors a lane (no block barriers,
  // many loads in flight per thread)
  if (K8 <= warp_max_k8 && M >= 1024)
    return {true, K8 <= 256 ? 8 : K8 <= 320 ? 10 : K8 <= 384 ? 12 : 16, 32 * kWarpRowsPerBlock};
  // at most 512 threads where two vectors a thread cover the row: four blocks (rows) per SM instead of two
  // (8192-wide SiLU rows over 8192 rows: 90.3 -> 64.2 us)
  for (int c = 1; c <= kMaxChunks; c *= 2)
    if (K8 <= (int64_t)(K8 <= 512 * kMaxChunks ? 512 : kMaxThreads) * c) {
      const int64_t per = (K8 + c - 1) / c;
      return {false, c, (int)((per + 31) / 32 * 32)};
    }
  return {false, 0, 0};
}

int launch_norm_rows(const NormRows& p, int style, cudaStream_t st) {
  static const int warp_max = [] {  // rows (in 16-byte vectors) up to which many-row norms take a warp per row
    const char* e = getenv("TBF16_NORM_WARP_MAX_K8");
    return e ? std::min(atoi(e), kWarpNormMaxK8) : kWarpNormMaxK8;  // 16 vectors a lane at most
  }();
  const RowLaunch L = row_launch(p.K8, p.M, warp_max);
  if (!L.nch || p.M > INT32_MAX) return TBF16_ERR_UNSUPPORTED;  // rows above TBF16_FUSED_MAX_ROW
  const unsigned blocks = (unsigned)(L.warp ? (p.M + kWarpRowsPerBlock - 1) / kWarpRowsPerBlock : p.M);
#define TBF16_NORM(N, S, W) norm_rows_kernel<N, S, W><<<blocks, L.threads, 0, st>>>(p)
#define TBF16_NORM_STYLE(N, W) \
  if (style == TBF16_NORM_SCALE_FP32) TBF16_NORM(N, TBF16_NORM_SCALE_FP32, W); else TBF16_NORM(N, TBF16_NORM_SCALE_BF16, W)
  if (L.warp) {
    switch (L.nch) {
      case 1: TBF16_NORM_STYLE(1, true); break;
      case 2: TBF16_NORM_STYLE(2, true); break;
      case 4: TBF16_NORM_STYLE(4, true); break;
      case 8: TBF16_NORM_STYLE(8, true); break;
      case 10: TBF16_NORM_STYLE(10, true); break;
      case 12: TBF16_NORM_STYLE(12, true); break;
      default: TBF16_NORM_STYLE(16, true); break;
    }
  } else {
    if (L.nch == 1) TBF16_NORM_STYLE(1, false);
    else TBF16_NORM_STYLE(2, false);
  }
#undef TBF16_NORM_STYLE
#undef TBF16_NORM
  return tbf16_host::check_launch();
}

}  // namespace

extern "C" {

int tbf16_glu_rows(const void* g, int64_t ldg, const void* u, int64_t ldu, int64_t M, int64_t I, int act,
                   int target_exp, void* y16, int64_t ldy, float* s_inv, void* h_out, int64_t ldo, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (M < 0 || I < 0 || ldg < I || ldu < I || ldy < I || (h_out && ldo < I) || !s_inv || !y16 || !g || !u ||
      target_exp < 0 || target_exp > 64 || (act != TBF16_ACT_SILU && act != TBF16_ACT_GELU_TANH))
    return TBF16_ERR_INVALID;
  if (I % 8 || ldg % 8 || ldu % 8 || ldy % 8 || (h_out && ldo % 8) || !tbf16_host::aligned16(g) ||
      !tbf16_host::aligned16(u) || !tbf16_host::aligned16(y16) || (h_out && !tbf16_host::aligned16(h_out)))
    return TBF16_ERR_ALIGN;
  if (M == 0 || I == 0) return TBF16_OK;
  const int64_t I8 = I / 8;
  const RowLaunch L = row_launch(I8, M, kWarpRowsMaxK8);
  if (!L.nch || M > INT32_MAX) return TBF16_ERR_UNSUPPORTED;  // rows above TBF16_FUSED_MAX_ROW
  auto st = static_cast<cudaStream_t>(stream);
  const uint4 *gp = static_cast<const uint4*>(g), *up = static_cast<const uint4*>(u);
  uint4 *yp = static_cast<uint4*>(y16), *op = static_cast<uint4*>(h_out);
  const unsigned blocks = (unsigned)(L.warp ? (M + kWarpRowsPerBlock - 1) / kWarpRowsPerBlock : M);
#define TBF16_GLU(N, A, W)                                                                                 \
  glu_rows_kernel<N, A, W><<<blocks, L.threads, 0, st>>>(gp, ldg / 8, up, ldu / 8, M, (int)I8, target_exp, yp, \
                                                         ldy / 8, s_inv, op, ldo / 8)
#define TBF16_GLU_ACT(N, W) \
  if (act == TBF16_ACT_SILU) TBF16_GLU(N, TBF16_ACT_SILU, W); else TBF16_GLU(N, TBF16_ACT_GELU_TANH, W)
  if (L.warp) {
    if (L.nch == 1) TBF16_GLU_ACT(1, true);
    else if (L.nch == 2) TBF16_GLU_ACT(2, true);
    else TBF16_GLU_ACT(4, true);
  } else {
    if (L.nch == 1) TBF16_GLU_ACT(1, false);
    else TBF16_GLU_ACT(2, false);
  }
#undef TBF16_GLU_ACT
#undef TBF16_GLU
  return tbf16_host::check_launch();
}

int tbf16_glu_bwd(const void* dh, int64_t ldh, const void* g, int64_t ldg, const void* u, int64_t ldu, int64_t M,
                  int64_t I, int act, void* dg, int64_t lddg, void* du, int64_t lddu, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (M < 0 || I < 0 || ldh < I || ldg < I || ldu < I || lddg < I || lddu < I || !dh || !g || !u || !dg || !du ||
      (act != TBF16_ACT_SILU && act != TBF16_ACT_GELU_TANH))
    return TBF16_ERR_INVALID;
  if (I % 8 || ldh % 8 || ldg % 8 || ldu % 8 || lddg % 8 || lddu % 8 || !tbf16_host::aligned16(dh) ||
      !tbf16_host::aligned16(g) || !tbf16_host::aligned16(u) || !tbf16_host::aligned16(dg) || !tbf16_host::aligned16(du))
    return TBF16_ERR_ALIGN;
  if (M == 0 || I == 0) return TBF16_OK;
  if (M > INT32_MAX || I / 8 > INT32_MAX) return TBF16_ERR_UNSUPPORTED;
  auto st = static_cast<cudaStream_t>(stream);
  const int I8 = (int)(I / 8);
  const int threads = I8 >= 256 ? 256 : (I8 + 31) / 32 * 32;
  const uint4 *hp = static_cast<const uint4*>(dh), *gp = static_cast<const uint4*>(g), *up = static_cast<const uint4*>(u);
  uint4 *gop = static_cast<uint4*>(dg), *uop = static_cast<uint4*>(du);
  if (act == TBF16_ACT_SILU)
    glu_bwd_kernel<TBF16_ACT_SILU><<<(unsigned)M, threads, 0, st>>>(hp, ldh / 8, gp, ldg / 8, up, ldu / 8, I8, gop,
                                                                     lddg / 8, uop, lddu / 8);
  else
    glu_bwd_kernel<TBF16_ACT_GELU_TANH><<<(unsigned)M, threads, 0, st>>>(hp, ldh / 8, gp, ldg / 8, up, ldu / 8, I8, gop,
                                                                          lddg / 8, uop, lddu / 8);
  return tbf16_host::check_launch();
}

int tbf16_rmsnorm_rope(const void* x, int64_t ldtok, const void* w, int64_t M, int64_t D, float eps, int style,
                       float offset, const void* cos, const void* sin, int64_t ldc, int64_t S, int64_t H, void* out,
                       int64_t ldo, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (M < 0 || S <= 0 || H <= 0 || M % H || ldtok < H * D || ldc < D || ldo < D || !x || !cos || !sin || !out ||
      !(eps >= 0.f) ||
      (style != TBF16_NORM_SCALE_FP32 && style != TBF16_NORM_SCALE_BF16))
    return TBF16_ERR_INVALID;
  if (D != 64 && D != 128 && D != 256 && D != 512) return TBF16_ERR_UNSUPPORTED;
  if (ldtok % 8 || ldc % 8 || ldo % 8 || !tbf16_host::aligned16(x) || (w && !tbf16_host::aligned16(w)) ||
      !tbf16_host::aligned16(cos) || !tbf16_host::aligned16(sin) || !tbf16_host::aligned16(out))
    return TBF16_ERR_ALIGN;
  if (M == 0) return TBF16_OK;
  auto st = static_cast<cudaStream_t>(stream);
  const unsigned blocks = (unsigned)((M + kWarpRowsPerBlock - 1) / kWarpRowsPerBlock);
  const uint4 *xp = static_cast<const uint4*>(x), *wp = static_cast<const uint4*>(w);
  const uint4 *cp = static_cast<const uint4*>(cos), *sp = static_cast<const uint4*>(sin);
  uint4* op = static_cast<uint4*>(out);
  const int D8 = (int)(D / 8);
#define TBF16_ROPE(N, S_, NORM)                                                                                     \
  norm_rope_kernel<N, S_, NORM><<<blocks, 32 * kWarpRowsPerBlock, 0, st>>>(xp, ldtok / 8, wp, M, D8, eps, offset, cp, sp, \
                                                                          ldc / 8, S, H, op, ldo / 8)
#define TBF16_ROPE_N(N)                                                                  \
  if (!w) TBF16_ROPE(N, TBF16_NORM_SCALE_FP32, false);                                   \
  else if (style == TBF16_NORM_SCALE_FP32) TBF16_ROPE(N, TBF16_NORM_SCALE_FP32, true);   \
  else TBF16_ROPE(N, TBF16_NORM_SCALE_BF16, true)
  if (D8 <= 32) {
    TBF16_ROPE_N(1);
  } else {
    TBF16_ROPE_N(2);
  }
#undef TBF16_ROPE_N
#undef TBF16_ROPE
  return tbf16_host::check_launch();
}


int tbf16_rmsnorm_rows(const void* x, int64_t ldx, const void* w, int64_t M, int64_t K, float eps, int style,
                       float offset, int target_exp, void* y16, int64_t ldy, float* s_inv, void* r_out, int64_t ldo,
                       void* stream) {
  if (!w) return TBF16_ERR_INVALID;
  return tbf16_add_rmsnorm_rows(x, ldx, nullptr, 0, nullptr, w, M, K, eps, style, offset, target_exp, nullptr, 0, y16,
                                ldy, s_inv, r_out, ldo, stream);
}

int tbf16_add_rmsnorm_rows(const void* x, int64_t ldx, const void* res, int64_t ldr, const void* wa, const void* wb,
                           int64_t M, int64_t K, float eps, int style, float offset, int target_exp, void* a_out,
                           int64_t lda, void* y16, int64_t ldy, float* s_inv, void* r_out, int64_t ldo, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (M < 0 || K < 0 || ldx < K || (res && ldr < K) || (a_out && lda < K) || (y16 && ldy < K) || (r_out && ldo < K) ||
      (y16 && !s_inv) || (!y16 && !r_out && !a_out) || (r_out && !wb && !wa && !res) || !x || !(eps >= 0.f) ||
      target_exp < 0 || target_exp > 64 || (style != TBF16_NORM_SCALE_FP32 && style != TBF16_NORM_SCALE_BF16))
    return TBF16_ERR_INVALID;
  auto a16 = [](const void* q) { return !q || tbf16_host::aligned16(q); };
  if (K % 8 || ldx % 8 || (res && ldr % 8) || (a_out && lda % 8) || (y16 && ldy % 8) || (r_out && ldo % 8) ||
      !tbf16_host::aligned16(x) || !a16(res) || !a16(wa) || !a16(wb) || !a16(a_out) || !a16(y16) || !a16(r_out))
    return TBF16_ERR_ALIGN;
  if (M == 0 || K == 0) return TBF16_OK;
  NormRows p;
  p.x = static_cast<const uint4*>(x);
  p.ldx8 = ldx / 8;
  p.res = static_cast<const uint4*>(res);
  p.ldr8 = ldr / 8;
  p.wa = static_cast<const uint4*>(wa);
  p.wb = static_cast<const uint4*>(wb);
  p.a_out = static_cast<uint4*>(a_out);
  p.lda8 = lda / 8;
  p.y16 = static_cast<uint4*>(y16);
  p.ldy8 = ldy / 8;
  p.s_inv = s_inv;
  p.r_out = static_cast<uint4*>(r_out);
  p.ldo8 = ldo / 8;
  p.M = M;
  p.K8 = (int)(K / 8);
  p.K = (int)K;
  p.t = target_exp;
  p.eps = eps;
  p.offset = offset;
  return launch_norm_rows(p, style, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
