// Scaled bf16 convolutions (the reference's tbf16/conv.py:34-60): one exact power-of-two scale per
// sample for the input (a convolution mixes positions, so rows cannot be scaled separately), one per
// output channel for the weight (prepared once, as a linear's rows), fp32 accumulation, and the two
// scales undone in the bf16 epilogue:
//
//   e[b]     = frexp_exp(max |x[b]|) - t      (zero samples count as max 1; t = _target_exp(K))
//   x16      = fp16_rn(x * 2^-e[b])
//   y[b,o,p] = bf16_rn((sum_k x16 w16[o,k]) * 2^e[b] * ws[o] + bias[o])
//
// groups == 1: im2col into fp16 rows (one row per output position, K = C kd kh kw columns zero-padded
// to a multiple of 8, each row carrying its sample's output scale) and the tcgen05 GEMM against the
// [O, K] weight rows; the output comes out channels-last. For C a multiple of 8 the rows are built from a
// scaled channels-last fp16 copy of the input by 16-byte copies, columns in (tap, channel) order. groups > 1 (depthwise and grouped convs, a few
// input channels per output): a direct kernel, one thread per output element. The reference ends in a
// cuDNN fp16 conv whose output is rounded to fp16 before the scales; here the fp32 sum is scaled and
// rounded to bf16 once. Geometry is passed as an array of int64 (TBF16_CONV_GEOM_LEN values, order in the header).
#include <utility>

#include "common.cuh"

using namespace tbf16;

namespace {

struct Geom {
  int64_t B, C, D, H, W;          // input (batch, channels, depth, height, width)
  int64_t sb, sc, sd, sh, sw;     // input strides in elements (any layout)
  int64_t kd, kh, kw;             // kernel extent
  int64_t std_, sth, stw;         // stride
  int64_t pd, ph, pw;             // zero padding
  int64_t dd, dh, dw;             // dilation
  int64_t Do, Ho, Wo;             // output extent
};

Geom load_geom(const int64_t* g) {
  Geom r;
  int64_t* f = &r.B;
  for (int i = 0; i < TBF16_CONV_GEOM_LEN; ++i) f[i] = g[i];
  return r;
}

// x * 2^-e exactly for any e (two steps when 2^-e alone would leave fp32's normal range).
__device__ __forceinline__ float scale_pow2(float v, int e) {
  const int ne = -e;
  if (ne >= -126 && ne <= 127) return v * exp2i(ne);
  const int h = ne / 2;
  return (v * exp2i(h)) * exp2i(ne - h);
}

// Per-sample max |x| over n dense elements of each sample (samples ld apart), merged with atomicMax:
// 16-byte loads when the sample is 16-byte aligned and n a multiple of 8, four of them in flight.
__global__ void __launch_bounds__(256) sample_amax_kernel(const __nv_bfloat16* __restrict__ x, int64_t n, int64_t ld,
                                                          int vec, float* __restrict__ amax) {
  const int64_t b = blockIdx.y;
  const __nv_bfloat16* xs = x + b * ld;
  float m = 0.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    const uint4* xv = reinterpret_cast<const uint4*>(xs);
    const int64_t n8 = n / 8;
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n8; i += 4 * stride) {
      uint4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = __ldg(xv + i + u * stride);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t w[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) m = fmaxf(m, fmaxf(fabsf(bf16lo(w[j])), fabsf(bf16hi(w[j]))));
      }
    }
    for (; i < n8; i += stride) {
      const uint4 q = __ldg(xv + i);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) m = fmaxf(m, fmaxf(fabsf(bf16lo(w[j])), fabsf(bf16hi(w[j]))));
    }
  } else {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
      m = fmaxf(m, fabsf(__bfloat162float(xs[i])));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<int*>(amax) + b, __float_as_int(m));
}

__global__ void sample_exp_kernel(const float* __restrict__ amax, int64_t B, int t, int32_t* __restrict__ e,
                                  float* __restrict__ out_scale) {
  const int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (b >= B) return;
  const float a = amax[b];
  const int eb = frexp_exp(a > 0.f ? a : 1.0f) - t;
  e[b] = eb;
  out_scale[b] = exp2i(eb);
}

// cols16[m, k] = fp16(x[b, c, od*s - p + z*d, ...] * 2^-e[b]) for output position m = (b, od, oh, ow) and
// k = ((c kd + z) kh + y) kw + x < K, 0 past K or in the padding; row_scale[m] = 2^e[b].
__global__ void __launch_bounds__(256) im2col_kernel(const __nv_bfloat16* __restrict__ xin, const Geom g, int64_t K,
                                                     int64_t Kp, const int32_t* __restrict__ e,
                                                     const float* __restrict__ out_scale, uint4* __restrict__ cols,
                                                     float* __restrict__ row_scale) {
  const int64_t K8 = Kp / 8;
  const int64_t M = g.B * g.Do * g.Ho * g.Wo;
  const int64_t kvol = g.kd * g.kh * g.kw;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < M * K8; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / K8, j = i - m * K8;
    int64_t r = m;
    const int64_t ow = r % g.Wo; r /= g.Wo;
    const int64_t oh = r % g.Ho; r /= g.Ho;
    const int64_t od = r % g.Do;
    const int64_t b = r / g.Do;
    const int eb = e[b];
    const __nv_bfloat16* xb = xin + b * g.sb;
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t k = j * 8 + u;
      float val = 0.f;
      if (k < K) {
        const int64_t c = k / kvol;
        int64_t q = k - c * kvol;
        const int64_t z = q / (g.kh * g.kw);
        q -= z * g.kh * g.kw;
        const int64_t yy = q / g.kw, xx = q - yy * g.kw;
        const int64_t id = od * g.std_ - g.pd + z * g.dd;
        const int64_t ih = oh * g.sth - g.ph + yy * g.dh;
        const int64_t iw = ow * g.stw - g.pw + xx * g.dw;
        if (id >= 0 && id < g.D && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W)
          val = scale_pow2(__bfloat162float(xb[c * g.sc + id * g.sd + ih * g.sh + iw * g.sw]), eb);
      }
      v[u] = val;
    }
    cols[i] = make_uint4(pack_f16(v[0], v[1]), pack_f16(v[2], v[3]), pack_f16(v[4], v[5]), pack_f16(v[6], v[7]));
    if (j == 0) row_scale[m] = out_scale[b];
  }
}

// Fast path for C % 8 == 0, in two passes. (1) x16cl[b, d, h, w, c] = fp16(x * 2^-e[b]) channels-last,
// 8 channels per thread (one 16-byte store). A channels-last input is read as the same flat array (one
// 16-byte load, the sample from one division); any other layout is gathered element by element.
// With amax non-null the exponents come from the sample maxima here (the rule of sample_exp_kernel), and
// the thread that converts a sample's first 8 channels also writes its e and output scale.
__global__ void __launch_bounds__(256) scale_cl_kernel(const __nv_bfloat16* __restrict__ xin, const Geom g,
                                                       int32_t* __restrict__ e, uint4* __restrict__ x16cl,
                                                       int flat, const float* __restrict__ amax = nullptr,
                                                       int t = 0, float* __restrict__ out_scale = nullptr) {
  pdl_launch_dependents();  // the implicit GEMM may start its prologue and weight loads meanwhile
  const int C8 = (int)(g.C / 8);
  const int64_t per_sample = g.D * g.H * g.W * C8;
  const int64_t total = g.B * per_sample;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / per_sample;
    int eb;
    if (amax) {
      const float a = __ldg(amax + b);
      eb = frexp_exp(a > 0.f ? a : 1.0f) - t;
      if (i == b * per_sample) {
        e[b] = eb;
        out_scale[b] = exp2i(eb);
      }
    } else {
      eb = e[b];
    }
    float v[8];
    if (flat) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(xin + b * g.sb) + (i - b * per_sample));
      v[0] = bf16lo(q.x); v[1] = bf16hi(q.x); v[2] = bf16lo(q.y); v[3] = bf16hi(q.y);
      v[4] = bf16lo(q.z); v[5] = bf16hi(q.z); v[6] = bf16lo(q.w); v[7] = bf16hi(q.w);
    } else {
      const int c8 = (int)(i % C8);
      int64_t r = i / C8;
      const int64_t w = r % g.W; r /= g.W;
      const int64_t h = r % g.H; r /= g.H;
      const int64_t d = r % g.D;
      const __nv_bfloat16* src = xin + b * g.sb + d * g.sd + h * g.sh + w * g.sw + (int64_t)c8 * 8 * g.sc;
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __bfloat162float(src[u * g.sc]);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = scale_pow2(v[u], eb);
    x16cl[i] = make_uint4(pack_f16(v[0], v[1]), pack_f16(v[2], v[3]), pack_f16(v[4], v[5]), pack_f16(v[6], v[7]));
  }
}

// (2) cols16[m, tap * C + c] = x16cl at the tap's input position (zero in the padding): one warp per
// output position (its coordinates decoded once), the lanes copying each tap's C / 8 16-byte chunks
// (coalesced on both sides) -- taps ordered (z, y, x), channels fastest, as the weight rows prepared
// for this path.
__global__ void __launch_bounds__(256) im2col_cl_kernel(const uint4* __restrict__ x16cl, const Geom g,
                                                        const float* __restrict__ out_scale, uint4* __restrict__ cols,
                                                        float* __restrict__ row_scale) {
  const int C8 = (int)(g.C / 8);
  const int kh = (int)g.kh, kw = (int)g.kw, taps = (int)(g.kd * g.kh * g.kw);
  const int lane = threadIdx.x & 31;
  const int64_t M = g.B * g.Do * g.Ho * g.Wo;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t m = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); m < M; m += warps) {
    int64_t r = m;
    const int64_t ow = r % g.Wo; r /= g.Wo;
    const int64_t oh = r % g.Ho; r /= g.Ho;
    const int64_t od = r % g.Do;
    const int64_t b = r / g.Do;
    const int64_t d0 = od * g.std_ - g.pd, h0 = oh * g.sth - g.ph, w0 = ow * g.stw - g.pw;
    const uint4* xb = x16cl + b * g.D * g.H * g.W * C8;
    uint4* row = cols + m * (int64_t)taps * C8;
    for (int tap = 0; tap < taps; ++tap) {
      const int z = tap / (kh * kw), yx = tap - z * kh * kw, yy = yx / kw, xx = yx - yy * kw;
      const int64_t id = d0 + z * g.dd, ih = h0 + yy * g.dh, iw = w0 + xx * g.dw;
      const bool in = id >= 0 && id < g.D && ih >= 0 && ih < g.H && iw >= 0 && iw < g.W;
      const uint4* src = xb + ((id * g.H + ih) * g.W + iw) * C8;
      for (int c8 = lane; c8 < C8; c8 += 32) row[tap * C8 + c8] = in ? __ldg(src + c8) : make_uint4(0, 0, 0, 0);
    }
    if (lane == 0) row_scale[m] = out_scale[b];
  }
}

// Grouped / depthwise convolution, one thread per output element of y (B, O, Do, Ho, Wo) contiguous:
// fp32 sum over the group's Cg input channels and the kernel window of fp16(x 2^-e) * w16.
__global__ void __launch_bounds__(256) conv_grouped_kernel(const __nv_bfloat16* __restrict__ xin, const Geom g,
                                                           int64_t O, int64_t groups,
                                                           const __half* __restrict__ w16,
                                                           const float* __restrict__ ws,
                                                           const __nv_bfloat16* __restrict__ bias,
                                                           const int32_t* __restrict__ e,
                                                           const float* __restrict__ out_scale,
                                                           __nv_bfloat16* __restrict__ y) {
  const int64_t total = g.B * O * g.Do * g.Ho * g.Wo;
  const int64_t Cg = g.C / groups, Og = O / groups;
  const int64_t kvol = g.kd * g.kh * g.kw;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i;
    const int64_t ow = r % g.Wo; r /= g.Wo;
    const int64_t oh = r % g.Ho; r /= g.Ho;
    const int64_t od = r % g.Do; r /= g.Do;
    const int64_t o = r % O;
    const int64_t b = r / O;
    const int eb = e[b];
    const int64_t c0 = (o / Og) * Cg;
    const __nv_bfloat16* xb = xin + b * g.sb;
    const __half* wo = w16 + o * Cg * kvol;
    float acc = 0.f;
    for (int64_t c = 0; c < Cg; ++c) {
      for (int64_t z = 0; z < g.kd; ++z) {
        const int64_t id = od * g.std_ - g.pd + z * g.dd;
        if (id < 0 || id >= g.D) continue;
        for (int64_t yy = 0; yy < g.kh; ++yy) {
          const int64_t ih = oh * g.sth - g.ph + yy * g.dh;
          if (ih < 0 || ih >= g.H) continue;
          for (int64_t xx = 0; xx < g.kw; ++xx) {
            const int64_t iw = ow * g.stw - g.pw + xx * g.dw;
            if (iw < 0 || iw >= g.W) continue;
            const float xv = __half2float(__float2half_rn(
                scale_pow2(__bfloat162float(xb[(c0 + c) * g.sc + id * g.sd + ih * g.sh + iw * g.sw]), eb)));
            acc = fmaf(xv, __half2float(wo[((c * g.kd + z) * g.kh + yy) * g.kw + xx]), acc);
          }
        }
      }
    }
    float v = (acc * out_scale[b]) * ws[o];
    if (bias) v += __bfloat162float(bias[o]);
    y[i] = __float2bfloat16_rn(v);
  }
}

// The implicit GEMM's conditions: one group (checked by the caller), channels a multiple of 64 (a K
// block is one tap's 64 channels; the weight rows are then the (tap, channel) rows of the im2col path),
// stride 1, and output rows that tile into 128-position boxes inside one (sample, depth) slice: Wo a
// power-of-two divisor of 128 or a multiple of 128, and Ho Wo a multiple of 128.
bool implicit_ok(const Geom& g, int64_t O) {
  if (g.C % 64 || O % 8 || g.std_ != 1 || g.sth != 1 || g.stw != 1) return false;
  const int64_t bx = g.Wo < 128 ? g.Wo : 128;
  if (bx <= 0 || g.Wo % bx || 128 % bx || (g.Ho * g.Wo) % 128) return false;
  const int64_t M = g.B * g.Do * g.Ho * g.Wo, K = g.kd * g.kh * g.kw * g.C;
  return M <= INT32_MAX && K <= INT32_MAX && O <= INT32_MAX && g.B * g.D * g.H * g.W <= INT32_MAX;
}

int grid_for(int64_t work) {
  const tbf16_host::DeviceInfo* d = tbf16_host::device_info();
  const int64_t cap = (int64_t)(d ? d->sms : 148) * 16;
  const int64_t g = (work + 255) / 256;
  return (int)(g < 1 ? 1 : (g < cap ? g : cap));
}

bool geom_ok(const Geom& g) {
  return g.B >= 0 && g.C > 0 && g.D > 0 && g.H > 0 && g.W > 0 && g.kd > 0 && g.kh > 0 && g.kw > 0 && g.std_ > 0 &&
         g.sth > 0 && g.stw > 0 && g.pd >= 0 && g.ph >= 0 && g.pw >= 0 && g.dd > 0 && g.dh > 0 && g.dw > 0 &&
         g.Do > 0 && g.Ho > 0 && g.Wo > 0 && g.sb >= 0 && g.sc >= 0 && g.sd >= 0 && g.sh >= 0 && g.sw >= 0 &&
         (g.Do - 1) * g.std_ + (g.kd - 1) * g.dd < g.D + 2 * g.pd && (g.Ho - 1) * g.sth + (g.kh - 1) * g.dh < g.H + 2 * g.ph &&
         (g.Wo - 1) * g.stw + (g.kw - 1) * g.dw < g.W + 2 * g.pw;
}

}  // namespace

namespace {
// amax_ws[b] = max |x| over sample b's n dense elements (samples ld apart).
int launch_sample_amax(const void* x, int64_t B, int64_t n, int64_t ld, float* amax_ws, cudaStream_t st) {
  if (cudaMemsetAsync(amax_ws, 0, sizeof(float) * B, st) != cudaSuccess) return TBF16_ERR_LAUNCH;
  if (n > 0) {
    // about four blocks per SM in all, each thread with a few 16-byte loads in flight
    const tbf16_host::DeviceInfo* d = tbf16_host::device_info();
    const int64_t want = ((int64_t)(d ? d->sms : 148) * 4 + B - 1) / B;
    const int64_t per = (n / 8 + 1023) / 1024;
    const unsigned gx = (unsigned)(per < 1 ? 1 : (per < want ? per : want));
    const int vec = n % 8 == 0 && ld % 8 == 0 && tbf16_host::aligned16(x);
    sample_amax_kernel<<<dim3(gx, (unsigned)B), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), n, ld, vec, amax_ws);
  }
  return TBF16_OK;
}

// The input's samples are dense blocks of C D H W elements (any order of the four strides).
bool dense_samples(const Geom& g) {
  int64_t sz[4] = {g.C, g.D, g.H, g.W}, sd[4] = {g.sc, g.sd, g.sh, g.sw};
  for (int i = 0; i < 4; ++i)  // sort the dimensions by stride (size-1 dimensions last)
    for (int j = i + 1; j < 4; ++j)
      if ((sz[j] > 1 && (sz[i] == 1 || sd[j] < sd[i]))) {
        std::swap(sz[i], sz[j]);
        std::swap(sd[i], sd[j]);
      }
  int64_t expect = 1;
  for (int i = 0; i < 4 && sz[i] > 1; ++i) {
    if (sd[i] != expect) return false;
    expect *= sz[i];
  }
  return g.B == 1 || g.sb >= expect;
}
}  // namespace

extern "C" {


int tbf16_conv_sample_scale(const void* x, int64_t B, int64_t n, int64_t ld, int target_exp, float* amax_ws,
                            int32_t* e, float* out_scale, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (B < 0 || n < 0 || ld < n || !x || !amax_ws || !e || !out_scale || target_exp < -126 || target_exp > 126)
    return TBF16_ERR_INVALID;
  if (B == 0) return TBF16_OK;
  auto st = static_cast<cudaStream_t>(stream);
  if (int rc = launch_sample_amax(x, B, n, ld, amax_ws, st)) return rc;
  sample_exp_kernel<<<(unsigned)((B + 255) / 256), 256, 0, st>>>(amax_ws, B, target_exp, e, out_scale);
  return tbf16_host::check_launch();
}

int tbf16_conv_im2col(const void* x, const int64_t* geom, int64_t K, int64_t Kp, const int32_t* e,
                      const float* out_scale, void* cols16, float* row_scale, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (!x || !geom || !e || !out_scale || !cols16 || !row_scale) return TBF16_ERR_INVALID;
  const Geom g = load_geom(geom);
  if (!geom_ok(g) || K != g.C * g.kd * g.kh * g.kw || Kp < K || Kp % 8) return TBF16_ERR_INVALID;
  if (!tbf16_host::aligned16(cols16)) return TBF16_ERR_ALIGN;
  const int64_t M = g.B * g.Do * g.Ho * g.Wo;
  if (M == 0) return TBF16_OK;
  im2col_kernel<<<grid_for(M * (Kp / 8)), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), g, K, Kp, e, out_scale, static_cast<uint4*>(cols16), row_scale);
  return tbf16_host::check_launch();
}

int tbf16_conv_im2col_cl(const void* x, const int64_t* geom, const int32_t* e, const float* out_scale, void* x16cl,
                         void* cols16, float* row_scale, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (!x || !geom || !e || !out_scale || !x16cl || !cols16 || !row_scale) return TBF16_ERR_INVALID;
  const Geom g = load_geom(geom);
  if (!geom_ok(g)) return TBF16_ERR_INVALID;
  if (g.C % 8) return TBF16_ERR_UNSUPPORTED;
  if (!tbf16_host::aligned16(x16cl) || !tbf16_host::aligned16(cols16)) return TBF16_ERR_ALIGN;
  const int64_t M = g.B * g.Do * g.Ho * g.Wo;
  if (M == 0) return TBF16_OK;
  auto st = static_cast<cudaStream_t>(stream);
  // the input is one flat channels-last array per sample when its strides say so (and 16-byte aligned)
  const int flat = g.sc == 1 && g.sw == g.C && g.sh == g.W * g.C && g.sd == g.H * g.W * g.C &&
                   (g.B == 1 || g.sb % 8 == 0) && tbf16_host::aligned16(x);
  scale_cl_kernel<<<grid_for(g.B * g.D * g.H * g.W * (g.C / 8)), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(x), g, const_cast<int32_t*>(e), static_cast<uint4*>(x16cl), flat);
  const tbf16_host::DeviceInfo* d = tbf16_host::device_info();
  const int64_t want = (int64_t)(d ? d->sms : 148) * 16, need = (M + 7) / 8;  // 8 output positions per block
  const int64_t blocks = need < want ? need : want;
  im2col_cl_kernel<<<(unsigned)blocks, 256, 0, st>>>(static_cast<const uint4*>(x16cl), g, out_scale,
                                                     static_cast<uint4*>(cols16), row_scale);
  return tbf16_host::check_launch();
}

int tbf16_conv_implicit_supported(const int64_t* geom, int64_t O) {
  if (!geom) return TBF16_ERR_INVALID;
  const Geom g = load_geom(geom);
  if (!geom_ok(g) || O <= 0) return TBF16_ERR_INVALID;
  return implicit_ok(g, O) ? TBF16_OK : TBF16_ERR_UNSUPPORTED;
}

int tbf16_conv_implicit(const void* x, const int64_t* geom, int target_exp, float* amax_ws, int32_t* e,
                        float* out_scale, void* x16cl, const void* wtap16, int64_t O, const float* ws, const void* bias,
                        void* y, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (!x || !geom || !amax_ws || !e || !out_scale || !x16cl || !wtap16 || !ws || !y || O <= 0 || target_exp < -126 ||
      target_exp > 126)
    return TBF16_ERR_INVALID;
  const Geom g = load_geom(geom);
  if (!geom_ok(g)) return TBF16_ERR_INVALID;
  if (!implicit_ok(g, O) || !dense_samples(g)) return TBF16_ERR_UNSUPPORTED;
  if (!tbf16_host::aligned16(x16cl) || !tbf16_host::aligned16(wtap16) || !tbf16_host::aligned16(y))
    return TBF16_ERR_ALIGN;
  const int64_t M = g.B * g.Do * g.Ho * g.Wo;
  if (M == 0) return TBF16_OK;
  auto st = static_cast<cudaStream_t>(stream);
  const int64_t n = g.C * g.D * g.H * g.W;
  if (int rc = launch_sample_amax(x, g.B, n, g.B > 1 ? g.sb : n, amax_ws, st)) return rc;
  const int flat = g.sc == 1 && g.sw == g.C && g.sh == g.W * g.C && g.sd == g.H * g.W * g.C &&
                   (g.B == 1 || g.sb % 8 == 0) && tbf16_host::aligned16(x);
  scale_cl_kernel<<<grid_for(g.B * g.D * g.H * g.W * (g.C / 8)), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(x), g, e, static_cast<uint4*>(x16cl), flat, amax_ws, target_exp, out_scale);
  if (int rc = tbf16_host::check_launch()) return rc;
  ConvGemm cv;
  cv.Wo = (int)g.Wo;
  cv.Ho = (int)g.Ho;
  cv.Do = (int)g.Do;
  cv.cb = (int)((g.C + 63) / 64);
  cv.kh = (int)g.kh;
  cv.kw = (int)g.kw;
  cv.pw = (int)g.pw;
  cv.ph = (int)g.ph;
  cv.pd = (int)g.pd;
  cv.dw = (int)g.dw;
  cv.dh = (int)g.dh;
  cv.dd = (int)g.dd;
  cv.sa_div = (int)(g.Do * g.Ho * g.Wo);
  const int64_t K = g.kd * g.kh * g.kw * cv.cb * 64;
  return tbf16_host::conv_gemm_pair(x16cl, g.B, g.D, g.H, g.W, g.C, cv, wtap16, K, (int)M, (int)O, out_scale, ws, bias,
                                    y, O, st);
}

int tbf16_conv_grouped(const void* x, const int64_t* geom, int64_t O, int64_t groups, const void* w16, const float* ws,
                       const void* bias, const int32_t* e, const float* out_scale, void* y, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (!x || !geom || !w16 || !ws || !e || !out_scale || !y || O <= 0 || groups <= 0) return TBF16_ERR_INVALID;
  const Geom g = load_geom(geom);
  if (!geom_ok(g) || g.C % groups || O % groups) return TBF16_ERR_INVALID;
  const int64_t total = g.B * O * g.Do * g.Ho * g.Wo;
  if (total == 0) return TBF16_OK;
  conv_grouped_kernel<<<grid_for(total), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), g, O, groups, static_cast<const __half*>(w16), ws,
      static_cast<const __nv_bfloat16*>(bias), e, out_scale, static_cast<__nv_bfloat16*>(y));
  return tbf16_host::check_launch();
}

}  // extern "C"
