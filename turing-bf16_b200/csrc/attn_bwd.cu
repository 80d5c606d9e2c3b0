// Scaled fp16 flash-attention backward for sm_100a (tcgen05 + TMA): the backward of the reference's
// ScaledSDPAFn (tbf16/autograd.py:166-193) with its per-call power-of-two scaling of dO.
//
//   G    = (12 - ceil(log2 D)) - max_{b,h}(head_exp(dout) + ev_q)      (t_do passed in, autograd.py:175-178)
//   dO16 = fp16(dout * 2^(ev_q + G)),  delta = rowsum(dO16 * O16)        (O16: the forward's fp16 output)
//   P    = exp(scale * q16 k16^T + mask - lse),  dS = P * (dO16 v16^T - delta)
//   dq = bf16(scale * dS k16 * 2^(a - G)), dk = bf16(scale * dS^T q16 * 2^(-a - G)), dv = bf16(P^T dO16 * 2^(-ev - G))
// with fp32 accumulation throughout and one bf16 rounding per gradient (the reference rounds dq16, dk16,
// dv16 to fp16 first and reduces GQA heads in fp32 afterwards; here the GQA sum happens in TMEM).
//
// Main kernel: one CTA per 128-key tile of one (batch, kv head), looping over the GQA group's query
// heads and 128-row query tiles. Everything is computed with keys as TMEM lanes, so no operand needs a
// transpose: the same shared tiles serve as K-major or MN-major UMMA operands.
//   warp 0     TMA: K, V once; Q_i, dO_i per query tile
//   warp 1     MMA: S^T = K Q^T, dP^T = V dO^T, dV += P^T dO, dK += dS^T Q, dQ = dS K
//   warps 2-5  one key per thread: P^T, dS^T (fp16, 128B-swizzled K-major tiles in shared memory);
//              at the end dK, dV from TMEM -> bf16
//   warps 6-9  one query per thread: dQ from TMEM, float4 atomic adds into an fp32 accumulator
// TMEM: S^T [0,128), dP^T / dQ [128,256), dV [256,256+D), dK [256+D,256+2D). Bounded waits throughout.
#include <algorithm>

#include "common.cuh"

using namespace tbf16;

namespace {

constexpr int BQ = 128;   // queries per tile
constexpr int BKV = 128;  // keys per CTA
constexpr int kThreads = 32 * 10;

struct AttnBwdParams {
  int B, Hq, Hkv, Sq, Sk, group;
  float scale, scale_log2;
  int causal;
  const float* lse;         // [B*Hq, lse_ld] natural log
  const float* delta;       // [B*Hq, lse_ld]
  int64_t lse_ld;           // row stride of lse and delta: Sq rounded up to a multiple of 128
  float* dq_acc;            // [B*Hq*Sq*D]
  __nv_bfloat16* dk;        // [B*Hkv*Sk*D]
  __nv_bfloat16* dv;
  const int32_t* a;         // scalar
  const int32_t* ev;        // [B*Hkv]
  const int32_t* G;         // scalar
  const uint16_t* mask;     // fp16 additive, nullable
  int64_t mb, mh, mi;
  unsigned int* err;
  unsigned int* flag;       // bit 2: non-finite values seen
  int q_tiles;
};

template <int D>
struct BwdCfg {
  static constexpr int ATOMS = D / 64;
  static constexpr int TILE = ATOMS * 16384;  // 128 rows x D fp16
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = K_OFF + TILE;
  static constexpr int Q_OFF = V_OFF + TILE;
  static constexpr int DO_OFF = Q_OFF + TILE;
  static constexpr int P_OFF = DO_OFF + TILE;
  static constexpr int DS_OFF = P_OFF + 32768;
  static constexpr int VEC_OFF = DS_OFF + 32768;  // lse (log2 units) and delta of the query tile
  static constexpr int BAR_OFF = VEC_OFF + 1024;
  static constexpr int SMEM = 1024 + BAR_OFF + 256;
  static constexpr uint32_t T_S = 0, T_DP = 128, T_DV = 256, T_DK = 256 + D;
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(256 + 2 * D <= 512, "TMEM");
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t swz_off(int r, int c) {
  return (uint32_t)((c >> 3) * 16384 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const AttnBwdParams p) {
  using C = BwdCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;
  uint64_t* qdo_empty = bars + 2;
  uint64_t* s_full = bars + 3;
  uint64_t* dp_full = bars + 4;
  uint64_t* p_ready = bars + 5;
  uint64_t* ds_ready = bars + 6;
  uint64_t* s_free = bars + 7;
  uint64_t* pds_free = bars + 8;
  uint64_t* dq_full = bars + 9;
  uint64_t* dq_empty = bars + 10;
  uint64_t* kv_done = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* lse_s = reinterpret_cast<float*>(smem + C::VEC_OFF);
  float* delta_s = lse_s + 128;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bhk = blockIdx.y;
  const int b = bhk / p.Hkv, hk = bhk % p.Hkv;
  const int k0 = blockIdx.x * BKV;
  const int i_first = p.causal ? k0 / BQ : 0;  // query tiles that see these keys (top-left causal)
  const int n_i = max(0, p.q_tiles - i_first);
  const int n_t = p.group * n_i;              // (query head, query tile) pairs

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(qdo_full, 1);
    mbar_init(qdo_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_ready, 4);
    mbar_init(ds_ready, 4);
    mbar_init(s_free, 4);
    mbar_init(pds_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 4);
    mbar_init(kv_done, 1);
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * C::TILE);
#pragma unroll
      for (int a = 0; a < C::ATOMS; ++a) {
        tma_load_3d(smem + C::K_OFF + a * 16384, &tmK, kv_full, a * 64, k0, bhk);
        tma_load_3d(smem + C::V_OFF + a * 16384, &tmV, kv_full, a * 64, k0, bhk);
      }
      for (int t = 0; t < n_t; ++t) {
        const int h = hk * p.group + t / n_i;
        const int q0 = (i_first + t % n_i) * BQ;
        const int bh = b * p.Hq + h;
        if (!mbar_wait(qdo_empty, (t & 1) ^ 1, abort, p.err)) break;
        mbar_arrive_expect_tx(qdo_full, 2 * C::TILE + 1024);
#pragma unroll
        for (int a = 0; a < C::ATOMS; ++a) {
          tma_load_3d(smem + C::Q_OFF + a * 16384, &tmQ, qdo_full, a * 64, q0, bh);
          tma_load_3d(smem + C::DO_OFF + a * 16384, &tmDO, qdo_full, a * 64, q0, bh);
        }
        // this tile's 128 lse and delta values (rows padded to 128, so always in bounds and aligned)
        bulk_load(lse_s, p.lse + (int64_t)bh * p.lse_ld + q0, 512, qdo_full);
        bulk_load(delta_s, p.delta + (int64_t)bh * p.lse_ld + q0, 512, qdo_full);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_sq = idesc_f16_f32(128, 128, false, false);  // S^T, dP^T
      constexpr uint32_t id_kd = idesc_f16_f32(128, D, false, true);     // dV, dK
      constexpr uint32_t id_q = idesc_f16_f32(128, D, true, true);       // dQ
      const uint32_t k_addr = smem_u32(smem + C::K_OFF), v_addr = smem_u32(smem + C::V_OFF);
      const uint32_t q_addr = smem_u32(smem + C::Q_OFF), do_addr = smem_u32(smem + C::DO_OFF);
      const uint32_t p_addr = smem_u32(smem + C::P_OFF), ds_addr = smem_u32(smem + C::DS_OFF);
      bool ok = mbar_wait(kv_full, 0, abort, p.err);
      for (int t = 0; ok && t < n_t; ++t) {
        const uint32_t ph = t & 1;
        if (!mbar_wait(qdo_full, ph, abort, p.err) || !mbar_wait(s_free, ph ^ 1, abort, p.err)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {  // S^T = K Q^T
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_f16_ss(tmem + C::T_S, smem_desc_sw128(k_addr + off, 16, 1024), smem_desc_sw128(q_addr + off, 16, 1024),
                      id_sq, kk > 0);
        }
        umma_commit(s_full);
        if (!mbar_wait(dq_empty, ph ^ 1, abort, p.err)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {  // dP^T = V dO^T
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_f16_ss(tmem + C::T_DP, smem_desc_sw128(v_addr + off, 16, 1024), smem_desc_sw128(do_addr + off, 16, 1024),
                      id_sq, kk > 0);
        }
        umma_commit(dp_full);
        if (!mbar_wait(p_ready, ph, abort, p.err)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {  // dV += P^T dO   (dO MN-major: D contiguous)
          umma_f16_ss(tmem + C::T_DV, smem_desc_sw128(p_addr + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                      smem_desc_sw128(do_addr + kk * 2048, 16384, 1024), id_kd, (t > 0 || kk > 0));
        }
        if (!mbar_wait(ds_ready, ph, abort, p.err)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {  // dK += dS^T Q   (Q MN-major)
          umma_f16_ss(tmem + C::T_DK, smem_desc_sw128(ds_addr + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                      smem_desc_sw128(q_addr + kk * 2048, 16384, 1024), id_kd, (t > 0 || kk > 0));
        }
        umma_commit(qdo_empty);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {  // dQ = dS K   (dS^T read MN-major, K MN-major)
          umma_f16_ss(tmem + C::T_DP, smem_desc_sw128(ds_addr + kk * 2048, 16384, 1024),
                      smem_desc_sw128(k_addr + kk * 2048, 16384, 1024), id_q, kk > 0);
        }
        umma_commit(dq_full);
        umma_commit(pds_free);
      }
      if (ok) umma_commit(kv_done);
    }
  } else if (warp < 6) {
    // ---------------------------------------------------------------- P^T and dS^T, one key per thread
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // key within the tile
    const int kj = k0 + r;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    bool ok = true;
    bool bad = false;
    for (int t = 0; t < n_t; ++t) {
      const uint32_t ph = t & 1;
      const int h = hk * p.group + t / n_i;
      const int q0 = (i_first + t % n_i) * BQ;
      // Q, dO, lse and delta of this tile have landed (qdo_full), and S^T is in TMEM (s_full)
      if (!mbar_wait_warp(qdo_full, ph, abort, p.err) || !mbar_wait_warp(s_full, ph, abort, p.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // P for this thread's key against the 128 queries, kept as packed fp16 pairs (the operand the dV
      // MMA consumes; dS below reuses it, so P is rounded once for both). 32 logits at a time.
      uint32_t pp[BQ / 2];
      // Fully valid tiles (no user mask, all keys and queries in range, whole tile below the causal
      // diagonal) skip the per-element checks: P = 2^(s * c - lse * log2 e).
      const bool full_tile = p.mask == nullptr && k0 + BKV <= p.Sk && q0 + BQ <= p.Sq && (!p.causal || k0 + BKV - 1 <= q0);
      const uint16_t* mrow = p.mask ? p.mask + b * p.mb + h * p.mh + (int64_t)q0 * p.mi + min(kj, p.Sk - 1) : nullptr;
#pragma unroll
      for (int c = 0; c < BQ / 32; ++c) {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_base + C::T_S + c * 32, rr);
        tmem_ld_wait();
        float pc[32];
        if (full_tile) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            pc[e] = ex2(fmaf(__uint_as_float(rr[e]), p.scale_log2, -lse_s[c * 32 + e] * 1.4426950408889634f));
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int col = c * 32 + e;
            const int qi = q0 + col;
            const bool valid = kj < p.Sk && qi < p.Sq && (!p.causal || kj <= qi);
            float s = __uint_as_float(rr[e]) * p.scale_log2;
            if (mrow && valid) s += __half2float(__ushort_as_half(mrow[(int64_t)col * p.mi])) * 1.4426950408889634f;
            pc[e] = valid ? ex2(s - lse_s[col] * 1.4426950408889634f) : 0.f;
          }
        }
#pragma unroll
        for (int e = 0; e < 32; e += 2) pp[c * 16 + e / 2] = pack_f16(pc[e], pc[e + 1]);
      }
      if (t > 0 && !mbar_wait_warp(pds_free, (t - 1) & 1, abort, p.err)) { ok = false; break; }
      uint8_t* pt = smem + C::P_OFF;
#pragma unroll
      for (int c = 0; c < BQ / 8; ++c)
        *reinterpret_cast<uint4*>(pt + swz_off(r, c)) = make_uint4(pp[4 * c], pp[4 * c + 1], pp[4 * c + 2], pp[4 * c + 3]);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
      if (!mbar_wait_warp(dp_full, ph, abort, p.err)) { ok = false; break; }
      tc_fence_after();
      uint8_t* dst = smem + C::DS_OFF;
#pragma unroll
      for (int c = 0; c < BQ / 32; ++c) {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_base + C::T_DP + c * 32, rr);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int col = c * 32 + e;
          const float p0 = f16lo(pp[col / 2]), p1 = f16hi(pp[col / 2]);
          // masked / padded queries have P = 0 (their delta slot may hold padding): dS = 0 there
          const float d0 = p0 != 0.f ? p0 * (__uint_as_float(rr[e]) - delta_s[col]) : 0.f;
          const float d1 = p1 != 0.f ? p1 * (__uint_as_float(rr[e + 1]) - delta_s[col + 1]) : 0.f;
          bad |= !isfinite(d0) || !isfinite(d1);
          pk[e / 2] = pack_f16(d0, d1);
        }
#pragma unroll
        for (int g = 0; g < 4; ++g)
          *reinterpret_cast<uint4*>(dst + swz_off(r, c * 4 + g)) = make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(ds_ready);
        mbar_arrive(s_free);
      }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(p.flag, kErrOverflow);
    // dK, dV epilogue
    if (ok && n_t > 0 && mbar_wait_warp(kv_done, 0, abort, p.err)) {
      tc_fence_after();
      const float sk = p.scale * exp2i(-__ldg(p.a) - __ldg(p.G));
      const float sv = exp2i(-__ldg(p.ev + bhk) - __ldg(p.G));
      const int64_t orow = ((int64_t)bhk * p.Sk + min(kj, p.Sk - 1)) * D;
      bool nf = false;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        __nv_bfloat16* dst = (which ? p.dk : p.dv) + orow;
        const float f = which ? sk : sv;
        const uint32_t col0 = which ? C::T_DK : C::T_DV;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + col0 + c * 32, o);
          tmem_ld_wait();
          if (kj < p.Sk) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              float v[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                v[e] = __uint_as_float(o[8 * g + e]) * f;
                nf |= !isfinite(v[e]);
              }
              *reinterpret_cast<uint4*>(dst + c * 32 + g * 8) =
                  make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
            }
          }
        }
      }
      if (__any_sync(0xffffffffu, nf) && lane == 0) atomicOr(p.flag, kErrOverflow);
    } else if (n_t == 0 && kj < p.Sk) {  // keys no query sees (causal, Sk > Sq): zero gradients
      const int64_t orow = ((int64_t)bhk * p.Sk + kj) * D;
      for (int c = 0; c < D; c += 8) {
        *reinterpret_cast<uint4*>(p.dk + orow + c) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(p.dv + orow + c) = make_uint4(0, 0, 0, 0);
      }
    }
  } else {
    // ---------------------------------------------------------------- dQ: one query per thread, atomics
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    for (int t = 0; t < n_t; ++t) {
      const int h = hk * p.group + t / n_i;
      const int qi = (i_first + t % n_i) * BQ + r;
      if (!mbar_wait_warp(dq_full, t & 1, abort, p.err)) break;
      tc_fence_after();
      float* dst = p.dq_acc + ((int64_t)(b * p.Hq + h) * p.Sq + min(qi, p.Sq - 1)) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + C::T_DP + c * 32, o);
        tmem_ld_wait();
        if (qi < p.Sq) {
#pragma unroll
          for (int g = 0; g < 8; ++g)
            atomicAdd(reinterpret_cast<float4*>(dst + c * 32 + 4 * g),
                      make_float4(__uint_as_float(o[4 * g]), __uint_as_float(o[4 * g + 1]), __uint_as_float(o[4 * g + 2]),
                                  __uint_as_float(o[4 * g + 3])));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_empty);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort) {
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 2000000ull) {
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// G = t_do - max_{b,h}(frexp(amax_do[b,h]) + ev[b, h / group]); one block.
__global__ void __launch_bounds__(256) attn_bwd_exp_kernel(const float* __restrict__ amax_do, int BHq, int Hq, int Hkv,
                                                           int group, const int32_t* __restrict__ ev, int t_do,
                                                           int32_t* __restrict__ G) {
  __shared__ int red[8];
  int e = INT_MIN;
  for (int i = threadIdx.x; i < BHq; i += blockDim.x) {
    const int b = i / Hq, h = i % Hq;
    e = max(e, frexp_exp(amax_do[i]) + ev[b * Hkv + h / group]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) e = max(e, __shfl_xor_sync(0xffffffffu, e, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = e;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 0; w < (int)blockDim.x / 32; ++w) e = max(e, red[w]);
    *G = t_do - e;
  }
}

// dO16 = fp16(dout * 2^(ev_q + G)) (contiguous, D columns, zero beyond D0) and delta = rowsum(dO16 * O16).
// One thread per 8 columns; D/8 threads per row.
template <int D>
__global__ void __launch_bounds__(256) attn_bwd_prep_kernel(const uint16_t* __restrict__ dout, int64_t sb, int64_t sh,
                                                            int64_t ss, int D0, const __half* __restrict__ o16,
                                                            const int32_t* __restrict__ ev, const int32_t* __restrict__ G,
                                                            int Hq, int Hkv, int group, int Sq, int64_t rows,
                                                            int64_t lse_ld, __half* __restrict__ do16,
                                                            float* __restrict__ delta) {
  constexpr int TPR = D / 8;
  const int64_t row = (int64_t)blockIdx.x * (256 / TPR) + threadIdx.x / TPR;
  const int c = (threadIdx.x % TPR) * 8;
  float acc = 0.f;
  if (row < rows) {
    const int64_t bh = row / Sq;
    const int i = (int)(row % Sq);
    const int b = (int)(bh / Hq), h = (int)(bh % Hq);
    const float sc = exp2i(__ldg(ev + b * Hkv + h / group) + __ldg(G));
    float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (c < D0) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(dout + b * sb + h * sh + (int64_t)i * ss + c));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        f[2 * j] = bf16lo(w[j]) * sc;
        f[2 * j + 1] = bf16hi(w[j]) * sc;
      }
    }
    uint4 hv;
    hv.x = pack_f16(f[0], f[1]); hv.y = pack_f16(f[2], f[3]); hv.z = pack_f16(f[4], f[5]); hv.w = pack_f16(f[6], f[7]);
    *reinterpret_cast<uint4*>(do16 + row * D + c) = hv;
    const uint4 ov = __ldg(reinterpret_cast<const uint4*>(o16 + row * D + c));
    const uint32_t dw[4] = {hv.x, hv.y, hv.z, hv.w}, owd[4] = {ov.x, ov.y, ov.z, ov.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) acc += f16lo(dw[j]) * f16lo(owd[j]) + f16hi(dw[j]) * f16hi(owd[j]);
  }
#pragma unroll
  for (int o = TPR / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (row < rows && threadIdx.x % TPR == 0) delta[(row / Sq) * lse_ld + row % Sq] = acc;
}

// dq = bf16(dq_acc * scale * 2^(a - G)), contiguous (B, Hq, Sq, D).
__global__ void __launch_bounds__(256) attn_bwd_dq_kernel(const float4* __restrict__ acc, int64_t n4, float scale,
                                                          const int32_t* __restrict__ a, const int32_t* __restrict__ G,
                                                          uint2* __restrict__ dq, unsigned int* flag) {
  const float f = scale * exp2i(__ldg(a) - __ldg(G));
  bool nf = false;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = acc[i];
    const float x0 = v.x * f, x1 = v.y * f, x2 = v.z * f, x3 = v.w * f;
    nf |= !isfinite(x0) || !isfinite(x1) || !isfinite(x2) || !isfinite(x3);
    dq[i] = make_uint2(pack_bf16(x0, x1), pack_bf16(x2, x3));
  }
  if (nf) atomicOr(flag, kErrOverflow);
}

struct Workspace {
  float* dq_acc;
  __half* do16;
  float* delta;
  float* amax;
};

int64_t lse_stride(int64_t Sq) { return (Sq + 127) / 128 * 128; }

Workspace carve(void* ws, int64_t B, int64_t Hq, int64_t Sq, int64_t D) {
  uint8_t* p = static_cast<uint8_t*>(ws);
  Workspace w;
  const int64_t n = B * Hq * Sq * D;
  w.dq_acc = reinterpret_cast<float*>(p);
  p += ((4 * n + 255) / 256) * 256;
  w.do16 = reinterpret_cast<__half*>(p);
  p += ((2 * n + 255) / 256) * 256;
  w.delta = reinterpret_cast<float*>(p);
  p += ((4 * B * Hq * lse_stride(Sq) + 255) / 256) * 256;
  w.amax = reinterpret_cast<float*>(p);
  return w;
}

int64_t workspace_bytes(int64_t B, int64_t Hq, int64_t Sq, int64_t D) {
  const int64_t n = B * Hq * Sq * D;
  return ((4 * n + 255) / 256) * 256 + ((2 * n + 255) / 256) * 256 + ((4 * B * Hq * lse_stride(Sq) + 255) / 256) * 256 +
         ((4 * B * Hq + 255) / 256) * 256;
}

template <int D>
int launch_bwd(const void* q16, const void* k16, const void* v16, const void* do16, const AttnBwdParams& prm,
               int64_t Sk, cudaStream_t st) {
  using C = BwdCfg<D>;
  const tbf16_host::DeviceInfo* dev = tbf16_host::device_info();
  CUtensorMap tq, tk, tv, tdo;
  const int64_t BHq = (int64_t)prm.B * prm.Hq, BHk = (int64_t)prm.B * prm.Hkv;
  if (int rc = tbf16_host::make_tmap_3d(&tq, q16, D, prm.Sq, BHq, D, (uint64_t)prm.Sq * D, 64, BQ)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tdo, do16, D, prm.Sq, BHq, D, (uint64_t)prm.Sq * D, 64, BQ)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tk, k16, D, Sk, BHk, D, (uint64_t)Sk * D, 64, BKV)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tv, v16, D, Sk, BHk, D, (uint64_t)Sk * D, 64, BKV)) return rc;
  static bool attr_done[64] = {false};
  if (!attr_done[dev->device & 63]) {
    if (cudaFuncSetAttribute(attn_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
      return tbf16_host::check_launch();
    attr_done[dev->device & 63] = true;
  }
  dim3 grid((unsigned)((Sk + BKV - 1) / BKV), (unsigned)BHk);
  attn_bwd_kernel<D><<<grid, kThreads, C::SMEM, st>>>(tq, tk, tv, tdo, prm);
  return tbf16_host::check_launch();
}

}  // namespace

extern "C" {

int64_t tbf16_attn_bwd_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D) {
  (void)Hkv;
  (void)Sk;
  if (B < 0 || Hq < 0 || Sq < 0 || D <= 0) return -1;
  return workspace_bytes(B, Hq, Sq, D);
}

int tbf16_attn_bwd(const void* q16, const void* k16, const void* v16, const void* o16, const float* lse, int64_t lse_ld,
                   const void* dout,
                   int64_t dout_sb, int64_t dout_sh, int64_t dout_ss, int64_t dout_d, const int32_t* a, const int32_t* ev,
                   int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, float scale, int causal,
                   const void* mask, int64_t mask_sb, int64_t mask_sh, int64_t mask_sq, int t_do, void* dq, void* dk,
                   void* dv, int32_t* G_out, unsigned int* flag, void* ws, int64_t ws_bytes, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Sq <= 0 || Sk <= 0 || dout_d <= 0 || dout_d > D || !a || !ev ||
      !lse || lse_ld != lse_stride(Sq) || !G_out || !flag || !ws || B * Hq > 65535 || B * Hkv > 65535)
    return TBF16_ERR_INVALID;
  if (D != 64 && D != 128) return TBF16_ERR_UNSUPPORTED;
  if (ws_bytes < workspace_bytes(B, Hq, Sq, D)) return TBF16_ERR_INVALID;
  if (!tbf16_host::aligned16(q16) || !tbf16_host::aligned16(k16) || !tbf16_host::aligned16(v16) ||
      !tbf16_host::aligned16(o16) || !tbf16_host::aligned16(dout) || !tbf16_host::aligned16(dq) ||
      !tbf16_host::aligned16(dk) || !tbf16_host::aligned16(dv) || !tbf16_host::aligned16(ws) || dout_d % 8 ||
      dout_sb % 8 || dout_sh % 8 || dout_ss % 8)
    return TBF16_ERR_ALIGN;
  const tbf16_host::DeviceInfo* dev = tbf16_host::device_info();
  auto st = static_cast<cudaStream_t>(stream);
  Workspace w = carve(ws, B, Hq, Sq, D);
  const int group = (int)(Hq / Hkv);
  // 1. G from the global max of head_exp(dout) + ev_q
  if (int rc = tbf16_head_amax(dout, TBF16_BF16, B, Hq, Sq, dout_d, dout_sb, dout_sh, dout_ss, w.amax, stream)) return rc;
  attn_bwd_exp_kernel<<<1, 256, 0, st>>>(w.amax, (int)(B * Hq), (int)Hq, (int)Hkv, group, ev, t_do, G_out);
  // 2. dO16 and delta
  const int64_t rows = B * Hq * Sq;
  const int rpb = 256 / (int)(D / 8);
  const unsigned pgrid = (unsigned)((rows + rpb - 1) / rpb);
  if (D == 64)
    attn_bwd_prep_kernel<64><<<pgrid, 256, 0, st>>>(static_cast<const uint16_t*>(dout), dout_sb, dout_sh, dout_ss,
                                                    (int)dout_d, static_cast<const __half*>(o16), ev, G_out, (int)Hq,
                                                    (int)Hkv, group, (int)Sq, rows, lse_ld, w.do16, w.delta);
  else
    attn_bwd_prep_kernel<128><<<pgrid, 256, 0, st>>>(static_cast<const uint16_t*>(dout), dout_sb, dout_sh, dout_ss,
                                                     (int)dout_d, static_cast<const __half*>(o16), ev, G_out, (int)Hq,
                                                     (int)Hkv, group, (int)Sq, rows, lse_ld, w.do16, w.delta);
  // 3. main kernel (dQ accumulated in fp32)
  if (cudaMemsetAsync(w.dq_acc, 0, sizeof(float) * rows * D, st) != cudaSuccess) return TBF16_ERR_LAUNCH;
  AttnBwdParams prm;
  prm.B = (int)B; prm.Hq = (int)Hq; prm.Hkv = (int)Hkv; prm.Sq = (int)Sq; prm.Sk = (int)Sk; prm.group = group;
  prm.scale = scale;
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.causal = causal;
  prm.lse = lse; prm.delta = w.delta; prm.dq_acc = w.dq_acc; prm.lse_ld = lse_ld;
  prm.dk = static_cast<__nv_bfloat16*>(dk);
  prm.dv = static_cast<__nv_bfloat16*>(dv);
  prm.a = a; prm.ev = ev; prm.G = G_out;
  prm.mask = static_cast<const uint16_t*>(mask);
  prm.mb = mask_sb; prm.mh = mask_sh; prm.mi = mask_sq;
  prm.err = dev->err;
  prm.flag = flag;
  prm.q_tiles = (int)((Sq + BQ - 1) / BQ);
  int rc = D == 64 ? launch_bwd<64>(q16, k16, v16, w.do16, prm, Sk, st) : launch_bwd<128>(q16, k16, v16, w.do16, prm, Sk, st);
  if (rc) return rc;
  // 4. dq
  const int64_t n4 = rows * D / 4;
  const int g = (int)std::min<int64_t>((n4 + 255) / 256, (int64_t)dev->sms * 16);
  attn_bwd_dq_kernel<<<g, 256, 0, st>>>(reinterpret_cast<const float4*>(w.dq_acc), n4, scale, a, G_out,
                                        static_cast<uint2*>(dq), flag);
  return tbf16_host::check_launch();
}

}  // extern "C"
