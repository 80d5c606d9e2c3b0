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
// transpose: the same shared tiles serve as K-major or MN-major UMMA operands. Four warpgroups, their
// registers re-split with setmaxnreg (96 for the control group, 128 for the key warps, 160 for dQ):
//   warp 0      TMA: K, V once; Q_i (+ lse, delta) per query tile, 2 stages
//   warp 1      MMA: S^T = K Q^T, dP^T = V dO^T, dV += P^T dO, dK += dS^T Q, dQ = dS K
//   warp 2      TMA: dO_i, 1 stage
//   warps 4-11  key warps, two per TMEM lane quadrant, each half of the query columns: P^T (packed
//               fp16 back into TMEM), dS^T (fp16, 128B-swizzled K-major tile in shared memory), and at
//               the end half the columns of dK, dV from TMEM -> bf16
//   warps 12-15 dQ warps, one per TMEM lane quadrant. D = 128: the tensor core computes dQ^T = K^T dS^T
//               (head dims as lanes), each thread reads its d's 128 query columns at once (which frees
//               them for the next dP) and adds them into the fp32 accumulator with red.global.add, the
//               warp's 32 consecutive d making each instruction one 128-byte segment (no shared-memory
//               staging). D = 64: dQ = dS K with queries as lanes, TMA reduce-adds of 32-column boxes
//               from two alternating staging buffers.
// The key warps only compute P and dS, so the tile loop is dS(t) -> P(t+1) -> dS(t+1) while the tensor
// core runs dQ(t), dK(t), dP(t+1), dV(t+1), S(t+2) and the dQ warps drain dQ(t) alongside.
// TMEM: S^T [0,128), dP^T / dQ [128,256), dV [256,256+D), dK [256+D,256+2D). Bounded waits throughout.
#include <algorithm>

#include "common.cuh"

using namespace tbf16;

namespace {

constexpr int BQ = 128;   // queries per tile
constexpr int BKV = 128;  // keys per CTA
constexpr int kThreads = 32 * 16;
// setmaxnreg shares per warpgroup (128 threads): control 96 (the MMA issuer keeps its operand
// descriptors in registers), key warps 128 (the launch value: no re-split), dQ warps 160 (all D = 128
// columns of a query row at once). Their sum must not exceed the 512-thread launch's 65536 registers.
constexpr uint32_t kRegsCtl = 96;
constexpr uint32_t kRegsKey = 128;
constexpr uint32_t kRegsDq = 160;
static_assert(128 * (kRegsCtl + 2 * kRegsKey + kRegsDq) <= 65536, "register split");

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
  // attention dropout (kernels instantiated with DROP): per-row hash keys [B*Hq, lse_ld] from the prep
  // kernel, keep threshold and 1 / keep probability (see drop_keep)
  const uint32_t* rowkey;
  uint32_t drop_thr;
  float inv_keep;
};

template <int D>
struct BwdCfg {
  static constexpr int ATOMS = D / 64;
  static constexpr int TILE = ATOMS * 16384;  // 128 rows x D fp16
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = K_OFF + TILE;
  static constexpr int Q_OFF = V_OFF + TILE;      // [2 stages]
  static constexpr int DO_OFF = Q_OFF + 2 * TILE; // one stage: its readers dP(t), dV(t) finish early
  static constexpr int DS_OFF = DO_OFF + TILE;
  // D = 128: dQ is computed transposed (head dims as TMEM lanes) and added into the fp32 accumulator with
  // coalesced reductions straight from registers; D = 64 keeps queries as lanes and stages 32 x 32 boxes
  // for TMA reduce-adds (4 warps x 2 boxes of 4 KB)
  static constexpr bool DQ_T = D == 128;
  static constexpr int DQS_OFF = DS_OFF + 32768;
  // [2 stages] of the query tile's lse (natural log), delta and (with dropout) row hash keys, 128 each
  static constexpr int VEC_OFF = DQS_OFF + (DQ_T ? 0 : 32768);
  static constexpr int VEC_STAGE = 1536;
  static constexpr int BAR_OFF = VEC_OFF + 2 * VEC_STAGE;
  // the dynamic shared window starts 1024-byte aligned (checked on entry), so no alignment slack
  static constexpr int SMEM = BAR_OFF + 256;
  static constexpr uint32_t T_S = 0, T_DP = 128, T_DV = 256, T_DK = 256 + D;
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(256 + 2 * D <= 512, "TMEM");
};

template <int D, bool DROP>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmDQ, const AttnBwdParams p) {
  using C = BwdCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {  // the layout below has no alignment slack
    if (threadIdx.x == 0) atomicOr(p.err, kErrSmemAlign);
    return;
  }
  uint8_t* smem = smem_raw;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;     // [2]: Q, lse, delta of a query tile
  uint64_t* q_empty = bars + 3;    // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* dp_full = bars + 6;
  uint64_t* p_ready = bars + 7;
  uint64_t* ds_ready = bars + 8;
  uint64_t* dq_full = bars + 9;
  uint64_t* dq_empty = bars + 10;
  uint64_t* kv_done = bars + 11;
  uint64_t* do_full = bars + 12;
  uint64_t* do_empty = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // (kv head) fastest, key tiles in increasing order: under a causal mask the low key tiles see the
  // most query tiles, so the longest CTAs start first
  const int bhk = blockIdx.x;
  const int b = bhk / p.Hkv, hk = bhk % p.Hkv;
  const int k0 = blockIdx.y * BKV;
  const int i_first = p.causal ? k0 / BQ : 0;  // query tiles that see these keys (top-left causal)
  const int n_i = max(0, p.q_tiles - i_first);
  const int n_t = p.group * n_i;              // (query head, query tile) pairs

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_ready, 8);
    mbar_init(ds_ready, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 4);
    mbar_init(kv_done, 1);
    mbar_init(do_full, 1);
    mbar_init(do_empty, 1);
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

  // each role's code sits under its warpgroup's register re-split
  if (warp < 4) {
    setmaxnreg_dec<kRegsCtl>();
    if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer: K, V, then Q (2 stages)
    if (lane == 0 && n_t > 0) {  // no copies in flight when the CTA has no query tile
      mbar_arrive_expect_tx(kv_full, 2 * C::TILE);
#pragma unroll
      for (int a = 0; a < C::ATOMS; ++a) {
        tma_load_3d(smem + C::K_OFF + a * 16384, &tmK, kv_full, a * 64, k0, bhk);
        tma_load_3d(smem + C::V_OFF + a * 16384, &tmV, kv_full, a * 64, k0, bhk);
      }
      // Q, lse and delta of query tile t go to stage t & 1: the next tile loads while this one runs
      for (int t = 0; t < n_t; ++t) {
        const int h = hk * p.group + t / n_i;
        const int q0 = (i_first + t % n_i) * BQ;
        const int bh = b * p.Hq + h;
        const int st = t & 1;
        if (!mbar_wait(&q_empty[st], ((t >> 1) & 1) ^ 1, abort, p.err)) break;
        mbar_arrive_expect_tx(&q_full[st], C::TILE + 1024 + (DROP ? 512 : 0));
#pragma unroll
        for (int a = 0; a < C::ATOMS; ++a)
          tma_load_3d(smem + C::Q_OFF + st * C::TILE + a * 16384, &tmQ, &q_full[st], a * 64, q0, bh);
        // this tile's 128 lse and delta values (rows padded to 128, so always in bounds and aligned)
        float* vec = reinterpret_cast<float*>(smem + C::VEC_OFF + st * C::VEC_STAGE);
        bulk_load(vec, p.lse + (int64_t)bh * p.lse_ld + q0, 512, &q_full[st]);
        bulk_load(vec + 128, p.delta + (int64_t)bh * p.lse_ld + q0, 512, &q_full[st]);
        if constexpr (DROP) bulk_load(vec + 256, p.rowkey + (int64_t)bh * p.lse_ld + q0, 512, &q_full[st]);
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- TMA producer: dO (one stage)
    if (lane == 0 && n_t > 0) {
      for (int t = 0; t < n_t; ++t) {
        const int h = hk * p.group + t / n_i;
        const int q0 = (i_first + t % n_i) * BQ;
        if (!mbar_wait(do_empty, (t & 1) ^ 1, abort, p.err)) break;
        mbar_arrive_expect_tx(do_full, C::TILE);
#pragma unroll
        for (int a = 0; a < C::ATOMS; ++a)
          tma_load_3d(smem + C::DO_OFF + a * 16384, &tmDO, do_full, a * 64, q0, b * p.Hq + h);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    // Order per query tile t: S(t) dP(t) | dV(t) S(t+1) | dK(t) dQ(t) | dP(t+1) ... so the key warps
    // find S(t+1) ready when they finish dS(t). The MMA pipe executes in issue order: S(t+1) overwrites
    // P^T(t) after dV(t) read it; dQ(t) overwrites dP^T(t) after the key warps read it (ds_ready); when
    // dP(t+1) completes, dK(t) and dQ(t) have read dS(t), so dS(t+1) may overwrite it.
    if (lane == 0 && n_t > 0) {
      constexpr uint32_t id_sq = idesc_f16_f32(128, 128, false, false);  // S^T, dP^T
      constexpr uint32_t id_kd = idesc_f16_f32(128, D, false, true);     // dV, dK
      // dQ (M = queries, N = D) or, with DQ_T, dQ^T (M = D, N = queries): both operands MN-major
      constexpr uint32_t id_q = C::DQ_T ? idesc_f16_f32(D, 128, true, true) : idesc_f16_f32(128, D, true, true);
      // a k16 step adds its byte offset / 16 to the 14-bit start-address field (no carry: < 2^18 bytes)
      const uint64_t kd = smem_desc_sw128(smem_u32(smem + C::K_OFF), 16, 1024);
      const uint64_t vd = smem_desc_sw128(smem_u32(smem + C::V_OFF), 16, 1024);
      const uint64_t qd = smem_desc_sw128(smem_u32(smem + C::Q_OFF), 16, 1024);
      const uint64_t dod = smem_desc_sw128(smem_u32(smem + C::DO_OFF), 16, 1024);
      const uint64_t qd_mn = smem_desc_sw128(smem_u32(smem + C::Q_OFF), 16384, 1024);
      const uint64_t dod_mn = smem_desc_sw128(smem_u32(smem + C::DO_OFF), 16384, 1024);  // one stage
      const uint64_t dsd = smem_desc_sw128(smem_u32(smem + C::DS_OFF), 16, 1024);
      const uint64_t dsd_mn = smem_desc_sw128(smem_u32(smem + C::DS_OFF), 16384, 1024);
      const uint64_t kd_mn = smem_desc_sw128(smem_u32(smem + C::K_OFF), 16384, 1024);
      constexpr uint32_t kTile16 = C::TILE >> 4;
      auto issue_s = [&](int t) {  // S^T = K Q^T
        const uint64_t q = qd + (t & 1) * kTile16;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off16 = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
          umma_f16_ss(tmem + C::T_S, kd + off16, q + off16, id_sq, kk > 0);
        }
        umma_commit(s_full);
      };
      auto issue_dp = [&]() {  // dP^T = V dO^T
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off16 = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
          umma_f16_ss(tmem + C::T_DP, vd + off16, dod + off16, id_sq, kk > 0);
        }
        umma_commit(dp_full);
      };
      bool ok = mbar_wait(kv_full, 0, abort, p.err) && mbar_wait(&q_full[0], 0, abort, p.err);
      if (ok) {
        tc_fence_after();
        issue_s(0);
        ok = mbar_wait(do_full, 0, abort, p.err);
        if (ok) {
          tc_fence_after();
          issue_dp();
        }
      }
      for (int t = 0; ok && t < n_t; ++t) {
        const int st = t & 1;
        const bool next = t + 1 < n_t;
        if (!mbar_wait(p_ready, t & 1, abort, p.err)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)  // dV += P^T dO   (P^T from TMEM: queries 64h.. at column 64h; dO MN-major)
          umma_f16_ts(tmem + C::T_DV, tmem + C::T_S + (kk >> 2) * 64 + (kk & 3) * 8, dod_mn + (kk * 2048 >> 4), id_kd,
                      (t > 0 || kk > 0));
        umma_commit(do_empty);  // dP(t) and dV(t) were the readers of dO(t)
        if (next) {
          if (!mbar_wait(&q_full[st ^ 1], ((t + 1) >> 1) & 1, abort, p.err)) break;
          tc_fence_after();
          issue_s(t + 1);
        }
        if (!mbar_wait(ds_ready, t & 1, abort, p.err)) break;
        tc_fence_after();
        // dQ first: its extraction (the dQ warps) gates dP(t+1)
        if constexpr (C::DQ_T) {
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)  // dQ^T = K^T dS^T   (K MN-major as A: m = d; dS^T MN-major as B)
            umma_f16_ss(tmem + C::T_DP, kd_mn + (kk * 2048 >> 4), dsd_mn + (kk * 2048 >> 4), id_q, kk > 0);
        } else {
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)  // dQ = dS K   (dS^T read MN-major, K MN-major)
            umma_f16_ss(tmem + C::T_DP, dsd_mn + (kk * 2048 >> 4), kd_mn + (kk * 2048 >> 4), id_q, kk > 0);
        }
        umma_commit(dq_full);
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {  // dK += dS^T Q   (Q MN-major)
          const uint32_t off16 = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
          umma_f16_ss(tmem + C::T_DK, dsd + off16, qd_mn + st * kTile16 + (kk * 2048 >> 4), id_kd, (t > 0 || kk > 0));
        }
        umma_commit(&q_empty[st]);
        if (next) {
          if (!mbar_wait(dq_empty, t & 1, abort, p.err) || !mbar_wait(do_full, (t + 1) & 1, abort, p.err)) break;
          tc_fence_after();
          issue_dp();
        }
      }
      if (ok) umma_commit(kv_done);
    }
    }
  } else if (warp < 12) {  // key warps keep the launch's kRegsKey registers
    // ---------------------------------------------------------------- key warps
    // Two warps per TMEM lane quadrant: warp w handles keys 32 (w % 4) .. (one key per thread, as TMEM
    // lanes) and half h = (w - 4) / 4 of every query tile's 128 columns, i.e. queries [64 h, 64 h + 64)
    // of P^T and dS^T, and half the D columns of dK, dV. Per query tile: dS(t), then P(t+1) (S(t+1) was
    // issued right after dV(t)) while the tensor core runs dQ(t), dK(t) and dP(t+1).
    const int quad = warp & 3;
    const int half = (warp - 4) >> 2;
    const int r = quad * 32 + lane;  // key within the tile
    const int kj = k0 + r;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const int cq = half * 64;        // this warp's query columns
    bool ok = true;
    bool bad = false;
    uint32_t pp[32];  // P of this thread's key against the warp's 64 queries, packed fp16 pairs
    uint64_t keep_bits = 0;  // dropout: bit c set when query column cq + c keeps this key

    // P(t): 2^(scale s - lse) for queries [cq, cq + 64), written to TMEM over S^T columns
    // [cq, cq + 32) (inside this warp's own S^T columns) as the A operand of dV += P^T dO
    auto compute_p = [&](int t) -> bool {
      const int h = hk * p.group + t / n_i;
      const int q0 = (i_first + t % n_i) * BQ;
      const float* lse_s = reinterpret_cast<const float*>(smem + C::VEC_OFF + (t & 1) * C::VEC_STAGE);
      if (!mbar_wait_warp(&q_full[t & 1], (t >> 1) & 1, abort, p.err) || !mbar_wait_warp(s_full, t & 1, abort, p.err))
        return false;
      tc_fence_after();
      // Fully valid tiles (no user mask, keys and queries in range, whole tile below the causal diagonal)
      // go straight to the exp; 3 of every 8 exp2 pairs run on the FMA pipe. The 64 columns go in two
      // halves of 32, so only 32 logits are live at a time. Other tiles first turn S^T into scaled,
      // masked logits (-inf where masked) in TMEM with a short loop, take the same exp path with c = 1,
      // and zero P outside this key's valid query columns afterwards (padded queries' lse slots are not
      // written by the forward). A fully unrolled per-element form of this once-per-CTA path cost more
      // in instruction fetch than the tile's arithmetic.
      const bool full_tile = p.mask == nullptr && k0 + BKV <= p.Sk && q0 + BQ <= p.Sq && (!p.causal || k0 + BKV - 1 <= q0);
      uint64_t vbits = ~0ull;  // bit c: query column cq + c is valid for this key
      if (!full_tile) {
        const int lo = p.causal ? kj - q0 : 0;      // valid columns: lo <= col < hi
        const int hi = kj < p.Sk ? p.Sq - q0 : 0;
        const uint16_t* mrow = p.mask ? p.mask + b * p.mb + h * p.mh + (int64_t)q0 * p.mi + min(kj, p.Sk - 1) : nullptr;
        const uint32_t s_tm = tmem + lane_base + C::T_S + cq;
#pragma unroll 1
        for (int c = 0; c < 64; c += 32) {
          uint32_t o[32];
          tmem_ld32(s_tm + c, o);
          tmem_ld_wait();
          if (mrow) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int col = cq + c + i;
              const bool valid = col >= lo && col < hi;
              float v = __uint_as_float(o[i]) * p.scale_log2;
              if (valid) v += __half2float(__ushort_as_half(mrow[(int64_t)col * p.mi])) * 1.4426950408889634f;
              o[i] = __float_as_uint(valid ? v : -INFINITY);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int col = cq + c + i;
              o[i] = __float_as_uint(col >= lo && col < hi ? __uint_as_float(o[i]) * p.scale_log2 : -INFINITY);
            }
          }
          tmem_st32(s_tm + c, o);
        }
        tmem_st_wait();
        const int va = max(0, min(64, lo - cq)), vz = max(0, min(64, hi - cq));
        auto below = [](int n) -> uint64_t { return n >= 64 ? ~0ull : ((1ull << n) - 1); };
        vbits = vz > va ? below(vz) & ~below(va) : 0ull;
      }
      const uint64_t c2 = full_tile ? f2_pack(p.scale_log2, p.scale_log2) : f2_pack(1.f, 1.f);
      const uint64_t nl2e = f2_pack(-1.4426950408889634f, -1.4426950408889634f);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_base + C::T_S + cq + 32 * hh, rr);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const int E = 32 * hh + e;
          const float4 ls = reinterpret_cast<const float4*>(lse_s)[(cq + E) >> 2];
#pragma unroll
          for (int u = 0; u < 4; u += 2) {
            float x0, x1, p0, p1;
            const uint64_t nl = f2_mul(u == 0 ? f2_pack(ls.x, ls.y) : f2_pack(ls.z, ls.w), nl2e);
            f2_unpack(f2_fma(f2_pack(__uint_as_float(rr[e + u]), __uint_as_float(rr[e + u + 1])), c2, nl), x0, x1);
            if ((((E + u) >> 1) & 7) >= 5) {
              ex2_poly2(x0, x1, p0, p1);
            } else {
              p0 = ex2(x0);
              p1 = ex2(x1);
            }
            pp[(E + u) >> 1] = pack_f16(p0, p1);
          }
        }
      }
      if (!full_tile) {
#pragma unroll
        for (int c = 0; c < 32; ++c)
          pp[c] &= ((vbits >> (2 * c)) & 1 ? 0x0000ffffu : 0u) | ((vbits >> (2 * c + 1)) & 1 ? 0xffff0000u : 0u);
      }
      // dV(t-1) has read the previous P^T: it precedes S(t) in the MMA pipe
      if constexpr (DROP) {
        // dV sees P with the dropped entries zeroed (1 / keep probability applied to dV at the end);
        // dS keeps the full P and this thread's keep bits
        const uint32_t* rks = reinterpret_cast<const uint32_t*>(lse_s) + 256;
        uint32_t pt[32];
        uint64_t kb = 0;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const bool k0b = drop_keep(rks[cq + 2 * c], (uint32_t)kj, p.drop_thr);
          const bool k1b = drop_keep(rks[cq + 2 * c + 1], (uint32_t)kj, p.drop_thr);
          pt[c] = pp[c] & ((k0b ? 0x0000ffffu : 0u) | (k1b ? 0xffff0000u : 0u));
          kb |= (uint64_t)((k0b ? 1u : 0u) | (k1b ? 2u : 0u)) << (2 * c);
        }
        keep_bits = kb;
        tmem_st32(tmem + lane_base + C::T_S + cq, pt);
      } else {
        tmem_st32(tmem + lane_base + C::T_S + cq, pp);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
      return true;
    };

    ok = n_t > 0 && compute_p(0);
    for (int t = 0; ok && t < n_t; ++t) {
      const float* delta_s = reinterpret_cast<const float*>(smem + C::VEC_OFF + (t & 1) * C::VEC_STAGE) + 128;
      // ---- dS(t) = P (dP - delta) for this warp's 64 queries (when dP(t) completes, dK(t-1) and
      // dQ(t-1) have read dS(t-1)); masked / padded queries have P = 0 and a finite dP and delta
      // (padding rows of delta are zeroed), so their dS is 0. A dS that does not fit fp16 raises the flag.
      if (!mbar_wait_warp(dp_full, t & 1, abort, p.err)) { ok = false; break; }
      tc_fence_after();
      {
        float dmax = 0.f;  // largest |dS|: a value >= 65520 rounds to an fp16 infinity (NaN also flags)
        const uint64_t m1 = f2_pack(-1.f, -1.f);
        uint8_t* dst = smem + C::DS_OFF;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {  // two halves of 32 columns: 32 dP values live at a time
          uint32_t rr[32];
          tmem_ld32(tmem + lane_base + C::T_DP + cq + 32 * hh, rr);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const int E = 32 * hh + e;
            const float4 dl = reinterpret_cast<const float4*>(delta_s)[(cq + E) >> 2];
#pragma unroll
            for (int u = 0; u < 4; u += 2) {
              const float2 pf = __half22float2(*reinterpret_cast<const __half2*>(&pp[(E + u) >> 1]));
              uint64_t dd;
              if constexpr (DROP) {  // dP of a dropped entry is 0; kept ones are scaled by 1 / keep probability
                const float g0 = (keep_bits >> (E + u)) & 1 ? p.inv_keep : 0.f;
                const float g1 = (keep_bits >> (E + u + 1)) & 1 ? p.inv_keep : 0.f;
                dd = f2_fma(f2_pack(__uint_as_float(rr[e + u]), __uint_as_float(rr[e + u + 1])), f2_pack(g0, g1),
                            f2_mul(u == 0 ? f2_pack(dl.x, dl.y) : f2_pack(dl.z, dl.w), m1));
              } else {
                dd = f2_fma(u == 0 ? f2_pack(dl.x, dl.y) : f2_pack(dl.z, dl.w), m1,
                            f2_pack(__uint_as_float(rr[e + u]), __uint_as_float(rr[e + u + 1])));
              }
              float d0, d1;
              f2_unpack(f2_mul(f2_pack(pf.x, pf.y), dd), d0, d1);
              pk[(e + u) >> 1] = pack_f16(d0, d1);
              dmax = fmaxf(dmax, fmaxf(fabsf(d0), fabsf(d1)));
            }
          }
#pragma unroll
          for (int g = 0; g < 4; ++g)
            *reinterpret_cast<uint4*>(dst + swz_off(r, half * 8 + 4 * hh + g)) =
                make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
        }
        bad |= !(dmax < 65520.f);
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_ready);
      // ---- P(t+1) while the tensor core runs dQ(t), dK(t) and dP(t+1)
      if (t + 1 < n_t && !compute_p(t + 1)) { ok = false; break; }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(p.flag, kErrOverflow);
    // dK, dV epilogue: this warp's D/2 columns of its 32 keys
    if (ok && n_t > 0 && mbar_wait_warp(kv_done, 0, abort, p.err)) {
      tc_fence_after();
      const float sk = p.scale * exp2i(-__ldg(p.a) - __ldg(p.G));
      const float sv = exp2i(-__ldg(p.ev + bhk) - __ldg(p.G)) * (DROP ? p.inv_keep : 1.f);
      const int64_t orow = ((int64_t)bhk * p.Sk + min(kj, p.Sk - 1)) * D + half * (D / 2);
      bool nf = false;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        __nv_bfloat16* dst = (which ? p.dk : p.dv) + orow;
        const float f = which ? sk : sv;
        const uint32_t col0 = (which ? C::T_DK : C::T_DV) + half * (D / 2);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
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
      const int64_t orow = ((int64_t)bhk * p.Sk + kj) * D + half * (D / 2);
      for (int c = 0; c < D / 2; c += 8) {
        *reinterpret_cast<uint4*>(p.dk + orow + c) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(p.dv + orow + c) = make_uint4(0, 0, 0, 0);
      }
    }
  } else {
    setmaxnreg_inc<kRegsDq>();
    // ---------------------------------------------------------------- dQ warps
    // dQ(t) = dS K lands in TMEM with queries as lanes: warp w reads all D columns of its 32 queries at
    // once (then the columns are free for dP(t+1)) and adds them into the fp32 accumulator with TMA
    // reductions of 32 x 32 boxes (rows past the sequence end are clipped), staged in two alternating
    // 4 KB 128B-swizzled buffers so a box waits only for the reduction issued two boxes earlier.
    const int quad = warp & 3;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    if constexpr (C::DQ_T) {
      // dQ^T(t) = K^T dS^T: lanes are head dims, columns queries. Thread d reads its 128 query columns at
      // once (freeing the columns for dP(t+1)), then adds each into dq_acc[q][d]: the warp's 32 lanes are
      // 32 consecutive d, so every reduction instruction covers one contiguous 128-byte segment.
      const int d = quad * 32 + lane;
      for (int t = 0; t < n_t; ++t) {
        const int h = hk * p.group + t / n_i;
        const int q0 = (i_first + t % n_i) * BQ;
        if (!mbar_wait_warp(dq_full, t & 1, abort, p.err)) break;
        tc_fence_after();
        uint32_t o[BQ];
#pragma unroll
        for (int c = 0; c < BQ / 32; ++c)
          tmem_ld32(tmem + lane_base + C::T_DP + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&o[c * 32]));
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_empty);
        float* dst = p.dq_acc + ((int64_t)(b * p.Hq + h) * p.Sq + q0) * D + d;
        const int nq = min(BQ, p.Sq - q0);
#pragma unroll
        for (int c = 0; c < BQ; ++c)
          if (c < nq) red_add_f32(dst + (int64_t)c * D, __uint_as_float(o[c]));
      }
    } else {
    uint8_t* stage = smem + C::DQS_OFF + (warp - 12) * 8192;
    int sb = 0;
    for (int t = 0; t < n_t; ++t) {
      const int h = hk * p.group + t / n_i;
      const int q0 = (i_first + t % n_i) * BQ;
      if (!mbar_wait_warp(dq_full, t & 1, abort, p.err)) break;
      tc_fence_after();
      uint32_t o[D];
#pragma unroll
      for (int c = 0; c < D / 32; ++c)
        tmem_ld32(tmem + lane_base + C::T_DP + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&o[c * 32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_empty);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        uint8_t* buf = stage + sb * 4096;
#pragma unroll
        for (int g = 0; g < 8; ++g)
          *reinterpret_cast<uint4*>(buf + lane * 128 + ((g ^ (lane & 7)) << 4)) =
              make_uint4(o[c * 32 + 4 * g], o[c * 32 + 4 * g + 1], o[c * 32 + 4 * g + 2], o[c * 32 + 4 * g + 3]);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_3d(&tmDQ, buf, c * 32, q0 + quad * 32, b * p.Hq + h);
          bulk_commit_group();
        }
        sb ^= 1;
      }
    }
    if (lane == 0) bulk_wait_group<0>();
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

// ------------------------------------------------------------------------------------------------------
// Head dim 256. The key-stationary design above keeps dK and dV of all D columns in TMEM (2 D columns per
// key); at D = 256 that is all 512 columns, so here each 128-key tile is split over two CTAs by OUTPUT
// columns: CTA dh (blockIdx.z) accumulates dK, dV and dQ for head dims [128 dh, 128 dh + 128). Both CTAs
// compute the full-D contractions S^T = K Q^T and dP^T = V dO^T (the softmax needs all of D), so those
// two products are done twice; everything downstream is split. Query tiles are 64 rows, so that K, V
// (64 KB each, resident) plus one 32 KB stage of Q and of dO fit in shared memory.
//   warp 0      TMA: K, V once; per query tile Q (4 atoms of 64 rows x 64 dims), lse and delta, one stage
//   warp 1      MMA, per query tile t (all 128-row M):
//                 S^T  = K Q^T          (N = 64 queries, K = 256)      -> TMEM [0, 64)
//                 dP^T = V dO^T         (N = 64, K = 256)              -> TMEM [64, 128)
//                 dV  += P^T dO_dh      (TS: P^T from TMEM; N = 128)   -> TMEM [256, 384)
//                 dK  += dS^T Q_dh      (dS^T from shared memory)      -> TMEM [384, 512)
//                 dQ^T = K_dh^T dS^T    (M = 128 head dims, N = 64)    -> TMEM [128, 192)
//               issued as dV(t) | dK(t) dQ^T(t) dP(t+1) S(t+1) | dV(t+1) ...: Q's stage is released by
//               dK(t) and reloaded while dQ^T(t) and dP(t+1) run
//   warp 2      TMA: dO per query tile, one stage (released by dV(t))
//   warps 4-11  key warps, two per TMEM lane quadrant, each 32 of the 64 query columns: P^T (packed fp16
//               back over its S^T columns), dS^T (fp16 into a 128B-swizzled 128 x 64 tile), and at the
//               end 64 of the 128 dK / dV columns
//   warps 12-15 dQ warps: dQ^T rows are head dims, so each thread adds its 64 query values into the fp32
//               accumulator with red.global.add, 32 consecutive head dims per warp instruction
namespace d256 {
constexpr int QROWS = 64;
constexpr int KROWS = 128;
constexpr int D = 256;
constexpr int K_OFF = 0;                    // 4 atoms x 128 rows x 128 B
constexpr int V_OFF = K_OFF + 65536;
constexpr int Q_OFF = V_OFF + 65536;        // 4 atoms x 64 rows x 128 B
constexpr int DO_OFF = Q_OFF + 32768;
constexpr int DS_OFF = DO_OFF + 32768;      // dS^T: 128 keys x 64 queries fp16, one atom
constexpr int VEC_OFF = DS_OFF + 16384;     // lse[64], delta[64], dropout row keys[64]
constexpr int BAR_OFF = VEC_OFF + 768;
constexpr int SMEM = BAR_OFF + 256;
constexpr uint32_t T_S = 0, T_DP = 64, T_DQ = 128, T_DV = 256, T_DK = 384;
static_assert(SMEM <= 227 * 1024, "shared memory");
}  // namespace d256

template <bool DROP>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_d256_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                         const AttnBwdParams p) {
  using namespace d256;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {
    if (threadIdx.x == 0) atomicOr(p.err, kErrSmemAlign);
    return;
  }
  uint8_t* smem = smem_raw;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;
  uint64_t* q_empty = bars + 2;
  uint64_t* do_full = bars + 3;
  uint64_t* do_empty = bars + 4;
  uint64_t* s_full = bars + 5;
  uint64_t* dp_full = bars + 6;
  uint64_t* p_ready = bars + 7;
  uint64_t* ds_ready = bars + 8;
  uint64_t* dq_full = bars + 9;
  uint64_t* dq_empty = bars + 10;
  uint64_t* kv_done = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bhk = blockIdx.x;
  const int b = bhk / p.Hkv, hk = bhk % p.Hkv;
  const int k0 = blockIdx.y * KROWS;
  const int dh = blockIdx.z;  // this CTA's half of the head dims for dK, dV and dQ
  const int i_first = p.causal ? k0 / QROWS : 0;
  const int n_i = max(0, p.q_tiles - i_first);
  const int n_t = p.group * n_i;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(do_full, 1);
    mbar_init(do_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_ready, 8);
    mbar_init(ds_ready, 8);
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
    // ---------------------------------------------------------------- TMA: K, V, then Q + lse + delta
    if (lane == 0 && n_t > 0) {
      mbar_arrive_expect_tx(kv_full, 2 * 65536);
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        tma_load_3d(smem + K_OFF + a * 16384, &tmK, kv_full, a * 64, k0, bhk);
        tma_load_3d(smem + V_OFF + a * 16384, &tmV, kv_full, a * 64, k0, bhk);
      }
      for (int t = 0; t < n_t; ++t) {
        const int h = hk * p.group + t / n_i;
        const int q0 = (i_first + t % n_i) * QROWS;
        const int bh = b * p.Hq + h;
        if (!mbar_wait(q_empty, (t & 1) ^ 1, abort, p.err)) break;
        mbar_arrive_expect_tx(q_full, 32768 + 512 + (DROP ? 256 : 0));
#pragma unroll
        for (int a = 0; a < 4; ++a) tma_load_3d(smem + Q_OFF + a * 8192, &tmQ, q_full, a * 64, q0, bh);
        float* vec = reinterpret_cast<float*>(smem + VEC_OFF);
        bulk_load(vec, p.lse + (int64_t)bh * p.lse_ld + q0, 256, q_full);
        bulk_load(vec + 64, p.delta + (int64_t)bh * p.lse_ld + q0, 256, q_full);
        if constexpr (DROP) bulk_load(vec + 128, p.rowkey + (int64_t)bh * p.lse_ld + q0, 256, q_full);
      }
    }
  } else if (warp == 2) {
    // ---------------------------------------------------------------- TMA: dO
    if (lane == 0 && n_t > 0) {
      for (int t = 0; t < n_t; ++t) {
        const int h = hk * p.group + t / n_i;
        const int q0 = (i_first + t % n_i) * QROWS;
        if (!mbar_wait(do_empty, (t & 1) ^ 1, abort, p.err)) break;
        mbar_arrive_expect_tx(do_full, 32768);
#pragma unroll
        for (int a = 0; a < 4; ++a) tma_load_3d(smem + DO_OFF + a * 8192, &tmDO, do_full, a * 64, q0, b * p.Hq + h);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && n_t > 0) {
      constexpr uint32_t id_s = idesc_f16_f32(128, QROWS, false, false);   // S^T, dP^T
      constexpr uint32_t id_kv = idesc_f16_f32(128, 128, false, true);  // dV, dK
      constexpr uint32_t id_qt = idesc_f16_f32(128, QROWS, true, true);    // dQ^T
      const uint32_t k_addr = smem_u32(smem + K_OFF), v_addr = smem_u32(smem + V_OFF);
      const uint32_t q_addr = smem_u32(smem + Q_OFF), do_addr = smem_u32(smem + DO_OFF);
      const uint32_t ds_addr = smem_u32(smem + DS_OFF);
      auto issue_full_d = [&](uint32_t a_addr, uint32_t b_addr, uint32_t d_col) {  // K = 256 head dims
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t in_atom = (kk & 3) * 32;
          umma_f16_ss(tmem + d_col, smem_desc_sw128(a_addr + (kk >> 2) * 16384 + in_atom, 16, 1024),
                      smem_desc_sw128(b_addr + (kk >> 2) * 8192 + in_atom, 16, 1024), id_s, kk > 0);
        }
      };
      bool ok = mbar_wait(kv_full, 0, abort, p.err) && mbar_wait(q_full, 0, abort, p.err);
      if (ok) {
        tc_fence_after();
        issue_full_d(k_addr, q_addr, T_S);
        umma_commit(s_full);
        ok = mbar_wait(do_full, 0, abort, p.err);
        if (ok) {
          tc_fence_after();
          issue_full_d(v_addr, do_addr, T_DP);
          umma_commit(dp_full);
        }
      }
      for (int t = 0; ok && t < n_t; ++t) {
        const bool next = t + 1 < n_t;
        if (!mbar_wait(p_ready, t & 1, abort, p.err)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < QROWS / 16; ++kk)  // dV += P^T dO_dh   (P^T: queries 32 w.. in packed columns 32 w..)
          umma_f16_ts(tmem + T_DV, tmem + T_S + (kk >> 1) * 32 + (kk & 1) * 8,
                      smem_desc_sw128(do_addr + dh * 16384 + kk * 2048, 8192, 1024), id_kv, (t > 0 || kk > 0));
        umma_commit(do_empty);  // dP(t) and dV(t) were dO(t)'s readers
        if (!mbar_wait(ds_ready, t & 1, abort, p.err)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < QROWS / 16; ++kk)  // dK += dS^T Q_dh
          umma_f16_ss(tmem + T_DK, smem_desc_sw128(ds_addr + kk * 32, 16, 1024),
                      smem_desc_sw128(q_addr + dh * 16384 + kk * 2048, 8192, 1024), id_kv, (t > 0 || kk > 0));
        umma_commit(q_empty);  // S(t) and dK(t) were Q(t)'s readers
        if (t > 0 && !mbar_wait(dq_empty, (t - 1) & 1, abort, p.err)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < KROWS / 16; ++kk)  // dQ^T = K_dh^T dS^T   (both MN-major)
          umma_f16_ss(tmem + T_DQ, smem_desc_sw128(k_addr + dh * 32768 + kk * 2048, 16384, 1024),
                      smem_desc_sw128(ds_addr + kk * 2048, 16384, 1024), id_qt, kk > 0);
        umma_commit(dq_full);
        if (next) {
          if (!mbar_wait(do_full, (t + 1) & 1, abort, p.err)) break;
          tc_fence_after();
          issue_full_d(v_addr, do_addr, T_DP);
          umma_commit(dp_full);
          if (!mbar_wait(q_full, (t + 1) & 1, abort, p.err)) break;
          tc_fence_after();
          issue_full_d(k_addr, q_addr, T_S);
          umma_commit(s_full);
        }
      }
      if (ok) umma_commit(kv_done);
    }
  } else if (warp >= 4 && warp < 12) {
    // ---------------------------------------------------------------- key warps
    const int quad = warp & 3;
    const int half = (warp - 4) >> 2;
    const int r = quad * 32 + lane;  // key within the tile
    const int kj = k0 + r;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const int cq = half * 32;        // this warp's 32 query columns
    const float* vec = reinterpret_cast<const float*>(smem + VEC_OFF);
    bool ok = true, bad = false;
    uint32_t pp[16];  // P of this thread's key against the warp's 32 queries, packed fp16 pairs
    uint32_t keep_bits = 0;  // dropout: bit c set when query column cq + c keeps this key

    auto compute_p = [&](int t) -> bool {
      const int h = hk * p.group + t / n_i;
      const int q0 = (i_first + t % n_i) * QROWS;
      if (!mbar_wait_warp(q_full, t & 1, abort, p.err) || !mbar_wait_warp(s_full, t & 1, abort, p.err)) return false;
      tc_fence_after();
      uint32_t rr[32];
      tmem_ld32(tmem + lane_base + T_S + cq, rr);
      tmem_ld_wait();
      const uint16_t* mrow = p.mask ? p.mask + b * p.mb + h * p.mh + (int64_t)q0 * p.mi + min(kj, p.Sk - 1) : nullptr;
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float pc[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int col = cq + e + u;
          const int qi = q0 + col;
          const bool valid = kj < p.Sk && qi < p.Sq && (!p.causal || kj <= qi);
          float sv = __uint_as_float(rr[e + u]) * p.scale_log2;
          if (mrow && valid) sv += __half2float(__ushort_as_half(mrow[(int64_t)col * p.mi])) * 1.4426950408889634f;
          pc[u] = valid ? ex2(sv - vec[col] * 1.4426950408889634f) : 0.f;
        }
        pp[e >> 1] = pack_f16(pc[0], pc[1]);
      }
      if constexpr (DROP) {  // dV sees P with dropped entries zeroed; dS keeps the full P and the keep bits
        const uint32_t* rks = reinterpret_cast<const uint32_t*>(vec) + 128;
        uint32_t pt[16];
        uint32_t kb = 0;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const bool k0b = drop_keep(rks[cq + 2 * c], (uint32_t)kj, p.drop_thr);
          const bool k1b = drop_keep(rks[cq + 2 * c + 1], (uint32_t)kj, p.drop_thr);
          pt[c] = pp[c] & ((k0b ? 0x0000ffffu : 0u) | (k1b ? 0xffff0000u : 0u));
          kb |= ((k0b ? 1u : 0u) | (k1b ? 2u : 0u)) << (2 * c);
        }
        keep_bits = kb;
        tmem_st16(tmem + lane_base + T_S + cq, pt);
      } else {
        tmem_st16(tmem + lane_base + T_S + cq, pp);  // P^T over this warp's own S^T columns
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
      return true;
    };

    ok = n_t > 0 && compute_p(0);
    for (int t = 0; ok && t < n_t; ++t) {
      if (!mbar_wait_warp(dp_full, t & 1, abort, p.err)) { ok = false; break; }
      tc_fence_after();
      {
        uint32_t rr[32];
        tmem_ld32(tmem + lane_base + T_DP + cq, rr);
        tmem_ld_wait();
        uint32_t pk[16];
        float dmax = 0.f;  // largest |dS|: a value >= 65520 rounds to an fp16 infinity (NaN also flags)
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float2 pf = __half22float2(*reinterpret_cast<const __half2*>(&pp[e >> 1]));
          float dp0 = __uint_as_float(rr[e]), dp1 = __uint_as_float(rr[e + 1]);
          if constexpr (DROP) {
            dp0 = (keep_bits >> e) & 1 ? dp0 * p.inv_keep : 0.f;
            dp1 = (keep_bits >> (e + 1)) & 1 ? dp1 * p.inv_keep : 0.f;
          }
          const float d0 = pf.x * (dp0 - vec[64 + cq + e]);
          const float d1 = pf.y * (dp1 - vec[64 + cq + e + 1]);
          pk[e >> 1] = pack_f16(d0, d1);
          dmax = fmaxf(dmax, fmaxf(fabsf(d0), fabsf(d1)));
        }
        bad |= !(dmax < 65520.f);
        // dS^T row r, queries [cq, cq + 32): 16-byte chunks 4 half .. 4 half + 3 of the 128-byte row
#pragma unroll
        for (int g = 0; g < 4; ++g)
          *reinterpret_cast<uint4*>(smem + DS_OFF + swz_off(r, half * 4 + g)) =
              make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_ready);
      if (t + 1 < n_t && !compute_p(t + 1)) { ok = false; break; }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(p.flag, kErrOverflow);
    // dK, dV: this warp's 64 of the CTA's 128 head-dim columns for its 32 keys
    const int64_t orow = ((int64_t)bhk * p.Sk + min(kj, p.Sk - 1)) * D + dh * 128 + half * 64;
    if (ok && n_t > 0 && mbar_wait_warp(kv_done, 0, abort, p.err)) {
      tc_fence_after();
      const float sk = p.scale * exp2i(-__ldg(p.a) - __ldg(p.G));
      const float sv = exp2i(-__ldg(p.ev + bhk) - __ldg(p.G)) * (DROP ? p.inv_keep : 1.f);
      bool nf = false;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        __nv_bfloat16* dst = (which ? p.dk : p.dv) + orow;
        const float f = which ? sk : sv;
        const uint32_t col0 = (which ? T_DK : T_DV) + half * 64;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
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
    } else if (n_t == 0 && kj < p.Sk) {  // keys no query sees: zero gradients
      for (int c = 0; c < 64; c += 8) {
        *reinterpret_cast<uint4*>(p.dk + orow + c) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(p.dv + orow + c) = make_uint4(0, 0, 0, 0);
      }
    }
  } else if (warp >= 12) {
    // ---------------------------------------------------------------- dQ warps
    const int quad = warp & 3;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const int d = dh * 128 + quad * 32 + lane;
    for (int t = 0; t < n_t; ++t) {
      const int h = hk * p.group + t / n_i;
      const int q0 = (i_first + t % n_i) * QROWS;
      if (!mbar_wait_warp(dq_full, t & 1, abort, p.err)) break;
      tc_fence_after();
      uint32_t o[QROWS];
      tmem_ld32(tmem + lane_base + T_DQ, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
      tmem_ld32(tmem + lane_base + T_DQ + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_empty);
      float* dst = p.dq_acc + ((int64_t)(b * p.Hq + h) * p.Sq + q0) * D + d;
      const int nq = min(QROWS, p.Sq - q0);
#pragma unroll
      for (int c = 0; c < QROWS; ++c)
        if (c < nq) red_add_f32(dst + (int64_t)c * D, __uint_as_float(o[c]));
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
                                                           const int32_t* __restrict__ e_floor, int32_t* __restrict__ G) {
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
    if (e_floor) e = max(e, *e_floor);  // head-sharded call: the maximum over every rank's heads
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
                                                            float* __restrict__ delta, uint32_t* __restrict__ rowkey,
                                                            uint32_t seed_lo, uint32_t seed_hi) {
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
  if (row < rows && threadIdx.x % TPR == 0) {
    delta[(row / Sq) * lse_ld + row % Sq] = acc;
    if (rowkey)
      rowkey[(row / Sq) * lse_ld + row % Sq] = drop_row_key(seed_lo, seed_hi, (uint32_t)(row / Sq), (uint32_t)(row % Sq));
  }
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
  uint32_t* rowkey;  // dropout row hash keys, [B*Hq, lse_ld]
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
  p += ((4 * B * Hq + 255) / 256) * 256;
  w.rowkey = reinterpret_cast<uint32_t*>(p);
  return w;
}

int64_t workspace_bytes(int64_t B, int64_t Hq, int64_t Sq, int64_t D) {
  const int64_t n = B * Hq * Sq * D;
  return ((4 * n + 255) / 256) * 256 + ((2 * n + 255) / 256) * 256 + 2 * ((4 * B * Hq * lse_stride(Sq) + 255) / 256) * 256 +
         ((4 * B * Hq + 255) / 256) * 256;
}

template <int D, bool DROP>
int launch_bwd(const void* q16, const void* k16, const void* v16, const void* do16, const AttnBwdParams& prm,
               int64_t Sk, cudaStream_t st) {
  using C = BwdCfg<D>;
  const tbf16_host::DeviceInfo* dev = tbf16_host::device_info();
  CUtensorMap tq, tk, tv, tdo, tdq;
  const int64_t BHq = (int64_t)prm.B * prm.Hq, BHk = (int64_t)prm.B * prm.Hkv;
  if (int rc = tbf16_host::make_tmap_3d(&tq, q16, D, prm.Sq, BHq, D, (uint64_t)prm.Sq * D, 64, BQ)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tdo, do16, D, prm.Sq, BHq, D, (uint64_t)prm.Sq * D, 64, BQ)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tk, k16, D, Sk, BHk, D, (uint64_t)Sk * D, 64, BKV)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tv, v16, D, Sk, BHk, D, (uint64_t)Sk * D, 64, BKV)) return rc;
  if (int rc = tbf16_host::make_tmap_3d_f32(&tdq, prm.dq_acc, D, prm.Sq, BHq, D, (uint64_t)prm.Sq * D, 32, 32)) return rc;
  static bool attr_done[64] = {false};
  if (!attr_done[dev->device & 63]) {
    if (cudaFuncSetAttribute(attn_bwd_kernel<D, DROP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
      return tbf16_host::check_launch();
    attr_done[dev->device & 63] = true;
  }
  dim3 grid((unsigned)BHk, (unsigned)((Sk + BKV - 1) / BKV));
  attn_bwd_kernel<D, DROP><<<grid, kThreads, C::SMEM, st>>>(tq, tk, tv, tdo, tdq, prm);
  return tbf16_host::check_launch();
}

template <bool DROP>
int launch_bwd_d256(const void* q16, const void* k16, const void* v16, const void* do16, AttnBwdParams prm, int64_t Sk,
                    cudaStream_t st) {
  const tbf16_host::DeviceInfo* dev = tbf16_host::device_info();
  constexpr int D = 256;
  CUtensorMap tq, tk, tv, tdo;
  const int64_t BHq = (int64_t)prm.B * prm.Hq, BHk = (int64_t)prm.B * prm.Hkv;
  if (int rc = tbf16_host::make_tmap_3d(&tq, q16, D, prm.Sq, BHq, D, (uint64_t)prm.Sq * D, 64, d256::QROWS)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tdo, do16, D, prm.Sq, BHq, D, (uint64_t)prm.Sq * D, 64, d256::QROWS)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tk, k16, D, Sk, BHk, D, (uint64_t)Sk * D, 64, d256::KROWS)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tv, v16, D, Sk, BHk, D, (uint64_t)Sk * D, 64, d256::KROWS)) return rc;
  static bool attr_done[64] = {false};
  if (!attr_done[dev->device & 63]) {
    if (cudaFuncSetAttribute(attn_bwd_d256_kernel<DROP>, cudaFuncAttributeMaxDynamicSharedMemorySize, d256::SMEM) !=
        cudaSuccess)
      return tbf16_host::check_launch();
    attr_done[dev->device & 63] = true;
  }
  prm.q_tiles = (int)((prm.Sq + d256::QROWS - 1) / d256::QROWS);
  dim3 grid((unsigned)BHk, (unsigned)((Sk + d256::KROWS - 1) / d256::KROWS), 2);
  attn_bwd_d256_kernel<DROP><<<grid, kThreads, d256::SMEM, st>>>(tq, tk, tv, tdo, prm);
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

}  // extern "C"

namespace {

int attn_bwd_impl(const void* q16, const void* k16, const void* v16, const void* o16, const float* lse, int64_t lse_ld,
                  const void* dout, int64_t dout_sb, int64_t dout_sh, int64_t dout_ss, int64_t dout_d, const int32_t* a,
                  const int32_t* ev, int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, float scale,
                  int causal, const void* mask, int64_t mask_sb, int64_t mask_sh, int64_t mask_sq, int t_do, void* dq,
                  void* dk, void* dv, int32_t* G_out, unsigned int* flag, void* ws, int64_t ws_bytes, float dropout_p,
                  uint64_t seed, const int32_t* e_floor, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  uint32_t thr = 0;
  float inv_keep = 1.f;
  if (!tbf16_host::dropout_params(dropout_p, &thr, &inv_keep)) return TBF16_ERR_INVALID;
  const bool drop = thr > 0;
  const uint32_t seed_lo = (uint32_t)seed, seed_hi = (uint32_t)(seed >> 32);
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Sq <= 0 || Sk <= 0 || dout_d <= 0 || dout_d > D || !a || !ev ||
      !lse || lse_ld != lse_stride(Sq) || !G_out || !flag || !ws || B * Hq > 65535 || B * Hkv > 65535)
    return TBF16_ERR_INVALID;
  if (D != 64 && D != 128 && D != 256) return TBF16_ERR_UNSUPPORTED;
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
  attn_bwd_exp_kernel<<<1, 256, 0, st>>>(w.amax, (int)(B * Hq), (int)Hq, (int)Hkv, group, ev, t_do, e_floor, G_out);
  // 2. dO16 and delta (the padding rows of delta are zeroed: the main kernel reads whole 128-row tiles)
  const int64_t rows = B * Hq * Sq;
  if (lse_ld != Sq && cudaMemsetAsync(w.delta, 0, sizeof(float) * B * Hq * lse_ld, st) != cudaSuccess)
    return TBF16_ERR_LAUNCH;
  const int rpb = 256 / (int)(D / 8);
  const unsigned pgrid = (unsigned)((rows + rpb - 1) / rpb);
  if (D == 64)
    attn_bwd_prep_kernel<64><<<pgrid, 256, 0, st>>>(static_cast<const uint16_t*>(dout), dout_sb, dout_sh, dout_ss,
                                                    (int)dout_d, static_cast<const __half*>(o16), ev, G_out, (int)Hq,
                                                    (int)Hkv, group, (int)Sq, rows, lse_ld, w.do16, w.delta,
                                                     drop ? w.rowkey : nullptr, seed_lo, seed_hi);
  else if (D == 128)
    attn_bwd_prep_kernel<128><<<pgrid, 256, 0, st>>>(static_cast<const uint16_t*>(dout), dout_sb, dout_sh, dout_ss,
                                                     (int)dout_d, static_cast<const __half*>(o16), ev, G_out, (int)Hq,
                                                     (int)Hkv, group, (int)Sq, rows, lse_ld, w.do16, w.delta,
                                                     drop ? w.rowkey : nullptr, seed_lo, seed_hi);
  else
    attn_bwd_prep_kernel<256><<<pgrid, 256, 0, st>>>(static_cast<const uint16_t*>(dout), dout_sb, dout_sh, dout_ss,
                                                     (int)dout_d, static_cast<const __half*>(o16), ev, G_out, (int)Hq,
                                                     (int)Hkv, group, (int)Sq, rows, lse_ld, w.do16, w.delta,
                                                     drop ? w.rowkey : nullptr, seed_lo, seed_hi);
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
  prm.rowkey = w.rowkey;
  prm.drop_thr = thr;
  prm.inv_keep = inv_keep;
  int rc;
  if (drop)
    rc = D == 64    ? launch_bwd<64, true>(q16, k16, v16, w.do16, prm, Sk, st)
         : D == 128 ? launch_bwd<128, true>(q16, k16, v16, w.do16, prm, Sk, st)
                    : launch_bwd_d256<true>(q16, k16, v16, w.do16, prm, Sk, st);
  else
    rc = D == 64    ? launch_bwd<64, false>(q16, k16, v16, w.do16, prm, Sk, st)
         : D == 128 ? launch_bwd<128, false>(q16, k16, v16, w.do16, prm, Sk, st)
                    : launch_bwd_d256<false>(q16, k16, v16, w.do16, prm, Sk, st);
  if (rc) return rc;
  // 4. dq
  const int64_t n4 = rows * D / 4;
  const int g = (int)std::min<int64_t>((n4 + 255) / 256, (int64_t)dev->sms * 16);
  attn_bwd_dq_kernel<<<g, 256, 0, st>>>(reinterpret_cast<const float4*>(w.dq_acc), n4, scale, a, G_out,
                                        static_cast<uint2*>(dq), flag);
  return tbf16_host::check_launch();
}

}  // namespace

extern "C" {

int tbf16_attn_bwd(const void* q16, const void* k16, const void* v16, const void* o16, const float* lse, int64_t lse_ld,
                   const void* dout,
                   int64_t dout_sb, int64_t dout_sh, int64_t dout_ss, int64_t dout_d, const int32_t* a, const int32_t* ev,
                   int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, float scale, int causal,
                   const void* mask, int64_t mask_sb, int64_t mask_sh, int64_t mask_sq, int t_do, void* dq, void* dk,
                   void* dv, int32_t* G_out, unsigned int* flag, void* ws, int64_t ws_bytes, void* stream) {
  return attn_bwd_impl(q16, k16, v16, o16, lse, lse_ld, dout, dout_sb, dout_sh, dout_ss, dout_d, a, ev, B, Hq, Hkv, Sq,
                       Sk, D, scale, causal, mask, mask_sb, mask_sh, mask_sq, t_do, dq, dk, dv, G_out, flag, ws, ws_bytes,
                       0.f, 0, nullptr, stream);
}

int tbf16_attn_bwd_dropout(const void* q16, const void* k16, const void* v16, const void* o16, const float* lse,
                           int64_t lse_ld, const void* dout, int64_t dout_sb, int64_t dout_sh, int64_t dout_ss,
                           int64_t dout_d, const int32_t* a, const int32_t* ev, int64_t B, int64_t Hq, int64_t Hkv,
                           int64_t Sq, int64_t Sk, int64_t D, float scale, int causal, const void* mask, int64_t mask_sb,
                           int64_t mask_sh, int64_t mask_sq, int t_do, void* dq, void* dk, void* dv, int32_t* G_out,
                           unsigned int* flag, void* ws, int64_t ws_bytes, float dropout_p, uint64_t seed,
                           void* stream) {
  return attn_bwd_impl(q16, k16, v16, o16, lse, lse_ld, dout, dout_sb, dout_sh, dout_ss, dout_d, a, ev, B, Hq, Hkv, Sq,
                       Sk, D, scale, causal, mask, mask_sb, mask_sh, mask_sq, t_do, dq, dk, dv, G_out, flag, ws, ws_bytes,
                       dropout_p, seed, nullptr, stream);
}

int tbf16_attn_bwd_sharded(const void* q16, const void* k16, const void* v16, const void* o16, const float* lse,
                           int64_t lse_ld, const void* dout, int64_t dout_sb, int64_t dout_sh, int64_t dout_ss,
                           int64_t dout_d, const int32_t* a, const int32_t* ev, int64_t B, int64_t Hq, int64_t Hkv,
                           int64_t Sq, int64_t Sk, int64_t D, float scale, int causal, const void* mask, int64_t mask_sb,
                           int64_t mask_sh, int64_t mask_sq, int t_do, void* dq, void* dk, void* dv, int32_t* G_out,
                           unsigned int* flag, void* ws, int64_t ws_bytes, float dropout_p, uint64_t seed,
                           const int32_t* e_global, void* stream) {
  if (!e_global) return TBF16_ERR_INVALID;
  return attn_bwd_impl(q16, k16, v16, o16, lse, lse_ld, dout, dout_sb, dout_sh, dout_ss, dout_d, a, ev, B, Hq, Hkv, Sq,
                       Sk, D, scale, causal, mask, mask_sb, mask_sh, mask_sq, t_do, dq, dk, dv, G_out, flag, ws, ws_bytes,
                       dropout_p, seed, e_global, stream);
}

}  // extern "C"
