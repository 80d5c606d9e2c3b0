// Scaled fp16 flash-attention forward for sm_100a (tcgen05 + TMA), the compute step of the
// reference's scaled SDPA (tbf16/attention.py:56-65 inference, tbf16/autograd.py:153-164 training).
//
// Inputs are the exact fp16 copies from prepare_qkv: q16 = q * 2^a, k16 = k * 2^-a (so q16 . k16 =
// q . k), v16 = v * 2^-ev. Output: out = bf16_rn(softmax(scale * q16 k16^T + mask) v16 * 2^ev), written
// straight from the fp32 accumulator (the reference rounds to fp16 first), plus the natural-log
// logsumexp per row for the backward pass.
//
// CTA = one 128-row query tile of one (batch, head); keys in 128-column tiles.
//   warp 0      TMA producer: Q once, then K and V tiles through 2-deep rings (3-D tensor maps over
//               (head, seq, dim), so tiles never cross heads; rows past the end read as zeros).
//   warp 1      MMA issuer: S_j = Q K_j^T into one of two TMEM S buffers (M=128, N=128, K=D), then
//               O += P_{j-1} V_{j-1} (M=128, N=D, K=128) with P from shared memory and V MN-major.
//   warps 2-5   softmax, one query row per thread: tcgen05.ld the S row, mask, online max with a lazy
//               rescale of O in TMEM (only when the running max grows by more than 2^8), exp2, row
//               sum, P -> fp16 into a 128B-swizzled K-major shared tile; epilogue O / l * 2^ev -> bf16.
// TMEM: S0 [0,128), S1 [128,256), O [256, 256+D). Every mbarrier wait is bounded.
#include <algorithm>
#include <memory>
#include <mutex>
#include <queue>
#include <vector>

#include "common.cuh"

using namespace tbf16;

namespace {

constexpr int BM = 128;  // query rows per CTA
constexpr int BN = 128;  // keys per tile
constexpr int kSoftmaxWarps = 4;
constexpr int kThreads = 32 * (2 + kSoftmaxWarps);
constexpr float kRescaleLog2 = 8.0f;  // keep a stale max until the true one exceeds it by 2^8
constexpr int kPolyPairsOf8 = 3;      // exp2 pairs (of every 8) computed on the FMA pipe

struct AttnFwdParams {
  int B, Hq, Hkv, Sq, Sk;
  int group;          // Hq / Hkv
  float scale_log2;   // softmax scale * log2(e)
  int causal;         // keys j <= query i (top-left aligned, as torch's is_causal)
  const int32_t* ev;  // [B * Hkv]: output multiplied by 2^ev
  __nv_bfloat16* out; // (B, Hq, Sq, D) with element strides osb, osh, oss (D contiguous)
  int64_t osb, osh, oss;
  float* lse;         // [B * Hq, lse_ld] natural-log logsumexp, nullable
  int64_t lse_ld;
  __half* o16;        // [B, Hq, Sq, D] fp16 O before the 2^ev scale (training), nullable
  void* split_ws;     // key-split launches of the head-dim-256 kernel: tickets, flags, parts' O
  const uint16_t* mask;  // additive fp16 bias, nullable; element (b,h,i,j) at b*mb + h*mh + i*mi + j
  int64_t mb, mh, mi;
  unsigned int* err;
  int m_tiles;
  // attention dropout (kernels instantiated with DROP): keep threshold, seed, 1 / keep probability
  uint32_t drop_thr, seed_lo, seed_hi;
  float inv_keep;
};

template <int D>
struct FwdCfg {
  static constexpr int ATOMS = D / 64;            // 64-column swizzle atoms per row
  static constexpr int TILE_BYTES = ATOMS * 128 * 128;  // 128 rows x D fp16
  static constexpr int Q_OFF = 0;
  // K/V ring depth: 2 stages up to D = 128; at D = 256 one stage fits in shared memory (the next V
  // tile loads while the softmax of the next S runs, so the single stage costs little).
  static constexpr int KS = D == 256 ? 1 : 2;
  static constexpr int K_OFF = Q_OFF + TILE_BYTES;
  static constexpr int V_OFF = K_OFF + KS * TILE_BYTES;
  static constexpr int P_OFF = V_OFF + KS * TILE_BYTES;
  static constexpr int P_BYTES = 2 * 128 * 128;        // 128 rows x 128 keys fp16
  static constexpr int BAR_OFF = P_OFF + P_BYTES;
  static constexpr int SMEM = 1024 + BAR_OFF + 256;
  static constexpr int O_COL = 256;
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// A tile that is not fully valid (sequence end, causal diagonal, user mask): S[row, k0 + e] -> the scaled,
// masked logit in log2 units (-inf where masked), in place in TMEM, 32 columns per step of a short
// loop. Keys k0 + e with e < lim are kept. The fully unrolled register form of this once-per-row-tile
// path cost about 9 us per tile on B200 (instruction fetch), more than the rest of the step.
__device__ __forceinline__ void mask_logits_tmem(uint32_t s_addr, int ncol, int k0, int qi, const AttnFwdParams& p,
                                                 const uint16_t* mrow) {
  const int lim = min(p.Sk, p.causal ? qi + 1 : p.Sk) - k0;
#pragma unroll 1
  for (int c = 0; c < ncol; c += 32) {
    uint32_t o[32];
    tmem_ld32(s_addr + c, o);
    tmem_ld_wait();
    if (mrow) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float v = __uint_as_float(o[i]) * p.scale_log2;
        if (c + i < lim) v += __half2float(__ushort_as_half(mrow[c + i])) * 1.4426950408889634f;
        o[i] = __float_as_uint(c + i < lim ? v : -INFINITY);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(c + i < lim ? __uint_as_float(o[i]) * p.scale_log2 : -INFINITY);
    }
    tmem_st32(s_addr + c, o);
  }
  tmem_st_wait();
}

template <int D, bool DROP>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnFwdParams p) {
  using C = FwdCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_empty = bars + 11; // [2]
  uint64_t* p_full = bars + 13;
  uint64_t* pv_done = bars + 14;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // causal: the grid is (heads, query tiles) so that CTAs start in order of their key count -- every
  // head's last (heaviest) query tile first -- and the light tiles fill in behind them
  const int bh = p.causal ? (int)blockIdx.x : (int)blockIdx.y;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int bhk = b * p.Hkv + h / p.group;
  const int m_tile = p.causal ? (p.m_tiles - 1 - (int)blockIdx.y) : (int)blockIdx.x;
  const int m0 = m_tile * BM;
  const int kv_end = p.causal ? min(p.Sk, m0 + BM) : p.Sk;
  const int n_kv = (kv_end + BN - 1) / BN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kSoftmaxWarps);
    }
    mbar_init(p_full, kSoftmaxWarps);
    mbar_init(pv_done, 1);
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && n_kv > 0) {
      mbar_arrive_expect_tx(q_full, C::TILE_BYTES);
#pragma unroll
      for (int a = 0; a < C::ATOMS; ++a) tma_load_3d(smem + C::Q_OFF + a * 16384, &tmQ, q_full, a * 64, m0, bh);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % C::KS;
        const uint32_t ph = (j / C::KS) & 1;
        if (!mbar_wait(&k_empty[st], ph ^ 1, abort, p.err)) break;
        mbar_arrive_expect_tx(&k_full[st], C::TILE_BYTES);
#pragma unroll
        for (int a = 0; a < C::ATOMS; ++a)
          tma_load_3d(smem + C::K_OFF + st * C::TILE_BYTES + a * 16384, &tmK, &k_full[st], a * 64, j * BN, bhk);
        if (!mbar_wait(&v_empty[st], ph ^ 1, abort, p.err)) break;
        mbar_arrive_expect_tx(&v_full[st], C::TILE_BYTES);
#pragma unroll
        for (int a = 0; a < C::ATOMS; ++a)
          tma_load_3d(smem + C::V_OFF + st * C::TILE_BYTES + a * 16384, &tmV, &v_full[st], a * 64, j * BN, bhk);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(BM, BN, false, false);
      constexpr uint32_t idesc_o = idesc_f16_f32(BM, D, false, true);
      const uint32_t q_addr = smem_u32(smem + C::Q_OFF);
      const uint32_t p_addr = smem_u32(smem + C::P_OFF);
      auto issue_pv = [&](int i) -> bool {
        const int st = i % C::KS;
        if (!mbar_wait(p_full, i & 1, abort, p.err)) return false;
        if (!mbar_wait(&v_full[st], (i / C::KS) & 1, abort, p.err)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + C::V_OFF + st * C::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t ad = smem_desc_sw128(p_addr + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          // V tile is MN-major: D contiguous (64-wide atoms 16 KB apart), keys = 8-row groups 1 KB apart.
          const uint64_t bd = smem_desc_sw128(v_addr + kk * 2048, 16384, 1024);
          umma_f16_ss(tmem + C::O_COL, ad, bd, idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(pv_done);
        umma_commit(&v_empty[st]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, abort, p.err);
      for (int j = 0; ok && j < n_kv; ++j) {
        const int sb = j & 1;  // S buffer in TMEM (always two)
        const int ks = j % C::KS;  // K stage in shared memory
        if (!mbar_wait(&k_full[ks], (j / C::KS) & 1, abort, p.err) ||
            !mbar_wait(&s_empty[sb], ((j >> 1) & 1) ^ 1, abort, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + C::K_OFF + ks * C::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_f16_ss(tmem + sb * BN, smem_desc_sw128(q_addr + off, 16, 1024), smem_desc_sw128(k_addr + off, 16, 1024),
                      idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[ks]);
        if (j >= 1) ok = issue_pv(j - 1);
      }
      if (ok) issue_pv(n_kv - 1);
    }
  } else {
    // ---------------------------------------------------------------- softmax + epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row within the tile
    const int qi = m0 + r;           // query index
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const uint32_t rk = DROP ? drop_row_key(p.seed_lo, p.seed_hi, (uint32_t)bh, (uint32_t)qi) : 0u;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int st = j & 1;
      if (!mbar_wait_warp(&s_full[st], (j >> 1) & 1, abort, p.err)) { ok = false; break; }
      tc_fence_after();
      const int k0 = j * BN;
      // Logits are kept raw (s) and scaled inside the exp: p = 2^(s * c - m) with c = scale * log2(e)
      // (scale > 0, so the max commutes with it). Partial tiles (sequence end, causal diagonal, user
      // mask) are first turned into scaled, masked values in TMEM and use c = 1. Reductions use 8
      // independent partial accumulators: a single softmax warp per sub-partition has no other latency
      // hiding.
      const bool full_tile = p.mask == nullptr && k0 + BN <= p.Sk && (!p.causal || k0 + BN - 1 <= m0);
      const float c_scale = full_tile ? p.scale_log2 : 1.f;
      if (!full_tile)
        mask_logits_tmem(tmem + lane_base + st * BN, BN, k0, qi, p,
                         p.mask ? p.mask + b * p.mb + h * p.mh + (int64_t)min(qi, p.Sq - 1) * p.mi + k0 : nullptr);
      float s[BN];
      {
        uint32_t rr[BN];  // all four 32-column loads in flight, one wait
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
          tmem_ld32(tmem + lane_base + st * BN + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&rr[c * 32]));
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < BN; ++e) s[e] = __uint_as_float(rr[e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[st]);
      float m8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) m8[e] = s[e];
#pragma unroll
      for (int c = 8; c < BN; ++c) m8[c & 7] = fmaxf(m8[c & 7], s[c]);
      const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * c_scale;
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_used + kRescaleLog2 || (m_used == -INFINITY && mx > -INFINITY)) {
        alpha = (m_used == -INFINITY) ? 0.f : ex2(m_used - mx);
        rescale = j > 0;
        m_used = mx;
        l *= alpha;
      }
      const float base = m_used == -INFINITY ? 0.f : m_used;
      float sum8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float p0 = ex2(fmaf(s[c], c_scale, -base)), p1 = ex2(fmaf(s[c + 1], c_scale, -base));
        sum8[(c >> 1) & 7] += p0 + p1;
        pk[c / 2] = pack_f16(p0, p1);
        if constexpr (DROP) pk[c / 2] &= drop_pair_mask(rk, (uint32_t)(k0 + c) >> 1, p.drop_thr);
      }
      l += ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      // O and the P buffer are free once the previous P.V has completed
      if (j > 0 && !mbar_wait_warp(pv_done, (j - 1) & 1, abort, p.err)) { ok = false; break; }
      tc_fence_after();
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + C::O_COL + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * (rescale ? alpha : 1.f));
          tmem_st32(tmem + lane_base + C::O_COL + c * 32, o);
        }
        tmem_st_wait();
      }
      uint8_t* pbuf = smem + C::P_OFF;
#pragma unroll
      for (int c = 0; c < BN / 8; ++c)
        *reinterpret_cast<uint4*>(pbuf + swz_off(r, c)) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && n_kv > 0 && mbar_wait_warp(pv_done, (n_kv - 1) & 1, abort, p.err)) {
      tc_fence_after();
      const float inv_l = l > 0.f ? (DROP ? p.inv_keep : 1.f) / l : 0.f;
      const float sc = exp2i(__ldg(p.ev + bhk));
      __nv_bfloat16* orow = p.out + (int64_t)(bh / p.Hq) * p.osb + (int64_t)(bh % p.Hq) * p.osh +
                            (int64_t)min(qi, p.Sq - 1) * p.oss;
      __half* o16row = p.o16 ? p.o16 + ((int64_t)bh * p.Sq + min(qi, p.Sq - 1)) * D : nullptr;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + C::O_COL + c * 32, o);
        tmem_ld_wait();
        if (qi < p.Sq) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(o[8 * g + 0]) * inv_l * sc, __uint_as_float(o[8 * g + 1]) * inv_l * sc);
            w.y = pack_bf16(__uint_as_float(o[8 * g + 2]) * inv_l * sc, __uint_as_float(o[8 * g + 3]) * inv_l * sc);
            w.z = pack_bf16(__uint_as_float(o[8 * g + 4]) * inv_l * sc, __uint_as_float(o[8 * g + 5]) * inv_l * sc);
            w.w = pack_bf16(__uint_as_float(o[8 * g + 6]) * inv_l * sc, __uint_as_float(o[8 * g + 7]) * inv_l * sc);
            *reinterpret_cast<uint4*>(orow + c * 32 + g * 8) = w;
            if (o16row) {
              uint4 h;
              h.x = pack_f16(__uint_as_float(o[8 * g + 0]) * inv_l, __uint_as_float(o[8 * g + 1]) * inv_l);
              h.y = pack_f16(__uint_as_float(o[8 * g + 2]) * inv_l, __uint_as_float(o[8 * g + 3]) * inv_l);
              h.z = pack_f16(__uint_as_float(o[8 * g + 4]) * inv_l, __uint_as_float(o[8 * g + 5]) * inv_l);
              h.w = pack_f16(__uint_as_float(o[8 * g + 6]) * inv_l, __uint_as_float(o[8 * g + 7]) * inv_l);
              *reinterpret_cast<uint4*>(o16row + c * 32 + g * 8) = h;
            }
          }
        }
      }
      if (p.lse && qi < p.Sq)
        p.lse[(int64_t)bh * p.lse_ld + qi] = (m_used + log2f(l)) * 0.6931471805599453f;
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

// ------------------------------------------------------------------------------------------------
// Head dims 64 and 128: a persistent kernel, one CTA per SM, whose work items are pairs of 128-row
// query tiles of one head ("tile 0" and "tile 1") that share every K and V tile. TMEM holds S and O
// of both tiles (S0 [0,128), O0 [128,256), S1 [256,384), O1 [384,512)); P is written back over its S
// columns as packed fp16 and the P.V MMA reads its A operand from TMEM. Within an item the MMA warp
// alternates the tiles,
//   S0_0 S1_0 | PV0_0 S0_1 | PV1_0 S1_1 | PV0_1 S0_2 | PV1_1 S1_2 | ...
// so the tensor core computes one tile's P.V and next S while the other tile's softmax runs. The
// MMA pipe executes one CTA's MMAs in issue order: S0_{j+1} overwrites P0_j only after PV0_j has
// read it, and when S0_{j+1} completes PV0_j has completed too (O0 may be rescaled without another
// wait). K and V go through two-stage rings that run on across items.
// Between items nothing drains: the Q tiles are released once the item's last S MMA completes (the
// next item's Q loads during the last P.V steps), the next item's first S MMAs run while the softmax
// warps write the previous item's output, and its first P.V (which overwrites O) waits for the
// softmax warps' first P of the new item, which they produce only after reading O out.
// Items are ordered heads fastest and heaviest (last) query pairs first for causal attention, query
// pairs fastest otherwise (CTAs in flight share a head's K and V in L2), and dealt to the CTAs in a
// snake order (round r gives item r * G + c to CTA c, or to CTA G - 1 - c when r is odd), which
// balances the causal triangle almost as well as longest-first list scheduling.
//   warps 0-3  softmax + epilogue of tile 0 (warp w reads TMEM lanes 32 (w % 4) ..)
//   warps 4-7  softmax + epilogue of tile 1
//   warp 8     TMA producer          warp 9  MMA issuer (+ TMEM allocation)     warps 10-11 idle
// The CTA launches with 168 registers per thread (12 warps); the third warpgroup (warps 8-11) drops
// to 72 and the two softmax warpgroups rise to 216, so a thread holds its whole 128-logit row with
// room for the exp pipeline: 72 * 128 + 216 * 256 = 64512 = 168 * 384 (and per sub-partition the
// 216 + 216 + 72 registers of its three warps fit its 16384).
constexpr int kPPThreads = 384;
constexpr uint32_t kPPRegsLaunch = 168, kPPRegsSoftmax = 216, kPPRegsOther = 72;
static_assert(kPPRegsOther * 128 + kPPRegsSoftmax * 256 <= kPPRegsLaunch * kPPThreads, "register split");

template <int D>
struct FwdPPCfg {
  static constexpr int ATOMS = D / 64;
  static constexpr int TILE_BYTES = ATOMS * 128 * 128;
  static constexpr int STAGES = 2;
  static constexpr int Q_OFF = 0;  // two Q tiles
  static constexpr int K_OFF = 2 * TILE_BYTES;
  static constexpr int V_OFF = K_OFF + STAGES * TILE_BYTES;
  static constexpr int BAR_OFF = V_OFF + STAGES * TILE_BYTES;
  static constexpr int SMEM = 1024 + BAR_OFF + 256;
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// One work item of the two-tile kernel: (batch * head, first query row, key tiles of each tile).
struct PPItem {
  int bh, m0, n0, n1;
};

// The CTA's r-th item (snake order over gridDim.x CTAs); false past the last item. Every role of the
// CTA walks the same sequence.
__device__ __forceinline__ bool pp_item(const AttnFwdParams& p, int r, PPItem& it) {
  const int G = (int)gridDim.x;
  const int pairs = (p.m_tiles + 1) >> 1;
  const int n_items = p.B * p.Hq * pairs;
  const int k = r * G + ((r & 1) ? G - 1 - (int)blockIdx.x : (int)blockIdx.x);
  if (k >= n_items) return false;
  const int BHq = p.B * p.Hq;
  int pair;
  if (p.causal) {
    pair = pairs - 1 - k / BHq;
    it.bh = k % BHq;
  } else {
    pair = k % pairs;
    it.bh = k / pairs;
  }
  it.m0 = pair * 2 * BM;
  // key tiles per query tile (tile 1 may lie past the end of the sequence: no work)
  auto kv_tiles = [&](int t) -> int {
    const int r0 = it.m0 + t * BM;
    if (r0 >= p.Sq) return 0;
    const int kv_end = p.causal ? min(p.Sk, r0 + BM) : p.Sk;
    return (kv_end + BN - 1) / BN;
  };
  it.n0 = kv_tiles(0);
  it.n1 = kv_tiles(1);
  return true;
}

template <int D, bool DROP>
__global__ void __launch_bounds__(kPPThreads, 1)
    attn_fwd_pp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const AttnFwdParams p) {
  using C = FwdPPCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;   // [2]
  uint64_t* k_empty = bars + 4;  // [2]
  uint64_t* v_full = bars + 6;   // [2]
  uint64_t* v_empty = bars + 8;  // [2]
  uint64_t* s_full = bars + 10;  // [tile]
  uint64_t* p_full = bars + 12;  // [tile]
  uint64_t* pv_done = bars + 14; // [tile]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 9) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // each role's code sits under its warpgroup's register re-split
  if (warp >= 8) {
    setmaxnreg_dec<kPPRegsOther>();
    if (warp == 8) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      uint32_t g = 0;  // K/V ring slots used so far (across items)
      PPItem it;
      for (int r = 0; pp_item(p, r, it); ++r) {
        const int bhk = (it.bh / p.Hq) * p.Hkv + (it.bh % p.Hq) / p.group;
        const int n_kv = max(it.n0, it.n1);
        // the previous item's S MMAs have all completed before its Q tiles are overwritten
        if (r > 0 && !mbar_wait(q_empty, (r - 1) & 1, abort, p.err)) break;
        mbar_arrive_expect_tx(q_full, 2 * C::TILE_BYTES);
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int a = 0; a < C::ATOMS; ++a)
            tma_load_3d(smem + C::Q_OFF + t * C::TILE_BYTES + a * 16384, &tmQ, q_full, a * 64, it.m0 + t * BM, it.bh);
        bool ok = true;
        for (int j = 0; j < n_kv; ++j, ++g) {
          const int st = g & 1;
          const uint32_t ph = (g >> 1) & 1;
          if (!mbar_wait(&k_empty[st], ph ^ 1, abort, p.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&k_full[st], C::TILE_BYTES);
#pragma unroll
          for (int a = 0; a < C::ATOMS; ++a)
            tma_load_3d(smem + C::K_OFF + st * C::TILE_BYTES + a * 16384, &tmK, &k_full[st], a * 64, j * BN, bhk);
          if (!mbar_wait(&v_empty[st], ph ^ 1, abort, p.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&v_full[st], C::TILE_BYTES);
#pragma unroll
          for (int a = 0; a < C::ATOMS; ++a)
            tma_load_3d(smem + C::V_OFF + st * C::TILE_BYTES + a * 16384, &tmV, &v_full[st], a * 64, j * BN, bhk);
        }
        if (!ok) break;
      }
    }
    } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs the loop so operands stay warp-uniform; one elected lane issues.
    constexpr uint32_t idesc_s = idesc_f16_f32(BM, BN, false, false);
    constexpr uint32_t idesc_o = idesc_f16_f32(BM, D, false, true);
    // descriptors: a k16 step adds its byte offset / 16 to the 14-bit start-address field (shared
    // addresses stay below 2^18 bytes, so it cannot carry out)
    const uint64_t qd0 = smem_desc_sw128(smem_u32(smem + C::Q_OFF), 16, 1024);
    const uint64_t kd0 = smem_desc_sw128(smem_u32(smem + C::K_OFF), 16, 1024);
    const uint64_t vd0 = smem_desc_sw128(smem_u32(smem + C::V_OFF), 16384, 1024);
    constexpr uint32_t kTile16 = C::TILE_BYTES >> 4;
    auto issue_s = [&](int t, uint32_t slot) {  // S_t = Q_t K^T (K in ring slot `slot`) into tile t's S columns
      const uint64_t qd = qd0 + t * kTile16, kd = kd0 + (slot & 1) * kTile16;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off16 = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
        umma_f16_ss(tmem + t * 256, qd + off16, kd + off16, idesc_s, kk > 0 ? 1u : 0u);
      }
      umma_commit(&s_full[t]);
    };
    auto issue_pv = [&](int t, uint32_t slot, bool first) {  // O_t (+)= P_t V, P (128 x 128 fp16) from TMEM
      const uint64_t vd = vd0 + (slot & 1) * kTile16;
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk)
        umma_f16_ts(tmem + t * 256 + 128, tmem + t * 256 + kk * 8, vd + (kk * 2048 >> 4), idesc_o,
                    (!first || kk > 0) ? 1u : 0u);
    };
    uint32_t g = 0;              // K/V ring slots consumed so far (across items)
    uint32_t pw[2] = {0u, 0u};   // p_full phases consumed per tile
    bool ok = true;
    PPItem it;
    for (int r = 0; ok && pp_item(p, r, it); ++r) {
      const int n_kv = max(it.n0, it.n1);
      ok = mbar_wait_warp(q_full, r & 1, abort, p.err) && mbar_wait_warp(&k_full[g & 1], (g >> 1) & 1, abort, p.err);
      if (!ok) break;
      tc_fence_after();
      if (elect_one()) {
        if (it.n0 > 0) issue_s(0, g);
        if (it.n1 > 0) issue_s(1, g);
        umma_commit(&k_empty[g & 1]);
        if (n_kv == 1) umma_commit(q_empty);
      }
      __syncwarp();
      for (int j = 0; j < n_kv; ++j) {
        const uint32_t gj = g + j;
        const int st = gj & 1;
        const bool next = j + 1 < n_kv;
        if (!mbar_wait_warp(&v_full[st], (gj >> 1) & 1, abort, p.err)) { ok = false; break; }
        if (next && !mbar_wait_warp(&k_full[st ^ 1], ((gj + 1) >> 1) & 1, abort, p.err)) { ok = false; break; }
        for (int t = 0; t < 2; ++t) {
          const int nt = t == 0 ? it.n0 : it.n1;
          if (j >= nt) continue;
          if (!mbar_wait_warp(&p_full[t], pw[t] & 1, abort, p.err)) { ok = false; break; }
          ++pw[t];
          tc_fence_after();
          if (elect_one()) {
            issue_pv(t, gj, j == 0);
            if (j + 1 < nt) issue_s(t, gj + 1);
            else umma_commit(&pv_done[t]);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) {
          umma_commit(&v_empty[st]);
          if (next) umma_commit(&k_empty[st ^ 1]);
          // every S MMA of the item has been issued: the Q tiles are free once they complete
          if (j == n_kv - 2) umma_commit(q_empty);
        }
        __syncwarp();
      }
      g += n_kv;
    }
    }
  } else {
    setmaxnreg_inc<kPPRegsSoftmax>();
    // ---------------------------------------------------------------- softmax + epilogue
    const int t = warp >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + t * 256;
    const uint32_t o_addr = s_addr + 128;
    uint32_t sw = 0, dw = 0;  // s_full and pv_done phases consumed
    bool ok = true;
    PPItem it;
    for (int ri = 0; ok && pp_item(p, ri, it); ++ri) {
      const int bh = it.bh;
      const int b = bh / p.Hq, h = bh % p.Hq;
      const int bhk = b * p.Hkv + h / p.group;
      const int m_t = it.m0 + t * BM;
      const int qi = m_t + r;
      const int nt = t == 0 ? it.n0 : it.n1;
      const uint32_t rk = DROP ? drop_row_key(p.seed_lo, p.seed_hi, (uint32_t)bh, (uint32_t)qi) : 0u;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nt; ++j) {
        if (!mbar_wait_warp(&s_full[t], sw & 1, abort, p.err)) { ok = false; break; }
        ++sw;
        tc_fence_after();
        const int k0 = j * BN;
        const bool full_tile = p.mask == nullptr && k0 + BN <= p.Sk && (!p.causal || k0 + BN - 1 <= m_t);
        // Logits of a full tile stay raw (s) and are scaled inside the exp, p = 2^(s * c - m) with
        // c = scale * log2(e) > 0 (the max commutes with it). A partial tile (sequence end, causal
        // diagonal, user mask) maps s to the scaled, masked logit first and uses c = 1.
        const float c_scale = full_tile ? p.scale_log2 : 1.f;
        if (!full_tile)
          mask_logits_tmem(s_addr, BN, k0, qi, p,
                           p.mask ? p.mask + b * p.mb + h * p.mh + (int64_t)min(qi, p.Sq - 1) * p.mi + k0 : nullptr);
        // the whole 128-column S row in registers: four loads in flight, one wait
        uint32_t rr[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&rr[c * 32]));
        tmem_ld_wait();
        // row max: 8 independent 3-input max chains
        float m8[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) m8[e] = __uint_as_float(rr[e]);
#pragma unroll
        for (int e = 8; e < BN; e += 2) m8[(e >> 1) & 7] = max3f(m8[(e >> 1) & 7], __uint_as_float(rr[e]), __uint_as_float(rr[e + 1]));
        const float mx = max3f(max3f(m8[0], m8[1], m8[2]), max3f(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7])) * c_scale;
        float alpha = 1.f;
        bool rescale = false;
        if (mx > m_used + kRescaleLog2 || (m_used == -INFINITY && mx > -INFINITY)) {
          alpha = (m_used == -INFINITY) ? 0.f : ex2(m_used - mx);
          rescale = j > 0;
          m_used = mx;
          l *= alpha;
        }
        // P = 2^(logit - m) packed to fp16 in place (pair e/2 overwrites a register already read); the
        // scaling and the row sum run on fp32 pairs, and three pairs in eight take the FMA-pipe exp2 so
        // the MUFU pipe is not the only exp unit
        const float base = m_used == -INFINITY ? 0.f : m_used;
        const uint64_t c2 = f2_pack(c_scale, c_scale), nb2 = f2_pack(-base, -base);
        uint64_t sum4[4] = {0, 0, 0, 0};
#pragma unroll
        for (int e = 0; e < BN; e += 2) {
          float x0, x1, p0, p1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(rr[e]), __uint_as_float(rr[e + 1])), c2, nb2), x0, x1);
          if (((e >> 1) & 7) >= 8 - kPolyPairsOf8) {
            ex2_poly2(x0, x1, p0, p1);
          } else {
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          sum4[(e >> 1) & 3] = f2_add(sum4[(e >> 1) & 3], f2_pack(p0, p1));
          rr[e >> 1] = pack_f16(p0, p1);
          // dropout: the row sum keeps every key; P.V sees only the kept ones (scaled back at the end)
          if constexpr (DROP) rr[e >> 1] &= drop_pair_mask(rk, (uint32_t)(k0 + e) >> 1, p.drop_thr);
        }
        {
          float a0, a1;
          f2_unpack(f2_add(f2_add(sum4[0], sum4[1]), f2_add(sum4[2], sum4[3])), a0, a1);
          l += a0 + a1;
        }
        // P of keys [0, 128) onto S columns [0, 64)
        tmem_st32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&rr[0]));
        tmem_st32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&rr[32]));
        // O is complete up to P.V_{j-1} (it precedes S_j in the MMA pipe): rescale it in place if needed,
        // the whole row in one TMEM round trip (the S registers are free again)
        if (__any_sync(0xffffffffu, rescale)) {
          uint32_t o[D];
#pragma unroll
          for (int c = 0; c < D / 32; ++c) tmem_ld32(o_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&o[c * 32]));
          tmem_ld_wait();
          const float a = rescale ? alpha : 1.f;
          const uint64_t a2 = f2_pack(a, a);
#pragma unroll
          for (int e = 0; e < D; e += 2) {
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(o[e]), __uint_as_float(o[e + 1])), a2, 0), x0, x1);
            o[e] = __float_as_uint(x0);
            o[e + 1] = __float_as_uint(x1);
          }
#pragma unroll
          for (int c = 0; c < D / 32; ++c) tmem_st32(o_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&o[c * 32]));
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
      if (!ok || nt == 0) continue;
      if (!mbar_wait_warp(&pv_done[t], dw & 1, abort, p.err)) { ok = false; break; }
      ++dw;
      tc_fence_after();
      // O leaves TMEM here; the next item's first P.V overwrites it only after this warp's next
      // p_full arrival, which follows these loads (tcgen05.wait::ld, then the fence before the arrive)
      const float inv_l = l > 0.f ? (DROP ? p.inv_keep : 1.f) / l : 0.f;
      const float sc = exp2i(__ldg(p.ev + bhk));
      __nv_bfloat16* orow = p.out + (int64_t)b * p.osb + (int64_t)h * p.osh + (int64_t)min(qi, p.Sq - 1) * p.oss;
      __half* o16row = p.o16 ? p.o16 + ((int64_t)bh * p.Sq + min(qi, p.Sq - 1)) * D : nullptr;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(o_addr + c * 32, o);
        tmem_ld_wait();
        if (qi < p.Sq) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(o[8 * g + e]) * inv_l;
            *reinterpret_cast<uint4*>(orow + c * 32 + g * 8) =
                make_uint4(pack_bf16(v[0] * sc, v[1] * sc), pack_bf16(v[2] * sc, v[3] * sc),
                           pack_bf16(v[4] * sc, v[5] * sc), pack_bf16(v[6] * sc, v[7] * sc));
            if (o16row)
              *reinterpret_cast<uint4*>(o16row + c * 32 + g * 8) = make_uint4(
                  pack_f16(v[0], v[1]), pack_f16(v[2], v[3]), pack_f16(v[4], v[5]), pack_f16(v[6], v[7]));
          }
        }
      }
      if (p.lse && qi < p.Sq) p.lse[(int64_t)bh * p.lse_ld + qi] = (m_used + log2f(l)) * 0.6931471805599453f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort) {
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 2000000ull) {
    }
  }
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool DROP>
int launch_fwd_pp(const void* q16, const void* k16, const void* v16, const AttnFwdParams& prm, cudaStream_t st) {
  using C = FwdPPCfg<D>;
  const tbf16_host::DeviceInfo* dev = tbf16_host::device_info();
  if (!dev) return TBF16_ERR_DEVICE;
  CUtensorMap tq, tk, tv;
  const int64_t BHq = (int64_t)prm.B * prm.Hq, BHk = (int64_t)prm.B * prm.Hkv;
  if (int rc = tbf16_host::make_tmap_3d(&tq, q16, D, prm.Sq, BHq, D, (uint64_t)prm.Sq * D, 64, BM)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tk, k16, D, prm.Sk, BHk, D, (uint64_t)prm.Sk * D, 64, BN)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tv, v16, D, prm.Sk, BHk, D, (uint64_t)prm.Sk * D, 64, BN)) return rc;
  static bool attr_done[64] = {false};
  if (!attr_done[dev->device & 63]) {
    if (cudaFuncSetAttribute(attn_fwd_pp_kernel<D, DROP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return tbf16_host::check_launch();
    attr_done[dev->device & 63] = true;
  }
  // one CTA per SM (shared memory and the 512 TMEM columns allow no second), never more than the items
  const int64_t items = BHq * ((prm.m_tiles + 1) / 2);
  if (items > INT32_MAX - 2 * (int64_t)dev->sms) return TBF16_ERR_INVALID;  // item indices are int
  const unsigned grid = (unsigned)std::min<int64_t>(items, dev->sms);
  attn_fwd_pp_kernel<D, DROP><<<grid, kPPThreads, C::SMEM, st>>>(tq, tk, tv, prm);
  return tbf16_host::check_launch();
}

template <int D, bool DROP>
int launch_fwd(const void* q16, const void* k16, const void* v16, const AttnFwdParams& prm, cudaStream_t st) {
  using C = FwdCfg<D>;
  const tbf16_host::DeviceInfo* dev = tbf16_host::device_info();
  if (!dev) return TBF16_ERR_DEVICE;
  CUtensorMap tq, tk, tv;
  const int64_t BHq = (int64_t)prm.B * prm.Hq, BHk = (int64_t)prm.B * prm.Hkv;
  if (int rc = tbf16_host::make_tmap_3d(&tq, q16, D, prm.Sq, BHq, D, (uint64_t)prm.Sq * D, 64, BM)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tk, k16, D, prm.Sk, BHk, D, (uint64_t)prm.Sk * D, 64, BN)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tv, v16, D, prm.Sk, BHk, D, (uint64_t)prm.Sk * D, 64, BN)) return rc;
  static bool attr_done[64] = {false};
  if (!attr_done[dev->device & 63]) {
    if (cudaFuncSetAttribute(attn_fwd_kernel<D, DROP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
      return tbf16_host::check_launch();
    attr_done[dev->device & 63] = true;
  }
  const dim3 grid = prm.causal ? dim3((unsigned)BHq, prm.m_tiles) : dim3(prm.m_tiles, (unsigned)BHq);
  attn_fwd_kernel<D, DROP><<<grid, kThreads, C::SMEM, st>>>(tq, tk, tv, prm);
  return tbf16_host::check_launch();
}

// ------------------------------------------------------------------------------------------------
// Head dim 256: a persistent kernel over CTA pairs (clusters of two, cta_group::2 MMAs issued by the
// even CTA), one pair per two SMs; a work item is 256 query rows of one head, CTA c of the pair
// owning rows m0 + 128 c .. + 127 (its TMEM lanes).
//   S = Q K^T    M = 256 (the pair's rows), N = 128 keys, K = 256: each CTA holds its own Q rows and
//                half of the key tile (keys 64 c .. 64 c + 63 of it, all 256 dims), 32 KB a stage
//   O += P V     M = 256, N = 256 dims, K = 128 keys: P is read from each CTA's TMEM (TS form), each
//                CTA holds dims 128 c .. 128 c + 127 of the V tile (128 keys), 32 KB a stage
// so that two K and two V stages fit beside the 64 KB Q tile. TMEM per CTA: S0 [0,128), S1 [128,256),
// O [256,512); P is written over its S buffer's first 64 columns as packed fp16. Steps are counted
// across items (the K/V rings, S buffers and barrier phases run on); per item the MMA warp issues
//   S_0 S_1 | PV_0 S_2 | PV_1 S_3 | ... | PV_n-1
// so each step's softmax runs while the tensor core computes the previous step's P.V and the next S.
// In issue order S_{j+2} (overwriting P_j) follows PV_j. The softmax rescales O (lazily, when its
// running max grows by more than 2^8) only after PV_{j-1} has completed, and PV_j waits for both
// CTAs' P_j, so the rescale lands between them. Between items: the Q tiles are released once the
// item's last S has completed (the next Q loads during the last steps), the next item's S_0 and S_1
// run while the softmax warps write the output, and its PV_0 (which overwrites O) waits for their
// first P of the new item, produced after they have read O out. Items are ordered heads fastest and
// heaviest first (causal) or row pairs fastest, and dealt to the pairs in snake order.
//   warps 0-3  softmax + epilogue (one query row per thread)    warp 4  TMA producer (both CTAs)
//   warp 5     MMA issuer (even CTA) + TMEM allocation (both)
namespace fwd256 {
constexpr int THREADS = 192;
constexpr int ROWS = 128;                 // query rows per CTA
constexpr int KEYS = 128;                 // keys per tile
constexpr int Q_BYTES = 4 * 16384;        // 128 rows x 256 dims, four 64-dim atoms
constexpr int KH_BYTES = 4 * 8192;        // 64 keys x 256 dims, four 64-dim atoms
constexpr int VH_BYTES = 2 * 16384;       // 128 keys x 128 dims, two 64-dim atoms
constexpr int Q_OFF = 0;
constexpr int K_OFF = Q_OFF + Q_BYTES;
constexpr int V_OFF = K_OFF + 2 * KH_BYTES;
constexpr int BAR_OFF = V_OFF + 2 * VH_BYTES;
constexpr int SMEM = 1024 + BAR_OFF + 256;
static_assert(SMEM <= 227 * 1024, "shared memory");

// Key-split launches. When the items are too few for the pairs (one 2048-token sequence of 8 heads is
// 64 items on 74 pairs, and the last 256 rows' 16 key tiles set the kernel's time), the host cuts the
// heaviest items into two parts over their key tiles and deals all parts to the pairs longest first
// (LPT). Both parts of an item end with their own (O, running max, row sum) for the same rows; per 32-row
// warp slot, whichever finishes first (a ticket in the workspace) writes its part there and raises a
// flag, the second one waits for that flag, adds the two parts and writes the output. The first never
// waits on anything but its own pair's MMAs, so the wait always ends.
constexpr int kSchedPairs = 80;      // >= the pairs of a 148-SM device
constexpr int kSchedEntries = 256;   // parts of one launch
constexpr int kSplitItems = 128;     // split items of one launch
constexpr int kSplitSlots = kSplitItems * 8;  // (item, CTA, softmax warp)
constexpr int64_t kSplitHdrBytes = 2 * kSplitSlots * 4;  // tickets, then flags
constexpr int kSlotFloats = 256 * 32 + 64;    // a warp's 32 rows x 256 dims of O, then 32 maxima, 32 sums
template <bool SPLIT>
struct Sched {
  uint16_t start[kSchedPairs + 1];  // pair c runs e[start[c]] .. e[start[c + 1] - 1] in order
  uint64_t e[kSchedEntries];        // bh | row pair << 16 | first key tile << 30 | key tiles << 43 | sid << 56
};
template <>
struct Sched<false> {
  int unused;
};

struct Item {
  int bh, m0, kb, n_kv, sid;  // key tiles kb .. kb + n_kv - 1; sid > 0: part of split item sid - 1
};
// The pair's r-th item; false past the last one. Every role of both CTAs walks the same sequence.
// Without a schedule: snake order over the gridDim.x / 2 pairs.
template <bool SPLIT>
__device__ __forceinline__ bool item_at(const AttnFwdParams& p, const Sched<SPLIT>& sc, int r, Item& it) {
  if constexpr (SPLIT) {
    const int c = (int)(blockIdx.x >> 1);
    const int k = sc.start[c] + r;
    if (k >= sc.start[c + 1]) return false;
    const uint64_t e = sc.e[k];
    it.bh = (int)(e & 0xffffu);
    it.m0 = (int)((e >> 16) & 0x3fffu) * 2 * ROWS;
    it.kb = (int)((e >> 30) & 0x1fffu);
    it.n_kv = (int)((e >> 43) & 0x1fffu);
    it.sid = (int)(e >> 56);
    return true;
  }
  const int G = (int)(gridDim.x >> 1), c = (int)(blockIdx.x >> 1);
  const int pairs = (p.Sq + 2 * ROWS - 1) / (2 * ROWS);
  const int BHq = p.B * p.Hq;
  const int k = r * G + ((r & 1) ? G - 1 - c : c);
  if (k >= BHq * pairs) return false;
  int pr;
  if (p.causal) {
    pr = pairs - 1 - k / BHq;
    it.bh = k % BHq;
  } else {
    pr = k % pairs;
    it.bh = k / pairs;
  }
  it.m0 = pr * 2 * ROWS;
  const int kv_end = p.causal ? min(p.Sk, it.m0 + 2 * ROWS) : p.Sk;
  it.kb = 0;
  it.n_kv = (kv_end + KEYS - 1) / KEYS;
  it.sid = 0;
  return true;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* f) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* f, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
// Warp-wide bounded wait for a flag another CTA raises: lane 0 polls, then every lane takes its own
// acquire so that its loads of the flagged data follow it.
__device__ __forceinline__ bool flag_wait_warp(const int* f, volatile int* abort, unsigned int* err,
                                               uint64_t timeout_ns = 2000000000ull) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0 && ld_acquire_gpu(f) == 0) {
    const uint64_t t0 = global_timer_ns();
    while (ld_acquire_gpu(f) == 0) {
      if (*abort) { ok = false; break; }
      if (global_timer_ns() - t0 > timeout_ns) {
        atomicOr(err, kErrWaitTimeout);
        *abort = 1;
        ok = false;
        break;
      }
      __nanosleep(100);
    }
  }
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  if (ok) (void)ld_acquire_gpu(f);
  return ok;
}
}  // namespace fwd256

template <bool DROP, bool SPLIT>
__global__ void __launch_bounds__(fwd256::THREADS, 1)
    attn_fwd_d256_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                              const __grid_constant__ CUtensorMap tmV, const AttnFwdParams p,
                              const __grid_constant__ fwd256::Sched<SPLIT> sched) {
  using namespace fwd256;
  constexpr int D = 256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* q_full = bars + 0;    // even CTA's: both CTAs' Q bytes
  uint64_t* q_empty = bars + 1;   // both (commit to both CTAs)
  uint64_t* k_full = bars + 2;    // [2] even CTA's
  uint64_t* v_full = bars + 4;    // [2] even CTA's
  uint64_t* k_empty = bars + 6;   // [2] both
  uint64_t* v_empty = bars + 8;   // [2] both
  uint64_t* s_full = bars + 10;   // [2] both
  uint64_t* p_full = bars + 12;   // [2] even CTA's: 4 softmax warps of each CTA
  uint64_t* pv_done = bars + 14;  // both
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);
    }
    mbar_init(pv_done, 1);
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 5) tmem_alloc_pair(tmem_slot, 512);
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      uint32_t g = 0;  // K/V ring slots used so far (across items)
      int r = 0;
      bool ok = true;
      Item it;
      for (; ok && item_at(p, sched, r, it); ++r) {
        const int bhk = (it.bh / p.Hq) * p.Hkv + (it.bh % p.Hq) / p.group;
        // the previous item's S MMAs have all completed before the Q tiles are overwritten
        if (r > 0 && !mbar_wait(q_empty, (r - 1) & 1, abort, p.err)) { ok = false; break; }
        if (leader) mbar_arrive_expect_tx(q_full, 2 * Q_BYTES);
#pragma unroll
        for (int a = 0; a < 4; ++a)
          tma_load_3d_pair(smem + Q_OFF + a * 16384, &tmQ, q_full, a * 64, it.m0 + (int)rank * ROWS, it.bh);
        for (int j = 0; j < it.n_kv; ++j, ++g) {
          const int st = g & 1;
          const uint32_t ph = (g >> 1) & 1;
          if (!mbar_wait(&k_empty[st], ph ^ 1, abort, p.err)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&k_full[st], 2 * KH_BYTES);
#pragma unroll
          for (int a = 0; a < 4; ++a)
            tma_load_3d_pair(smem + K_OFF + st * KH_BYTES + a * 8192, &tmK, &k_full[st], a * 64,
                             (it.kb + j) * KEYS + (int)rank * (KEYS / 2), bhk);
          if (!mbar_wait(&v_empty[st], ph ^ 1, abort, p.err)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&v_full[st], 2 * VH_BYTES);
#pragma unroll
          for (int a = 0; a < 2; ++a)
            tma_load_3d_pair(smem + V_OFF + st * VH_BYTES + a * 16384, &tmV, &v_full[st], (int)rank * 128 + a * 64,
                             (it.kb + j) * KEYS, bhk);
        }
      }
      // the even CTA's last releases of this CTA's Q tiles and ring stages have landed before the CTA
      // may exit
      if (ok && r > 0) ok = mbar_wait(q_empty, (r - 1) & 1, abort, p.err);
      for (int st = 0; ok && st < 2; ++st) {
        const uint32_t uses = (g + 1 - st) / 2;
        if (uses > 0)
          ok = mbar_wait(&k_empty[st], (uses - 1) & 1, abort, p.err) && mbar_wait(&v_empty[st], (uses - 1) & 1, abort, p.err);
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA issuer (even CTA)
    if (leader && lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16_f32(2 * ROWS, KEYS, false, false);
      constexpr uint32_t idesc_o = idesc_f16_f32(2 * ROWS, D, false, true);
      const uint64_t qd0 = smem_desc_sw128(smem_u32(smem + Q_OFF), 16, 1024);
      const uint64_t kd0 = smem_desc_sw128(smem_u32(smem + K_OFF), 16, 1024);
      const uint64_t vd0 = smem_desc_sw128(smem_u32(smem + V_OFF), 16384, 1024);
      auto issue_s = [&](uint32_t gs) -> bool {  // S of ring slot gs into S buffer gs & 1 of both CTAs
        const int st = gs & 1;
        if (!mbar_wait(&k_full[st], (gs >> 1) & 1, abort, p.err)) return false;
        tc_fence_after();
        const uint64_t kd = kd0 + (uint64_t)((st * KH_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t offq = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
          const uint32_t offk = ((kk >> 2) * 8192 + (kk & 3) * 32) >> 4;
          umma_f16_ss_pair(tmem + st * KEYS, qd0 + offq, kd + offk, idesc_s, kk > 0 ? 1u : 0u);
        }
        umma_commit_pair(&s_full[st], 0x3);
        umma_commit_pair(&k_empty[st], 0x3);
        return true;
      };
      auto issue_pv = [&](uint32_t gs, bool first) -> bool {  // O (+)= P V of slot gs, P from both CTAs' TMEM
        const int st = gs & 1;
        if (!mbar_wait_cluster(&p_full[st], (gs >> 1) & 1, abort, p.err)) return false;
        if (!mbar_wait(&v_full[st], (gs >> 1) & 1, abort, p.err)) return false;
        tc_fence_after();
        const uint64_t vd = vd0 + (uint64_t)((st * VH_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < KEYS / 16; ++kk)
          umma_f16_ts_pair(tmem + 256, tmem + st * KEYS + kk * 8, vd + ((kk * 2048) >> 4), idesc_o,
                           (!first || kk > 0) ? 1u : 0u);
        umma_commit_pair(&v_empty[st], 0x3);
        umma_commit_pair(pv_done, 0x3);
        return true;
      };
      uint32_t g = 0;  // steps (ring slots) issued so far (across items)
      bool ok = true;
      Item it;
      for (int r = 0; ok && item_at(p, sched, r, it); ++r) {
        const int n = it.n_kv;
        ok = mbar_wait(q_full, r & 1, abort, p.err) && issue_s(g) && (n < 2 || issue_s(g + 1));
        if (ok && n <= 2) umma_commit_pair(q_empty, 0x3);  // every S of the item issued
        for (int j = 0; ok && j < n; ++j) {
          ok = issue_pv(g + j, j == 0) && (j + 2 >= n || issue_s(g + j + 2));
          if (ok && j + 2 == n - 1) umma_commit_pair(q_empty, 0x3);
        }
        g += n;
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax + epilogue (both CTAs)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    const uint32_t o_addr = tmem + lane_base + 256;
    uint32_t g = 0;  // steps consumed so far (across items)
    bool ok = true;
    Item it;
    for (int ri = 0; ok && item_at(p, sched, ri, it); ++ri) {
      const int bh = it.bh;
      const int b = bh / p.Hq, h = bh % p.Hq;
      const int bhk = b * p.Hkv + h / p.group;
      const int mc = it.m0 + (int)rank * ROWS;  // this CTA's first query row
      const int qi = mc + r;
      const int n_kv = it.n_kv;
      const uint32_t rk = DROP ? drop_row_key(p.seed_lo, p.seed_hi, (uint32_t)bh, (uint32_t)qi) : 0u;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < n_kv; ++j) {
        const uint32_t gs = g + j;
        const int sb = gs & 1;
        if (!mbar_wait_warp(&s_full[sb], (gs >> 1) & 1, abort, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t s_addr = tmem + lane_base + sb * KEYS;
        const int k0 = (it.kb + j) * KEYS;
        uint32_t rr[KEYS];
        float alpha = 1.f;
        bool rescale = false;
        const bool dead = p.causal && k0 > mc + ROWS - 1;
        if (dead) {
          // every key of the tile lies after every row of this CTA (the pair's last tile, even CTA): P = 0
#pragma unroll
          for (int e = 0; e < KEYS / 2; ++e) rr[e] = 0u;
        } else {
          const bool full_tile = p.mask == nullptr && k0 + KEYS <= p.Sk && (!p.causal || k0 + KEYS - 1 <= mc);
          const float c_scale = full_tile ? p.scale_log2 : 1.f;
          if (!full_tile)
            mask_logits_tmem(s_addr, KEYS, k0, qi, p,
                             p.mask ? p.mask + b * p.mb + h * p.mh + (int64_t)min(qi, p.Sq - 1) * p.mi + k0 : nullptr);
#pragma unroll
          for (int c = 0; c < KEYS / 32; ++c) tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&rr[c * 32]));
          tmem_ld_wait();
          float m8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) m8[e] = __uint_as_float(rr[e]);
#pragma unroll
          for (int e = 8; e < KEYS; e += 2)
            m8[(e >> 1) & 7] = max3f(m8[(e >> 1) & 7], __uint_as_float(rr[e]), __uint_as_float(rr[e + 1]));
          const float mx = max3f(max3f(m8[0], m8[1], m8[2]), max3f(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7])) * c_scale;
          if (mx > m_used + kRescaleLog2 || (m_used == -INFINITY && mx > -INFINITY)) {
            alpha = (m_used == -INFINITY) ? 0.f : ex2(m_used - mx);
            rescale = j > 0;
            m_used = mx;
            l *= alpha;
          }
          const float base = m_used == -INFINITY ? 0.f : m_used;
          const uint64_t c2 = f2_pack(c_scale, c_scale), nb2 = f2_pack(-base, -base);
          uint64_t sum4[4] = {0, 0, 0, 0};
#pragma unroll
          for (int e = 0; e < KEYS; e += 2) {
            float x0, x1, p0, p1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(rr[e]), __uint_as_float(rr[e + 1])), c2, nb2), x0, x1);
            if (((e >> 1) & 7) >= 8 - kPolyPairsOf8) {
              ex2_poly2(x0, x1, p0, p1);
            } else {
              p0 = ex2(x0);
              p1 = ex2(x1);
            }
            sum4[(e >> 1) & 3] = f2_add(sum4[(e >> 1) & 3], f2_pack(p0, p1));
            rr[e >> 1] = pack_f16(p0, p1);
            if constexpr (DROP) rr[e >> 1] &= drop_pair_mask(rk, (uint32_t)(k0 + e) >> 1, p.drop_thr);
          }
          {
            float a0, a1;
            f2_unpack(f2_add(f2_add(sum4[0], sum4[1]), f2_add(sum4[2], sum4[3])), a0, a1);
            l += a0 + a1;
          }
        }
        // O is complete once P.V of the previous step has: wait for it at every step of the item (the
        // epilogue waited for the last one of the previous item), so that no phase of the barrier is
        // skipped, then rescale O if this row's max moved. This step's P.V cannot start before this
        // warp's arrival below, so the barrier is never more than one phase ahead of the wait.
        if (j > 0) {
          if (!mbar_wait_warp(pv_done, (gs - 1) & 1, abort, p.err)) { ok = false; break; }
          tc_fence_after();
        }
        if (!dead && __any_sync(0xffffffffu, rescale)) {
          const float a = rescale ? alpha : 1.f;
          const uint64_t a2 = f2_pack(a, a);
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t o[64];
            tmem_ld32(o_addr + c * 64, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
            tmem_ld32(o_addr + c * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 64; e += 2) {
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(o[e]), __uint_as_float(o[e + 1])), a2, 0), x0, x1);
              o[e] = __float_as_uint(x0);
              o[e + 1] = __float_as_uint(x1);
            }
            tmem_st32(o_addr + c * 64, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
            tmem_st32(o_addr + c * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
          }
        }
        // P of the tile's 128 keys onto the S buffer's columns [0, 64)
        tmem_st32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&rr[0]));
        tmem_st32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&rr[32]));
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader) mbar_arrive(&p_full[sb]);
          else mbar_arrive_remote_tmem(&p_full[sb], 0);
        }
      }
      if (!ok) break;
      g += n_kv;
      // a split item's part takes its ticket once its last P is handed over, so the atomic's round trip
      // overlaps the last P.V (which part is first only decides who writes and who adds)
      const int slot = ((it.sid - 1) * 2 + (int)rank) * 4 + quad;
      int ticket_v = 0;
      if constexpr (SPLIT)
        if (it.sid > 0 && lane == 0) ticket_v = atomicAdd(static_cast<int*>(p.split_ws) + slot, 1);
      // epilogue: O leaves TMEM here; the next item's first P.V overwrites it only after this warp's
      // next p_full arrival, which follows these loads
      if (!mbar_wait_warp(pv_done, (g - 1) & 1, abort, p.err)) { ok = false; break; }
      tc_fence_after();
      float f_own = 1.f, f_oth = 0.f;  // weights of this part's O and of the other part's
      const float4* oth = nullptr;     // the other part's O (a split item's second part to finish)
      if constexpr (SPLIT) {
        if (it.sid > 0) {
          int* flag = static_cast<int*>(p.split_ws) + kSplitSlots + slot;
          float* part =
              reinterpret_cast<float*>(static_cast<uint8_t*>(p.split_ws) + kSplitHdrBytes) + (int64_t)slot * kSlotFloats;
          const int t = __shfl_sync(0xffffffffu, ticket_v, 0);
          if (t == 0) {
            // first part to finish: O (groups of 4 dims, lanes fastest), then its max and sum, to the slot
            float4* o4 = reinterpret_cast<float4*>(part);
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
              uint32_t o[32];
              tmem_ld32(o_addr + c * 32, o);
              tmem_ld_wait();
#pragma unroll
              for (int q = 0; q < 8; ++q)
                __stcg(o4 + (c * 8 + q) * 32 + lane,
                       make_float4(__uint_as_float(o[4 * q]), __uint_as_float(o[4 * q + 1]),
                                   __uint_as_float(o[4 * q + 2]), __uint_as_float(o[4 * q + 3])));
            }
            __stcg(part + D * 32 + lane, m_used);
            __stcg(part + D * 32 + 32 + lane, l);
            __threadfence();
            __syncwarp();
            if (lane == 0) st_release_gpu(flag, 1);
            continue;
          }
          if (!flag_wait_warp(flag, abort, p.err)) { ok = false; break; }
          const float m2 = __ldcg(part + D * 32 + lane), l2 = __ldcg(part + D * 32 + 32 + lane);
          const float mn = fmaxf(m_used, m2);
          f_own = m_used == -INFINITY ? 0.f : ex2(m_used - mn);
          f_oth = m2 == -INFINITY ? 0.f : ex2(m2 - mn);
          // products and sum rounded separately (no FMA), so the result does not depend on which part
          // finished first
          l = __fadd_rn(__fmul_rn(l, f_own), __fmul_rn(l2, f_oth));
          m_used = mn;
          oth = reinterpret_cast<const float4*>(part);
        }
      }
      const float inv_l = l > 0.f ? (DROP ? p.inv_keep : 1.f) / l : 0.f;
      const float sc = exp2i(__ldg(p.ev + bhk));
      __nv_bfloat16* orow = p.out + (int64_t)b * p.osb + (int64_t)h * p.osh + (int64_t)min(qi, p.Sq - 1) * p.oss;
      __half* o16row = p.o16 ? p.o16 + ((int64_t)bh * p.Sq + min(qi, p.Sq - 1)) * D : nullptr;
      // 8 output values of dims 8 gg .. of chunk c, normalised here: bf16 times 2^ev, and the fp16 copy
      auto emit8 = [&](int c, int gg, float (&v)[8]) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] *= inv_l;
        *reinterpret_cast<uint4*>(orow + c * 32 + gg * 8) =
            make_uint4(pack_bf16(v[0] * sc, v[1] * sc), pack_bf16(v[2] * sc, v[3] * sc),
                       pack_bf16(v[4] * sc, v[5] * sc), pack_bf16(v[6] * sc, v[7] * sc));
        if (o16row)
          *reinterpret_cast<uint4*>(o16row + c * 32 + gg * 8) = make_uint4(
              pack_f16(v[0], v[1]), pack_f16(v[2], v[3]), pack_f16(v[4], v[5]), pack_f16(v[6], v[7]));
      };
      bool combined = false;
      if constexpr (SPLIT) {
        if (oth) {
          // the other part's O added chunk by chunk; its loads run two chunks ahead of this loop's stores
          // (a load cannot move past a store that may alias it, so loaded in place each group would be
          // one L2 round trip)
          constexpr int NC = D / 32;
          float4 pa[8], pb[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            pa[q] = __ldcg(oth + q * 32 + lane);
            pb[q] = __ldcg(oth + (8 + q) * 32 + lane);
          }
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            float4 cur[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              cur[q] = (c & 1) ? pb[q] : pa[q];
              if (c + 2 < NC) {
                if (c & 1) pb[q] = __ldcg(oth + ((c + 2) * 8 + q) * 32 + lane);
                else pa[q] = __ldcg(oth + ((c + 2) * 8 + q) * 32 + lane);
              }
            }
            uint32_t o[32];
            tmem_ld32(o_addr + c * 32, o);
            tmem_ld_wait();
            if (qi < p.Sq) {
#pragma unroll
              for (int gg = 0; gg < 4; ++gg) {
                const float w[8] = {cur[2 * gg].x,     cur[2 * gg].y,     cur[2 * gg].z,     cur[2 * gg].w,
                                    cur[2 * gg + 1].x, cur[2 * gg + 1].y, cur[2 * gg + 1].z, cur[2 * gg + 1].w};
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; ++e)
                  v[e] = __fadd_rn(__fmul_rn(__uint_as_float(o[8 * gg + e]), f_own), __fmul_rn(w[e], f_oth));
                emit8(c, gg, v);
              }
            }
          }
          combined = true;
        }
      }
      if (!combined) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(o_addr + c * 32, o);
          tmem_ld_wait();
          if (qi < p.Sq) {
#pragma unroll
            for (int gg = 0; gg < 4; ++gg) {
              float v[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(o[8 * gg + e]);
              emit8(c, gg, v);
            }
          }
        }
      }
      if (p.lse && qi < p.Sq) p.lse[(int64_t)bh * p.lse_ld + qi] = (m_used + log2f(l)) * 0.6931471805599453f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort) {  // let copies and MMAs already in flight land before the CTA's memory goes away
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 2000000ull) {
    }
  }
  cluster_sync();  // the even CTA's MMAs have finished reading the odd CTA's shared memory and TMEM
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// ---------------------------------------------------------------- key-split planning (host)
// Cost of a part in key-tile steps of a pair (~2 us each at S = 1-4k): its tiles, plus kItemSteps for the
// pipeline fill (~1.5 us) and the output write (~3.4 us) a part adds, plus kCombineSteps for the exchange
// through the workspace (put on the second part: ~3.6 us to write a part's O, ~1.5 us more to add it).
// Figures from a %globaltimer trace of the kernel; a split is taken when the estimate drops below
// kSplitGain of the plain schedule's (measured: estimates of 0.59 / 0.62 / 0.76 ran 0.71 / 0.89 / 0.90 of
// the plain time, 0.81 / 0.87 ran 1.07 / 1.02).
constexpr double kItemSteps = 2.5, kCombineSteps = 2.0, kSplitGain = 0.78;

struct SplitPlan {
  bool split = false;
  int pairs = 0;   // pairs in the grid
  int splits = 0;  // split items
  fwd256::Sched<true> sched;
};

struct SplitPart {
  double w;
  uint64_t e;
};

// Longest-processing-time list schedule of the parts on G pairs (parts sorted longest first, each to
// the least-loaded pair, ties to the lower pair); returns the largest load, and each pair's parts in
// order when `assign` is given.
double lpt_schedule(std::vector<SplitPart>& parts, int G, std::vector<std::vector<int>>* assign) {
  std::stable_sort(parts.begin(), parts.end(), [](const SplitPart& a, const SplitPart& b) { return a.w > b.w; });
  using Load = std::pair<double, int>;
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
  for (int c = 0; c < G; ++c) heap.push({0.0, c});
  double span = 0.0;
  for (size_t i = 0; i < parts.size(); ++i) {
    Load ld = heap.top();
    heap.pop();
    ld.first += parts[i].w + kItemSteps;
    span = std::max(span, ld.first);
    if (assign) (*assign)[ld.second].push_back((int)i);
    heap.push(ld);
  }
  return span;
}

uint64_t sched_entry(int64_t bh, int pr, int kb, int n, int sid) {
  return (uint64_t)bh | (uint64_t)pr << 16 | (uint64_t)kb << 30 | (uint64_t)n << 43 | (uint64_t)sid << 56;
}

// The parts of every item when those longer than `target` steps are cut in two (the first part as long
// as the target allows, the rest second); empty when the cut exceeds the schedule's limits.
std::vector<SplitPart> split_parts(int64_t BHq, int rpairs, int Sk, bool causal, double target, int* splits) {
  std::vector<SplitPart> parts;
  *splits = 0;
  for (int pr = 0; pr < rpairs; ++pr) {
    const int kv_end = causal ? std::min(Sk, (pr + 1) * 2 * fwd256::ROWS) : Sk;
    const int n = (kv_end + fwd256::KEYS - 1) / fwd256::KEYS;
    for (int64_t bh = 0; bh < BHq; ++bh) {
      if (target > 0 && n >= 2 && n + kItemSteps > target) {
        const int a = std::max(1, std::min(n - 1, (int)(target - kItemSteps - kCombineSteps)));
        const int sid = ++*splits;
        if (sid > fwd256::kSplitItems) return {};
        parts.push_back({(double)a, sched_entry(bh, pr, 0, a, sid)});
        parts.push_back({(double)(n - a) + kCombineSteps, sched_entry(bh, pr, a, n - a, sid)});
      } else {
        parts.push_back({(double)n, sched_entry(bh, pr, 0, n, 0)});
      }
      if ((int)parts.size() > fwd256::kSchedEntries) return {};
    }
  }
  return parts;
}

// Split plan for a head-dim-256 launch: cut items over their key tiles when the estimated schedule
// length drops below kSplitGain of the plain one (few items for the pairs: short sequences, few heads).
void plan_split(int64_t BHq, int Sq, int Sk, bool causal, int max_pairs, SplitPlan& plan) {
  plan = SplitPlan{};
  const int rpairs = (Sq + 2 * fwd256::ROWS - 1) / (2 * fwd256::ROWS);
  const int n_max = (Sk + fwd256::KEYS - 1) / fwd256::KEYS;
  if (BHq * rpairs > fwd256::kSchedEntries || n_max > 8191 || max_pairs > fwd256::kSchedPairs || max_pairs < 1) return;
  int splits = 0;
  std::vector<SplitPart> whole = split_parts(BHq, rpairs, Sk, causal, 0.0, &splits);
  double total = 0.0;
  for (const SplitPart& q : whole) total += q.w + kItemSteps;
  const double base = lpt_schedule(whole, (int)std::min<int64_t>((int64_t)whole.size(), max_pairs), nullptr);
  double best = base, best_target = 0.0;
  const int lo = std::max(2, (int)(total / max_pairs)), hi = n_max + 2;
  const int step = std::max(1, (hi - lo) / 48);
  for (int t = lo; t <= hi; t += step) {
    std::vector<SplitPart> parts = split_parts(BHq, rpairs, Sk, causal, (double)t, &splits);
    if (parts.empty() || splits == 0) continue;
    const double span = lpt_schedule(parts, (int)std::min<size_t>(parts.size(), (size_t)max_pairs), nullptr);
    if (span < best) {
      best = span;
      best_target = t;
    }
  }
  if (best_target == 0.0 || best > kSplitGain * base) return;
  std::vector<SplitPart> parts = split_parts(BHq, rpairs, Sk, causal, best_target, &splits);
  const int G = (int)std::min<size_t>(parts.size(), (size_t)max_pairs);
  std::vector<std::vector<int>> assign(G);
  lpt_schedule(parts, G, &assign);
  int k = 0;
  for (int c = 0; c < G; ++c) {
    plan.sched.start[c] = (uint16_t)k;
    for (int i : assign[c]) plan.sched.e[k++] = parts[i].e;
  }
  for (int c = G; c <= fwd256::kSchedPairs; ++c) plan.sched.start[c] = (uint16_t)k;
  plan.split = true;
  plan.pairs = G;
  plan.splits = splits;
}

// Plans by shape, computed once each (a handful of shapes per model).
std::shared_ptr<const SplitPlan> split_plan(int64_t BHq, int Sq, int Sk, bool causal, int max_pairs) {
  struct Entry {
    int64_t BHq;
    int Sq, Sk, causal, max_pairs;
    std::shared_ptr<const SplitPlan> plan;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  std::lock_guard<std::mutex> lock(mu);
  for (const Entry& e : cache)
    if (e.BHq == BHq && e.Sq == Sq && e.Sk == Sk && e.causal == (int)causal && e.max_pairs == max_pairs) return e.plan;
  auto plan = std::make_shared<SplitPlan>();
  plan_split(BHq, Sq, Sk, causal, max_pairs, *plan);
  if (cache.size() >= 64) cache.erase(cache.begin());
  cache.push_back({BHq, Sq, Sk, (int)causal, max_pairs, plan});
  return plan;
}

int64_t split_ws_bytes(const SplitPlan& plan) {
  return plan.split ? fwd256::kSplitHdrBytes + (int64_t)plan.splits * 8 * fwd256::kSlotFloats * 4 : 0;
}

// plan: a key-split schedule (prm.split_ws holds split_ws_bytes(*plan)), or null for the plain order.
template <bool DROP, bool SPLIT>
int launch_fwd_d256_pair(const void* q16, const void* k16, const void* v16, const AttnFwdParams& prm,
                         const SplitPlan* plan, cudaStream_t st) {
  const tbf16_host::DeviceInfo* dev = tbf16_host::device_info();
  if (!dev) return TBF16_ERR_DEVICE;
  CUtensorMap tq, tk, tv;
  const int64_t BHq = (int64_t)prm.B * prm.Hq, BHk = (int64_t)prm.B * prm.Hkv;
  if (int rc = tbf16_host::make_tmap_3d(&tq, q16, 256, prm.Sq, BHq, 256, (uint64_t)prm.Sq * 256, 64, fwd256::ROWS)) return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tk, k16, 256, prm.Sk, BHk, 256, (uint64_t)prm.Sk * 256, 64, fwd256::KEYS / 2))
    return rc;
  if (int rc = tbf16_host::make_tmap_3d(&tv, v16, 256, prm.Sk, BHk, 256, (uint64_t)prm.Sk * 256, 64, fwd256::KEYS))
    return rc;
  auto kern = attn_fwd_d256_pair_kernel<DROP, SPLIT>;
  static bool attr_done[64] = {false};
  if (!attr_done[dev->device & 63]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, fwd256::SMEM) != cudaSuccess)
      return tbf16_host::check_launch();
    attr_done[dev->device & 63] = true;
  }
  // one pair per two SMs (shared memory and the 512 TMEM columns allow no second CTA), never more than
  // the items
  const int64_t items = BHq * ((prm.Sq + 2 * fwd256::ROWS - 1) / (2 * fwd256::ROWS));
  if (items > INT32_MAX - dev->sms) return TBF16_ERR_INVALID;  // item indices are int
  const int64_t pairs = SPLIT ? plan->pairs : std::min<int64_t>(items, dev->sms / 2);
  fwd256::Sched<SPLIT> sched{};
  if constexpr (SPLIT) {
    sched = plan->sched;
    // tickets and flags start at zero every launch
    if (cudaMemsetAsync(prm.split_ws, 0, fwd256::kSplitHdrBytes, st) != cudaSuccess) return tbf16_host::check_launch();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(fwd256::THREADS);
  cfg.dynamicSmemBytes = fwd256::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, tq, tk, tv, prm, sched) != cudaSuccess) return tbf16_host::check_launch();
  return tbf16_host::check_launch();
}

}  // namespace

extern "C" int tbf16_attn_fwd(const void* q16, const void* k16, const void* v16, int64_t B, int64_t Hq, int64_t Hkv,
                              int64_t Sq, int64_t Sk, int64_t D, float scale, int causal, const int32_t* ev,
                              const void* mask, int64_t mask_sb, int64_t mask_sh, int64_t mask_sq, void* out, float* lse,
                              int64_t lse_ld, void* o16, void* stream) {
  return tbf16_attn_fwd_out(q16, k16, v16, B, Hq, Hkv, Sq, Sk, D, scale, causal, ev, mask, mask_sb, mask_sh, mask_sq, out,
                            Hq * Sq * D, Sq * D, D, lse, lse_ld, o16, stream);
}

// TBF16_ATTN_FWD=1 selects the one-tile kernels, =2 the two-tile / CTA-pair kernels whatever the shape
static bool attn_one_cta() {
  const char* e = getenv("TBF16_ATTN_FWD");
  return e && e[0] == '1';
}
static bool attn_multi_tile() {
  const char* e = getenv("TBF16_ATTN_FWD");
  return e && e[0] == '2';
}

static int attn_fwd_impl(const void* q16, const void* k16, const void* v16, int64_t B, int64_t Hq, int64_t Hkv,
                         int64_t Sq, int64_t Sk, int64_t D, float scale, int causal, const int32_t* ev,
                         const void* mask, int64_t mask_sb, int64_t mask_sh, int64_t mask_sq, void* out, int64_t out_sb,
                         int64_t out_sh, int64_t out_ss, float* lse, int64_t lse_ld, void* o16, float dropout_p,
                         uint64_t seed, void* ws, int64_t ws_bytes, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  uint32_t thr = 0;
  float inv_keep = 1.f;
  if (!tbf16_host::dropout_params(dropout_p, &thr, &inv_keep)) return TBF16_ERR_INVALID;
  const bool drop = thr > 0;
  if (B < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Sq < 0 || Sk < 0 || !ev || !out || B * Hq > 65535 ||
      Sq > INT32_MAX || Sk > INT32_MAX)
    return TBF16_ERR_INVALID;
  if (D != 64 && D != 128 && D != 256) return TBF16_ERR_UNSUPPORTED;
  if (!tbf16_host::aligned16(q16) || !tbf16_host::aligned16(k16) || !tbf16_host::aligned16(v16) ||
      !tbf16_host::aligned16(out) || !tbf16_host::aligned16(o16))
    return TBF16_ERR_ALIGN;
  if (out_sb < 0 || out_sh < 0 || out_ss < 0 || out_sb % 8 || out_sh % 8 || out_ss % 8) return TBF16_ERR_ALIGN;
  if (B == 0 || Sq == 0) return TBF16_OK;
  const tbf16_host::DeviceInfo* dev = tbf16_host::device_info();
  AttnFwdParams prm;
  prm.B = (int)B; prm.Hq = (int)Hq; prm.Hkv = (int)Hkv; prm.Sq = (int)Sq; prm.Sk = (int)Sk;
  prm.group = (int)(Hq / Hkv);
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.causal = causal;
  prm.ev = ev;
  prm.out = static_cast<__nv_bfloat16*>(out);
  prm.osb = out_sb;
  prm.osh = out_sh;
  prm.oss = out_ss;
  prm.lse = lse;
  prm.lse_ld = lse_ld;
  if (lse && lse_ld < Sq) return TBF16_ERR_INVALID;
  prm.o16 = static_cast<__half*>(o16);
  prm.split_ws = nullptr;
  prm.mask = static_cast<const uint16_t*>(mask);
  prm.mb = mask_sb; prm.mh = mask_sh; prm.mi = mask_sq;
  prm.err = dev->err;
  prm.m_tiles = (int)((Sq + BM - 1) / BM);
  prm.drop_thr = thr;
  prm.seed_lo = (uint32_t)seed;
  prm.seed_hi = (uint32_t)(seed >> 32);
  prm.inv_keep = inv_keep;
  if (Sk == 0) return TBF16_ERR_UNSUPPORTED;
  auto st = static_cast<cudaStream_t>(stream);
  // D <= 128: the persistent two-query-tile kernel, D = 256: the CTA-pair kernel (P in TMEM in both);
  // TBF16_ATTN_FWD=1 selects the one-tile kernel
  static const bool one_cta = attn_one_cta();
  // D <= 128 with no more two-tile items (256 query rows) than SMs: the two-tile kernel would leave SMs
  // idle, and the one-tile kernel's twice as many CTAs win (graph-timed, causal, D = 128, 2048 tokens:
  // 64 items 31.6 against 46.3 us, 96 items 33.1 against 48.4, 128 items 36.3 against 48.0; from 192
  // items, 1.3 waves, the two-tile kernel is faster: 49.4 against 57.4)
  static const bool multi = attn_multi_tile();
  const bool one = one_cta || (!multi && D <= 128 && (int64_t)B * Hq * ((Sq + 2 * BM - 1) / (2 * BM)) <= dev->sms);
  if (D == 256 && !one_cta && ws && ws_bytes > 0 && tbf16_host::aligned16(ws)) {
    // a key-split schedule when the caller's workspace holds it (tbf16_attn_fwd_ws_size)
    std::shared_ptr<const SplitPlan> plan = split_plan(B * Hq, (int)Sq, (int)Sk, causal != 0, dev->sms / 2);
    if (plan->split && ws_bytes >= split_ws_bytes(*plan)) {
      prm.split_ws = ws;
      return drop ? launch_fwd_d256_pair<true, true>(q16, k16, v16, prm, plan.get(), st)
                  : launch_fwd_d256_pair<false, true>(q16, k16, v16, prm, plan.get(), st);
    }
  }
  if (drop) {
    if (D == 64) return one ? launch_fwd<64, true>(q16, k16, v16, prm, st) : launch_fwd_pp<64, true>(q16, k16, v16, prm, st);
    if (D == 128)
      return one ? launch_fwd<128, true>(q16, k16, v16, prm, st) : launch_fwd_pp<128, true>(q16, k16, v16, prm, st);
    return one_cta ? launch_fwd<256, true>(q16, k16, v16, prm, st)
                   : launch_fwd_d256_pair<true, false>(q16, k16, v16, prm, nullptr, st);
  }
  if (D == 64) return one ? launch_fwd<64, false>(q16, k16, v16, prm, st) : launch_fwd_pp<64, false>(q16, k16, v16, prm, st);
  if (D == 128)
    return one ? launch_fwd<128, false>(q16, k16, v16, prm, st) : launch_fwd_pp<128, false>(q16, k16, v16, prm, st);
  return one_cta ? launch_fwd<256, false>(q16, k16, v16, prm, st)
                 : launch_fwd_d256_pair<false, false>(q16, k16, v16, prm, nullptr, st);
}

// Head-dim-256 forwards with few items for the pairs run a key-split schedule in a caller's workspace.
extern "C" int64_t tbf16_attn_fwd_ws_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D,
                                          int causal) {
  if (D != 256 || B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Sq <= 0 || Sk <= 0 || B * Hq > 65535 ||
      Sq > INT32_MAX || Sk > INT32_MAX || attn_one_cta())
    return 0;
  const tbf16_host::DeviceInfo* dev = tbf16_host::device_info();
  if (!dev) return 0;
  return split_ws_bytes(*split_plan(B * Hq, (int)Sq, (int)Sk, causal != 0, dev->sms / 2));
}

extern "C" int tbf16_attn_fwd_ws(const void* q16, const void* k16, const void* v16, int64_t B, int64_t Hq, int64_t Hkv,
                                 int64_t Sq, int64_t Sk, int64_t D, float scale, int causal, const int32_t* ev,
                                 const void* mask, int64_t mask_sb, int64_t mask_sh, int64_t mask_sq, void* out,
                                 int64_t out_sb, int64_t out_sh, int64_t out_ss, float* lse, int64_t lse_ld, void* o16,
                                 float dropout_p, uint64_t seed, void* ws, int64_t ws_bytes, void* stream) {
  return attn_fwd_impl(q16, k16, v16, B, Hq, Hkv, Sq, Sk, D, scale, causal, ev, mask, mask_sb, mask_sh, mask_sq, out,
                       out_sb, out_sh, out_ss, lse, lse_ld, o16, dropout_p, seed, ws, ws_bytes, stream);
}

extern "C" int tbf16_attn_fwd_out(const void* q16, const void* k16, const void* v16, int64_t B, int64_t Hq,
                                  int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, float scale, int causal,
                                  const int32_t* ev, const void* mask, int64_t mask_sb, int64_t mask_sh,
                                  int64_t mask_sq, void* out, int64_t out_sb, int64_t out_sh, int64_t out_ss,
                                  float* lse, int64_t lse_ld, void* o16, void* stream) {
  return attn_fwd_impl(q16, k16, v16, B, Hq, Hkv, Sq, Sk, D, scale, causal, ev, mask, mask_sb, mask_sh, mask_sq, out,
                       out_sb, out_sh, out_ss, lse, lse_ld, o16, 0.f, 0, nullptr, 0, stream);
}

extern "C" int tbf16_attn_fwd_dropout(const void* q16, const void* k16, const void* v16, int64_t B, int64_t Hq,
                                      int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, float scale, int causal,
                                      const int32_t* ev, const void* mask, int64_t mask_sb, int64_t mask_sh,
                                      int64_t mask_sq, void* out, int64_t out_sb, int64_t out_sh, int64_t out_ss,
                                      float* lse, int64_t lse_ld, void* o16, float dropout_p, uint64_t seed,
                                      void* stream) {
  return attn_fwd_impl(q16, k16, v16, B, Hq, Hkv, Sq, Sk, D, scale, causal, ev, mask, mask_sb, mask_sh, mask_sq, out,
                       out_sb, out_sh, out_ss, lse, lse_ld, o16, dropout_p, seed, nullptr, 0, stream);
}

namespace {
__global__ void dropout_keep_kernel(uint8_t* __restrict__ keep, int64_t BH, int64_t Sq, int64_t Sk, uint32_t thr,
                                    uint32_t seed_lo, uint32_t seed_hi) {
  const int64_t n = BH * Sq * Sk;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = idx / Sk;
    const uint32_t j = (uint32_t)(idx % Sk);
    const uint32_t rk = drop_row_key(seed_lo, seed_hi, (uint32_t)(row / Sq), (uint32_t)(row % Sq));
    keep[idx] = drop_keep(rk, j, thr) ? 1 : 0;
  }
}
}  // namespace

extern "C" int tbf16_attn_dropout_keep(uint8_t* keep, int64_t BH, int64_t Sq, int64_t Sk, float dropout_p,
                                       uint64_t seed, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  uint32_t thr = 0;
  float inv_keep = 1.f;
  if (!keep || BH < 0 || Sq < 0 || Sk < 0 || !tbf16_host::dropout_params(dropout_p, &thr, &inv_keep))
    return TBF16_ERR_INVALID;
  const int64_t n = BH * Sq * Sk;
  if (n == 0) return TBF16_OK;
  const tbf16_host::DeviceInfo* dev = tbf16_host::device_info();
  const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)dev->sms * 32);
  dropout_keep_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(keep, BH, Sq, Sk, thr, (uint32_t)seed,
                                                                           (uint32_t)(seed >> 32));
  return tbf16_host::check_launch();
}
