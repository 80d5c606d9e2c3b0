// Scaled bf16-on-fp16 GEMM for sm_100a: TMA -> (converter warps) -> tcgen05.mma (fp32 in TMEM) ->
// epilogue warps -> bf16.
//
//   y[m, n] = bf16_rn((sum_k A16[m,k] * B16[n,k]) * sa[m] * sb[n] + bias[n])
//
// A16 is either an fp16 operand in memory (K-major or MN-major) or, in the fused linear, the bf16
// activation x converted in shared memory to fp16(x[m,k] / sa[m]) by converter warps (exact for
// values inside fp16's range: sa is a power of two). B16 is fp16 (K-major or MN-major).
//
// One CTA per SM, persistent over 128 x BN output tiles (grouped raster for L2 reuse):
//   warp 0      TMA producer: one elected lane streams 128x64 A and BNx64 B tiles (128-byte swizzle)
//               into a STAGES-deep ring guarded by full/empty mbarriers.
//   warp 1      MMA issuer: allocates 2*BN TMEM columns (two fp32 accumulators), one lane issues
//               tcgen05.mma.kind::f16 (M=128, N=BN, K=16) x 4 per stage and commits to the stage's
//               empty barrier, and to the accumulator's full barrier after the last k-block.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time, apply the scales and bias, store bf16;
//               the other accumulator is being filled meanwhile.
//   warps 6-9   converters (fused linear only): bf16 -> fp16 with the row's power-of-two scale,
//               in place in the A stage, then fence.proxy.async and arrive on the stage's conv barrier.
// Every mbarrier wait is bounded (2 s); on timeout the kernel records it in the device error word,
// every role leaves its loop, and the CTA drains and frees its TMEM before returning.
//
// The CTA-pair kernel (scaled_gemm_pair_kernel, further down) is the one large products use: clusters
// of two CTAs compute 256 x PN tiles with tcgen05.mma.cta_group::2 (PN = 256, or 192 / 160 / 128 when
// the last wave of 256-wide tiles would leave most pairs idle), and its CONV form reads A as an implicit
// convolution through a 5-D tensor map. Inside tbf16_linear both kernels launch as programmatic
// dependents of the call's own row pass (first weight tiles before griddepcontrol.wait, A after).
#include <algorithm>

#include "common.cuh"

using namespace tbf16;

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // one 128-byte swizzle atom of 16-bit elements
constexpr int kEpiWarps = 4;
constexpr int kConvWarps = 4;
constexpr int kGroupM = 16;  // M tiles per raster group (TBF16_GEMM_GROUP overrides, for tuning)

struct GemmParams {
  int M, N, K;
  const float* sa;            // [M]
  const float* sb;            // [N] or null
  const __nv_bfloat16* bias;  // [N] or null
  __nv_bfloat16* y;
  int64_t ldy;
  unsigned int* err;
  int tiles_m, tiles_n;
  int group_m;    // M tiles per raster group
  int tma_store;  // pair kernel: epilogue through shared memory and TMA stores (else direct 16-byte stores)
  ConvGemm cv;    // pair kernel, implicit convolution only
};

template <int BN, int STAGES, bool CONVERT>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int WARPS = 2 + kEpiWarps + (CONVERT ? kConvWarps : 0);
  static constexpr int THREADS = 32 * WARPS;
  static constexpr int TMEM_COLS = 2 * BN;  // power of two >= 32
  static constexpr int BAR_BYTES = 8 * (3 * STAGES + 4) + 16;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
  static_assert(TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM columns");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// Grouped raster: group_m M tiles x all N tiles per group, M fastest, so the CTAs in flight share a few
// A panels and B panels in L2.
__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int group_m, int& tm, int& tn) {
  const int per_group = group_m * tiles_n;
  const int group = tile / per_group;
  const int first = group * group_m;
  const int gsize = min(tiles_m - first, group_m);
  const int r = tile % per_group;
  tm = first + r % gsize;
  tn = r / gsize;
}

template <int BN, int STAGES, bool CONVERT, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(Cfg<BN, STAGES, CONVERT>::THREADS, 1)
    scaled_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const GemmParams p) {
  using C = Cfg<BN, STAGES, CONVERT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* conv = full + STAGES;
  uint64_t* empty = conv + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.tiles_m * p.tiles_n;
  const int KB = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], kConvWarps);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);
    }
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // A programmatic dependent of the kernel that writes A's row scales (and, for fp16 A, A itself):
    // the first stages' weight tiles load before griddepcontrol.wait, A only after.
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool first = true;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort; tile += gridDim.x) {
        int tm, tn;
        tile_coords(tile, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
        const int m0 = tm * BM, n0 = tn * BN;
        auto load_a = [&](uint8_t* sA, uint64_t* bar, int kb) {
          if (!A_MN) {
            tma_load_2d(sA, &tmA, bar, kb * BK, m0);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(sA + j * 64 * BK * 2, &tmA, bar, m0 + j * 64, kb * BK);
          }
        };
        auto load_b = [&](uint8_t* sB, uint64_t* bar, int kb) {
          if (!B_MN) {
            tma_load_2d(sB, &tmB, bar, kb * BK, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sB + j * 64 * BK * 2, &tmB, bar, n0 + j * 64, kb * BK);
          }
        };
        int kb0 = 0;
        if (first) {  // every stage is free: weight tiles first, then (after the wait) the A tiles
          first = false;
          const int pre = KB < STAGES ? KB : STAGES;
          for (int kb = 0; kb < pre; ++kb) {
            mbar_arrive_expect_tx(&full[kb], C::STAGE_BYTES);
            load_b(smem + kb * C::STAGE_BYTES + C::A_BYTES, &full[kb], kb);
          }
          pdl_wait();
          for (int kb = 0; kb < pre; ++kb) load_a(smem + kb * C::STAGE_BYTES, &full[kb], kb);
          stage = pre == STAGES ? 0 : pre;
          phase = pre == STAGES ? 1u : 0u;
          kb0 = pre;
        }
        for (int kb = kb0; kb < KB; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort, p.err)) break;
          uint8_t* sA = smem + stage * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          load_a(sA, &full[stage], kb);
          load_b(sA + C::A_BYTES, &full[stage], kb);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(CONVERT ? &conv[stage] : &full[stage], phase, abort, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // K-major: advance 32 bytes inside the swizzle atom; MN-major: two 8-row K groups (2 KB).
            const uint64_t ad = A_MN ? smem_desc_sw128(a_addr + k * 2048, 64 * BK * 2, 1024)
                                     : smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc_sw128(b_addr + k * 2048, 64 * BK * 2, 1024)
                                     : smem_desc_sw128(b_addr + k * 32, 16, 1024);
            umma_f16_ss(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  } else if (warp < 2 + kEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;
    // sa may be written by the grid this one was launched early behind: wait for it here too rather
    // than rely on the producer's wait being ordered before these loads (a no-op for plain launches).
    pdl_wait();
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort, p.err)) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(tile, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
      const int m = tm * BM + row;
      const bool mok = m < p.M;
      const float a = mok ? __ldg(p.sa + m) : 0.f;
      __nv_bfloat16* yrow = p.y + (int64_t)(mok ? m : 0) * p.ldy;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + acc * BN + c * 32 + ((uint32_t)(quad * 32) << 16), r);
        tmem_ld_wait();
        const int n0 = tn * BN + c * 32;
        if (mok && n0 < p.N) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int n = n0 + 8 * j;
            if (n < p.N) {
              float v[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float sbv = p.sb ? __ldg(p.sb + n + e) : 1.f;
                v[e] = (__uint_as_float(r[8 * j + e]) * a) * sbv;
                if (p.bias) v[e] += __bfloat162float(p.bias[n + e]);
              }
              uint4 o;
              o.x = pack_bf16(v[0], v[1]);
              o.y = pack_bf16(v[2], v[3]);
              o.z = pack_bf16(v[4], v[5]);
              o.w = pack_bf16(v[6], v[7]);
              *reinterpret_cast<uint4*>(yrow + n) = o;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  } else if (CONVERT) {
    // ------------------------------------------------------------ converters: bf16 -> fp16(x * s) in place
    const int row = (warp - 2 - kEpiWarps) * 32 + lane;  // 0..127, one row of the A tile per thread
    pdl_wait();  // sa comes from the row pass (a no-op for plain launches)
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int tm, tn;
      tile_coords(tile, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
      const int m = tm * BM + row;
      const float s = m < p.M ? 1.0f / __ldg(p.sa + m) : 0.f;  // exact: sa is a power of two
      bool ok = true;
      for (int kb = 0; kb < KB; ++kb) {
        if (!mbar_wait_warp(&full[stage], phase, abort, p.err)) { ok = false; break; }
        uint8_t* rowp = smem + stage * C::STAGE_BYTES + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          // Rotate the chunk order by row so the 8 threads of a quarter-warp hit distinct banks.
          uint4* q = reinterpret_cast<uint4*>(rowp + ((c + row) & 7) * 16);
          const uint4 v = *q;
          uint4 o;
          o.x = pack_f16(bf16lo(v.x) * s, bf16hi(v.x) * s);
          o.y = pack_f16(bf16lo(v.y) * s, bf16hi(v.y) * s);
          o.z = pack_f16(bf16lo(v.z) * s, bf16hi(v.z) * s);
          o.w = pack_f16(bf16lo(v.w) * s, bf16hi(v.w) * s);
          *q = o;
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (*abort) {  // let copies and MMAs already in flight land before the CTA's memory goes away
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 2000000ull) {
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <int BN, int STAGES, bool CONVERT, bool A_MN, bool B_MN>
int launch_gemm(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, const float* sa,
                const float* sb, const void* bias, void* y, int64_t ldy, cudaStream_t st, bool pdl = false) {
  using C = Cfg<BN, STAGES, CONVERT>;
  const tbf16_host::DeviceInfo* d = tbf16_host::device_info();
  if (!d) return TBF16_ERR_DEVICE;
  CUtensorMap ta, tb;
  int rc = A_MN ? tbf16_host::make_tmap_2d(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, 64, 64)
                : tbf16_host::make_tmap_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, 64, BM);
  if (rc) return rc;
  rc = B_MN ? tbf16_host::make_tmap_2d(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, 64)
            : tbf16_host::make_tmap_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, 64, BN);
  if (rc) return rc;
  auto kern = scaled_gemm_kernel<BN, STAGES, CONVERT, A_MN, B_MN>;
  static bool attr_done[64] = {false};
  if (!attr_done[d->device & 63]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
      return tbf16_host::check_launch();
    attr_done[d->device & 63] = true;
  }
  GemmParams p;
  p.M = M; p.N = N; p.K = K;
  p.sa = sa; p.sb = sb;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.ldy = ldy;
  p.err = d->err;
  p.tiles_m = (M + BM - 1) / BM;
  static const int group_env = [] {
    const char* e = getenv("TBF16_GEMM_GROUP");
    return e ? atoi(e) : 0;
  }();
  p.group_m = group_env > 0 ? group_env : kGroupM;
  p.tiles_n = (N + BN - 1) / BN;
  const int tiles = p.tiles_m * p.tiles_n;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(tiles, d->sms));
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  // pdl: the kernel before it is this call's own row pass, which writes only A's operand and row scales,
  // so the GEMM may start early and load its first weight tiles before griddepcontrol.wait (see the
  // producer). Any other predecessor may write the weights (prepare_weight's pass does), so other
  // launches are plain: the wait is then a no-op and every load follows the predecessor's completion.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, kern, ta, tb, p) != cudaSuccess) return tbf16_host::check_launch();
  return tbf16_host::check_launch();
}

// ------------------------------------------------------------------------------------------------
// CTA-pair GEMM (fp16 operands): a cluster of two CTAs on two SMs computes a 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256: each CTA holds 128 rows of A and of the accumulator; N = 256:
// each CTA holds half of the B tile). Per SM and k16 step the tensor core reads 8 KB of shared memory
// instead of 12 KB, and each SM loads 32 KB per 64-wide K block instead of 48 KB. The even CTA's
// thread issues the MMAs; both CTAs' TMA loads count their bytes on the even CTA's full barrier; the
// MMA completion is multicast to both CTAs' empty / accumulator-full barriers; both CTAs' epilogue
// warps release an accumulator on the even CTA's barrier. No multicast loads.
constexpr int kPairStages = 6;
// PN: the pair tile's width (256 x PN outputs; 256 for the headline shapes, 192 / 160 / 128 for products
// whose last wave of 256-wide tiles would leave most pairs idle, 320 for products that fit one wave of
// 320-wide tiles but not of 256-wide ones, e.g. 2048 x 2560: 64 tiles on 74 pairs instead of 80).
// PN = 320 (WIDE) issues two N = 160 MMAs per k16 step into one 320-column accumulator: TMEM holds only
// one, so the next tile's MMAs wait for the epilogue -- it is chosen only when no pair gets a second tile.
template <int PN>
struct PairCfg {
  static_assert((PN % 32 == 0 && PN >= 128 && PN <= 256) || PN == 320, "pair tile width");
  static constexpr bool WIDE = PN > 256;
  static constexpr int NACC = WIDE ? 1 : 2;            // PN-column accumulators in TMEM
  static constexpr int STAGES = WIDE ? 5 : kPairStages;
  static constexpr int A_BYTES = BM * BK * 2;          // this CTA's 128 rows
  static constexpr int B_BYTES = (PN / 2) * BK * 2;    // this CTA's half of the PN B rows
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int THREADS = 32 * (2 + kEpiWarps);
  static constexpr int TMEM_COLS = 512;
  static constexpr int EPI_BYTES = kEpiWarps * 2 * 32 * 64;  // per epilogue warp two 32 x 32 bf16 tiles
  static constexpr int BAR_BYTES = 8 * (2 * STAGES + 4) + 16;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(NACC * PN <= TMEM_COLS, "TMEM");
};

template <bool A_MN, bool B_MN, bool CONV, int PN>
__global__ void __launch_bounds__(PairCfg<PN>::THREADS, 1)
    scaled_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            const __grid_constant__ CUtensorMap tmY, const GemmParams p) {
  using C = PairCfg<PN>;
  static_assert(PN == 256 || (!B_MN && !CONV), "narrow and wide pair tiles take K-major B only");
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * C::STAGE_BYTES + C::EPI_BYTES);  // even CTA's are used
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;                                             // even CTA's are used
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cid = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int num_tiles = p.tiles_m * p.tiles_n;  // in 256 x 256 pair tiles
  const int KB = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);
    }
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    // Launched as a programmatic dependent of the kernel that writes A and its row scales (the row pass
    // or a fused producer): the first stages' weight tiles load before griddepcontrol.wait, A only after.
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool first = true;
      for (int tile = cid; tile < num_tiles && !*abort; tile += nclusters) {
        int tm, tn;
        tile_coords(tile, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
        const int m0 = tm * 256 + (int)rank * 128, n0 = tn * PN + (int)rank * (PN / 2);
        int cx = 0, cy = 0, cz = 0, cbat = 0;  // CONV: input coordinates of the A box at tap (0, 0, 0)
        if (CONV) {
          int r = m0;
          const int xo = r % p.cv.Wo;
          r /= p.cv.Wo;
          const int yo = r % p.cv.Ho;
          r /= p.cv.Ho;
          const int zo = r % p.cv.Do;
          cbat = r / p.cv.Do;  // past the last sample for the second half of a ragged last pair: zero fill
          cx = xo - p.cv.pw;
          cy = yo - p.cv.ph;
          cz = zo - p.cv.pd;
        }
        int cblk = 0, kx = 0, ky = 0, kz = 0;  // CONV: K block kb = ((kz kh + ky) kw + kx) cb + cblk
        auto load_a = [&](uint8_t* sA, uint64_t* bar, int kb) {  // K blocks in order (CONV steps its counters)
          if (CONV) {
            tma_load_5d_pair(sA, &tmA, bar, cblk * BK, cx + kx * p.cv.dw, cy + ky * p.cv.dh, cz + kz * p.cv.dd, cbat);
            if (++cblk == p.cv.cb) {
              cblk = 0;
              if (++kx == p.cv.kw) {
                kx = 0;
                if (++ky == p.cv.kh) {
                  ky = 0;
                  ++kz;
                }
              }
            }
          } else if (!A_MN) {
            tma_load_2d_pair(sA, &tmA, bar, kb * BK, m0);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d_pair(sA + j * 64 * BK * 2, &tmA, bar, m0 + j * 64, kb * BK);
          }
        };
        auto load_b = [&](uint8_t* sB, uint64_t* bar, int kb) {
          if (C::WIDE) {
            // two boxes of PN / 4 rows: tile columns [PN/4 rank, +PN/4) and [PN/2 + PN/4 rank, +PN/4), so
            // that the first N = PN/2 MMA (PN/4 rows from each CTA) writes tile columns [0, PN/2) and the
            // second [PN/2, PN) in order
            tma_load_2d_pair(sB, &tmB, bar, kb * BK, tn * PN + (int)rank * (PN / 4));
            tma_load_2d_pair(sB + (PN / 4) * BK * 2, &tmB, bar, kb * BK, tn * PN + PN / 2 + (int)rank * (PN / 4));
          } else if (!B_MN) {
            tma_load_2d_pair(sB, &tmB, bar, kb * BK, n0);
          } else {
#pragma unroll
            for (int j = 0; j < 2; ++j) tma_load_2d_pair(sB + j * 64 * BK * 2, &tmB, bar, n0 + j * 64, kb * BK);
          }
        };
        int kb0 = 0;
        if (first) {  // every stage is free: weight tiles first, then (after the wait) the A tiles
          first = false;
          const int pre = KB < S ? KB : S;
          for (int kb = 0; kb < pre; ++kb) {
            if (leader) mbar_arrive_expect_tx(&full[kb], 2 * C::STAGE_BYTES);  // both CTAs' bytes
            load_b(smem + kb * C::STAGE_BYTES + C::A_BYTES, &full[kb], kb);
          }
          pdl_wait();
          for (int kb = 0; kb < pre; ++kb) load_a(smem + kb * C::STAGE_BYTES, &full[kb], kb);
          stage = pre == S ? 0 : pre;
          phase = pre == S ? 1u : 0u;
          kb0 = pre;
        }
        for (int kb = kb0; kb < KB; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort, p.err)) break;
          uint8_t* sA = smem + stage * C::STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);  // both CTAs' bytes
          load_a(sA, &full[stage], kb);
          load_b(sA + C::A_BYTES, &full[stage], kb);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(256, C::WIDE ? PN / 2 : PN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = cid; tile < num_tiles && !*abort; tile += nclusters) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort, p.err)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * PN;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? smem_desc_sw128(a_addr + k * 2048, 64 * BK * 2, 1024)
                                     : smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc_sw128(b_addr + k * 2048, 64 * BK * 2, 1024)
                                     : smem_desc_sw128(b_addr + k * 32, 16, 1024);
            umma_f16_ss_pair(d_tmem, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
            if constexpr (C::WIDE)
              umma_f16_ss_pair(d_tmem + PN / 2, ad, smem_desc_sw128(b_addr + (PN / 4) * BK * 2 + k * 32, 16, 1024),
                               idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == S) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 0x3);
        if (++acc == C::NACC) { acc = 0; acc_phase ^= 1; }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs, own 128 rows)
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    // TMA-store path: each warp converts 32 columns of its 32 rows into one of two 2 KB shared tiles
    // (64-byte swizzle, conflict-free 16-byte writes) and one lane stores the tile with TMA; the buffer
    // is rewritten only after the store issued from it two chunks earlier has read it.
    uint8_t* ebuf = smem + S * C::STAGE_BYTES + (warp - 2) * 2 * 2048;
    pdl_wait();  // sa (and the conv's sample scales) come from the pass this GEMM may launch behind
    int eb = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = cid; tile < num_tiles; tile += nclusters) {
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort, p.err)) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(tile, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
      const int m = tm * 256 + (int)rank * 128 + row;
      const bool mok = m < p.M;
      const float a = mok ? __ldg(p.sa + (CONV ? m / p.cv.sa_div : m)) : 0.f;
      if (p.tma_store) {
        const int row0 = tm * 256 + (int)rank * 128 + quad * 32;
#pragma unroll 1
        for (int c = 0; c < PN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem_base + acc * PN + c * 32 + ((uint32_t)(quad * 32) << 16), r);
          tmem_ld_wait();
          const int n0 = tn * PN + c * 32;
          if (n0 >= p.N) break;  // the rest of this tile lies past the last column
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
          uint8_t* buf = ebuf + eb * 2048;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int n = n0 + 8 * j;
            uint4 o = make_uint4(0, 0, 0, 0);
            if (n < p.N) {  // N is a multiple of 8: the 8 columns are all inside or all outside
              float v[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float sbv = p.sb ? __ldg(p.sb + n + e) : 1.f;
                v[e] = (__uint_as_float(r[8 * j + e]) * a) * sbv;
                if (p.bias) v[e] += __bfloat162float(p.bias[n + e]);
              }
              o.x = pack_bf16(v[0], v[1]);
              o.y = pack_bf16(v[2], v[3]);
              o.z = pack_bf16(v[4], v[5]);
              o.w = pack_bf16(v[6], v[7]);
            }
            *reinterpret_cast<uint4*>(buf + lane * 64 + ((j ^ ((lane >> 1) & 3)) * 16)) = o;
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmY, buf, n0, row0);
            bulk_commit_group();
          }
          eb ^= 1;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(&tempty[acc], 0);
        if (++acc == C::NACC) { acc = 0; acc_phase ^= 1; }
        continue;
      }
      __nv_bfloat16* yrow = p.y + (int64_t)(mok ? m : 0) * p.ldy;
#pragma unroll 1
      for (int c = 0; c < PN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + acc * PN + c * 32 + ((uint32_t)(quad * 32) << 16), r);
        tmem_ld_wait();
        const int n0 = tn * PN + c * 32;
        if (mok && n0 < p.N) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int n = n0 + 8 * j;
            if (n < p.N) {
              float v[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float sbv = p.sb ? __ldg(p.sb + n + e) : 1.f;
                v[e] = (__uint_as_float(r[8 * j + e]) * a) * sbv;
                if (p.bias) v[e] += __bfloat162float(p.bias[n + e]);
              }
              uint4 o;
              o.x = pack_bf16(v[0], v[1]);
              o.y = pack_bf16(v[2], v[3]);
              o.z = pack_bf16(v[4], v[5]);
              o.w = pack_bf16(v[6], v[7]);
              *reinterpret_cast<uint4*>(yrow + n) = o;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(&tempty[acc], 0);  // the even CTA's MMA may reuse the accumulator
      if (++acc == C::NACC) { acc = 0; acc_phase ^= 1; }
    }
  }

  if (warp >= 2 && lane == 0) bulk_wait_group<0>();  // the epilogue's TMA stores have completed
  tc_fence_before();
  __syncthreads();
  if (*abort) {  // let copies and MMAs already in flight land before the CTA's memory goes away
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 2000000ull) {
    }
  }
  cluster_sync();  // the even CTA's MMAs have finished reading the odd CTA's shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

// The pair kernel with A's tensor map already built (a matrix, or the conv input for CONV).
template <bool A_MN, bool B_MN, bool CONV, int PN>
int launch_pair_core(const CUtensorMap& ta, const void* B, int64_t ldb, int M, int N, int K, const float* sa,
                     const float* sb, const void* bias, void* y, int64_t ldy, const ConvGemm* cv, cudaStream_t st,
                     bool pdl) {
  using C = PairCfg<PN>;
  const tbf16_host::DeviceInfo* d = tbf16_host::device_info();
  if (!d) return TBF16_ERR_DEVICE;
  CUtensorMap tb;
  int rc = B_MN ? tbf16_host::make_tmap_2d(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, 64)
                : tbf16_host::make_tmap_2d(&tb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, 64, C::WIDE ? PN / 4 : PN / 2);
  if (rc) return rc;
  CUtensorMap ty;
  rc = tbf16_host::make_tmap_2d_out(&ty, y, (uint64_t)N, (uint64_t)M, (uint64_t)ldy, 32, 32);
  if (rc) return rc;
  auto kern = scaled_gemm_pair_kernel<A_MN, B_MN, CONV, PN>;
  static bool attr_done[64] = {false};
  if (!attr_done[d->device & 63]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
      return tbf16_host::check_launch();
    attr_done[d->device & 63] = true;
  }
  GemmParams p;
  p.M = M; p.N = N; p.K = K;
  p.sa = sa; p.sb = sb;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.ldy = ldy;
  p.err = d->err;
  p.tiles_m = (M + 255) / 256;
  p.tiles_n = (N + PN - 1) / PN;
  static const int group_env = [] {
    const char* e = getenv("TBF16_GEMM_GROUP");
    return e ? atoi(e) : 0;
  }();
  p.group_m = group_env > 0 ? group_env : kGroupM / 2;
  static const int epi_env = [] {  // TBF16_GEMM_EPI=0 selects the direct-store epilogue (for comparison)
    const char* e = getenv("TBF16_GEMM_EPI");
    return e ? atoi(e) : 1;
  }();
  p.tma_store = epi_env != 0 && tbf16_host::aligned16(y) ? 1 : 0;
  if (cv) p.cv = *cv;
  const int tiles = p.tiles_m * p.tiles_n;
  const int clusters = std::min(tiles, d->sms / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // pdl: may start while the kernel before it runs -- only when that kernel is known to write just A and
  // its row scales (this call's own row pass, the conv's scale pass): the producer loads the first
  // weight tiles before griddepcontrol.wait. Other launches are plain (see launch_gemm).
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, kern, ta, tb, ty, p) != cudaSuccess) return tbf16_host::check_launch();
  return tbf16_host::check_launch();
}

// Pair tile width for a product with K-major B: the one with the least work per SM counted as waves of
// tiles x (tile width + a fixed 32-column share for its prologue / epilogue). Measured (linear_q, CUDA
// graph): 600 x 1000 x 1024 16.7 -> 13.1 us at 128; 2048 x 2560 x 2048 33.1 -> 31.4 us and x 10240
// 109.7 -> 107.5 us at 160 -- far less than the waves suggest, because a narrow tile moves more operand
// bytes per flop and the kernel is close to the L2 -> shared-memory rate with every SM loading (4096^3:
// 101.6 us at 256, 128 us at 160). 320 (one tile per pair at most, see PairCfg) moves fewer operand bytes
// per flop than 256 and is taken whenever it has the least cost. TBF16_GEMM_PN = 320 / 256 / 192 / 160 /
// 128 forces one.
int pair_width(int M, int N, int pairs) {
  static const int env = [] {
    const char* e = getenv("TBF16_GEMM_PN");
    return e ? atoi(e) : 0;
  }();
  if (env == 320 || env == 256 || env == 192 || env == 160 || env == 128) return env;
  const int64_t tm = (M + 255) / 256;
  auto cost = [&](int pn) {
    const int64_t tiles = tm * ((N + pn - 1) / pn);
    return (tiles + pairs - 1) / pairs * (pn + 32);
  };
  // a narrower tile moves more operand bytes per flop (at 160, 30 % more per SM), so it has to save at
  // least a tenth of the waves' time to be taken
  int best = 256;
  int64_t best_cost = cost(256) * 9 / 10;
  for (int pn : {192, 160, 128}) {
    if (cost(pn) < best_cost) {
      best_cost = cost(pn);
      best = pn;
    }
  }
  if (tm * ((N + 319) / 320) <= pairs && cost(320) < best_cost) best = 320;
  return best;
}

template <bool A_MN, bool B_MN>
int launch_gemm_pair(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, const float* sa,
                     const float* sb, const void* bias, void* y, int64_t ldy, cudaStream_t st, bool pdl = false) {
  CUtensorMap ta;
  int rc = A_MN ? tbf16_host::make_tmap_2d(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, 64, 64)
                : tbf16_host::make_tmap_2d(&ta, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, 64, BM);
  if (rc) return rc;
  if (!B_MN) {
    const tbf16_host::DeviceInfo* d = tbf16_host::device_info();
    switch (pair_width(M, N, d ? d->sms / 2 : 74)) {
      case 320: return launch_pair_core<A_MN, false, false, 320>(ta, B, ldb, M, N, K, sa, sb, bias, y, ldy, nullptr, st, pdl);
      case 192: return launch_pair_core<A_MN, false, false, 192>(ta, B, ldb, M, N, K, sa, sb, bias, y, ldy, nullptr, st, pdl);
      case 160: return launch_pair_core<A_MN, false, false, 160>(ta, B, ldb, M, N, K, sa, sb, bias, y, ldy, nullptr, st, pdl);
      case 128: return launch_pair_core<A_MN, false, false, 128>(ta, B, ldb, M, N, K, sa, sb, bias, y, ldy, nullptr, st, pdl);
      default: break;
    }
  }
  return launch_pair_core<A_MN, B_MN, false, 256>(ta, B, ldb, M, N, K, sa, sb, bias, y, ldy, nullptr, st, pdl);
}

// The pair kernel whenever both dimensions span two or more 256 tiles (it moves a third less data from
// L2 per SM for the same CTA count; measured faster from M = N = 512 up), or the product fills the
// GPU with pair tiles; TBF16_GEMM_PAIR=0 / 1 forces the single-CTA / pair kernel.
bool use_pair(int M, int N) {
  static const int env = [] {
    const char* e = getenv("TBF16_GEMM_PAIR");
    return e ? atoi(e) : -1;
  }();
  if (env >= 0) return env != 0;
  return (M >= 512 && N >= 512) || (int64_t)((M + 255) / 256) * ((N + 255) / 256) >= 148;
}

bool ok8(int64_t v) { return v % 8 == 0; }

}  // namespace

namespace tbf16_host {

int conv_gemm_pair(const void* x16cl, int64_t B, int64_t D, int64_t H, int64_t W, int64_t C, const ConvGemm& cv,
                   const void* w16, int64_t ldw, int M, int N, const float* sa, const float* sb, const void* bias,
                   void* y, int64_t ldy, cudaStream_t st) {
  const int bx = cv.Wo < 128 ? cv.Wo : 128;
  CUtensorMap ta;
  if (int rc = make_tmap_conv_in(&ta, x16cl, B, D, H, W, C, bx, 128 / bx)) return rc;
  // K = taps x cb x 64: the weight rows are exactly one K long
  return launch_pair_core<false, false, true, 256>(ta, w16, ldw, M, N, (int)ldw, sa, sb, bias, y, ldy, &cv, st, true);
}

}  // namespace tbf16_host

extern "C" {

int tbf16_linear(const void* x, int64_t M, int64_t K, int64_t ldx, const void* w16, int64_t N, int64_t ldw,
                 const float* ws, const void* bias, void* y, int64_t ldy, float* x_sinv, void* x16_ws, int target_exp,
                 int l1, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (M < 0 || N < 0 || K < 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || ldx < K || ldw < K || ldy < N ||
      !ws || !x_sinv || !y)
    return TBF16_ERR_INVALID;
  if (!ok8(K) || !ok8(N) || !ok8(ldx) || !ok8(ldw) || !ok8(ldy) || !tbf16_host::aligned16(x) ||
      !tbf16_host::aligned16(w16) || !tbf16_host::aligned16(y))
    return TBF16_ERR_ALIGN;
  if (M == 0 || N == 0) return TBF16_OK;
  if (K == 0) return TBF16_ERR_UNSUPPORTED;
  if (x16_ws) {
    // Materialise fp16(x * s) once in the row pass (one HBM read of x), then the fp16-operand GEMM:
    // converting inside the GEMM would redo it for every N tile and compete with the tensor core for
    // shared-memory bandwidth.
    if (!tbf16_host::aligned16(x16_ws)) return TBF16_ERR_ALIGN;
    if (target_exp < 0 || target_exp > 64) return TBF16_ERR_INVALID;
    auto st = static_cast<cudaStream_t>(stream);
    if (int rc = tbf16_host::row_pass(x, M, K, ldx, target_exp, l1, 1, x16_ws, K, x_sinv, nullptr, st)) return rc;
    if (tbf16_host::use_skinny((int)M, (int)N))
      return tbf16_host::skinny_gemm(x16_ws, K, w16, ldw, (int)M, (int)N, (int)K, x_sinv, ws, bias, y, ldy, st,
                                       true);
    if (use_pair((int)M, (int)N))
      return launch_gemm_pair<false, false>(x16_ws, K, w16, ldw, (int)M, (int)N, (int)K, x_sinv, ws, bias, y, ldy, st,
                                            true);
    return launch_gemm<256, 4, false, false, false>(x16_ws, K, w16, ldw, (int)M, (int)N, (int)K, x_sinv, ws, bias, y,
                                                    ldy, st, true);
  }
  if (int st = tbf16_row_scale(x, M, K, ldx, target_exp, l1, x_sinv, nullptr, nullptr, 0, stream)) return st;
  return tbf16_linear_scaled(x, M, K, ldx, w16, N, ldw, ws, bias, y, ldy, x_sinv, stream);
}

int tbf16_linear_scaled(const void* x, int64_t M, int64_t K, int64_t ldx, const void* w16, int64_t N, int64_t ldw,
                        const float* ws, const void* bias, void* y, int64_t ldy, const float* x_sinv, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (M < 0 || N < 0 || K <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || ldx < K || ldw < K || ldy < N ||
      !ws || !x_sinv || !y)
    return TBF16_ERR_INVALID;
  if (!ok8(K) || !ok8(N) || !ok8(ldx) || !ok8(ldw) || !ok8(ldy) || !tbf16_host::aligned16(x) ||
      !tbf16_host::aligned16(w16) || !tbf16_host::aligned16(y))
    return TBF16_ERR_ALIGN;
  if (M == 0 || N == 0) return TBF16_OK;
  return launch_gemm<256, 4, true, false, false>(x, ldx, w16, ldw, (int)M, (int)N, (int)K, x_sinv, ws, bias, y, ldy,
                                                 static_cast<cudaStream_t>(stream));
}

int tbf16_gemm_f16(const void* a16, int a_mn, int64_t lda, const void* b16, int b_mn, int64_t ldb, int64_t M, int64_t N,
                   int64_t K, const float* sa, const float* sb, const void* bias, void* y, int64_t ldy, void* stream) {
  if (int st = tbf16_host::require_sm100()) return st;
  if (M < 0 || N < 0 || K <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || ldy < N || !sa || !y)
    return TBF16_ERR_INVALID;
  if (lda < (a_mn ? M : K) || ldb < (b_mn ? N : K)) return TBF16_ERR_INVALID;
  // K is a row length (must give 16-byte rows) only for a K-major operand; MN-major operands run along K
  // by rows of stride lda / ldb, and TMA fills the tail past K with zeros.
  if (((!a_mn || !b_mn) && !ok8(K)) || !ok8(N) || !ok8(lda) || !ok8(ldb) || !ok8(ldy) ||
      !tbf16_host::aligned16(a16) || !tbf16_host::aligned16(b16) || !tbf16_host::aligned16(y))
    return TBF16_ERR_ALIGN;
  if (M == 0 || N == 0) return TBF16_OK;
  auto st = static_cast<cudaStream_t>(stream);
  const int m = (int)M, n = (int)N, k = (int)K;
  if (!a_mn && !b_mn && tbf16_host::use_skinny(m, n))
    return tbf16_host::skinny_gemm(a16, lda, b16, ldb, m, n, k, sa, sb, bias, y, ldy, st, false);
  if (use_pair(m, n)) {
    if (!a_mn && !b_mn) return launch_gemm_pair<false, false>(a16, lda, b16, ldb, m, n, k, sa, sb, bias, y, ldy, st);
    if (!a_mn && b_mn) return launch_gemm_pair<false, true>(a16, lda, b16, ldb, m, n, k, sa, sb, bias, y, ldy, st);
    if (a_mn && !b_mn) return launch_gemm_pair<true, false>(a16, lda, b16, ldb, m, n, k, sa, sb, bias, y, ldy, st);
    return launch_gemm_pair<true, true>(a16, lda, b16, ldb, m, n, k, sa, sb, bias, y, ldy, st);
  }
  if (!a_mn && !b_mn) return launch_gemm<256, 4, false, false, false>(a16, lda, b16, ldb, m, n, k, sa, sb, bias, y, ldy, st);
  if (!a_mn && b_mn) return launch_gemm<256, 4, false, false, true>(a16, lda, b16, ldb, m, n, k, sa, sb, bias, y, ldy, st);
  if (a_mn && !b_mn) return launch_gemm<256, 4, false, true, false>(a16, lda, b16, ldb, m, n, k, sa, sb, bias, y, ldy, st);
  return launch_gemm<256, 4, false, true, true>(a16, lda, b16, ldb, m, n, k, sa, sb, bias, y, ldy, st);
}

}  // extern "C"
