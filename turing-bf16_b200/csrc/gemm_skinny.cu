// Scaled GEMM for few activation rows (9 <= M <= 256 in the linear; any M <= 256 in tbf16_gemm_f16):
//
//   y[m, n] = bf16_rn((sum_k A16[m,k] * B16[n,k]) * sa[m] * sb[n] + bias[n])
//
// the same result as scaled_gemm_kernel, shaped for the weight-streaming regime. With one 128-row M
// tile the output-tiled GEMM keeps only N / 256 CTAs busy (16 at N = 4096), each bound by its own SM's
// load bandwidth; here the product is computed transposed and split over K:
//   * the weight B supplies the MMA's 128-row operand (its rows are the TMEM lanes) and the activation A
//     the MMA's N operand (Mp = M rounded up to 16 columns; rows past M are TMA zero fill);
//   * a cluster of S CTAs (S <= 8, one per SM) shares one 128-row weight tile and splits its K blocks,
//     so N / 128 * S CTAs stream the weight (128 at N = 4096 with S = 4);
//   * after the main loop every CTA pushes its fp32 partial accumulator, 16 columns at a time, into the
//     shared memory of the CTA that owns those columns (distributed shared memory, no workspace, no
//     second launch); the owner adds the S partials in rank order and applies the scales and bias.
// Roles: warp 0 TMA producer (one lane), warp 1 TMEM allocation + MMA issue (one lane), warps 2-5
// epilogue (TMEM lane quadrant = warp % 4). Every mbarrier wait is bounded; the two cluster barriers
// are reached by every thread of every CTA whatever happened before them.
#include <algorithm>

#include "common.cuh"

using namespace tbf16;

namespace {

constexpr int kRowsW = 128;                 // weight rows per tile: MMA M, TMEM lanes
constexpr int kBK = 64;                     // one 128-byte swizzle atom of fp16
constexpr int kWBytes = kRowsW * kBK * 2;   // 16 KB weight tile per stage
constexpr int kMaxStages = 8;
constexpr int kStageArea = 192 * 1024;      // stage ring, reused as the partial-sum receive area
constexpr int kThreads = 192;
constexpr int kMaxSplit = 8;                // portable cluster size
constexpr int kBarBytes = 8 * (2 * kMaxStages + 1) + 16;
constexpr int kSmem = 1024 + kStageArea + kBarBytes;
static_assert(kSmem <= 227 * 1024, "shared memory");

struct SkinnyParams {
  int M, N, Mp, S, stages, kb_total;
  int kbs;  // K blocks per stage (consecutive 64-wide boxes of the same rows)
  int pdl;  // launched as a programmatic dependent of the row pass that writes A and sa
  uint32_t idesc;
  uint32_t tmem_cols;
  const float* sa;            // [M]
  const float* sb;            // [N] or null
  const __nv_bfloat16* bias;  // [N] or null
  __nv_bfloat16* y;
  int64_t ldy;
  unsigned int* err;
};

// Receive slot of (source rank, owned group j, weight row): 16 fp32 = four 16-byte chunks; chunk c
// lives at c ^ ((row >> 1) & 3) so the 8 rows of a quarter-warp cover all 32 banks.
__device__ __forceinline__ uint32_t recv_off(int src, int j, int J, int row) {
  return (uint32_t)(((src * J + j) * kRowsW + row) * 64);
}
__device__ __forceinline__ uint32_t chunk_off(int c, int row) { return (uint32_t)((c ^ ((row >> 1) & 3)) * 16); }

__global__ void __launch_bounds__(kThreads, 1)
    scaled_gemm_skinny_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                              const SkinnyParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStageArea);
  uint64_t* empty = full + kMaxStages;
  uint64_t* tfull = empty + kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = (int)cluster_ctarank();  // == blockIdx.x: the grid's x extent is the cluster size S
  const int n0 = blockIdx.y * kRowsW;
  const int kb0 = rank * p.kb_total / p.S, kb1 = (rank + 1) * p.kb_total / p.S;  // >= 1 block: S <= kb_total
  const int x_bytes = p.Mp * kBK * 2;
  const int stage_bytes = p.kbs * (kWBytes + x_bytes);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    *abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) tmem_alloc(tmem_slot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      // The weight does not depend on the preceding row pass: fill the ring's weight tiles first, then
      // wait for the row pass (activation rows and their scales) and add the activation tiles.
      const int pre = min(p.stages, (kb1 - kb0 + p.kbs - 1) / p.kbs);
      for (int i = 0; i < pre; ++i) {
        const int kb = kb0 + i * p.kbs, nb = min(p.kbs, kb1 - kb);
        uint8_t* sW = smem + i * stage_bytes;
        mbar_arrive_expect_tx(&full[i], (uint32_t)(nb * (kWBytes + x_bytes)));
        for (int b = 0; b < nb; ++b) tma_load_2d(sW + b * kWBytes, &tmW, &full[i], (kb + b) * kBK, n0);
      }
      if (p.pdl) pdl_wait();
      for (int i = 0; i < pre; ++i) {
        const int kb = kb0 + i * p.kbs, nb = min(p.kbs, kb1 - kb);
        uint8_t* sX = smem + i * stage_bytes + p.kbs * kWBytes;
        for (int b = 0; b < nb; ++b) tma_load_2d(sX + b * x_bytes, &tmX, &full[i], (kb + b) * kBK, 0);
      }
      int stage = pre == p.stages ? 0 : pre;
      uint32_t phase = pre == p.stages ? 1 : 0;
      for (int kb = kb0 + pre * p.kbs; kb < kb1; kb += p.kbs) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort, p.err)) break;
        const int nb = min(p.kbs, kb1 - kb);
        uint8_t* sW = smem + stage * stage_bytes;
        uint8_t* sX = sW + p.kbs * kWBytes;
        mbar_arrive_expect_tx(&full[stage], (uint32_t)(nb * (kWBytes + x_bytes)));
        for (int b = 0; b < nb; ++b) tma_load_2d(sW + b * kWBytes, &tmW, &full[stage], (kb + b) * kBK, n0);
        for (int b = 0; b < nb; ++b) tma_load_2d(sX + b * x_bytes, &tmX, &full[stage], (kb + b) * kBK, 0);
        if (++stage == p.stages) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer: D[128 x Mp] += W . X^T
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; kb += p.kbs) {
        if (!mbar_wait(&full[stage], phase, abort, p.err)) { ok = false; break; }
        tc_fence_after();
        const int nb = min(p.kbs, kb1 - kb);
        const uint32_t w_base = smem_u32(smem + stage * stage_bytes);
        const uint32_t x_base = w_base + p.kbs * kWBytes;
        for (int b = 0; b < nb; ++b) {
          const uint32_t w_addr = w_base + b * kWBytes, x_addr = x_base + b * x_bytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_f16_ss(tmem_base, smem_desc_sw128(w_addr + k * 32, 16, 1024),
                        smem_desc_sw128(x_addr + k * 32, 16, 1024), p.idesc, (kb != kb0 || b != 0 || k != 0) ? 1u : 0u);
        }
        umma_commit(&empty[stage]);
        if (++stage == p.stages) { stage = 0; phase ^= 1; }
      }
      if (ok) umma_commit(tfull);
    }
  }

  // ---------------------------------------------------------------- split-K reduction and epilogue
  const bool epi = warp >= 2;
  const int quad = warp & 3;  // TMEM lane quadrant this warp may access
  const int row = quad * 32 + lane;
  const int G = p.Mp / 16, J = (G + p.S - 1) / p.S;
  bool have = false;
  if (epi) {
    have = mbar_wait_warp(tfull, 0, abort, p.err);
    tc_fence_after();
  }
  __syncwarp();
  // Every CTA of the cluster is past its main loop: all stage memory is free to receive partials.
  cluster_sync();
  if (epi && have) {
    const uint32_t base = smem_u32(smem);
#pragma unroll 1
    for (int g = 0; g < G; ++g) {
      uint32_t r[16];
      tmem_ld16(tmem_base + g * 16 + ((uint32_t)(quad * 32) << 16), r);
      tmem_ld_wait();
      const uint32_t dst = mapa_u32(base + recv_off(rank, g / p.S, J, row), (uint32_t)(g % p.S));
#pragma unroll
      for (int c = 0; c < 4; ++c) st_cluster_v4(dst + chunk_off(c, row), r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
    }
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // all partials have landed in their owners' shared memory
  if (epi && have && !*abort) {
    if (p.pdl) pdl_wait();  // sa comes from the row pass
    const int n = n0 + row;
    const bool nok = n < p.N;
    const float sbv = (nok && p.sb) ? __ldg(p.sb + n) : 1.f;
    const float bv = (nok && p.bias) ? __bfloat162float(p.bias[n]) : 0.f;
#pragma unroll 1
    for (int j = 0; j < J; ++j) {
      const int g = j * p.S + rank;
      if (g >= G) break;
      float acc[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) acc[e] = 0.f;
#pragma unroll 1
      for (int src = 0; src < p.S; ++src) {
        const uint8_t* slot = smem + recv_off(src, j, J, row);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float4 v = *reinterpret_cast<const float4*>(slot + chunk_off(c, row));
          acc[4 * c] += v.x;
          acc[4 * c + 1] += v.y;
          acc[4 * c + 2] += v.z;
          acc[4 * c + 3] += v.w;
        }
      }
      if (nok) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int m = g * 16 + e;
          if (m < p.M) {
            float v = (acc[e] * __ldg(p.sa + m)) * sbv;
            if (p.bias) v += bv;
            p.y[(int64_t)m * p.ldy + n] = __float2bfloat16_rn(v);
          }
        }
      }
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
    tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

}  // namespace

namespace tbf16_host {

bool use_skinny(int M, int N) {
  (void)N;
  static const int env = [] {
    const char* e = getenv("TBF16_GEMM_SKINNY");
    return e ? atoi(e) : -1;
  }();
  if (M > kSkinnyMaxRows || env == 0) return false;
  return true;
}

int skinny_gemm(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, const float* sa,
                const float* sb, const void* bias, void* y, int64_t ldy, cudaStream_t st, bool after_row_pass) {
  const DeviceInfo* d = device_info();
  if (!d) return TBF16_ERR_DEVICE;
  if (M <= 0 || M > kSkinnyMaxRows || N <= 0 || K <= 0) return TBF16_ERR_INVALID;
  const int Mp = (M + 15) / 16 * 16;
  const int tiles = (N + kRowsW - 1) / kRowsW;
  const int kb_total = (K + kBK - 1) / kBK;
  // Tuning overrides: TBF16_SKINNY_SPLIT (cluster size, power of two <= 8), TBF16_SKINNY_KBS (K blocks
  // per stage, 1..4).
  static const int split_env = [] {
    const char* e = getenv("TBF16_SKINNY_SPLIT");
    return e ? atoi(e) : 0;
  }();
  static const int kbs_env = [] {
    const char* e = getenv("TBF16_SKINNY_KBS");
    return e ? atoi(e) : 0;
  }();
  int S = 1;
  if (split_env > 0) {
    while (2 * S <= std::min(split_env, kMaxSplit) && 2 * S <= kb_total) S *= 2;
  } else {
    while (2 * S <= kMaxSplit && (int64_t)tiles * 2 * S <= d->sms && 2 * S <= kb_total) S *= 2;
  }
  // Two consecutive K blocks per stage while a stage stays <= 36 KB (Mp <= 128): each weight row is then
  // read in 256-byte runs, measured a few percent faster than 128-byte runs.
  const int kbs = (kbs_env >= 1 && kbs_env <= 4) ? kbs_env : (Mp <= 128 ? 2 : 1);
  const int stage_bytes = kbs * (kWBytes + Mp * kBK * 2);
  if (stage_bytes > kStageArea / 2) return TBF16_ERR_UNSUPPORTED;
  CUtensorMap tw, tx;
  if (int rc = make_tmap_2d(&tw, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, kBK, kRowsW)) return rc;
  if (int rc = make_tmap_2d(&tx, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, kBK, (uint32_t)Mp)) return rc;
  static bool attr_done[64] = {false};
  if (!attr_done[d->device & 63]) {
    if (cudaFuncSetAttribute(scaled_gemm_skinny_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) !=
        cudaSuccess)
      return check_launch();
    attr_done[d->device & 63] = true;
  }
  SkinnyParams p;
  p.M = M; p.N = N; p.Mp = Mp; p.S = S; p.kbs = kbs;
  p.pdl = after_row_pass ? 1 : 0;
  p.stages = std::min(kMaxStages, kStageArea / stage_bytes);
  p.kb_total = kb_total;
  p.idesc = idesc_f16_f32(kRowsW, Mp, false, false);
  uint32_t cols = 32;
  while ((int)cols < Mp) cols *= 2;
  p.tmem_cols = cols;
  p.sa = sa; p.sb = sb;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.ldy = ldy;
  p.err = d->err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(S, tiles);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // After the linear's own row pass (which writes only A and sa), start early and stream the weight while
  // the row pass runs; the kernel waits for the row pass before it reads A or sa.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = after_row_pass ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, scaled_gemm_skinny_kernel, tw, tx, p) != cudaSuccess) return check_launch();
  return check_launch();
}

}  // namespace tbf16_host
