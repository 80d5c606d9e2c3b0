// Shared device helpers for the sm_100a kernels: status codes, power-of-two scale rules, bf16/fp16
// packing, and inline-PTX wrappers for mbarriers, TMA and tcgen05 (TMEM, UMMA).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tbf16_sm100.h"

namespace tbf16 {

// ------------------------------------------------------------------ device error word
// Kernels that give up on a wait set a bit in a per-device word (defined in runtime.cu, passed to
// kernels as a pointer) and return. Read and cleared through tbf16_device_status().
constexpr unsigned int kErrWaitTimeout = 1u;
constexpr unsigned int kErrOverflow = 2u;
constexpr unsigned int kErrSmemAlign = 4u;  // dynamic shared window not 1024-byte aligned

// ------------------------------------------------------------------ scale rules
// The scale is an exact power of two built from exponent bits, never exp2/log2.

// Biased exponent of a non-negative fp32, clamped to [1, 252] (zero and subnormal behave like the
// smallest normal, inf/NaN like 2^125) -- tbf16/csrc/small_kernels.cu:13-14, gemm_sm75.cu:20-21.
__device__ __forceinline__ int clamped_biased_exp(float amax) {
  int e = (__float_as_int(amax) >> 23) & 0xFF;
  return min(max(e, 1), 252);
}

// Biased exponent of s with amax*s in [2^(t-1), 2^t): small_kernels.cu:15-16 clamps it to [1, 254].
__device__ __forceinline__ int scale_biased_exp_small(float amax, int t) {
  int se = 126 + t - (clamped_biased_exp(amax) - 127);
  return min(max(se, 1), 254);
}

// The fused GEMM's variant, gemm_sm75.cu:22: only the upper clamp.
__device__ __forceinline__ int scale_biased_exp_fused(float amax, int t) {
  return max(min(253 + t - clamped_biased_exp(amax), 254), 0);
}

// 2^(se-127) and its exact inverse 2^(127-se) from a biased exponent in [1, 254]. The inverse of
// 2^127 is the subnormal 2^-127, built from bits so that no flush to zero can touch it.
__device__ __forceinline__ float pow2_from_biased(int se) { return __int_as_float(se << 23); }
__device__ __forceinline__ float inv_pow2_from_biased(int se) {
  const int ie = 254 - se;  // biased exponent of 2^(127-se)
  return ie >= 1 ? __int_as_float(ie << 23) : __int_as_float(0x00400000);  // ie == 0 only for se == 254
}

// Exact 2^e for an integer e (normal, subnormal, 0 or inf at the extremes), from bits.
__device__ __forceinline__ float exp2i(int e) {
  if (e >= 128) return __int_as_float(0x7f800000);
  if (e >= -126) return __int_as_float((e + 127) << 23);
  if (e >= -149) return __int_as_float(1 << (e + 149));
  return 0.f;
}

// Exponent of frexp: |x| = m * 2^e with m in [0.5, 1); 0 for zero, inf and NaN (torch.frexp).
__device__ __forceinline__ int frexp_exp(float x) {
  const unsigned a = __float_as_uint(x) & 0x7fffffffu;
  if (a == 0 || a >= 0x7f800000u) return 0;
  const int e = (int)(a >> 23);
  if (e == 0) return -126 - (__clz(a) - 9);  // subnormal: leading zeros of the 23-bit mantissa
  return e - 126;
}

// ------------------------------------------------------------------ packing
__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ float f16lo(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xffff))); }
__device__ __forceinline__ float f16hi(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v >> 16))); }
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after timeout_ns (or at once when *abort is set by another thread of the
// CTA), records kErrWaitTimeout in *err, sets *abort and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, unsigned int* err,
                                          uint64_t timeout_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > timeout_ns) {
      atomicOr(err, kErrWaitTimeout);
      *abort = 1;
      return false;
    }
  }
}

// Warp-wide bounded wait: lane 0 polls (so 32 lanes do not hammer the barrier word), then every lane
// takes its own acquire of the completed phase. Safe when the barrier cannot complete its next phase
// before this warp has consumed the current one (true for every ring below).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort, unsigned int* err,
                                               uint64_t timeout_ns = 2000000000ull) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort, err, timeout_ns);
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  if (ok) (void)mbar_try_wait(bar, parity);
  return ok;
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// 2-D tiled load, no multicast. x is the innermost coordinate (elements, a multiple of 8 for 16-bit data).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// 1-D bulk copy global -> shared (no multicast); both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Make this thread's generic-proxy shared-memory writes visible to the async proxy (UMMA reads).
// Element-wise add of a shared tile into global memory through a 3-D tensor map (TMA reduction, no
// multicast); x (innermost) must be a multiple of 16 bytes and no coordinate may be negative.
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* m, const void* src, int x, int y, int z) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(m)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// 2-D tiled store from shared memory (bulk group completion). Coordinates must be >= 0 and x * 2 bytes a
// multiple of 16; TMA writes only the part of the box inside the tensor.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
// Fire-and-forget fp32 add into global memory (red.global.add: no return value, resolved in L2).
__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed bulk groups of this thread still read their shared source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N committed bulk groups of this thread are incomplete.
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------ tcgen05
// TMEM allocation: executed by one full warp; the allocated address lands in *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
// Warpgroup register re-split (all four warps of a warpgroup execute the same one). The shares of all
// warpgroups must add up to at most the registers the CTA was launched with, else an increase waits
// forever.
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (fp16/bf16 in, fp32 accumulate). One thread issues.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// D[tmem] (+)= A[tmem] * B[smem]^T.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Instruction descriptor, kind::f16 with fp16 A/B and fp32 D (bit layout of the PTX ISA's
// instruction descriptor table: D format [4,6), A/B format [7,10)/[10,13), A/B major [15]/[16],
// N>>3 [17,23), M>>4 [24,29)).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand tile (version 1, layout
// SWIZZLE_128B = 2 in bits [61,64)). lbo/sbo in bytes. K-major: sbo = 1024 (8 rows of 128 B), lbo
// unused (16). MN-major: lbo = stride between 64-element MN blocks, sbo = stride between 8-row K groups.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// 32 lanes x 32 bits, 32 consecutive columns: thread i of the warp gets row (lane base + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]));
}
// 32 lanes x 32 bits, 16 consecutive columns.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
}
// 32 lanes x 32 bits, 16 consecutive columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(pred));
  return pred != 0;
}

// ------------------------------------------------------------------ programmatic dependent launch
// Lets the next kernel of the stream, when launched with the programmatic-serialization attribute, start
// before this grid ends (no-op otherwise).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Waits until the preceding grid of the stream has completed and its memory is visible (returns at once
// for a kernel launched without the attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------ CTA pairs (cluster of 2, cta_group::2)
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// All threads of both CTAs of the cluster.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared::cluster address of the same shared offset in CTA `cta` of the cluster.
__device__ __forceinline__ uint32_t mapa_u32(uint32_t saddr, uint32_t cta) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(saddr), "r"(cta));
  return remote;
}
// 16-byte store into (possibly another CTA's) distributed shared memory.
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}
// Arrive on the mbarrier at the same shared offset in CTA `cta` of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(uint64_t* bar_local, uint32_t cta) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(bar_local)), "r"(cta));
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}
// Arrive on the mbarrier at the same shared offset in CTA `cta` with the instruction's default
// (release, CTA-scope) semantics: no cluster-wide fence, about 0.7 us cheaper per arrival than
// mbar_arrive_remote on B200. For handing over TMEM that the arriving thread has written and completed
// (tcgen05.wait::st, then tcgen05.fence::before_thread_sync) to a tcgen05.mma the other CTA issues
// after its wait and tcgen05.fence::after_thread_sync.
__device__ __forceinline__ void mbar_arrive_remote_tmem(uint64_t* bar_local, uint32_t cta) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(bar_local)), "r"(cta));
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}
// 2-D tiled load into this CTA's shared memory whose completion (bytes) is counted on the pair's even
// CTA's mbarrier at the same offset (bit 24 of the cluster shared address selects the CTA of the pair).
// No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* m, uint64_t* bar_local, int x, int y) {
  const uint32_t mbar = smem_u32(bar_local) & 0xFEFFFFFFu;
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(mbar), "r"(x), "r"(y)
      : "memory");
}
// 5-D tiled load for a CTA pair (no multicast), completing on the even CTA's barrier like tma_load_2d_pair.
__device__ __forceinline__ void tma_load_5d_pair(void* dst, const CUtensorMap* m, uint64_t* bar_local, int c0, int c1,
                                                 int c2, int c3, int c4) {
  const uint32_t mbar = smem_u32(bar_local) & 0xFEFFFFFFu;
  asm volatile(
      "cp.async.bulk.tensor.5d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(mbar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}
// 3-D tiled load for a CTA pair (no multicast), completing on the even CTA's barrier like tma_load_2d_pair.
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* m, uint64_t* bar_local, int x, int y,
                                                 int z) {
  const uint32_t mbar = smem_u32(bar_local) & 0xFEFFFFFFu;
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(mbar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// Bounded wait with cluster-scope acquire, for a phase completed by arrivals from the other CTA of the
// pair (its writes, released at cluster scope by the arrive, are visible after it).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, "
      "0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                  unsigned int* err, uint64_t timeout_ns = 2000000000ull) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > timeout_ns) {
      atomicOr(err, kErrWaitTimeout);
      *abort = 1;
      return false;
    }
  }
}
// TMEM allocation / release for a CTA pair: one warp with the same warp index in each CTA.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols));
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
// D[tmem of both CTAs] (+)= A[smem of both CTAs] * B[smem of both CTAs]^T with M = 256 split over the
// pair's TMEM and N split over the pair's shared B tiles. Issued by one thread of the even CTA.
__device__ __forceinline__ void umma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// D[tmem of both CTAs] (+)= A[tmem of both CTAs] * B[smem of both CTAs]: the TS form of umma_f16_ss_pair
// (each CTA's TMEM holds its 128 rows of A).
__device__ __forceinline__ void umma_f16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Arrive once on the mbarrier at this offset in every CTA of `mask` when the pair's MMAs issued so far complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar_local, uint16_t mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   smem_u32(bar_local)),
               "h"(mask)
               : "memory");
}

// ------------------------------------------------------------------ softmax arithmetic (attention)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100 executes one f32x2 add / mul / fma per lane per instruction).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ void f2_unpack(uint64_t d, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(d));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair of x <= 0 (or -inf) on the FMA pipe: Cody-Waite split x = n + f with n = rint(x)
// (adding 1.5 * 2^23 rounds to an integer in the low mantissa bits), 2^f on [-1/2, 1/2] by a degree-3
// polynomial fitted here for minimum maximum relative error (7.5e-5, below fp16's half ulp 2.4e-4,
// the precision P is kept in), and 2^n added into the exponent field. Inputs below -120 give 2^-120,
// which rounds to zero in fp16 and is negligible in the fp32 row sum.
__device__ __forceinline__ void ex2_poly2(float x0, float x1, float& p0, float& p1) {
  const uint64_t x = f2_pack(fmaxf(x0, -120.f), fmaxf(x1, -120.f));
  const uint64_t t = f2_add(x, f2_pack(12582912.f, 12582912.f));
  const uint64_t n = f2_add(t, f2_pack(-12582912.f, -12582912.f));
  const uint64_t f = f2_fma(n, f2_pack(-1.f, -1.f), x);
  uint64_t q = f2_fma(f2_pack(0.0551716685295105f, 0.0551716685295105f), f, f2_pack(0.2426111400127411f, 0.2426111400127411f));
  q = f2_fma(q, f, f2_pack(0.6932609677314758f, 0.6932609677314758f));
  q = f2_fma(q, f, f2_pack(0.9999280571937561f, 0.9999280571937561f));
  float q0, q1, t0, t1;
  f2_unpack(q, q0, q1);
  f2_unpack(t, t0, t1);
  p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
  p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}

// ------------------------------------------------------------------ attention dropout
// keep(bh, i, j) for query row i and key j of head bh, identical in the forward and backward kernels: a
// counter-based hash (murmur3's 32-bit finaliser) of a per-row key and the key pair j / 2 gives 32 bits,
// 16 per key of the pair; a key is kept when its 16 bits are >= thr = round(p * 65536), so the keep
// probability is exactly (65536 - thr) / 65536 and kept values are scaled by its inverse.
__host__ __device__ __forceinline__ uint32_t fmix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x85ebca6bu;
  x ^= x >> 13;
  x *= 0xc2b2ae35u;
  x ^= x >> 16;
  return x;
}
__host__ __device__ __forceinline__ uint32_t drop_row_key(uint32_t seed_lo, uint32_t seed_hi, uint32_t bh, uint32_t i) {
  return fmix32((fmix32(bh ^ seed_lo) + i * 0x9e3779b9u) ^ seed_hi);
}
__host__ __device__ __forceinline__ uint32_t drop_pair_bits(uint32_t row_key, uint32_t j_pair) {
  return fmix32(row_key ^ (j_pair * 0x7feb352du));
}
// Keep mask of keys (2 jp, 2 jp + 1) as a packed-fp16 lane mask (0xffff per kept half).
__device__ __forceinline__ uint32_t drop_pair_mask(uint32_t row_key, uint32_t j_pair, uint32_t thr) {
  const uint32_t bits = drop_pair_bits(row_key, j_pair);
  return ((bits & 0xffffu) >= thr ? 0x0000ffffu : 0u) | ((bits >> 16) >= thr ? 0xffff0000u : 0u);
}
// Whether key j is kept in row `row_key` (the backward's per-element form).
__device__ __forceinline__ bool drop_keep(uint32_t row_key, uint32_t j, uint32_t thr) {
  const uint32_t bits = drop_pair_bits(row_key, j >> 1);
  return ((j & 1) ? (bits >> 16) : (bits & 0xffffu)) >= thr;
}

// Byte offset of 16-byte chunk c (0..15 for 128 fp16 columns) of row r in a K-major tile made of
// 64-column 128B-swizzled atoms of 128 rows each.
__device__ __forceinline__ uint32_t swz_off(int r, int c) {
  return (uint32_t)((c >> 3) * 16384 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

}  // namespace tbf16

// Host helpers shared by the .cu files.
// Implicit convolution (the pair kernel's CONV form): A is not a matrix but the scaled channels-last
// fp16 input [B, D, H, W, C] seen through a 5-D tensor map. Row m of the product is output position
// (b, z, y, x) of a stride-1 convolution, K block kb is (tap = kb / cb, 64-channel block kb % cb), and a
// 128-row A tile -- bx x by output positions of one (b, z) slice -- is one box load at the tap's input
// offset: padding and the channels past C arrive as the load's zero fill.
struct ConvGemm {
  int Wo, Ho, Do;     // output extent
  int cb;             // 64-channel blocks per tap
  int kh, kw;         // kernel extent (kd = taps / (kh kw))
  int pw, ph, pd;     // zero padding
  int dw, dh, dd;     // dilation
  int sa_div;         // rows per sample: the row scale of row m is sa[m / sa_div]
};

namespace tbf16_host {
struct DeviceInfo {
  int device = -1;
  int sms = 0;
  int cc_major = 0, cc_minor = 0;
  unsigned int* err = nullptr;  // device address of the error word
};
// Info for the current device, filled once per device (not thread-safe against concurrent first use
// on the same device from two host threads; each field is written idempotently).
const DeviceInfo* device_info();
// TBF16_OK, or TBF16_ERR_DEVICE when the current device is not sm_100.
int require_sm100();
// 5-D tensor map of a channels-last fp16 tensor [B, D, H, W, C] (C % 8 == 0, 16-byte aligned) for the
// implicit convolution: box of 64 channels x bx x by positions x 1 x 1, 128-byte swizzle, zero fill.
int make_tmap_conv_in(CUtensorMap* map, const void* base, int64_t B, int64_t D, int64_t H, int64_t W, int64_t C,
                      int bx, int by);
// Implicit-GEMM convolution on the pair kernel (gemm.cu): y[M, N] (rows = output positions (b, z, y, x)
// of a stride-1 conv, M = B Do Ho Wo) = scaled products of x16cl [B, D, H, W, C] and w16 [N, taps x cb x 64]
// (row stride ldw = taps x cb x 64, channels zero-padded per tap); sa per sample. Validated by the caller.
int conv_gemm_pair(const void* x16cl, int64_t B, int64_t D, int64_t H, int64_t W, int64_t C, const ConvGemm& cv,
                   const void* w16, int64_t ldw, int M, int N, const float* sa, const float* sb, const void* bias,
                   void* y, int64_t ldy, cudaStream_t st);
// Maps the last CUDA error to a status (clears it).
int check_launch();
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
// Row amax / L1 -> power-of-two scale (fused rule if fused_rule, else the small-kernel rule), s_inv and
// optional int8 log2(s); with y non-null also y = fp16_rn(x * s) (row stride ldy). Rows up to 8192
// elements take one HBM read (row in registers). Arguments already validated by the caller.
int row_pass(const void* x, int64_t rows, int64_t K, int64_t ldx, int t, int l1, int fused_rule, void* y, int64_t ldy,
             float* s_inv, int8_t* exp_out, cudaStream_t st);
// Scaled GEMM for few activation rows (M <= kSkinnyMaxRows), both operands K-major fp16:
// y[m, n] = bf16((sum_k A[m,k] B[n,k]) * sa[m] * sb[n] + bias[n]) (gemm_skinny.cu). Validated by the caller.
constexpr int kSkinnyMaxRows = 256;
// after_row_pass: the preceding kernel of the stream is the row pass that writes A and sa (and nothing
// the GEMM reads otherwise); the GEMM is then launched as its programmatic dependent.
int skinny_gemm(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, const float* sa,
                const float* sb, const void* bias, void* y, int64_t ldy, cudaStream_t st, bool after_row_pass);
// Whether skinny_gemm takes an M x N product (TBF16_GEMM_SKINNY=0 / 1 forces it off / on for M <= 256).
bool use_skinny(int M, int N);
// Encode a 2-D tiled tensor map (16-bit elements, 128-byte swizzle) for a row-major [rows, cols]
// matrix with leading dimension ld (elements). Returns 0 on success.
int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols,
                 uint32_t box_rows);
// 3-D tiled tensor map (16-bit elements, 128-byte swizzle): dims {d0 (contiguous), d1, d2}, element
// strides of dims 1 and 2, box {box0, box1, 1}.
int make_tmap_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                 uint64_t stride2, uint32_t box0, uint32_t box1);
// Output map for TMA stores of bf16 tiles: rows of box_cols = 32 elements (64 bytes, 64-byte swizzle:
// 16-byte chunk c of row r sits at chunk c ^ ((r >> 1) & 3) in shared memory).
int make_tmap_2d_out(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols,
                     uint32_t box_rows);
// The same for fp32 elements with a 64- or 128-byte swizzle (box0 * 4 <= the swizzle span).
int make_tmap_3d_f32(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1,
                     uint64_t stride2, uint32_t box0, uint32_t box1, int swizzle_bytes = 128);
// Attention dropout: threshold (a key is kept when its 16 hash bits are >= thr) and 1 / keep probability
// for dropout_p in [0, 1); false outside that range.
inline bool dropout_params(float dropout_p, uint32_t* thr, float* inv_keep) {
  if (!(dropout_p >= 0.f && dropout_p < 1.f)) return false;
  const uint32_t t = (uint32_t)lrintf(dropout_p * 65536.f);
  if (t >= 65536u) return false;
  *thr = t;
  *inv_keep = 65536.f / (float)(65536u - t);
  return true;
}

}  // namespace tbf16_host
