/*
 * libtbf16_sm100 -- C ABI of the B200 (sm_100a) kernels behind tbf16's scaled bf16-on-fp16 path.
 *
 * Conventions
 *   - Plain pointers to device memory, sizes and strides in ELEMENTS, an explicit CUDA stream
 *     (a cudaStream_t passed as void*; NULL = the legacy default stream). Every call is
 *     asynchronous on that stream and never synchronises the host.
 *   - The library never allocates or frees device memory: outputs and any workspace are passed in.
 *   - bf16 / fp16 tensors are passed as void* holding 16-bit values; dtype codes below.
 *   - Returns 0 (TBF16_OK) or a status code. Argument checks (shape, alignment, dtype) happen on
 *     the host before any launch; a kernel that gives up on a bounded wait records it in a device
 *     word read by tbf16_device_status().
 *   - Requires an sm_100 device (B200). The reference's compute_75 kernels are replaced, not wrapped.
 *
 * Each entry point names the reference interface it replaces (tech-cosmos/turing-bf16; paths relative
 * to that project's root).
 */
#ifndef TBF16_SM100_H
#define TBF16_SM100_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum tbf16_status {
  TBF16_OK = 0,
  TBF16_ERR_INVALID = 1,     /* bad shape / stride / argument */
  TBF16_ERR_ALIGN = 2,       /* pointer or leading dimension not aligned for 16-byte / TMA access */
  TBF16_ERR_DTYPE = 3,       /* unsupported dtype code */
  TBF16_ERR_LAUNCH = 4,      /* CUDA launch or runtime error */
  TBF16_ERR_DEVICE = 5,      /* not an sm_100 device */
  TBF16_ERR_UNSUPPORTED = 6, /* a valid request this build does not implement */
  TBF16_ERR_TIMEOUT = 7      /* a kernel gave up on a bounded wait (see tbf16_device_status) */
};

enum tbf16_dtype { TBF16_BF16 = 0, TBF16_F16 = 1 };

/* ------------------------------------------------------------------ library */

/* ABI version (major * 100 + minor). */
int tbf16_abi_version(void);
/* Human-readable text for a status code. */
const char* tbf16_status_string(int status);
/* TBF16_OK if `device` is an sm_100 GPU this build runs on. */
int tbf16_device_check(int device);
/* Bits set by kernels on the current device since the last reset (1 = a bounded wait timed out,
 * 2 = attention backward produced a non-finite value, 4 = a kernel found its dynamic shared memory
 * window not 1024-byte aligned and did nothing). Synchronises the device; reset != 0 clears. */
int tbf16_device_status(unsigned int* bits, int reset);
/* Failure-path self-test (no counterpart in the reference): one warp waits on an mbarrier that nothing
 * arrives on, through the bounded-wait helper the pipelined kernels use, with the limit timeout_ns
 * (1 ns .. 1 s) instead of their 2 s. The wait gives up, sets bit 1 of the device status word and the
 * kernel returns, leaving the context usable; read and clear the bit with tbf16_device_status. */
int tbf16_selftest_bounded_wait(uint64_t timeout_ns, void* stream);

/* ------------------------------------------------------------------ row / column power-of-two scales */

/* Row scales of the fused GEMM's pre-pass. Replaces row_scale(x, t, l1)
 * (tbf16/csrc/gemm_sm75.cu:243-253, kernel :27-47). x: bf16 [rows, K], row stride ldx.
 * s_inv[r] = 1 / s[r], s[r] = 2^(min(253 + t - e, 254) - 127) with e the clamped biased exponent of
 * the row max (l1 = 0) or L1 norm (l1 = 1). exp_out (nullable): int8 log2(s[r]). t must be >= 0.
 * y16 (nullable): also write fp16_rn(x * s[r]) there (row stride ldy) in the same read of x, the
 * operand the fused kernel converts on the fly (gemm_sm75.cu:108,132). Rows up to 8192 elements are
 * read once (held in registers). */
int tbf16_row_scale(const void* x, int64_t rows, int64_t K, int64_t ldx, int target_exp, int l1, float* s_inv,
                    int8_t* exp_out, void* y16, int64_t ldy, void* stream);

/* Row quantisation. Replaces quantize_rows(x, t, l1) (tbf16/csrc/small_kernels.cu:275-287, kernel
 * :35-74; Python tbf16/ops.py:74-89). y16 = fp16_rn(x * s[r]) with s from small_kernels.cu:12-18
 * (row amax or L1 norm into [2^(t-1), 2^t)); s_inv = 1 / s. y16 row stride ldy. */
int tbf16_quantize_rows(const void* x, int64_t rows, int64_t K, int64_t ldx, int target_exp, int l1, void* y16,
                        int64_t ldy, float* s_inv, void* stream);

/* Column quantisation. Replaces quantize_cols(x, t, row_mul) (tbf16/csrc/small_kernels.cu:318-340,
 * kernels :136-184; Python tbf16/autograd.py:26-36). amax[c] = max_r |x[r,c]| * |row_mul[r]|,
 * s[c] from small_kernels.cu:12-18, y16 = fp16_rn(x * row_mul[r] * s[c]) (row stride ldy), s_inv[c] = 1/s[c].
 * row_mul nullable. amax_ws: workspace of K floats (overwritten). rows == 0 gives s_inv = 1. */
int tbf16_quantize_cols(const void* x, int64_t rows, int64_t K, int64_t ldx, int target_exp, const float* row_mul,
                        void* y16, int64_t ldy, float* s_inv, float* amax_ws, void* stream);

/* Allocation-free variant of tbf16_quantize_cols, for callers that cannot allocate device memory where
 * they call in (an arena that owns every allocation, a plugin without access to its host's allocator, a
 * path where cudaMalloc's implicit synchronisation is not allowed). Same inputs, outputs and results;
 * the K-float column-maximum workspace lives in a file-scope device array of TBF16_NOALLOC_MAX_COLS
 * floats (256 KB) that every GPU loading the library holds until exit. K > TBF16_NOALLOC_MAX_COLS
 * returns TBF16_ERR_INVALID. No cudaMalloc / cudaFree. All calls on a GPU share the array: calls that
 * overlap on the GPU race. The first call on each device resolves the array's address
 * (cudaGetSymbolAddress); make that first call before any stream capture. The address is kept for the
 * life of the process: after cudaDeviceReset (or anything else that destroys and re-creates the
 * device's primary context) the library's module is loaded again and the array may move, so do not
 * call this entry point on that device afterwards.
 * No counterpart in the reference (its extension allocates every workspace with torch::empty). */
#define TBF16_NOALLOC_MAX_COLS 65536
int tbf16_quantize_cols_noalloc(const void* x, int64_t rows, int64_t K, int64_t ldx, int target_exp,
                                const float* row_mul, void* y16, int64_t ldy, float* s_inv, void* stream);

/* ------------------------------------------------------------------ attention scales */

/* Per-(b, h) amax of a strided (B, H, S, D) tensor with contiguous D. Replaces head_amax(x)
 * (tbf16/csrc/small_kernels.cu:342-359, kernel :221-243). amax: fp32 [B*H], overwritten. */
int tbf16_head_amax(const void* x, int dtype, int64_t B, int64_t H, int64_t S, int64_t D, int64_t sb, int64_t sh,
                    int64_t ss, float* amax, void* stream);

/* head_exp (tbf16/attention.py:24-27): e[b*H+h] = frexp exponent of amax (0 for all-zero heads).
 * amax_ws: workspace of B*H floats. */
int tbf16_head_exp(const void* x, int dtype, int64_t B, int64_t H, int64_t S, int64_t D, int64_t sb, int64_t sh,
                   int64_t ss, int32_t* e, float* amax_ws, void* stream);

/* y (contiguous B, H, S, D) = cast(x * 2^e[b, h]). Replaces head_scale_cast(x, e, dtype)
 * (tbf16/csrc/small_kernels.cu:361-379, kernel :246-263; Python attention.py:30-35). e is int32
 * indexed e[b * e_sb + h * e_sh] (broadcast strides may be 0). */
int tbf16_head_scale_cast(const void* x, int in_dtype, int64_t B, int64_t H, int64_t S, int64_t D, int64_t sb,
                          int64_t sh, int64_t ss, const int32_t* e, int64_t e_sb, int64_t e_sh, void* y, int out_dtype,
                          void* stream);

/* prepare_qkv (tbf16/attention.py:38-48) on the device, no host sync: eq, ek = max over (b, h) of the
 * frexp exponents of q and k head maxima; a = clamp(floor((ek - eq) / 2), ek - 14, 14 - eq);
 * ev[b, hk] = head_exp(v) - v_exp; q16 = fp16(q * 2^a), k16 = fp16(k * 2^-a), v16 = fp16(v * 2^-ev),
 * all contiguous (B, H, S, D). q is (B, Hq, Sq, D), k and v (B, Hkv, Sk, D), each with its own
 * strides (sb, sh, ss) and contiguous D. a_out: one int32; ev_out: int32 [B*Hkv].
 * ws: workspace of (B*Hq + 2*B*Hkv) floats. */
int tbf16_prepare_qkv(const void* q, int64_t qsb, int64_t qsh, int64_t qss, const void* k, int64_t ksb, int64_t ksh,
                      int64_t kss, const void* v, int64_t vsb, int64_t vsh, int64_t vss, int64_t B, int64_t Hq,
                      int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, int v_exp, void* q16, void* k16, void* v16,
                      int32_t* a_out, int32_t* ev_out, float* ws, void* stream);

/* tbf16_prepare_qkv in two phases for attention sharded over heads (this build's head-parallel form of
 * attention.py:38-48; the reference runs on one GPU): eq and ek are maxima over ALL (b, h), so each rank
 * computes its own, the caller all-reduces them (MAX), and the second phase scales with the result.
 * Phase 1: eqk[0..1] (int32, device) = this rank's eq, ek (INT_MIN when B = 0); ws (B*Hq + 2*B*Hkv
 * floats) keeps the per-head maxima, v's included. Phase 2: a from the all-reduced eqk (same rule as
 * tbf16_prepare_qkv), ev from ws's v maxima, q16 / k16 / v16 as tbf16_prepare_qkv writes them. Same
 * arguments and layouts as tbf16_prepare_qkv; ws must be the one phase 1 filled. */
int tbf16_qkv_local_exponents(const void* q, int64_t qsb, int64_t qsh, int64_t qss, const void* k, int64_t ksb,
                              int64_t ksh, int64_t kss, const void* v, int64_t vsb, int64_t vsh, int64_t vss, int64_t B,
                              int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, int32_t* eqk, float* ws,
                              void* stream);
int tbf16_prepare_qkv_global(const void* q, int64_t qsb, int64_t qsh, int64_t qss, const void* k, int64_t ksb,
                             int64_t ksh, int64_t kss, const void* v, int64_t vsb, int64_t vsh, int64_t vss, int64_t B,
                             int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, int v_exp, const int32_t* eqk,
                             const float* ws, void* q16, void* k16, void* v16, int32_t* a_out, int32_t* ev_out,
                             void* stream);

/* ------------------------------------------------------------------ scaled GEMMs (tcgen05) */

/* Fused scaled linear. Replaces linear(x, w16, ws, bias, cfg, t, l1) (tbf16/csrc/gemm_sm75.cu:257-284,
 * kernel :78-226) and, since the cuBLAS small-M branch is gone, scaled_linear for every M
 * (tbf16/ops.py:153-164). x bf16 [M, K] (row stride ldx); w16 fp16 [N, K] (ldw); ws fp32 [N];
 * bias bf16 [N] or NULL; y bf16 [M, N] (ldy).
 *   s_inv[m] = row_scale(x, t, l1)                           (written to x_sinv, M floats)
 *   y[m, n]  = bf16_rn((sum_k fp16(x[m,k] / s_inv[m]) * w16[n,k]) * s_inv[m] * ws[n] + bias[n])
 * with fp32 accumulation in TMEM and no fp16 rounding of the product. K, N, ldx, ldw multiples of 8.
 * x16_ws (nullable): fp16 [M, K] workspace. Given, the row pass writes fp16(x / s_inv) there in the same
 * read of x and the GEMM takes fp16 operands (the fast path); NULL converts x inside the GEMM. */
int tbf16_linear(const void* x, int64_t M, int64_t K, int64_t ldx, const void* w16, int64_t N, int64_t ldw,
                 const float* ws, const void* bias, void* y, int64_t ldy, float* x_sinv, void* x16_ws, int target_exp,
                 int l1, void* stream);

/* The GEMM half of tbf16_linear with the row scales given (x_sinv: M powers of two, e.g. from
 * tbf16_row_scale or from a producer kernel that already knows its rows' maxima). Same semantics as the
 * reference's gemm_kernel (tbf16/csrc/gemm_sm75.cu:78-226) launched after its row_scale pre-pass. */
int tbf16_linear_scaled(const void* x, int64_t M, int64_t K, int64_t ldx, const void* w16, int64_t N, int64_t ldw,
                        const float* ws, const void* bias, void* y, int64_t ldy, const float* x_sinv, void* stream);

/* Scaled fp16 GEMM with a bf16 epilogue: y[m, n] = bf16_rn((sum_k A[m,k] B[n,k]) * sa[m] * sb[n] + bias[n]).
 * Replaces the cuBLAS GEMM + epilogue pair of linear_q (tbf16/ops.py:167-178, small_kernels.cu:289-302)
 * and _scaled_mm (tbf16/autograd.py:114-120), i.e. the training dX and dW contractions.
 * A is a16 [M, K] (a_mn = 0, row stride lda) or a16 [K, M] (a_mn = 1); B is b16 [N, K] (b_mn = 0)
 * or b16 [K, N] (b_mn = 1). sb and bias nullable. Contiguous dimensions and leading dimensions
 * must be multiples of 8. */
int tbf16_gemm_f16(const void* a16, int a_mn, int64_t lda, const void* b16, int b_mn, int64_t ldb, int64_t M, int64_t N,
                   int64_t K, const float* sa, const float* sb, const void* bias, void* y, int64_t ldy, void* stream);

/* Few-row linear for decode: y[m, n] = bf16_rn((sum_k x[m,k] w16[n,k]) * ws[n] + bias[n]) for M <= 8 rows,
 * fp32 products of bf16 x and fp16 w (no activation scaling). Replaces the reference's single-row gemv
 * (tbf16/csrc/small_kernels.cu:107-132, called by tbf16/ops.py:207-218) and extends it to 8 rows that
 * share one pass over the weight. x bf16 [M, K] (row stride ldx), w16 fp16 [N, K] (ldw), ws fp32 [N],
 * bias bf16 [N] nullable, y bf16 [M, N] (ldy). K, ldx, ldw multiples of 8; x, w16 16-byte aligned.
 * M > TBF16_GEMV_MAX_ROWS returns TBF16_ERR_UNSUPPORTED (use tbf16_linear). */
#define TBF16_GEMV_MAX_ROWS 8
int tbf16_gemv(const void* x, int64_t M, int64_t K, int64_t ldx, const void* w16, int64_t N, int64_t ldw,
               const float* ws, const void* bias, void* y, int64_t ldy, void* stream);

/* ------------------------------------------------------------------ producer fusion */
/* The kernels that produce a linear's input also give its row scales, so the linear needs no row pass:
 * pass the y16 / s_inv they write to tbf16_gemm_f16 (A = y16, sa = s_inv) or tbf16_linear_scaled. The
 * reference runs these as separate passes (torch's activation or norm, then its quantize / row_scale
 * kernel: tbf16/ops.py:74-89, tbf16/csrc/gemm_sm75.cu:27-47); its own notes name them as the cost that
 * dominates at small token counts. Rows up to 16384 elements (TBF16_ERR_UNSUPPORTED above). */
#define TBF16_ACT_SILU 0
#define TBF16_ACT_GELU_TANH 1
#define TBF16_FUSED_MAX_ROW 16384

/* Gated MLP activation: h[m, i] = bf16_rn(bf16_rn(act(g[m, i])) * u[m, i]) (act in fp32 with the fast
 * exp and division: silu x / (1 + exp(-x)), or GELU with the tanh approximation), torch's act(g) * u on
 * bf16 tensors to within one bf16 ulp (identical in all but ~1e-4 of the elements);
 * then s_inv[m] = the fused rule's power-of-two row scale of h (row max, target target_exp, as
 * tbf16_row_scale) and y16[m, i] = fp16_rn(h[m, i] / s_inv[m]). h is also written to h_out when non-null.
 * g, u bf16 [M, I] (row strides ldg, ldu), y16 fp16 [M, I] (ldy), h_out bf16 (ldo). I and the strides
 * multiples of 8, pointers 16-byte aligned. */
int tbf16_glu_rows(const void* g, int64_t ldg, const void* u, int64_t ldu, int64_t M, int64_t I, int act,
                   int target_exp, void* y16, int64_t ldy, float* s_inv, void* h_out, int64_t ldo, void* stream);

/* Backward of the gated activation for training, as torch's autograd differentiates act(g) * u on bf16
 * tensors: with a = bf16_rn(act(g)) recomputed, du = bf16_rn(dh * a), da = bf16_rn(dh * u) and
 * dg = bf16_rn(da * act'(g)) (act' in fp32: silu s (1 + g (1 - s)), s = 1 / (1 + exp(-g)); tanh-GELU
 * 0.5 (1 + t) + 0.5 g (1 - t^2) sqrt(2/pi) (1 + 3 * 0.044715 g^2)). One read of dh, g, u and one write of
 * dg, du instead of torch's four elementwise passes. No reference counterpart (the reference leaves the
 * activation to torch). All bf16 [M, I], strides and I multiples of 8, pointers 16-byte aligned. */
int tbf16_glu_bwd(const void* dh, int64_t ldh, const void* g, int64_t ldg, const void* u, int64_t ldu, int64_t M,
                  int64_t I, int act, void* dg, int64_t lddg, void* du, int64_t lddu, void* stream);

/* Attention operands: per-head RMSNorm (optional) and rotary embedding in one pass, as a model computes
 * them on bf16 tensors. x: bf16 rows of D values, one per head of a token: row r is head r % H of token
 * r / H, at x + (r / H) * ldtok + (r % H) * D, position (r / H) % S -- a (B, S, H, D) tensor whose heads
 * are contiguous and whose tokens are ldtok >= H * D elements apart (a column slice of a fused QKV
 * projection, or contiguous with ldtok = H * D). M a multiple of H. out: rows ldo apart. With w non-null, y = rmsnorm over the row as
 * tbf16_rmsnorm_rows (style, offset, eps); else y = x. Then out = bf16_rn(bf16_rn(y * cos) + bf16_rn(rot(y) *
 * sin)), rot(y) = (-y[D/2:], y[:D/2]) (rotate-half), cos / sin bf16 [S, D] rows (row stride ldc). Replaces
 * the norm + five elementwise passes (mul, neg, cat, mul, add) before the attention's scale passes; no
 * reference counterpart (the reference leaves both to the model). D = 64, 128, 256 or 512
 * (TBF16_ERR_UNSUPPORTED otherwise); strides multiples of 8, pointers 16-byte aligned. */
int tbf16_rmsnorm_rope(const void* x, int64_t ldtok, const void* w, int64_t M, int64_t D, float eps, int style,
                       float offset, const void* cos, const void* sin, int64_t ldc, int64_t S, int64_t H, void* out,
                       int64_t ldo, void* stream);

/* RMSNorm: ms[m] = mean_k x[m, k]^2 (fp32), rs = rsqrt(ms + eps) and
 *   style TBF16_NORM_SCALE_FP32: r[m, k] = bf16_rn((x[m, k] * rs) * (w[k] + offset))   (Gemma: offset 1)
 *   style TBF16_NORM_SCALE_BF16: r[m, k] = bf16_rn(w[k] * bf16_rn(x[m, k] * rs))        (Llama: offset unused)
 * then s_inv and y16 of r as tbf16_glu_rows; r also written to r_out when non-null. With y16 NULL (and
 * r_out given) it is a plain RMSNorm for norms that feed no linear. x bf16 [M, K] (ldx), w bf16 [K]. */
#define TBF16_NORM_SCALE_FP32 0
#define TBF16_NORM_SCALE_BF16 1
int tbf16_rmsnorm_rows(const void* x, int64_t ldx, const void* w, int64_t M, int64_t K, float eps, int style,
                       float offset, int target_exp, void* y16, int64_t ldy, float* s_inv, void* r_out, int64_t ldo,
                       void* stream);

/* The norm with a layer's residual add folded in, each step optional: a = RMSNorm_wa(x) (skipped when wa
 * is NULL), a = bf16_rn(res + a) (skipped when res is NULL), a written to a_out (nullable); then
 * r = RMSNorm_wb(a) (skipped when wb is NULL) with y16 / s_inv / r_out as tbf16_rmsnorm_rows. Both
 * norms use style, offset and eps. Covers x + norm(y) (wa, res, a_out: Gemma's post-norms), the
 * pre-norm rows of a residual sum (res, wb, y16: Llama), and both at once (Gemma's post-attention norm,
 * residual and pre-feed-forward norm in one pass). tbf16_rmsnorm_rows is this call with wb only. All
 * rows [M, K] bf16 (fp16 for y16), strides multiples of 8, pointers 16-byte aligned. */
int tbf16_add_rmsnorm_rows(const void* x, int64_t ldx, const void* res, int64_t ldr, const void* wa, const void* wb,
                           int64_t M, int64_t K, float eps, int style, float offset, int target_exp, void* a_out,
                           int64_t lda, void* y16, int64_t ldy, float* s_inv, void* r_out, int64_t ldo, void* stream);

/* ------------------------------------------------------------------ scaled convolutions */
/* The reference's scaled convolutions (tbf16/conv.py:34-60): one power-of-two scale per input sample,
 * the weight prepared as a linear's rows (tbf16_quantize_rows on [O, C kd kh kw], t = _target_exp(K)):
 *   e[b] = frexp_exp(max |x[b]|) - t (a zero sample counts as max 1), x16 = fp16_rn(x * 2^-e[b]),
 *   y[b, o, p] = bf16_rn((sum_k x16 w16[o, k]) * 2^e[b] * ws[o] + bias[o])   (fp32 sum, one rounding).
 * Geometry: an array of TBF16_CONV_GEOM_LEN int64 in this order: B, C, D, H, W (input extents; 1-D and
 * 2-D convolutions use D = H = 1 or D = 1), the input strides in elements for b, c, d, h, w (any
 * layout), the kernel extents kd, kh, kw, the strides, the zero paddings and the dilations (each d, h,
 * w), and the output extents Do, Ho, Wo. */
#define TBF16_CONV_GEOM_LEN 25

/* Per-sample exponents: x holds B samples of n dense elements, ld elements apart (contiguous or
 * channels-last); writes e[b] and out_scale[b] = 2^e[b] (fp32; B floats of amax_ws as scratch). */
int tbf16_conv_sample_scale(const void* x, int64_t B, int64_t n, int64_t ld, int target_exp, float* amax_ws,
                            int32_t* e, float* out_scale, void* stream);

/* groups == 1: cols16 fp16 [B Do Ho Wo, Kp] (one row per output position, column k = ((c kd + z) kh + y)
 * kw + x as in the weight's [O, C, kd, kh, kw] layout, zero in the padding and for K <= k < Kp) and
 * row_scale[m] = out_scale of the row's sample; then tbf16_gemm_f16(cols16, 0, Kp, w16 [O, Kp], 0, Kp,
 * M, O, Kp, row_scale, ws, bias, y, O) gives y channels-last [B, Do, Ho, Wo, O]. Kp: K rounded up to 8. */
int tbf16_conv_im2col(const void* x, const int64_t* geom, int64_t K, int64_t Kp, const int32_t* e,
                      const float* out_scale, void* cols16, float* row_scale, void* stream);

/* The same for C a multiple of 8, in two passes of 16-byte vectors: x16cl fp16 [B, D, H, W, C]
 * (channels-last, fp16(x * 2^-e[b])), then cols16 [B Do Ho Wo, taps C] with column tap * C + c, tap =
 * (z kh + y) kw + x -- so the weight rows for this path are the weight permuted to [O, kd, kh, kw, C].
 * TBF16_ERR_UNSUPPORTED when C % 8 != 0. */
int tbf16_conv_im2col_cl(const void* x, const int64_t* geom, const int32_t* e, const float* out_scale, void* x16cl,
                         void* cols16, float* row_scale, void* stream);

/* Implicit-GEMM convolution (one group): the whole scaled convolution in one call, without im2col rows.
 * Per-sample amax into amax_ws (B floats, overwritten) and the exponents e / output scales out_scale
 * (B each, as tbf16_conv_sample_scale with this target_exp); x16cl receives the scaled channels-last fp16
 * copy [B, D, H, W, C] (as in tbf16_conv_im2col_cl); the GEMM's TMA then loads each (tap, 64-channel)
 * block of 128 output positions straight from it, the padding as zero fill. wtap16: fp16 [O, taps * C]
 * rows, taps (z, y, x) outer and channels fastest (the rows of the im2col_cl path). y: bf16
 * [B * Do * Ho * Wo, O] (channels-last output, row stride O) =
 * bf16_rn((sum x16cl w16) * out_scale[b] * ws[o] + bias[o]). Replaces the same reference call as the
 * im2col path (tbf16/conv.py:34-60). TBF16_ERR_UNSUPPORTED unless tbf16_conv_implicit_supported says so:
 * C % 64 == 0, O % 8 == 0, stride 1, Wo a power-of-two divisor of 128 or a multiple of 128, and
 * Ho * Wo a multiple of 128 (other convs take the im2col path); also unless each sample of x is one
 * dense block (contiguous or channels-last). */
int tbf16_conv_implicit_supported(const int64_t* geom, int64_t O);
int tbf16_conv_implicit(const void* x, const int64_t* geom, int target_exp, float* amax_ws, int32_t* e,
                        float* out_scale, void* x16cl, const void* wtap16, int64_t O, const float* ws, const void* bias,
                        void* y, void* stream);

/* groups > 1 (grouped and depthwise): direct convolution into y bf16 [B, O, Do, Ho, Wo] contiguous; w16
 * fp16 [O, C / groups, kd, kh, kw] contiguous, ws fp32 [O], bias bf16 [O] nullable. */
int tbf16_conv_grouped(const void* x, const int64_t* geom, int64_t O, int64_t groups, const void* w16, const float* ws,
                       const void* bias, const int32_t* e, const float* out_scale, void* y, void* stream);

/* ------------------------------------------------------------------ scaled attention (tcgen05) */

/* Flash-attention forward on the fp16 copies from tbf16_prepare_qkv. Replaces the torch fp16 SDPA call of
 * the reference's sdpa (tbf16/attention.py:63-65) and the efficient-attention forward of ScaledSDPAFn
 * (tbf16/autograd.py:159-164). q16 (B, Hq, Sq, D), k16 and v16 (B, Hkv, Sk, D), contiguous fp16; GQA by
 * Hq / Hkv. out (B, Hq, Sq, D) bf16 = bf16_rn(softmax(scale * q16 k16^T + mask) v16 * 2^ev[b, h / (Hq/Hkv)]);
 * causal keeps key j <= query i (top-left). mask: optional additive fp16 bias, element (b, h, i, j) at
 * b*mask_sb + h*mask_sh + i*mask_sq + j (strides may be 0 to broadcast). lse (nullable): fp32 (B*Hq, lse_ld)
 * natural-log logsumexp of the scaled, masked logits (the backward wants lse_ld = Sq rounded up to a
 * multiple of 128). o16 (nullable): fp16 (B, Hq, Sq, D) copy of the output before the 2^ev scale (the
 * reference's out16, kept for the backward). D in {64, 128, 256}. */
int tbf16_attn_fwd(const void* q16, const void* k16, const void* v16, int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq,
                   int64_t Sk, int64_t D, float scale, int causal, const int32_t* ev, const void* mask, int64_t mask_sb,
                   int64_t mask_sh, int64_t mask_sq, void* out, float* lse, int64_t lse_ld, void* o16, void* stream);
/* tbf16_attn_fwd with the output's element strides given: out element (b, h, i, d) at
 * b * out_sb + h * out_sh + i * out_ss + d (D contiguous; strides multiples of 8). out_sb = Sq Hq D,
 * out_sh = D, out_ss = Hq D writes (B, Sq, Hq, D) order, the rows the output projection reads, so the
 * transpose + reshape a model does next is free. tbf16_attn_fwd is this call with contiguous strides. */
int tbf16_attn_fwd_out(const void* q16, const void* k16, const void* v16, int64_t B, int64_t Hq, int64_t Hkv,
                       int64_t Sq, int64_t Sk, int64_t D, float scale, int causal, const int32_t* ev, const void* mask,
                       int64_t mask_sb, int64_t mask_sh, int64_t mask_sq, void* out, int64_t out_sb, int64_t out_sh,
                       int64_t out_ss, float* lse, int64_t lse_ld, void* o16, void* stream);

/* Bytes of workspace tbf16_attn_bwd needs (fp32 dQ accumulator, fp16 dO16, delta, head maxima). */
int64_t tbf16_attn_bwd_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D);

/* Flash-attention backward with the reference's per-call power-of-two dO scaling. Replaces the
 * efficient-attention backward of ScaledSDPAFn.backward (tbf16/autograd.py:166-193):
 *   G = t_do - max_{b,h}(head_exp(dout) + ev_q)          (t_do = 12 - ceil(log2 D), minus 8 per retry)
 *   dO16 = fp16(dout * 2^(ev_q + G)); P, dS from q16, k16, v16, lse, delta = rowsum(dO16 * o16)
 *   dq = bf16(dq16 * 2^(a - G)), dk = bf16(dk16 * 2^(-a - G)), dv = bf16(dv16 * 2^(-ev - G))
 * (GQA heads summed in fp32 inside the kernel). q16, k16, v16, o16, lse, a, ev come from
 * tbf16_prepare_qkv (v_exp = 0) and tbf16_attn_fwd; lse_ld must be Sq rounded up to a multiple of 128
 * (each 128-row block of lse is bulk-copied). dout: bf16 (B, Hq, Sq, dout_d) with strides
 * (dout_sb, dout_sh, dout_ss) and contiguous last dim (dout_d <= D; missing columns are zero).
 * dq (B, Hq, Sq, D), dk, dv (B, Hkv, Sk, D): contiguous bf16. G_out: one int32 (device). flag: device
 * word, bit 2 set if any dS or gradient is non-finite (the caller's overflow check). ws: workspace of
 * tbf16_attn_bwd_workspace_size bytes. D in {64, 128, 256}. */
int tbf16_attn_bwd(const void* q16, const void* k16, const void* v16, const void* o16, const float* lse, int64_t lse_ld,
                   const void* dout,
                   int64_t dout_sb, int64_t dout_sh, int64_t dout_ss, int64_t dout_d, const int32_t* a, const int32_t* ev,
                   int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, float scale, int causal,
                   const void* mask, int64_t mask_sb, int64_t mask_sh, int64_t mask_sq, int t_do, void* dq, void* dk,
                   void* dv, int32_t* G_out, unsigned int* flag, void* ws, int64_t ws_bytes, void* stream);

/* Attention dropout, the dropout_p of the reference's ScaledSDPAFn / sdpa (tbf16/autograd.py:159-160,
 * 179-181, passed there to torch's memory-efficient attention): tbf16_attn_fwd_dropout and
 * tbf16_attn_bwd_dropout are tbf16_attn_fwd_out and tbf16_attn_bwd with the softmax weights of dropped
 * (query, key) pairs zeroed for P.V and dV (kept ones scaled by 1 / keep probability; the row sum, lse
 * and delta are those of the undropped softmax, so the output is the unbiased dropout estimate and the
 * gradients are exact for that output). dropout_p in [0, 1); seed selects the mask, which depends only on
 * (seed, batch*head, query, key), so the backward with the same seed sees the forward's mask. The mask is
 * a counter-based hash (murmur3's 32-bit finaliser), not torch's Philox stream: masks differ from the
 * reference's, their distribution does not. tbf16_attn_dropout_keep writes the mask (1 = kept) as bytes
 * [BH, Sq, Sk] for checking. */
int tbf16_attn_fwd_dropout(const void* q16, const void* k16, const void* v16, int64_t B, int64_t Hq, int64_t Hkv,
                           int64_t Sq, int64_t Sk, int64_t D, float scale, int causal, const int32_t* ev,
                           const void* mask, int64_t mask_sb, int64_t mask_sh, int64_t mask_sq, void* out,
                           int64_t out_sb, int64_t out_sh, int64_t out_ss, float* lse, int64_t lse_ld, void* o16,
                           float dropout_p, uint64_t seed, void* stream);
int tbf16_attn_bwd_dropout(const void* q16, const void* k16, const void* v16, const void* o16, const float* lse,
                           int64_t lse_ld, const void* dout, int64_t dout_sb, int64_t dout_sh, int64_t dout_ss,
                           int64_t dout_d, const int32_t* a, const int32_t* ev, int64_t B, int64_t Hq, int64_t Hkv,
                           int64_t Sq, int64_t Sk, int64_t D, float scale, int causal, const void* mask, int64_t mask_sb,
                           int64_t mask_sh, int64_t mask_sq, int t_do, void* dq, void* dk, void* dv, int32_t* G_out,
                           unsigned int* flag, void* ws, int64_t ws_bytes, float dropout_p, uint64_t seed, void* stream);
int tbf16_attn_dropout_keep(uint8_t* keep, int64_t BH, int64_t Sq, int64_t Sk, float dropout_p, uint64_t seed,
                            void* stream);

/* tbf16_attn_fwd_dropout (dropout_p = 0: tbf16_attn_fwd_out) with a device workspace. Head dim 256 with
 * few 256-row query blocks for the device's CTA pairs (one short sequence, few heads: a 2048-token
 * prefill of 8 heads is 64 blocks on 74 pairs) cuts the longest blocks into two parts over their key
 * tiles, run by different pairs and added in fp32 through ws; each part rounds its softmax weights to
 * fp16 against its own running max, so outputs match the plain call's within that rounding, and are the
 * same bits whichever part finishes first. tbf16_attn_fwd_ws_size gives the bytes (0: the plain schedule,
 * ws may be null); a smaller or null ws runs the plain schedule. ws: 16-byte aligned, not shared with a
 * concurrent call. Same replacement as tbf16_attn_fwd (tbf16/attention.py:63-65,
 * tbf16/autograd.py:159-164). */
int64_t tbf16_attn_fwd_ws_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D, int causal);
int tbf16_attn_fwd_ws(const void* q16, const void* k16, const void* v16, int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq,
                      int64_t Sk, int64_t D, float scale, int causal, const int32_t* ev, const void* mask,
                      int64_t mask_sb, int64_t mask_sh, int64_t mask_sq, void* out, int64_t out_sb, int64_t out_sh,
                      int64_t out_ss, float* lse, int64_t lse_ld, void* o16, float dropout_p, uint64_t seed, void* ws,
                      int64_t ws_bytes, void* stream);

/* The backward of one rank's heads in a head-sharded call (no counterpart in the reference, whose
 * ScaledSDPAFn sees every head in one process): tbf16_attn_bwd_dropout with the dO exponent taken as
 * max(this rank's heads, *e_global), where e_global (device int32) is the all_reduce(MAX) over the ranks
 * of max_{b,h}(head_exp(dout) + ev_q) (autograd.py:175 there), so G, and with it every gradient, equals
 * the unsharded call's without a host round trip. dropout_p = 0 for no dropout. */
int tbf16_attn_bwd_sharded(const void* q16, const void* k16, const void* v16, const void* o16, const float* lse,
                           int64_t lse_ld, const void* dout, int64_t dout_sb, int64_t dout_sh, int64_t dout_ss,
                           int64_t dout_d, const int32_t* a, const int32_t* ev, int64_t B, int64_t Hq, int64_t Hkv,
                           int64_t Sq, int64_t Sk, int64_t D, float scale, int causal, const void* mask, int64_t mask_sb,
                           int64_t mask_sh, int64_t mask_sq, int t_do, void* dq, void* dk, void* dv, int32_t* G_out,
                           unsigned int* flag, void* ws, int64_t ws_bytes, float dropout_p, uint64_t seed,
                           const int32_t* e_global, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TBF16_SM100_H */
