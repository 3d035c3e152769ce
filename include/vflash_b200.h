/*
 * vflash_b200 — C ABI of the B200 (sm_100a) quantised-linear hot path.
 *
 * Every entry point is stream-ordered, allocates nothing (the caller owns
 * every buffer) and returns 0 on success or a VFB_E* code; the message of the
 * last failure on the calling host thread is available from vfb_last_error().
 * Pointers are CUDA device pointers of the current device unless stated.
 * Row strides ("ld*") are in elements.  `stream` is a cudaStream_t (0 = the
 * legacy default stream).  Shapes are validated before any launch; nothing is
 * retried and there is no fallback arithmetic.
 *
 * The reference interfaces these replace live in Hansimov/vflash
 * (paths relative to its repository root):
 *   src/vflash/native/h3_fp8_activation.py   quantize_activation / _rows_fp8
 *   src/vflash/native/h3_fp8_linear.py       RowFP8Execution.linear (w8a8)
 *   src/vflash/native/h3_nvfp4_linear.py     NVFP4Execution.linear
 *   src/vflash/native/h3_fused_ops.py        triton_strict_bf16_* epilogues
 */
#ifndef VFLASH_B200_H
#define VFLASH_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VFB_API __attribute__((visibility("default")))
#else
#define VFB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define VFB_OK 0
#define VFB_EINVAL 1      /* shape, stride, alignment or pointer rejected   */
#define VFB_ECUDA 2       /* a CUDA runtime call failed                     */
#define VFB_EDEVICE 3     /* current device is not compute capability 10.0  */
#define VFB_ETIMEOUT 4    /* a kernel's bounded wait expired (device flag)  */

/* Message of the last error raised on this host thread ("" if none). */
VFB_API const char *vfb_last_error(void);

/* Library version string, e.g. "vflash_b200 0.1.0 sm_100a". */
VFB_API const char *vfb_version(void);

/* Read (and optionally clear) the device-side status word of the current
 * device.  Kernels whose bounded waits expire record VFB_ETIMEOUT there and
 * return instead of hanging.  Synchronises the device. */
VFB_API int vfb_device_status(int *status, int clear);

/* Bounded-wait self-test: launches one thread that waits on a barrier nothing
 * completes; the wait gives up after timeout_ns (1 ms .. 10 s), records
 * VFB_ETIMEOUT in the device status word (read it with vfb_device_status) and
 * the kernel ends normally, leaving the context usable.  No reference
 * counterpart: it exercises the failure path every pipeline wait of the GEMMs
 * takes (their limit is 4 s) without stalling a real kernel. */
VFB_API int vfb_wait_selftest(int64_t timeout_ns, void *stream);

/* ---- FP8 per-token activation quantisation -------------------------------
 * Replaces quantize_activation / _rows_fp8
 * (src/vflash/native/h3_fp8_activation.py:13-55) and the portable expression
 * _quantize_activation_torch (src/vflash/native/h3_fp8_linear.py:18-31):
 *   amax   = max_k |x[m,k]|                       (fp32)
 *   scale  = amax > 0 ? max(amax / 448, FLT_MIN) : 1   (IEEE division)
 *   codes  = e4m3_rn(clamp(x / scale, -448, 448))      (IEEE division)
 * x: bf16 [M,K] with row stride ldx >= K.  codes: e4m3 [M_pad,K] contiguous,
 * scales: fp32 [M_pad].  Rows M..M_pad-1 get codes 0 and scale 1.
 * Requires 1 <= K <= 32768 and M_pad >= M. */
VFB_API int vfb_fp8_quant_rows(const void *x, int64_t M, int64_t K, int64_t ldx,
                       void *codes, float *scales, int64_t M_pad,
                       void *stream);

/* Row maxima only: amax[m] = max_k |x[m,k]| (NaN for a row holding a NaN).
 * With vfb_fp8_quant_rows_amax this quantises a row that is split over several
 * ranks (tensor parallelism) exactly as the unsplit row: each rank takes its
 * slice's maxima, the ranks combine them with a MAX all-reduce, and each
 * quantises its slice with the full row's maxima.  No reference counterpart:
 * the reference's tensor-parallel block (src/vflash/native/h3_parallel.py:
 * 220-250) runs in BF16 and never quantises a split row. */
VFB_API int vfb_fp8_row_absmax(const void *x, int64_t M, int64_t K, int64_t ldx, float *amax,
                               void *stream);

/* vfb_fp8_quant_rows with the row maxima given (amax[M], device) instead of
 * computed: scale = amax > 0 ? max(amax / 448, FLT_MIN) : 1 (1 for NaN). */
VFB_API int vfb_fp8_quant_rows_amax(const void *x, int64_t M, int64_t K, int64_t ldx,
                                    const float *amax, void *codes, float *scales, int64_t M_pad,
                                    void *stream);

/* RMSNorm + AdaLN modulate + per-token e4m3 quantisation of the result, in
 * one pass.  Replaces the sequence the reference block runs before its QKV and
 * FFN-input projections (src/vflash/native/h3_native_denoiser.py:534-541 and
 * 561-568): _rms_norm (231-243, torch's fused rms_norm: fp32 upcast,
 * rsqrt(mean(x^2) + eps), (x * rstd) * w rounded once to bf16), then
 * triton_strict_bf16_modulate (src/vflash/native/h3_fused_ops.py:52-122,
 * 575-611: bf16(bf16(n * bf16(1 + scale)) + shift)), then the quantiser above
 * applied to the modulated rows.
 * x: bf16 [M,K], row stride ldx; norm_weight: bf16 [K] or NULL (no weight);
 * scale / shift: bf16 [tokens, K] with row strides *_token_stride (0 = one
 * row for all tokens), row r uses row r % tokens.  Outputs as
 * vfb_fp8_quant_rows.  Requires K % 8 == 0, 8 <= K <= 32768, 16-byte aligned
 * rows of x, weight, scale and shift, 8-byte aligned codes, eps >= 0.  rstd
 * is accumulated in fp32 in this kernel's order and rounded from fp64, so it
 * may differ from torch's by one fp32 ulp. */
VFB_API int vfb_fp8_norm_modulate_quant(const void *x, int64_t M, int64_t K, int64_t ldx,
                                        const void *norm_weight, float eps, const void *scale,
                                        int64_t scale_token_stride, const void *shift,
                                        int64_t shift_token_stride, int64_t tokens, void *codes,
                                        float *scales, int64_t M_pad, void *stream);

/* ---- FP8 row-scaled GEMM with fused epilogues ----------------------------
 * Replaces torch._scaled_mm(codes, weight.t(), scale_a, scale_b.t(),
 * out_dtype=bf16) plus the following bias add
 * (src/vflash/native/h3_fp8_linear.py:109-121) and, per epilogue kind, the
 * separate strict-BF16 elementwise launch that follows the linear:
 *   y[m,n] = bf16( sa[m] * sw[n] * sum_k A[m,k] W[n,k] )     (fp32 accumulate)
 *   y      = bf16( y + bias[n] )                    if bias != NULL
 * then the epilogue `kind`:
 *   VFB_EPI_STORE     out = y, optionally merged with three LoRA branches
 *                     (triton_strict_bf16_qkv_direct_merge,
 *                     src/vflash/native/h3_fused_ops.py:901-979):
 *                     out = bf16(y + bf16(adapter_p[m,c] * scaling[p]))
 *   VFB_EPI_GELU_TANH out = bf16(gelu_tanh(y))
 *   VFB_EPI_SWIGLU    out[m,j] = bf16(v * bf16(silu(g))) with v = y[m,j] and
 *                     g = y[m,F+j] (triton_strict_bf16_silu_mul,
 *                     src/vflash/native/h3_fused_ops.py:185-224,660-700);
 *                     N is the packed width 2F, the output is [M,F]
 *   VFB_EPI_RESIDUAL  out = bf16(residual + bf16(gate[t,n] * y)) with
 *                     t = m % tokens, or bf16(residual + y) when gate == NULL
 *                     (triton_strict_bf16_gate_residual,
 *                     src/vflash/native/h3_fused_ops.py:125-170,614-657)
 *   VFB_EPI_QKV_NORM_ROPE  STORE into three planes (Q, K, V; adapters as
 *                     STORE), then on every 128-column head of the Q and K
 *                     planes the block's QK-norm and rotary embedding
 *                     (_qk_norm_rotary, src/vflash/native/h3_native_denoiser.py:
 *                     409-419): n = bf16((q * rstd) * norm_w) with rstd =
 *                     rsqrt(mean(q^2) + qk_eps) over the head (fp32 sum, rounded
 *                     from fp64), then out = bf16(bf16(n * cos[t,d]) +
 *                     bf16(partner * sin[t,d])), partner = -n[d+64] for d < 64,
 *                     n[d-64] otherwise (triton_strict_bf16_rotary,
 *                     src/vflash/native/h3_fused_ops.py:421-510), t = m % tokens;
 *                     rotary over the whole head (cos/sin [tokens, 128]).
 * Output column n of a STORE/GELU/RESIDUAL epilogue goes to plane
 * p = n / plane_width (plane_width = 0: one plane of width N) at
 *   out + p * plane_stride + m * ldo + (n % plane_width),
 * which writes the Q, K and V planes of a merged projection directly.
 * wire_chunks = c > 0 (STORE or QKV_NORM_ROPE with three planes) stores the
 * planes instead in the destination-major wire layout of pack_qkv
 * (src/vflash/native/h3_parallel_relayout.py:214-256): each plane's columns
 * are split into 2c groups of W = plane_width / (2c) columns (W % 32 == 0),
 * group g = d * c + k (destination d in {0, 1}, chunk k) of plane p going to
 * slab s = (k * 2 + d) * 3 + p at
 *   out + s * plane_stride + m * ldo + (n % W),
 * i.e. out is [c][2][3][M][W] with ldo = W and plane_stride = M * W.
 * A: e4m3 [M rows, K] with row stride lda bytes (multiple of 16); sa: [>=M].
 * W: e4m3 [N,K] row-major with row stride ldw bytes (multiple of 16);
 * sw: [N].  K % 16 == 0.  N % 32 == 0 (SWIGLU: F % 32 == 0).
 * ---------------------------------------------------------------------- */
#define VFB_EPI_STORE 0
#define VFB_EPI_GELU_TANH 1
#define VFB_EPI_SWIGLU 2
#define VFB_EPI_RESIDUAL 3
#define VFB_EPI_QKV_NORM_ROPE 4

typedef struct vfb_epilogue {
  int32_t kind;              /* VFB_EPI_*                                   */
  int32_t wire_chunks;       /* 0, or chunks of the pack_qkv wire layout    */
  void *out;                 /* bf16 output                                 */
  int64_t ldo;               /* output row stride (elements)                */
  int64_t plane_width;       /* 0 or a multiple of 32 dividing N            */
  int64_t plane_stride;      /* elements between output planes              */
  const void *bias;          /* bf16 [N] or NULL                            */
  /* STORE: optional LoRA branches, one per plane (NULL = none)             */
  const void *adapter[3];    /* bf16 [M, plane_width], row stride adapter_ld*/
  int64_t adapter_ld;
  float scaling[3];
  int32_t reserved1;
  /* RESIDUAL                                                               */
  const void *residual;      /* bf16 [M, N], row stride ldr                 */
  int64_t ldr;
  const void *gate;          /* bf16 [tokens, N] strided, or NULL           */
  int64_t gate_token_stride; /* elements                                    */
  int64_t gate_hidden_stride;/* elements                                    */
  int64_t tokens;            /* gate / rotary row = m % tokens              */
  /* QKV_NORM_ROPE (head_dim 128, rotary over the whole head)               */
  const void *q_norm;        /* bf16 [128] or NULL (no weight)              */
  const void *k_norm;        /* bf16 [128] or NULL                          */
  const void *rope_cos;      /* bf16 [tokens, 128], row stride rope_token_stride */
  const void *rope_sin;      /* bf16 [tokens, 128], same stride             */
  int64_t rope_token_stride; /* elements, multiple of 8                     */
  float qk_eps;              /* > 0                                         */
  int32_t reserved2;
} vfb_epilogue;

VFB_API int vfb_fp8_gemm(const void *A, int64_t lda, const float *sa,
                 const void *W, int64_t ldw, const float *sw,
                 int64_t M, int64_t N, int64_t K,
                 const vfb_epilogue *ep, void *stream);

/* Low-rank adapter products: out = bf16(A @ W^T), bf16
 * operands, fp32 accumulation on the same CTA-pair tensor-core pipeline
 * (tcgen05.mma kind::f16).  Replaces the two functional.linear calls of
 * _residual_linear_unscaled (src/vflash/native/h3_native_denoiser.py:288-299):
 * the down product states @ down^T ([M, r]; the three QKV branches' downs
 * concatenated into one [3r, H] weight) and the up product low @ up^T
 * ([M, inner]), whose result the STORE adapters of vfb_fp8_gemm then scale and
 * merge.  A: bf16 [M, K] with row stride lda ELEMENTS; W: bf16 [N, K], row
 * stride ldw elements; K % 8 == 0, strides multiples of 8, 16-byte aligned
 * bases; N % 8 == 0.  ep: kind VFB_EPI_STORE with out, ldo (elements,
 * multiple of 8, >= N) and nothing else: one plane, no bias, no adapters, no
 * wire layout (the reference's low-rank linears have no bias). */
VFB_API int vfb_bf16_gemm(const void *A, int64_t lda, const void *W, int64_t ldw,
                  int64_t M, int64_t N, int64_t K, const vfb_epilogue *ep, void *stream);

/* Fused FP8 FFN in one call: replaces the FFN input and output linears of
 * the H3 block (src/vflash/native/h3_native_denoiser.py:561-576) with the
 * reference's per-token activation quantiser before each
 * (h3_fp8_linear.py:92-121):
 *   vfb_fp8_quant_rows(x)
 *   -> up GEMM with the activation epilogue (VFB_EPI_GELU_TANH with w_up
 *      [F, H], or VFB_EPI_SWIGLU with the packed w_up [2F, H]; bias_up)
 *   -> per-token e4m3 requantisation of the bf16 intermediate [M, F] over
 *      its full row (the quantiser's arithmetic, h3_fp8_activation.py:16-19)
 *   -> down GEMM (w_down [H, F]; bias_down; RESIDUAL with residual [M, H]
 *      (row stride ldr) and optional gate [tokens, H] (row stride
 *      gate_token_stride), else STORE) into out [M, H] (row stride ldo).
 * The same bits as vfb_fp8_gemm / vfb_fp8_quant_rows called step by step,
 * which is how it runs: three launches after the input quantiser, the
 * fastest order measured on the B200 at the benchmark's size (see
 * vfb_fp8_ffn_one_kernel).  x: bf16 [M, H], row stride ldx; s_up [n_up], s_down
 * [H] fp32.  H and F multiples of 32, at most 32768.  The intermediates live
 * in `workspace` (256-byte aligned, at least vfb_fp8_ffn_workspace_bytes(M,
 * H, F) bytes, F = intermediate width); the call allocates nothing.
 * vfb_fp8_ffn_workspace_bytes returns -1 for an invalid shape. */
VFB_API int64_t vfb_fp8_ffn_workspace_bytes(int64_t M, int64_t H, int64_t F);
VFB_API int vfb_fp8_ffn(const void *x, int64_t M, int64_t H, int64_t ldx,
                const void *w_up, const float *s_up, int64_t n_up,
                const void *w_down, const float *s_down, int32_t activation,
                const void *bias_up, const void *bias_down,
                const void *residual, int64_t ldr,
                const void *gate, int64_t gate_token_stride, int64_t tokens,
                void *out, int64_t ldo, void *workspace, int64_t workspace_bytes, void *stream);

/* vfb_fp8_ffn with the up GEMM, the requantisation and the down GEMM in ONE
 * persistent kernel (same arguments, same bits), for F % 256 == 0 (GELU) or
 * F % 128 == 0 (SwiGLU); other widths run the three launches.  No reference
 * counterpart: the reference runs the FFN's linears and its quantiser as
 * separate launches.  CTA pairs take up and down tiles from one counter in
 * row-block groups; each up tile's epilogue stores its bf16 tile (L2
 * evict_last) and merges its rows' maxima, and once a row block's up tiles
 * are all done the warps that stored it requantise it to e4m3 and drop the
 * bf16 lines from L2; the row block's down tiles then read the codes.  The
 * bf16 intermediate stays in L2 only while a group's intermediate fits next
 * to the weight tiles in use.  Measured on the B200 at H 4096, F 16384
 * (GELU), this path is slower than vfb_fp8_ffn at every M from 512 to 32760
 * (1.4-1.7x at M <= 2048, 1.35x at 32760): the down tiles wait for their
 * row blocks' conversion and the up epilogue carries the conversion work. */
VFB_API int vfb_fp8_ffn_one_kernel(const void *x, int64_t M, int64_t H, int64_t ldx,
                const void *w_up, const float *s_up, int64_t n_up,
                const void *w_down, const float *s_down, int32_t activation,
                const void *bias_up, const void *bias_down,
                const void *residual, int64_t ldr,
                const void *gate, int64_t gate_token_stride, int64_t tokens,
                void *out, int64_t ldo, void *workspace, int64_t workspace_bytes, void *stream);

/* vfb_fp8_ffn on an input that is already quantised per token: x_codes e4m3
 * [M, H] (row stride H, 16-byte aligned), x_scales fp32 [>= M], e.g. the
 * output of vfb_fp8_norm_modulate_quant (the block's RMSNorm + AdaLN
 * modulate fused into the quantiser).  Everything else as vfb_fp8_ffn. */
VFB_API int vfb_fp8_ffn_quantized(const void *x_codes, const float *x_scales, int64_t M, int64_t H,
                const void *w_up, const float *s_up, int64_t n_up,
                const void *w_down, const float *s_down, int32_t activation,
                const void *bias_up, const void *bias_down,
                const void *residual, int64_t ldr,
                const void *gate, int64_t gate_token_stride, int64_t tokens,
                void *out, int64_t ldo, void *workspace, int64_t workspace_bytes, void *stream);

/* vfb_fp8_ffn for callers that cannot allocate device memory: a process that
 * embeds this library in a runtime which has already reserved the GPU's
 * memory for its own pool, or code that runs where cudaMalloc's implicit
 * synchronisation is not allowed.  This entry point has no counterpart in
 * the reference.  Same arguments and result as vfb_fp8_ffn without the
 * workspace: the intermediates live in a fixed 64 MiB array of device memory
 * owned by the library, which every GPU that loads the library holds until
 * the process exits.  Shapes whose intermediates need more
 * (vfb_fp8_ffn_workspace_bytes(M, H, F) > 64 MiB) are rejected with
 * VFB_EINVAL.  The first call on a device looks the array's address up
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * A cudaDeviceReset gives the device a new context in which the array has a
 * new address: the first call after it looks the address up again (the
 * library keeps each cached address with the id of its context), so that
 * call, too, belongs before any capture.
 * All calls on a device share the array: calls whose kernels may overlap on
 * the GPU (other streams, unordered host threads) race, so order them. */
VFB_API int vfb_fp8_ffn_noalloc(const void *x, int64_t M, int64_t H, int64_t ldx,
                const void *w_up, const float *s_up, int64_t n_up,
                const void *w_down, const float *s_down, int32_t activation,
                const void *bias_up, const void *bias_down,
                const void *residual, int64_t ldr,
                const void *gate, int64_t gate_token_stride, int64_t tokens,
                void *out, int64_t ldo, void *stream);

/* ---- NVFP4 ----------------------------------------------------------------
 * Activation quantiser: replaces FlashInfer nvfp4_quantize(x, global_scale,
 * sfLayout=128x4, do_shuffle=False) as NVFP4Execution.linear calls it
 * (src/vflash/native/h3_nvfp4_linear.py:102).  x: [M,K] bf16 (dtype 0) or fp16
 * (dtype 1), row stride ldx; global_scale: device fp32 scalar (gsf).  Per 16
 * elements: sf = e4m3(gsf * amax / 6), codes = e2m1(x / (sf / gsf)) with the
 * reference's rcp.approx.ftz arithmetic.  codes: [M, K/2] bytes (element 2i in
 * the low nibble); sf: ceil128(M) * ceil4(K/16) bytes in the 128x4 layout,
 * padding written as 0.  K % 16 == 0. */
VFB_API int vfb_nvfp4_quant_rows(const void *x, int32_t dtype, int64_t M, int64_t K, int64_t ldx,
                                 const float *global_scale, void *codes, void *sf, void *stream);

/* RMSNorm + AdaLN modulate + NVFP4 quantisation in one pass: the codes and
 * scales vfb_nvfp4_quant_rows would give for the bf16 tensor
 *   bf16(bf16(rms_norm(x) * bf16(1 + scale[t])) + shift[t]),  t = row % tokens,
 * computed exactly as vfb_fp8_norm_modulate_quant computes it (rms_norm:
 * src/vflash/native/h3_native_denoiser.py:231-243 with the norm weight
 * norm_weight [K] or none; modulate: h3_fused_ops.py:52-122), so the block's
 * norm and modulate before an NVFP4 linear cost one HBM pass.  x bf16 [M, K]
 * (row stride ldx), scale / shift bf16 rows of K (token strides in
 * elements, 0 for one row), global_scale the linear's input_scale (device
 * fp32 scalar); codes [M, K/2], sf ceil128(M) * K/16 bytes (128x4, padding
 * rows 0).  K % 64 == 0, K <= 32768; rows and weights 16-byte aligned. */
VFB_API int vfb_nvfp4_norm_modulate_quant(const void *x, int64_t M, int64_t K, int64_t ldx,
                                          const void *norm_weight, float eps, const void *scale,
                                          int64_t scale_token_stride, const void *shift,
                                          int64_t shift_token_stride, int64_t tokens,
                                          const float *global_scale, void *codes, void *sf, void *stream);

/* Block-scaled GEMM: replaces FlashInfer mm_fp4(codes, packed.T, scales,
 * weight_scales.T, alpha, bf16, backend="cutlass") and the bias add
 * (src/vflash/native/h3_nvfp4_linear.py:118-139):
 *   out = bf16(alpha * sum_k A(m,k) W(n,k)) [then bf16(out + bias)]
 * A: [M, K/2] codes with scales sfa (128x4 layout, ceil128(M) rows); W: the
 * NVFP4Weight packed [N, K/2] codes and scales [N, K/16] (128x4 layout).
 * alpha: device fp32 scalar.  out: bf16 [planes, M, N/planes] contiguous
 * (planes = 1: [M, N]).  K % 64 == 0, N % 128 == 0. */
VFB_API int vfb_nvfp4_gemm(const void *A, const void *sfa, const void *W, const void *sfw,
                           const float *alpha, int64_t M, int64_t N, int64_t K, const void *bias,
                           void *out, int64_t planes, void *stream);

/* vfb_nvfp4_gemm with the fused epilogues of vfb_fp8_gemm, for the QAD visual
 * linears (src/vflash/adapters/h3_qad.py:206-218) whose outputs go through
 * the same strict-BF16 steps as the FP8 block's:
 *   y = bf16(alpha * sum_k A(m,k) W(n,k)), alpha = alpha[0] / alpha_div[0]
 *       (one IEEE fp32 division on the device, as NVFP4Execution.linear's
 *       weight.alpha / weight.input_scale, h3_nvfp4_linear.py:124-125;
 *       alpha_div NULL: alpha[0] as is)
 *   y = bf16(y + bias[n])  if ep->bias != NULL   (h3_nvfp4_linear.py:139)
 * then ep->kind as for vfb_fp8_gemm: VFB_EPI_STORE (planes via plane_width /
 * plane_stride / ldo, optional LoRA branches merged per plane:
 * triton_strict_bf16_qkv_direct_merge), VFB_EPI_GELU_TANH, VFB_EPI_SWIGLU
 * (packed W [2F, K/2] with F % 128 == 0: value rows first, their scales the
 * first F/128 blocks of the 128x4 layout; out [M, F]) or VFB_EPI_RESIDUAL
 * (gate optional).  No wire layout and no QK-norm epilogue.  Operands as
 * vfb_nvfp4_gemm; K % 64 == 0, N % 128 == 0. */
VFB_API int vfb_nvfp4_gemm_ex(const void *A, const void *sfa, const void *W, const void *sfw,
                              const float *alpha, const float *alpha_div, int64_t M, int64_t N, int64_t K,
                              const vfb_epilogue *ep, void *stream);

/* vfb_nvfp4_gemm_ex whose result leaves the kernel quantised for the next
 * NVFP4 linear instead of as bf16: the bf16 values the epilogue would store
 * (VFB_EPI_STORE with one plane and no adapters, VFB_EPI_GELU_TANH or
 * VFB_EPI_SWIGLU) are quantised as vfb_nvfp4_quant_rows(values,
 * out_global_scale) would quantise them, bit for bit: out_codes e2m1
 * [M, W/2] (contiguous) and out_sf 128x4 scales for ceil128(M) rows and W/16
 * groups (padding rows 0), W = N (SWIGLU: N/2), W % 64 == 0.  ep->out, ldo,
 * plane_width and plane_stride are not used.  No reference counterpart: the
 * reference stores the bf16 activation output and the next
 * NVFP4Execution.linear quantises it again (h3_nvfp4_linear.py:102), so the
 * intermediate of a QAD FFN round-trips HBM in bf16 and costs a quantiser
 * launch; here it stays as codes. */
VFB_API int vfb_nvfp4_gemm_quant(const void *A, const void *sfa, const void *W, const void *sfw,
                                 const float *alpha, const float *alpha_div, int64_t M, int64_t N,
                                 int64_t K, const vfb_epilogue *ep, const float *out_global_scale,
                                 void *out_codes, void *out_sf, void *stream);

/* ---- strict-BF16 elementwise steps -----------------------------------------
 * Standalone versions of the epilogues above, for callers whose GEMM is not
 * this library's.  bf16 tensors; the last dimension is contiguous and its
 * width a multiple of 8; other strides as stated.  Rounding boundaries follow
 * the reference kernels in src/vflash/native/h3_fused_ops.py (line ranges
 * given per entry point).  `out` may not alias inputs unless stated. */

/* triton_strict_bf16_silu_mul (h3_fused_ops.py:185-224, 660-700):
 * packed [rows, 2*width] -> out[r, c] = bf16(v * bf16(silu(g))), v = packed[r, c],
 * g = packed[r, width + c]; out row stride out_ld (out may be the value half
 * of packed itself, out_ld = 2*width). */
VFB_API int vfb_silu_mul(const void *packed, int64_t rows, int64_t width, void *out,
                         int64_t out_ld, void *stream);

/* triton_strict_bf16_ffn_adapter_silu (h3_fused_ops.py:254-284, 703-762):
 * base/adapter [rows, 2*width]; value and gate halves each merged as
 * bf16(b + bf16(a * scaling)), then out = bf16(value * bf16(silu(gate))).
 * out row stride out_ld; out may be the value half of base (reuse_base). */
VFB_API int vfb_ffn_adapter_silu(const void *base, const void *adapter, int64_t rows,
                                 int64_t width, float scaling, void *out, int64_t out_ld,
                                 void *stream);

/* triton_strict_bf16_gate_residual (h3_fused_ops.py:125-170, 614-657):
 * residual/projected [rows, hidden] contiguous (rows = batch * tokens),
 * gate [tokens, hidden] with row stride gate_token_stride:
 * out = bf16(residual + bf16(gate[r % tokens] * projected)). */
VFB_API int vfb_gate_residual(const void *residual, const void *gate, int64_t gate_token_stride,
                              const void *projected, int64_t rows, int64_t tokens,
                              int64_t hidden, void *out, void *stream);

/* triton_strict_bf16_modulate (h3_fused_ops.py:52-122, 575-611):
 * value [rows, hidden] contiguous (rows = batch * tokens), scale / shift
 * [tokens, hidden] with row strides scale_token_stride / shift_token_stride:
 * out = bf16(bf16(value * bf16(1 + scale[r % tokens])) + shift[r % tokens]). */
VFB_API int vfb_modulate(const void *value, const void *scale, int64_t scale_token_stride,
                         const void *shift, int64_t shift_token_stride, int64_t rows,
                         int64_t tokens, int64_t hidden, void *out, void *stream);

/* triton_strict_bf16_rotary (h3_fused_ops.py:421-510, 1031-1085), split-half
 * RoPE on value [rows, heads, head_dim] contiguous (rows = batch * tokens) with
 * cos / sin [tokens, rotary_dim] (row strides *_token_stride, unit column
 * stride): for d < rotary_dim,
 *   out[d] = bf16(bf16(x[d] * cos[d]) + bf16(partner[d] * sin[d])),
 *   partner[d] = d < rotary_dim/2 ? -x[d + rotary_dim/2] : x[d - rotary_dim/2];
 * out[d] = x[d] for d >= rotary_dim.  rotary_dim even, <= head_dim. */
VFB_API int vfb_rotary(const void *value, const void *cos, int64_t cos_token_stride, const void *sin,
                       int64_t sin_token_stride, int64_t rows, int64_t tokens, int64_t heads,
                       int64_t head_dim, int64_t rotary_dim, void *out, void *stream);

/* triton_strict_bf16_adapter_gate_residual (h3_fused_ops.py:342-415, 982-1028):
 * out = bf16(residual + bf16(gate * bf16(base + bf16(adapter * scaling)))). */
VFB_API int vfb_adapter_gate_residual(const void *base, const void *adapter, const void *residual,
                                      const void *gate, int64_t gate_token_stride, int64_t rows,
                                      int64_t tokens, int64_t hidden, float scaling, void *out,
                                      void *stream);

/* triton_strict_bf16_adapter_merge / _qkv_adapter_merge (h3_fused_ops.py:298-339,
 * 765-838): base/adapter [rows, width], `branches` (1..3) equal column
 * branches: out = bf16(base + bf16(adapter * scalings[branch])). */
VFB_API int vfb_adapter_merge(const void *base, const void *adapter, int64_t rows, int64_t width,
                              int32_t branches, const float *scalings, void *out, void *stream);

/* triton_strict_bf16_qkv_direct_merge (h3_fused_ops.py:901-979), in place:
 * base [rows, 3*width]; base[:, b*width:(b+1)*width] =
 * bf16(base_b + bf16(adapter_b * scalings[b])) for b = q, k, v.
 * `scalings` is a host pointer to three floats. */
VFB_API int vfb_qkv_direct_merge(void *base, const void *adapter_q, const void *adapter_k,
                                 const void *adapter_v, int64_t rows, int64_t width,
                                 const float *scalings, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* VFLASH_B200_H */
