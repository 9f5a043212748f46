/*
 * isp_b200.h — C ABI of the B200 (sm_100a) quantized-linear hot path.
 *
 * Plain C: raw device pointers, sizes, host scalars and a CUDA stream.  No
 * function allocates, synchronizes or throws; every one validates shapes,
 * dtypes and alignment on the host before launching and returns an
 * isp_status.  Work is stream-ordered on the caller's stream, so calls can be
 * captured into CUDA graphs.  All matrices are row-major and contiguous.
 *
 * Each entry point names the reference interface it replaces
 * (xiro2416/inspark_proper_format, paths relative to its root).
 *
 * Ordering: the GEMM, convolution and norm-quant kernels use programmatic
 * dependent launch, so a kernel may start while the preceding kernel of this
 * library on the same stream finishes.  Before waiting for it, a GEMM or
 * convolution reads only its weight operand (W / W13 / w_packed and NVFP4 weight
 * scales; for M <= 128 also the per-column w_scale and bias); every activation,
 * activation scale, residual and output (and, for M > 128, w_scale and bias) is
 * touched only after the preceding kernel has completed.  A weight, w_scale or
 * bias must therefore not be the output of the immediately preceding call into
 * this library on the same stream (put any other stream operation, e.g. an event
 * record, in between).
 */
#ifndef ISP_B200_H
#define ISP_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t; 0 is the legacy default stream. */
typedef struct CUstream_st *isp_stream_t;

enum isp_status {
  ISP_OK = 0,
  ISP_ERR_SHAPE = 1,    /* a size is out of the supported range           */
  ISP_ERR_ALIGN = 2,    /* a pointer/row stride breaks a 16-byte rule      */
  ISP_ERR_DTYPE = 3,    /* unsupported dtype combination                   */
  ISP_ERR_ARCH = 4,     /* current device is not sm_100                    */
  ISP_ERR_LAUNCH = 5,   /* the CUDA launch itself failed                   */
  ISP_ERR_TIMEOUT = 6,  /* a bounded device-side wait expired (see below)  */
  ISP_ERR_ARG = 7       /* a required pointer is NULL / bad enum value     */
};

enum isp_dtype {
  ISP_BF16 = 0, ISP_F32 = 1, ISP_F16 = 2, ISP_E4M3 = 3, ISP_I8 = 4, ISP_E2M1 = 5, ISP_I32 = 6
};

/* Row normalization applied before quantization. */
enum isp_norm {
  ISP_NORM_NONE = 0,
  /* gpt_fast RMSNorm: bf16/f32(x*rsqrt(mean(x^2)+eps)) * gamma (FP32)
     models/indextts2/upstream/s2mel/modules/gpt_fast/model.py:246-258 */
  ISP_NORM_RMS_GPTFAST = 1,
  /* Qwen-style RMSNorm: round_to_input_dtype(x*rsqrt(mean(x^2)+eps)*gamma)
     models/indextts2/dspark/draft.py:12-23 */
  ISP_NORM_RMS_QWEN = 2,
  /* Zipformer BiasNorm: round_to_input_dtype(x * mean((x-b)^2)^-1/2 * out_mul)
     models/zipvoice/reference/models/modules/scaling.py:337-370 */
  ISP_NORM_BIAS = 3
};

/* Activation quantization formats. */
enum isp_qfmt {
  /* codes = e4m3_rne(clamp(y / scale, +-448)); build/unified_acoustic_export.py:22-36 */
  ISP_Q_E4M3_STATIC = 0,
  /* s[m] = max(amax_m/448, 1e-12); codes = e4m3(y / s[m]); ops/triton/fp8.py:11-17 */
  ISP_Q_E4M3_ROW = 1,
  /* codes = clamp(rne(y / smooth[k] / scale), -128, 127);
     build/unified_acoustic_export.py:160-162, 27-29 */
  ISP_Q_INT8_STATIC = 2,
  /* NVFP4: 16-element blocks, E4M3 block scale e4m3(amax_b / (6 g)), E2M1
     codes of y / (s_b g) packed low nibble = even k;
     scripts/export_nvfp4_weights.py:25-42 */
  ISP_Q_NVFP4 = 3,
  /* NVFP4 as above, block scales written in the tensor-core layout consumed by
     isp_nvfp4_gemm: 128-row x 4-block chunks of 512 bytes, byte
     ((m/128)*(K/64) + k16/4)*512 + (m%32)*16 + ((m%128)/32)*4 + k16%4
     (scales_out holds ceil(M/128)*128*K/16 bytes; K % 64 == 0). */
  ISP_Q_NVFP4_MMA = 4
};

int isp_version(void);
const char *isp_status_string(int status);

/* Returns ISP_OK when the current CUDA device is a compute capability 10.0
   part the library was built for, ISP_ERR_ARCH otherwise. */
int isp_device_check(void);

/* Device-side error word shared by all kernels with bounded waits.  A wait
   that gives up records ISP_ERR_TIMEOUT there and the kernel returns early.
   Reads (and with clear != 0, resets) the word for the current device;
   synchronizes `stream`. */
int isp_read_device_error(int *error_out, int clear, isp_stream_t stream);

/* Self-test of the bounded-wait path (a library diagnostic; the reference has no
   device-side waits to bound): launches one CTA that holds TMEM, waits on a
   barrier nothing arrives on for limit_ns nanoseconds (1e3 .. 1e8), records
   ISP_ERR_TIMEOUT in the device error word, unwinds its other roles through the
   abort flag and frees TMEM, exactly as a GEMM whose wait expires.  Returns the
   launch status; the timeout is read back with isp_read_device_error. */
int isp_wait_selftest(int64_t limit_ns, isp_stream_t stream);

/*
 * Fused row normalization -> quantization.
 *
 * Replaces: RMSNorm/BiasNorm followed by the separate quantize step of
 *   _QDQ.forward            build/unified_acoustic_export.py:22-36
 *   inspark_custom::fp8_quantize  ops/tensorrt/cfm_gated_up_plugin.py:17-31
 *   _quantize (per-row)     ops/triton/fp8.py:11-17
 *   ExportWeightOp INT8 SmoothQuant input path  build/unified_acoustic_export.py:160-162
 *   NVFP4 dynamic activation quantization  quantization/nvfp4.py:66
 *
 * x:      [M, K] in x_dtype (ISP_BF16 or ISP_F32); K % 16 == 0.
 * gamma:  [K] FP32 (RMS kinds), bias: [K] FP32 (ISP_NORM_BIAS), else NULL.
 * out_mul: exp(log_scale) for ISP_NORM_BIAS (ignored otherwise).
 * scale:  ISP_Q_E4M3_STATIC / ISP_Q_INT8_STATIC: the per-tensor scale;
 *         NVFP4 formats: the FP32 global scale g; ignored for ISP_Q_E4M3_ROW.
 *         Must lie in [2^-100, 2^100] (quotients are then exactly rounded).
 * smooth: [K] FP32 SmoothQuant divisor (ISP_Q_INT8_STATIC) or NULL.
 * codes:  [M, K] uint8/int8 codes, or [M, K/2] packed E2M1 for NVFP4.
 * scales_out: FP32 [M] (ISP_Q_E4M3_ROW), E4M3 [M, K/16] (ISP_Q_NVFP4), the
 *   tensor-core layout (ISP_Q_NVFP4_MMA: ceil(M/128)*128*K/16 bytes, K % 64
 *   == 0; bytes of rows >= M are not written and do not affect rows < M of an
 *   isp_nvfp4_gemm), else NULL.
 */
int isp_norm_quant(const void *x, int x_dtype, int64_t M, int K,
                   const float *gamma, const float *bias, float eps, float out_mul,
                   int norm_kind, int qfmt, float scale, const float *smooth,
                   void *codes, void *scales_out, isp_stream_t stream);

/*
 * gpt_fast AdaptiveLayerNorm fused with the quantizer:
 *   y = ada_w[g] * RMSNorm_gptfast(x) + ada_b[g],   g = row / rows_per_group,
 * multiply and add as separate FP32 roundings, then quantized as isp_norm_quant.
 *
 * Replaces: AdaptiveLayerNorm.forward  models/indextts2/upstream/s2mel/modules/gpt_fast/model.py:18-32
 *   (the DiT's attention/FFN norms) followed by its Q/DQ.
 *
 * ada_w, ada_b: [M / rows_per_group, K] FP32 (the split projection of each
 * utterance's conditioning embedding), 16-byte aligned; M % rows_per_group == 0.
 * Other arguments as isp_norm_quant with norm_kind ISP_NORM_RMS_GPTFAST.
 */
int isp_adaln_quant(const void *x, int x_dtype, int64_t M, int K, const float *gamma, float eps,
                    const float *ada_w, const float *ada_b, int64_t rows_per_group, int qfmt,
                    float scale, const float *smooth, void *codes, void *scales_out,
                    isp_stream_t stream);

/*
 * Reorders E4M3 block scales [R, K/16] (row-major, the ModelOpt storage order
 * of scripts/export_nvfp4_weights.py:38) into the tensor-core layout described
 * at ISP_Q_NVFP4_MMA.  dst must hold ceil(R/128)*128*K/16 bytes; padding rows
 * are written as zero.  K % 64 == 0.
 */
int isp_nvfp4_scales_to_mma(const void *src, int64_t R, int K, void *dst, isp_stream_t stream);

/*
 * Quantized learned convolutions (groups 1, zero padding) as one phase-folded
 * implicit GEMM on tcgen05.  Conv1d (stride S): rows are output times, K runs
 * over (tap, 128 channels) boxes of channels-last codes.  ConvTranspose1d
 * (stride S): output time q * S + r is row q and column co * S + r, and K runs
 * over the window of input rows q + R that any phase reads, so every product of
 * the reference's zero-insertion rewrite and gather kernel is formed once,
 * without the (S - 1) / S zero rows (taps that do not reach a (phase, row)
 * pair are zero weights).  Three calls: pack the weight once, quantize the
 * input, run the convolution.
 *
 * Replaces: ops/triton/fp8_conv.py:24-62 (conv1d, the FP8 MatrixConv path of
 *   ops/matrix.py:21-31 with weights from quantization/precision.py:15-56) and
 *   ExportWeightOp.forward for conv roles (build/unified_acoustic_export.py:
 *   156-216, static FP8 / INT8 SmoothQuant Q/DQ, zero-insertion rewrite).
 */

/* Phases P (1, or the ConvTranspose1d stride) and window slots W of a geometry,
 * for sizing the packed weight [CO * P, W, C_pad].  W <= 128. */
int isp_conv1d_geometry(int KW, int stride, int dilation, int padding, int transposed,
                        int *phases, int *taps);

/*
 * Weight codes [CI * KW, ldw] (E4M3 or INT8 bytes; row ci * KW + tap, column
 * co: the packed [K, N] layout of quantization/weights.py:5-17, whose per-
 * output-channel scales are used unchanged; for ConvTranspose1d the rows come
 * from weight.permute(1, 0, 2) as in quantization/precision.py:34-36) ->
 * w_packed [CO * P, W, C_pad], zero past CI and where no tap reaches.
 * ldw >= CO; C_pad % 128 == 0, C_pad >= CI; w_packed 16-byte aligned.
 */
int isp_conv1d_pack_weight(const void *codes, int64_t ldw, int CO, int CI, int KW, int stride,
                           int dilation, int padding, int transposed, void *w_packed, int C_pad,
                           isp_stream_t stream);

/*
 * Input quantization: x [B, C, T] (x_dtype ISP_F32 or ISP_BF16, channels first)
 * -> channels-last codes xq [B, T_rows, C_pad], T_rows = T rounded up to a
 * multiple of row_multiple (the Conv1d stride; 1 for ConvTranspose1d), rows >= T
 * and channels >= C coded 0.
 *   static scale (amax == NULL, in_scale > 0): E4M3 e4m3(clamp(x / in_scale)),
 *     INT8 rne(x / smooth[c] / in_scale) saturated (smooth may be NULL);
 *   dynamic per-utterance scale (amax != NULL, in_scale == 0, E4M3 only): the
 *     call writes amax[b] = max |x[b]| and codes x / max(amax[b] / 448, 1e-12)
 *     (ops/triton/fp8_conv.py:6-22); pass the same amax to isp_conv1d.
 */
int isp_conv1d_quant(const void *x, int x_dtype, int64_t B, int C, int64_t T, int row_multiple,
                     const float *smooth, float in_scale, float *amax, int code_dtype, void *xq,
                     int C_pad, isp_stream_t stream);

/*
 * y[b, co, t] = acc * s_in * w_scale[co] + bias[co] with acc the exact-product,
 * FP32-accumulated sum over (tap, ci) of xq codes times weight codes, s_in =
 * in_scale (static) or max(amax[b] / 448, 1e-12) (dynamic).  T_out must equal
 * (T_in + 2 padding - dilation (KW - 1) - 1) / stride + 1 (Conv1d) or
 * (T_in - 1) stride - 2 padding + dilation (KW - 1) + output_padding + 1
 * (ConvTranspose1d).  xq from isp_conv1d_quant with the same geometry; ab_dtype
 * ISP_E4M3 or ISP_I8; y [B, CO, T_out] in ISP_F32, ISP_BF16 or ISP_F16.
 */
int isp_conv1d(const void *xq, int ab_dtype, int64_t B, int C_pad, int64_t T_in, const void *w_packed,
               int CO, int KW, int stride, int dilation, int padding, int output_padding,
               int transposed, int64_t T_out, float in_scale, const float *amax,
               const float *w_scale, const float *bias, void *y, int out_dtype, isp_stream_t stream);

/*
 * BigVGAN anti-aliased Snake activation: 2x 12-tap polyphase upsample with
 * replicate padding, Snake v + inv_beta[c] * sin(alpha[c] v)^2, 12-tap
 * stride-2 replicate-padded low-pass, fused in one pass over x.
 *
 * Replaces: Activation1d  models/indextts2/upstream/s2mel/modules/bigvgan/alias_free_activation/torch/act.py:16-21
 *   FusedAliasFree         ops/triton/alias_free.py:28-43 (_up_snake + _down)
 *   inspark_custom::small_fir_activation[_tiled]  ops/tensorrt/vocoder_tiled_fir_plugin.py:11-36
 *   inspark_custom::small_fir_activation_quantized  deployment/multibatch/fir_quant_plugin.py:11-26
 *
 * x: [rows, T] FP32 with rows = B*C and channel = row % C; 16-byte aligned
 *    (rows with T % 4 == 0 are streamed by bulk async copies).
 * up, down: 12 FP32 taps each, in HOST memory (model constants; they are
 *   passed by value to the kernel so every FMA reads them from the constant
 *   bank).  alpha, inv_beta: [C] FP32 on the device (linear alpha;
 *   inv_beta = 1/(beta + 1e-9)).
 * out_dtype ISP_F32: y [rows, T] FP32.
 * out_dtype ISP_I8: y = clamp(rint((v / smooth[c]) / scale), -128, 127) int8.
 */
int isp_fir_snake(const float *x, int64_t rows, int C, int64_t T,
                  const float *up, const float *down, const float *alpha, const float *inv_beta,
                  void *y, int out_dtype, const float *smooth, float scale, isp_stream_t stream);

/*
 * W8A8 scaled GEMM on tcgen05 tensor cores: out = epilogue(A[M,K] . W[N,K]^T).
 *
 * Replaces: _gemm/_reduce   ops/triton/fp8.py:19-45 (and ops.matrix.linear)
 *   FP8Linear.forward       runtime/zipvoice_fp8/quantization.py:75-82
 *   FusedProjectionResidual ops/tensorrt/zipvoice_fp8_b128/b128/residual_kernel.py:4-11
 *   i8_residual             ops/tensorrt/zipvoice/a1007/b1/i8_residual_runtime_kernel.py:5-21
 *   TRT native FP8 / INT8 GEMMs under explicit Q/DQ
 *
 * ab_dtype: ISP_E4M3 (FP32 accumulate) or ISP_I8 (exact int32 accumulate).
 * K % 16 == 0, N % 16 == 0, A/W 16-byte aligned.
 * v = ((acc * a_s[m]) * w_scale[n]) + bias[n] + residual[m, n], where a_s is
 *   a_scale_rows[m] when given, else the scalar a_scale; w_scale NULL means 1.
 * out: out_dtype ISP_BF16 / ISP_F16 / ISP_F32 value, or ISP_E4M3 codes of
 *   clamp(v * out_inv_scale, +-448) (next-layer static requant by the
 *   reciprocal scale, as the residual plugin's `Inv`).
 * out2 (optional): E4M3 codes of clamp(v * out2_inv_scale, +-448) — the
 *   second output of the residual plugin.  residual: [M, N] in residual_dtype
 *   (ISP_F32 or ISP_BF16) or NULL.
 */
int isp_scaled_gemm(const void *A, const void *W, int ab_dtype, int64_t M, int N, int K,
                    float a_scale, const float *a_scale_rows, const float *w_scale,
                    const float *bias, const void *residual, int residual_dtype,
                    void *out, int out_dtype, float out_inv_scale, void *out2, float out2_inv_scale,
                    isp_stream_t stream);

/*
 * CFM gated-up: h = silu(A.W1^T * s1[n]) * (A.W3^T * s3[n]), then static E4M3
 * requant q = e4m3(clamp(h * (1/out_scale), +-448)).
 *
 * Replaces: _paired / GatedUp  ops/triton/cfm_gated_up.py:7-51
 *   inspark_custom::fp8_gated_up  ops/tensorrt/cfm_gated_up_plugin.py:33-49
 *   _interleaved / fp8_gated_up_interleaved  ops/triton/cfm_interleaved.py:19-55,
 *                                            ops/tensorrt/cfm_interleaved_plugin.py:15-41
 *
 * interleaved == 0: W1, W3 are [N, K] E4M3 and s1, s3 [N] FP32.
 * interleaved != 0: W1 is [2N, K] with row 2n = gate n, row 2n+1 = up n;
 *   s1 is [2N]; W3 and s3 must be NULL.
 * out_dtype ISP_E4M3: codes [M, N]; ISP_F32: q * out_scale (DEQUANT=True).
 */
int isp_gated_up(const void *A, const void *W1, const void *W3, int interleaved,
                 int64_t M, int N, int K, const float *s1, const float *s3,
                 float out_scale, void *out, int out_dtype, isp_stream_t stream);

/*
 * INT8 nonlinear-value projection: three INT8 GEMMs sharing one activation,
 *   z_j[m, n] = acc_j[m, n] * (a_scale * w_scale[jN + n]) + bias[jN + n],
 *   acc_j = sum_k Q[m, k] * W[jN + n, k] (exact int32), j = 0, 1, 2,
 * stored as value = tanhf(z0) * z1 and gate = z2 (every step one FP32 rounding,
 * in the reference's order; tanhf is CUDA's, the function libdevice.tanh calls).
 *
 * Replaces: int8_nonlinear_value (Triton, TensorRT plugin
 *   zipvoice_int8_b*::OriginalInt8NonlinearValue*)
 *   ops/tensorrt/zipvoice/a1007/b1/int8_nonlinear_value_runtime_kernel.py:6-34,
 *   ops/tensorrt/zipvoice/a1007/b1/int8_nonlinear_value_plugin.py:7-35
 *
 * Q: [M, K] int8 codes, rows m = t * groups + b (the plugin's [T, B, K]).
 * W: [3N, K] int8 (the three projections stacked, the exported [1152, 512]).
 * w_scale, bias: [3N] FP32; a_scale > 0 (the per-tensor input scale AS).
 * value: [groups, M / groups, N] FP32 (row (b, t) = input row t * groups + b);
 * gate: [M, N] FP32.  N % 16 == 0, K % 16 == 0, M % groups == 0; every pointer
 * 16-byte aligned.
 */
int isp_int8_nonlinear_value(const void *Q, const void *W, int64_t M, int N, int K, int groups,
                             float a_scale, const float *w_scale, const float *bias,
                             float *value, float *gate, isp_stream_t stream);

/*
 * NVFP4 block-scaled GEMM on tcgen05 tensor cores (kind::mxf4nvf4, 16-element
 * K blocks, E4M3 block scales):
 *   v[m, n] = alpha * sum_k (e2m1(A[m,k]) sa[m,k/16]) (e2m1(W[n,k]) sw[n,k/16])
 *             + bias[n] + residual[m, n]
 * with alpha = activation global scale * weight global scale.
 *
 * Replaces: MatrixWeightOp.forward with the ModelOpt NVFP4 quantizers applied
 *   (build/nvfp4_graph.py:73-87, installed by quantization/nvfp4.py:11-56),
 *   i.e. TensorRT's native FP4 GEMM behind NVFP4 Q/DQ.
 *
 * A: [M, K/2] packed E2M1 (low nibble = even k); A_sf: A's block scales in
 *   the tensor-core layout (ISP_Q_NVFP4_MMA, as written by isp_norm_quant).
 * W: [N, K/2] packed E2M1; W_sf: the weight's scales in the same layout
 *   (isp_nvfp4_scales_to_mma of the exporter's [N, K/16] block_scale).
 * K % 64 == 0, N % 8 == 0; A, W, A_sf, W_sf, out 16-byte aligned.
 * out: [M, N] in out_dtype (ISP_BF16, ISP_F16 or ISP_F32).  bias: [N] FP32 or
 *   NULL; residual: [M, N] ISP_F32 / ISP_BF16 or NULL.
 */
int isp_nvfp4_gemm(const void *A, const void *A_sf, const void *W, const void *W_sf,
                   int64_t M, int N, int K, float alpha, const float *bias,
                   const void *residual, int residual_dtype, void *out, int out_dtype,
                   isp_stream_t stream);

/*
 * NVFP4 CFM gated-up: gate = alpha_gate * (A . W1^T), up = alpha_up * (A . W3^T),
 * h = silu(gate) * up, requantized to NVFP4 with the FP32 global scale h_scale
 * (the down projection's calibrated activation global scale):
 *   s_b = e4m3(min(amax_b / (6 h_scale), 448)) (an all-zero block: 1),
 *   code = e2m1(h / (s_b h_scale)).
 *
 * Replaces: FeedForward.forward w1/w3/silu (gpt_fast/model.py:235-244) under the
 *   NVFP4 recipe (quantization/nvfp4.py:58-68): two native FP4 GEMMs, the
 *   SiLU-gate, and the dynamic block quantization of the w2 input.
 *
 * A, A_sf: as isp_nvfp4_gemm (K % 64 == 0).
 * W13: [2N, K/2] packed E2M1, gate and up rows stacked in blocks of 64:
 *   rows [128 j, 128 j + 64) = W1 rows [64 j, 64 j + 64), rows
 *   [128 j + 64, 128 j + 128) = W3 rows [64 j, 64 j + 64); W13_sf: its scales in
 *   the tensor-core layout.  N % 64 == 0.
 * h_codes: [M, N/2] packed E2M1; h_sf: ceil(M/128)*128*N/16 bytes, the
 *   tensor-core layout of an [M, N] operand (feeds isp_nvfp4_gemm directly).
 * h_scale must lie in [2^-100, 2^100].
 */
int isp_nvfp4_gated_up(const void *A, const void *A_sf, const void *W13, const void *W13_sf,
                       int64_t M, int N, int K, float alpha_gate, float alpha_up, float h_scale,
                       void *h_codes, void *h_sf, isp_stream_t stream);

/*
 * No reference counterpart: an addition of this library for callers that cannot
 * allocate device memory at call time -- an inference-engine plugin whose enqueue
 * receives only pre-sized buffers, or a streaming audio worker that keeps the
 * allocator (and its locks) off its per-chunk path.
 *
 * The dynamic-scale FP8 convolution (isp_conv1d_quant with amax != NULL, then
 * isp_conv1d) in one call, with the per-utterance maxima kept in a static device
 * array inside the library instead of a caller buffer.  xq is still the caller's
 * [B, T_rows, C_pad] code buffer (sized as for isp_conv1d_quant); every other
 * argument as isp_conv1d.
 *   - B <= 8192 (ISP_ERR_SHAPE beyond); the call allocates nothing.  The array is
 *     8192 floats (32 KB), held by every GPU that loads the library until exit.
 *   - The first call on each device resolves the array's address on that device
 *     (device must be current); make that first call before any stream capture.
 *     The address is cached per device: after cudaDeviceReset the library must be
 *     reloaded before this entry point is called again.
 *   - The maxima are cleared at the start of each call.  One array per process and
 *     device: calls that overlap in time (other streams, other threads) race on it
 *     and must be serialized by the caller.
 */
int isp_conv1d_dynamic_noalloc(const void *x, int x_dtype, int64_t B, int C, int64_t T, void *xq,
                               int C_pad, const void *w_packed, int CO, int KW, int stride,
                               int dilation, int padding, int output_padding, int transposed,
                               int64_t T_out, const float *w_scale, const float *bias, void *y,
                               int out_dtype, isp_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* ISP_B200_H */
