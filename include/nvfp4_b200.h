/*
 * nvfp4_b200.h -- C ABI of the B200 (sm_100a) NVFP4 hot path.
 *
 * Plain C: raw device pointers, 64-bit sizes, a cudaStream_t passed as void*,
 * an int status return.  No allocation happens behind any entry point unless
 * its comment says so; all work is enqueued asynchronously on `stream`.
 * Device pointers must stay valid until the work on `stream` completes.
 *
 * Data formats (identical to the reference, float4utils.py / cutlass_mm_fp4.cu):
 *   - bf16 inputs: row-major, 16-byte aligned base.
 *   - packed E2M1 ("q"): [rows, k/2] bytes, element 2j in the low nibble
 *     (float4utils.py:141).
 *   - E4M3 block scales ("s"): one byte per 1x16 block along k, stored in the
 *     128x4-atom swizzled layout of [round_up(rows,128), round_up(k/16,4)]
 *     bytes: byte offset of block (r, c) is
 *       ((r/128)*(pad_cols/4) + c/4)*512 + (r%32)*16 + ((r%128)/32)*4 + c%4
 *     (float4utils.py:118-122).  Padding is written as 0 by the quantizers.
 *   - optional per-tensor global scale g (device float*): block scale =
 *     e4m3((amax_blk/6)/g), dequantised value = e2m1 * e4m3 * g.  NULL means
 *     g = 1, which is bit-identical to the reference quantizer.
 */
#ifndef NVFP4_B200_H
#define NVFP4_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NVFP4B200_API_VERSION 4

enum nvfp4b200_status {
  NVFP4B200_OK = 0,
  NVFP4B200_ERR_INVALID_ARG = 1,      /* NULL pointer where one is required, bad enum   */
  NVFP4B200_ERR_BAD_SHAPE = 2,        /* size constraint violated (see each function)   */
  NVFP4B200_ERR_MISALIGNED = 3,       /* pointer not aligned as documented               */
  NVFP4B200_ERR_UNSUPPORTED_DEVICE = 4, /* current device is not compute capability 10.0 */
  NVFP4B200_ERR_LAUNCH = 5,           /* the kernel launch failed                        */
  NVFP4B200_ERR_TIMEOUT = 6,          /* a bounded device-side wait gave up              */
  NVFP4B200_ERR_CUDA = 7              /* another CUDA runtime/driver call failed         */
};

enum nvfp4b200_dtype { NVFP4B200_BF16 = 0, NVFP4B200_F32 = 1 };
enum nvfp4b200_epilogue { NVFP4B200_EPI_NONE = 0, NVFP4B200_EPI_RELU = 1, NVFP4B200_EPI_RELU2 = 2 };

/* Library / device information. */
int nvfp4b200_api_version(void);
const char* nvfp4b200_status_string(int status);
/* NVFP4B200_OK when the current CUDA device can run this library. */
int nvfp4b200_device_check(void);
/* Reads and clears the device-side error word that bounded waits set when
 * they give up (synchronises the current device).  *out = 0 when none. */
int nvfp4b200_get_device_error(int* out);

/* Caps the number of SMs the persistent GEMM kernel occupies on every device
 * (0 = all SMs, the default; values are rounded down to whole CTA pairs,
 * minimum one pair).  Process-wide.  A data-parallel training step lowers it
 * so that collective kernels (NCCL all-reduce of the gradient buckets) find
 * free SMs while GEMMs run, instead of waiting for them to finish.  No
 * counterpart in the reference (its GEMM is a library call).  Returns
 * NVFP4B200_ERR_INVALID_ARG for negative values. */
int nvfp4b200_set_gemm_max_sms(int max_sms);

/* Failure-path self-test (no reference counterpart): one warp runs the GEMM
 * pipeline's bounded mbarrier wait on a barrier that nothing arrives on.
 * After limit_cycles SM cycles (1 .. 2^32) the wait gives up, the kernel
 * records NVFP4B200_ERR_TIMEOUT in the device error word (read and cleared by
 * nvfp4b200_get_device_error) and returns; the context stays usable. */
int nvfp4b200_wait_selftest(int64_t limit_cycles, void* stream);

/* Gate/up GEMM with the SwiGLU activation in its epilogue (new: the MLP
 * forward; no counterpart in the reference).  b: [n, k/2] packed, whose rows
 * interleave gate and up weights in blocks of 128 (rows 256 t .. 256 t + 127
 * are gate rows 128 t.., the next 128 the matching up rows); n % 256 == 0.
 * h: bf16 [m, n/2], h[:, 128 t + j] = silu(gate_j) * up_j computed from the
 * bf16-rounded gate/up values (the product scale_a * scale_b applied first).
 * gu: bf16 [m, n] gate/up values in b's row order, or NULL (not stored).
 * ws (2 x u32, zero on entry, left zero) with h_global_scale_out: device
 * global scale of h, amax(|h|)/(6*448) (1 when the amax is 0 or not finite),
 * or both NULL. */
int nvfp4b200_gemm_swiglu(const void* a, const void* b, const void* sfa, const void* sfb, const float* scale_a,
                          const float* scale_b, void* h, void* gu, uint32_t* ws, float* h_global_scale_out,
                          int64_t m, int64_t n, int64_t k, void* stream);

/* dh GEMM with the SwiGLU backward in its epilogue (new: the MLP backward; no
 * counterpart in the reference).  The product dh = scale_a * scale_b * (A . B^T)
 * ([m, n]) is rounded to bf16 and never stored; gu: bf16 [m, 2n] gate/up
 * values interleaved in blocks of 128 (nvfp4b200_gemm_swiglu's layout);
 * dgu: bf16 [m, 2n] in the same layout, exactly nvfp4b200_swiglu_bwd(gu, dh,
 * interleave = 128).  n % 256 == 0.  ws (2 x u32, zero on entry, left zero)
 * with dgu_global_scale_out: device global scale of dgu, or both NULL. */
int nvfp4b200_gemm_dswiglu(const void* a, const void* b, const void* sfa, const void* sfb, const float* scale_a,
                           const float* scale_b, const void* gu, void* dgu, uint32_t* ws,
                           float* dgu_global_scale_out, int64_t m, int64_t n, int64_t k, void* stream);

/* ------------------------------------------------------------------------ */
/* Quantizers                                                               */
/* ------------------------------------------------------------------------ */

/* quant_nvfp4_fused (float4utils.py:327-357, kernel :79-148).
 * x: bf16 [rows, k]; q: u8 [rows, k/2]; s: u8 swizzled [round_up(rows,128),
 * round_up(k/16,4)] (every byte written, padding = 0).  k % 16 == 0.
 * global_scale: device float or NULL (g = 1: reference-exact). */
int nvfp4b200_quant_nvfp4(const void* x, void* q, void* s, int64_t rows, int64_t k,
                          const float* global_scale, void* stream);

/* Quantize y = (x * row_scale[r]) * gamma[c] along k, with both factors
 * optional (NULL); row_scale is fp32 [rows], gamma bf16 [k].  With both NULL
 * this is nvfp4b200_quant_nvfp4; with row_scale = 1/RMS it is the second
 * phase of the reference's fused RMSNorm kernel (float4utils.py:233-294). */
int nvfp4b200_scaled_quant_nvfp4(const void* x, const float* row_scale, const void* gamma,
                                 void* q, void* s, int64_t rows, int64_t k,
                                 const float* global_scale, void* stream);

/* rmsnorm_quant_nvfp4_fused (float4utils.py:359-401, kernel :169-295):
 * inv_rms[r] = rsqrtf(sum(x^2)/k + eps), then y = (x * inv_rms) [* gamma]
 * quantized as above.  gamma (bf16 [k]) is optional (NULL = reference).
 * k % 16 == 0.  Rows up to 8192 wide are read once (held in registers);
 * wider rows take a 1/RMS pass and a second read. */
int nvfp4b200_rmsnorm_quant_nvfp4(const void* x, const void* gamma, void* q, void* s,
                                  float* inv_rms, int64_t rows, int64_t k, float eps,
                                  const float* global_scale, void* stream);

/* Row statistics for the global-scale RMSNorm path (no reference
 * counterpart): inv_rms as above, and the global scale of the normalised
 * tensor y = (x*inv_rms)*gamma: *global_scale_out = amax(|y|)/(6*448)
 * (1.0 when that amax is 0 or not finite).  `ws` is a caller-owned device
 * workspace of 2 uint32 that must be zero before the first call; every call
 * leaves it zero again.  Calls sharing one `ws` must not overlap.
 * k % 16 == 0 and k <= 16384.  The sum of squares is not reduced in the
 * reference kernel's order (this path has none), so inv_rms may differ from
 * nvfp4b200_rmsnorm_quant_nvfp4's by about one ulp. */
int nvfp4b200_rmsnorm_stats(const void* x, const void* gamma, float* inv_rms,
                            int64_t rows, int64_t k, float eps,
                            uint32_t* ws, float* global_scale_out, void* stream);

/* Transposed quantize (no reference counterpart; the NVFP4 backward needs
 * operands blocked along the other dimension): y = ((x*row_scale[r])*gamma[c])^T,
 * x bf16 [rows, cols] -> q u8 [cols, rows/2] and s swizzled for (cols, rows).
 * rows % 16 == 0, cols % 2 == 0; row_scale / gamma optional. */
int nvfp4b200_quant_nvfp4_t(const void* x, const float* row_scale, const void* gamma,
                            void* q, void* s, int64_t rows, int64_t cols,
                            const float* global_scale, void* stream);

/* Global scale of a bf16 tensor of n elements: *global_scale_out =
 * amax(|x|)/(6*448), NaN ignored, 1.0 when the amax is 0 or not finite.
 * If amax_out is non-NULL it receives the amax.  `ws` as for
 * nvfp4b200_rmsnorm_stats. */
int nvfp4b200_global_scale(const void* x, int64_t n, uint32_t* ws, float* global_scale_out,
                           float* amax_out, void* stream);

/* Same result as nvfp4b200_global_scale, for callers that cannot allocate
 * device memory (an arena or pool that owns all device memory, a plugin host
 * that hands over only the call's tensors, or code that must not call
 * cudaMalloc/cudaFree because those may synchronise the device).  No
 * counterpart in the reference.  Allocates nothing: its scratch is a fixed
 * ~16 KB array inside the library's device memory, held by every GPU that
 * loads the library until the process exits.  Limit: n <= 2^30 elements
 * (larger n returns NVFP4B200_ERR_BAD_SHAPE).  Every call looks up the
 * array's device address in the current context, so a cudaDeviceReset
 * between calls is safe; the first call on a device may load the library's
 * device code for that device (make it before any stream capture).  All
 * calls share the array: calls that overlap on the GPU race. */
int nvfp4b200_global_scale_noalloc(const void* x, int64_t n, float* global_scale_out, float* amax_out,
                                   void* stream);

/* ------------------------------------------------------------------------ */
/* Block-scaled GEMM (tcgen05.mma kind::mxf4nvf4)                           */
/* ------------------------------------------------------------------------ */

/* gn_kernels::cutlass_sm120a_nvfp4_mm (cutlass_mm_fp4.cu:167-272):
 *   d = bf16(output_scale * (A . B^T) + bias)
 * a: packed [m, k/2]; b: packed [n, k/2] (the reference's column-major B,
 * i.e. b.mT of a row-major [n, k/2]); sfa / sfb: swizzled scales of A and B;
 * output_scale: device float (NULL = 1); bias: bf16 [n] or NULL;
 * d: bf16 [m, n] row-major.  Constraints: k % 32 == 0, n % 8 == 0, all
 * pointers 16-byte aligned. */
/* gn_kernels::cutlass_sm120a_mxfp4_mm (cutlass_mm_fp4.cu:71-165): MXFP4
 *   d = bf16(A . B^T + bias)
 * with E2M1 operands and one UE8M0 scale (2^(e-127)) per 1x32 block along k.
 * a: packed [m, k/2]; b: packed [n, k/2]; sfa / sfb: the 128x4-atom swizzled
 * layout with one column per 32 k, i.e. [round_up(rows, 128),
 * round_up(k/32, 4)] bytes; padding entries must not be 0xFF (NaN).
 * bias: bf16 [n] or NULL; d: bf16 [m, n].  k % 32 == 0, n % 8 == 0, all
 * pointers 16-byte aligned. */
int nvfp4b200_mxfp4_mm(const void* a, const void* b, const void* sfa, const void* sfb, const void* bias, void* d,
                       int64_t m, int64_t n, int64_t k, void* stream);

int nvfp4b200_nvfp4_mm(const void* a, const void* b, const void* sfa, const void* sfb,
                       const float* output_scale, const void* bias, void* d,
                       int64_t m, int64_t n, int64_t k, void* stream);
/* gn_kernels::cutlass_sm120a_nvfp4_mm_relu (cutlass_mm_fp4.cu:274-374):
 * d = bf16(relu(output_scale * (A . B^T) + bias)). */
int nvfp4b200_nvfp4_mm_relu(const void* a, const void* b, const void* sfa, const void* sfb,
                            const float* output_scale, const void* bias, void* d,
                            int64_t m, int64_t n, int64_t k, void* stream);
/* gn_kernels::cutlass_sm120a_nvfp4_mm_relu_2 (cutlass_mm_fp4.cu:377-477):
 * d = bf16(relu(output_scale * (A . B^T) + bias)^2). */
int nvfp4b200_nvfp4_mm_relu_2(const void* a, const void* b, const void* sfa, const void* sfb,
                              const float* output_scale, const void* bias, void* d,
                              int64_t m, int64_t n, int64_t k, void* stream);

/* General form used by the training step (no reference counterpart):
 * alpha = (scale_a ? *scale_a : 1) * (scale_b ? *scale_b : 1);
 * v = epilogue(alpha * (A . B^T) + bias) + residual; d_dtype BF16 stores
 * bf16(v), F32 stores v, or adds v into d when accumulate != 0 (F32 only).
 * d and residual (bf16, optional) are [m, n] with row stride ldd elements
 * (ldd >= n, ldd % 8 == 0). */
int nvfp4b200_gemm(const void* a, const void* b, const void* sfa, const void* sfb,
                   const float* scale_a, const float* scale_b, const void* bias,
                   const void* residual, void* d, int d_dtype, int accumulate, int epilogue,
                   int64_t m, int64_t n, int64_t k, int64_t ldd, void* stream);

/* ------------------------------------------------------------------------ */
/* Training-step element-wise kernels (no reference counterpart: the        */
/* reference's backward is bf16, float4utils.py:653-683)                     */
/* ------------------------------------------------------------------------ */

/* h = silu(gate) * up with gu bf16 [tokens, 2*ff], h bf16 [tokens, ff].
 * interleave = 0: each gu row is [gate | up]; interleave = 128: gate and up
 * alternate in blocks of 128 columns (the layout nvfp4b200_gemm_swiglu
 * writes; ff % 128 == 0).  If ws and global_scale_out are non-NULL, also
 * writes the global scale of h (as nvfp4b200_global_scale). */
int nvfp4b200_swiglu_fwd(const void* gu, void* h, int64_t tokens, int64_t ff, int interleave,
                         uint32_t* ws, float* global_scale_out, void* stream);

/* d(gate), d(up) of the above given dh bf16 [tokens, ff] -> dgu bf16
 * [tokens, 2*ff] in gu's layout.  Optional global scale of dgu as above. */
int nvfp4b200_swiglu_bwd(const void* gu, const void* dh, void* dgu, int64_t tokens, int64_t ff, int interleave,
                         uint32_t* ws, float* global_scale_out, void* stream);

/* RMSNorm backward for y = (x*inv_rms)*gamma given dy bf16 [rows, k]:
 * dx = inv_rms*(dy*gamma - xn*mean(dy*gamma*xn)) [+ dres], written bf16;
 * dgamma_acc (fp32 [k]) += sum_r dy*xn.  dres / dgamma_acc optional. */
int nvfp4b200_rmsnorm_bwd(const void* x, const void* gamma, const float* inv_rms,
                          const void* dy, const void* dres, void* dx, float* dgamma_acc,
                          int64_t rows, int64_t k, void* stream);

/* Element-wise y = a + b over n bf16 elements (residual add). */
int nvfp4b200_add_bf16(const void* a, const void* b, void* y, int64_t n, void* stream);

/* AdamW on a bf16 parameter with fp32 moments (no master copy):
 * g = grad * grad_scale (grad bf16 or fp32 per grad_dtype);
 * m = b1*m + (1-b1)*g; v = b2*v + (1-b2)*(g*g);
 * p = p - lr*((m/bc1)/(sqrt(v/bc2)+eps) + wd*p), rounded to bf16.
 * Every operation is rounded once in this order.  An update below half a
 * bf16 ulp of p is lost; nvfp4b200_adamw_master_step keeps it. */
int nvfp4b200_adamw_step(void* param, const void* grad, int grad_dtype, float* m, float* v,
                         int64_t n, float lr, float beta1, float beta2, float eps,
                         float weight_decay, float bias_corr1, float bias_corr2,
                         float grad_scale, void* stream);

/* AdamW with an fp32 master copy of a bf16 parameter (no counterpart in the
 * reference, which trains with torch's optimizers): master, m and v are fp32
 * [n]; param (bf16 [n]) is overwritten with bf16(master) after the update.
 * The order of operations is torch.optim.AdamW's, each rounded once:
 *   g = grad * grad_scale;  w = w * one_minus_lr_wd;
 *   m = m + one_minus_beta1 * (g - m);  v = beta2*v + one_minus_beta2*(g*g);
 *   w = w - step_size * (m / (sqrt(v)/bias_corr2_sqrt + eps))
 * with one_minus_lr_wd = 1 - lr*wd, step_size = lr / (1 - beta1^t) and
 * bias_corr2_sqrt = sqrt(1 - beta2^t) computed by the caller.  Updates below
 * half a bf16 ulp of the parameter accumulate in the master instead of
 * being rounded away.  amax_bits (device uint32, optional): the largest
 * |bf16 parameter| written by this call, as float bits, combined into
 * *amax_bits with an atomic max (zero it before the first call; NaN is
 * ignored).  It lets the weights' global scale for the next quantization be
 * taken from the update itself instead of another pass over the weights. */
int nvfp4b200_adamw_master_step(void* param, float* master, const void* grad, int grad_dtype, float* m, float* v,
                                int64_t n, float one_minus_lr_wd, float one_minus_beta1, float beta2,
                                float one_minus_beta2, float eps, float step_size, float bias_corr2_sqrt,
                                float grad_scale, uint32_t* amax_bits, void* stream);

/* Global scales from amaxes (no reference counterpart): for i < n,
 * global_scale_out[i] = amax_i/(6*448), amax_i = float bits amax_bits[i],
 * and 1.0 when that amax is 0 or not finite -- exactly what
 * nvfp4b200_global_scale computes from the tensor.  n <= 2^20. */
int nvfp4b200_global_scale_from_amax(const uint32_t* amax_bits, float* global_scale_out, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_B200_H */
