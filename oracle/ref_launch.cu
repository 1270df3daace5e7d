// Host launchers for the REFERENCE quantizer kernels -- checker build only.
//
// This translation unit contains no kernel code of its own.  oracle/build_ref.py
// extracts the reference's NVRTC kernel source strings from float4utils.py
// (``_KERNEL_NVFP4_FUSED`` float4utils.py:62-150 and
// ``_KERNEL_RMSNORM_NVFP4_SMEM`` float4utils.py:152-297) into a temporary file
// and force-includes it here with ``nvcc -include``; the result goes only to
// oracle/_ref/ (git-ignored).  The launch geometry below is the reference
// wrappers' (float4utils.py:350-355 and :384-399).  It exists so that golden
// vectors can be produced by the reference's own kernels, to pin the numpy
// oracle; nothing in the product links it.
#include <cuda_runtime.h>

#if defined(REF_QUANT)
extern "C" int ref_quant_nvfp4(const void* x_bf16, void* q_u8, void* s_u8,
                               int num_blocks16, int cols, int pad_cols,
                               void* stream) {
  const int threads = 256;
  const int grid = (num_blocks16 + threads - 1) / threads;
  if (grid == 0) return 0;
  quant_nvfp4_fused_opt<<<grid, threads, 0, (cudaStream_t)stream>>>(
      (const unsigned short*)x_bf16, (unsigned char*)q_u8, (unsigned char*)s_u8,
      num_blocks16, cols, pad_cols);
  return (int)cudaGetLastError();
}
#elif defined(REF_RMSNORM)
extern "C" int ref_rmsnorm_quant_nvfp4(const void* x_bf16, void* q_u8, void* s_u8,
                                       float* inv_rms, int R, int K, int pad_cols,
                                       float epsilon, void* stream) {
  const int threads = 256;
  const int smem = K * 2;
  if (R == 0) return 0;
  cudaError_t e = cudaFuncSetAttribute(rmsnorm_quant_nvfp4_smem_opt,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, 98304);
  if (e != cudaSuccess) return (int)e;
  rmsnorm_quant_nvfp4_smem_opt<<<R, threads, smem, (cudaStream_t)stream>>>(
      (const unsigned short*)x_bf16, (unsigned char*)q_u8, (unsigned char*)s_u8,
      inv_rms, R, K, pad_cols, epsilon);
  return (int)cudaGetLastError();
}
#else
#error "define REF_QUANT or REF_RMSNORM"
#endif
