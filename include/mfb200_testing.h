/* mfb200_testing.h -- single-kernel entry points of libmfb200 used by the unit
 * tests. They have no counterpart in the reference (which has per-kernel
 * GPU-vs-host smoke checks inside its CUDA backend,
 * src/nn/cuda/cuda_kernels.cu:1872-3197); each call allocates its own device
 * buffers and is not meant for production use. Returns 0 on success. */
#ifndef MFB200_TESTING_H
#define MFB200_TESTING_H
#include <stdint.h>
#ifndef MFB200_API
#define MFB200_API __attribute__((visibility("default")))
#endif
#ifdef __cplusplus
extern "C" {
#endif

/* out[M,N] (bf16 bits) = epilogue(A[M,K] . W[N,K]^T) through the tcgen05 GEMM.
 * A/W are bf16 bits (fp8 = 0) or e4m3 bytes (fp8 = 1); resid is fp32; out is
 * fp32 when out_f32 = 1, else bf16 bits. mode: 0 store
 * act(scale*acc+bias), 1 resid + alpha*(scale*acc+bias), 2 row LayerNorm of
 * act(scale*acc+bias) (N == bn). */
MFB200_API int mfb200_debug_gemm(int M, int N, int K, int bn, int fp8, const void *A, const void *W,
                      const float *bias, int mode, int act, const float *resid, float alpha,
                      const float *ln_gamma, const float *ln_beta, float ln_eps,
                      const float *col_scale, float a_scale, int out_f32, void *out,
                      unsigned *status_out);

#ifdef __cplusplus
}
#endif
#endif
