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

/* Allow (1, the default) or forbid (0) the CTA-pair GEMM kernel in GEMMs
 * planned afterwards (tests run both kernels). */
MFB200_API void mfb200_debug_set_gemm_pairs(int enable);

/* Run the bf16 encoder of forwards planned afterwards with (1, the default)
 * or without (0) the deferred LayerNorm: residual GEMMs that store the
 * un-normalised stream with row statistics and consumer GEMMs that fold the
 * normalisation into their epilogue, instead of separate ln1 / ln2 passes. */
MFB200_API void mfb200_debug_set_fold_ln(int enable);

/* Split K (1, the default) or not (0) in the GEMMs of forwards planned
 * afterwards whose output tiles would occupy at most half of the SMs (small
 * batches): fp32 partial products, then one reduction + epilogue kernel. */
MFB200_API void mfb200_debug_set_auto_split(int enable);

/* Launch the kernels of forwards planned afterwards with (1, the default) or
 * without (0) programmatic dependent launch. */
MFB200_API void mfb200_debug_set_pdl(int enable);

/* out[M,N] (bf16 bits) = epilogue(A[M,K] . W[N,K]^T) through the tcgen05 GEMM.
 * A/W are bf16 bits (fp8 = 0), e4m3 bytes (fp8 = 1) or fp16 bits (fp8 = 2); resid is fp32; out is
 * fp32 when out_f32 = 1, fp16 bits when out_f32 = 2, else bf16 bits. mode: 0
 * store act(scale*acc+bias), 1 resid + alpha*(scale*acc+bias), 3 the same
 * computed in place (the output buffer starts as resid, rounded to the output
 * format, and the GEMM adds alpha*(scale*acc+bias) into it). k_splits > 1: split-K,
 * `out` receives k_splits fp32 partial products [k_splits, M, N] (no bias).
 * ln_gamma/ln_beta/ln_eps are unused. */
MFB200_API int mfb200_debug_gemm(int M, int N, int K, int bn, int fp8, const void *A, const void *W,
                      const float *bias, int mode, int act, const float *resid, float alpha,
                      const float *ln_gamma, const float *ln_beta, float ln_eps,
                      const float *col_scale, float a_scale, int out_f32, int k_splits, void *out,
                      unsigned *status_out);

/* Residual + LayerNorm GEMM: y = resid + alpha*(A.W^T + bias) (A, W bf16
 * bits, resid fp32), out_f32 = LN(y)*gamma + beta and out_bf16 = the same in
 * bf16; N must be bn times a cluster size of 1, 2, 4 or 8. */
MFB200_API int mfb200_debug_gemm_ln(int M, int N, int K, int bn, const void *A, const void *W,
                                    const float *bias, const float *resid, float alpha,
                                    const float *gamma, const float *beta, float eps,
                                    float *out_f32, uint16_t *out_bf16, unsigned *status_out);

/* Mean device time (ms) of `iters` back-to-back launches of one GEMM on
 * pseudo-random device operands (for profiling the kernel in isolation); mode and
 * out_f32 as for mfb200_debug_gemm (mode 2: residual + LayerNorm); dtype 0 bf16,
 * 1 e4m3, 2 fp16 operands. */
MFB200_API int mfb200_debug_gemm_bench(int M, int N, int K, int bn, int mode, int act, int out_f32,
                                       int iters, int dtype, float *ms_out);

/* As mfb200_debug_gemm_bench, also returning the kernel's per-role clock-cycle
 * counters summed over the timed launches and all CTAs: [0] epilogue waiting
 * for an accumulator, [1] epilogue processing, [2] MMA issuer waiting for a
 * free accumulator, [3] MMA issuer waiting for operands, [4] producer waiting
 * for a free stage, [5] CTA lifetime, [6] epilogue tiles (per warp), [7] unused. */
MFB200_API int mfb200_debug_gemm_trace(int M, int N, int K, int bn, int mode, int act, int out_f32,
                                       int iters, int dtype, float *ms_out,
                                       unsigned long long *trace_out);

/* Bounded-wait error path of the GEMM kernels: an M x N x K bf16 GEMM
 * (random operands, BN 256; the CTA-pair kernel when pair = 1, which needs
 * K >= 768 and M > 128) in which CTA 0 (pair 0) announces the bytes of its
 * first pipeline stage but never loads them, with every barrier wait limited
 * to wait_ns nanoseconds. The waits on that stage run out; the kernel records
 * a timeout code in the status word, drains its loads and MMAs, frees its
 * TMEM and returns. Returns 0 when the kernel returned (the code is in
 * *status_out), nonzero if it could not be launched. */
MFB200_API int mfb200_debug_gemm_withheld(int M, int N, int K, int pair,
                                          unsigned long long wait_ns, unsigned *status_out);

/* One eager forward on the handle in which layer 0's QKV GEMM withholds its
 * first stage as above (waits limited to wait_ns). Returns the error the
 * forward reports (nonzero; mfb200_last_error names the timeout); later calls
 * on the handle are unaffected. */
struct mfb200_handle;
MFB200_API int mfb200_debug_forward_withheld(struct mfb200_handle *h, int batch,
                                             unsigned long long wait_ns);

#ifdef __cplusplus
}
#endif
#endif
