// debug_api.cu -- self-contained kernel entry points for unit tests
// (include/mfb200_testing.h). Each call allocates its own device buffers,
// copies host inputs in, runs ONE kernel and copies the result back.
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <cstdio>
#include <cstring>
#include <vector>

#include "../../include/mfb200_testing.h"
#include "gemm_host.h"

using namespace mfb200;

namespace {
struct DevBuf {
  void *p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  bool alloc(size_t n) { return cudaMalloc(&p, n ? n : 16) == cudaSuccess; }
};
}  // namespace

extern "C" void mfb200_debug_set_gemm_pairs(int enable) { set_gemm_pairs(enable != 0); }

extern "C" void mfb200_debug_set_pdl(int enable) { set_pdl(enable != 0); }

extern "C" int mfb200_debug_gemm(int M, int N, int K, int bn, int fp8, const void *A,
                                 const void *W, const float *bias, int mode, int act,
                                 const float *resid, float alpha, const float *ln_gamma,
                                 const float *ln_beta, float ln_eps, const float *col_scale,
                                 float a_scale, int out_f32, int k_splits, void *out,
                                 unsigned *status_out) {
  (void)ln_gamma;
  (void)ln_beta;
  (void)ln_eps;
  const int sp = k_splits > 1 ? k_splits : 1;
  const size_t es = fp8 == 1 ? 1 : 2;  // fp8: 0 bf16, 1 e4m3, 2 fp16 operands
  DevBuf dA, dW, dB, dR, dO, dG, dBe, dCs, dS;
  if (!dA.alloc(size_t(M) * K * es) || !dW.alloc(size_t(N) * K * es) || !dB.alloc(N * 4) ||
      !dR.alloc(size_t(M) * N * 4) || !dO.alloc(size_t(sp) * M * N * 4) || !dG.alloc(N * 4) ||
      !dBe.alloc(N * 4) || !dCs.alloc(N * 4) || !dS.alloc(4))
    return 1;
  cudaMemcpy(dA.p, A, size_t(M) * K * es, cudaMemcpyHostToDevice);
  cudaMemcpy(dW.p, W, size_t(N) * K * es, cudaMemcpyHostToDevice);
  if (bias) cudaMemcpy(dB.p, bias, N * 4, cudaMemcpyHostToDevice);
  if (resid) cudaMemcpy(dR.p, resid, size_t(M) * N * 4, cudaMemcpyHostToDevice);
  if (col_scale) cudaMemcpy(dCs.p, col_scale, N * 4, cudaMemcpyHostToDevice);
  cudaMemset(dO.p, 0, size_t(sp) * M * N * 4);
  if (mode == kEpiAccum && resid) {  // accumulate in place: the output starts as the residual
    if (out_f32 == 2) {
      std::vector<__half> h(size_t(M) * N);
      for (size_t i = 0; i < h.size(); ++i) h[i] = __float2half_rn(resid[i]);
      cudaMemcpy(dO.p, h.data(), h.size() * 2, cudaMemcpyHostToDevice);
    } else {
      cudaMemcpy(dO.p, resid, size_t(M) * N * 4, cudaMemcpyHostToDevice);
    }
  }
  cudaMemset(dS.p, 0, 4);
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.mode = mode;
  a.act = act;
  a.bias = bias ? static_cast<float *>(dB.p) : nullptr;
  a.out = dO.p;
  a.ldo = N;
  a.resid = static_cast<const float *>(dR.p);
  a.ldr = N;
  a.alpha = alpha;
  a.k_splits = sp;
  a.split_stride = static_cast<long long>(M) * N;
  a.col_scale = col_scale ? static_cast<float *>(dCs.p) : nullptr;
  a.a_scale = a_scale;
  a.status = static_cast<unsigned *>(dS.p);
  a.out_f32 = out_f32 == 1;
  a.out_f16 = out_f32 == 2;  // 2: fp16 output
  GemmLaunch g;
  a.ab_f16 = fp8 == 2;
  a.no_pair = gemm_pairs_enabled() ? 0 : 1;
  if (plan_gemm(g, dA.p, K, dW.p, K, bn, fp8 == 1, a)) return 2;
  if (launch_gemm(g, 0) != cudaSuccess) return 3;
  if (cudaDeviceSynchronize() != cudaSuccess) return 4;
  cudaMemcpy(out, dO.p, size_t(sp) * M * N * (sp > 1 || out_f32 == 1 ? 4 : 2), cudaMemcpyDeviceToHost);
  unsigned st = 0;
  cudaMemcpy(&st, dS.p, 4, cudaMemcpyDeviceToHost);
  if (status_out) *status_out = st;
  return st ? 5 : 0;
}

// Times `iters` back-to-back launches of one GEMM on random device data
// (bf16, bias, optional fp32 output); returns the mean ms per launch.
// Pseudo-random operand fill (an integer hash of the index): values in
// [-1, 1) for 16-bit formats, e4m3 codes of magnitude below 1 for 8-bit.
// Random operands matter for timing: tensor-core power, and so the clock the
// GPU holds under its power cap, depends on how many bits toggle.
__global__ void fill_random_kernel(uint16_t *p, long long n, int dtype, uint32_t seed) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t h = static_cast<uint32_t>(i) * 0x9E3779B1u ^ seed;
  h ^= h >> 15;
  h *= 0x85EBCA77u;
  h ^= h >> 13;
  h *= 0xC2B2AE3Du;
  h ^= h >> 16;
  const float f = static_cast<float>(h & 0xFFFFu) / 32768.0f - 1.0f;
  if (dtype == 1) {  // two e4m3 values per 16-bit word
    const uint16_t lo = static_cast<uint16_t>((h & 0x80u) | ((h >> 8) & 0x37u));
    const uint16_t hi = static_cast<uint16_t>(((h >> 16) & 0x80u) | ((h >> 24) & 0x37u));
    p[i] = static_cast<uint16_t>(lo | (hi << 8));
  } else if (dtype == 2) {
    p[i] = __half_as_ushort(__float2half_rn(f));
  } else {
    p[i] = __bfloat16_as_ushort(__float2bfloat16_rn(f));
  }
}

static int gemm_bench_impl(int M, int N, int K, int bn, int mode, int act, int out_f32, int iters,
                           int dtype, float *ms_out, unsigned long long *trace_out);

extern "C" int mfb200_debug_gemm_bench(int M, int N, int K, int bn, int mode, int act,
                                       int out_f32, int iters, int dtype, float *ms_out) {
  return gemm_bench_impl(M, N, K, bn, mode, act, out_f32, iters, dtype, ms_out, nullptr);
}

// As mfb200_debug_gemm_bench, and the kernel's per-role cycle counters
// (GemmArgs::trace, 8 values summed over the `iters` timed launches).
extern "C" int mfb200_debug_gemm_trace(int M, int N, int K, int bn, int mode, int act,
                                       int out_f32, int iters, int dtype, float *ms_out,
                                       unsigned long long *trace_out) {
  return gemm_bench_impl(M, N, K, bn, mode, act, out_f32, iters, dtype, ms_out, trace_out);
}

static int gemm_bench_impl(int M, int N, int K, int bn, int mode, int act, int out_f32, int iters,
                           int dtype, float *ms_out, unsigned long long *trace_out) {
  DevBuf dA, dW, dB, dR, dO, dS, dO2, dG, dRS;
  if (!dA.alloc(size_t(M) * K * 2) || !dW.alloc(size_t(N) * K * 2) || !dB.alloc(N * 4) ||
      !dR.alloc(size_t(M) * N * 4) || !dO.alloc(size_t(M) * N * 4) || !dS.alloc(4) ||
      !dO2.alloc(size_t(M) * N * 2) || !dG.alloc(N * 4) || !dRS.alloc(size_t(M) * 16 * 8))
    return 1;
  cudaMemset(dG.p, 0, N * 4);
  {
    const long long na = static_cast<long long>(M) * K * (dtype == 1 ? 1 : 2) / 2;
    const long long nw = static_cast<long long>(N) * K * (dtype == 1 ? 1 : 2) / 2;
    fill_random_kernel<<<static_cast<unsigned>((na + 255) / 256), 256>>>(
        static_cast<uint16_t *>(dA.p), na, dtype, 1u);
    fill_random_kernel<<<static_cast<unsigned>((nw + 255) / 256), 256>>>(
        static_cast<uint16_t *>(dW.p), nw, dtype, 2u);
  }
  cudaMemset(dB.p, 0, N * 4);
  cudaMemset(dR.p, 0, size_t(M) * N * 4);
  cudaMemset(dS.p, 0, 4);
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.mode = mode;
  a.act = act;
  a.bias = static_cast<float *>(dB.p);
  a.out = dO.p;
  a.ldo = N;
  a.resid = static_cast<const float *>(dR.p);
  a.ldr = N;
  a.alpha = 1.0f;
  a.a_scale = 1.0f;
  a.out_f32 = out_f32 == 1;
  a.out_f16 = out_f32 == 2;  // 2: fp16 output
  a.ab_f16 = dtype == 2;
  a.status = static_cast<unsigned *>(dS.p);
  if (mode == kEpiAccum && !a.out_f16) a.out_f32 = 1;
  if (mode == kEpiResidLN) {  // fused residual + LayerNorm (N / bn CTAs per cluster)
    a.out_f32 = 0;
    a.out2 = dO2.p;
    a.ldo2 = N;
    a.ln_gamma = static_cast<float *>(dG.p);
    a.ln_beta = static_cast<float *>(dG.p);
    a.ln_eps = 1e-3f;
    a.cluster_n = N / bn;
    a.row_stats = static_cast<float2 *>(dRS.p);
  }
  if (mode == kEpiResidNorm) {  // deferred-LayerNorm residual GEMM: fp16 stream in place
    a.out_f32 = 0;
    a.out_f16 = 1;
    a.resid16 = static_cast<const __half *>(dO.p);
    a.ldr16 = N;
    a.rn_stats = reinterpret_cast<const float2 *>(dRS.p);  // (0, 0): normalised residual = beta
    a.rn_gamma = static_cast<float *>(dG.p);
    a.rn_beta = static_cast<float *>(dG.p);
    a.stats_out = reinterpret_cast<float2 *>(dR.p);
    a.ln_eps = 1e-3f;
    cudaMemset(dRS.p, 0, size_t(M) * 8);
  }
  GemmLaunch g;
  a.no_pair = gemm_pairs_enabled() ? 0 : 1;
  if (plan_gemm(g, dA.p, K, dW.p, K, bn, dtype == 1, a)) return 2;
  for (int i = 0; i < 2; ++i)
    if (launch_gemm(g, 0) != cudaSuccess) return 3;
  DevBuf dT;
  if (trace_out) {
    if (!dT.alloc(8 * 8)) return 1;
    cudaMemset(dT.p, 0, 64);
    g.args.trace = static_cast<unsigned long long *>(dT.p);
  }
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, 0);
  for (int i = 0; i < iters; ++i) launch_gemm(g, 0);
  cudaEventRecord(e1, 0);
  if (cudaDeviceSynchronize() != cudaSuccess) return 4;
  float ms = 0;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *ms_out = ms / iters;
  if (trace_out) cudaMemcpy(trace_out, dT.p, 64, cudaMemcpyDeviceToHost);
  unsigned st = 0;
  cudaMemcpy(&st, dS.p, 4, cudaMemcpyDeviceToHost);
  return st ? 5 : 0;
}

// A GEMM on random operands whose first pipeline stage in CTA 0 (or CTA
// pair 0) is announced on its barrier but never loaded, with every barrier
// wait limited to wait_ns: the waits on that stage run out, the kernel
// records a timeout code in the status word, drains and returns.
extern "C" int mfb200_debug_gemm_withheld(int M, int N, int K, int pair,
                                          unsigned long long wait_ns, unsigned *status_out) {
  DevBuf dA, dW, dO, dS;
  if (!dA.alloc(size_t(M) * K * 2) || !dW.alloc(size_t(N) * K * 2) ||
      !dO.alloc(size_t(M) * N * 2) || !dS.alloc(4))
    return 1;
  fill_random_kernel<<<static_cast<unsigned>((size_t(M) * K + 255) / 256), 256>>>(
      static_cast<uint16_t *>(dA.p), static_cast<long long>(M) * K, 0, 1u);
  fill_random_kernel<<<static_cast<unsigned>((size_t(N) * K + 255) / 256), 256>>>(
      static_cast<uint16_t *>(dW.p), static_cast<long long>(N) * K, 0, 2u);
  cudaMemset(dS.p, 0, 4);
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.out = dO.p;
  a.ldo = N;
  a.alpha = 1.0f;
  a.a_scale = 1.0f;
  a.status = static_cast<unsigned *>(dS.p);
  a.wait_ns = wait_ns;
  a.debug_withhold = 1;
  a.no_pair = pair ? 0 : 1;
  GemmLaunch g;
  if (plan_gemm(g, dA.p, K, dW.p, K, 256, false, a)) return 2;
  if (pair && !g.pair) return 6;
  if (launch_gemm(g, 0) != cudaSuccess) return 3;
  if (cudaDeviceSynchronize() != cudaSuccess) return 4;
  unsigned st = 0;
  cudaMemcpy(&st, dS.p, 4, cudaMemcpyDeviceToHost);
  if (status_out) *status_out = st;
  return 0;
}

// Residual + LayerNorm GEMM (kEpiResidLN): y = resid + alpha*(A.W^T + bias),
// out_f32 = LN(y)*gamma + beta (fp32) and out_bf16 = the same in bf16. The
// row spans N / bn CTAs of one thread-block cluster.
extern "C" int mfb200_debug_gemm_ln(int M, int N, int K, int bn, const void *A, const void *W,
                                    const float *bias, const float *resid, float alpha,
                                    const float *gamma, const float *beta, float eps,
                                    float *out_f32, uint16_t *out_bf16, unsigned *status_out) {
  DevBuf dA, dW, dB, dR, dG, dBe, dO, dO2, dRS, dS;
  const int C = N / bn;
  if (!dA.alloc(size_t(M) * K * 2) || !dW.alloc(size_t(N) * K * 2) || !dB.alloc(N * 4) ||
      !dR.alloc(size_t(M) * N * 4) || !dG.alloc(N * 4) || !dBe.alloc(N * 4) ||
      !dO.alloc(size_t(M) * N * 4) || !dO2.alloc(size_t(M) * N * 2) ||
      !dRS.alloc(size_t(M) * 2 * C * 8) || !dS.alloc(4))
    return 1;
  cudaMemcpy(dA.p, A, size_t(M) * K * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(dW.p, W, size_t(N) * K * 2, cudaMemcpyHostToDevice);
  cudaMemcpy(dB.p, bias, N * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dR.p, resid, size_t(M) * N * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dG.p, gamma, N * 4, cudaMemcpyHostToDevice);
  cudaMemcpy(dBe.p, beta, N * 4, cudaMemcpyHostToDevice);
  cudaMemset(dS.p, 0, 4);
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.mode = kEpiResidLN;
  a.bias = static_cast<float *>(dB.p);
  a.resid = static_cast<const float *>(dR.p);
  a.ldr = N;
  a.alpha = alpha;
  a.a_scale = 1.0f;
  a.out = dO.p;
  a.ldo = N;
  a.out2 = dO2.p;
  a.ldo2 = N;
  a.ln_gamma = static_cast<float *>(dG.p);
  a.ln_beta = static_cast<float *>(dBe.p);
  a.ln_eps = eps;
  a.cluster_n = C;
  a.row_stats = static_cast<float2 *>(dRS.p);
  a.status = static_cast<unsigned *>(dS.p);
  GemmLaunch g;
  a.no_pair = gemm_pairs_enabled() ? 0 : 1;
  if (const char *e = plan_gemm(g, dA.p, K, dW.p, K, bn, false, a)) {
    std::fprintf(stderr, "%s\n", e);
    return 2;
  }
  if (launch_gemm(g, 0) != cudaSuccess) return 3;
  if (cudaDeviceSynchronize() != cudaSuccess) return 4;
  cudaMemcpy(out_f32, dO.p, size_t(M) * N * 4, cudaMemcpyDeviceToHost);
  cudaMemcpy(out_bf16, dO2.p, size_t(M) * N * 2, cudaMemcpyDeviceToHost);
  unsigned st = 0;
  cudaMemcpy(&st, dS.p, 4, cudaMemcpyDeviceToHost);
  if (status_out) *status_out = st;
  return st ? 5 : 0;
}
