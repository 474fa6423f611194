// noalloc.cu -- split-K GEMM that allocates nothing.
//
// Some callers cannot call cudaMalloc: code that runs inside another
// framework's memory pool, or a real-time search thread that must not take
// the driver's allocation locks or risk an out-of-memory failure in the
// middle of a game. For them this file provides one entry point,
// mfb200_splitk_gemm_noalloc, that computes
//     out[M,N] (fp32) = A[M,K] . W[N,K]^T + bias
// with the tcgen05 GEMM split along K, keeping the per-slice partial products
// in a fixed file-scope device array instead of a caller- or
// library-allocated workspace. The caller passes device pointers for inputs
// and output only.
#include <cstdio>
#include <mutex>

#include "../../include/mfb200.h"
#include "gemm_host.h"

namespace {

// Scratch for the partial products: k_splits * M * N fp32 values at most.
constexpr long long kScratchFloats = 2LL * 1024 * 1024;  // 8 MiB per GPU
constexpr long long kPartialFloats = kScratchFloats - 64;  // the tail holds the status word
static __device__ __align__(256) float g_splitk_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
float *g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

thread_local char t_err[256];

int fail(const char *msg) {
  std::snprintf(t_err, sizeof(t_err), "%s", msg);
  return 1;
}

// out[r, c] = bias[c] + sum_s part[s, r, c]; NaN everywhere if a barrier
// wait of the GEMM timed out (*status != 0), whose partials are incomplete.
__global__ void splitk_sum_kernel(const float *__restrict__ part, int splits, long long stride,
                                  long long total, int n, const float *__restrict__ bias,
                                  const unsigned *__restrict__ status, float *__restrict__ out) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  if (*status != 0u) {
    out[i] = __int_as_float(0x7FC00000);
    return;
  }
  float acc = bias ? bias[i % n] : 0.0f;
  for (int s = 0; s < splits; ++s) acc += part[s * stride + i];
  out[i] = acc;
}

}  // namespace

extern "C" MFB200_API const char *mfb200_noalloc_last_error(void) { return t_err; }

extern "C" MFB200_API int mfb200_splitk_gemm_noalloc(const void *d_A, const void *d_W, int M,
                                                     int N, int K, int k_splits,
                                                     const float *d_bias, float *d_out,
                                                     void *stream) {
  if (!d_A || !d_W || !d_out) return fail("mfb200_splitk_gemm_noalloc: null pointer");
  if (M <= 0 || N <= 0 || K <= 0 || k_splits <= 0)
    return fail("mfb200_splitk_gemm_noalloc: sizes must be positive");
  if (N % 32 || K % 8)
    return fail("mfb200_splitk_gemm_noalloc: N must be a multiple of 32 and K of 8");
  if (static_cast<long long>(k_splits) * M * N > kPartialFloats)
    return fail("mfb200_splitk_gemm_noalloc: k_splits*M*N exceeds the 2097088-float scratch "
                "limit; use fewer splits or a smaller problem");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail("mfb200_splitk_gemm_noalloc: no current CUDA device");
  float *scratch = nullptr;
  {
    // first call on a device: resolve the device address of the scratch
    // array (the name itself is only a host-side stand-in)
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
      void *p = nullptr;
      if (cudaGetSymbolAddress(&p, g_splitk_scratch) != cudaSuccess || !p)
        return fail("mfb200_splitk_gemm_noalloc: cudaGetSymbolAddress failed");
      g_scratch_ptr[dev] = static_cast<float *>(p);
    }
    scratch = g_scratch_ptr[dev];
  }
  using namespace mfb200;
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.mode = kEpiStore;
  a.act = kActNone;
  a.out = scratch;
  a.ldo = N;
  a.out_f32 = 1;
  a.a_scale = 1.0f;
  a.alpha = 1.0f;
  a.k_splits = k_splits;
  a.split_stride = static_cast<long long>(M) * N;
  // The GEMM's device status word (set only on a barrier timeout) lives in
  // the scratch tail, which the partials never reach; it must start at zero.
  a.status = reinterpret_cast<unsigned *>(scratch + kPartialFloats);
  GemmLaunch g;
  if (const char *err = plan_gemm(g, d_A, K, d_W, K, N >= 256 ? 256 : (N >= 128 ? 128 : 64),
                                  false, a))
    return fail(err);
  const int splits = g.args.k_splits;  // planning may merge empty K slices
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(a.status, 0, sizeof(unsigned), s) != cudaSuccess)
    return fail("mfb200_splitk_gemm_noalloc: status clear failed");
  if (launch_gemm(g, s) != cudaSuccess) return fail("mfb200_splitk_gemm_noalloc: GEMM launch failed");
  const long long total = static_cast<long long>(M) * N;
  splitk_sum_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(
      scratch, splits, total, total, N, d_bias, a.status, d_out);
  if (cudaGetLastError() != cudaSuccess) return fail("mfb200_splitk_gemm_noalloc: reduce launch failed");
  return 0;
}
