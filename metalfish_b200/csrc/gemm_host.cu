// gemm_host.cu -- host side of the tcgen05 GEMM: TMA descriptor creation,
// launch configuration and the template instantiations.
#include <cstdio>
#include <algorithm>
#include <atomic>
#include <mutex>

#include "gemm_host.h"

namespace mfb200 {

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int g_num_sms = 0;
std::atomic<bool> g_pairs{true};
}  // namespace

void set_gemm_pairs(bool enable) { g_pairs = enable; }
bool gemm_pairs_enabled() { return g_pairs; }

int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

bool make_kmajor_tmap(CUtensorMap *tm, const void *base, bool fp8, uint64_t k, uint64_t rows,
                      uint64_t row_stride_bytes, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const uint32_t elem = fp8 ? 1 : 2;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_stride_bytes & 15) || k == 0 || rows == 0)
    return false;
  cuuint64_t dims[2] = {k, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {128u / elem, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r =
      fn(tm, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
         const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// General tiled tensor map (rank 2 or 3, innermost dimension first).
static bool make_tmap(CUtensorMap *tm, const void *base, CUtensorMapDataType dt, int rank,
                      const uint64_t *dims, const uint64_t *stride_bytes, const uint32_t *box,
                      CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15)) return false;
  cuuint64_t d[3], st[2];
  cuuint32_t b[3], e[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    if (dims[i] == 0) return false;
  }
  for (int i = 0; i + 1 < rank; ++i) {
    st[i] = stride_bytes[i];
    if (st[i] & 15) return false;
  }
  return fn(tm, dt, rank, const_cast<void *>(base), d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
            swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <int BN, bool FP8, bool LN, int EPI>
static cudaError_t launch_t(const GemmLaunch &g, cudaStream_t stream) {
  using S = GemmShape<BN, FP8, LN>;
  // the shared-memory opt-in is a per-device function attribute
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_sm100_kernel<BN, FP8, LN, EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         S::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  // the CTAs covering one row block of the LN epilogue form a cluster
  const int cluster = (g.args.mode == kEpiResidLN && g.args.cluster_n > 1) ? g.args.cluster_n : 1;
  const cudaError_t e = launch_k(gemm_sm100_kernel<BN, FP8, LN, EPI>, g.grid, dim3(S::THREADS),
                                 S::SMEM_BYTES, stream, cluster, g.tmA, g.tmB, g.tmOut, g.tmOut2,
                                 g.tmRes, g.args);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// How many clusters of `csize` CTAs of this GEMM can be co-resident on the
// current device (GPC boundaries make this smaller than SMs / csize).
template <int BN, bool FP8>
static int max_clusters_t(int csize) {
  using S = GemmShape<BN, FP8, true>;
  static int cache[64][9] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || csize < 1 || csize > 8) return 0;
  if (cache[dev][csize]) return cache[dev][csize];
  cudaFuncSetAttribute(gemm_sm100_kernel<BN, FP8, true, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       S::SMEM_BYTES);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(csize * 64));
  cfg.blockDim = dim3(S::THREADS);
  cfg.dynamicSmemBytes = S::SMEM_BYTES;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(csize);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_sm100_kernel<BN, FP8, true, 0>, &cfg) != cudaSuccess || n <= 0)
    n = num_sms() / csize;
  cudaGetLastError();
  cache[dev][csize] = n;
  return n;
}

// Co-resident clusters of two CTAs of the pair kernel.
template <bool FP8>
static int max_pairs_t() {
  using S = PairShape<FP8>;
  static int cache[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 0;
  if (cache[dev]) return cache[dev];
  cudaFuncSetAttribute(gemm_pair_kernel<FP8, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       S::SMEM_BYTES);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 64);
  cfg.blockDim = dim3(S::THREADS);
  cfg.dynamicSmemBytes = S::SMEM_BYTES;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<FP8, 0>, &cfg) != cudaSuccess || n <= 0)
    n = num_sms() / 2;
  cudaGetLastError();
  cache[dev] = n;
  return n;
}

template <bool FP8, int EPI>
static cudaError_t launch_pair_t(const GemmLaunch &g, cudaStream_t stream) {
  using S = PairShape<FP8>;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel<FP8, EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  return launch_k(gemm_pair_kernel<FP8, EPI>, g.grid, dim3(S::THREADS), S::SMEM_BYTES, stream, 2, g.tmA,
                  g.tmB, g.tmOut, g.tmOut2, g.tmRes, g.args);
}

static int max_clusters(int bn, bool fp8, int csize) {
  if (fp8) return bn == 256 ? max_clusters_t<256, true>(csize)
                            : (bn == 128 ? max_clusters_t<128, true>(csize) : max_clusters_t<64, true>(csize));
  return bn == 256 ? max_clusters_t<256, false>(csize)
                   : (bn == 128 ? max_clusters_t<128, false>(csize) : max_clusters_t<64, false>(csize));
}

// One kernel instance per (tile width, operand width, epilogue selector).
template <bool FP8, int EPI>
static cudaError_t launch_sel(const GemmLaunch &g, cudaStream_t stream) {
  if (g.pair) return launch_pair_t<FP8, EPI>(g, stream);
  switch (g.bn) {
  case 256: return launch_t<256, FP8, false, EPI>(g, stream);
  case 128: return launch_t<128, FP8, false, EPI>(g, stream);
  case 64: return launch_t<64, FP8, false, EPI>(g, stream);
  }
  return cudaErrorInvalidValue;
}

template <bool FP8>
static cudaError_t launch_fmt(const GemmLaunch &g, cudaStream_t stream) {
  if (g.args.mode == kEpiResidLN) {  // the cluster LayerNorm epilogue has its own kernel
    switch (g.bn) {
    case 256: return launch_t<256, FP8, true, 0>(g, stream);
    case 128: return launch_t<128, FP8, true, 0>(g, stream);
    case 64: return launch_t<64, FP8, true, 0>(g, stream);
    }
    return cudaErrorInvalidValue;
  }
  switch (epi_select(g.args.mode, g.args.act, g.args.k_splits)) {
  case kActNone: return launch_sel<FP8, kActNone>(g, stream);
  case kActRelu: return launch_sel<FP8, kActRelu>(g, stream);
  case kActRelu2: return launch_sel<FP8, kActRelu2>(g, stream);
  case kActTanh: return launch_sel<FP8, kActTanh>(g, stream);
  case kActSigmoid: return launch_sel<FP8, kActSigmoid>(g, stream);
  case kActSwish: return launch_sel<FP8, kActSwish>(g, stream);
  case kActMish: return launch_sel<FP8, kActMish>(g, stream);
  case kActSelu: return launch_sel<FP8, kActSelu>(g, stream);
  case kSelResid: return launch_sel<FP8, kSelResid>(g, stream);
  case kSelAccum: return launch_sel<FP8, kSelAccum>(g, stream);
  case kSelResidNorm: return launch_sel<FP8, kSelResidNorm>(g, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_gemm(const GemmLaunch &g, cudaStream_t stream) {
  return g.fp8 ? launch_fmt<true>(g, stream) : launch_fmt<false>(g, stream);
}

// Second half of a split-K GEMM: one warp per (row, 32-column chunk), lane =
// column. Sums the K slices' fp32 partial products [splits, M, N] in slice
// order and applies the epilogue the single-pass kernel would have applied
// (activation scale, deferred-LayerNorm fold, column scale, bias, then the
// store / accumulate / residual / residual-norm mode and the output format).
__global__ void __launch_bounds__(256)
    splitk_epilogue_kernel(const float *__restrict__ part, int splits, long long stride,
                           const GemmArgs a) {
  pdl_wait();
  pdl_launch();
  const int chunks = a.N / 32;
  const long long w = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<long long>(a.M) * chunks) return;
  const int row = static_cast<int>(w / chunks), ch = static_cast<int>(w % chunks);
  const int c = ch * 32 + lane;
  const float *p = part + static_cast<long long>(row) * a.N + c;
  float v = 0.0f;
  int s = 0;
  for (; s + 4 <= splits; s += 4) {
    const float x0 = __ldcg(p + s * stride), x1 = __ldcg(p + (s + 1) * stride);
    const float x2 = __ldcg(p + (s + 2) * stride), x3 = __ldcg(p + (s + 3) * stride);
    v += x0;
    v += x1;
    v += x2;
    v += x3;
  }
  for (; s < splits; ++s) v += __ldcg(p + s * stride);
  float as = a.a_scale_ptr ? a.a_scale * __ldg(a.a_scale_ptr) : a.a_scale;
  if (a.a_row_scale) as *= __ldcg(a.a_row_scale + row);
  if (as != 1.0f) v *= as;
  if (a.fold_stats) {
    const float2 st = __ldcg(a.fold_stats + row);
    v = st.y * (v - st.x * __ldg(a.fold_colsum + c));
  }
  if (a.col_scale) v *= __ldg(a.col_scale + c);
  if (a.bias) v += __ldg(a.bias + c);
  if (a.mode == kEpiAccum) {
    v *= a.alpha;
    if (a.out_f32) {
      float *o = static_cast<float *>(a.out) + static_cast<long long>(row) * a.ldo + c;
      *o += v;
    } else {
      __half *o = static_cast<__half *>(a.out) + static_cast<long long>(row) * a.ldo + c;
      *o = __float2half_rn(__half2float(*o) + v);
    }
    return;
  }
  if (a.mode == kEpiResidNorm) {
    float r = __half2float(a.resid16[static_cast<long long>(row) * a.ldr16 + c]);
    if (a.rn_stats) {
      const float2 st = __ldcg(a.rn_stats + row);
      r = (r - st.x) * st.y * __ldg(a.rn_gamma + c) + __ldg(a.rn_beta + c);
    }
    const float y = r + a.alpha * v;
    static_cast<__half *>(a.out)[static_cast<long long>(row) * a.ldo + c] = __float2half_rn(y);
    float sum = y, sq = y * y;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      sum += __shfl_xor_sync(0xffffffffu, sum, o);
      sq += __shfl_xor_sync(0xffffffffu, sq, o);
    }
    if (lane == 0)
      a.stats_out[static_cast<long long>(ch) * a.M + row] =
          make_float2(sum, fmaxf(sq - sum * sum * (1.0f / 32.0f), 0.0f));
    return;
  }
  if (a.mode == kEpiResid) v = a.resid[static_cast<long long>(row) * a.ldr + c] + a.alpha * v;
  else v = apply_act(v, a.act);
  const bool second = a.out2 && c >= a.split;
  void *base = second ? a.out2 : a.out;
  const long long idx = static_cast<long long>(row) * (second ? a.ldo2 : a.ldo) + (second ? c - a.split : c);
  if (a.out_f32) {
    static_cast<float *>(base)[idx] = v;
  } else if (a.out_fp8) {
    const float is = a.out_scale_ptr ? 1.0f / __ldg(a.out_scale_ptr) : a.out_inv_scale;
    if (a.out_i8)
      static_cast<int8_t *>(base)[idx] = static_cast<int8_t>(quant_s8(v * is));
    else
      static_cast<__nv_fp8_e4m3 *>(base)[idx] = __nv_fp8_e4m3(v * is);
  } else if (a.out_f16) {
    static_cast<__half *>(base)[idx] = __float2half_rn(v);
  } else {
    static_cast<__nv_bfloat16 *>(base)[idx] = __float2bfloat16_rn(v);
  }
}

// kEpiResidNorm of a split-K GEMM with the row statistics finalised in the
// same pass: one CTA (N threads, one column each) per row, so the mean and
// variance come from the whole row (two-pass, as the LayerNorm kernel).
__global__ void __launch_bounds__(1024)
    splitk_residnorm_row_kernel(const float *__restrict__ part, int splits, long long stride,
                                const GemmArgs a) {
  pdl_wait();
  pdl_launch();
  __shared__ float red[32];
  const int row = blockIdx.x, c = threadIdx.x, lane = c & 31, warp = c >> 5;
  const int warps = blockDim.x >> 5;
  const float *p = part + static_cast<long long>(row) * a.N + c;
  float v = 0.0f;
  int s = 0;
  for (; s + 4 <= splits; s += 4) {
    const float x0 = __ldcg(p + s * stride), x1 = __ldcg(p + (s + 1) * stride);
    const float x2 = __ldcg(p + (s + 2) * stride), x3 = __ldcg(p + (s + 3) * stride);
    v += x0;
    v += x1;
    v += x2;
    v += x3;
  }
  for (; s < splits; ++s) v += __ldcg(p + s * stride);
  if (a.bias) v += __ldg(a.bias + c);
  float r = __half2float(a.resid16[static_cast<long long>(row) * a.ldr16 + c]);
  if (a.rn_stats) {
    const float2 st = __ldcg(a.rn_stats + row);
    r = (r - st.x) * st.y * __ldg(a.rn_gamma + c) + __ldg(a.rn_beta + c);
  }
  const float y = r + a.alpha * v;
  static_cast<__half *>(a.out)[static_cast<long long>(row) * a.ldo + c] = __float2half_rn(y);
  // block sums: mean, then the squared deviations from it
  float t = y;
#pragma unroll
  for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  if (lane == 0) red[warp] = t;
  __syncthreads();
  float sum = 0.0f;
  for (int w = 0; w < warps; ++w) sum += red[w];
  const float mean = sum / static_cast<float>(a.N);
  __syncthreads();
  t = (y - mean) * (y - mean);
#pragma unroll
  for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  if (lane == 0) red[warp] = t;
  __syncthreads();
  if (c == 0) {
    float sq = 0.0f;
    for (int w = 0; w < warps; ++w) sq += red[w];
    a.stats_final[row] = make_float2(mean, 1.0f / sqrtf(sq / static_cast<float>(a.N) + a.ln_eps));
  }
}

cudaError_t launch_splitk_epilogue(const float *part, int splits, const GemmArgs &a,
                                   cudaStream_t stream) {
  if (a.mode == kEpiResidNorm && a.stats_final && a.N <= 1024 && a.N % 32 == 0 &&
      a.a_scale == 1.0f && !a.a_scale_ptr && !a.a_row_scale && !a.col_scale && !a.fold_stats)
    return launch_k(splitk_residnorm_row_kernel, dim3(static_cast<unsigned>(a.M)),
                    dim3(static_cast<unsigned>(a.N)), 0, stream, 1, part, splits,
                    static_cast<long long>(a.M) * a.N, a);
  if (a.stats_final) return cudaErrorInvalidValue;  // finalised statistics need the row kernel
  const long long warps = static_cast<long long>(a.M) * (a.N / 32);
  return launch_k(splitk_epilogue_kernel, dim3(static_cast<unsigned>((warps + 7) / 8)), dim3(256),
                  0, stream, 1, part, splits, static_cast<long long>(a.M) * a.N, a);
}

const char *plan_gemm(GemmLaunch &g, const void *A, long long lda_elems, const void *W,
                      long long ldw_elems, int bn, bool fp8, const GemmArgs &args) {
  if (bn != 64 && bn != 128 && bn != 256) return "gemm: BN must be 64, 128 or 256";
  if (args.M <= 0 || args.N <= 0 || args.K <= 0) return "gemm: empty problem";
  if (args.N % 32) return "gemm: N must be a multiple of 32";
  if (args.out2 && args.split % 32) return "gemm: split column must be a multiple of 32";
  if (args.mode == kEpiResidLN) {
    const int C = args.cluster_n;
    if (C != 1 && C != 2 && C != 4 && C != 8) return "gemm: LN epilogue cluster size must be 1, 2, 4 or 8";
    if (args.N != C * bn) return "gemm: LN epilogue needs N == cluster_n * BN";
    if (!args.row_stats || !args.ln_gamma || !args.ln_beta || !args.resid)
      return "gemm: LN epilogue needs row_stats, gamma, beta and a residual";
    if (args.k_splits > 1) return "gemm: LN epilogue cannot be split along K";
  }
  if (args.mode == kEpiAccum && ((!args.out_f32 && !args.out_f16) || args.out2 || args.out_fp8))
    return "gemm: the accumulate epilogue adds into one fp32 or fp16 output";
  if (args.out_f16 && (args.out_f32 || args.out_fp8)) return "gemm: one output format";
  if (args.ab_i8 && (!fp8 || args.mode == kEpiResidLN))
    return "gemm: 8-bit integer operands need the 8-bit kernels (no LN epilogue)";
  if (args.out_i8 && !args.out_fp8) return "gemm: integer 8-bit output is an 8-bit output (out_fp8)";
  if (args.mode == kEpiResidNorm) {
    if (!args.out_f16 || args.out2 || args.k_splits > 1 || !args.resid16 || !args.stats_out)
      return "gemm: the residual-norm epilogue writes one fp16 output and its row statistics "
             "from an fp16 residual (no K split)";
    if (args.rn_stats && (!args.rn_gamma || !args.rn_beta))
      return "gemm: normalising the residual needs its LayerNorm gamma and beta";
  }
  if (args.fold_stats && (args.mode != kEpiStore || args.k_splits > 1 || args.K % 32 ||
                          !args.fold_colsum || fp8))
    return "gemm: a folded LayerNorm input needs the store epilogue, K a multiple of 32, "
           "column sums and 16-bit operands (no K split)";
  if (args.k_splits > 1 && (args.bias || args.mode != kEpiStore || args.out2))
    return "gemm: split-K writes raw fp32 partials (no bias, residual or column split)";
  const uint32_t elem = fp8 ? 1 : 2;
  g = GemmLaunch{};
  g.bn = bn;
  g.fp8 = fp8;
  g.args = args;
  // CTA pairs for the large store / accumulate / residual GEMMs with at
  // least 8 K steps (K >= 512 in 16-bit, K >= 1024 in 8-bit). With fewer, a
  // tile is bound by its epilogue, and the pair's shared accumulator
  // hand-off (both CTAs must drain an accumulator before it is reused) costs
  // more than the halved W traffic saves. Measured on B200 (M=65536, one
  // process, back-to-back launches): bf16 K=1024 N=1024 gains 14%; 8-bit
  // K=1024 gains 7% (N=3104) and 15% (N=1024, accumulate epilogue); bf16
  // K=256 (4 steps) loses 20%.
  const int ksteps = (args.K + (fp8 ? 127 : 63)) / (fp8 ? 128 : 64);
  g.pair = !args.no_pair && bn == 256 && args.k_splits <= 1 && args.mode != kEpiResidLN &&
           args.M > 128 && ksteps >= 8;
  {
    // every K slice must be non-empty
    const int kblocks = (args.K + (fp8 ? 128 : 64) - 1) / (fp8 ? 128 : 64);
    int splits = args.k_splits > 1 ? args.k_splits : 1;
    if (splits > kblocks) splits = kblocks;
    const int per = (kblocks + splits - 1) / splits;
    g.args.k_splits = (kblocks + per - 1) / per;
  }
  if (!make_kmajor_tmap(&g.tmA, A, fp8, static_cast<uint64_t>(args.K),
                        static_cast<uint64_t>(args.M), static_cast<uint64_t>(lda_elems) * elem, 128))
    return "gemm: cannot build TMA descriptor for A (alignment?)";
  if (!make_kmajor_tmap(&g.tmB, W, fp8, static_cast<uint64_t>(args.K),
                        static_cast<uint64_t>(args.N), static_cast<uint64_t>(ldw_elems) * elem,
                        g.pair ? bn / 2 : bn))
    return "gemm: cannot build TMA descriptor for W (alignment?)";
  {
    // epilogue tensor maps: 32-row x 32-column boxes in the output format
    const bool f32 = g.args.k_splits > 1 || args.out_f32;
    const CUtensorMapDataType odt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                        : (args.out_fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                                        : (args.out_f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                        : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16));
    const uint64_t oel = f32 ? 4 : (args.out_fp8 ? 1 : 2);
    const CUtensorMapSwizzle oswz = f32 ? CU_TENSOR_MAP_SWIZZLE_128B
                                        : (args.out_fp8 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                        : CU_TENSOR_MAP_SWIZZLE_64B);
    const uint32_t box3[3] = {32, 32, 1};
    if (g.args.k_splits > 1) {
      if (args.split_stride != static_cast<long long>(args.M) * args.ldo)
        return "gemm: split-K partials must be packed [splits, M, ldo]";
      const uint64_t dims[3] = {uint64_t(args.N), uint64_t(args.M), uint64_t(g.args.k_splits)};
      const uint64_t st[2] = {uint64_t(args.ldo) * 4, uint64_t(args.split_stride) * 4};
      if (!make_tmap(&g.tmOut, args.out, odt, 3, dims, st, box3, oswz))
        return "gemm: cannot build the split-K output tensor map";
    } else if (args.mode == kEpiResidLN) {
      const uint64_t dims[2] = {uint64_t(args.N), uint64_t(args.M)};
      const uint64_t st[1] = {uint64_t(args.ldo) * 4};
      if (!make_tmap(&g.tmOut, args.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dims, st, box3,
                     CU_TENSOR_MAP_SWIZZLE_128B))
        return "gemm: cannot build the LN fp32 output tensor map";
      if (args.out2) {
        const uint64_t lel = args.out_fp8 ? 1 : 2;
        const uint64_t s2[1] = {uint64_t(args.ldo2) * lel};
        if (!make_tmap(&g.tmOut2, args.out2,
                       args.out_fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                       2, dims, s2, box3,
                       args.out_fp8 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B))
          return "gemm: cannot build the LN low-precision output tensor map";
      }
    } else {
      const int n_main = args.out2 ? args.split : args.N;
      const uint64_t dims[2] = {uint64_t(n_main), uint64_t(args.M)};
      const uint64_t st[1] = {uint64_t(args.ldo) * oel};
      if (!make_tmap(&g.tmOut, args.out, odt, 2, dims, st, box3, oswz))
        return "gemm: cannot build the output tensor map (alignment?)";
      if (args.out2) {
        const uint64_t d2[2] = {uint64_t(args.N - args.split), uint64_t(args.M)};
        const uint64_t s2[1] = {uint64_t(args.ldo2) * oel};
        if (!make_tmap(&g.tmOut2, args.out2, odt, 2, d2, s2, box3, oswz))
          return "gemm: cannot build the second output tensor map";
      }
    }
    if (args.mode == kEpiResidNorm) {
      const uint64_t dims[2] = {uint64_t(args.N), uint64_t(args.M)};
      const uint64_t st[1] = {uint64_t(args.ldr16) * 2};
      if (!make_tmap(&g.tmRes, args.resid16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, dims, st, box3,
                     CU_TENSOR_MAP_SWIZZLE_64B))
        return "gemm: cannot build the fp16 residual tensor map";
    }
    if (args.mode == kEpiResid || args.mode == kEpiResidLN) {
      const uint64_t dims[2] = {uint64_t(args.N), uint64_t(args.M)};
      const uint64_t st[1] = {uint64_t(args.ldr) * 4};
      if (!make_tmap(&g.tmRes, args.resid, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dims, st, box3,
                     CU_TENSOR_MAP_SWIZZLE_128B))
        return "gemm: cannot build the residual tensor map";
    }
  }
  const long long tiles = static_cast<long long>((args.M + 127) / 128) *
                          ((args.N + bn - 1) / bn) * g.args.k_splits;
  const int sms = num_sms();
  if (args.mode == kEpiResidLN) {
    // whole clusters; each cluster walks row blocks
    const long long tiles_m = (args.M + 127) / 128;
    const long long clusters = std::min<long long>(tiles_m, max_clusters(bn, fp8, args.cluster_n));
    g.grid = dim3(static_cast<unsigned>(clusters * args.cluster_n));
    return nullptr;
  }
  if (g.pair) {
    const long long units = static_cast<long long>((args.M + 255) / 256) * ((args.N + 255) / 256);
    const long long pairs = std::min<long long>(units, fp8 ? max_pairs_t<true>() : max_pairs_t<false>());
    g.grid = dim3(static_cast<unsigned>(2 * pairs));
    return nullptr;
  }
  g.grid = dim3(static_cast<unsigned>(tiles < sms ? tiles : sms));
  return nullptr;
}

}  // namespace mfb200
