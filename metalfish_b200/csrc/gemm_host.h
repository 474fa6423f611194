// gemm_host.h -- planning and launching of the tcgen05 GEMM.
#pragma once
#include "gemm_sm100.cuh"

namespace mfb200 {

// A fully prepared launch: both TMA descriptors and the epilogue arguments.
// Plans are built once per (buffer set, batch size) and replayed (directly or
// inside a CUDA graph).
struct GemmLaunch {
  CUtensorMap tmA, tmB;        // operands (K-major, 128-byte swizzle)
  CUtensorMap tmOut, tmOut2;   // epilogue TMA stores (32 x 32 boxes)
  CUtensorMap tmRes;           // residual TMA loads (fp32, 32 x 32 boxes)
  GemmArgs args;
  int bn = 256;
  bool fp8 = false;
  bool pair = false;  // CTA-pair kernel (gemm_pair_kernel), clusters of 2
  dim3 grid;
};

// Whether plan_gemm may choose the CTA-pair kernel (default on).
void set_gemm_pairs(bool enable);
// Whether GEMMs planned from now on may use the CTA-pair kernel (tests can forbid it).
bool gemm_pairs_enabled();

int num_sms();

bool make_kmajor_tmap(CUtensorMap *tm, const void *base, bool fp8, uint64_t k, uint64_t rows,
                      uint64_t row_stride_bytes, uint32_t box_rows);

// Returns nullptr on success, else a static error message.
const char *plan_gemm(GemmLaunch &g, const void *A, long long lda_elems, const void *W,
                      long long ldw_elems, int bn, bool fp8, const GemmArgs &args);

cudaError_t launch_gemm(const GemmLaunch &g, cudaStream_t stream);

// The reduction and epilogue of a GEMM whose K slices were computed by a
// split-K launch into `part` ([splits, a.M, a.N] fp32): applies `a`'s
// epilogue (any mode but the LayerNorm cluster one) to the sums.
cudaError_t launch_splitk_epilogue(const float *part, int splits, const GemmArgs &a,
                                   cudaStream_t stream);

}  // namespace mfb200
