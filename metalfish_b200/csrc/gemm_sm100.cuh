// gemm_sm100.cuh -- persistent tcgen05/TMEM GEMM with fused epilogues.
//
//   C[M,N] = epilogue( A[M,K] . W[N,K]^T )
//
// A (activations) and W (weights, the reference's [out, in] layout) are both
// K-major in HBM. Each CTA owns a 128 x BN output tile (optionally one K
// slice of it, split-K) at a time; the CTA is persistent over work units
// (grid = number of SMs) and warp-specialised:
//   warp 0     TMA producer: one lane streams 128-byte-swizzled K slices of A
//              and W into a STAGES-deep shared-memory ring (no multicast);
//   warp 1     MMA issuer: allocates 2*BN TMEM columns (two fp32
//              accumulators, so the epilogue of tile i overlaps the MMAs of
//              tile i+1) and issues tcgen05.mma (M=128, N=BN, K=16 bf16 or
//              K=32 fp8 per instruction) from one lane;
//   warps 2-17 epilogue: four warps per TMEM lane quarter (TMEM lane =
//              tile row), each taking every fourth 32-column chunk (in the
//              cluster-LayerNorm variant warps 2-9, two teams of four that
//              alternate tiles, each warp covering all columns of its 32
//              rows); tcgen05.ld the
//              accumulator, apply scale / bias / activation / residual
//              (residual tiles fetched by TMA), write each 32 x 32 chunk into
//              a per-warp swizzled shared-memory tile in the output format
//              (bf16, fp16, e4m3, int8 or fp32) and TMA-store it
//              asynchronously.
// Each kernel instance carries one epilogue (template parameter EPI), and
// gemm_pair_kernel runs the same roles over a cluster of two CTAs
// (tcgen05 cta_group::2, 256-row tiles).
// All barrier waits are bounded (sm100_ptx.cuh).
#pragma once
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "pdl.cuh"
#include "sm100_ptx.cuh"

namespace mfb200 {

enum EpiMode : int {
  kEpiStore = 0,    // act(scale*acc + bias)
  kEpiResid = 1,    // resid + alpha * (scale*acc + bias)
  kEpiResidLN = 2,  // y = resid + alpha * (scale*acc + bias); LN(y) over the full row
                    // (the row spans the cluster_n CTAs of a thread-block cluster)
  kEpiAccum = 3,    // out (fp32 or fp16, holding the residual) += alpha * (scale*acc + bias),
                    // added in place by TMA reduce stores: no residual reads
  kEpiResidNorm = 4,  // y = LN_prev(resid16) + alpha * (scale*acc + bias), stored fp16 (in place
                      // over resid16 allowed), with per-32-column row statistics of y written
                      // to stats_out; LN_prev applies the row statistics rn_stats of the
                      // residual with rn_gamma / rn_beta (rn_stats == nullptr: residual as is)
};

enum Act : int {
  kActNone = 0, kActRelu, kActRelu2, kActTanh, kActSigmoid, kActSwish, kActMish, kActSelu
};

struct GemmArgs {
  int M, N, K;
  int ab_f16;                 // 16-bit operands are fp16 (else bf16); both A and W
  int ab_i8;                  // 8-bit operands are signed integers (kind::i8, int32
                              // accumulator converted to float) instead of e4m3
  const float *a_row_scale;   // if set: the accumulator of row m is multiplied by a_row_scale[m]
                              // (per-row dequantisation scale of 8-bit integer activations)
  int out_i8;                 // store signed 8-bit integers round(v / *out_scale_ptr), saturated
  int mode, act;
  const float *bias;          // [N] or nullptr
  void *out;                  // [M, ldo] bf16 (or e4m3 / fp32)
  long long ldo;
  void *out2;                 // columns n >= split go to out2[m, n - split]
  long long ldo2;
  int split;
  const float *resid;         // kEpiResid: fp32 residual parent [M, ldr]
  long long ldr;
  float alpha;
  const float *col_scale;     // per-output-channel scale (fp8 weights) or nullptr
  float a_scale;              // activation scale (fp8) ; 1 for bf16
  int out_f32;                // store fp32 instead of bf16
  int out_f16;                // store fp16 instead of bf16
  int out_fp8;                // store e4m3 instead of bf16 ...
  float out_inv_scale;        // ... after multiplying by this
  const float *a_scale_ptr;   // if set: activation scale multiplied by *a_scale_ptr
  const float *out_scale_ptr; // if set (e4m3 out): stored value = v / *out_scale_ptr
  const float *ln_gamma, *ln_beta;  // kEpiResidLN: LN affine parameters [N]
  float ln_eps;
  int cluster_n;              // kEpiResidLN: CTAs per row (cluster size, N = cluster_n * BN)
  float2 *row_stats;          // kEpiResidLN: [M, 2*cluster_n] per-row partial (sum, sum of squares)
  int k_splits;               // >1: split-K; K slice s writes fp32 partials at
  long long split_stride;     //     out + s * split_stride (raw accumulator)
  unsigned *status;           // device status word
  unsigned long long wait_ns; // limit of every barrier wait (0: kWaitLimitNs)
  int debug_withhold;         // tests only: CTA 0 (pair 0) announces its first stage's bytes
                              // but never loads them, so the waits on it run out
  int no_pair;                // never use the CTA-pair kernel for this GEMM
  unsigned long long *trace;  // profiling only (null in the product): per-role clock-cycle sums,
                              // see gemm_trace_add
  // Deferred LayerNorm (the residual stream is kept un-normalised). The
  // residual GEMM writes per-row partials: float2 (chunk sum, chunk sum of
  // squared deviations from the chunk mean) per 32-column chunk, chunk-major
  // [N / 32, M] so that a warp's 32 rows store 256 contiguous bytes;
  // launch_row_stats turns them into per-row float2 (mean, 1/sqrt(var + eps)).
  const __half *resid16;      // kEpiResidNorm: fp16 residual [M, ldr16]
  long long ldr16;
  const float2 *rn_stats;     // kEpiResidNorm: (mean, rstd) [M] of the residual rows, or nullptr
  const float *rn_gamma, *rn_beta;  // kEpiResidNorm: affine parameters of that LayerNorm [N]
  float2 *stats_out;          // kEpiResidNorm: partials of the stored rows [N / 32, M]
  const float2 *fold_stats;   // kEpiStore: A holds un-normalised rows with (mean, rstd) [M];
                              // W holds gamma-scaled rows and the epilogue computes
                              // rstd * (acc - mean * fold_colsum) before the bias
  const float *fold_colsum;   // [N] column sums of the gamma-scaled W
  float2 *stats_final;        // kEpiResidNorm through the split-K epilogue kernel (N <= 1024):
                              // the rows' (mean, rstd) [M] written directly (stats_out unused)
};

// mish(x) = x * tanh(softplus(x)). With e = exp(x), tanh(log(1 + e)) =
// ((1+e)^2 - 1) / ((1+e)^2 + 1) = n / (n + 2) where n = e * (e + 2): one
// exponential and one division instead of exp, log1p and tanh, both the fast
// forms (relative error ~1e-6, far inside the bf16 rounding of the output).
// For x > 20 the ratio is 1 to fp32 precision (and e*e would overflow), so
// mish(x) = x.
__device__ __forceinline__ float mish_fast(float v) {
  if (v > 20.0f) return v;
  const float e = __expf(v);
  const float n = e * (e + 2.0f);
  return v * __fdividef(n, n + 2.0f);
}

// Activations of the reference CPU backend (src/nn/cpu/cpu_network.cpp:303-324).
template <int ACT>
__device__ __forceinline__ float act_t(float v) {
  if constexpr (ACT == kActRelu) return fmaxf(v, 0.0f);
  else if constexpr (ACT == kActRelu2) { const float r = fmaxf(v, 0.0f); return r * r; }
  else if constexpr (ACT == kActTanh) return tanhf(v);
  else if constexpr (ACT == kActSigmoid) return 1.0f / (1.0f + expf(-v));
  else if constexpr (ACT == kActSwish)
    // fast exponential and division: relative error ~1e-6, far inside the
    // bf16 rounding of every consumer; for v < ~-87 the divisor overflows
    // and the result is 0 (the true value is below 1e-36)
    return __fdividef(v, 1.0f + __expf(-v));
  else if constexpr (ACT == kActMish) return mish_fast(v);
  else if constexpr (ACT == kActSelu) return 1.05070098f * (v > 0.0f ? v : 1.67326324f * (expf(v) - 1.0f));
  else return v;
}

__device__ __forceinline__ float apply_act(float v, int act) {
  switch (act) {
  case kActRelu: return act_t<kActRelu>(v);
  case kActRelu2: return act_t<kActRelu2>(v);
  case kActTanh: return act_t<kActTanh>(v);
  case kActSigmoid: return act_t<kActSigmoid>(v);
  case kActSwish: return act_t<kActSwish>(v);
  case kActMish: return act_t<kActMish>(v);
  case kActSelu: return act_t<kActSelu>(v);
  default: return v;
  }
}

// Epilogue staging: every epilogue warp owns a 4 KB tile (1024-byte aligned)
// that holds one 32-row x 32-column chunk in the exact byte layout the TMA
// unit expects for the output tensor map: fp32 rows of 128 B with the 128-byte
// swizzle, bf16 rows of 64 B with the 64-byte swizzle, e4m3 rows of 32 B with
// the 32-byte swizzle (16-byte group q of row r stored at group q ^ f(r)). With
// one row per lane these layouts make the shared-memory writes conflict-free,
// and one elected lane then issues an asynchronous TMA store of the chunk.
// Residual tiles arrive the same way, by TMA load into the staging tile.
// Epilogue warps: 16 (four per TMEM lane quarter, every fourth 32-column
// chunk each) in the store / accumulate kernels, 8 in the LayerNorm kernels.
constexpr int kEpiWarpsLN = 8;
constexpr int kEpiWarpsMax = 16;
constexpr int kStageBytes = 32 * 32 * 4;

struct EpiCtx {
  const CUtensorMap *out, *out2, *res;
  uint8_t *stage;      // this warp's staging tile
  uint64_t *res_bar;   // this warp's mbarrier for residual tile loads
  uint32_t res_loads;  // residual loads issued so far (phase parity)
  int lane;
  volatile int *abort_flag;
  uint64_t *xbar;      // row-statistics barrier (kEpiResidLN)
  uint32_t xtiles;     // row-statistics exchanges completed (phase parity)
  uint32_t rank;       // CTA rank in the cluster
  uint8_t *stage2;     // second staging tile (kEpiResidLN kernels)
  uint32_t chunks;     // chunks staged so far (selects the half of a 2-byte-output tile)
  uint32_t res_issued; // residual loads issued (kEpiResidNorm prefetch)
  float2 rowst;        // deferred LayerNorm: this lane's row (mean, rstd), loaded by epi_pre
  float arow;          // this lane's row scale (args.a_row_scale), loaded by epi_pre
};

// Deferred LayerNorm, issued before the accumulator wait so that the latency
// overlaps the mainloop: this lane's row (mean, rstd) and, into L1, the
// tile's gamma / beta / column-sum lines.
__device__ __forceinline__ void epi_pre(const GemmArgs &args, EpiCtx &e, int row0, int n0, int bn) {
  if (args.a_row_scale)
    e.arow = __ldcg(args.a_row_scale + (row0 + e.lane < args.M ? row0 + e.lane : args.M - 1));
  const float2 *st = args.mode == kEpiResidNorm ? args.rn_stats : args.fold_stats;
  if (!st) return;
  const int row = row0 + e.lane < args.M ? row0 + e.lane : args.M - 1;
  e.rowst = __ldcg(st + row);
  if (e.lane < bn / 32 && n0 + 32 * e.lane < args.N) {
    if (args.mode == kEpiResidNorm) {
      prefetch_l1(args.rn_gamma + n0 + 32 * e.lane);
      prefetch_l1(args.rn_beta + n0 + 32 * e.lane);
    } else {
      prefetch_l1(args.fold_colsum + n0 + 32 * e.lane);
    }
  }
}

// kEpiResidNorm: before the accumulator is ready, lane 0 of each epilogue
// warp pulls the fp16 residual chunks of its rows (at most two 32 x 32
// chunks per tile: one per staging half) into its staging tile by TMA.
template <int BN, int EW>
__device__ __forceinline__ void resid_issue(const GemmArgs &args, EpiCtx &e, int row0, int n0,
                                            int group) {
  constexpr int STEP = 32 * (EW / 4);
  static_assert(BN / STEP <= 2, "at most two residual chunks per warp and tile");
  int nch = 0;
  for (int c = group * 32; c < BN && n0 + c < args.N; c += STEP) ++nch;
  if (nch == 0) return;
  if (e.lane == 0) {
    bulk_wait_read0();  // earlier stores have finished reading the staging tile
    mbar_arrive_expect_tx(e.res_bar, static_cast<uint32_t>(nch) * (kStageBytes / 2));
    int i = 0;
    for (int c = group * 32; c < BN && n0 + c < args.N; c += STEP, ++i)
      tma_load_2d(e.stage + i * (kStageBytes / 2), e.res, e.res_bar, n0 + c, row0);
  }
  ++e.res_issued;
}

// Profiling counters (args.trace, 8 values, summed over all CTAs with
// atomics): 0 epilogue cycles waiting for an accumulator, 1 epilogue cycles
// processing tiles, 2 MMA-issuer cycles waiting for a free accumulator,
// 3 MMA-issuer cycles waiting for operands, 4 producer cycles waiting for a
// free stage, 5 CTA cycles from start to end, 6 epilogue tiles (per warp),
// 7 producer cycles issuing loads.
__device__ __forceinline__ long long trace_clock(const GemmArgs &a) {
  return a.trace ? clock64() : 0;
}
__device__ __forceinline__ void gemm_trace_add(const GemmArgs &a, int i, long long v) {
  if (a.trace && v) atomicAdd(a.trace + i, static_cast<unsigned long long>(v));
}

__device__ __forceinline__ unsigned long long wait_limit(const GemmArgs &a) {
  return a.wait_ns ? a.wait_ns : kWaitLimitNs;
}

// An epilogue warp that stopped early waits (bounded) for a residual load it
// issued and never consumed before the CTA releases its shared memory.
__device__ __forceinline__ void resid_drain(const GemmArgs &args, EpiCtx &e) {
  if (args.mode != kEpiResidNorm || e.res_issued == e.res_loads) return;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(e.res_bar, e.res_loads & 1)) {
    if (global_ns() - t0 > wait_limit(args)) {
      atomicCAS(args.status, 0u, static_cast<unsigned>(kErrTimeoutDrain));
      break;
    }
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2_f(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&h);
}

__device__ __forceinline__ uint32_t pack_f16x2_f(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&h);
}

// Round to the nearest integer (ties to even) and saturate to [-127, 127].
__device__ __forceinline__ int quant_s8(float x) {
  const int r = __float2int_rn(x);
  return r > 127 ? 127 : (r < -127 ? -127 : r);
}

__device__ __forceinline__ void stage_row(const GemmArgs &args, uint8_t *st, int r,
                                          const float (&v)[32], bool f32, float out_is) {
  if (f32) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      *reinterpret_cast<float4 *>(st + r * 128 + ((q ^ (r & 7)) << 4)) =
          make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else if (args.out_fp8) {
    const float is = out_is;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t x = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint32_t byte;
          if (args.out_i8) {
            byte = static_cast<uint32_t>(quant_s8(v[16 * q + 4 * k + e] * is)) & 0xFFu;
          } else {
            const __nv_fp8_e4m3 f(v[16 * q + 4 * k + e] * is);
            byte = f.__x;
          }
          x |= byte << (8 * e);
        }
        w[k] = x;
      }
      *reinterpret_cast<uint4 *>(st + r * 32 + ((q ^ ((r >> 2) & 1)) << 4)) =
          make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else if (args.out_f16) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4 *>(st + r * 64 + ((q ^ ((r >> 1) & 3)) << 4)) =
          make_uint4(pack_f16x2_f(v[8 * q], v[8 * q + 1]), pack_f16x2_f(v[8 * q + 2], v[8 * q + 3]),
                     pack_f16x2_f(v[8 * q + 4], v[8 * q + 5]), pack_f16x2_f(v[8 * q + 6], v[8 * q + 7]));
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4 *>(st + r * 64 + ((q ^ ((r >> 1) & 3)) << 4)) =
          make_uint4(pack_bf16x2_f(v[8 * q], v[8 * q + 1]), pack_bf16x2_f(v[8 * q + 2], v[8 * q + 3]),
                     pack_bf16x2_f(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2_f(v[8 * q + 6], v[8 * q + 7]));
  }
}

// The chunks of one tile owned by this warp (every other 32-column chunk,
// starting at `group`*32), with the TMEM load of the next chunk in flight
// while the current one is processed. Returns false on a barrier timeout.
template <int BN, int MODE, int ACT, int EW, bool OP8>
__device__ __forceinline__ bool epilogue_tile(const GemmArgs &args, EpiCtx &e, uint32_t taddr,
                                              int row0, int n0, int group, int ks) {
  constexpr int STEP = 32 * (EW / 4);  // columns between this warp's chunks
  const int lane = e.lane;
  const bool f32 = ks >= 0 || args.out_f32;
  const float a_scale = args.a_scale_ptr ? args.a_scale * __ldg(args.a_scale_ptr) : args.a_scale;
  const float out_is = args.out_scale_ptr ? 1.0f / __ldg(args.out_scale_ptr) : args.out_inv_scale;
  // With 8 epilogue warps the TMEM load of the next chunk is issued before
  // the current one is processed; with 16 the other warps hide that latency
  // and the registers of a second chunk are not available.
  constexpr bool PREFETCH = EW <= 8;
  uint32_t raw[32];
  int c = group * 32;
  if (c >= BN) return true;
  // consumer side of the deferred LayerNorm: this row's statistics
  const bool fold = MODE == kEpiStore && ks < 0 && args.fold_stats != nullptr;
  const float f_mean = fold ? e.rowst.x : 0.0f, f_rstd = fold ? e.rowst.y : 1.0f;
  // kEpiResidNorm: the residual chunks (prefetched by resid_issue into staging
  // halves 0 and 1) have landed; each lane later reads its own row of a chunk
  // and overwrites the same bytes with its output row, so the chunk is staged
  // for its store in place
  float r_mean = 0.0f, r_rstd = 1.0f;
  if constexpr (MODE == kEpiResidNorm) {
    if (e.res_issued != e.res_loads) {
      if (!mbar_wait(e.res_bar, e.res_loads & 1, args.status, kErrTimeoutEpilogue, e.abort_flag, wait_limit(args)))
        return false;
      ++e.res_loads;
    }
    if (args.rn_stats) {
      r_mean = e.rowst.x;
      r_rstd = e.rowst.y;
    }
  }
  int ci = 0;  // this warp's chunk index within the tile
  if (PREFETCH) tmem_ld32(taddr + c, raw);
  for (; c < BN; c += STEP, ++ci) {
    if (!PREFETCH) tmem_ld32(taddr + c, raw);
    tmem_wait_ld();
    float v[32];
    if (OP8 && args.ab_i8) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = static_cast<float>(static_cast<int>(raw[j]));
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]);
    }
    if (PREFETCH && c + STEP < BN) tmem_ld32(taddr + c + STEP, raw);  // warp-collective prefetch
    const int nb = n0 + c;
    if (nb >= args.N) continue;
    // A chunk of 2- or 1-byte outputs fills at most half of the 4 KB tile, so
    // the two halves alternate and only the store before last must have
    // finished reading; fp32 chunks (and residual tiles) use the whole tile.
    const bool halves = !f32 && MODE != kEpiResid;
    uint8_t *st = MODE == kEpiResidNorm ? e.stage + ci * (kStageBytes / 2)
                                        : (halves ? e.stage + (e.chunks & 1u) * (kStageBytes / 2) : e.stage);
    ++e.chunks;
    if (MODE != kEpiResidNorm) {  // (residual-norm: resid_issue waited for all earlier stores)
      if (lane == 0) {
        if (halves) bulk_wait_read1(); else bulk_wait_read0();
      }
      __syncwarp();
    }
    if (ks < 0) {
      const float as = (OP8 && args.a_row_scale) ? a_scale * e.arow : a_scale;
      if (as != 1.0f) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] *= as;
      }
      if (fold) {
        const float4 *cs = reinterpret_cast<const float4 *>(args.fold_colsum + nb);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 f = __ldg(cs + q);
          v[4 * q] = f_rstd * (v[4 * q] - f_mean * f.x);
          v[4 * q + 1] = f_rstd * (v[4 * q + 1] - f_mean * f.y);
          v[4 * q + 2] = f_rstd * (v[4 * q + 2] - f_mean * f.z);
          v[4 * q + 3] = f_rstd * (v[4 * q + 3] - f_mean * f.w);
        }
      }
      if (args.col_scale) {
        const float4 *cs = reinterpret_cast<const float4 *>(args.col_scale + nb);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 f = __ldg(cs + q);
          v[4 * q] *= f.x; v[4 * q + 1] *= f.y; v[4 * q + 2] *= f.z; v[4 * q + 3] *= f.w;
        }
      }
      if (args.bias) {
        const float4 *bp = reinterpret_cast<const float4 *>(args.bias + nb);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 f = __ldg(bp + q);
          v[4 * q] += f.x; v[4 * q + 1] += f.y; v[4 * q + 2] += f.z; v[4 * q + 3] += f.w;
        }
      }
    }
    if constexpr (MODE == kEpiAccum) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= args.alpha;
    } else if constexpr (MODE == kEpiResidNorm) {
      // y = LN_prev(r) + alpha * v (stored as fp16 by stage_row) and this
      // chunk's statistics of y (fp32, before the rounding to fp16)
      float s = 0.0f, sq = 0.0f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 w = *reinterpret_cast<const uint4 *>(st + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4));
        const uint32_t w4[4] = {w.x, w.y, w.z, w.w};
        float r[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w4[k]));
          r[2 * k] = f.x;
          r[2 * k + 1] = f.y;
        }
        if (args.rn_stats) {
          const float4 *gp = reinterpret_cast<const float4 *>(args.rn_gamma + nb + 8 * q);
          const float4 *bp = reinterpret_cast<const float4 *>(args.rn_beta + nb + 8 * q);
          const float4 g0 = __ldg(gp), g1 = __ldg(gp + 1), b0 = __ldg(bp), b1 = __ldg(bp + 1);
          const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
          const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
          for (int k = 0; k < 8; ++k) r[k] = (r[k] - r_mean) * r_rstd * g[k] + b[k];
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int j = 8 * q + k;
          v[j] = r[k] + args.alpha * v[j];
          s += v[j];
          sq += v[j] * v[j];
        }
      }
      // chunk sum of squared deviations from the chunk mean
      const float m2 = fmaxf(sq - s * s * (1.0f / 32.0f), 0.0f);
      if (row0 + lane < args.M)
        args.stats_out[static_cast<long long>(nb / 32) * args.M + row0 + lane] = make_float2(s, m2);
    } else if constexpr (MODE == kEpiResid) {
      if (lane == 0) {
        mbar_arrive_expect_tx(e.res_bar, kStageBytes);
        tma_load_2d(e.stage, e.res, e.res_bar, nb, row0);
      }
      if (!mbar_wait(e.res_bar, e.res_loads & 1, args.status, kErrTimeoutEpilogue, e.abort_flag, wait_limit(args)))
        return false;
      ++e.res_loads;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 rv =
            *reinterpret_cast<const float4 *>(e.stage + lane * 128 + ((q ^ (lane & 7)) << 4));
        v[4 * q] = rv.x + args.alpha * v[4 * q];
        v[4 * q + 1] = rv.y + args.alpha * v[4 * q + 1];
        v[4 * q + 2] = rv.z + args.alpha * v[4 * q + 2];
        v[4 * q + 3] = rv.w + args.alpha * v[4 * q + 3];
      }
      __syncwarp();  // every lane has read its residual row before the tile is overwritten
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = act_t<ACT>(v[j]);
    }
    stage_row(args, st, lane, v, f32, out_is);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (MODE == kEpiAccum)
        tma_reduce_add_2d(e.out, st, nb, row0);
      else if (ks >= 0)
        tma_store_3d(e.out, st, nb, row0, ks);
      else if (args.out2 && nb >= args.split)
        tma_store_2d(e.out2, st, nb - args.split, row0);
      else
        tma_store_2d(e.out, st, nb, row0);
      bulk_commit();
    }
  }
  return true;
}

// Residual + LayerNorm epilogue (the reference's LN(parent + alpha*x),
// src/nn/cpu/cpu_network.cpp:424-460, one-pass fp32 statistics).
// In LN kernels the eight epilogue warps form two teams of four (one warp per
// TMEM lane quarter); team t handles every other tile, in accumulator t, so
// one team's memory traffic overlaps the other's. Each warp covers all BN
// columns of its 32 rows.
// Pass 1, per 32-column chunk of this lane's row: y = resid + alpha*(scale*acc
// + bias) with the residual read once (vector loads, next chunk in flight),
// row sum and sum of squares accumulated, and y written back over the
// accumulator's own TMEM columns. The row statistics are then published:
// each thread writes its row's partial to row_stats[row][rank]; after a
// __syncwarp one lane per warp arrives (release, cluster scope) on the team's
// barrier in every cluster CTA; once it completes (acquire) each thread sums
// the cluster_n partials of its row. Pass 2 reads y back from TMEM, normalises
// it and TMA-stores an fp32 copy (`out`, the next residual parent) and a
// bf16 / e4m3 copy (`out2`, the next GEMM's input).
template <int BN>
__device__ __forceinline__ bool epilogue_tile_ln(const GemmArgs &args, EpiCtx &e, uint32_t taddr,
                                                 int row0, int n0) {
  const int lane = e.lane;
  const int row = row0 + lane;
  const int rrow = row < args.M ? row : args.M - 1;  // clamp loads of rows past M
  const float a_scale = args.a_scale_ptr ? args.a_scale * __ldg(args.a_scale_ptr) : args.a_scale;
  const float out_is = args.out_scale_ptr ? 1.0f / __ldg(args.out_scale_ptr) : args.out_inv_scale;
  const int C = args.cluster_n;
  const float *rbase = args.resid + static_cast<long long>(rrow) * args.ldr;
  float s = 0.0f, sq = 0.0f;
  float4 rv[8];
  {
    const float4 *rp = reinterpret_cast<const float4 *>(rbase + n0);
#pragma unroll
    for (int q = 0; q < 8; ++q) rv[q] = __ldg(rp + q);
  }
  for (int c = 0; c < BN; c += 32) {
    const int nb = n0 + c;
    uint32_t raw[32];
    tmem_ld32(taddr + c, raw);
    float4 cur[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) cur[q] = rv[q];
    if (c + 32 < BN) {  // next chunk's residual in flight
      const float4 *rp = reinterpret_cast<const float4 *>(rbase + nb + 32);
#pragma unroll
      for (int q = 0; q < 8; ++q) rv[q] = __ldg(rp + q);
    }
    tmem_wait_ld();
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]) * a_scale;
    if (args.col_scale) {
      const float4 *cs = reinterpret_cast<const float4 *>(args.col_scale + nb);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 f = __ldg(cs + q);
        v[4 * q] *= f.x; v[4 * q + 1] *= f.y; v[4 * q + 2] *= f.z; v[4 * q + 3] *= f.w;
      }
    }
    const float4 *bp = reinterpret_cast<const float4 *>(args.bias + nb);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 b = args.bias ? __ldg(bp + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[4 * q] = cur[q].x + args.alpha * (v[4 * q] + b.x);
      v[4 * q + 1] = cur[q].y + args.alpha * (v[4 * q + 1] + b.y);
      v[4 * q + 2] = cur[q].z + args.alpha * (v[4 * q + 2] + b.z);
      v[4 * q + 3] = cur[q].w + args.alpha * (v[4 * q + 3] + b.w);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      s += v[j];
      sq += v[j] * v[j];
      raw[j] = __float_as_uint(v[j]);
    }
    tmem_st32(taddr + c, raw);
  }
  tmem_wait_st();
  // publish this thread's partial and signal every CTA of the cluster
  if (row < args.M)
    args.row_stats[static_cast<long long>(row) * C + e.rank] = make_float2(s, sq);
  const uint32_t bar = smem_u32(e.xbar);
  // __syncwarp orders the lanes' writes before lane 0's (cumulative) release
  __syncwarp();
  if (lane == 0)
    for (int p = 0; p < C; ++p) mbar_arrive_remote(mapa_shared(bar, static_cast<uint32_t>(p)));
  if (!mbar_wait_cluster(e.xbar, e.xtiles & 1, args.status, kErrTimeoutRowStats, e.abort_flag, wait_limit(args)))
    return false;
  ++e.xtiles;
  float ts = 0.0f, tq = 0.0f;
  {
    const float2 *rs = args.row_stats + static_cast<long long>(rrow) * C;
    for (int k = 0; k < C; ++k) {
      const float2 x = __ldcg(rs + k);  // L2: written by other SMs
      ts += x.x;
      tq += x.y;
    }
  }
  const float mean = ts / static_cast<float>(args.N);
  float var = tq / static_cast<float>(args.N) - mean * mean;
  var = var < 0.0f ? 0.0f : var;
  const float rstd = 1.0f / sqrtf(var + args.ln_eps);
  uint32_t raw[32];
  tmem_ld32(taddr, raw);
  for (int c = 0; c < BN; c += 32) {
    const int nb = n0 + c;
    tmem_wait_ld();
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]);
    if (c + 32 < BN) tmem_ld32(taddr + c + 32, raw);
    const float4 *gp = reinterpret_cast<const float4 *>(args.ln_gamma + nb);
    const float4 *bp = reinterpret_cast<const float4 *>(args.ln_beta + nb);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 g = __ldg(gp + q), b = __ldg(bp + q);
      v[4 * q] = (v[4 * q] - mean) * rstd * g.x + b.x;
      v[4 * q + 1] = (v[4 * q + 1] - mean) * rstd * g.y + b.y;
      v[4 * q + 2] = (v[4 * q + 2] - mean) * rstd * g.z + b.z;
      v[4 * q + 3] = (v[4 * q + 3] - mean) * rstd * g.w + b.w;
    }
    // two staging tiles (LN kernels): the fp32 and the bf16/e4m3 copies go
    // out through different tiles, so only the store two back must have
    // finished reading before a tile is rewritten
    if (lane == 0) bulk_wait_read1();
    __syncwarp();
    stage_row(args, e.stage, lane, v, true, out_is);  // fp32 copy
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(e.out, e.stage, nb, row0);
      bulk_commit();
    }
    if (args.out2) {
      if (lane == 0) bulk_wait_read1();
      __syncwarp();
      stage_row(args, e.stage2, lane, v, false, out_is);  // bf16 / e4m3 copy
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(e.out2, e.stage2, nb, row0);
        bulk_commit();
      }
    }
  }
  return true;
}

// Epilogue selector, a template parameter of the GEMM kernels: 0-7 the store
// epilogue with that activation (kAct*), then the residual, accumulate and
// residual-norm modes. Each kernel instance carries only its own epilogue:
// with every variant behind a runtime switch the kernel's code was large
// enough that instruction fetch stalled its epilogue warps (measured: the
// K = 256 generator shape 11% and the e4m3 N = 1024 shape 7% slower).
enum EpiSel : int { kSelResid = 8, kSelAccum = 9, kSelResidNorm = 10, kSelCount = 11 };

__host__ __device__ constexpr int epi_select(int mode, int act, int k_splits) {
  return k_splits > 1 ? static_cast<int>(kActNone)
                      : (mode == kEpiResid ? kSelResid
                                           : (mode == kEpiAccum ? kSelAccum
                                                                : (mode == kEpiResidNorm ? kSelResidNorm : act)));
}

template <int BN, bool LN, int EW, int EPI, bool OP8>
__device__ __forceinline__ bool epilogue_dispatch(const GemmArgs &args, EpiCtx &e, uint32_t taddr,
                                                  int row0, int n0, int group, int ks) {
  if constexpr (LN) {
    return epilogue_tile_ln<BN>(args, e, taddr, row0, n0);
  } else if constexpr (EPI == kSelResid) {
    return epilogue_tile<BN, kEpiResid, kActNone, EW, OP8>(args, e, taddr, row0, n0, group, ks);
  } else if constexpr (EPI == kSelAccum) {
    return epilogue_tile<BN, kEpiAccum, kActNone, EW, OP8>(args, e, taddr, row0, n0, group, ks);
  } else if constexpr (EPI == kSelResidNorm) {
    static_assert(EW == kEpiWarpsMax, "the residual-norm epilogue needs 16 epilogue warps");
    return epilogue_tile<BN, kEpiResidNorm, kActNone, EW, OP8>(args, e, taddr, row0, n0, group, ks);
  } else {
    return epilogue_tile<BN, kEpiStore, EPI, EW, OP8>(args, e, taddr, row0, n0, group, ks);
  }
}

template <int BN, bool FP8, bool LN = false>
struct GemmShape {
  static constexpr int BM = 128;
  static constexpr int BK = FP8 ? 128 : 64;  // elements per 128-byte swizzled row
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int EW = LN ? kEpiWarpsLN : kEpiWarpsMax;  // epilogue warps
  // LN kernels trade one pipeline stage for a second staging tile per warp;
  // the others give 64 KB to the 16 epilogue warps' staging tiles
  static constexpr int STAGES = LN ? (BN == 256 ? 3 : (BN == 128 ? 4 : 5))
                                   : (BN == 256 ? 3 : (BN == 128 ? 5 : 6));
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int STAGE_BYTES = (LN ? 2 : 1) * EW * kStageBytes;  // epilogue staging
  static constexpr int SMEM_BYTES = STAGES * (A_BYTES + B_BYTES) + STAGE_BYTES + 1024 + 512;
  static constexpr int THREADS = 64 + 32 * EW;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

template <int BN, bool FP8, bool LN, int EPI>
__global__ void __launch_bounds__(64 + 32 * (LN ? kEpiWarpsLN : kEpiWarpsMax), 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmOut,
                      const __grid_constant__ CUtensorMap tmOut2,
                      const __grid_constant__ CUtensorMap tmRes, const GemmArgs args) {
  using S = GemmShape<BN, FP8, LN>;
  constexpr int STAGES = S::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *smA = base;
  uint8_t *smB = base + STAGES * S::A_BYTES;
  uint8_t *stage_base = smB + STAGES * S::B_BYTES;
  uint64_t *full = reinterpret_cast<uint64_t *>(smB + STAGES * S::B_BYTES + S::STAGE_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *tfull = empty + STAGES;
  uint64_t *tempty = tfull + 2;
  uint64_t *res_bars = tempty + 2;  // one per epilogue warp
  uint64_t *drain = res_bars + S::EW;
  uint64_t *xbar = drain + 1;  // row-statistics exchange, one per LN team
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(xbar + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (args.M + S::BM - 1) / S::BM;
  const int tiles_n = (args.N + BN - 1) / BN;
  const int splits = args.k_splits > 1 ? args.k_splits : 1;
  const int units = tiles_m * tiles_n * splits;
  const int kblocks = (args.K + S::BK - 1) / S::BK;
  const int kb_per = (kblocks + splits - 1) / splits;
  // Work units: normally u enumerates (tile, K slice) pairs over the whole
  // grid; with the LayerNorm epilogue the CTAs of one cluster walk the same
  // row blocks, CTA `rank` owning column block `rank`.
  constexpr bool ln = LN;  // launched for args.mode == kEpiResidLN
  const int C = ln ? args.cluster_n : 1;
  const uint32_t rank = ln ? cluster_ctarank() : 0u;
  const int u_begin = ln ? static_cast<int>(blockIdx.x) / C : static_cast<int>(blockIdx.x);
  const int u_step = ln ? static_cast<int>(gridDim.x) / C : static_cast<int>(gridDim.x);
  const int u_end = ln ? tiles_m : units;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], LN ? 32 * S::EW / 2 : 32 * S::EW);
    }
    for (int w = 0; w < S::EW; ++w) mbar_init(&res_bars[w], 1);
    mbar_init(drain, 1);
    mbar_init(&xbar[0], static_cast<uint32_t>(C * S::EW / 2));
    mbar_init(&xbar[1], static_cast<uint32_t>(C * S::EW / 2));
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (ln) cluster_sync();  // peers' barriers are initialised before any remote arrive
  const uint32_t tmem_base = *tmem_slot;
  // Weight tiles do not depend on the previous kernel: the producer announces
  // the first stages of its first work unit and loads their W tiles before
  // the grid-dependency wait, so that their latency overlaps the previous
  // kernel's tail (small batches, where a GEMM follows a short kernel whose
  // CTAs leave room for this one's). A tiles, outputs and everything else
  // are touched only after the wait.
  int pre = 0;  // stages whose W tile is already in flight
  if (warp == 0 && lane == 0 && u_begin < u_end &&
      !(args.debug_withhold && blockIdx.x == 0)) {
    const int t = ln ? u_begin * tiles_n + static_cast<int>(rank) : u_begin / splits;
    const int ks = ln ? 0 : u_begin % splits;
    const int n0 = (t % tiles_n) * BN;
    const int kb0 = ks * kb_per, kb1 = min(kblocks, (ks + 1) * kb_per);
    pre = min(STAGES, max(0, kb1 - kb0));
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], S::A_BYTES + S::B_BYTES);
      tma_load_2d(smB + i * S::B_BYTES, &tmB, &full[i], (kb0 + i) * S::BK, n0);
    }
  }
  pdl_wait();
  pdl_launch();
  const long long t_start = trace_clock(args);
  long long tr_a = 0, tr_b = 0, tr_c = 0;  // per-role trace sums

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int stage = 0;
      uint32_t round = 0;
      long long issued = 0;
      bool ok = true;
      for (int u = u_begin; u < u_end && ok; u += u_step) {
        const int t = ln ? u * tiles_n + static_cast<int>(rank) : u / splits;
        const int ks = ln ? 0 : u % splits;
        const int m0 = (t / tiles_n) * S::BM;
        const int n0 = (t % tiles_n) * BN;
        const int kb1 = min(kblocks, (ks + 1) * kb_per);
        if (ln) {
          // pull this tile's residual into L2 while its mainloop runs
          for (int y = m0; y < min(m0 + S::BM, args.M); y += 32)
            for (int x = n0; x < min(n0 + BN, args.N); x += 32) tma_prefetch_l2_2d(&tmRes, x, y);
        }
        for (int kb = ks * kb_per; kb < kb1; ++kb) {
          if (issued < pre) {  // W already in flight (announced before the wait)
            tma_load_2d(smA + stage * S::A_BYTES, &tmA, &full[stage], kb * S::BK, m0);
            ++issued;
            if (++stage == STAGES) { stage = 0; ++round; }
            continue;
          }
          const long long tw = trace_clock(args);
          const bool got = mbar_wait(&empty[stage], (round & 1) ^ 1, args.status, kErrTimeoutProducer,
                         abort_flag, wait_limit(args));
          tr_a += trace_clock(args) - tw;
          if (!got) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], S::A_BYTES + S::B_BYTES);
          // (tests: the first stage of CTA 0 is announced but never loaded)
          if (!(args.debug_withhold && blockIdx.x == 0 && issued == 0)) {
            tma_load_2d(smA + stage * S::A_BYTES, &tmA, &full[stage], kb * S::BK, m0);
            tma_load_2d(smB + stage * S::B_BYTES, &tmB, &full[stage], kb * S::BK, n0);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; ++round; }
        }
      }
      if (!ok) {
        // Drain: let every load still in flight land before the CTA exits.
        const long long first = issued > STAGES ? issued - STAGES : 0;
        for (long long i = first; i < issued; ++i) {
          const unsigned long long t0 = global_ns();
          while (!mbar_try_wait(&full[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1))) {
            if (global_ns() - t0 > wait_limit(args)) {
              atomicCAS(args.status, 0u, static_cast<unsigned>(kErrTimeoutDrain));
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issuer
      const bool i8 = FP8 && args.ab_i8;
      const uint32_t idesc = FP8 ? (i8 ? umma_idesc_s8(128, BN) : umma_idesc(128, BN, kFmtE4M3, kFmtE4M3))
                                 : (args.ab_f16 ? umma_idesc(128, BN, kFmtF16, kFmtF16)
                                                : umma_idesc(128, BN, kFmtBF16, kFmtBF16));
      int stage = 0;
      uint32_t round = 0;
      int local = 0;
      bool ok = true;
      for (int u = u_begin; u < u_end && ok; u += u_step, ++local) {
        const int ks = ln ? 0 : u % splits;
        const int acc = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        const long long tw = trace_clock(args);
        const bool got = mbar_wait(&tempty[acc], aphase ^ 1, args.status, kErrTimeoutMma, abort_flag, wait_limit(args));
        tr_a += trace_clock(args) - tw;
        if (!got) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        const int kb0 = ks * kb_per, kb1 = min(kblocks, kb0 + kb_per);
        for (int kb = kb0; kb < kb1; ++kb) {
          const long long tw = trace_clock(args);
          const bool got = mbar_wait(&full[stage], round & 1, args.status, kErrTimeoutMma, abort_flag, wait_limit(args));
          tr_b += trace_clock(args) - tw;
          if (!got) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_kmajor_desc(smem_u32(smA + stage * S::A_BYTES));
          const uint64_t bd = sw128_kmajor_desc(smem_u32(smB + stage * S::B_BYTES));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            // advance 32 bytes along K inside the 128-byte swizzled row
            const uint32_t accumulate = (kb > kb0 || kk > 0) ? 1u : 0u;
            if (FP8 && i8)
              umma_i8(d, ad + 2 * kk, bd + 2 * kk, idesc, accumulate);
            else if (FP8)
              umma_f8(d, ad + 2 * kk, bd + 2 * kk, idesc, accumulate);
            else
              umma_f16(d, ad + 2 * kk, bd + 2 * kk, idesc, accumulate);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; ++round; }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
      if (!ok) {
        // Aborted: wait (bounded) until every MMA already issued has retired
        // before the TMEM is released.
        umma_commit(drain);
        const unsigned long long t0 = global_ns();
        while (!mbar_try_wait(drain, 0)) {
          if (global_ns() - t0 > wait_limit(args)) {
            atomicCAS(args.status, 0u, static_cast<unsigned>(kErrTimeoutDrain));
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;        // TMEM lane quarter this warp may access
    const int group = (warp - 2) >> 2;   // which alternate 32-column chunks
    EpiCtx e{&tmOut, &tmOut2, &tmRes, stage_base + (warp - 2) * kStageBytes, &res_bars[warp - 2],
             0u, lane, abort_flag, &xbar[group], 0u, rank,
             LN ? stage_base + (S::EW + warp - 2) * kStageBytes : nullptr, 0u};
    if (lane == 0) {
      tma_prefetch_desc(&tmOut);
      if (args.out2) tma_prefetch_desc(&tmOut2);
      if (args.mode == kEpiResid || args.mode == kEpiResidNorm) tma_prefetch_desc(&tmRes);
    }
    int local = 0;
    for (int u = u_begin; u < u_end; u += u_step, ++local) {
      if (ln && (local & 1) != group) continue;  // LN: team `group` takes every other tile
      const int t = ln ? u * tiles_n + static_cast<int>(rank) : u / splits;
      const int ks = (!ln && splits > 1) ? u % splits : -1;
      const int acc = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      const int m0 = (t / tiles_n) * S::BM;
      const int n0 = (t % tiles_n) * BN;
      if (ks < 0 && lane < BN / 32 && n0 + 32 * lane < args.N) {
        // the tile's bias / column scales (one 128-byte line per 32 columns)
        // reach L1 while the accumulator is still being computed
        if (args.bias) prefetch_l1(args.bias + n0 + 32 * lane);
        if (args.col_scale) prefetch_l1(args.col_scale + n0 + 32 * lane);
      }
      if constexpr (!LN) {
        if (ks < 0 && args.mode == kEpiResidNorm)
          resid_issue<BN, S::EW>(args, e, m0 + quarter * 32, n0, group);
        if (ks < 0) epi_pre(args, e, m0 + quarter * 32, n0, BN);
      }
      const long long tw = trace_clock(args);
      const bool got = mbar_wait(&tfull[acc], aphase, args.status, kErrTimeoutEpilogue, abort_flag, wait_limit(args));
      tr_a += trace_clock(args) - tw;
      if (!got) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const long long te = trace_clock(args);
      const bool ok = epilogue_dispatch<BN, LN, S::EW, EPI, FP8>(args, e, taddr, m0 + quarter * 32, n0, group, ks);
      tr_b += trace_clock(args) - te;
      tr_c += 1;
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (!ok) break;
    }
    resid_drain(args, e);
    if (lane == 0) bulk_wait0();  // all TMA stores of this warp have landed
  }

  if (args.trace && lane == 0) {
    if (warp == 0) {
      gemm_trace_add(args, 4, tr_a);
    } else if (warp == 1) {
      gemm_trace_add(args, 2, tr_a);
      gemm_trace_add(args, 3, tr_b);
    } else {
      gemm_trace_add(args, 0, tr_a);
      gemm_trace_add(args, 1, tr_b);
      gemm_trace_add(args, 6, tr_c);
    }
    if (threadIdx.x == 0) gemm_trace_add(args, 5, trace_clock(args) - t_start);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
  if (ln) cluster_sync();  // no CTA leaves while a peer may still signal it
}

// ---------------------------------------------------------------------------
// CTA-pair GEMM (tcgen05 .cta_group::2). A cluster of two CTAs owns a
// 256 x 256 output tile: CTA r stages rows [128r, 128r+128) of the A tile and
// rows [128r, 128r+128) of the W tile (half of the tile's N) in its shared
// memory, rank 0 issues M=256 N=256 MMAs that read both CTAs' operands, and
// each CTA's TMEM receives its own 128 rows x 256 columns. Per SM this halves
// the W bytes staged and read by the tensor core (32 KB per K step instead of
// 48 KB), which leaves room for six pipeline stages. Roles as in
// gemm_sm100_kernel; the producer of each CTA loads its halves and counts the
// bytes on rank 0's `full` barrier, rank 0's commits arrive on both CTAs'
// `empty` / `tfull` barriers, and every epilogue warp of both CTAs arrives on
// rank 0's `tempty` barrier. Store / accumulate / residual epilogues, no
// split-K.
template <bool FP8>
struct PairShape {
  static constexpr int BM = 128;                 // rows per CTA (256 per pair)
  static constexpr int BN = 256;                 // columns per tile
  static constexpr int BK = FP8 ? 128 : 64;
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = (BN / 2) * 128; // this CTA's half of W
  static constexpr int EW = kEpiWarpsMax;         // epilogue warps
  static constexpr int STAGES = 5;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int STAGE_BYTES = EW * kStageBytes;
  static constexpr int SMEM_BYTES = STAGES * (A_BYTES + B_BYTES) + STAGE_BYTES + 1024 + 256;
  static constexpr int THREADS = 64 + 32 * EW;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

template <bool FP8, int EPI>
__global__ void __launch_bounds__(64 + 32 * kEpiWarpsMax, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmOut,
                     const __grid_constant__ CUtensorMap tmOut2,
                     const __grid_constant__ CUtensorMap tmRes, const GemmArgs args) {
  using S = PairShape<FP8>;
  constexpr int STAGES = S::STAGES;
  constexpr int BN = S::BN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *smA = base;
  uint8_t *smB = base + STAGES * S::A_BYTES;
  uint8_t *stage_base = smB + STAGES * S::B_BYTES;
  uint64_t *full = reinterpret_cast<uint64_t *>(stage_base + S::STAGE_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *tfull = empty + STAGES;
  uint64_t *tempty = tfull + 2;
  uint64_t *res_bars = tempty + 2;
  uint64_t *drain = res_bars + S::EW;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int tiles_m = (args.M + 2 * S::BM - 1) / (2 * S::BM);
  const int tiles_n = (args.N + BN - 1) / BN;
  const int units = tiles_m * tiles_n;
  const int kblocks = (args.K + S::BK - 1) / S::BK;
  const int u_begin = static_cast<int>(blockIdx.x >> 1);
  const int u_step = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * S::EW);  // one arrive per epilogue warp of the pair
    }
    for (int w = 0; w < S::EW; ++w) mbar_init(&res_bars[w], 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive or load
  const uint32_t tmem_base = *tmem_slot;
  // (no W loads before the wait here, unlike gemm_sm100_kernel: measured
  // slower at batch 32 and 1024, where a pair kernel follows a kernel whose
  // CTAs it cannot share an SM with)
  pdl_wait();
  pdl_launch();
  const long long t_start = trace_clock(args);
  long long tr_a = 0, tr_b = 0, tr_c = 0;  // per-role trace sums

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int stage = 0;
      uint32_t round = 0;
      long long issued = 0;
      bool ok = true;
      for (int u = u_begin; u < units && ok; u += u_step) {
        const int m0 = (u / tiles_n) * 2 * S::BM + static_cast<int>(rank) * S::BM;
        const int nb0 = (u % tiles_n) * BN + static_cast<int>(rank) * (BN / 2);
        // (no L2 prefetch of the residual tile: the producer's prefetches
        // delayed its operand loads; measured 5% slower with them)
        for (int kb = 0; kb < kblocks; ++kb) {
          const long long tw = trace_clock(args);
          const bool got = mbar_wait(&empty[stage], (round & 1) ^ 1, args.status, kErrTimeoutProducer,
                         abort_flag, wait_limit(args));
          tr_a += trace_clock(args) - tw;
          if (!got) {
            ok = false;
            break;
          }
          const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (S::A_BYTES + S::B_BYTES));
          // (tests: the first stage of pair 0 is announced but never loaded)
          if (!(args.debug_withhold && (blockIdx.x >> 1) == 0 && issued == 0)) {
            tma_load_2d_pair(smA + stage * S::A_BYTES, &tmA, fb, kb * S::BK, m0);
            tma_load_2d_pair(smB + stage * S::B_BYTES, &tmB, fb, kb * S::BK, nb0);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; ++round; }
        }
      }
      if (!ok && rank == 0) {
        // Drain: the loads of both CTAs complete on rank 0's barriers.
        const long long first = issued > STAGES ? issued - STAGES : 0;
        for (long long i = first; i < issued; ++i) {
          const unsigned long long t0 = global_ns();
          while (!mbar_try_wait(&full[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1))) {
            if (global_ns() - t0 > wait_limit(args)) {
              atomicCAS(args.status, 0u, static_cast<unsigned>(kErrTimeoutDrain));
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------------------------------------------------- MMA issuer
      const bool i8 = FP8 && args.ab_i8;
      const uint32_t idesc = FP8 ? (i8 ? umma_idesc_s8(256, BN) : umma_idesc(256, BN, kFmtE4M3, kFmtE4M3))
                                 : (args.ab_f16 ? umma_idesc(256, BN, kFmtF16, kFmtF16)
                                                : umma_idesc(256, BN, kFmtBF16, kFmtBF16));
      int stage = 0;
      uint32_t round = 0;
      int local = 0;
      bool ok = true;
      bool issued_any = false;
      for (int u = u_begin; u < units && ok; u += u_step, ++local) {
        const int acc = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        const long long tw = trace_clock(args);
        const bool got = mbar_wait_cluster(&tempty[acc], aphase ^ 1, args.status, kErrTimeoutMma, abort_flag, wait_limit(args));
        tr_a += trace_clock(args) - tw;
        if (!got) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          const long long tw = trace_clock(args);
          const bool got = mbar_wait(&full[stage], round & 1, args.status, kErrTimeoutMma, abort_flag, wait_limit(args));
          tr_b += trace_clock(args) - tw;
          if (!got) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_kmajor_desc(smem_u32(smA + stage * S::A_BYTES));
          const uint64_t bd = sw128_kmajor_desc(smem_u32(smB + stage * S::B_BYTES));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t accumulate = (kb > 0 || kk > 0) ? 1u : 0u;
            if (FP8 && i8)
              umma_i8_pair(d, ad + 2 * kk, bd + 2 * kk, idesc, accumulate);
            else if (FP8)
              umma_f8_pair(d, ad + 2 * kk, bd + 2 * kk, idesc, accumulate);
            else
              umma_f16_pair(d, ad + 2 * kk, bd + 2 * kk, idesc, accumulate);
          }
          issued_any = true;
          umma_commit_pair_mc(&empty[stage], 0x3);
          if (++stage == STAGES) { stage = 0; ++round; }
        }
        if (ok) umma_commit_pair_mc(&tfull[acc], 0x3);
      }
      if (!ok && issued_any) {
        // Aborted: wait (bounded) until every MMA already issued has retired.
        umma_commit_pair(drain);
        const unsigned long long t0 = global_ns();
        while (!mbar_try_wait(drain, 0)) {
          if (global_ns() - t0 > wait_limit(args)) {
            atomicCAS(args.status, 0u, static_cast<unsigned>(kErrTimeoutDrain));
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int group = (warp - 2) >> 2;
    EpiCtx e{&tmOut, &tmOut2, &tmRes, stage_base + (warp - 2) * kStageBytes, &res_bars[warp - 2],
             0u, lane, abort_flag, nullptr, 0u, rank, nullptr, 0u};
    if (lane == 0) {
      tma_prefetch_desc(&tmOut);
      if (args.out2) tma_prefetch_desc(&tmOut2);
      if (args.mode == kEpiResid || args.mode == kEpiResidNorm) tma_prefetch_desc(&tmRes);
    }
    const uint32_t tempty0 = mapa_shared(smem_u32(&tempty[0]), 0);
    const uint32_t tempty1 = mapa_shared(smem_u32(&tempty[1]), 0);
    int local = 0;
    for (int u = u_begin; u < units; u += u_step, ++local) {
      const int acc = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      const int m0 = (u / tiles_n) * 2 * S::BM + static_cast<int>(rank) * S::BM;
      const int n0 = (u % tiles_n) * BN;
      if (lane < BN / 32 && n0 + 32 * lane < args.N) {
        if (args.bias) prefetch_l1(args.bias + n0 + 32 * lane);
        if (args.col_scale) prefetch_l1(args.col_scale + n0 + 32 * lane);
      }
      if (args.mode == kEpiResidNorm) resid_issue<BN, S::EW>(args, e, m0 + quarter * 32, n0, group);
      epi_pre(args, e, m0 + quarter * 32, n0, BN);
      const long long tw = trace_clock(args);
      const bool got = mbar_wait(&tfull[acc], aphase, args.status, kErrTimeoutEpilogue, abort_flag, wait_limit(args));
      tr_a += trace_clock(args) - tw;
      if (!got) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const long long te = trace_clock(args);
      const bool ok = epilogue_dispatch<BN, false, S::EW, EPI, FP8>(args, e, taddr, m0 + quarter * 32, n0, group, -1);
      tr_b += trace_clock(args) - te;
      tr_c += 1;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acc ? tempty1 : tempty0);
      if (!ok) break;
    }
    resid_drain(args, e);
    if (lane == 0) bulk_wait0();
  }

  if (args.trace && lane == 0) {
    if (warp == 0) {
      gemm_trace_add(args, 4, tr_a);
    } else if (warp == 1) {
      gemm_trace_add(args, 2, tr_a);
      gemm_trace_add(args, 3, tr_b);
    } else {
      gemm_trace_add(args, 0, tr_a);
      gemm_trace_add(args, 1, tr_b);
      gemm_trace_add(args, 6, tr_c);
    }
    if (threadIdx.x == 0) gemm_trace_add(args, 5, trace_clock(args) - t_start);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // rank 0's MMAs and both CTAs' loads are finished before release
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, S::TMEM_COLS);
  }
}

}  // namespace mfb200
