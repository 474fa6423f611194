// gemm_sm100.cuh -- persistent tcgen05/TMEM GEMM with fused epilogues.
//
//   C[M,N] = epilogue( A[M,K] . W[N,K]^T )
//
// A (activations) and W (weights, the reference's [out, in] layout) are both
// K-major in HBM. Each CTA owns a 128 x BN output tile at a time; the CTA is
// persistent over tiles (grid = number of SMs) and warp-specialised:
//   warp 0     TMA producer: one lane streams 128-byte-swizzled K slices of A
//              and W into a STAGES-deep shared-memory ring (no multicast);
//   warp 1     MMA issuer: allocates 2*BN TMEM columns (two fp32
//              accumulators, so the epilogue of tile i overlaps the MMAs of
//              tile i+1) and issues tcgen05.mma (M=128, N=BN, K=16 bf16 or
//              K=32 fp8 per instruction) from one lane;
//   warps 2-5  epilogue: tcgen05.ld the accumulator (TMEM lane = tile row),
//              apply scale / bias / activation / residual / row-LayerNorm and
//              store bf16 (or e4m3) to HBM.
// All barrier waits are bounded (sm100_ptx.cuh).
#pragma once
#include <cuda_fp8.h>

#include "sm100_ptx.cuh"

namespace mfb200 {

enum EpiMode : int {
  kEpiStore = 0,  // act(scale*acc + bias)
  kEpiResid = 1,  // resid + alpha * (scale*acc + bias)
  kEpiRowLN = 2,  // LN(act(scale*acc + bias)) over the full row (requires N == BN)
};

enum Act : int {
  kActNone = 0, kActRelu, kActRelu2, kActTanh, kActSigmoid, kActSwish, kActMish, kActSelu
};

// Activations of the reference CPU backend (src/nn/cpu/cpu_network.cpp:303-324),
// written with CUDA's own expf/tanhf/log1pf.
__device__ __forceinline__ float apply_act(float v, int act) {
  switch (act) {
  case kActRelu: return fmaxf(v, 0.0f);
  case kActRelu2: { const float r = fmaxf(v, 0.0f); return r * r; }
  case kActTanh: return tanhf(v);
  case kActSigmoid: return 1.0f / (1.0f + expf(-v));
  case kActSwish: return v / (1.0f + expf(-v));
  case kActMish: return v * tanhf(log1pf(expf(v)));
  case kActSelu: return 1.05070098f * (v > 0.0f ? v : 1.67326324f * (expf(v) - 1.0f));
  default: return v;
  }
}

struct GemmArgs {
  int M, N, K;
  int mode, act;
  const float *bias;          // [N] or nullptr
  void *out;                  // [M, ldo] bf16 (or e4m3 when out_fp8)
  long long ldo;
  void *out2;                 // columns n >= split go to out2[m, n - split]
  long long ldo2;
  int split;
  const float *resid;         // kEpiResid: fp32 residual parent [M, ldr]
  long long ldr;
  float alpha;
  const float *ln_gamma, *ln_beta;  // kEpiRowLN
  float ln_eps;
  const float *col_scale;     // per-output-channel scale (fp8 weights) or nullptr
  float a_scale;              // activation scale (fp8) ; 1 for bf16
  int out_f32;                // store fp32 instead of bf16
  int out_fp8;                // store e4m3 instead of bf16 ...
  float out_inv_scale;        // ... after multiplying by this
  unsigned *status;           // device status word
};

template <int BN, bool FP8>
struct GemmShape {
  static constexpr int BM = 128;
  static constexpr int BK = FP8 ? 128 : 64;        // elements per 128-byte swizzled row
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGES = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * (A_BYTES + B_BYTES) + 1024 + 256;
  static constexpr int THREADS = 192;
};

template <int BN, bool FP8>
__global__ void __launch_bounds__(192, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
  using S = GemmShape<BN, FP8>;
  constexpr int STAGES = S::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *smA = base;
  uint8_t *smB = base + STAGES * S::A_BYTES;
  uint64_t *full = reinterpret_cast<uint64_t *>(smB + STAGES * S::B_BYTES);
  uint64_t *empty = full + STAGES;
  uint64_t *tfull = empty + STAGES;
  uint64_t *tempty = tfull + 2;
  uint64_t *drain = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (args.M + S::BM - 1) / S::BM;
  const int tiles_n = (args.N + BN - 1) / BN;
  const int tiles = tiles_m * tiles_n;
  const int kblocks = (args.K + S::BK - 1) / S::BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
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
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      int stage = 0;
      uint32_t round = 0;
      long long issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int m0 = (t / tiles_n) * S::BM;
        const int n0 = (t % tiles_n) * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], (round & 1) ^ 1, args.status, kErrTimeoutProducer,
                         abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], S::A_BYTES + S::B_BYTES);
          tma_load_2d(smA + stage * S::A_BYTES, &tmA, &full[stage], kb * S::BK, m0);
          tma_load_2d(smB + stage * S::B_BYTES, &tmB, &full[stage], kb * S::BK, n0);
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
            if (global_ns() - t0 > kWaitLimitNs) {
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
      constexpr uint32_t idesc =
          FP8 ? umma_idesc(128, BN, kFmtE4M3, kFmtE4M3) : umma_idesc(128, BN, kFmtBF16, kFmtBF16);
      int stage = 0;
      uint32_t round = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t aphase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aphase ^ 1, args.status, kErrTimeoutMma, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], round & 1, args.status, kErrTimeoutMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_kmajor_desc(smem_u32(smA + stage * S::A_BYTES));
          const uint64_t bd = sw128_kmajor_desc(smem_u32(smB + stage * S::B_BYTES));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            // advance 32 bytes along K inside the 128-byte swizzled row
            if (FP8)
              umma_f8(d, ad + 2 * kk, bd + 2 * kk, idesc, (kb | kk) != 0);
            else
              umma_f16(d, ad + 2 * kk, bd + 2 * kk, idesc, (kb | kk) != 0);
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
          if (global_ns() - t0 > kWaitLimitNs) {
            atomicCAS(args.status, 0u, static_cast<unsigned>(kErrTimeoutDrain));
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int local = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t aphase = (local >> 1) & 1;
      if (!mbar_wait(&tfull[acc], aphase, args.status, kErrTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      const int m0 = (t / tiles_n) * S::BM;
      const int n0 = (t % tiles_n) * BN;
      const int row = m0 + row_in_tile;
      const bool row_ok = row < args.M;
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const float ascale = args.a_scale;

      float mean = 0.0f, inv_std = 1.0f;
      if (args.mode == kEpiRowLN) {
        // pass 1: row statistics over the whole tile (N == BN)
        float s = 0.0f, sq = 0.0f;
        for (int c = 0; c < BN; c += 16) {
          uint32_t r[16];
          tmem_ld16(taddr + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int n = n0 + c + j;
            float v = __uint_as_float(r[j]) * ascale;
            if (args.col_scale) v *= args.col_scale[n];
            if (args.bias) v += args.bias[n];
            v = apply_act(v, args.act);
            s += v;
            sq += v * v;
          }
        }
        mean = s / static_cast<float>(BN);
        float var = sq / static_cast<float>(BN) - mean * mean;
        var = var < 0.0f ? 0.0f : var;
        inv_std = 1.0f / sqrtf(var + args.ln_eps);
      }

      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + c, r);
        tmem_wait_ld();
        const int nb = n0 + c;
        if (!row_ok || nb >= args.N) continue;
        float v[16];
        float res[16];
        if (args.mode == kEpiResid) {
          const float4 *rp =
              reinterpret_cast<const float4 *>(args.resid + static_cast<long long>(row) * args.ldr + nb);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 f = rp[q];
            res[4 * q] = f.x;
            res[4 * q + 1] = f.y;
            res[4 * q + 2] = f.z;
            res[4 * q + 3] = f.w;
          }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int n = nb + j;
          float x = __uint_as_float(r[j]) * ascale;
          if (args.col_scale) x *= args.col_scale[n];
          if (args.bias) x += args.bias[n];
          if (args.mode == kEpiResid) {
            x = res[j] + args.alpha * x;
          } else {
            x = apply_act(x, args.act);
            if (args.mode == kEpiRowLN)
              x = (x - mean) * inv_std * args.ln_gamma[n] + args.ln_beta[n];
          }
          v[j] = x;
        }
        void *dst_base = args.out;
        long long ld = args.ldo;
        int col = nb;
        if (args.out2 && nb >= args.split) {
          dst_base = args.out2;
          ld = args.ldo2;
          col = nb - args.split;
        }
        if (args.out_f32) {
          float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(dst_base) + row * ld + col);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        } else if (args.out_fp8) {
          __nv_fp8_e4m3 *dst = static_cast<__nv_fp8_e4m3 *>(dst_base) + row * ld + col;
          uint32_t packed[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __nv_fp8_e4m3 f(v[q * 4 + e] * args.out_inv_scale);
              w |= static_cast<uint32_t>(f.__x) << (8 * e);
            }
            packed[q] = w;
          }
          *reinterpret_cast<uint4 *>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        } else {
          __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(dst_base) + row * ld + col;
          uint32_t packed[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * q], v[2 * q + 1]);
            packed[q] = *reinterpret_cast<const uint32_t *>(&h);
          }
          uint4 *d4 = reinterpret_cast<uint4 *>(dst);
          d4[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
          d4[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, S::TMEM_COLS);
  }
}

}  // namespace mfb200
