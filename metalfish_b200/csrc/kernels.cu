// kernels.cu -- memory-bound and small-matmul kernels of the BT4 forward.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <atomic>
#include <type_traits>

#include "gemm_sm100.cuh"
#include "../../include/mfb200.h"
#include "kernels.cuh"
#include "pdl.cuh"

namespace mfb200 {

namespace {
std::atomic<bool> g_pdl{true};
}
bool pdl_enabled() { return g_pdl; }
void set_pdl(bool enable) { g_pdl = enable; }


// ------------------------------------------------------------------ helpers
// Two values rounded to the nearest integer and saturated to [-127, 127],
// as the low and high byte of a 16-bit word.
__device__ __forceinline__ uint16_t pack_s8x2(float a, float b) {
  int x = __float2int_rn(a), y = __float2int_rn(b);
  x = x > 127 ? 127 : (x < -127 ? -127 : x);
  y = y > 127 ? 127 : (y < -127 ? -127 : y);
  return static_cast<uint16_t>((static_cast<uint32_t>(x) & 0xFFu) | ((static_cast<uint32_t>(y) & 0xFFu) << 8));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t w) {
  const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162 *>(&w);
  return make_float2(__low2float(h), __high2float(h));
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
}
// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ------------------------------------------------------------------ unpack
// One CTA per position, 128 threads. Reference semantics: an unpacked plane
// square is `value` where the mask bit is set, else 0
// (src/nn/cpu/cpu_network.cpp:599-605 + the inverse of
// src/nn/input_plane_packing.h:39-61). The PE input is the first 12 planes in
// square-major order (src/nn/cpu/cpu_network.cpp:731-747).
__global__ void unpack_kernel(const uint64_t *__restrict__ masks, const float *__restrict__ values,
                              __nv_bfloat16 *__restrict__ x0, __nv_bfloat16 *__restrict__ p) {
  pdl_wait();
  pdl_launch();
  const int b = blockIdx.x;
  __shared__ uint64_t sm[kPlanes];
  __shared__ float sv[kPlanes];
  for (int i = threadIdx.x; i < kPlanes; i += blockDim.x) {
    sm[i] = masks[static_cast<long long>(b) * kPlanes + i];
    sv[i] = values[static_cast<long long>(b) * kPlanes + i];
  }
  __syncthreads();
  // X0 rows: 64 squares x 192 columns; each thread writes pairs of columns.
  for (int idx = threadIdx.x; idx < kSquares * (kEmbIn / 2); idx += blockDim.x) {
    const int sq = idx / (kEmbIn / 2);
    const int c = 2 * (idx % (kEmbIn / 2));
    if (c >= kPlanes && c < kEmbIn - 16) continue;  // PE columns: written by pe_concat
    float v0 = 0.0f, v1 = 0.0f;
    if (c < kPlanes) {
      v0 = ((sm[c] >> sq) & 1ull) ? sv[c] : 0.0f;
      v1 = ((sm[c + 1] >> sq) & 1ull) ? sv[c + 1] : 0.0f;
    }
    reinterpret_cast<uint32_t *>(x0)[((static_cast<long long>(b) * kSquares + sq) * kEmbIn + c) /
                                     2] = pack_bf16x2(v0, v1);
  }
  for (int idx = threadIdx.x; idx < kPeInputs / 2; idx += blockDim.x) {
    const int e = 2 * idx;
    const int sq = e / 12, pl = e % 12;  // pl even, pl+1 < 12
    const float v0 = ((sm[pl] >> sq) & 1ull) ? sv[pl] : 0.0f;
    const float v1 = ((sm[pl + 1] >> sq) & 1ull) ? sv[pl + 1] : 0.0f;
    reinterpret_cast<uint32_t *>(p)[(static_cast<long long>(b) * kPeInputs + e) / 2] =
        pack_bf16x2(v0, v1);
  }
}

void launch_unpack(const uint64_t *masks, const float *values, int batch, __nv_bfloat16 *x0,
                   __nv_bfloat16 *p, cudaStream_t s) {
  launch_k(unpack_kernel, dim3(batch), dim3(128), 0, s, 1, masks, values, x0, p);
}

// PEo[b, sq*pe + e] -> X0[b*64 + sq, 112 + e]; 8 columns (16 bytes) per thread.
__global__ void pe_concat_kernel(const __nv_bfloat16 *__restrict__ peo, int total_rows, int pe,
                                 __nv_bfloat16 *__restrict__ x0) {
  pdl_wait();
  pdl_launch();
  const int chunks = pe / 8;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(total_rows) * chunks) return;
  const long long row = i / chunks;
  const int c = static_cast<int>(i % chunks) * 8;
  const uint4 v = *reinterpret_cast<const uint4 *>(peo + row * pe + c);
  // X0 column 112 + c: byte offset (row*192 + 112 + c)*2 is 16-byte aligned
  *reinterpret_cast<uint4 *>(x0 + row * kEmbIn + kPlanes + c) = v;
}

void launch_pe_concat(const __nv_bfloat16 *peo, int batch, int pe, __nv_bfloat16 *x0,
                      cudaStream_t s) {
  const long long n = static_cast<long long>(batch) * kSquares * (pe / 8);
  launch_k(pe_concat_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, s, 1, peo,
           batch * kSquares, pe, x0);
}

// ------------------------------------------------------------------ layernorm
// Loads of G consecutive values (G = 4 or 8) as fp32.
template <Fmt F, int G>
__device__ __forceinline__ void load_g(const void *base, long long i, float *v) {
  if constexpr (F == Fmt::F32) {
    const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(base) + i);
#pragma unroll
    for (int k = 0; k < G / 4; ++k) {
      const float4 f = p[k];
      v[4 * k] = f.x; v[4 * k + 1] = f.y; v[4 * k + 2] = f.z; v[4 * k + 3] = f.w;
    }
  } else {
    uint32_t w[G / 2];
    if constexpr (G == 8) {
      const uint4 u = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(base) + i);
      w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w;
    } else {
      const uint2 u = *reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(base) + i);
      w[0] = u.x; w[1] = u.y;
    }
#pragma unroll
    for (int k = 0; k < G / 2; ++k) {
      const float2 f = F == Fmt::F16 ? __half22float2(*reinterpret_cast<const __half2 *>(&w[k]))
                                     : unpack_bf16x2(w[k]);
      v[2 * k] = f.x;
      v[2 * k + 1] = f.y;
    }
  }
}

// One warp per row of W = 32*VPL columns. Lane l owns the G-column groups
// starting at q*32*G + l*G (G = 8 when W is a multiple of 256, else 4), so
// each load and store instruction of the warp moves 32*G contiguous values
// with 16-byte (fp16/bf16) accesses.
template <int VPL, Fmt IN, Fmt RES>
__global__ void __launch_bounds__(256)
    layernorm_warp_kernel(const void *__restrict__ in_, int rows,
                          const float *__restrict__ gamma, const float *__restrict__ beta,
                          float eps, const float *__restrict__ multT,
                          const float *__restrict__ addT, __nv_bfloat16 *__restrict__ out,
                          void *__restrict__ out_res, uint8_t *__restrict__ out8,
                          const float *__restrict__ scale8, float *__restrict__ row_scale8) {
  pdl_wait();
  pdl_launch();
  constexpr int W = 32 * VPL;
  constexpr int G = (VPL % 8 == 0) ? 8 : 4;
  constexpr int NG = VPL / G;  // groups per lane
  const int warps = blockDim.x >> 5;
  const long long row = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[VPL];
#pragma unroll
  for (int q = 0; q < NG; ++q) load_g<IN, G>(in_, row * W + q * 32 * G + lane * G, v + q * G);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) s += v[i];
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / static_cast<float>(W);
  float sq = 0.0f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const float t = v[i] - mean;
    sq += t * t;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float inv = 1.0f / sqrtf(sq / static_cast<float>(W) + eps);
  const int sqr = static_cast<int>(row % kSquares);
  const bool e4m3 = out8 && !row_scale8;
  const float inv8 = e4m3 ? 1.0f / __ldg(scale8) : 0.0f;
#pragma unroll
  for (int q = 0; q < NG; ++q) {
    const int c = q * 32 * G + lane * G;
    float r[G], g[G], b[G];
    load_g<Fmt::F32, G>(gamma, c, g);
    load_g<Fmt::F32, G>(beta, c, b);
#pragma unroll
    for (int e = 0; e < G; ++e) r[e] = (v[q * G + e] - mean) * inv * g[e] + b[e];
    if (multT) {
      float mt[G], at[G];
      load_g<Fmt::F32, G>(multT, static_cast<long long>(sqr) * W + c, mt);
      load_g<Fmt::F32, G>(addT, static_cast<long long>(sqr) * W + c, at);
#pragma unroll
      for (int e = 0; e < G; ++e) r[e] = r[e] * mt[e] + at[e];
    }
#pragma unroll
    for (int e = 0; e < G; ++e) v[q * G + e] = r[e];  // kept for the 8-bit integer copy
    const long long o = row * W + c;
    if (out) {
      uint32_t w[G / 2];
#pragma unroll
      for (int k = 0; k < G / 2; ++k) w[k] = pack_bf16x2(r[2 * k], r[2 * k + 1]);
      if constexpr (G == 8) *reinterpret_cast<uint4 *>(out + o) = make_uint4(w[0], w[1], w[2], w[3]);
      else *reinterpret_cast<uint2 *>(out + o) = make_uint2(w[0], w[1]);
    }
    if (e4m3) {
      uint32_t w[G / 4];
#pragma unroll
      for (int k = 0; k < G / 4; ++k) {
        const __nv_fp8_e4m3 a(r[4 * k] * inv8), bb(r[4 * k + 1] * inv8), c2(r[4 * k + 2] * inv8),
            d(r[4 * k + 3] * inv8);
        w[k] = uint32_t(a.__x) | (uint32_t(bb.__x) << 8) | (uint32_t(c2.__x) << 16) |
               (uint32_t(d.__x) << 24);
      }
      if constexpr (G == 8) *reinterpret_cast<uint2 *>(out8 + o) = make_uint2(w[0], w[1]);
      else *reinterpret_cast<uint32_t *>(out8 + o) = w[0];
    }
    if (out_res) {
      if constexpr (RES == Fmt::F16) {
        uint32_t w[G / 2];
#pragma unroll
        for (int k = 0; k < G / 2; ++k) {
          const __half2 h = __floats2half2_rn(r[2 * k], r[2 * k + 1]);
          w[k] = *reinterpret_cast<const uint32_t *>(&h);
        }
        __half *dst = static_cast<__half *>(out_res) + o;
        if constexpr (G == 8) *reinterpret_cast<uint4 *>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        else *reinterpret_cast<uint2 *>(dst) = make_uint2(w[0], w[1]);
      } else {
        float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(out_res) + o);
#pragma unroll
        for (int k = 0; k < G / 4; ++k)
          dst[k] = make_float4(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3]);
      }
    }
  }
  if (out8 && row_scale8) {
    // 8-bit integer copy with a per-row scale: absmax / 127, values rounded
    // to the nearest integer (the GEMM multiplies its int32 accumulator of
    // the row by this scale)
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = fmaxf(amax, 1e-20f) * (1.0f / 127.0f);
    const float is = 1.0f / scale;
    if (lane == 0) row_scale8[row] = scale;
#pragma unroll
    for (int q = 0; q < NG; ++q) {
      const long long o = row * W + q * 32 * G + lane * G;
      uint32_t w[G / 4];
#pragma unroll
      for (int k = 0; k < G / 4; ++k) {
        uint32_t x = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          int t = __float2int_rn(v[q * G + 4 * k + e] * is);
          t = t > 127 ? 127 : (t < -127 ? -127 : t);
          x |= (static_cast<uint32_t>(t) & 0xFFu) << (8 * e);
        }
        w[k] = x;
      }
      if constexpr (G == 8) *reinterpret_cast<uint2 *>(out8 + o) = make_uint2(w[0], w[1]);
      else *reinterpret_cast<uint32_t *>(out8 + o) = w[0];
    }
  }
}

// One CTA (T threads: 256, or 1024 when there are few rows, so that a small
// batch's row is spread over more threads) per row for wide rows (smolgen's
// H*g = 8192): the row is read once into registers (VPT values per thread in
// 8-value groups, each warp instruction covering 512 contiguous bytes), then
// mean, variance and the normalised output come from the registers.
template <int VPT, int T = 256>
__global__ void __launch_bounds__(T)
    layernorm_block_kernel(const __nv_bfloat16 *__restrict__ in, int width,
                           const float *__restrict__ gamma, const float *__restrict__ beta,
                           float eps, __nv_bfloat16 *__restrict__ out) {
  pdl_wait();
  pdl_launch();
  constexpr int NG = VPT / 8;
  const long long row = blockIdx.x;
  const __nv_bfloat16 *src = in + row * width;
  __shared__ float red[T / 32];
  float v[VPT];
#pragma unroll
  for (int q = 0; q < NG; ++q) {
    const uint4 u = *reinterpret_cast<const uint4 *>(src + q * (8 * T) + threadIdx.x * 8);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16x2(w[e]);
      v[8 * q + 2 * e] = f.x;
      v[8 * q + 2 * e + 1] = f.y;
    }
  }
  auto block_sum = [&](float x) {
#pragma unroll
    for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    __syncthreads();  // red[] of the previous reduction has been read
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < T / 32; ++i) t += red[i];
    return t;
  };
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) s += v[i];
  const float mean = block_sum(s) / static_cast<float>(width);
  float sq = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const float t = v[i] - mean;
    sq += t * t;
  }
  const float inv = 1.0f / sqrtf(block_sum(sq) / static_cast<float>(width) + eps);
#pragma unroll
  for (int q = 0; q < NG; ++q) {
    const int c = q * (8 * T) + threadIdx.x * 8;
    float g[8], b[8];
    load_g<Fmt::F32, 8>(gamma, c, g);
    load_g<Fmt::F32, 8>(beta, c, b);
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      o[e] = pack_bf16x2((v[8 * q + 2 * e] - mean) * inv * g[2 * e] + b[2 * e],
                         (v[8 * q + 2 * e + 1] - mean) * inv * g[2 * e + 1] + b[2 * e + 1]);
    *reinterpret_cast<uint4 *>(out + row * width + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <int VPL, Fmt IN>
static void ln_warp_in(const void *in, int rows, const float *gamma, const float *beta, float eps,
                       const float *multT, const float *addT, __nv_bfloat16 *out, void *out_res,
                       Fmt res_fmt, uint8_t *out8, const float *scale8, float *row_scale8,
                       cudaStream_t s) {
  const int wpb = 8;
  const unsigned grid = static_cast<unsigned>((rows + wpb - 1) / wpb);
  if (res_fmt == Fmt::F16)
    launch_k(layernorm_warp_kernel<VPL, IN, Fmt::F16>, dim3(grid), dim3(32 * wpb), 0, s, 1, in, rows, gamma, beta, eps, multT, addT, out, out_res, out8, scale8, row_scale8);
  else
    launch_k(layernorm_warp_kernel<VPL, IN, Fmt::F32>, dim3(grid), dim3(32 * wpb), 0, s, 1, in, rows, gamma, beta, eps, multT, addT, out, out_res, out8, scale8, row_scale8);
}

template <int VPL>
static void ln_warp(const void *in, Fmt in_fmt, int rows, const float *gamma, const float *beta,
                    float eps, const float *multT, const float *addT, __nv_bfloat16 *out,
                    void *out_res, Fmt res_fmt, uint8_t *out8, const float *scale8,
                    float *row_scale8, cudaStream_t s) {
  switch (in_fmt) {
  case Fmt::F32:
    ln_warp_in<VPL, Fmt::F32>(in, rows, gamma, beta, eps, multT, addT, out, out_res, res_fmt, out8, scale8, row_scale8, s);
    return;
  case Fmt::F16:
    ln_warp_in<VPL, Fmt::F16>(in, rows, gamma, beta, eps, multT, addT, out, out_res, res_fmt, out8, scale8, row_scale8, s);
    return;
  default:
    ln_warp_in<VPL, Fmt::BF16>(in, rows, gamma, beta, eps, multT, addT, out, out_res, res_fmt, out8, scale8, row_scale8, s);
    return;
  }
}

// Deferred LayerNorm: (mean, 1/sqrt(var + eps)) of each row from its CH
// per-32-column partials (chunk sum, chunk sum of squared deviations from the
// chunk mean; written chunk-major [CH, rows] by the residual GEMM epilogue):
// var = (sum_i M2_i + sum_i (s_i - 32 mean)^2 / 32) / width, the
// decomposition of the two-pass variance the LayerNorm kernel computes
// (src/nn/cpu/cpu_network.cpp:424-460 normalises with the row's mean and
// variance). One thread per row, all CH loads in flight at once, each
// warp-wide load 256 contiguous bytes.
template <int CH>
__global__ void __launch_bounds__(256)
    row_stats_kernel(const float2 *__restrict__ part, int rows, float eps,
                     float2 *__restrict__ out) {
  pdl_wait();
  pdl_launch();
  const long long row = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  float2 v[CH];
#pragma unroll
  for (int i = 0; i < CH; ++i) v[i] = __ldcg(part + static_cast<long long>(i) * rows + row);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < CH; ++i) s += v[i].x;
  constexpr float width = 32.0f * CH;
  const float mean = s / width;
  float m2 = 0.0f;
#pragma unroll
  for (int i = 0; i < CH; ++i) {
    const float dv = v[i].x - 32.0f * mean;
    m2 += v[i].y + dv * dv * (1.0f / 32.0f);
  }
  out[row] = make_float2(mean, 1.0f / sqrtf(m2 / width + eps));
}

void launch_row_stats(const float2 *part, int rows, int width, float eps, float2 *out,
                      cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>((rows + 255) / 256)), block(256);
  switch (width) {
  case 128: launch_k(row_stats_kernel<4>, grid, block, 0, s, 1, part, rows, eps, out); return;
  case 256: launch_k(row_stats_kernel<8>, grid, block, 0, s, 1, part, rows, eps, out); return;
  case 512: launch_k(row_stats_kernel<16>, grid, block, 0, s, 1, part, rows, eps, out); return;
  case 1024: launch_k(row_stats_kernel<32>, grid, block, 0, s, 1, part, rows, eps, out); return;
  default: return;
  }
}

void launch_layernorm_q(const void *in, Fmt in_fmt, int rows, int width, const float *gamma,
                        const float *beta, float eps, const float *multT, const float *addT,
                        __nv_bfloat16 *out, void *out_res, Fmt res_fmt, uint8_t *out8,
                        const float *scale8, cudaStream_t s, float *row_scale8) {
#define MFB_LN(V) ln_warp<V>(in, in_fmt, rows, gamma, beta, eps, multT, addT, out, out_res, res_fmt, out8, scale8, row_scale8, s)
  switch (width) {
  case 128: MFB_LN(4); return;
  case 256: MFB_LN(8); return;
  case 512: MFB_LN(16); return;
  case 1024: MFB_LN(32); return;
  default: return;
  }
#undef MFB_LN
}

void launch_layernorm(const void *in, bool in_f32, int rows, int width, const float *gamma,
                      const float *beta, float eps, const float *multT, const float *addT,
                      __nv_bfloat16 *out, float *out_f32, cudaStream_t s) {
  if (width != 128 && width != 256 && width != 512 && width != 1024) {
    // wide bf16 rows (smolgen's H*g, a multiple of 2048 up to 16384); no
    // gates, no fp32 output on this path
    const __nv_bfloat16 *src = static_cast<const __nv_bfloat16 *>(in);
    switch (width) {
    case 2048: launch_k(layernorm_block_kernel<8>, dim3(rows), dim3(256), 0, s, 1, src, width, gamma, beta, eps, out); return;
    case 4096: launch_k(layernorm_block_kernel<16>, dim3(rows), dim3(256), 0, s, 1, src, width, gamma, beta, eps, out); return;
    case 6144: launch_k(layernorm_block_kernel<24>, dim3(rows), dim3(256), 0, s, 1, src, width, gamma, beta, eps, out); return;
    case 8192:
      if (rows <= 64)  // small batch: a row over 1024 threads
        launch_k(layernorm_block_kernel<8, 1024>, dim3(rows), dim3(1024), 0, s, 1, src, width, gamma, beta, eps, out);
      else
        launch_k(layernorm_block_kernel<32>, dim3(rows), dim3(256), 0, s, 1, src, width, gamma, beta, eps, out);
      return;
    case 12288: launch_k(layernorm_block_kernel<48>, dim3(rows), dim3(256), 0, s, 1, src, width, gamma, beta, eps, out); return;
    case 16384: launch_k(layernorm_block_kernel<64>, dim3(rows), dim3(256), 0, s, 1, src, width, gamma, beta, eps, out); return;
    default: return;
    }
  }
  launch_layernorm_q(in, in_f32 ? Fmt::F32 : Fmt::BF16, rows, width, gamma, beta, eps, multT, addT,
                     out, out_f32, Fmt::F32, nullptr, nullptr, s);
}

// ------------------------------------------------------------------ split-K reduce
// out[r] = LN(act(sum_s part[s][r] + bias)) for rows of width 32*VPL; one warp
// per row (the smolgen dense1 stage: dense, bias, activation, LN eps 1e-3,
// src/nn/cpu/cpu_network.cpp:1143-1157).
template <int VPL>
__global__ void splitk_act_ln_kernel(const float *__restrict__ part, int splits, long long stride,
                                     int rows, const float *__restrict__ bias, int act,
                                     const float *__restrict__ gamma, const float *__restrict__ beta,
                                     float eps, __nv_bfloat16 *__restrict__ out) {
  pdl_wait();
  pdl_launch();
  constexpr int W = 32 * VPL;
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[VPL];
#pragma unroll
  for (int q = 0; q < VPL / 4; ++q) {
    const int c = q * 128 + lane * 4;
    float4 a = *reinterpret_cast<const float4 *>(bias + c);
    // slices in order; four loads in flight at a time
    int sidx = 0;
    for (; sidx + 4 <= splits; sidx += 4) {
      float4 f[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        f[k] = __ldcg(reinterpret_cast<const float4 *>(part + (sidx + k) * stride + row * W + c));
#pragma unroll
      for (int k = 0; k < 4; ++k) { a.x += f[k].x; a.y += f[k].y; a.z += f[k].z; a.w += f[k].w; }
    }
    for (; sidx < splits; ++sidx) {
      const float4 f = __ldcg(reinterpret_cast<const float4 *>(part + sidx * stride + row * W + c));
      a.x += f.x; a.y += f.y; a.z += f.z; a.w += f.w;
    }
    v[4 * q] = apply_act(a.x, act);
    v[4 * q + 1] = apply_act(a.y, act);
    v[4 * q + 2] = apply_act(a.z, act);
    v[4 * q + 3] = apply_act(a.w, act);
  }
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) s += v[i];
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / static_cast<float>(W);
  float sq = 0.0f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) sq += (v[i] - mean) * (v[i] - mean);
#pragma unroll
  for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float inv = 1.0f / sqrtf(sq / static_cast<float>(W) + eps);
#pragma unroll
  for (int q = 0; q < VPL / 4; ++q) {
    const int c = q * 128 + lane * 4;
    float r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) r[e] = (v[4 * q + e] - mean) * inv * gamma[c + e] + beta[c + e];
    *reinterpret_cast<uint2 *>(out + row * W + c) = make_uint2(pack_bf16x2(r[0], r[1]), pack_bf16x2(r[2], r[3]));
  }
}

// The same for a few rows (small batches): one CTA per row and one thread
// per column, so every slice of a column is loaded at once instead of one
// warp walking the slices of a whole row (the latency of one small batch's
// smolgen dense1 step).
__global__ void __launch_bounds__(1024)
    splitk_act_ln_row_kernel(const float *__restrict__ part, int splits, long long stride,
                             const float *__restrict__ bias, int act,
                             const float *__restrict__ gamma, const float *__restrict__ beta,
                             float eps, __nv_bfloat16 *__restrict__ out) {
  pdl_wait();
  pdl_launch();
  __shared__ float red[32];
  const int row = blockIdx.x, c = threadIdx.x, lane = c & 31, warp = c >> 5;
  const int width = blockDim.x, warps = width >> 5;
  const float *p = part + static_cast<long long>(row) * width + c;
  float x[16];
  const int n = splits < 16 ? splits : 16;
#pragma unroll
  for (int k = 0; k < 16; ++k) x[k] = k < n ? __ldcg(p + k * stride) : 0.0f;
  float v = __ldg(bias + c);
#pragma unroll
  for (int k = 0; k < 16; ++k) v += x[k];  // slices in order
  for (int k = 16; k < splits; ++k) v += __ldcg(p + k * stride);
  v = apply_act(v, act);
  auto bsum = [&](float t) {
#pragma unroll
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    __syncthreads();
    if (lane == 0) red[warp] = t;
    __syncthreads();
    float r = 0.0f;
    for (int w = 0; w < warps; ++w) r += red[w];
    return r;
  };
  const float mean = bsum(v) / static_cast<float>(width);
  const float inv = 1.0f / sqrtf(bsum((v - mean) * (v - mean)) / static_cast<float>(width) + eps);
  out[static_cast<long long>(row) * width + c] =
      __float2bfloat16_rn((v - mean) * inv * __ldg(gamma + c) + __ldg(beta + c));
}

bool launch_splitk_act_ln(const float *part, int splits, long long stride, int rows, int width,
                          const float *bias, int act, const float *gamma, const float *beta,
                          float eps, __nv_bfloat16 *out, cudaStream_t s) {
  if (rows <= 64 && width % 32 == 0 && width <= 1024) {
    launch_k(splitk_act_ln_row_kernel, dim3(static_cast<unsigned>(rows)),
             dim3(static_cast<unsigned>(width)), 0, s, 1, part, splits, stride, bias, act, gamma,
             beta, eps, out);
    return true;
  }
  const int wpb = 8;
  const unsigned grid = static_cast<unsigned>((rows + wpb - 1) / wpb);
  switch (width) {
  case 128: launch_k(splitk_act_ln_kernel<4>, dim3(grid), dim3(32 * wpb), 0, s, 1, part, splits, stride, rows, bias, act, gamma, beta, eps, out); return true;
  case 256: launch_k(splitk_act_ln_kernel<8>, dim3(grid), dim3(32 * wpb), 0, s, 1, part, splits, stride, rows, bias, act, gamma, beta, eps, out); return true;
  case 512: launch_k(splitk_act_ln_kernel<16>, dim3(grid), dim3(32 * wpb), 0, s, 1, part, splits, stride, rows, bias, act, gamma, beta, eps, out); return true;
  case 1024: launch_k(splitk_act_ln_kernel<32>, dim3(grid), dim3(32 * wpb), 0, s, 1, part, splits, stride, rows, bias, act, gamma, beta, eps, out); return true;
  default: return false;
  }
}

// ------------------------------------------------------------------ attention
// One CTA (4 warps) per (position, head); head depth 32. Warp w owns query
// rows 16w..16w+15. S = Q K^T via mma.sync (2 k-steps x 8 key tiles), plus
// the smolgen bias, row softmax in registers, then O = P V (4 k-steps x 4
// tiles) and O / rowsum (src/nn/cpu/cpu_network.cpp:1175-1254 and the
// softmax of :405-422: exp(x - max) / sum).
//
// The softmax runs in base 2: the smolgen generator GEMM writes the bias
// already multiplied by log2(e), the scores are scaled by log2(e)/sqrt(dh),
// and exp(x - max) = 2^(x' - max') with one ex2.approx per element. The bias
// arrives in "fragment order" (the generator's output columns are permuted
// when the weights are packed, attention_bias_column()): thread (warp w,
// lane l) finds the 32 values its score fragments need as four 16-byte
// pieces at w*1024 + i*256 + l*8 (i = 0..3), so each warp-wide load reads
// 512 contiguous bytes, issued while Q, K and V are still in flight. P stays
// unnormalised through P V; the 16 outputs of each thread are divided by the
// row sum at the end, staged in the warp's own 16 rows of sQ (no other warp
// reads them) and written back as whole 16-byte pieces of each context row.
constexpr int kDh = 32;
constexpr int kQkvStride = 40;   // padded smem row (80 bytes): conflict-free ldmatrix

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// OUT: the context format, 0 bf16, 1 e4m3, 2 signed 8-bit integers (one
// kernel instance each).
template <int OUT>
__global__ void __launch_bounds__(128)
    attention_kernel(const __nv_bfloat16 *__restrict__ qkv, long long ldq,
                     const __nv_bfloat16 *__restrict__ bias, int heads, int d,
                     __nv_bfloat16 *__restrict__ ctx, uint8_t *__restrict__ ctx8,
                     const float *__restrict__ scale8) {
  pdl_wait();
  pdl_launch();
  __shared__ __align__(16) __nv_bfloat16 sQ[kSquares * kQkvStride];
  __shared__ __align__(16) __nv_bfloat16 sK[kSquares * kQkvStride];
  __shared__ __align__(16) __nv_bfloat16 sV[kSquares * kQkvStride];
  const int bh = blockIdx.x;
  const int b = bh / heads, h = bh % heads;
  const int tid = threadIdx.x;
  const __nv_bfloat16 *base = qkv + static_cast<long long>(b) * kSquares * ldq + h * kDh;
  // Q, K, V: 64 rows x 64 bytes = 4 chunks of 16 B each
  for (int i = tid; i < kSquares * 4; i += 128) {
    const int r = i >> 2, c = (i & 3) * 8;
    const __nv_bfloat16 *g = base + r * ldq + c;
    cp_async16(&sQ[r * kQkvStride + c], g);
    cp_async16(&sK[r * kQkvStride + c], g + d);
    cp_async16(&sV[r * kQkvStride + c], g + 2 * d);
  }
  cp_async_commit();
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int q0 = warp * 16;
  // this thread's 32 bias values (fragment order), word 2j: row g, keys
  // 8j+2t and 8j+2t+1; word 2j+1: row g+8, the same keys
  uint32_t bw[16];
  {
    const uint4 *bp = reinterpret_cast<const uint4 *>(
        bias + static_cast<long long>(bh) * kSquares * kSquares + warp * 1024 + lane * 8);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 v = __ldg(bp + 32 * i);
      bw[4 * i] = v.x;
      bw[4 * i + 1] = v.y;
      bw[4 * i + 2] = v.z;
      bw[4 * i + 3] = v.w;
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- S = Q K^T
  float S[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) S[j][e] = 0.0f;
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    uint32_t a[4];
    {
      const int mat = lane >> 3;
      const int r = q0 + (lane & 7) + 8 * (mat & 1);
      const int c = ks * 16 + 8 * (mat >> 1);
      ldmatrix_x4(a, &sQ[r * kQkvStride + c]);
    }
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      uint32_t bf[4];
      const int mat = lane >> 3;
      const int key = 8 * (j + (mat >> 1)) + (lane & 7);
      const int c = ks * 16 + 8 * (mat & 1);
      ldmatrix_x4(bf, &sK[key * kQkvStride + c]);
      mma_bf16_16816(S[j], a, bf[0], bf[1]);
      mma_bf16_16816(S[j + 1], a, bf[2], bf[3]);
    }
  }
  // ---- x = S log2(e) / sqrt(dh) + bias log2(e); rows g and g+8 of this warp
  const float c2 = 1.4426950408889634f / sqrtf(static_cast<float>(kDh));
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float2 b0 = unpack_bf16x2(bw[2 * j]);
    const float2 b1 = unpack_bf16x2(bw[2 * j + 1]);
    S[j][0] = fmaf(S[j][0], c2, b0.x);
    S[j][1] = fmaf(S[j][1], c2, b0.y);
    S[j][2] = fmaf(S[j][2], c2, b1.x);
    S[j][3] = fmaf(S[j][3], c2, b1.y);
    mx0 = fmaxf(mx0, fmaxf(S[j][0], S[j][1]));
    mx1 = fmaxf(mx1, fmaxf(S[j][2], S[j][3]));
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
  }
  float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    S[j][0] = ex2_approx(S[j][0] - mx0);
    S[j][1] = ex2_approx(S[j][1] - mx0);
    S[j][2] = ex2_approx(S[j][2] - mx1);
    S[j][3] = ex2_approx(S[j][3] - mx1);
    sum0 += S[j][0] + S[j][1];
    sum1 += S[j][2] + S[j][3];
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    sum0 += __shfl_xor_sync(0xffffffffu, sum0, o);
    sum1 += __shfl_xor_sync(0xffffffffu, sum1, o);
  }
  const float inv0 = 1.0f / sum0, inv1 = 1.0f / sum1;
  // ---- O = P V (P unnormalised, each entry in (0, 1])
  float O[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) O[j][e] = 0.0f;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    uint32_t a[4];
    a[0] = pack_bf16x2(S[2 * ks][0], S[2 * ks][1]);
    a[1] = pack_bf16x2(S[2 * ks][2], S[2 * ks][3]);
    a[2] = pack_bf16x2(S[2 * ks + 1][0], S[2 * ks + 1][1]);
    a[3] = pack_bf16x2(S[2 * ks + 1][2], S[2 * ks + 1][3]);
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      uint32_t bf[4];
      const int mat = lane >> 3;
      const int key = ks * 16 + 8 * (mat & 1) + (lane & 7);
      const int c = 8 * (j + (mat >> 1));
      ldmatrix_x4_trans(bf, &sV[key * kQkvStride + c]);
      mma_bf16_16816(O[j], a, bf[0], bf[1]);
      mma_bf16_16816(O[j + 1], a, bf[2], bf[3]);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    O[j][0] *= inv0;
    O[j][1] *= inv0;
    O[j][2] *= inv1;
    O[j][3] *= inv1;
  }
  const long long base_off = (static_cast<long long>(b) * kSquares + q0) * d + h * kDh;
  // stage this warp's 16 x 32 outputs in its own rows of sQ (80-byte rows)
  uint8_t *stage = reinterpret_cast<uint8_t *>(&sQ[q0 * kQkvStride]);
  constexpr int kRowBytes = kQkvStride * 2;
  if constexpr (OUT != 0) {
    // 8-bit context for an 8-bit output projection: value / *scale8 as e4m3
    // or (OUT 2) as a saturated signed integer; 32-byte rows
    const float inv = 1.0f / __ldg(scale8);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = 8 * j + 2 * t;
      uint16_t lo, hi;
      if constexpr (OUT == 2) {
        lo = pack_s8x2(O[j][0] * inv, O[j][1] * inv);
        hi = pack_s8x2(O[j][2] * inv, O[j][3] * inv);
      } else {
        lo = __nv_fp8x2_e4m3(make_float2(O[j][0] * inv, O[j][1] * inv)).__x;
        hi = __nv_fp8x2_e4m3(make_float2(O[j][2] * inv, O[j][3] * inv)).__x;
      }
      *reinterpret_cast<uint16_t *>(stage + g * kRowBytes + col) = lo;
      *reinterpret_cast<uint16_t *>(stage + (g + 8) * kRowBytes + col) = hi;
    }
    __syncwarp();
    const int r = lane >> 1, half = lane & 1;
    *reinterpret_cast<uint4 *>(ctx8 + base_off + static_cast<long long>(r) * d + 16 * half) =
        *reinterpret_cast<const uint4 *>(stage + r * kRowBytes + 16 * half);
    return;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int col = 8 * j + 2 * t;
    *reinterpret_cast<uint32_t *>(stage + g * kRowBytes + 2 * col) = pack_bf16x2(O[j][0], O[j][1]);
    *reinterpret_cast<uint32_t *>(stage + (g + 8) * kRowBytes + 2 * col) =
        pack_bf16x2(O[j][2], O[j][3]);
  }
  __syncwarp();
  __nv_bfloat16 *out = ctx + base_off;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int piece = lane + 32 * p, r = piece >> 2, c = (piece & 3) * 8;
    *reinterpret_cast<uint4 *>(out + static_cast<long long>(r) * d + c) =
        *reinterpret_cast<const uint4 *>(stage + r * kRowBytes + 2 * c);
  }
}

void launch_attention(const __nv_bfloat16 *qkv, long long ldq, const __nv_bfloat16 *bias,
                      int batch, int heads, int d, __nv_bfloat16 *ctx, cudaStream_t s,
                      uint8_t *ctx8, const float *scale8, int ctx_i8) {
  const dim3 grid(batch * heads);
  if (!ctx8)
    launch_k(attention_kernel<0>, grid, dim3(128), 0, s, 1, qkv, ldq, bias, heads, d, ctx, ctx8, scale8);
  else if (ctx_i8)
    launch_k(attention_kernel<2>, grid, dim3(128), 0, s, 1, qkv, ldq, bias, heads, d, ctx, ctx8, scale8);
  else
    launch_k(attention_kernel<1>, grid, dim3(128), 0, s, 1, qkv, ldq, bias, heads, d, ctx, ctx8, scale8);
}

// ------------------------------------------------------------------ legal-move priors
// The MCTS leaf step after the forward: gather each legal move's raw policy
// logit (src/mcts/evaluator.cpp:182-226; an index outside [0, 1858) gives
// logit 0) and normalise as ApplyNNPolicyToNode does
// (src/mcts/search.cpp:127-197): the first n = min(moves, 256) moves, their
// max, e = FastExp((l - max) * inv_temp), the sum in move order, uniform 1/n
// if the sum is not positive, else e * (1/sum); moves past the 256th get 0.
// FastExp (src/mcts/core.h:38-44) is Schraudolph's exponential: clamp to
// [-88, 88], then the float whose bits are trunc(x * 12102203) + (127 << 23).
// One warp per position; the sum runs on one lane so that it adds in the
// reference's order and the priors are bit-identical to it.
__device__ __forceinline__ float fast_exp_mcts(float x) {
  x = x < 88.0f ? x : 88.0f;
  x = -88.0f < x ? x : -88.0f;
  return __int_as_float(__float2int_rz(__fmul_rn(x, 12102203.0f)) + 1065353216);
}

constexpr int kMaxEdges = 256;

// Policy index of a move given as from | to << 6 | promotion << 12 for a
// position with the given side to move and canonicalisation transform, as the
// evaluator computes it: vertical mirror for black (src/mcts/evaluator.cpp:
// 24-36, 195-200), then NN::MoveToNNIndex (src/nn/policy_map.cpp:303-360):
// both squares transformed (rank reversed for mirror / transpose, file for
// flip / transpose), looked up in table[promotion][from][to].
__device__ __forceinline__ int move_index(uint32_t raw, bool black, int transform,
                                          const int16_t *__restrict__ table) {
  int from = raw & 63, to = (raw >> 6) & 63;
  const int kind = static_cast<int>(raw >> 12);
  if (kind > 4) return -1;
  if (black) {
    from ^= 56;
    to ^= 56;
  }
  if (transform) {
    if (transform & 6) {
      from ^= 56;
      to ^= 56;
    }
    if (transform & 5) {
      from ^= 7;
      to ^= 7;
    }
  }
  return table[kind * 4096 + from * 64 + to];
}

// index: policy index per move, or (raw != nullptr) the moves themselves,
// mapped through move_index with the side to move of each history's last
// board and the encoder's transform.
__global__ void __launch_bounds__(256)
    priors_kernel(const float *__restrict__ policy, int batch, const int32_t *__restrict__ offsets,
                  const int16_t *__restrict__ index, float inv_temp, float *__restrict__ priors,
                  const uint16_t *__restrict__ raw, const int16_t *__restrict__ table,
                  const mfb200_board *__restrict__ boards, const int32_t *__restrict__ hist_off,
                  const int32_t *__restrict__ transforms) {
  pdl_wait();
  pdl_launch();
  __shared__ float se[8][kMaxEdges];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * 8 + warp;
  if (b >= batch) return;
  const int lo = offsets[b] - offsets[0];
  const int moves = offsets[b + 1] - offsets[b];
  const int n = moves < kMaxEdges ? moves : kMaxEdges;
  float *e = se[warp];
  const float *pol = policy + static_cast<long long>(b) * kPolicy;
  float mx = -INFINITY;
  bool black = false;
  int transform = 0;
  if (raw) {
    const int last = hist_off[b + 1] - hist_off[0] - 1;
    black = hist_off[b + 1] > hist_off[b] && boards[last].black_to_move != 0;
    transform = transforms[b];
  }
  for (int i = lane; i < n; i += 32) {
    const int idx = raw ? move_index(raw[lo + i], black, transform, table) : index[lo + i];
    const float l = (idx >= 0 && idx < kPolicy) ? pol[idx] : 0.0f;
    e[i] = l;
    mx = l > mx ? l : mx;
  }
  for (int i = n + lane; i < moves; i += 32) priors[lo + i] = 0.0f;
  if (n == 0) return;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float t = __shfl_xor_sync(0xffffffffu, mx, o);
    mx = t > mx ? t : mx;
  }
  __syncwarp();
  for (int i = lane; i < n; i += 32) e[i] = fast_exp_mcts(__fmul_rn(__fsub_rn(e[i], mx), inv_temp));
  __syncwarp();
  float sum = 0.0f;
  if (lane == 0)
    for (int i = 0; i < n; ++i) sum = __fadd_rn(sum, e[i]);
  sum = __shfl_sync(0xffffffffu, sum, 0);
  if (sum <= 0.0f) {
    const float u = 1.0f / static_cast<float>(n);
    for (int i = lane; i < n; i += 32) priors[lo + i] = u;
    return;
  }
  const float inv_sum = 1.0f / sum;
  for (int i = lane; i < n; i += 32) priors[lo + i] = __fmul_rn(e[i], inv_sum);
}

void launch_priors(const float *policy, int batch, const int32_t *offsets, const int16_t *index,
                   float softmax_temp, float *priors, cudaStream_t s) {
  if (batch <= 0) return;
  launch_k(priors_kernel, dim3((batch + 7) / 8), dim3(256), 0, s, 1, policy, batch, offsets, index,
           1.0f / softmax_temp, priors, static_cast<const uint16_t *>(nullptr),
           static_cast<const int16_t *>(nullptr), static_cast<const mfb200_board *>(nullptr),
           static_cast<const int32_t *>(nullptr), static_cast<const int32_t *>(nullptr));
}

void launch_leaf_priors(const float *policy, int batch, const int32_t *offsets,
                        const uint16_t *moves, const int16_t *table, const mfb200_board *boards,
                        const int32_t *hist_off, const int32_t *transforms, float softmax_temp,
                        float *priors, cudaStream_t s) {
  if (batch <= 0) return;
  launch_k(priors_kernel, dim3((batch + 7) / 8), dim3(256), 0, s, 1, policy, batch, offsets,
           static_cast<const int16_t *>(nullptr), 1.0f / softmax_temp, priors, moves, table, boards,
           hist_off, transforms);
}

// ------------------------------------------------------------------ absmax
// slot = max(slot, max |x|) over n values (non-negative floats order like
// their bit patterns, so an integer atomicMax suffices). FP8 calibration.
template <typename T>
__global__ void absmax_kernel(const T *__restrict__ x, long long n, float *__restrict__ slot) {
  pdl_wait();
  pdl_launch();
  float m = 0.0f;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float v;
    if constexpr (std::is_same_v<T, __nv_bfloat16>) v = __bfloat162float(x[i]);
    else if constexpr (std::is_same_v<T, __half>) v = __half2float(x[i]);
    else v = x[i];
    m = fmaxf(m, fabsf(v));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<int *>(slot), __float_as_int(m));
}

void launch_absmax(const void *x, Fmt fmt, long long n, float *slot, cudaStream_t s) {
  if (fmt == Fmt::F32)
    launch_k(absmax_kernel<float>, dim3(296), dim3(256), 0, s, 1, static_cast<const float *>(x), n, slot);
  else if (fmt == Fmt::F16)
    launch_k(absmax_kernel<__half>, dim3(296), dim3(256), 0, s, 1, static_cast<const __half *>(x), n, slot);
  else
    launch_k(absmax_kernel<__nv_bfloat16>, dim3(296), dim3(256), 0, s, 1, static_cast<const __nv_bfloat16 *>(x), n, slot);
}

// scales[i] = max(absmax[i], tiny) / qmax (448, e4m3's largest finite value,
// or 127 for signed 8-bit integers)
__global__ void absmax_to_scale_kernel(const float *absmax, int n, float *scales, float qmax) {
  pdl_wait();
  pdl_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) scales[i] = fmaxf(absmax[i], 1e-6f) / qmax;
}

void launch_absmax_to_scale(const float *absmax, int n, float *scales, cudaStream_t s, float qmax) {
  launch_k(absmax_to_scale_kernel, dim3((n + 127) / 128), dim3(128), 0, s, 1, absmax, n, scales, qmax);
}

// ------------------------------------------------------------------ policy
// One CTA (4 warps) per position. raw[i][j] = (q_i . k_j) / sqrt(dp) by
// mma.sync over dp in 64-wide chunks (double-buffered cp.async), then the
// promotion logits and the 1858 gather (src/nn/cpu/cpu_network.cpp:892-1025):
//   promo p: raw[48 + (p%64)/8][56 + p%8] + k[56 + (p%24)/3] . ppo3[p%3]
constexpr int kPolChunk = 64;
constexpr int kPolStride = 72;  // padded smem row (144 bytes)

__global__ void __launch_bounds__(128)
    policy_map_kernel(const __nv_bfloat16 *__restrict__ qk, int dp, const float *__restrict__ ppo3,
                      const int16_t *__restrict__ gather, float *__restrict__ policy) {
  pdl_wait();
  pdl_launch();
  // q/k double buffers; after the k-loop the same bytes hold the raw logits
  __shared__ __align__(16) __nv_bfloat16 sQK[4][kSquares * kPolStride];
  __nv_bfloat16(*sQ)[kSquares * kPolStride] = sQK;
  __nv_bfloat16(*sK)[kSquares * kPolStride] = sQK + 2;
  float *raw = reinterpret_cast<float *>(sQK);
  static_assert(sizeof(float) * kSquares * (kSquares + 1) <= sizeof(__nv_bfloat16) * 4 * kSquares * kPolStride,
                "raw logits must fit in the q/k buffers");
  __shared__ float pk[8 * 3];
  const int b = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long ld = 2LL * dp;
  const __nv_bfloat16 *qbase = qk + static_cast<long long>(b) * kSquares * ld;
  const __nv_bfloat16 *kbase = qbase + dp;
  const int nchunks = dp / kPolChunk;
  auto load = [&](int chunk, int buf) {
    for (int i = tid; i < kSquares * 8; i += 128) {
      const int r = i >> 3, c = (i & 7) * 8;
      cp_async16(&sQ[buf][r * kPolStride + c], qbase + r * ld + chunk * kPolChunk + c);
      cp_async16(&sK[buf][r * kPolStride + c], kbase + r * ld + chunk * kPolChunk + c);
    }
    cp_async_commit();
  };
  const int g = lane >> 2, t = lane & 3;
  const int q0 = warp * 16;
  float S[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) S[j][e] = 0.0f;
  load(0, 0);
  for (int ch = 0; ch < nchunks; ++ch) {
    if (ch + 1 < nchunks) {
      load(ch + 1, (ch + 1) & 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16 *Q = sQ[ch & 1];
    const __nv_bfloat16 *K = sK[ch & 1];
#pragma unroll
    for (int ks = 0; ks < kPolChunk / 16; ++ks) {
      uint32_t a[4];
      {
        const int mat = lane >> 3;
        const int r = q0 + (lane & 7) + 8 * (mat & 1);
        const int c = ks * 16 + 8 * (mat >> 1);
        ldmatrix_x4(a, &Q[r * kPolStride + c]);
      }
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        uint32_t bf[4];
        const int mat = lane >> 3;
        const int key = 8 * (j + (mat >> 1)) + (lane & 7);
        const int c = ks * 16 + 8 * (mat & 1);
        ldmatrix_x4(bf, &K[key * kPolStride + c]);
        mma_bf16_16816(S[j], a, bf[0], bf[1]);
        mma_bf16_16816(S[j + 1], a, bf[2], bf[3]);
      }
    }
    __syncthreads();
  }
  const float scale = 1.0f / sqrtf(static_cast<float>(dp));
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int col = 8 * j + 2 * t;
    raw[(q0 + g) * (kSquares + 1) + col] = S[j][0] * scale;
    raw[(q0 + g) * (kSquares + 1) + col + 1] = S[j][1] * scale;
    raw[(q0 + g + 8) * (kSquares + 1) + col] = S[j][2] * scale;
    raw[(q0 + g + 8) * (kSquares + 1) + col + 1] = S[j][3] * scale;
  }
  // promotion key terms: k[56+i] . ppo3[r], 24 dot products; warp w does i = 2w, 2w+1
  for (int pr = warp * 6; pr < warp * 6 + 6; ++pr) {
    const int i = pr / 3, r = pr % 3;
    const __nv_bfloat16 *krow = kbase + (56 + i) * ld;
    float acc = 0.0f;
    for (int c = lane * 2; c < dp; c += 64) {
      const float2 kv = unpack_bf16x2(*reinterpret_cast<const uint32_t *>(krow + c));
      acc += kv.x * ppo3[r * dp + c] + kv.y * ppo3[r * dp + c + 1];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) pk[i * 3 + r] = acc;
  }
  __syncthreads();
  float *out = policy + static_cast<long long>(b) * kPolicy;
  for (int p = tid; p < kPolicy; p += 128) {
    const int idx = gather[p];
    float v;
    if (idx < kSquares * kSquares) {
      v = raw[(idx >> 6) * (kSquares + 1) + (idx & 63)];
    } else {
      const int promo = idx - kSquares * kSquares;
      const int pair = promo % 64;
      v = raw[(48 + pair / 8) * (kSquares + 1) + 56 + pair % 8] + pk[((promo % 24) / 3) * 3 + promo % 3];
    }
    out[p] = v;
  }
}

void launch_policy_map(const __nv_bfloat16 *qk, int batch, int dp, const float *ppo3,
                       const int16_t *gather, float *policy, cudaStream_t s) {
  launch_k(policy_map_kernel, dim3(batch), dim3(128), 0, s, 1, qk, dp, ppo3, gather, policy);
}

// ------------------------------------------------------------------ heads
// One warp per position: WDL = softmax(W2v h_v + b2v), moves_left =
// relu(W2m h_m + b2m) (src/nn/network_execution_plan.cpp:1061-1111).
__global__ void heads_kernel(const __nv_bfloat16 *__restrict__ h, int batch, int vh, int mh,
                             const float *__restrict__ w2v, const float *__restrict__ b2v,
                             const float *__restrict__ w2m, const float *__restrict__ b2m,
                             float *__restrict__ wdl, float *__restrict__ mlh) {
  pdl_wait();
  pdl_launch();
  const int warps = blockDim.x >> 5;
  const int b = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= batch) return;
  const __nv_bfloat16 *x = h + static_cast<long long>(b) * (vh + mh);
  float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, am = 0.0f;
  for (int i = lane; i < vh; i += 32) {
    const float v = __bfloat162float(x[i]);
    a0 += w2v[i] * v;
    a1 += w2v[vh + i] * v;
    a2 += w2v[2 * vh + i] * v;
  }
  for (int i = lane; i < mh; i += 32) am += w2m[i] * __bfloat162float(x[vh + i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    a0 += __shfl_xor_sync(0xffffffffu, a0, o);
    a1 += __shfl_xor_sync(0xffffffffu, a1, o);
    a2 += __shfl_xor_sync(0xffffffffu, a2, o);
    am += __shfl_xor_sync(0xffffffffu, am, o);
  }
  if (lane == 0) {
    a0 += b2v[0];
    a1 += b2v[1];
    a2 += b2v[2];
    const float m = fmaxf(a0, fmaxf(a1, a2));
    const float e0 = expf(a0 - m), e1 = expf(a1 - m), e2 = expf(a2 - m);
    const float inv = 1.0f / (e0 + e1 + e2);
    wdl[3 * b + 0] = e0 * inv;
    wdl[3 * b + 1] = e1 * inv;
    wdl[3 * b + 2] = e2 * inv;
    mlh[b] = fmaxf(am + b2m[0], 0.0f);
  }
}

void launch_heads(const __nv_bfloat16 *h, int batch, int vh, int mh, const float *w2v,
                  const float *b2v, const float *w2m, const float *b2m, float *wdl, float *mlh,
                  cudaStream_t s) {
  const int wpb = 8;
  launch_k(heads_kernel, dim3((batch + wpb - 1) / wpb), dim3(32 * wpb), 0, s, 1, h, batch, vh, mh, w2v, b2v, w2m, b2m,
                                                           wdl, mlh);
}

}  // namespace mfb200
