// kernels.cuh -- the memory-bound / small-matmul kernels of the BT4 forward.
// (The large projections run through the tcgen05 GEMM in gemm_sm100.cuh.)
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace mfb200 {

constexpr int kPlanes = 112;
constexpr int kSquares = 64;
constexpr int kPolicy = 1858;
constexpr int kPeInputs = 12 * kSquares;  // 12 position planes, square-major
constexpr int kEmbIn = 192;               // 112 planes + 64 PE, padded to 3 x 64

// Element formats of activation buffers.
enum class Fmt : int { BF16 = 0, F32 = 1, F16 = 2 };

// Input unpack: packed (mask, value) planes -> X0[M, 192] (planes in columns
// 0..111, columns 176..191 zeroed; columns 112..175 are filled by pe_concat)
// and the square-major PE input P[B, 768].
void launch_unpack(const uint64_t *masks, const float *values, int batch, __nv_bfloat16 *x0,
                   __nv_bfloat16 *p, cudaStream_t s);

// X0[:, 112:112+pe] = PEo[B, 64*pe] viewed as [B*64, pe].
void launch_pe_concat(const __nv_bfloat16 *peo, int batch, int pe, __nv_bfloat16 *x0,
                      cudaStream_t s);

// Row LayerNorm (two-pass mean/variance in fp32) of bf16 or fp32 rows
// (`in_f32`); optional square gates multT/addT [64][width] applied after the
// norm. Writes bf16 `out` and, when `out_f32` is non-null, an fp32 copy.
// Widths 128/256/512/1024 use one warp per row; other widths (bf16 input
// only, no gates, no fp32 copy) one CTA per row.
void launch_layernorm(const void *in, bool in_f32, int rows, int width, const float *gamma,
                      const float *beta, float eps, const float *multT, const float *addT,
                      __nv_bfloat16 *out, float *out_f32, cudaStream_t s);

// out = LN(act(sum of `splits` fp32 partials + bias)) per row (split-K
// epilogue of a skinny GEMM); width 128/256/512/1024. Returns false for other
// widths.
bool launch_splitk_act_ln(const float *part, int splits, long long stride, int rows, int width,
                          const float *bias, int act, const float *gamma, const float *beta,
                          float eps, __nv_bfloat16 *out, cudaStream_t s);

// Same, with the input in any Fmt, the full-precision copy `out_res` in
// `res_fmt` (F32 or F16: the residual stream) and an optional e4m3 copy
// out8 = value / *scale8 (FP8 GEMM input); `out` may be null when only the
// other copies are needed. Widths 128/256/512/1024 only.
// Deferred LayerNorm: per-row (mean, 1/sqrt(var + eps)) [rows] from the
// per-32-column partials [width / 32, rows] of a residual GEMM (width <= 1024).
void launch_row_stats(const float2 *part, int rows, int width, float eps, float2 *out,
                      cudaStream_t s);

void launch_layernorm_q(const void *in, Fmt in_fmt, int rows, int width, const float *gamma,
                        const float *beta, float eps, const float *multT, const float *addT,
                        __nv_bfloat16 *out, void *out_res, Fmt res_fmt, uint8_t *out8,
                        const float *scale8, cudaStream_t s, float *row_scale8 = nullptr);

// Fragment order of the smolgen attention bias: the generator GEMM's output
// column c (its weight row) holds the reference's bias entry q * 64 + k
// returned here (query q, key k), so that each attention thread finds its 32
// values as four 16-byte pieces and each warp-wide 16-byte load reads 512
// contiguous bytes: c = w * 1024 + i * 256 + lane * 8 + jj * 4 + e, with
// j = 2i + jj, query 16w + lane/4 + 8*(e/2) and key 8j + 2*(lane%4) + e%2
// (the accumulator fragment layout of mma.m16n8k16).
inline int attention_bias_column(int c) {
  const int w = c >> 10, i = (c >> 8) & 3, lane = (c >> 3) & 31, jj = (c >> 2) & 1, e = c & 3;
  const int j = 2 * i + jj;
  const int q = 16 * w + (lane >> 2) + 8 * (e >> 1);
  const int k = 8 * j + 2 * (lane & 3) + (e & 1);
  return q * 64 + k;
}

// 64-token attention per (position, head) with the smolgen bias added before
// the softmax: ctx[b*64+q, h*dh:..] = softmax(Q K^T / sqrt(dh) + bias) V.
// qkv: [B*64, ldq] with Q at column 0, K at d, V at 2d. bias: [B*H, 4096],
// each row in fragment order (attention_bias_column) and multiplied by log2(e).
// With ctx8 set, the context is written as e4m3 (value / *scale8) instead,
// or with ctx_i8 as signed 8-bit integers round(value / *scale8), saturated.
void launch_attention(const __nv_bfloat16 *qkv, long long ldq, const __nv_bfloat16 *bias,
                      int batch, int heads, int d, __nv_bfloat16 *ctx, cudaStream_t s,
                      uint8_t *ctx8 = nullptr, const float *scale8 = nullptr, int ctx_i8 = 0);

}  // namespace mfb200
extern "C" {
typedef struct mfb200_board mfb200_board;
}
namespace mfb200 {
// Position histories (CSR over offsets [batch + 1]) -> packed planes
// masks / values [batch, 112] and transforms [batch] (encoder.cu).
void launch_encode(const mfb200_board *boards, const int32_t *offsets, int batch, int fmt,
                   uint64_t *masks, float *values, int32_t *transforms, cudaStream_t s);

// Legal-move priors of `batch` positions from their policy logits
// [batch, 1858]: offsets [batch + 1] (CSR into index, offsets[0] need not be
// 0), index = policy index of each legal move; priors has offsets[batch] -
// offsets[0] entries (see priors_kernel).
void launch_priors(const float *policy, int batch, const int32_t *offsets, const int16_t *index,
                   float softmax_temp, float *priors, cudaStream_t s);
// Same from the moves themselves (from | to << 6 | promotion << 12), mapped to
// policy indices on the device with `table` [5][64][64], each history's side
// to move (its last board) and the encoder's transforms.
void launch_leaf_priors(const float *policy, int batch, const int32_t *offsets,
                        const uint16_t *moves, const int16_t *table, const mfb200_board *boards,
                        const int32_t *hist_off, const int32_t *transforms, float softmax_temp,
                        float *priors, cudaStream_t s);

// FP8 calibration: *slot = max(*slot, max|x|) over n values of format `fmt`;
// and scales[i] = absmax[i] / 448.
void launch_absmax(const void *x, Fmt fmt, long long n, float *slot, cudaStream_t s);
void launch_absmax_to_scale(const float *absmax, int n, float *scales, cudaStream_t s,
                            float qmax = 448.0f);

// Attention-policy logits: raw = q k^T / sqrt(dp) (64x64), the 8x24 promotion
// logits, gathered onto the 1858 moves. qk: [B*64, 2*dp] (q | k);
// ppo3: [3, dp] = ip4_pol_w[r] + ip4_pol_w[3].
void launch_policy_map(const __nv_bfloat16 *qk, int batch, int dp, const float *ppo3,
                       const int16_t *gather, float *policy, cudaStream_t s);

// Value (WDL softmax) and moves-left (relu) output layers from the hidden
// vector h[B, vh + mh] (value hidden first).
void launch_heads(const __nv_bfloat16 *h, int batch, int vh, int mh, const float *w2v,
                  const float *b2v, const float *w2m, const float *b2m, float *wdl, float *mlh,
                  cudaStream_t s);

}  // namespace mfb200
