// encoder.cu -- position histories -> packed input planes on the GPU.
//
// NN::EncodePositionForNN (src/nn/encoder.cpp:249-466) with 8 history planes
// and FillEmptyHistory::FEN_ONLY, for every input format of
// src/nn/proto/net.proto:256-263, followed by PackInputPlaneRaw
// (src/nn/input_plane_packing.h:30-61): the output is the (mask, value) pair
// per plane that the forward's unpack kernel reads. One thread per position
// works on bitboards: a plane is its 64-bit occupancy plus the value of its
// set squares, which is exactly the packed form, so the 112 x 64 float planes
// of the reference are never built.
#include <cstdint>

#include "../../include/mfb200.h"
#include "kernels.cuh"
#include "pdl.cuh"

namespace mfb200 {
namespace {

constexpr int kFlip = 1, kMirror = 2, kTranspose = 4;
constexpr int kWOO = 1, kWOOO = 2, kBOO = 4, kBOOO = 8;
constexpr int kAux = 104;  // first auxiliary plane (13 planes x 8 history boards)

// Bit i of byte j moved to bit 7-i (files mirrored a<->h), encoder.cpp:46-51.
__device__ __forceinline__ uint64_t files_mirrored(uint64_t v) {
  v = ((v >> 1) & 0x5555555555555555ull) | ((v & 0x5555555555555555ull) << 1);
  v = ((v >> 2) & 0x3333333333333333ull) | ((v & 0x3333333333333333ull) << 2);
  v = ((v >> 4) & 0x0F0F0F0F0F0F0F0Full) | ((v & 0x0F0F0F0F0F0F0F0Full) << 4);
  return v;
}
// Ranks mirrored (byte order reversed), encoder.cpp:53-58.
__device__ __forceinline__ uint64_t ranks_mirrored(uint64_t v) {
  const uint32_t lo = static_cast<uint32_t>(v), hi = static_cast<uint32_t>(v >> 32);
  return (static_cast<uint64_t>(__byte_perm(lo, 0, 0x0123)) << 32) | __byte_perm(hi, 0, 0x0123);
}
// Transpose of the 8x8 bit matrix along the a1-h8 diagonal, encoder.cpp:60-68.
__device__ __forceinline__ uint64_t transposed(uint64_t v) {
  v = (v & 0xAA00AA00AA00AA00ull) >> 9 | (v & 0x0055005500550055ull) << 9 | (v & 0x55AA55AA55AA55AAull);
  v = (v & 0xCCCC0000CCCC0000ull) >> 18 | (v & 0x0000333300003333ull) << 18 | (v & 0x3333CCCC3333CCCCull);
  v = (v & 0xF0F0F0F000000000ull) >> 36 | (v & 0x000000000F0F0F0Full) << 36 | (v & 0x0F0F0F0FF0F0F0F0ull);
  return v;
}
__device__ __forceinline__ uint64_t transform_board(uint64_t b, int t) {
  if (b == 0 || b == ~0ull) return b;
  if (t & kFlip) b = files_mirrored(b);
  if (t & kMirror) b = ranks_mirrored(b);
  if (t & kTranspose) b = transposed(b);
  return b;
}
// -1, 0, 1 as the (flipped / mirrored) board compares with its transpose,
// encoder.cpp:88-102.
__device__ __forceinline__ int transpose_order(uint64_t b, int t) {
  if (t & kFlip) b = files_mirrored(b);
  if (t & kMirror) b = ranks_mirrored(b);
  const uint64_t alt = transposed(b);
  return b < alt ? -1 : (b > alt ? 1 : 0);
}

__device__ __forceinline__ uint64_t of_kind(const mfb200_board &p, int k) {
  return p.pieces[0][k] | p.pieces[1][k];
}
__device__ __forceinline__ uint64_t of_side(const mfb200_board &p, int c) {
  return p.pieces[c][0] | p.pieces[c][1] | p.pieces[c][2] | p.pieces[c][3] | p.pieces[c][4] |
         p.pieces[c][5];
}

// The canonicalisation of the position to evaluate, encoder.cpp:104-170:
// none while any castling right remains; flip so our king is on files e-h;
// with pawns on the board nothing more; otherwise mirror so the king is on
// ranks 1-4 and transpose when it is below the diagonal, ties on the
// diagonal broken by comparing piece sets with their transposes.
__device__ int choose_transform(const mfb200_board &p, int us) {
  if (p.castling) return 0;
  uint64_t king = p.pieces[us][5];
  int t = 0;
  if (king & 0x0F0F0F0F0F0F0F0Full) {
    t |= kFlip;
    king = files_mirrored(king);
  }
  if (of_kind(p, 0)) return t;
  if (king & 0xFFFFFFFF00000000ull) {
    t |= kMirror;
    king = ranks_mirrored(king);
  }
  if (king & 0xE0C08000ull) return t | kTranspose;
  if (king & 0x10204080ull) {
    const uint64_t keys[7] = {of_side(p, 0) | of_side(p, 1), of_side(p, us), of_kind(p, 5),
                              of_kind(p, 4), of_kind(p, 3), of_kind(p, 1), of_kind(p, 2)};
    for (int i = 0; i < 7; ++i) {
      const int o = transpose_order(keys[i], t);
      if (o) return o < 0 ? t : (t | kTranspose);
    }
  }
  return t;
}

// IsStartPosition, encoder.cpp:214-238.
__device__ bool is_start_position(const mfb200_board &p) {
  if (p.black_to_move || p.game_ply != 0 || p.rule50 != 0 || p.ep_square >= 0 || p.castling != 15)
    return false;
  const uint64_t white[6] = {0xFF00ull, 0x42ull, 0x24ull, 0x81ull, 0x08ull, 0x10ull};
  for (int k = 0; k < 6; ++k)
    if (p.pieces[0][k] != white[k] || p.pieces[1][k] != ranks_mirrored(white[k])) return false;
  return true;
}

// Castling rights with our side in bits 0-1 (O-O, O-O-O), encoder.cpp:338-360.
__device__ __forceinline__ int castling_for(const mfb200_board &p, int us) {
  const int c = p.castling;
  const int w = ((c & kWOO) ? 1 : 0) | ((c & kWOOO) ? 2 : 0);
  const int b = ((c & kBOO) ? 1 : 0) | ((c & kBOOO) ? 2 : 0);
  return us ? (b | (w << 2)) : (w | (b << 2));
}

__global__ void __launch_bounds__(128)
    encode_kernel(const mfb200_board *__restrict__ boards, const int32_t *__restrict__ offsets,
                  int batch, int fmt, uint64_t *__restrict__ masks, float *__restrict__ values,
                  int32_t *__restrict__ transforms) {
  pdl_wait();
  pdl_launch();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const mfb200_board *h = boards + (offsets[b] - offsets[0]);
  const int n = offsets[b + 1] - offsets[b];
  uint64_t *M = masks + static_cast<long long>(b) * kPlanes;
  float *V = values + static_cast<long long>(b) * kPlanes;
  for (int p = 0; p < kPlanes; ++p) {
    M[p] = 0;
    V[p] = 0.0f;
  }
  // planes of set squares (value 1) and uniform planes (every square = v)
  auto bits = [&](int p, uint64_t m) {
    M[p] = m;
    V[p] = m ? 1.0f : 0.0f;
  };
  auto uniform = [&](int p, float v) {
    M[p] = v != 0.0f ? ~0ull : 0ull;
    V[p] = v;
  };
  if (n <= 0) {
    if (transforms) transforms[b] = 0;
    return;
  }
  const mfb200_board cur = h[n - 1];
  const int us = cur.black_to_move ? 1 : 0, them = 1 - us;
  const bool canonical = fmt == 3 || fmt == 4 || fmt == 5 || fmt == 132 || fmt == 133;
  const bool v2 = fmt == 5 || fmt == 133;
  const bool hecto = fmt == 4 || fmt == 5 || fmt == 132 || fmt == 133;
  const bool arma = fmt == 132 || fmt == 133;
  const int transform = canonical ? choose_transform(cur, us) : 0;
  // auxiliary planes, encoder.cpp:279-336
  if (fmt == 1) {
    const int c = castling_for(cur, us);  // ours O-O, O-O-O, theirs O-O, O-O-O
    uniform(kAux + 0, (c & 2) ? 1.0f : 0.0f);
    uniform(kAux + 1, (c & 1) ? 1.0f : 0.0f);
    uniform(kAux + 2, (c & 8) ? 1.0f : 0.0f);
    uniform(kAux + 3, (c & 4) ? 1.0f : 0.0f);
  } else {
    // rook squares from our side: queenside a1 / a8, kingside h1 / h8
    const int c = castling_for(cur, us);
    bits(kAux + 0, ((c & 2) ? 1ull : 0ull) | ((c & 8) ? (1ull << 56) : 0ull));
    bits(kAux + 1, ((c & 1) ? (1ull << 7) : 0ull) | ((c & 4) ? (1ull << 63) : 0ull));
  }
  if (canonical)
    bits(kAux + 4, cur.ep_square >= 0 ? (1ull << cur.ep_square) : 0ull);
  else
    uniform(kAux + 4, us ? 1.0f : 0.0f);
  uniform(kAux + 5, hecto ? static_cast<float>(cur.rule50) / 100.0f : static_cast<float>(cur.rule50));
  uniform(kAux + 6, (arma && us) ? 1.0f : 0.0f);
  uniform(kAux + 7, 1.0f);
  // history planes, encoder.cpp:362-437. Before the first record the oldest
  // one is repeated (synthesised history); that stops after 8 entries, where
  // the reference would not stop (V2, non-start oldest record with a nonzero
  // rule50 and no repetition).
  const int root = castling_for(cur, us);
  for (int i = 0, hi = n - 1; i < 8; ++i, --hi) {
    if (hi < -8) break;
    const mfb200_board &p = h[hi >= 0 ? hi : 0];
    if (hi < 0 && is_start_position(p)) break;
    if (canonical && hi < n - 1) {
      if (castling_for(p, us) != root) break;
      if (p.ep_square >= 0) break;
    }
    const bool rep = p.repetition != 0;
    if (v2 && i > 0 && !rep) {
      if (p.rule50 == 0) break;
      --i;
      continue;
    }
    const int base = i * 13;
    for (int k = 0; k < 6; ++k) {
      uint64_t o = p.pieces[us][k], t = p.pieces[them][k];
      if (us) {
        o = ranks_mirrored(o);
        t = ranks_mirrored(t);
      }
      bits(base + k, o);
      bits(base + 6 + k, t);
    }
    uniform(base + 12, rep ? 1.0f : 0.0f);
    if (hi < 0 && p.ep_square >= 0) {
      // the pawn that just made the double step, put back on its start rank
      const int e = p.ep_square;
      if (e < 8)
        bits(base + 0, M[base + 0] + ((0x0000000000000100ull - 0x0000000001000000ull) << e));
      else if (e >= 56)
        bits(base + 6, M[base + 6] + ((0x0001000000000000ull - 0x0000000100000000ull) << (e - 56)));
    }
    if (canonical && p.rule50 == 0) break;
  }
  // canonicalisation of the board planes, encoder.cpp:439-455
  if (transform) {
    for (int p = 0; p <= kAux + 4; ++p) {
      if (V[p] != 1.0f) continue;  // all planes here hold 0 or 1
      M[p] = transform_board(M[p], transform);
    }
  }
  if (transforms) transforms[b] = transform;
}

}  // namespace

void launch_encode(const mfb200_board *boards, const int32_t *offsets, int batch, int fmt,
                   uint64_t *masks, float *values, int32_t *transforms, cudaStream_t s) {
  if (batch <= 0) return;
  launch_k(encode_kernel, dim3((batch + 127) / 128), dim3(128), 0, s, 1, boards, offsets, batch, fmt,
           masks, values, transforms);
}

}  // namespace mfb200
