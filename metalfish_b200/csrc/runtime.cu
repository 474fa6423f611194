// runtime.cu -- the B200 BT4 forward behind the C ABI of include/mfb200.h.
//
// A handle owns, per GPU: the packed weights (one arena), an activation
// workspace sized for max_batch, a stream, per-batch-size launch plans and
// (optionally) one CUDA graph per batch size. A batch is sharded contiguously
// across the handle's GPUs with one host thread per GPU; there is no
// collective (positions are independent).
//
// The kernel schedule follows the reference execution plan
// (src/nn/network_execution_plan.cpp:155-223) with the per-stage semantics of
// the reference CPU backend (src/nn/cpu/cpu_network.cpp:580-1491):
//   unpack -> PE dense -> concat -> embedding dense+act -> LN+gates
//   -> embedding FFN -> LN(x + a*ffn)
//   -> per layer: QKV(+smolgen compress) -> smolgen dense1+act+LN
//      -> dense2+act -> LN -> global generator (bias) -> attention
//      -> out-proj + residual -> LN -> FFN1+act -> FFN2 + residual -> LN
//   -> policy embedding+act -> wq|wk -> policy map
//   -> value|moves-left per-square dense+act -> flattened dense+act -> output layers.
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <atomic>
#include <array>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "../../include/mfb200.h"
#include "../../include/mfb200_testing.h"
#include "gemm_host.h"
#include "kernels.cuh"

using namespace mfb200;

namespace {

thread_local std::string t_last_error;
constexpr int kMaxSplits = 32;  // split-K slices of the smolgen dense1 GEMM

struct Fail : std::runtime_error {
  using std::runtime_error::runtime_error;
};

void check(cudaError_t e, const char *what) {
  if (e != cudaSuccess) throw Fail(std::string(what) + ": " + cudaGetErrorString(e));
}

uint16_t f2bf(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

// ------------------------------------------------------------ weight slots
// Global and per-layer tensor slots, in the order of metalfish_b200/layout.py.
enum G {
  G_PREPROC_W, G_PREPROC_B, G_EMB_W, G_EMB_B, G_EMB_LN_G, G_EMB_LN_B, G_MULT_GATE, G_ADD_GATE,
  G_EFFN_W1, G_EFFN_B1, G_EFFN_W2, G_EFFN_B2, G_EFFN_LN_G, G_EFFN_LN_B, G_SMOLGEN_W,
  G_POL_W, G_POL_B, G_POL_WQ, G_POL_BQ, G_POL_WK, G_POL_BK, G_POL_PPO,
  G_VAL_W, G_VAL_B, G_VAL_W1, G_VAL_B1, G_VAL_W2, G_VAL_B2,
  G_MOV_W, G_MOV_B, G_MOV_W1, G_MOV_B1, G_MOV_W2, G_MOV_B2, G_COUNT
};
enum L {
  L_Q_W, L_Q_B, L_K_W, L_K_B, L_V_W, L_V_B, L_O_W, L_O_B,
  L_SG_COMPRESS, L_SG_W1, L_SG_B1, L_SG_LN1_G, L_SG_LN1_B, L_SG_W2, L_SG_B2, L_SG_LN2_G,
  L_SG_LN2_B, L_LN1_G, L_LN1_B, L_FFN_W1, L_FFN_B1, L_FFN_W2, L_FFN_B2, L_LN2_G, L_LN2_B, L_COUNT
};

void slot_sizes(const mfb200_net_desc &n, std::vector<size_t> &g, std::vector<size_t> &l) {
  const size_t d = n.embedding, T = 64, pe = n.pe, ed = n.emb_dff, dp = n.policy_d;
  const size_t c = n.smolgen_compress, h1 = n.smolgen_hidden, hg = size_t(n.heads) * n.smolgen_gen;
  g.assign(G_COUNT, 0);
  g[G_PREPROC_W] = T * pe * 12 * T;
  g[G_PREPROC_B] = T * pe;
  g[G_EMB_W] = d * (112 + pe);
  g[G_EMB_B] = d;
  g[G_EMB_LN_G] = g[G_EMB_LN_B] = d;
  g[G_MULT_GATE] = g[G_ADD_GATE] = d * T;
  g[G_EFFN_W1] = ed * d;
  g[G_EFFN_B1] = ed;
  g[G_EFFN_W2] = d * ed;
  g[G_EFFN_B2] = d;
  g[G_EFFN_LN_G] = g[G_EFFN_LN_B] = d;
  g[G_SMOLGEN_W] = T * T * size_t(n.smolgen_gen);
  g[G_POL_W] = dp * d;
  g[G_POL_B] = dp;
  g[G_POL_WQ] = g[G_POL_WK] = dp * dp;
  g[G_POL_BQ] = g[G_POL_BK] = dp;
  g[G_POL_PPO] = 4 * dp;
  g[G_VAL_W] = size_t(n.value_emb) * d;
  g[G_VAL_B] = n.value_emb;
  g[G_VAL_W1] = size_t(n.value_hidden) * T * n.value_emb;
  g[G_VAL_B1] = n.value_hidden;
  g[G_VAL_W2] = 3 * size_t(n.value_hidden);
  g[G_VAL_B2] = 3;
  g[G_MOV_W] = size_t(n.mlh_emb) * d;
  g[G_MOV_B] = n.mlh_emb;
  g[G_MOV_W1] = size_t(n.mlh_hidden) * T * n.mlh_emb;
  g[G_MOV_B1] = n.mlh_hidden;
  g[G_MOV_W2] = n.mlh_hidden;
  g[G_MOV_B2] = 1;
  l.assign(L_COUNT, 0);
  l[L_Q_W] = l[L_K_W] = l[L_V_W] = l[L_O_W] = d * d;
  l[L_Q_B] = l[L_K_B] = l[L_V_B] = l[L_O_B] = d;
  l[L_SG_COMPRESS] = c * d;
  l[L_SG_W1] = h1 * T * c;
  l[L_SG_B1] = l[L_SG_LN1_G] = l[L_SG_LN1_B] = h1;
  l[L_SG_W2] = hg * h1;
  l[L_SG_B2] = l[L_SG_LN2_G] = l[L_SG_LN2_B] = hg;
  l[L_LN1_G] = l[L_LN1_B] = l[L_LN2_G] = l[L_LN2_B] = d;
  l[L_FFN_W1] = size_t(n.dff) * d;
  l[L_FFN_B1] = n.dff;
  l[L_FFN_W2] = d * n.dff;
  l[L_FFN_B2] = d;
}

size_t blob_floats(const mfb200_net_desc &n) {
  std::vector<size_t> g, l;
  slot_sizes(n, g, l);
  size_t t = 0;
  for (size_t v : g) t += v;
  size_t tl = 0;
  for (size_t v : l) tl += v;
  return t + tl * size_t(n.layers);
}

const char *validate(const mfb200_net_desc &n) {
  if (n.embedding <= 0 || n.embedding % 64) return "embedding must be a positive multiple of 64";
  if (n.layers <= 0) return "layers must be positive";
  if (n.heads <= 0 || n.embedding / n.heads != 32 || n.embedding % n.heads)
    return "head depth (embedding/heads) must be 32";
  if (n.dff <= 0 || n.dff % 16 || n.emb_dff <= 0 || n.emb_dff % 16) return "dff must be a multiple of 16";
  if (n.pe <= 0 || n.pe % 8 || 112 + n.pe > kEmbIn) return "pe must be a multiple of 8, at most 80";
  if (n.smolgen_compress <= 0 || n.smolgen_compress % 16) return "smolgen compress must be a multiple of 16";
  if (n.smolgen_hidden != 128 && n.smolgen_hidden != 256 && n.smolgen_hidden != 512 &&
      n.smolgen_hidden != 1024)
    return "smolgen hidden must be 128, 256, 512 or 1024";
  if (n.smolgen_gen <= 0 || n.smolgen_gen % 16) return "smolgen gen must be a multiple of 16";
  {
    const int hg = n.heads * n.smolgen_gen;  // width of the smolgen LN rows
    bool ok = hg == 128 || hg == 256 || hg == 512 || hg == 1024;
    for (int k : {1, 2, 3, 4, 6, 8}) ok = ok || hg == 2048 * k;
    if (!ok) return "heads x smolgen gen must be 128, 256, 512, 1024 or 2048 x {1,2,3,4,6,8}";
  }
  if (n.policy_d <= 0 || n.policy_d % 64) return "policy embedding must be a multiple of 64";
  if (n.value_emb <= 0 || n.mlh_emb <= 0 || n.value_emb + n.mlh_emb > 64)
    return "value + moves-left embeddings must fit in 64 columns";
  if (n.value_hidden <= 0 || n.mlh_hidden <= 0 || (n.value_hidden + n.mlh_hidden) % 16)
    return "value + moves-left hidden widths must sum to a multiple of 16";
  for (int a : {n.act_default, n.act_smolgen, n.act_ffn})
    if (a < 0 || a > 7) return "unknown activation code";
  const int w = n.embedding;
  if (w != 128 && w != 256 && w != 512 && w != 1024) return "embedding must be 128, 256, 512 or 1024";
  return nullptr;
}

// Policy gather table: policy index -> raw index (64*64 + 8*24 layout of
// src/nn/tables/attention_policy_map.h:15), built from the move geometry of
// the 1858-move encoding (src/nn/policy_map.cpp): every queen/knight move
// from each square in ascending (from, to) order, then the 7th-rank
// underpromotions from_file*24 + to_file*3 + piece for |df| <= 1.
std::vector<int16_t> build_gather() {
  std::vector<int16_t> gather(kPolicy, -1);
  int next = 0;
  for (int from = 0; from < 64; ++from)
    for (int to = 0; to < 64; ++to) {
      if (to == from) continue;
      const int dr = to / 8 - from / 8, df = to % 8 - from % 8;
      const int adr = dr < 0 ? -dr : dr, adf = df < 0 ? -df : df;
      if (dr == 0 || df == 0 || adr == adf || (adr == 1 && adf == 2) || (adr == 2 && adf == 1))
        gather[next++] = static_cast<int16_t>(from * 64 + to);
    }
  for (int ff = 0; ff < 8; ++ff)
    for (int tf = 0; tf < 8; ++tf)
      for (int piece = 0; piece < 3; ++piece)
        if (tf - ff >= -1 && tf - ff <= 1)
          gather[next++] = static_cast<int16_t>(4096 + ff * 24 + tf * 3 + piece);
  if (next != kPolicy) throw Fail("internal: policy map has wrong size");
  return gather;
}

// Policy index of every move (NN::MoveToNNIndex, src/nn/policy_map.cpp:
// 316-360) by promotion kind (0 none, 1 queen, 2 rook, 3 bishop, 4 knight),
// from and to square, derived from the move list of build_gather: plain moves
// and knight promotions by (from, to) among the 1792 queen-line and knight
// moves, queen / rook / bishop promotions from the seventh rank by (from
// file, to file, piece). -1 where the reference has no entry. [5][64][64].
std::vector<int16_t> build_move_index() {
  const std::vector<int16_t> g = build_gather();
  std::vector<int16_t> t(5 * 4096, -1);
  for (int i = 0; i < kPolicy; ++i) {
    if (g[i] < 4096) {
      t[g[i]] = static_cast<int16_t>(i);
      t[4 * 4096 + g[i]] = static_cast<int16_t>(i);
    } else {
      const int r = g[i] - 4096, ff = r / 24, tf = (r % 24) / 3, piece = r % 3;
      t[(1 + piece) * 4096 + (48 + ff) * 64 + 56 + tf] = static_cast<int16_t>(i);
    }
  }
  return t;
}

// ------------------------------------------------------------ device state
struct Mat {  // a weight matrix [rows, ld] on the device (bf16, fp16, e4m3 or int8)
  void *w = nullptr;
  const float *scale = nullptr;  // per-row (output channel) scale for e4m3 / int8
  int rows = 0, ld = 0;
  bool fp8 = false;  // 8-bit (e4m3, or signed integers when i8)
  bool i8 = false;
  bool f16 = false;  // fp16: multiplies the fp16 residual stream directly
};

struct LayerW {
  Mat qkvc, o, f1, f2, sg1, sg2;
  Mat qkvc8, o8, f1_8, f2_8;  // 8-bit copies (e4m3 in FP8 handles, int8 in INT8 handles)
  // Deferred-LayerNorm copies (bf16 handles): QKV+compress scaled by the
  // preceding LayerNorm's gamma along K, FFN1 by ln1's gamma; with their
  // column sums and biases b + W.beta
  Mat qkvc_f, f1_f;
  float *cs_qkvc = nullptr, *bb_qkvc = nullptr, *cs_f1 = nullptr, *bb_f1 = nullptr;
  float *b_qkvc, *b_o, *ln1_g, *ln1_b, *b_f1, *b_f2, *ln2_g, *ln2_b;
  float *b_sg1, *sg_ln1_g, *sg_ln1_b, *b_sg2, *sg_ln2_g, *sg_ln2_b;
};

struct Weights {
  Mat pe, emb, effn1, effn2, sg_global, pol, qk, vm, vm1;
  Mat effn1_8, effn2_8;  // 8-bit copies (FP8 / INT8 handles)
  float *b_pe, *b_emb, *ln_emb_g, *ln_emb_b, *multT, *addT, *b_effn1, *b_effn2, *ln_effn_g,
      *ln_effn_b, *b_pol, *b_qk, *ppo3, *b_vm, *b_vm1, *w2v, *b2v, *w2m, *b2m;
  int16_t *gather;
  std::vector<LayerW> layers;
};

// Builds the packed arena on the host, then one copy to the device.
class ArenaBuilder {
 public:
  size_t add(size_t bytes) {
    const size_t off = (host.size() + 255) & ~size_t(255);
    host.resize(off + bytes);
    return off;
  }
  std::vector<uint8_t> host;
};

// Legal moves per position the priors buffers hold on average (the
// reference keeps at most 256 edges per node, src/mcts/search.cpp:49).
constexpr int kMoveCapacity = 256;
// History records per position the encoder buffers hold on average.
constexpr int kHistoryCapacity = 128;

struct Shard {  // one GPU
  int device = 0;
  cudaStream_t stream = nullptr;
  void *arena = nullptr;
  size_t arena_bytes = 0;
  Weights w;
  // workspace
  void *ws = nullptr;
  size_t ws_bytes = 0;
  uint64_t *masks;
  float *values;
  __nv_bfloat16 *x0, *p, *peo, *QKV, *C, *S1, *S2pre, *S2, *BIAS, *CTX, *H, *E, *QK,
      *VM, *VH;
  __half *Xh, *X1h;  // fp16 residual stream (LN outputs; the residual GEMMs add into it in place)
  float *T, *SK;     // fp32 embedding sum, split-K partials
  float2 *STA, *STB;  // deferred LayerNorm: per-chunk row partials [d / 32, M] of the fp16 stream
  float2 *SA, *SB;    //   and the rows' (mean, rstd) [M]
  float *SPK = nullptr;      // split-K partial products of small-batch GEMMs
  long long spk_floats = 0;
  uint8_t *X8, *X1_8, *CTX8, *H8;  // 8-bit GEMM inputs (FP8 / INT8 handles)
  float *RSX, *RSX1;  // INT8 handles: per-row scales of X8 / X1_8 [M]
  bool int8 = false;  // INT8 handle: the 8-bit GEMMs use signed integer operands
  float *scales, *absmax;    // per-tensor activation scales / calibration maxima
  float *policy, *wdl, *mlh;
  int32_t *move_off;      // legal-move priors: CSR offsets [max_batch + 1]
  int16_t *move_idx;      //   policy index per legal move [max_batch * 256]
  float *priors;          //   priors per legal move [max_batch * 256]
  mfb200_board *boards;   // encoder input: history records [max_batch * 128]
  int32_t *hist_off;      //   CSR offsets [max_batch + 1]
  int32_t *transforms;    //   canonicalisation transform per position [max_batch]
  uint16_t *moves;        // legal moves (from | to << 6 | promotion << 12) [max_batch * 256]
  int16_t *move_table;    // build_move_index() [5 * 4096]
  unsigned *status;
  cudaEvent_t ev[4];
  cudaEvent_t done[4];  // completion of the asynchronous submission in each ticket slot
  // Asynchronous submissions (mfb200_submit_leaves) run in three stages on
  // three streams so that consecutive submissions overlap: the inputs of
  // slot k are copied in on copy_in (in_done[k]), the encode + forward +
  // priors run on `stream` (comp_done[k]) and the outputs go back on
  // copy_out (done[k]). Each slot has its own device inputs and outputs; the
  // forward's workspace is shared (its users are serialised on `stream`).
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  cudaEvent_t in_done[4], comp_done[4];
  struct SlotBufs {
    mfb200_board *boards;
    int32_t *hist_off, *move_off, *transforms;
    uint16_t *moves;
    float *priors, *wdl, *mlh;
    unsigned *status;  // the status word as it was after this slot's forward
  } slots[4] = {};
  void *slot_mem = nullptr;
  struct Step {
    std::string name;
    double flops = 0;
    bool is_gemm = false;
    GemmLaunch g;
    std::function<void(cudaStream_t)> fn;
  };
  struct Plan {
    std::vector<Step> steps;
    cudaGraphExec_t graph = nullptr;
    // test switches (mfb200_testing.h), read once when the plan is built
    bool auto_split = true, pairs = true;
  };
  std::map<int, std::unique_ptr<Plan>> plans;
};

}  // namespace

struct mfb200_handle {
  mfb200_net_desc desc;
  mfb200_config cfg;
  std::vector<std::unique_ptr<Shard>> shards;
  std::mutex mu;
  std::string last_error;
  size_t weight_bytes = 0, ws_bytes = 0;
  std::string device_name;
  bool calibrated = false;  // FP8 activation scales set
  // asynchronous submissions (mfb200_submit_leaves): ticket t uses slot
  // t % kTickets; pending[slot] is the ticket not yet waited for, 0 if none
  static constexpr int kTickets = 4;
  uint64_t next_ticket = 1;
  uint64_t pending[kTickets] = {};
  // errors of finished submissions, kept for mfb200_wait (oldest dropped first)
  std::map<uint64_t, std::string> ticket_errors;
};

namespace {

// FP8 and INT8 handles run the 8-bit plan (e4m3 or signed-integer operands).
bool eight_bit(const mfb200_config &c) {
  return c.precision == MFB200_PRECISION_FP8 || c.precision == MFB200_PRECISION_INT8;
}

// ------------------------------------------------------------ packing
struct Packer {
  const mfb200_net_desc &n;
  const float *blob;
  std::vector<const float *> gp;
  std::vector<std::vector<const float *>> lp;
  Packer(const mfb200_net_desc &n_, const float *b) : n(n_), blob(b) {
    std::vector<size_t> g, l;
    slot_sizes(n, g, l);
    const float *p = blob;
    gp.resize(G_COUNT);
    for (int i = 0; i < G_COUNT; ++i) {
      gp[i] = p;
      p += g[i];
    }
    lp.resize(n.layers);
    for (int k = 0; k < n.layers; ++k) {
      lp[k].resize(L_COUNT);
      for (int i = 0; i < L_COUNT; ++i) {
        lp[k][i] = p;
        p += l[i];
      }
    }
  }
};

// Lays the packed weights out in `ab`; records host offsets in `off` for
// pointer fix-up after the device copy.
struct Layout {
  std::vector<std::pair<void **, size_t>> fix;  // (pointer field, arena offset)
};

template <class T>
void put_f32(ArenaBuilder &ab, Layout &lay, T **field, const float *src, size_t n) {
  const size_t off = ab.add(n * 4);
  if (src) std::memcpy(ab.host.data() + off, src, n * 4);
  lay.fix.push_back({reinterpret_cast<void **>(field), off});
}

// bf16 (or, with f16, fp16) matrix of `rows` x `ld` (zero padded), filled by
// `at(r, c)` for c < cols.
template <class F>
void put_mat(ArenaBuilder &ab, Layout &lay, Mat &m, int rows, int cols, int ld, F at,
             bool f16 = false) {
  const size_t off = ab.add(size_t(rows) * ld * 2);
  uint16_t *dst = reinterpret_cast<uint16_t *>(ab.host.data() + off);
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < ld; ++c) {
      const float v = c < cols ? at(r, c) : 0.0f;
      dst[size_t(r) * ld + c] = f16 ? __half_as_ushort(__float2half_rn(v)) : f2bf(v);
    }
  m.rows = rows;
  m.ld = ld;
  m.fp8 = false;
  m.f16 = f16;
  lay.fix.push_back({&m.w, off});
}

// Host float -> e4m3 (round to nearest, ties to even; saturating at +-448).
// e4m3: 1 sign, 4 exponent bits (bias 7), 3 mantissa bits, no infinities.
uint8_t f2e4m3(float x) {
  static const std::array<float, 127> table = [] {
    std::array<float, 127> t{};
    for (int b = 0; b < 127; ++b) {
      const int e = b >> 3, m = b & 7;
      t[b] = e == 0 ? std::ldexp(m / 8.0f, -6) : std::ldexp(1.0f + m / 8.0f, e - 7);
    }
    return t;
  }();
  const uint8_t sign = std::signbit(x) ? 0x80 : 0;
  float a = std::fabs(x);
  if (!(a == a)) return 0x7F;
  if (a >= table[126]) return sign | 126;
  int lo = 0, hi = 126;  // table[lo] <= a < table[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) / 2;
    (table[mid] <= a ? lo : hi) = mid;
  }
  const float dlo = a - table[lo], dhi = table[hi] - a;
  const int idx = (dhi < dlo || (dhi == dlo && (hi % 2 == 0))) ? hi : lo;
  return sign | static_cast<uint8_t>(idx);
}

// e4m3 matrix with a per-row (output channel) scale: row r is stored as
// round(W[r]/scale[r]) where scale[r] = max|W[r]| / 448.
template <class F>
void put_mat_fp8(ArenaBuilder &ab, Layout &lay, Mat &m, int rows, int cols, int ld, F at) {
  const size_t off = ab.add(size_t(rows) * ld);
  std::vector<float> sc(rows);
  for (int r = 0; r < rows; ++r) {
    float mx = 0.0f;
    for (int c = 0; c < cols; ++c) mx = std::max(mx, std::fabs(at(r, c)));
    sc[r] = mx > 0.0f ? mx / 448.0f : 1.0f;
  }
  uint8_t *dst = ab.host.data() + off;
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < ld; ++c) dst[size_t(r) * ld + c] = c < cols ? f2e4m3(at(r, c) / sc[r]) : 0;
  m.rows = rows;
  m.ld = ld;
  m.fp8 = true;
  lay.fix.push_back({&m.w, off});
  put_f32(ab, lay, const_cast<float **>(&m.scale), sc.data(), sc.size());
}

// Signed 8-bit integer matrix with a per-row (output channel) scale: row r is
// stored as round(W[r] / scale[r]) (nearest, ties away from zero) where
// scale[r] = max|W[r]| / 127.
template <class F>
void put_mat_i8(ArenaBuilder &ab, Layout &lay, Mat &m, int rows, int cols, int ld, F at) {
  const size_t off = ab.add(size_t(rows) * ld);
  std::vector<float> sc(rows);
  for (int r = 0; r < rows; ++r) {
    float mx = 0.0f;
    for (int c = 0; c < cols; ++c) mx = std::max(mx, std::fabs(at(r, c)));
    sc[r] = mx > 0.0f ? mx / 127.0f : 1.0f;
  }
  int8_t *dst = reinterpret_cast<int8_t *>(ab.host.data() + off);
  for (int r = 0; r < rows; ++r)
    for (int c = 0; c < ld; ++c) {
      const float q = c < cols ? std::round(at(r, c) / sc[r]) : 0.0f;
      dst[size_t(r) * ld + c] = static_cast<int8_t>(std::max(-127.0f, std::min(127.0f, q)));
    }
  m.rows = rows;
  m.ld = ld;
  m.fp8 = true;
  m.i8 = true;
  lay.fix.push_back({&m.w, off});
  put_f32(ab, lay, const_cast<float **>(&m.scale), sc.data(), sc.size());
}

// A matrix that multiplies the output of a LayerNorm z = (y - mean) * rstd *
// gamma + beta, prepared for un-normalised input rows y: stored (fp16) as
// W[r][c] * gamma[c], with colsum[r] = sum_c of those stored values and
// bias[r] = b[r] + sum_c W[r][c] * beta[c], so that
// z . W^T + b = rstd * (y . Wg^T - mean * colsum) + bias.
template <class F>
void put_folded(ArenaBuilder &ab, Layout &lay, Mat &m, float **colsum, float **bias, int rows,
                int K, F at, const float *gamma, const float *beta, const float *b) {
  put_mat(ab, lay, m, rows, K, K, [&](int r, int c) { return at(r, c) * gamma[c]; }, true);
  const size_t off = lay.fix.back().second;
  std::vector<float> cs(rows), bb(rows);
  for (int r = 0; r < rows; ++r) {
    const uint16_t *row = reinterpret_cast<const uint16_t *>(ab.host.data() + off) + size_t(r) * K;
    double sc = 0.0, sb = b ? b[r] : 0.0;
    for (int c = 0; c < K; ++c) {
      sc += __half2float(__ushort_as_half(row[c]));
      sb += double(at(r, c)) * beta[c];
    }
    cs[r] = static_cast<float>(sc);
    bb[r] = static_cast<float>(sb);
  }
  put_f32(ab, lay, colsum, cs.data(), cs.size());
  put_f32(ab, lay, bias, bb.data(), bb.size());
}

void pack_weights(const mfb200_net_desc &n, const float *blob, ArenaBuilder &ab, Layout &lay,
                  Weights &W, bool fp8, bool i8) {
  Packer P(n, blob);
  const int d = n.embedding, T = 64, dp = n.policy_d, pe = n.pe;
  const auto &g = P.gp;
  auto dense = [&](Mat &m, const float *src, int rows, int cols, bool f16 = false) {
    put_mat(ab, lay, m, rows, cols, cols, [&](int r, int c) { return src[size_t(r) * cols + c]; },
            f16);
  };
  dense(W.pe, g[G_PREPROC_W], T * pe, 12 * T);
  put_f32(ab, lay, &W.b_pe, g[G_PREPROC_B], size_t(T) * pe);
  put_mat(ab, lay, W.emb, d, 112 + pe, kEmbIn,
          [&](int r, int c) { return g[G_EMB_W][size_t(r) * (112 + pe) + c]; });
  put_f32(ab, lay, &W.b_emb, g[G_EMB_B], d);
  put_f32(ab, lay, &W.ln_emb_g, g[G_EMB_LN_G], d);
  put_f32(ab, lay, &W.ln_emb_b, g[G_EMB_LN_B], d);
  {
    // gates: reference layout is channel-major [d][64] (cpu_network.cpp:1290-1296);
    // stored square-major [64][d] so the LN kernel reads them contiguously.
    std::vector<float> mt(size_t(T) * d), at(size_t(T) * d);
    for (int c = 0; c < d; ++c)
      for (int s = 0; s < T; ++s) {
        mt[size_t(s) * d + c] = g[G_MULT_GATE][size_t(c) * T + s];
        at[size_t(s) * d + c] = g[G_ADD_GATE][size_t(c) * T + s];
      }
    put_f32(ab, lay, &W.multT, mt.data(), mt.size());
    put_f32(ab, lay, &W.addT, at.data(), at.size());
  }
  auto dense8 = [&](Mat &m, const float *src, int rows, int cols) {
    if (i8)
      put_mat_i8(ab, lay, m, rows, cols, cols, [&](int r, int c) { return src[size_t(r) * cols + c]; });
    else
      put_mat_fp8(ab, lay, m, rows, cols, cols, [&](int r, int c) { return src[size_t(r) * cols + c]; });
  };
  // matrices applied to the fp16 residual stream are stored in fp16
  dense(W.effn1, g[G_EFFN_W1], n.emb_dff, d, true);
  if (fp8) {
    dense8(W.effn1_8, g[G_EFFN_W1], n.emb_dff, d);
    dense8(W.effn2_8, g[G_EFFN_W2], d, n.emb_dff);
  }
  put_f32(ab, lay, &W.b_effn1, g[G_EFFN_B1], n.emb_dff);
  dense(W.effn2, g[G_EFFN_W2], d, n.emb_dff);
  put_f32(ab, lay, &W.b_effn2, g[G_EFFN_B2], d);
  put_f32(ab, lay, &W.ln_effn_g, g[G_EFFN_LN_G], d);
  put_f32(ab, lay, &W.ln_effn_b, g[G_EFFN_LN_B], d);
  // shared smolgen generator [4096, gen], its output columns (rows here) in
  // the attention kernel's fragment order
  put_mat(ab, lay, W.sg_global, T * T, n.smolgen_gen, n.smolgen_gen, [&](int r, int c) {
    return g[G_SMOLGEN_W][size_t(attention_bias_column(r)) * n.smolgen_gen + c];
  });
  dense(W.pol, g[G_POL_W], dp, d, true);
  put_f32(ab, lay, &W.b_pol, g[G_POL_B], dp);
  // wq and wk as one [2*dp, dp] matrix (q rows first)
  put_mat(ab, lay, W.qk, 2 * dp, dp, dp, [&](int r, int c) {
    return r < dp ? g[G_POL_WQ][size_t(r) * dp + c] : g[G_POL_WK][size_t(r - dp) * dp + c];
  });
  {
    std::vector<float> b(2 * size_t(dp));
    std::memcpy(b.data(), g[G_POL_BQ], dp * 4);
    std::memcpy(b.data() + dp, g[G_POL_BK], dp * 4);
    put_f32(ab, lay, &W.b_qk, b.data(), b.size());
    std::vector<float> p3(3 * size_t(dp));
    for (int r = 0; r < 3; ++r)
      for (int c = 0; c < dp; ++c)
        p3[size_t(r) * dp + c] = g[G_POL_PPO][size_t(r) * dp + c] + g[G_POL_PPO][size_t(3) * dp + c];
    put_f32(ab, lay, &W.ppo3, p3.data(), p3.size());
  }
  // value | moves-left per-square embedding as one [64, d] matrix
  const int ve = n.value_emb, me = n.mlh_emb, vh = n.value_hidden, mh = n.mlh_hidden;
  put_mat(ab, lay, W.vm, 64, d, d, [&](int r, int c) {
    if (r < ve) return g[G_VAL_W][size_t(r) * d + c];
    if (r < ve + me) return g[G_MOV_W][size_t(r - ve) * d + c];
    return 0.0f;
  }, true);
  {
    std::vector<float> b(64, 0.0f);
    std::memcpy(b.data(), g[G_VAL_B], ve * 4);
    std::memcpy(b.data() + ve, g[G_MOV_B], me * 4);
    put_f32(ab, lay, &W.b_vm, b.data(), 64);
  }
  // flattened dense over the [64 squares x 64 columns] view of that output
  put_mat(ab, lay, W.vm1, vh + mh, 64 * 64, 64 * 64, [&](int r, int k) {
    const int s = k / 64, c = k % 64;
    if (r < vh) return c < ve ? g[G_VAL_W1][size_t(r) * 64 * ve + size_t(s) * ve + c] : 0.0f;
    if (c >= ve && c < ve + me) return g[G_MOV_W1][size_t(r - vh) * 64 * me + size_t(s) * me + (c - ve)];
    return 0.0f;
  });
  {
    std::vector<float> b(vh + mh);
    std::memcpy(b.data(), g[G_VAL_B1], vh * 4);
    std::memcpy(b.data() + vh, g[G_MOV_B1], mh * 4);
    put_f32(ab, lay, &W.b_vm1, b.data(), b.size());
  }
  put_f32(ab, lay, &W.w2v, g[G_VAL_W2], 3 * size_t(vh));
  put_f32(ab, lay, &W.b2v, g[G_VAL_B2], 3);
  put_f32(ab, lay, &W.w2m, g[G_MOV_W2], mh);
  put_f32(ab, lay, &W.b2m, g[G_MOV_B2], 1);
  {
    const std::vector<int16_t> gather = build_gather();
    const size_t off = ab.add(gather.size() * 2);
    std::memcpy(ab.host.data() + off, gather.data(), gather.size() * 2);
    lay.fix.push_back({reinterpret_cast<void **>(&W.gather), off});
  }
  W.layers.resize(n.layers);
  const int c = n.smolgen_compress, h1 = n.smolgen_hidden, hg = n.heads * n.smolgen_gen;
  for (int k = 0; k < n.layers; ++k) {
    const auto &l = P.lp[k];
    LayerW &Lw = W.layers[k];
    // Q | K | V | smolgen compress as one [3d + c, d] matrix
    auto qkvc_at = [&](int r, int col) {
      if (r < d) return l[L_Q_W][size_t(r) * d + col];
      if (r < 2 * d) return l[L_K_W][size_t(r - d) * d + col];
      if (r < 3 * d) return l[L_V_W][size_t(r - 2 * d) * d + col];
      return l[L_SG_COMPRESS][size_t(r - 3 * d) * d + col];
    };
    put_mat(ab, lay, Lw.qkvc, 3 * d + c, d, d, qkvc_at, true);
    if (fp8) {
      if (i8)
        put_mat_i8(ab, lay, Lw.qkvc8, 3 * d + c, d, d, qkvc_at);
      else
        put_mat_fp8(ab, lay, Lw.qkvc8, 3 * d + c, d, d, qkvc_at);
      dense8(Lw.o8, l[L_O_W], d, d);
      dense8(Lw.f1_8, l[L_FFN_W1], n.dff, d);
      dense8(Lw.f2_8, l[L_FFN_W2], d, n.dff);
    }
    {
      std::vector<float> b(3 * size_t(d) + c, 0.0f);
      std::memcpy(b.data(), l[L_Q_B], d * 4);
      std::memcpy(b.data() + d, l[L_K_B], d * 4);
      std::memcpy(b.data() + 2 * d, l[L_V_B], d * 4);
      put_f32(ab, lay, &Lw.b_qkvc, b.data(), b.size());
    }
    dense(Lw.o, l[L_O_W], d, d);
    put_f32(ab, lay, &Lw.b_o, l[L_O_B], d);
    put_f32(ab, lay, &Lw.ln1_g, l[L_LN1_G], d);
    put_f32(ab, lay, &Lw.ln1_b, l[L_LN1_B], d);
    dense(Lw.f1, l[L_FFN_W1], n.dff, d, true);
    if (!fp8) {
      // deferred LayerNorm: QKV reads the stream before the preceding LN
      // (the embedding FFN's for layer 0, else the previous layer's ln2)
      const float *pg = k == 0 ? g[G_EFFN_LN_G] : P.lp[k - 1][L_LN2_G];
      const float *pb = k == 0 ? g[G_EFFN_LN_B] : P.lp[k - 1][L_LN2_B];
      std::vector<float> bq(3 * size_t(d) + c, 0.0f);
      std::memcpy(bq.data(), l[L_Q_B], d * 4);
      std::memcpy(bq.data() + d, l[L_K_B], d * 4);
      std::memcpy(bq.data() + 2 * d, l[L_V_B], d * 4);
      put_folded(ab, lay, Lw.qkvc_f, &Lw.cs_qkvc, &Lw.bb_qkvc, 3 * d + c, d, qkvc_at, pg, pb, bq.data());
      put_folded(ab, lay, Lw.f1_f, &Lw.cs_f1, &Lw.bb_f1, n.dff, d,
                 [&](int r, int col) { return l[L_FFN_W1][size_t(r) * d + col]; }, l[L_LN1_G],
                 l[L_LN1_B], l[L_FFN_B1]);
    }
    put_f32(ab, lay, &Lw.b_f1, l[L_FFN_B1], n.dff);
    dense(Lw.f2, l[L_FFN_W2], d, n.dff);
    put_f32(ab, lay, &Lw.b_f2, l[L_FFN_B2], d);
    put_f32(ab, lay, &Lw.ln2_g, l[L_LN2_G], d);
    put_f32(ab, lay, &Lw.ln2_b, l[L_LN2_B], d);
    dense(Lw.sg1, l[L_SG_W1], h1, 64 * c);
    put_f32(ab, lay, &Lw.b_sg1, l[L_SG_B1], h1);
    put_f32(ab, lay, &Lw.sg_ln1_g, l[L_SG_LN1_G], h1);
    put_f32(ab, lay, &Lw.sg_ln1_b, l[L_SG_LN1_B], h1);
    dense(Lw.sg2, l[L_SG_W2], hg, h1);
    put_f32(ab, lay, &Lw.b_sg2, l[L_SG_B2], hg);
    put_f32(ab, lay, &Lw.sg_ln2_g, l[L_SG_LN2_G], hg);
    put_f32(ab, lay, &Lw.sg_ln2_b, l[L_SG_LN2_B], hg);
  }
}

// ------------------------------------------------------------ workspace
void alloc_workspace(Shard &S, const mfb200_net_desc &n, int max_batch, bool fp8) {
  const size_t B = max_batch, M = B * 64, d = n.embedding;
  const size_t hg = size_t(n.heads) * n.smolgen_gen;
  const size_t hid = std::max<size_t>(n.dff, n.emb_dff);
  std::vector<std::pair<void **, size_t>> parts = {
      {reinterpret_cast<void **>(&S.masks), B * kPlanes * 8},
      {reinterpret_cast<void **>(&S.values), B * kPlanes * 4},
      {reinterpret_cast<void **>(&S.x0), M * kEmbIn * 2},
      {reinterpret_cast<void **>(&S.p), B * kPeInputs * 2},
      {reinterpret_cast<void **>(&S.peo), B * 64 * n.pe * 2},
      {reinterpret_cast<void **>(&S.T), M * d * 4},
      {reinterpret_cast<void **>(&S.Xh), M * d * 2},
      {reinterpret_cast<void **>(&S.SK), size_t(kMaxSplits) * B * n.smolgen_hidden * 4},
      {reinterpret_cast<void **>(&S.X1h), M * d * 2},
      {reinterpret_cast<void **>(&S.STA), M * (d / 32) * 8},
      {reinterpret_cast<void **>(&S.STB), M * (d / 32) * 8},
      {reinterpret_cast<void **>(&S.SA), M * 8},
      {reinterpret_cast<void **>(&S.SPK), size_t(num_sms()) * 128 * 256 * 4},
      {reinterpret_cast<void **>(&S.SB), M * 8},
      {reinterpret_cast<void **>(&S.QKV), M * 3 * d * 2},
      {reinterpret_cast<void **>(&S.C), M * n.smolgen_compress * 2},
      {reinterpret_cast<void **>(&S.S1), B * n.smolgen_hidden * 2},
      {reinterpret_cast<void **>(&S.S2pre), B * hg * 2},
      {reinterpret_cast<void **>(&S.S2), B * hg * 2},
      {reinterpret_cast<void **>(&S.BIAS), B * n.heads * 4096 * 2},
      {reinterpret_cast<void **>(&S.CTX), M * d * 2},
      {reinterpret_cast<void **>(&S.H), M * hid * 2},
      {reinterpret_cast<void **>(&S.E), M * n.policy_d * 2},
      {reinterpret_cast<void **>(&S.QK), M * 2 * n.policy_d * 2},
      {reinterpret_cast<void **>(&S.VM), M * 64 * 2},
      {reinterpret_cast<void **>(&S.VH), B * (n.value_hidden + n.mlh_hidden) * 2},
      {reinterpret_cast<void **>(&S.policy), B * kPolicy * 4},
      {reinterpret_cast<void **>(&S.wdl), B * 3 * 4},
      {reinterpret_cast<void **>(&S.mlh), B * 4},
      {reinterpret_cast<void **>(&S.move_off), (B + 1) * 4},
      {reinterpret_cast<void **>(&S.move_idx), B * kMoveCapacity * 2},
      {reinterpret_cast<void **>(&S.priors), B * kMoveCapacity * 4},
      {reinterpret_cast<void **>(&S.boards), B * kHistoryCapacity * sizeof(mfb200_board)},
      {reinterpret_cast<void **>(&S.hist_off), (B + 1) * 4},
      {reinterpret_cast<void **>(&S.transforms), B * 4},
      {reinterpret_cast<void **>(&S.moves), B * kMoveCapacity * 2},
      {reinterpret_cast<void **>(&S.move_table), 5 * 4096 * 2},
      {reinterpret_cast<void **>(&S.status), 256},
      {reinterpret_cast<void **>(&S.scales), size_t(2 + 4 * n.layers) * 4},
      {reinterpret_cast<void **>(&S.absmax), size_t(2 + 4 * n.layers) * 4},
      {reinterpret_cast<void **>(&S.X8), fp8 ? M * d : 16},
      {reinterpret_cast<void **>(&S.X1_8), fp8 ? M * d : 16},
      {reinterpret_cast<void **>(&S.CTX8), fp8 ? M * d : 16},
      {reinterpret_cast<void **>(&S.H8), fp8 ? M * hid : 16},
      {reinterpret_cast<void **>(&S.RSX), fp8 ? M * 4 : 16},
      {reinterpret_cast<void **>(&S.RSX1), fp8 ? M * 4 : 16},
  };
  size_t total = 0;
  std::vector<size_t> offs;
  for (auto &p : parts) {
    offs.push_back(total);
    total += (p.second + 1023) & ~size_t(1023);
  }
  S.spk_floats = static_cast<long long>(num_sms()) * 128 * 256;
  check(cudaMalloc(&S.ws, total), "workspace allocation");
  S.ws_bytes = total;
  check(cudaMemset(S.ws, 0, total), "workspace clear");
  for (size_t i = 0; i < parts.size(); ++i)
    *parts[i].first = static_cast<uint8_t *>(S.ws) + offs[i];
}

// Device inputs / outputs of the asynchronous submission slots, their copy
// streams and events.
void alloc_slots(Shard &S, int max_batch) {
  const size_t B = max_batch;
  const size_t sizes[] = {B * kHistoryCapacity * sizeof(mfb200_board), (B + 1) * 4, (B + 1) * 4,
                          B * 4, B * kMoveCapacity * 2, B * kMoveCapacity * 4, B * 12, B * 4, 256};
  size_t per = 0;
  for (size_t x : sizes) per += (x + 255) & ~size_t(255);
  check(cudaMalloc(&S.slot_mem, per * 4), "submission buffers");
  check(cudaMemset(S.slot_mem, 0, per * 4), "submission buffers clear");
  for (int k = 0; k < 4; ++k) {
    uint8_t *p = static_cast<uint8_t *>(S.slot_mem) + per * k;
    void *ptrs[9];
    for (int i = 0; i < 9; ++i) {
      ptrs[i] = p;
      p += (sizes[i] + 255) & ~size_t(255);
    }
    Shard::SlotBufs &b = S.slots[k];
    b.boards = static_cast<mfb200_board *>(ptrs[0]);
    b.hist_off = static_cast<int32_t *>(ptrs[1]);
    b.move_off = static_cast<int32_t *>(ptrs[2]);
    b.transforms = static_cast<int32_t *>(ptrs[3]);
    b.moves = static_cast<uint16_t *>(ptrs[4]);
    b.priors = static_cast<float *>(ptrs[5]);
    b.wdl = static_cast<float *>(ptrs[6]);
    b.mlh = static_cast<float *>(ptrs[7]);
    b.status = static_cast<unsigned *>(ptrs[8]);
    check(cudaEventCreateWithFlags(&S.in_done[k], cudaEventDisableTiming), "event");
    check(cudaEventCreateWithFlags(&S.comp_done[k], cudaEventDisableTiming), "event");
  }
  check(cudaStreamCreateWithFlags(&S.copy_in, cudaStreamNonBlocking), "stream");
  check(cudaStreamCreateWithFlags(&S.copy_out, cudaStreamNonBlocking), "stream");
}

// ------------------------------------------------------------ plan
// Split K for GEMMs whose output tiles fill at most half the SMs (small
// batches); the unit tests also run it off.
std::atomic<bool> g_auto_split{true};

int pick_bn(int M, int N) {
  if (N < 128) return 64;
  if (N < 256) return 128;
  const long long tiles256 = static_cast<long long>((M + 127) / 128) * ((N + 255) / 256);
  if (tiles256 >= num_sms()) return 256;
  const long long tiles128 = static_cast<long long>((M + 127) / 128) * ((N + 127) / 128);
  return tiles128 >= num_sms() ? 128 : (tiles128 * 2 <= num_sms() ? 64 : 128);
}

GemmArgs base_args(Shard &S, int M, int N, int K) {
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.a_scale = 1.0f;
  a.alpha = 1.0f;
  a.out_inv_scale = 1.0f;
  a.status = S.status;
  return a;
}

void add_fn(Shard::Plan &P, const char *name, double flops, std::function<void(cudaStream_t)> fn);

// Returns true when the GEMM was split along K (its epilogue then runs in the
// split-K epilogue kernel, which also finalises residual-norm row statistics
// into a.stats_final when that is set).
bool add_gemm(Shard::Plan &P, Shard &S, const char *name, const void *A, long long lda,
              const Mat &W, GemmArgs a) {
  Shard::Step st;
  st.name = name;
  st.is_gemm = true;
  st.flops = 2.0 * a.M * double(a.N) * a.K;
  const int bn = pick_bn(a.M, a.N);
  a.ab_f16 = W.f16 ? 1 : 0;
  // Small M (few positions): the output tiles would occupy only a fraction of
  // the SMs, each streaming its weight rows through the whole K loop. Split K
  // instead so that about one CTA per SM streams a slice of the weights
  // (fp32 partials in S.SPK), and apply the epilogue in a second kernel.
  const long long tiles = static_cast<long long>((a.M + 127) / 128) * ((a.N + bn - 1) / bn);
  const int kblocks = (a.K + (W.fp8 ? 127 : 63)) / (W.fp8 ? 128 : 64);
  a.no_pair = P.pairs ? 0 : 1;
  if (P.auto_split && a.k_splits <= 1 && a.mode != kEpiResidLN && tiles * 2 <= num_sms() &&
      kblocks >= 2) {
    const int splits = static_cast<int>(std::min<long long>({kblocks, num_sms() / tiles, 16}));
    // (at least 3 slices: below that the extra kernel costs more than it saves)
    if (splits >= 3 && static_cast<long long>(splits) * a.M * a.N <= S.spk_floats) {
      GemmArgs p = base_args(S, a.M, a.N, a.K);
      p.ab_f16 = a.ab_f16;
      p.ab_i8 = a.ab_i8;
      p.no_pair = a.no_pair;
      p.out = S.SPK;
      p.out_f32 = 1;
      p.ldo = a.N;
      p.k_splits = splits;
      p.split_stride = static_cast<long long>(a.M) * a.N;
      if (const char *err = plan_gemm(st.g, A, lda, W.w, W.ld, bn, W.fp8, p))
        throw Fail(std::string(name) + " (split-K): " + err);
      const int used = st.g.args.k_splits;
      P.steps.push_back(std::move(st));
      float *part = S.SPK;
      add_fn(P, (std::string(name) + "_splitk").c_str(), 0, [part, used, a](cudaStream_t s) {
        check(launch_splitk_epilogue(part, used, a, s), "split-K epilogue");
      });
      return true;
    }
  }
  if (const char *err = plan_gemm(st.g, A, lda, W.w, W.ld, bn, W.fp8, a))
    throw Fail(std::string(name) + ": " + err);
  P.steps.push_back(std::move(st));
  return false;
}

void add_fn(Shard::Plan &P, const char *name, double flops, std::function<void(cudaStream_t)> fn) {
  Shard::Step st;
  st.name = name;
  st.flops = flops;
  st.fn = std::move(fn);
  P.steps.push_back(std::move(st));
}

// Plan modes: bf16 forward, FP8 forward (e4m3 encoder/embedding-FFN GEMMs
// with per-tensor activation scales read from S.scales), and the bf16 forward
// with absmax probes that calibrates those scales.
enum PlanMode { kPlanBF16 = 0, kPlanFP8 = 1, kPlanCalibrate = 2 };

// Deferred LayerNorm in the bf16 forward (default on; the unit tests also run
// it off). The encoder's ln1 / ln2 are not separate passes: the residual GEMMs
// (output projection, FFN2, embedding FFN2) store the un-normalised sum
// y = LN_prev(stream) + alpha * (x W^T + b) in fp16 with per-32-column row
// statistics, and the GEMMs that read the stream (QKV, FFN1) fold the
// normalisation into their epilogue (rstd * (acc - mean * colsum) + bias, with
// gamma folded into W and beta into the bias). Only the last layer's ln2 runs
// as a kernel, for the heads.
std::atomic<bool> g_fold_ln{true};

// activation-scale slots: embedding LN output, embedding FFN hidden, then per
// layer l: layer input, attention context, ln1 output, FFN hidden
inline int slot_x(int l) { return 2 + 4 * l; }
inline int slot_ctx(int l) { return 3 + 4 * l; }
inline int slot_x1(int l) { return 4 + 4 * l; }
inline int slot_h(int l) { return 5 + 4 * l; }

std::unique_ptr<Shard::Plan> build_plan(Shard &S, const mfb200_net_desc &n, int B, int mode,
                                        int fp8_gemms) {
  auto P = std::make_unique<Shard::Plan>();
  P->auto_split = g_auto_split;
  P->pairs = gemm_pairs_enabled();
  const bool fp8_plan = mode == kPlanFP8, cal = mode == kPlanCalibrate;
  const bool fold = mode == kPlanBF16 && g_fold_ln.load() && !S.w.layers.empty() &&
                    S.w.layers[0].qkvc_f.w != nullptr &&
                    (n.embedding == 128 || n.embedding == 256 || n.embedding == 512 ||
                     n.embedding == 1024);
  // Which GEMM groups run in e4m3 under FP8 (mfb200_config.fp8_gemms bit
  // mask: 1 embedding FFN, 2 QKV, 4 output projection, 8 FFN1, 16 FFN2).
  // INT8 handles: signed 8-bit operands; the LayerNorm outputs (inputs of
  // the embedding FFN1, QKV, FFN1) carry per-row scales, the attention
  // context and the FFN hidden calibrated per-tensor scales.
  const bool i8 = fp8_plan && S.int8;
  const int fp8_mask = fp8_gemms ? fp8_gemms : (S.int8 ? 15 : 31);
  const bool f8e = fp8_plan && (fp8_mask & 1), f8q = fp8_plan && (fp8_mask & 2),
             f8o = fp8_plan && (fp8_mask & 4), f8f1 = fp8_plan && (fp8_mask & 8),
             f8f2 = fp8_plan && (fp8_mask & 16);
  const bool f8e2 = i8 ? f8f2 : f8e;  // the embedding FFN2 (reads the FFN hidden)
  float *rs_x = i8 ? S.RSX : nullptr, *rs_x1 = i8 ? S.RSX1 : nullptr;
  // A operand of an 8-bit GEMM: per-row scales (INT8, LayerNorm outputs) or
  // the per-tensor scale of calibration slot `slot`
  auto set_a8 = [&](GemmArgs &a, const Mat &Wm, const float *row_scale, int slot) {
    a.col_scale = Wm.scale;
    a.ab_i8 = Wm.i8 ? 1 : 0;
    if (Wm.i8 && row_scale)
      a.a_row_scale = row_scale;
    else
      a.a_scale_ptr = S.scales + slot;
  };
  const long long Md = static_cast<long long>(B) * 64 * n.embedding;
  auto probe = [&](const char *name, const void *x, Fmt fmt, long long cnt, int slot) {
    if (cal)
      add_fn(*P, name, 0, [&S, x, fmt, cnt, slot](cudaStream_t s) {
        launch_absmax(x, fmt, cnt, S.absmax + slot, s);
      });
  };
  const int M = B * 64, d = n.embedding, dp = n.policy_d, H = n.heads;
  const int hg = n.heads * n.smolgen_gen, vh = n.value_hidden, mh = n.mlh_hidden;
  const float alpha = std::pow(2.0f * static_cast<float>(n.layers), -0.25f);  // plan :1152-1162
  const float eps = 1e-3f;  // PE_DENSE epsilons (plan :1164-1193)
  Weights &W = S.w;
  auto row_stats = [&](float2 *part, float2 *out) {
    add_fn(*P, "row_stats", 0, [part, out, M, d, eps](cudaStream_t s) {
      launch_row_stats(part, M, d, eps, out, s);
    });
  };

  add_fn(*P, "unpack", 0, [&S, B](cudaStream_t s) { launch_unpack(S.masks, S.values, B, S.x0, S.p, s); });
  {
    GemmArgs a = base_args(S, B, 64 * n.pe, kPeInputs);
    a.bias = W.b_pe;
    a.out = S.peo;
    a.ldo = 64 * n.pe;
    add_gemm(*P, S, "pe_dense", S.p, kPeInputs, W.pe, a);
  }
  add_fn(*P, "pe_concat", 0, [&S, B, pe = n.pe](cudaStream_t s) { launch_pe_concat(S.peo, B, pe, S.x0, s); });
  {
    GemmArgs a = base_args(S, M, d, kEmbIn);
    a.bias = W.b_emb;
    a.act = n.act_default;
    a.out = S.T;
    a.out_f32 = 1;
    a.ldo = d;
    add_gemm(*P, S, "emb_dense", S.x0, kEmbIn, W.emb, a);
  }
  add_fn(*P, "emb_ln_gates", 0, [&S, &W, M, d, eps, f8e, rs_x1](cudaStream_t s) {
    launch_layernorm_q(S.T, Fmt::F32, M, d, W.ln_emb_g, W.ln_emb_b, eps, W.multT, W.addT,
                       nullptr, S.X1h, Fmt::F16, f8e ? S.X1_8 : nullptr, S.scales + 0, s, f8e ? rs_x1 : nullptr);
  });
  probe("absmax_emb_x", S.X1h, Fmt::F16, Md, 0);
  {
    GemmArgs a = base_args(S, M, n.emb_dff, d);
    a.bias = W.b_effn1;
    a.act = n.act_ffn;
    a.out = S.H;
    a.ldo = n.emb_dff;
    if (f8e2) {  // 8-bit hidden for an 8-bit embedding FFN2
      a.out = S.H8;
      a.out_fp8 = 1;
      a.out_i8 = i8 ? 1 : 0;
      a.out_scale_ptr = S.scales + 1;
    }
    if (f8e) {
      set_a8(a, W.effn1_8, rs_x1, 0);
      add_gemm(*P, S, "emb_ffn1", S.X1_8, d, W.effn1_8, a);
    } else {
      add_gemm(*P, S, "emb_ffn1", S.X1h, d, W.effn1, a);
    }
    probe("absmax_emb_h", S.H, Fmt::BF16, static_cast<long long>(M) * n.emb_dff, 1);
    GemmArgs b = base_args(S, M, d, n.emb_dff);
    // x1 (fp16 stream) += alpha * ffn (in place; the LN below reads the sum)
    b.mode = kEpiAccum;
    if (fold) {  // same sum, plus its row statistics for layer 0's folded QKV
      b.mode = kEpiResidNorm;
      b.resid16 = S.X1h;
      b.ldr16 = d;
      b.stats_out = S.STA;
      b.stats_final = S.SA;
      b.ln_eps = eps;
    }
    b.bias = W.b_effn2;
    b.alpha = alpha;
    b.out = S.X1h;
    b.out_f16 = 1;
    b.ldo = d;
    if (f8e2) {
      set_a8(b, W.effn2_8, nullptr, 1);
      add_gemm(*P, S, "emb_ffn2", S.H8, n.emb_dff, W.effn2_8, b);
    } else {
      if (!add_gemm(*P, S, "emb_ffn2", S.H, n.emb_dff, W.effn2, b) && fold) row_stats(S.STA, S.SA);
    }
  }
  if (!fold)
    add_fn(*P, "emb_ffn_ln", 0, [&S, &W, M, d, eps, f8q, rs_x](cudaStream_t s) {
      launch_layernorm_q(S.X1h, Fmt::F16, M, d, W.ln_effn_g, W.ln_effn_b, eps, nullptr, nullptr,
                         nullptr, S.Xh, Fmt::F16, f8q ? S.X8 : nullptr, S.scales + slot_x(0), s, f8q ? rs_x : nullptr);
    });
  probe("absmax_x", S.Xh, Fmt::F16, Md, slot_x(0));
  for (int k = 0; k < n.layers; ++k) {
    LayerW &Lw = W.layers[k];
    {
      GemmArgs a = base_args(S, M, 3 * d + n.smolgen_compress, d);
      a.bias = Lw.b_qkvc;
      a.out = S.QKV;
      a.ldo = 3 * d;
      a.out2 = S.C;
      a.ldo2 = n.smolgen_compress;
      a.split = 3 * d;
      if (f8q) {
        set_a8(a, Lw.qkvc8, rs_x, slot_x(k));
        add_gemm(*P, S, "qkv", S.X8, d, Lw.qkvc8, a);
      } else if (fold) {
        a.bias = Lw.bb_qkvc;
        a.fold_stats = S.SA;
        a.fold_colsum = Lw.cs_qkvc;
        a.ln_eps = eps;
        add_gemm(*P, S, "qkv", S.X1h, d, Lw.qkvc_f, a);
      } else {
        add_gemm(*P, S, "qkv", S.Xh, d, Lw.qkvc, a);
      }
    }
    {
      // smolgen dense1 over the flattened [B, 64*c] compress output: M = B is
      // skinny and K = 64*c long, so split K across CTAs, then one kernel sums
      // the partials and applies bias, activation and LN (eps 1e-3).
      const int h1 = n.smolgen_hidden, K1 = 64 * n.smolgen_compress;
      GemmArgs a = base_args(S, B, h1, K1);
      const long long tiles = static_cast<long long>((B + 127) / 128) * ((h1 + 255) / 256);
      a.k_splits = static_cast<int>(std::max<long long>(1, std::min<long long>(kMaxSplits, num_sms() / tiles)));
      a.out = S.SK;
      a.ldo = h1;
      a.out_f32 = 1;
      a.split_stride = static_cast<long long>(B) * h1;
      add_gemm(*P, S, "smolgen_dense1", S.C, K1, Lw.sg1, a);
      const int splits = P->steps.back().g.args.k_splits;
      add_fn(*P, "smolgen_dense1_reduce_ln", 0, [&S, &Lw, B, h1, splits, act = n.act_smolgen, eps](cudaStream_t s) {
        launch_splitk_act_ln(S.SK, splits, static_cast<long long>(B) * h1, B, h1, Lw.b_sg1, act,
                             Lw.sg_ln1_g, Lw.sg_ln1_b, eps, S.S1, s);
      });
    }
    {
      GemmArgs a = base_args(S, B, hg, n.smolgen_hidden);
      a.bias = Lw.b_sg2;
      a.act = n.act_smolgen;
      a.out = S.S2pre;
      a.ldo = hg;
      add_gemm(*P, S, "smolgen_dense2", S.S1, n.smolgen_hidden, Lw.sg2, a);
    }
    add_fn(*P, "smolgen_ln2", 0, [&S, &Lw, B, hg, eps](cudaStream_t s) {
      launch_layernorm(S.S2pre, false, B, hg, Lw.sg_ln2_g, Lw.sg_ln2_b, eps, nullptr, nullptr, S.S2, nullptr, s);
    });
    {
      GemmArgs a = base_args(S, B * H, 4096, n.smolgen_gen);
      a.out = S.BIAS;
      a.ldo = 4096;
      a.a_scale = 1.4426950408889634f;  // log2(e): the attention's softmax runs in base 2
      add_gemm(*P, S, "smolgen_global", S.S2, n.smolgen_gen, W.sg_global, a);
    }
    add_fn(*P, "attention", 4.0 * B * H * 64.0 * 64.0 * 32.0, [&S, B, H, d, f8o, i8, k](cudaStream_t s) {
      launch_attention(S.QKV, 3LL * d, S.BIAS, B, H, d, S.CTX, s, f8o ? S.CTX8 : nullptr,
                       S.scales + slot_ctx(k), i8 ? 1 : 0);
    });
    probe("absmax_ctx", S.CTX, Fmt::BF16, Md, slot_ctx(k));
    {
      GemmArgs a = base_args(S, M, d, d);
      // x (fp16 stream) += alpha * attention output (in place; ln1 reads the sum)
      a.mode = kEpiAccum;
      a.bias = Lw.b_o;
      a.alpha = alpha;
      a.out = S.Xh;
      a.out_f16 = 1;
      a.ldo = d;
      if (fold) {
        // stream y (X1h) -> LN_prev(y) + alpha * attention output, in place
        a.mode = kEpiResidNorm;
        a.out = S.X1h;
        a.resid16 = S.X1h;
        a.ldr16 = d;
        a.rn_stats = S.SA;
        a.rn_gamma = k == 0 ? W.ln_effn_g : W.layers[k - 1].ln2_g;
        a.rn_beta = k == 0 ? W.ln_effn_b : W.layers[k - 1].ln2_b;
        a.stats_out = S.STB;
        a.stats_final = S.SB;
        a.ln_eps = eps;
      }
      if (f8o) {
        set_a8(a, Lw.o8, nullptr, slot_ctx(k));
        add_gemm(*P, S, "out_proj", S.CTX8, d, Lw.o8, a);
      } else {
        if (!add_gemm(*P, S, "out_proj", S.CTX, d, Lw.o, a) && fold) row_stats(S.STB, S.SB);
      }
    }
    if (!fold)
      add_fn(*P, "ln1", 0, [&S, &Lw, M, d, eps, f8f1, k, rs_x1](cudaStream_t s) {
        launch_layernorm_q(S.Xh, Fmt::F16, M, d, Lw.ln1_g, Lw.ln1_b, eps, nullptr, nullptr,
                           nullptr, S.X1h, Fmt::F16, f8f1 ? S.X1_8 : nullptr, S.scales + slot_x1(k), s,
                           f8f1 ? rs_x1 : nullptr);
      });
    probe("absmax_x1", S.X1h, Fmt::F16, Md, slot_x1(k));
    {
      GemmArgs a = base_args(S, M, n.dff, d);
      a.bias = Lw.b_f1;
      a.act = n.act_ffn;
      a.out = S.H;
      a.ldo = n.dff;
      if (f8f2) {  // 8-bit hidden for an 8-bit FFN2
        a.out = S.H8;
        a.out_fp8 = 1;
        a.out_i8 = i8 ? 1 : 0;
        a.out_scale_ptr = S.scales + slot_h(k);
      }
      if (f8f1) {
        set_a8(a, Lw.f1_8, rs_x1, slot_x1(k));
        add_gemm(*P, S, "ffn1", S.X1_8, d, Lw.f1_8, a);
      } else if (fold) {
        a.bias = Lw.bb_f1;
        a.fold_stats = S.SB;
        a.fold_colsum = Lw.cs_f1;
        a.ln_eps = eps;
        add_gemm(*P, S, "ffn1", S.X1h, d, Lw.f1_f, a);
      } else {
        add_gemm(*P, S, "ffn1", S.X1h, d, Lw.f1, a);
      }
      probe("absmax_h", S.H, Fmt::BF16, static_cast<long long>(M) * n.dff, slot_h(k));
      GemmArgs b = base_args(S, M, d, n.dff);
      // x1 (fp16 stream) += alpha * ffn (in place; ln2 reads the sum)
      b.mode = kEpiAccum;
      b.bias = Lw.b_f2;
      b.alpha = alpha;
      b.out = S.X1h;
      b.out_f16 = 1;
      b.ldo = d;
      if (fold) {
        b.mode = kEpiResidNorm;
        b.resid16 = S.X1h;
        b.ldr16 = d;
        b.rn_stats = S.SB;
        b.rn_gamma = Lw.ln1_g;
        b.rn_beta = Lw.ln1_b;
        b.stats_out = S.STA;
        b.stats_final = S.SA;
        b.ln_eps = eps;
      }
      if (f8f2) {
        set_a8(b, Lw.f2_8, nullptr, slot_h(k));
        add_gemm(*P, S, "ffn2", S.H8, n.dff, Lw.f2_8, b);
      } else {
        if (!add_gemm(*P, S, "ffn2", S.H, n.dff, Lw.f2, b) && fold) row_stats(S.STA, S.SA);
      }
    }
    {
      // the last layer's output feeds the bf16 heads; earlier ones feed the
      // next layer's (e4m3, under FP8) QKV projection
      const bool last = k + 1 == n.layers;
      const bool q8 = f8q && !last;
      if (!fold || last)  // deferred LayerNorm: only the heads' input is normalised here
        add_fn(*P, "ln2", 0, [&S, &Lw, M, d, eps, q8, k, rs_x](cudaStream_t s) {
          launch_layernorm_q(S.X1h, Fmt::F16, M, d, Lw.ln2_g, Lw.ln2_b, eps, nullptr, nullptr,
                             nullptr, S.Xh, Fmt::F16, q8 ? S.X8 : nullptr, S.scales + slot_x(k + 1), s,
                             q8 ? rs_x : nullptr);
        });
      if (!last) probe("absmax_x", S.Xh, Fmt::F16, Md, slot_x(k + 1));
    }
  }
  {
    GemmArgs a = base_args(S, M, dp, d);
    a.bias = W.b_pol;
    a.act = n.act_default;
    a.out = S.E;
    a.ldo = dp;
    add_gemm(*P, S, "policy_embed", S.Xh, d, W.pol, a);
    GemmArgs b = base_args(S, M, 2 * dp, dp);
    b.bias = W.b_qk;
    b.out = S.QK;
    b.ldo = 2 * dp;
    add_gemm(*P, S, "policy_qk", S.E, dp, W.qk, b);
  }
  add_fn(*P, "policy_map", 2.0 * B * 64.0 * 64.0 * dp, [&S, &W, B, dp](cudaStream_t s) {
    launch_policy_map(S.QK, B, dp, W.ppo3, W.gather, S.policy, s);
  });
  {
    GemmArgs a = base_args(S, M, 64, d);
    a.bias = W.b_vm;
    a.act = n.act_default;
    a.out = S.VM;
    a.ldo = 64;
    add_gemm(*P, S, "value_mlh_embed", S.Xh, d, W.vm, a);
    GemmArgs b = base_args(S, B, vh + mh, 64 * 64);
    b.bias = W.b_vm1;
    b.act = n.act_default;
    b.out = S.VH;
    b.ldo = vh + mh;
    add_gemm(*P, S, "value_mlh_dense1", S.VM, 64 * 64, W.vm1, b);
  }
  add_fn(*P, "heads", 0, [&S, &W, B, vh, mh](cudaStream_t s) {
    launch_heads(S.VH, B, vh, mh, W.w2v, W.b2v, W.w2m, W.b2m, S.wdl, S.mlh, s);
  });
  return P;
}

void run_steps(Shard::Plan &P, cudaStream_t s) {
  for (auto &st : P.steps) {
    if (st.is_gemm)
      check(launch_gemm(st.g, s), st.name.c_str());
    else
      st.fn(s);
  }
  check(cudaGetLastError(), "kernel launch");
}

Shard::Plan &get_plan(mfb200_handle *h, Shard &S, int B, int mode = -1) {
  if (mode < 0) mode = eight_bit(h->cfg) ? kPlanFP8 : kPlanBF16;
  if (mode == kPlanFP8 && !h->calibrated)
    throw Fail("FP8 handle used before mfb200_calibrate set its activation scales");
  const int key = B * 4 + mode;
  auto it = S.plans.find(key);
  if (it != S.plans.end()) return *it->second;
  auto P = build_plan(S, h->desc, B, mode, h->cfg.fp8_gemms);
  if (mode == kPlanCalibrate) {  // run eagerly, never captured
    Shard::Plan &ref = *P;
    S.plans[key] = std::move(P);
    return ref;
  }
  // First run eagerly (also sets kernel attributes), then capture a graph.
  run_steps(*P, S.stream);
  check(cudaStreamSynchronize(S.stream), "first forward");
  if (h->cfg.use_graphs) {
    cudaGraph_t graph;
    check(cudaStreamBeginCapture(S.stream, cudaStreamCaptureModeThreadLocal), "graph capture begin");
    run_steps(*P, S.stream);
    check(cudaStreamEndCapture(S.stream, &graph), "graph capture end");
    check(cudaGraphInstantiate(&P->graph, graph, 0), "graph instantiate");
    cudaGraphDestroy(graph);
  }
  Shard::Plan &ref = *P;
  S.plans[key] = std::move(P);
  return ref;
}

void forward(mfb200_handle *h, Shard &S, int B, cudaStream_t s) {
  Shard::Plan &P = get_plan(h, S, B);
  if (P.graph)
    check(cudaGraphLaunch(P.graph, s), "graph launch");
  else
    run_steps(P, s);
}

void check_status(Shard &S) {
  unsigned st = 0;
  check(cudaMemcpy(&st, S.status, 4, cudaMemcpyDeviceToHost), "status read");
  if (st) {
    cudaMemset(S.status, 0, 4);
    throw Fail("device wait timed out in a GEMM (code " + std::to_string(st) + ")");
  }
}

int fail(mfb200_handle *h, const std::string &msg) {
  t_last_error = msg;
  if (h) h->last_error = msg;
  return 1;
}

}  // namespace

// ============================================================ C ABI
extern "C" void mfb200_debug_set_fold_ln(int enable) { g_fold_ln = enable != 0; }

// One eager forward of `batch` positions on the handle's first GPU in which
// layer 0's QKV GEMM announces its first pipeline stage but never loads it,
// with that GEMM's barrier waits limited to wait_ns. Returns the error the
// forward reports (nonzero, "device wait timed out ..."); the handle stays
// usable.
extern "C" int mfb200_debug_forward_withheld(mfb200_handle *h, int batch,
                                             unsigned long long wait_ns) {
  if (!h) return fail(nullptr, "mfb200_debug_forward_withheld: null handle");
  std::lock_guard<std::mutex> lock(h->mu);
  try {
    Shard &S = *h->shards[0];
    check(cudaSetDevice(S.device), "cudaSetDevice");
    if (batch <= 0 || batch > h->cfg.max_batch / static_cast<int>(h->shards.size()))
      throw Fail("batch out of range");
    Shard::Plan &P = get_plan(h, S, batch);
    bool injected = false;
    for (auto &st : P.steps) {
      if (st.is_gemm && !injected && st.name == "qkv") {
        GemmLaunch g = st.g;
        g.args.debug_withhold = 1;
        g.args.wait_ns = wait_ns;
        check(launch_gemm(g, S.stream), "withheld qkv");
        injected = true;
      } else if (st.is_gemm) {
        check(launch_gemm(st.g, S.stream), st.name.c_str());
      } else {
        st.fn(S.stream);
      }
    }
    check(cudaStreamSynchronize(S.stream), "forward");
    check_status(S);
  } catch (const std::exception &e) {
    return fail(h, std::string("mfb200_debug_forward_withheld: ") + e.what());
  }
  return 0;
}

extern "C" void mfb200_debug_set_auto_split(int enable) { g_auto_split = enable != 0; }

extern "C" size_t mfb200_weight_bytes(const mfb200_net_desc *desc) {
  return desc ? blob_floats(*desc) * sizeof(float) : 0;
}

extern "C" int mfb200_create(const mfb200_net_desc *desc, const void *weights, size_t bytes,
                             const mfb200_config *cfg, mfb200_handle **out) {
  if (!desc || !weights || !cfg || !out) return fail(nullptr, "mfb200_create: null argument");
  *out = nullptr;
  if (const char *err = validate(*desc)) return fail(nullptr, std::string("mfb200_create: ") + err);
  if (bytes != blob_floats(*desc) * sizeof(float))
    return fail(nullptr, "mfb200_create: weight blob has " + std::to_string(bytes) +
                             " bytes, expected " + std::to_string(blob_floats(*desc) * 4));
  if (cfg->precision != MFB200_PRECISION_BF16 && cfg->precision != MFB200_PRECISION_FP8 &&
      cfg->precision != MFB200_PRECISION_INT8)
    return fail(nullptr, "mfb200_create: unknown precision");
  if (cfg->max_batch <= 0) return fail(nullptr, "mfb200_create: max_batch must be positive");
  auto h = std::make_unique<mfb200_handle>();
  h->desc = *desc;
  h->cfg = *cfg;
  if (h->cfg.num_devices <= 0) h->cfg.num_devices = 1;
  try {
    int count = 0;
    check(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if (cfg->device < 0 || cfg->device + h->cfg.num_devices > count)
      throw Fail("requested devices " + std::to_string(cfg->device) + ".." +
                 std::to_string(cfg->device + h->cfg.num_devices - 1) + " but " +
                 std::to_string(count) + " visible");
    ArenaBuilder ab;
    Layout lay;
    Weights proto;
    pack_weights(*desc, static_cast<const float *>(weights), ab, lay, proto, eight_bit(*cfg),
                 cfg->precision == MFB200_PRECISION_INT8);
    const int per = (cfg->max_batch + h->cfg.num_devices - 1) / h->cfg.num_devices;
    for (int i = 0; i < h->cfg.num_devices; ++i) {
      auto S = std::make_unique<Shard>();
      S->device = cfg->device + i;
      check(cudaSetDevice(S->device), "cudaSetDevice");
      cudaDeviceProp prop;
      check(cudaGetDeviceProperties(&prop, S->device), "cudaGetDeviceProperties");
      if (prop.major != 10) throw Fail(std::string("device is not an sm_100 GPU: ") + prop.name);
      h->device_name = prop.name;
      check(cudaStreamCreateWithFlags(&S->stream, cudaStreamNonBlocking), "stream");
      for (auto &e : S->ev) check(cudaEventCreate(&e), "event");
      for (auto &e : S->done) check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
      check(cudaMalloc(&S->arena, ab.host.size()), "weight allocation");
      S->arena_bytes = ab.host.size();
      check(cudaMemcpy(S->arena, ab.host.data(), ab.host.size(), cudaMemcpyHostToDevice),
            "weight upload");
      // point the weight directory at this device's arena, then copy it
      for (auto &f : lay.fix) *f.first = static_cast<uint8_t *>(S->arena) + f.second;
      S->w = proto;
      alloc_workspace(*S, *desc, per, eight_bit(*cfg));
      S->int8 = cfg->precision == MFB200_PRECISION_INT8;
      alloc_slots(*S, per);
      {
        const std::vector<int16_t> table = build_move_index();
        check(cudaMemcpy(S->move_table, table.data(), table.size() * 2, cudaMemcpyHostToDevice),
              "move table upload");
      }
      h->weight_bytes = S->arena_bytes;
      h->ws_bytes = S->ws_bytes;
      h->shards.push_back(std::move(S));
    }
  } catch (const std::exception &e) {
    for (auto &S : h->shards) {
      cudaSetDevice(S->device);
      if (S->arena) cudaFree(S->arena);
      if (S->ws) cudaFree(S->ws);
      if (S->stream) cudaStreamDestroy(S->stream);
    }
    return fail(nullptr, std::string("mfb200_create: ") + e.what());
  }
  *out = h.release();
  return 0;
}

namespace {
int eval_shard(mfb200_handle *h, Shard &S, const uint64_t *masks, const float *values, int B,
               float *policy, float *wdl, float *mlh, float *ms) {
  check(cudaSetDevice(S.device), "cudaSetDevice");
  cudaStream_t s = S.stream;
  check(cudaEventRecord(S.ev[0], s), "event");
  check(cudaMemcpyAsync(S.masks, masks, size_t(B) * kPlanes * 8, cudaMemcpyHostToDevice, s), "H2D masks");
  check(cudaMemcpyAsync(S.values, values, size_t(B) * kPlanes * 4, cudaMemcpyHostToDevice, s), "H2D values");
  check(cudaEventRecord(S.ev[1], s), "event");
  forward(h, S, B, s);
  check(cudaEventRecord(S.ev[2], s), "event");
  if (policy)
    check(cudaMemcpyAsync(policy, S.policy, size_t(B) * kPolicy * 4, cudaMemcpyDeviceToHost, s), "D2H policy");
  if (wdl) check(cudaMemcpyAsync(wdl, S.wdl, size_t(B) * 12, cudaMemcpyDeviceToHost, s), "D2H wdl");
  if (mlh) check(cudaMemcpyAsync(mlh, S.mlh, size_t(B) * 4, cudaMemcpyDeviceToHost, s), "D2H mlh");
  check(cudaEventRecord(S.ev[3], s), "event");
  check(cudaStreamSynchronize(s), "forward");
  check_status(S);
  cudaEventElapsedTime(&ms[0], S.ev[0], S.ev[1]);
  cudaEventElapsedTime(&ms[1], S.ev[1], S.ev[2]);
  cudaEventElapsedTime(&ms[2], S.ev[2], S.ev[3]);
  cudaEventElapsedTime(&ms[3], S.ev[0], S.ev[3]);
  return 0;
}
// The forward followed by the legal-move priors of the shard's positions;
// offsets/index/priors are the shard's slices of the caller's CSR arrays.
int eval_shard_priors(mfb200_handle *h, Shard &S, const uint64_t *masks, const float *values,
                      int B, const int32_t *offsets, const int16_t *index, float temp,
                      float *priors, float *wdl, float *mlh, float *ms) {
  check(cudaSetDevice(S.device), "cudaSetDevice");
  cudaStream_t s = S.stream;
  const int32_t nmoves = offsets[B] - offsets[0];
  check(cudaEventRecord(S.ev[0], s), "event");
  check(cudaMemcpyAsync(S.masks, masks, size_t(B) * kPlanes * 8, cudaMemcpyHostToDevice, s), "H2D masks");
  check(cudaMemcpyAsync(S.values, values, size_t(B) * kPlanes * 4, cudaMemcpyHostToDevice, s), "H2D values");
  check(cudaMemcpyAsync(S.move_off, offsets, size_t(B + 1) * 4, cudaMemcpyHostToDevice, s), "H2D offsets");
  if (nmoves > 0)
    check(cudaMemcpyAsync(S.move_idx, index, size_t(nmoves) * 2, cudaMemcpyHostToDevice, s), "H2D moves");
  check(cudaEventRecord(S.ev[1], s), "event");
  forward(h, S, B, s);
  launch_priors(S.policy, B, S.move_off, S.move_idx, temp, S.priors, s);
  check(cudaGetLastError(), "priors launch");
  check(cudaEventRecord(S.ev[2], s), "event");
  if (priors && nmoves > 0)
    check(cudaMemcpyAsync(priors, S.priors, size_t(nmoves) * 4, cudaMemcpyDeviceToHost, s), "D2H priors");
  if (wdl) check(cudaMemcpyAsync(wdl, S.wdl, size_t(B) * 12, cudaMemcpyDeviceToHost, s), "D2H wdl");
  if (mlh) check(cudaMemcpyAsync(mlh, S.mlh, size_t(B) * 4, cudaMemcpyDeviceToHost, s), "D2H mlh");
  check(cudaEventRecord(S.ev[3], s), "event");
  check(cudaStreamSynchronize(s), "forward");
  check_status(S);
  cudaEventElapsedTime(&ms[0], S.ev[0], S.ev[1]);
  cudaEventElapsedTime(&ms[1], S.ev[1], S.ev[2]);
  cudaEventElapsedTime(&ms[2], S.ev[2], S.ev[3]);
  cudaEventElapsedTime(&ms[3], S.ev[0], S.ev[3]);
  return 0;
}
// Upload one shard's histories and encode them into S.masks / S.values.
void encode_shard(Shard &S, const mfb200_board *boards, const int32_t *offsets, int B, int fmt,
                  cudaStream_t s) {
  const int32_t nb = offsets[B] - offsets[0];
  check(cudaMemcpyAsync(S.hist_off, offsets, size_t(B + 1) * 4, cudaMemcpyHostToDevice, s), "H2D offsets");
  if (nb > 0)
    check(cudaMemcpyAsync(S.boards, boards, size_t(nb) * sizeof(mfb200_board), cudaMemcpyHostToDevice, s),
          "H2D boards");
  launch_encode(S.boards, S.hist_off, B, fmt, S.masks, S.values, S.transforms, s);
  check(cudaGetLastError(), "encode launch");
}

const char *check_histories(const int32_t *offsets, int batch, int fmt, int shards, int per) {
  if (fmt != 1 && fmt != 2 && fmt != 3 && fmt != 4 && fmt != 5 && fmt != 132 && fmt != 133)
    return "unknown input format";
  for (int b = 0; b < batch; ++b)
    if (offsets[b + 1] < offsets[b]) return "history_offsets must be non-decreasing";
  for (int i = 0; i < shards; ++i) {
    const int lo = i * per, hi = std::min(batch, lo + per);
    if (lo < hi && offsets[hi] - offsets[lo] > int64_t(per) * kHistoryCapacity)
      return "more than 128 history records per position on average";
  }
  return nullptr;
}
}  // namespace

extern "C" int mfb200_encode_history(mfb200_handle *h, const mfb200_board *boards,
                                     const int32_t *history_offsets, int batch, int input_format,
                                     uint64_t *masks, float *values, int32_t *transforms) {
  if (!h) return fail(nullptr, "mfb200_encode_history: null handle");
  std::lock_guard<std::mutex> lock(h->mu);
  if (batch <= 0) return 0;
  if (batch > h->cfg.max_batch / static_cast<int>(h->shards.size()))
    return fail(h, "mfb200_encode_history: batch exceeds one device's share of max_batch");
  if (!history_offsets || (!boards && history_offsets[batch] != history_offsets[0]))
    return fail(h, "mfb200_encode_history: null input");
  if (const char *e = check_histories(history_offsets, batch, input_format, 1, batch))
    return fail(h, std::string("mfb200_encode_history: ") + e);
  try {
    Shard &S = *h->shards[0];
    check(cudaSetDevice(S.device), "cudaSetDevice");
    cudaStream_t s = S.stream;
    encode_shard(S, boards, history_offsets, batch, input_format, s);
    if (masks) check(cudaMemcpyAsync(masks, S.masks, size_t(batch) * kPlanes * 8, cudaMemcpyDeviceToHost, s), "D2H");
    if (values) check(cudaMemcpyAsync(values, S.values, size_t(batch) * kPlanes * 4, cudaMemcpyDeviceToHost, s), "D2H");
    if (transforms) check(cudaMemcpyAsync(transforms, S.transforms, size_t(batch) * 4, cudaMemcpyDeviceToHost, s), "D2H");
    check(cudaStreamSynchronize(s), "encode");
  } catch (const std::exception &e) {
    return fail(h, std::string("mfb200_encode_history: ") + e.what());
  }
  return 0;
}

extern "C" int mfb200_evaluate_history(mfb200_handle *h, const mfb200_board *boards,
                                       const int32_t *history_offsets, int batch,
                                       int input_format, float *policy, float *wdl, float *mlh,
                                       int32_t *transforms, mfb200_timing *timing) {
  if (!h) return fail(nullptr, "mfb200_evaluate_history: null handle");
  std::lock_guard<std::mutex> lock(h->mu);
  if (batch <= 0) return 0;
  if (batch > h->cfg.max_batch)
    return fail(h, "mfb200_evaluate_history: batch " + std::to_string(batch) + " exceeds max_batch " +
                       std::to_string(h->cfg.max_batch));
  if (!history_offsets || (!boards && history_offsets[batch] != history_offsets[0]))
    return fail(h, "mfb200_evaluate_history: null input");
  const int nd = static_cast<int>(h->shards.size());
  const int per = (batch + nd - 1) / nd;
  if (const char *e = check_histories(history_offsets, batch, input_format, nd, per))
    return fail(h, std::string("mfb200_evaluate_history: ") + e);
  std::vector<std::array<float, 4>> ms(nd, {0, 0, 0, 0});
  std::vector<std::string> errs(nd);
  auto work = [&](int i) {
    const int lo = i * per, hi = std::min(batch, lo + per);
    if (lo >= hi) return;
    Shard &S = *h->shards[i];
    const int B = hi - lo;
    try {
      check(cudaSetDevice(S.device), "cudaSetDevice");
      cudaStream_t s = S.stream;
      float *m = ms[i].data();
      check(cudaEventRecord(S.ev[0], s), "event");
      encode_shard(S, boards + (history_offsets[lo] - history_offsets[0]), history_offsets + lo, B,
                   input_format, s);
      check(cudaEventRecord(S.ev[1], s), "event");
      forward(h, S, B, s);
      check(cudaEventRecord(S.ev[2], s), "event");
      if (policy)
        check(cudaMemcpyAsync(policy + size_t(lo) * kPolicy, S.policy, size_t(B) * kPolicy * 4,
                              cudaMemcpyDeviceToHost, s), "D2H policy");
      if (wdl) check(cudaMemcpyAsync(wdl + size_t(lo) * 3, S.wdl, size_t(B) * 12, cudaMemcpyDeviceToHost, s), "D2H wdl");
      if (mlh) check(cudaMemcpyAsync(mlh + lo, S.mlh, size_t(B) * 4, cudaMemcpyDeviceToHost, s), "D2H mlh");
      if (transforms)
        check(cudaMemcpyAsync(transforms + lo, S.transforms, size_t(B) * 4, cudaMemcpyDeviceToHost, s), "D2H");
      check(cudaEventRecord(S.ev[3], s), "event");
      check(cudaStreamSynchronize(s), "forward");
      check_status(S);
      cudaEventElapsedTime(&m[0], S.ev[0], S.ev[1]);
      cudaEventElapsedTime(&m[1], S.ev[1], S.ev[2]);
      cudaEventElapsedTime(&m[2], S.ev[2], S.ev[3]);
      cudaEventElapsedTime(&m[3], S.ev[0], S.ev[3]);
    } catch (const std::exception &e) {
      errs[i] = e.what();
    }
  };
  if (nd == 1) {
    work(0);
  } else {
    std::vector<std::thread> th;
    for (int i = 0; i < nd; ++i) th.emplace_back(work, i);
    for (auto &t : th) t.join();
  }
  for (auto &e : errs)
    if (!e.empty()) return fail(h, "mfb200_evaluate_history: " + e);
  if (timing) {
    *timing = mfb200_timing{0, 0, 0, 0};
    for (auto &m : ms) {
      timing->h2d_ms = std::max(timing->h2d_ms, m[0]);
      timing->forward_ms = std::max(timing->forward_ms, m[1]);
      timing->d2h_ms = std::max(timing->d2h_ms, m[2]);
      timing->total_ms = std::max(timing->total_ms, m[3]);
    }
  }
  return 0;
}

extern "C" int mfb200_policy_index_table(int16_t *out) {
  if (!out) return 1;
  const std::vector<int16_t> t = build_move_index();
  // TransformSquare (src/nn/policy_map.cpp:303-312): rank reversed for
  // mirror / transpose, file reversed for flip / transpose
  auto sq = [](int s, int tr) {
    if (tr & 6) s ^= 56;
    if (tr & 5) s ^= 7;
    return s;
  };
  for (int tr = 0; tr < 8; ++tr)
    for (int k = 0; k < 5; ++k)
      for (int from = 0; from < 64; ++from)
        for (int to = 0; to < 64; ++to)
          out[((tr * 5 + k) * 64 + from) * 64 + to] = t[k * 4096 + sq(from, tr) * 64 + sq(to, tr)];
  return 0;
}

namespace {
// Blocks until the submission in `slot` has completed on every device and
// checks the devices' status words; the slot is free afterwards.
// Any error is recorded for the ticket (mfb200_wait returns it, also after
// the slot has been reused) and returned as a message, empty if none.
std::string finish_ticket(mfb200_handle *h, int slot) {
  const uint64_t t = h->pending[slot];
  if (!t) return {};
  h->pending[slot] = 0;
  std::string err;
  for (auto &S : h->shards) {
    try {
      check(cudaSetDevice(S->device), "cudaSetDevice");
      check(cudaEventSynchronize(S->done[slot]), "submission");
      unsigned st = 0;
      check(cudaMemcpy(&st, S->slots[slot].status, 4, cudaMemcpyDeviceToHost), "status read");
      if (st) throw Fail("device wait timed out in a GEMM (code " + std::to_string(st) + ")");
    } catch (const std::exception &e) {
      if (err.empty()) err = e.what();
    }
  }
  if (!err.empty()) {
    h->ticket_errors[t] = err;
    while (h->ticket_errors.size() > 64) h->ticket_errors.erase(h->ticket_errors.begin());
  }
  return err;
}

// mfb200_evaluate_leaves, synchronous (ticket == nullptr) or enqueued into
// ticket slot `slot` (returns at once; the caller's buffers must stay valid
// until the ticket is waited for).
int leaves_impl(mfb200_handle *h, const mfb200_board *boards, const int32_t *history_offsets,
                int batch, int input_format, const uint16_t *moves, const int32_t *move_offsets,
                float softmax_temp, float *priors, float *wdl, float *mlh, mfb200_timing *timing,
                uint64_t *ticket, const char *fn) {
  if (batch <= 0) return 0;
  if (batch > h->cfg.max_batch)
    return fail(h, std::string(fn) + ": batch " + std::to_string(batch) + " exceeds max_batch " +
                       std::to_string(h->cfg.max_batch));
  if (!history_offsets || !move_offsets ||
      (!boards && history_offsets[batch] != history_offsets[0]) ||
      (!moves && move_offsets[batch] != move_offsets[0]))
    return fail(h, std::string(fn) + ": null input");
  if (!(softmax_temp > 0.0f)) return fail(h, std::string(fn) + ": softmax_temp must be positive");
  const int nd = static_cast<int>(h->shards.size());
  const int per = (batch + nd - 1) / nd;
  if (const char *e = check_histories(history_offsets, batch, input_format, nd, per))
    return fail(h, std::string(fn) + ": " + e);
  for (int b = 0; b < batch; ++b)
    if (move_offsets[b + 1] < move_offsets[b])
      return fail(h, std::string(fn) + ": move_offsets must be non-decreasing");
  for (int i = 0; i < nd; ++i) {
    const int lo = i * per, hi = std::min(batch, lo + per);
    if (lo < hi && move_offsets[hi] - move_offsets[lo] > int64_t(per) * kMoveCapacity)
      return fail(h, std::string(fn) + ": more than 256 legal moves per position on average");
  }
  int slot = -1;
  if (ticket) {
    const uint64_t t = h->next_ticket++;
    slot = static_cast<int>(t % mfb200_handle::kTickets);
    finish_ticket(h, slot);  // at most kTickets in flight (an error stays with its ticket)
    h->pending[slot] = t;
    *ticket = t;
  }
  std::vector<std::array<float, 4>> ms(nd, {0, 0, 0, 0});
  std::vector<std::string> errs(nd);
  auto work = [&](int i) {
    const int lo = i * per, hi = std::min(batch, lo + per);
    Shard &S = *h->shards[i];
    const int B = hi - lo;
    try {
      check(cudaSetDevice(S.device), "cudaSetDevice");
      cudaStream_t s = S.stream;
      if (slot >= 0) {
        // asynchronous: copy in / compute / copy out on three streams
        Shard::SlotBufs &sb = S.slots[slot];
        if (B > 0) {
          const int32_t mbase = move_offsets[lo] - move_offsets[0];
          const int32_t nmoves = move_offsets[hi] - move_offsets[lo];
          const int32_t hbase = history_offsets[lo] - history_offsets[0];
          const int32_t nb = history_offsets[hi] - history_offsets[lo];
          check(cudaMemcpyAsync(sb.hist_off, history_offsets + lo, size_t(B + 1) * 4,
                                cudaMemcpyHostToDevice, S.copy_in), "H2D offsets");
          if (nb > 0)
            check(cudaMemcpyAsync(sb.boards, boards + hbase, size_t(nb) * sizeof(mfb200_board),
                                  cudaMemcpyHostToDevice, S.copy_in), "H2D boards");
          check(cudaMemcpyAsync(sb.move_off, move_offsets + lo, size_t(B + 1) * 4,
                                cudaMemcpyHostToDevice, S.copy_in), "H2D move offsets");
          if (nmoves > 0)
            check(cudaMemcpyAsync(sb.moves, moves + mbase, size_t(nmoves) * 2,
                                  cudaMemcpyHostToDevice, S.copy_in), "H2D moves");
          check(cudaEventRecord(S.in_done[slot], S.copy_in), "event");
          check(cudaStreamWaitEvent(s, S.in_done[slot], 0), "wait inputs");
          launch_encode(sb.boards, sb.hist_off, B, input_format, S.masks, S.values, sb.transforms, s);
          check(cudaGetLastError(), "encode launch");
          forward(h, S, B, s);
          launch_leaf_priors(S.policy, B, sb.move_off, sb.moves, S.move_table, sb.boards, sb.hist_off,
                             sb.transforms, softmax_temp, sb.priors, s);
          check(cudaGetLastError(), "priors launch");
          check(cudaMemcpyAsync(sb.wdl, S.wdl, size_t(B) * 12, cudaMemcpyDeviceToDevice, s), "wdl");
          check(cudaMemcpyAsync(sb.mlh, S.mlh, size_t(B) * 4, cudaMemcpyDeviceToDevice, s), "mlh");
          // the status word now holds this submission's errors only
          check(cudaMemcpyAsync(sb.status, S.status, 4, cudaMemcpyDeviceToDevice, s), "status");
          check(cudaMemsetAsync(S.status, 0, 4, s), "status clear");
          check(cudaEventRecord(S.comp_done[slot], s), "event");
          check(cudaStreamWaitEvent(S.copy_out, S.comp_done[slot], 0), "wait forward");
          if (priors && nmoves > 0)
            check(cudaMemcpyAsync(priors + mbase, sb.priors, size_t(nmoves) * 4,
                                  cudaMemcpyDeviceToHost, S.copy_out), "D2H priors");
          if (wdl)
            check(cudaMemcpyAsync(wdl + size_t(lo) * 3, sb.wdl, size_t(B) * 12,
                                  cudaMemcpyDeviceToHost, S.copy_out), "D2H wdl");
          if (mlh)
            check(cudaMemcpyAsync(mlh + lo, sb.mlh, size_t(B) * 4, cudaMemcpyDeviceToHost,
                                  S.copy_out), "D2H mlh");
        } else {
          check(cudaMemsetAsync(sb.status, 0, 4, S.copy_out), "status clear");
        }
        check(cudaEventRecord(S.done[slot], S.copy_out), "event");
        return;
      }
      if (B > 0) {
        const int32_t mbase = move_offsets[lo] - move_offsets[0];
        const int32_t nmoves = move_offsets[hi] - move_offsets[lo];
        check(cudaEventRecord(S.ev[0], s), "event");
        encode_shard(S, boards + (history_offsets[lo] - history_offsets[0]), history_offsets + lo, B,
                     input_format, s);
        check(cudaMemcpyAsync(S.move_off, move_offsets + lo, size_t(B + 1) * 4, cudaMemcpyHostToDevice, s),
              "H2D move offsets");
        if (nmoves > 0)
          check(cudaMemcpyAsync(S.moves, moves + mbase, size_t(nmoves) * 2, cudaMemcpyHostToDevice, s),
                "H2D moves");
        check(cudaEventRecord(S.ev[1], s), "event");
        forward(h, S, B, s);
        launch_leaf_priors(S.policy, B, S.move_off, S.moves, S.move_table, S.boards, S.hist_off,
                           S.transforms, softmax_temp, S.priors, s);
        check(cudaGetLastError(), "priors launch");
        check(cudaEventRecord(S.ev[2], s), "event");
        if (priors && nmoves > 0)
          check(cudaMemcpyAsync(priors + mbase, S.priors, size_t(nmoves) * 4, cudaMemcpyDeviceToHost, s),
                "D2H priors");
        if (wdl) check(cudaMemcpyAsync(wdl + size_t(lo) * 3, S.wdl, size_t(B) * 12, cudaMemcpyDeviceToHost, s), "D2H wdl");
        if (mlh) check(cudaMemcpyAsync(mlh + lo, S.mlh, size_t(B) * 4, cudaMemcpyDeviceToHost, s), "D2H mlh");
        check(cudaEventRecord(S.ev[3], s), "event");
      }
      if (B <= 0) return;
      check(cudaStreamSynchronize(s), "forward");
      check_status(S);
      float *m = ms[i].data();
      cudaEventElapsedTime(&m[0], S.ev[0], S.ev[1]);
      cudaEventElapsedTime(&m[1], S.ev[1], S.ev[2]);
      cudaEventElapsedTime(&m[2], S.ev[2], S.ev[3]);
      cudaEventElapsedTime(&m[3], S.ev[0], S.ev[3]);
    } catch (const std::exception &e) {
      errs[i] = e.what();
    }
  };
  if (nd == 1) {
    work(0);
  } else {
    std::vector<std::thread> th;
    for (int i = 0; i < nd; ++i) th.emplace_back(work, i);
    for (auto &t : th) t.join();
  }
  for (auto &e : errs)
    if (!e.empty()) return fail(h, std::string(fn) + ": " + e);
  if (timing) {
    *timing = mfb200_timing{0, 0, 0, 0};
    for (auto &m : ms) {
      timing->h2d_ms = std::max(timing->h2d_ms, m[0]);
      timing->forward_ms = std::max(timing->forward_ms, m[1]);
      timing->d2h_ms = std::max(timing->d2h_ms, m[2]);
      timing->total_ms = std::max(timing->total_ms, m[3]);
    }
  }
  return 0;
}
}  // namespace

extern "C" int mfb200_evaluate_leaves(mfb200_handle *h, const mfb200_board *boards,
                                      const int32_t *history_offsets, int batch, int input_format,
                                      const uint16_t *moves, const int32_t *move_offsets,
                                      float softmax_temp, float *priors, float *wdl, float *mlh,
                                      mfb200_timing *timing) {
  if (!h) return fail(nullptr, "mfb200_evaluate_leaves: null handle");
  std::lock_guard<std::mutex> lock(h->mu);
  return leaves_impl(h, boards, history_offsets, batch, input_format, moves, move_offsets,
                     softmax_temp, priors, wdl, mlh, timing, nullptr, "mfb200_evaluate_leaves");
}

extern "C" int mfb200_submit_leaves(mfb200_handle *h, const mfb200_board *boards,
                                    const int32_t *history_offsets, int batch, int input_format,
                                    const uint16_t *moves, const int32_t *move_offsets,
                                    float softmax_temp, float *priors, float *wdl, float *mlh,
                                    uint64_t *ticket) {
  if (!h) return fail(nullptr, "mfb200_submit_leaves: null handle");
  if (!ticket) return fail(h, "mfb200_submit_leaves: null ticket");
  std::lock_guard<std::mutex> lock(h->mu);
  *ticket = 0;
  return leaves_impl(h, boards, history_offsets, batch, input_format, moves, move_offsets,
                     softmax_temp, priors, wdl, mlh, nullptr, ticket, "mfb200_submit_leaves");
}

extern "C" int mfb200_wait(mfb200_handle *h, uint64_t ticket) {
  if (!h) return fail(nullptr, "mfb200_wait: null handle");
  std::lock_guard<std::mutex> lock(h->mu);
  if (ticket == 0 || ticket >= h->next_ticket) return fail(h, "mfb200_wait: unknown ticket");
  const int slot = static_cast<int>(ticket % mfb200_handle::kTickets);
  if (h->pending[slot] == ticket) finish_ticket(h, slot);
  // (a ticket whose slot was reused was finished then; its error, if any, is kept)
  auto it = h->ticket_errors.find(ticket);
  if (it != h->ticket_errors.end()) return fail(h, "mfb200_wait: " + it->second);
  return 0;
}

extern "C" int mfb200_evaluate_priors(mfb200_handle *h, const uint64_t *masks,
                                      const float *values, int batch,
                                      const int32_t *move_offsets, const int16_t *move_index,
                                      float softmax_temp, float *priors, float *wdl, float *mlh,
                                      mfb200_timing *timing) {
  if (!h) return fail(nullptr, "mfb200_evaluate_priors: null handle");
  std::lock_guard<std::mutex> lock(h->mu);
  if (batch <= 0) return 0;
  if (batch > h->cfg.max_batch)
    return fail(h, "mfb200_evaluate_priors: batch " + std::to_string(batch) + " exceeds max_batch " +
                       std::to_string(h->cfg.max_batch));
  if (!masks || !values || !move_offsets || (!move_index && move_offsets[batch] != move_offsets[0]))
    return fail(h, "mfb200_evaluate_priors: null input");
  if (!(softmax_temp > 0.0f)) return fail(h, "mfb200_evaluate_priors: softmax_temp must be positive");
  for (int b = 0; b < batch; ++b)
    if (move_offsets[b + 1] < move_offsets[b])
      return fail(h, "mfb200_evaluate_priors: move_offsets must be non-decreasing");
  const int nd = static_cast<int>(h->shards.size());
  const int per = (batch + nd - 1) / nd;
  for (int i = 0; i < nd; ++i) {
    const int lo = i * per, hi = std::min(batch, lo + per);
    if (lo < hi && move_offsets[hi] - move_offsets[lo] > int64_t(per) * kMoveCapacity)
      return fail(h, "mfb200_evaluate_priors: more than " + std::to_string(kMoveCapacity) +
                         " legal moves per position on average");
  }
  std::vector<std::array<float, 4>> ms(nd, {0, 0, 0, 0});
  std::vector<std::string> errs(nd);
  auto work = [&](int i) {
    const int lo = i * per, hi = std::min(batch, lo + per);
    if (lo >= hi) return;
    const int32_t base = move_offsets[lo] - move_offsets[0];
    try {
      eval_shard_priors(h, *h->shards[i], masks + size_t(lo) * kPlanes, values + size_t(lo) * kPlanes,
                        hi - lo, move_offsets + lo, move_index ? move_index + base : nullptr,
                        softmax_temp, priors ? priors + base : nullptr,
                        wdl ? wdl + size_t(lo) * 3 : nullptr, mlh ? mlh + lo : nullptr, ms[i].data());
    } catch (const std::exception &e) {
      errs[i] = e.what();
    }
  };
  if (nd == 1) {
    work(0);
  } else {
    std::vector<std::thread> th;
    for (int i = 0; i < nd; ++i) th.emplace_back(work, i);
    for (auto &t : th) t.join();
  }
  for (auto &e : errs)
    if (!e.empty()) return fail(h, "mfb200_evaluate_priors: " + e);
  if (timing) {
    *timing = mfb200_timing{0, 0, 0, 0};
    for (auto &m : ms) {
      timing->h2d_ms = std::max(timing->h2d_ms, m[0]);
      timing->forward_ms = std::max(timing->forward_ms, m[1]);
      timing->d2h_ms = std::max(timing->d2h_ms, m[2]);
      timing->total_ms = std::max(timing->total_ms, m[3]);
    }
  }
  return 0;
}

extern "C" int mfb200_evaluate(mfb200_handle *h, const uint64_t *masks, const float *values,
                               int batch, float *policy, float *wdl, float *mlh,
                               mfb200_timing *timing) {
  if (!h) return fail(nullptr, "mfb200_evaluate: null handle");
  std::lock_guard<std::mutex> lock(h->mu);
  if (batch <= 0) return 0;
  if (batch > h->cfg.max_batch)
    return fail(h, "mfb200_evaluate: batch " + std::to_string(batch) + " exceeds max_batch " +
                       std::to_string(h->cfg.max_batch));
  if (!masks || !values) return fail(h, "mfb200_evaluate: null input");
  const int nd = static_cast<int>(h->shards.size());
  const int per = (batch + nd - 1) / nd;
  std::vector<std::array<float, 4>> ms(nd, {0, 0, 0, 0});
  std::vector<std::string> errs(nd);
  auto work = [&](int i) {
    const int lo = i * per, hi = std::min(batch, lo + per);
    if (lo >= hi) return;
    try {
      eval_shard(h, *h->shards[i], masks + size_t(lo) * kPlanes, values + size_t(lo) * kPlanes,
                 hi - lo, policy ? policy + size_t(lo) * kPolicy : nullptr,
                 wdl ? wdl + size_t(lo) * 3 : nullptr, mlh ? mlh + lo : nullptr, ms[i].data());
    } catch (const std::exception &e) {
      errs[i] = e.what();
    }
  };
  if (nd == 1) {
    work(0);
  } else {
    std::vector<std::thread> th;
    for (int i = 0; i < nd; ++i) th.emplace_back(work, i);
    for (auto &t : th) t.join();
  }
  for (auto &e : errs)
    if (!e.empty()) return fail(h, "mfb200_evaluate: " + e);
  if (timing) {
    *timing = mfb200_timing{0, 0, 0, 0};
    for (auto &m : ms) {
      timing->h2d_ms = std::max(timing->h2d_ms, m[0]);
      timing->forward_ms = std::max(timing->forward_ms, m[1]);
      timing->d2h_ms = std::max(timing->d2h_ms, m[2]);
      timing->total_ms = std::max(timing->total_ms, m[3]);
    }
  }
  return 0;
}

extern "C" int mfb200_evaluate_device(mfb200_handle *h, const uint64_t *d_masks,
                                      const float *d_values, int batch, float *d_policy,
                                      float *d_wdl, float *d_mlh, void *stream) {
  if (!h) return fail(nullptr, "mfb200_evaluate_device: null handle");
  std::lock_guard<std::mutex> lock(h->mu);
  if (batch <= 0) return 0;
  Shard &S = *h->shards[0];
  if (batch > h->cfg.max_batch / static_cast<int>(h->shards.size()) + 1 && h->shards.size() > 1)
    return fail(h, "mfb200_evaluate_device: batch exceeds one device's share of max_batch");
  if (batch > h->cfg.max_batch) return fail(h, "mfb200_evaluate_device: batch exceeds max_batch");
  try {
    check(cudaSetDevice(S.device), "cudaSetDevice");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : S.stream;
    if (d_masks != S.masks)
      check(cudaMemcpyAsync(S.masks, d_masks, size_t(batch) * kPlanes * 8, cudaMemcpyDeviceToDevice, s), "masks");
    if (d_values != S.values)
      check(cudaMemcpyAsync(S.values, d_values, size_t(batch) * kPlanes * 4, cudaMemcpyDeviceToDevice, s), "values");
    if (stream && !S.plans.count(batch * 4 + (eight_bit(h->cfg) ? 1 : 0))) {
      // build (and capture) on the handle's own stream first
      check(cudaStreamSynchronize(s), "sync");
      get_plan(h, S, batch);
    }
    forward(h, S, batch, s);
    if (d_policy)
      check(cudaMemcpyAsync(d_policy, S.policy, size_t(batch) * kPolicy * 4, cudaMemcpyDeviceToDevice, s), "policy");
    if (d_wdl) check(cudaMemcpyAsync(d_wdl, S.wdl, size_t(batch) * 12, cudaMemcpyDeviceToDevice, s), "wdl");
    if (d_mlh) check(cudaMemcpyAsync(d_mlh, S.mlh, size_t(batch) * 4, cudaMemcpyDeviceToDevice, s), "mlh");
  } catch (const std::exception &e) {
    return fail(h, std::string("mfb200_evaluate_device: ") + e.what());
  }
  return 0;
}

extern "C" int mfb200_calibrate(mfb200_handle *h, const uint64_t *masks, const float *values,
                                int count) {
  if (!h) return fail(nullptr, "mfb200_calibrate: null handle");
  std::lock_guard<std::mutex> lock(h->mu);
  if (!eight_bit(h->cfg))
    return fail(h, "mfb200_calibrate: only FP8 / INT8 handles have activation scales");
  if (!masks || !values || count <= 0) return fail(h, "mfb200_calibrate: no calibration positions");
  try {
    Shard &S0 = *h->shards[0];
    check(cudaSetDevice(S0.device), "cudaSetDevice");
    const int nscale = 2 + 4 * h->desc.layers;
    check(cudaMemsetAsync(S0.absmax, 0, nscale * 4, S0.stream), "absmax clear");
    const int chunk = h->cfg.max_batch / static_cast<int>(h->shards.size());
    for (int lo = 0; lo < count; lo += chunk) {
      const int b = std::min(chunk, count - lo);
      check(cudaMemcpyAsync(S0.masks, masks + size_t(lo) * kPlanes, size_t(b) * kPlanes * 8,
                            cudaMemcpyHostToDevice, S0.stream), "H2D masks");
      check(cudaMemcpyAsync(S0.values, values + size_t(lo) * kPlanes, size_t(b) * kPlanes * 4,
                            cudaMemcpyHostToDevice, S0.stream), "H2D values");
      run_steps(get_plan(h, S0, b, kPlanCalibrate), S0.stream);
    }
    launch_absmax_to_scale(S0.absmax, nscale, S0.scales, S0.stream,
                           h->cfg.precision == MFB200_PRECISION_INT8 ? 127.0f : 448.0f);
    check(cudaStreamSynchronize(S0.stream), "calibration");
    check_status(S0);
    std::vector<float> sc(nscale);
    check(cudaMemcpy(sc.data(), S0.scales, nscale * 4, cudaMemcpyDeviceToHost), "scales");
    for (size_t i = 1; i < h->shards.size(); ++i) {
      check(cudaSetDevice(h->shards[i]->device), "cudaSetDevice");
      check(cudaMemcpy(h->shards[i]->scales, sc.data(), nscale * 4, cudaMemcpyHostToDevice), "scales");
    }
    h->calibrated = true;
  } catch (const std::exception &e) {
    return fail(h, std::string("mfb200_calibrate: ") + e.what());
  }
  return 0;
}

extern "C" int mfb200_capabilities(mfb200_handle *h, mfb200_caps *caps) {
  if (!h || !caps) return fail(h, "mfb200_capabilities: null argument");
  std::memset(caps, 0, sizeof(*caps));
  caps->max_batch = h->cfg.max_batch;
  caps->precision = h->cfg.precision;
  caps->num_devices = static_cast<int>(h->shards.size());
  caps->device = h->cfg.device;
  caps->has_wdl = 1;
  caps->has_moves_left = 1;
  caps->weight_bytes = static_cast<int64_t>(h->weight_bytes);
  caps->workspace_bytes = static_cast<int64_t>(h->ws_bytes);
  std::snprintf(caps->device_name, sizeof(caps->device_name), "%s", h->device_name.c_str());
  return 0;
}

extern "C" int mfb200_profile(mfb200_handle *h, int batch, int iters, float *stage_ms,
                              double *stage_flops, char *names, size_t names_len, int max_stages) {
  if (!h) return -1;
  std::lock_guard<std::mutex> lock(h->mu);
  try {
    Shard &S = *h->shards[0];
    check(cudaSetDevice(S.device), "cudaSetDevice");
    if (batch <= 0 || batch > h->cfg.max_batch / static_cast<int>(h->shards.size()))
      throw Fail("profile batch out of range");
    Shard::Plan &P = get_plan(h, S, batch);
    const int n = static_cast<int>(P.steps.size());
    std::vector<cudaEvent_t> ev(n + 1);
    for (auto &e : ev) check(cudaEventCreate(&e), "event");
    std::vector<double> acc(n, 0.0);
    for (int it = 0; it < std::max(1, iters); ++it) {
      check(cudaEventRecord(ev[0], S.stream), "event");
      for (int i = 0; i < n; ++i) {
        auto &st = P.steps[i];
        if (st.is_gemm)
          check(launch_gemm(st.g, S.stream), st.name.c_str());
        else
          st.fn(S.stream);
        check(cudaEventRecord(ev[i + 1], S.stream), "event");
      }
      check(cudaStreamSynchronize(S.stream), "profile");
      for (int i = 0; i < n; ++i) {
        float ms = 0;
        cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
        acc[i] += ms;
      }
    }
    check_status(S);
    for (auto &e : ev) cudaEventDestroy(e);
    std::string all;
    for (int i = 0; i < n && i < max_stages; ++i) {
      if (stage_ms) stage_ms[i] = static_cast<float>(acc[i] / std::max(1, iters));
      if (stage_flops) stage_flops[i] = P.steps[i].flops;
      all += P.steps[i].name + "\n";
    }
    if (names && names_len) {
      std::snprintf(names, names_len, "%s", all.c_str());
    }
    return n;
  } catch (const std::exception &e) {
    fail(h, std::string("mfb200_profile: ") + e.what());
    return -2;
  }
}

extern "C" const char *mfb200_last_error(mfb200_handle *h) {
  if (!t_last_error.empty()) return t_last_error.c_str();
  return h ? h->last_error.c_str() : "";
}

extern "C" void mfb200_destroy(mfb200_handle *h) {
  if (!h) return;
  for (auto &S : h->shards) {
    cudaSetDevice(S->device);
    cudaStreamSynchronize(S->stream);
    for (auto &kv : S->plans)
      if (kv.second->graph) cudaGraphExecDestroy(kv.second->graph);
    for (auto &e : S->ev) cudaEventDestroy(e);
    for (auto &e : S->done) cudaEventDestroy(e);
    if (S->copy_in) {
      cudaStreamSynchronize(S->copy_in);
      cudaStreamSynchronize(S->copy_out);
      for (auto &e : S->in_done) cudaEventDestroy(e);
      for (auto &e : S->comp_done) cudaEventDestroy(e);
      cudaStreamDestroy(S->copy_in);
      cudaStreamDestroy(S->copy_out);
    }
    if (S->slot_mem) cudaFree(S->slot_mem);
    if (S->arena) cudaFree(S->arena);
    if (S->ws) cudaFree(S->ws);
    cudaStreamDestroy(S->stream);
  }
  delete h;
}
