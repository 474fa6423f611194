// b200_network.cpp -- see b200_network.h.
#include "b200_network.h"

#include <algorithm>
#include <cstring>
#include <limits>
#include <sstream>
#include <stdexcept>

#include "../../include/mfb200.h"
#include "nn/input_plane_packing.h"
#include "nn/network_format.h"
#include "nn/weights.h"

namespace MetalFish {
namespace NN {
namespace B200 {
namespace {

int ActivationCode(const std::string &name) {
  if (name == "relu") return MFB200_ACT_RELU;
  if (name == "relu_2") return MFB200_ACT_RELU2;
  if (name == "tanh") return MFB200_ACT_TANH;
  if (name == "sigmoid") return MFB200_ACT_SIGMOID;
  if (name == "swish") return MFB200_ACT_SWISH;
  if (name == "mish") return MFB200_ACT_MISH;
  if (name == "selu") return MFB200_ACT_SELU;
  throw std::runtime_error("B200 backend: unsupported activation " + name);
}

void Require(bool ok, const std::string &what) {
  if (!ok) throw std::runtime_error("B200 backend does not support this network: " + what);
}

// The shape of the attention-body network, inferred from tensor sizes.
mfb200_net_desc DescribeNet(const WeightsFile &file, const MultiHeadWeights &w,
                            const MultiHeadWeights::PolicyHead &pol,
                            const MultiHeadWeights::ValueHead &val) {
  const NetworkFormatDescriptor f = DescribeNetworkFormat(file);
  Require(f.attention_body, "not an attention-body network");
  Require(f.attention_policy, "policy head is not attention policy");
  Require(f.wdl && f.moves_left, "needs WDL value and moves-left heads");
  Require(f.input_embedding == INPUT_EMBEDDING_PE_DENSE, "input embedding is not PE_DENSE");
  Require(!w.encoder.empty() && w.encoder[0].mha.has_smolgen && w.has_smolgen,
          "encoder without smolgen");
  Require(pol.pol_encoder.empty(), "policy-head encoder layers");
  mfb200_net_desc d{};
  d.embedding = static_cast<int32_t>(w.ip_emb_b.size());
  d.layers = static_cast<int32_t>(w.encoder.size());
  d.heads = w.encoder_head_count;
  d.dff = static_cast<int32_t>(w.encoder[0].ffn.dense1_b.size());
  d.emb_dff = static_cast<int32_t>(w.ip_emb_ffn.dense1_b.size());
  d.pe = static_cast<int32_t>(w.ip_emb_preproc_b.size() / 64);
  d.smolgen_compress = static_cast<int32_t>(w.encoder[0].mha.smolgen.compress.size() / d.embedding);
  d.smolgen_hidden = static_cast<int32_t>(w.encoder[0].mha.smolgen.dense1_b.size());
  d.smolgen_gen = static_cast<int32_t>(w.smolgen_w.size() / 4096);
  d.policy_d = static_cast<int32_t>(pol.ip_pol_b.size());
  d.value_emb = static_cast<int32_t>(val.ip_val_b.size());
  d.value_hidden = static_cast<int32_t>(val.ip1_val_b.size());
  d.mlh_emb = static_cast<int32_t>(w.ip_mov_b.size());
  d.mlh_hidden = static_cast<int32_t>(w.ip1_mov_b.size());
  d.act_default = ActivationCode(f.activations.default_activation);
  d.act_smolgen = ActivationCode(f.activations.smolgen_activation);
  d.act_ffn = ActivationCode(f.activations.ffn_activation);
  return d;
}

// Concatenate every tensor in the library's slot order (the order of
// metalfish_b200/layout.py: globals, then each encoder layer).
std::vector<float> WeightBlob(const MultiHeadWeights &w, const MultiHeadWeights::PolicyHead &pol,
                              const MultiHeadWeights::ValueHead &val) {
  std::vector<float> blob;
  using List = std::initializer_list<const std::vector<float> *>;
  auto put = [&](const std::vector<float> &v) { blob.insert(blob.end(), v.begin(), v.end()); };
  for (const auto *v : List{&w.ip_emb_preproc_w, &w.ip_emb_preproc_b, &w.ip_emb_w, &w.ip_emb_b,
                        &w.ip_emb_ln_gammas, &w.ip_emb_ln_betas, &w.ip_mult_gate, &w.ip_add_gate,
                        &w.ip_emb_ffn.dense1_w, &w.ip_emb_ffn.dense1_b, &w.ip_emb_ffn.dense2_w,
                        &w.ip_emb_ffn.dense2_b, &w.ip_emb_ffn_ln_gammas, &w.ip_emb_ffn_ln_betas,
                        &w.smolgen_w})
    put(*v);
  for (const auto *v : List{&pol.ip_pol_w, &pol.ip_pol_b, &pol.ip2_pol_w, &pol.ip2_pol_b,
                        &pol.ip3_pol_w, &pol.ip3_pol_b, &pol.ip4_pol_w})
    put(*v);
  for (const auto *v : List{&val.ip_val_w, &val.ip_val_b, &val.ip1_val_w, &val.ip1_val_b,
                        &val.ip2_val_w, &val.ip2_val_b})
    put(*v);
  for (const auto *v : List{&w.ip_mov_w, &w.ip_mov_b, &w.ip1_mov_w, &w.ip1_mov_b, &w.ip2_mov_w,
                        &w.ip2_mov_b})
    put(*v);
  for (const auto &e : w.encoder) {
    const auto &m = e.mha;
    const auto &s = m.smolgen;
    for (const auto *v : List{&m.q_w, &m.q_b, &m.k_w, &m.k_b, &m.v_w, &m.v_b, &m.dense_w, &m.dense_b,
                          &s.compress, &s.dense1_w, &s.dense1_b, &s.ln1_gammas, &s.ln1_betas,
                          &s.dense2_w, &s.dense2_b, &s.ln2_gammas, &s.ln2_betas, &e.ln1_gammas,
                          &e.ln1_betas, &e.ffn.dense1_w, &e.ffn.dense1_b, &e.ffn.dense2_w,
                          &e.ffn.dense2_b, &e.ln2_gammas, &e.ln2_betas})
      put(*v);
  }
  return blob;
}

// One history entry as the GPU encoder reads it (include/mfb200.h).
mfb200_board ToBoard(const Position &p) {
  mfb200_board r{};
  const PieceType kinds[6] = {PAWN, KNIGHT, BISHOP, ROOK, QUEEN, KING};
  for (int c = 0; c < 2; ++c)
    for (int k = 0; k < 6; ++k) r.pieces[c][k] = p.pieces(c ? BLACK : WHITE, kinds[k]);
  r.rule50 = p.rule50_count();
  r.game_ply = p.game_ply();
  r.ep_square = p.ep_square() == SQ_NONE ? std::int8_t(-1) : std::int8_t(p.ep_square());
  r.castling = std::uint8_t((p.can_castle(WHITE_OO) ? 1 : 0) | (p.can_castle(WHITE_OOO) ? 2 : 0) |
                            (p.can_castle(BLACK_OO) ? 4 : 0) | (p.can_castle(BLACK_OOO) ? 8 : 0));
  r.black_to_move = p.side_to_move() == BLACK ? 1 : 0;
  r.repetition = p.is_repetition(std::numeric_limits<int>::max()) ? 1 : 0;
  return r;
}

// from | to << 6 | promotion << 12 (1 queen, 2 rook, 3 bishop, 4 knight).
std::uint16_t ToRawMove(Move m) {
  int kind = 0;
  if (m.type_of() == PROMOTION) {
    const PieceType pt = m.promotion_type();
    kind = pt == QUEEN ? 1 : pt == ROOK ? 2 : pt == BISHOP ? 3 : 4;
  }
  return std::uint16_t(int(m.from_sq()) | (int(m.to_sq()) << 6) | (kind << 12));
}

B200Options FromConfig(const BackendConfig &config) {
  B200Options o;
  o.device = config.cuda_device >= 0 ? config.cuda_device : 0;
  o.use_graphs = config.cuda_graph_execution;
  if (config.cuda_stable_execution_batch_size > 0)
    o.max_batch = config.cuda_stable_execution_batch_size;
  return o;
}

}  // namespace

B200Network::B200Network(const WeightsFile &weights, const BackendConfig &config)
    : B200Network(weights, FromConfig(config)) {}

B200Network::B200Network(const WeightsFile &weights, const B200Options &options)
    : options_(options) {
  const MultiHeadWeights w(weights.weights());
  const auto &pol = w.policy_heads.at(SelectPolicyHeadName(w));
  const auto &val = w.value_heads.at(SelectValueHeadName(w));
  const mfb200_net_desc desc = DescribeNet(weights, w, pol, val);
  const std::vector<float> blob = WeightBlob(w, pol, val);
  if (blob.size() * sizeof(float) != mfb200_weight_bytes(&desc))
    throw std::runtime_error("B200 backend: weight tensors do not match the inferred shape");
  mfb200_config cfg{};
  cfg.device = options.device;
  cfg.num_devices = options.num_devices;
  cfg.precision = MFB200_PRECISION_BF16;
  cfg.max_batch = options.max_batch;
  cfg.use_graphs = options.use_graphs ? 1 : 0;
  if (mfb200_create(&desc, blob.data(), blob.size() * sizeof(float), &cfg, &handle_) != 0)
    throw std::runtime_error(std::string("B200 backend unavailable: ") + mfb200_last_error(nullptr));
  std::ostringstream info;
  info << "B200 transformer backend (d=" << desc.embedding << " layers=" << desc.layers
       << " heads=" << desc.heads << " dff=" << desc.dff << ", "
       << GetBackendCapabilities().Summary() << ")";
  info_ = info.str();
}

B200Network::~B200Network() { mfb200_destroy(handle_); }

NetworkOutput B200Network::Evaluate(const InputPlanes &input) {
  return EvaluateBatch(std::vector<InputPlanes>{input}).front();
}

std::vector<NetworkOutput> B200Network::EvaluateBatch(const std::vector<InputPlanes> &inputs) {
  std::vector<NetworkOutput> out(inputs.size());
  if (inputs.empty()) return out;
  std::lock_guard<std::mutex> lock(mutex_);
  const int n = static_cast<int>(inputs.size());
  masks_.resize(size_t(n) * kPackedInputPlaneCount);
  values_.resize(size_t(n) * kPackedInputPlaneCount);
  for (int b = 0; b < n; ++b)
    for (int p = 0; p < kPackedInputPlaneCount; ++p)
      PackInputPlaneRaw(inputs[b][p].data(), p, masks_[size_t(b) * kPackedInputPlaneCount + p],
                        values_[size_t(b) * kPackedInputPlaneCount + p]);
  policy_.resize(size_t(n) * kPolicyOutputs);
  wdl_.resize(size_t(n) * 3);
  mlh_.resize(n);
  for (int lo = 0; lo < n; lo += options_.max_batch) {
    const int cnt = std::min(options_.max_batch, n - lo);
    if (mfb200_evaluate(handle_, masks_.data() + size_t(lo) * kPackedInputPlaneCount,
                        values_.data() + size_t(lo) * kPackedInputPlaneCount, cnt,
                        policy_.data() + size_t(lo) * kPolicyOutputs, wdl_.data() + size_t(lo) * 3,
                        mlh_.data() + lo, nullptr) != 0)
      throw std::runtime_error(std::string("B200 backend: ") + mfb200_last_error(handle_));
  }
  // NetworkOutput decoding as src/nn/network_output_decoder.cpp:49-75.
  for (int b = 0; b < n; ++b) {
    NetworkOutput &o = out[b];
    std::memcpy(o.policy.data(), policy_.data() + size_t(b) * kPolicyOutputs,
                sizeof(float) * kPolicyOutputs);
    o.has_wdl = true;
    o.wdl[0] = wdl_[3 * b];
    o.wdl[1] = wdl_[3 * b + 1];
    o.wdl[2] = wdl_[3 * b + 2];
    o.value = o.wdl[0] - o.wdl[2];
    o.has_moves_left = true;
    o.moves_left = mlh_[b];
  }
  return out;
}

std::vector<B200Network::LeafResult>
B200Network::EvaluatePriors(const std::vector<InputPlanes> &inputs,
                            const std::vector<std::vector<std::int16_t>> &move_indices,
                            float softmax_temp) {
  if (move_indices.size() != inputs.size())
    throw std::invalid_argument("legal move list count must match input count");
  std::vector<LeafResult> out(inputs.size());
  if (inputs.empty()) return out;
  std::lock_guard<std::mutex> lock(mutex_);
  const int n = static_cast<int>(inputs.size());
  masks_.resize(size_t(n) * kPackedInputPlaneCount);
  values_.resize(size_t(n) * kPackedInputPlaneCount);
  for (int b = 0; b < n; ++b)
    for (int p = 0; p < kPackedInputPlaneCount; ++p)
      PackInputPlaneRaw(inputs[b][p].data(), p, masks_[size_t(b) * kPackedInputPlaneCount + p],
                        values_[size_t(b) * kPackedInputPlaneCount + p]);
  move_offsets_.assign(1, 0);
  move_index_.clear();
  for (const auto &m : move_indices) {
    move_index_.insert(move_index_.end(), m.begin(), m.end());
    move_offsets_.push_back(static_cast<std::int32_t>(move_index_.size()));
  }
  priors_.resize(move_index_.size());
  wdl_.resize(size_t(n) * 3);
  mlh_.resize(n);
  for (int lo = 0; lo < n; lo += options_.max_batch) {
    const int cnt = std::min(options_.max_batch, n - lo);
    const std::int32_t base = move_offsets_[lo];
    if (mfb200_evaluate_priors(handle_, masks_.data() + size_t(lo) * kPackedInputPlaneCount,
                               values_.data() + size_t(lo) * kPackedInputPlaneCount, cnt,
                               move_offsets_.data() + lo, move_index_.data() + base, softmax_temp,
                               priors_.data() + base, wdl_.data() + size_t(lo) * 3,
                               mlh_.data() + lo, nullptr) != 0)
      throw std::runtime_error(std::string("B200 backend: ") + mfb200_last_error(handle_));
  }
  for (int b = 0; b < n; ++b) {
    LeafResult &r = out[b];
    r.priors.assign(priors_.begin() + move_offsets_[b], priors_.begin() + move_offsets_[b + 1]);
    r.wdl[0] = wdl_[3 * b];
    r.wdl[1] = wdl_[3 * b + 1];
    r.wdl[2] = wdl_[3 * b + 2];
    r.value = r.wdl[0] - r.wdl[2];
    r.moves_left = mlh_[b];
  }
  return out;
}

std::vector<B200Network::LeafResult>
B200Network::EvaluateLeaves(const std::vector<std::vector<const Position *>> &histories,
                            const std::vector<std::vector<Move>> &legal_moves, float softmax_temp,
                            int input_format) {
  if (legal_moves.size() != histories.size())
    throw std::invalid_argument("legal move list count must match history count");
  std::vector<LeafResult> out(histories.size());
  if (histories.empty()) return out;
  std::lock_guard<std::mutex> lock(mutex_);
  const int n = static_cast<int>(histories.size());
  boards_.clear();
  history_offsets_.assign(1, 0);
  moves_.clear();
  move_offsets_.assign(1, 0);
  for (int b = 0; b < n; ++b) {
    for (const Position *p : histories[b]) boards_.push_back(ToBoard(*p));
    history_offsets_.push_back(static_cast<std::int32_t>(boards_.size()));
    for (Move m : legal_moves[b]) moves_.push_back(ToRawMove(m));
    move_offsets_.push_back(static_cast<std::int32_t>(moves_.size()));
  }
  priors_.resize(moves_.size());
  wdl_.resize(size_t(n) * 3);
  mlh_.resize(n);
  for (int lo = 0; lo < n; lo += options_.max_batch) {
    const int cnt = std::min(options_.max_batch, n - lo);
    if (mfb200_evaluate_leaves(handle_, boards_.data() + history_offsets_[lo],
                               history_offsets_.data() + lo, cnt, input_format,
                               moves_.data() + move_offsets_[lo], move_offsets_.data() + lo,
                               softmax_temp, priors_.data() + move_offsets_[lo],
                               wdl_.data() + size_t(lo) * 3, mlh_.data() + lo, nullptr) != 0)
      throw std::runtime_error(std::string("B200 backend: ") + mfb200_last_error(handle_));
  }
  for (int b = 0; b < n; ++b) {
    LeafResult &r = out[b];
    r.priors.assign(priors_.begin() + move_offsets_[b], priors_.begin() + move_offsets_[b + 1]);
    r.wdl[0] = wdl_[3 * b];
    r.wdl[1] = wdl_[3 * b + 1];
    r.wdl[2] = wdl_[3 * b + 2];
    r.value = r.wdl[0] - r.wdl[2];
    r.moves_left = mlh_[b];
  }
  return out;
}

std::string B200Network::GetNetworkInfo() const { return info_; }

BackendCapabilities B200Network::GetBackendCapabilities() const {
  mfb200_caps c{};
  BackendCapabilities caps;
  caps.actual_backend = "b200";
  caps.has_wdl = true;
  caps.has_moves_left = true;
  if (mfb200_capabilities(handle_, &c) == 0) {
    caps.max_batch_size = c.max_batch;
    caps.device_name = c.device_name;
  }
  return caps;
}

}  // namespace B200
}  // namespace NN
}  // namespace MetalFish
