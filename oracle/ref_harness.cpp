// Reference harness -- TEST INFRASTRUCTURE ONLY (never linked into the product).
//
// Drives the reference's own, unmodified CPU code (compiled from the
// reference source tree against the protobuf shim in oracle/shim):
//
//   gen-inputs <seed> <count> <out.mfin>
//       Seeded uniform-random legal playouts of 0-80 plies from the start
//       position (per-position RNG seed = seed XOR index, std::mt19937_64),
//       encoded with EncodePositionForNN(INPUT_112_WITH_CANONICALIZATION_V2,
//       history <= 8, FillEmptyHistory::FEN_ONLY) -- the call the reference
//       benchmark makes (tests/test_nn_comparison.cpp:1518-1524) -- and packed
//       with PackInputPlanesRaw (src/nn/input_plane_packing.h:63-83).
//
//   eval <net.mfnt> <in.mfin> <out.mfot> [threads] [first] [count]
//       Builds a MetalFishNN::Net in memory with FLOAT32 layers (the pattern of
//       tests/test_mcts_module.cpp:91-103), constructs the reference
//       Cpu::CpuNetwork through NN::CreateNetwork(weights, "cpu")
//       (src/nn/network.cpp:188-190) and runs EvaluateBatch on contiguous
//       chunks, one std::thread per chunk (CpuNetwork::RunBatch is const and
//       reentrant, src/nn/cpu/cpu_network.cpp:580). Prints one JSON line with
//       the wall time of the EvaluateBatch calls.
//
//   to-pb <net.mfnt> <out.pb>
//       Serialises the same in-memory Net as a protobuf .pb weights file.
//
//   eval-backend <cpu|b200> ...  (b200 only in the b200_harness build)
//       As eval, through the named backend; "b200" constructs the B200
//       Network subclass (metalfish_b200/host) from the same WeightsFile.
//
// File formats (all little-endian) are produced/consumed by
// metalfish_b200/netfile.py.
#include "nn/encoder.h"
#include "nn/input_plane_packing.h"
#include "nn/network.h"
#include "core/bitboard.h"
#include "core/movegen.h"
#include "core/position.h"
#include "mcts/core.h"
#include "nn/policy_map.h"
#ifdef MFB_WITH_B200
#include "../metalfish_b200/host/b200_network.h"
#endif

#include <chrono>
#include <cstdio>
#include <cstring>
#include <deque>
#include <fstream>
#include <iostream>
#include <limits>
#include <map>
#include <random>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

using namespace MetalFish;
namespace NN = MetalFish::NN;

namespace {

constexpr char kStartFen[] = "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1";

std::string ReadFile(const std::string &path) {
  std::ifstream in(path, std::ios::binary);
  if (!in) throw std::runtime_error("cannot open " + path);
  return std::string((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
}

struct Reader {
  const std::string &s;
  std::size_t off = 0;
  template <class T> T get() {
    if (off + sizeof(T) > s.size()) throw std::runtime_error("truncated file");
    T v; std::memcpy(&v, s.data() + off, sizeof(T)); off += sizeof(T); return v;
  }
  std::string bytes(std::size_t n) {
    if (off + n > s.size()) throw std::runtime_error("truncated file");
    std::string r = s.substr(off, n); off += n; return r;
  }
};

// ------------------------------------------------------------------ inputs
struct Inputs {
  std::vector<std::uint64_t> masks;
  std::vector<float> values;
  int count = 0;
};

Inputs ReadInputs(const std::string &path) {
  const std::string s = ReadFile(path);
  Reader r{s};
  if (r.bytes(4) != "MFIN") throw std::runtime_error("bad input magic");
  (void)r.get<std::uint32_t>();
  Inputs in;
  in.count = int(r.get<std::uint32_t>());
  const std::uint32_t planes = r.get<std::uint32_t>();
  if (planes != 112) throw std::runtime_error("bad plane count");
  in.masks.resize(std::size_t(in.count) * 112);
  in.values.resize(std::size_t(in.count) * 112);
  std::memcpy(in.masks.data(), r.bytes(in.masks.size() * 8).data(), in.masks.size() * 8);
  std::memcpy(in.values.data(), r.bytes(in.values.size() * 4).data(), in.values.size() * 4);
  return in;
}

NN::InputPlanes Unpack(const Inputs &in, int b) {
  NN::InputPlanes planes{};
  for (int p = 0; p < 112; ++p) {
    const std::uint64_t m = in.masks[std::size_t(b) * 112 + p];
    const float v = in.values[std::size_t(b) * 112 + p];
    for (int sq = 0; sq < 64; ++sq) planes[p][sq] = ((m >> sq) & 1ULL) ? v : 0.0f;
  }
  return planes;
}

// One seeded random-playout game: position i of a fixture is the final
// position of a uniformly random legal line of 0..80 plies from the start
// position (per-position seed = seed ^ i), with the whole game history kept
// so the encoder can look back (src/nn/encoder.cpp:371-400).
struct Game {
  std::vector<std::unique_ptr<Position>> positions;
  std::vector<std::unique_ptr<StateInfo>> roots;
  std::vector<std::deque<StateInfo>> stacks;
  std::vector<const Position *> ptrs;
};

void BuildGame(std::uint64_t seed, int i, Game &g, const char *fen = kStartFen) {
  std::mt19937_64 rng(seed ^ std::uint64_t(i));
  const int target_plies = int(rng() % 81);
  // Play the line once to fix the moves.
  std::vector<Move> line;
  {
    Position pos;
    StateInfo root;
    std::deque<StateInfo> states;
    pos.set(fen, false, &root);
    for (int ply = 0; ply < target_plies; ++ply) {
      MoveList<LEGAL> legal(pos);
      if (legal.size() == 0) break;
      const Move m = *(legal.begin() + (rng() % legal.size()));
      line.push_back(m);
      states.emplace_back();
      pos.do_move(m, states.back());
    }
  }
  // Rebuild the full game history, each position replayed from the start so
  // that every Position keeps its own StateInfo chain (as build_history does
  // in tests/test_nn_comparison.cpp:280-302).
  const int total = int(line.size());
  g.stacks.resize(total + 1);
  for (int ply = 0; ply <= total; ++ply) {
    g.positions.push_back(std::make_unique<Position>());
    g.roots.push_back(std::make_unique<StateInfo>());
    g.positions.back()->set(fen, false, g.roots.back().get());
    auto &stack = g.stacks[ply];
    for (int k = 0; k < ply; ++k) {
      stack.emplace_back();
      g.positions.back()->do_move(line[k], stack.back());
    }
    g.ptrs.push_back(g.positions.back().get());
  }
}

int GenInputs(std::uint64_t seed, int count, const std::string &out_path) {
  Bitboards::init();
  Position::init();
  std::vector<std::uint64_t> masks(std::size_t(count) * 112);
  std::vector<float> values(std::size_t(count) * 112);
  for (int i = 0; i < count; ++i) {
    Game g;
    BuildGame(seed, i, g);
    int transform = 0;
    const NN::InputPlanes planes = NN::EncodePositionForNN(
        MetalFishNN::NetworkFormat::INPUT_112_WITH_CANONICALIZATION_V2, g.ptrs,
        NN::kMoveHistory, NN::FillEmptyHistory::FEN_ONLY, &transform);
    std::vector<std::uint64_t> m;
    std::vector<float> v;
    NN::PackInputPlanesRaw(planes[0].data(), 1, m, v);
    std::memcpy(&masks[std::size_t(i) * 112], m.data(), 112 * 8);
    std::memcpy(&values[std::size_t(i) * 112], v.data(), 112 * 4);
  }
  std::ofstream out(out_path, std::ios::binary);
  const std::uint32_t hdr[3] = {1, std::uint32_t(count), 112};
  out.write("MFIN", 4);
  out.write(reinterpret_cast<const char *>(hdr), sizeof(hdr));
  out.write(reinterpret_cast<const char *>(masks.data()), masks.size() * 8);
  out.write(reinterpret_cast<const char *>(values.data()), values.size() * 4);
  return out.good() ? 0 : 1;
}

// ------------------------------------------------------------------ legal moves
// The evaluator's vertical mirror for black to move
// (src/mcts/evaluator.cpp:24-36, a file-local helper there): both squares
// mirrored; promotions keep their piece, every other move becomes a plain
// from-to move.
Move MirrorVertical(Move m) {
  auto mirror = [](Square sq) { return make_square(file_of(sq), Rank(7 - rank_of(sq))); };
  if (m.type_of() == PROMOTION)
    return Move::make<PROMOTION>(mirror(m.from_sq()), mirror(m.to_sq()), m.promotion_type());
  return Move(mirror(m.from_sq()), mirror(m.to_sq()));
}

// For the fixture positions of GenInputs: the policy index of every legal
// move, in MoveList<LEGAL> order, as the evaluator maps it
// (src/mcts/evaluator.cpp:195-206: mirror for black, then
// NN::MoveToNNIndex(move, transform) with the encoder's transform).
// Output "MFMV", u32 version, u32 count, i32 offsets[count+1], i16 index[total],
// u16 raw[total] (the move itself: from | to << 6 | promotion << 12 with
// 0 none, 1 queen, 2 rook, 3 bishop, 4 knight).
int GenMoves(std::uint64_t seed, int count, const std::string &out_path) {
  Bitboards::init();
  Position::init();
  NN::InitPolicyTables();
  std::vector<std::int32_t> offsets(1, 0);
  std::vector<std::int16_t> index;
  std::vector<std::uint16_t> raw;  // from | to << 6 | promotion << 12 (1 Q, 2 R, 3 B, 4 N)
  for (int i = 0; i < count; ++i) {
    Game g;
    BuildGame(seed, i, g);
    int transform = 0;
    (void)NN::EncodePositionForNN(MetalFishNN::NetworkFormat::INPUT_112_WITH_CANONICALIZATION_V2,
                                  g.ptrs, NN::kMoveHistory, NN::FillEmptyHistory::FEN_ONLY,
                                  &transform);
    const Position &pos = *g.ptrs.back();
    for (Move m : MoveList<LEGAL>(pos)) {
      const Move pm = pos.side_to_move() == BLACK ? MirrorVertical(m) : m;
      index.push_back(std::int16_t(NN::MoveToNNIndex(pm, transform)));
      int kind = 0;
      if (m.type_of() == PROMOTION) {
        const PieceType pt = m.promotion_type();
        kind = pt == QUEEN ? 1 : pt == ROOK ? 2 : pt == BISHOP ? 3 : 4;
      }
      raw.push_back(std::uint16_t(int(m.from_sq()) | (int(m.to_sq()) << 6) | (kind << 12)));
    }
    offsets.push_back(std::int32_t(index.size()));
  }
  std::ofstream out(out_path, std::ios::binary);
  const std::uint32_t hdr[2] = {1, std::uint32_t(count)};
  out.write("MFMV", 4);
  out.write(reinterpret_cast<const char *>(hdr), sizeof(hdr));
  out.write(reinterpret_cast<const char *>(offsets.data()), offsets.size() * 4);
  out.write(reinterpret_cast<const char *>(index.data()), index.size() * 2);
  out.write(reinterpret_cast<const char *>(raw.data()), raw.size() * 2);
  return out.good() ? 0 : 1;
}

// Every position of each fixture game (oldest first) as the board records
// the GPU encoder takes (include/mfb200.h, mfb200_board), read through the
// reference's Position accessors, plus the transform the reference encoder
// chose for the final position. Output "MFHB", u32 version, u32 count,
// i32 offsets[count+1], 112-byte records, i32 transforms[count].
struct BoardRecord {
  std::uint64_t pieces[2][6];
  std::int32_t rule50, game_ply;
  std::int8_t ep_square;
  std::uint8_t castling, black_to_move, repetition;
  std::uint32_t reserved;
};
static_assert(sizeof(BoardRecord) == 112, "board record layout");

BoardRecord Record(const Position &p) {
  BoardRecord r{};
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

// After the V2 transforms: u32 n_all, then for each of the seven input
// formats: i32 format, u64 masks[n_all*112], f32 values[n_all*112],
// i32 transforms[n_all] -- the reference encoding of the first n_all
// positions in every format.
int GenHistory(std::uint64_t seed, int count, int n_all, const std::string &out_path,
               const char *fen = kStartFen) {
  using IF = MetalFishNN::NetworkFormat;
  const IF::InputFormat formats[7] = {
      IF::INPUT_CLASSICAL_112_PLANE, IF::INPUT_112_WITH_CASTLING_PLANE,
      IF::INPUT_112_WITH_CANONICALIZATION, IF::INPUT_112_WITH_CANONICALIZATION_HECTOPLIES,
      IF::INPUT_112_WITH_CANONICALIZATION_V2,
      IF::INPUT_112_WITH_CANONICALIZATION_HECTOPLIES_ARMAGEDDON,
      IF::INPUT_112_WITH_CANONICALIZATION_V2_ARMAGEDDON};
  Bitboards::init();
  Position::init();
  n_all = std::min(n_all, count);
  std::vector<std::int32_t> offsets(1, 0), transforms;
  std::vector<BoardRecord> boards;
  std::vector<std::uint64_t> fm[7];
  std::vector<float> fv[7];
  std::vector<std::int32_t> ft[7];
  for (int i = 0; i < count; ++i) {
    Game g;
    BuildGame(seed, i, g, fen);
    for (const Position *p : g.ptrs) boards.push_back(Record(*p));
    offsets.push_back(std::int32_t(boards.size()));
    int transform = 0;
    (void)NN::EncodePositionForNN(IF::INPUT_112_WITH_CANONICALIZATION_V2, g.ptrs,
                                  NN::kMoveHistory, NN::FillEmptyHistory::FEN_ONLY, &transform);
    transforms.push_back(transform);
    if (i < n_all) {
      for (int f = 0; f < 7; ++f) {
        int t = 0;
        const NN::InputPlanes planes = NN::EncodePositionForNN(
            formats[f], g.ptrs, NN::kMoveHistory, NN::FillEmptyHistory::FEN_ONLY, &t);
        std::vector<std::uint64_t> m;
        std::vector<float> v;
        NN::PackInputPlanesRaw(planes[0].data(), 1, m, v);
        fm[f].insert(fm[f].end(), m.begin(), m.end());
        fv[f].insert(fv[f].end(), v.begin(), v.end());
        ft[f].push_back(t);
      }
    }
  }
  std::ofstream out(out_path, std::ios::binary);
  const std::uint32_t hdr[2] = {1, std::uint32_t(count)};
  out.write("MFHB", 4);
  out.write(reinterpret_cast<const char *>(hdr), sizeof(hdr));
  out.write(reinterpret_cast<const char *>(offsets.data()), offsets.size() * 4);
  out.write(reinterpret_cast<const char *>(boards.data()), boards.size() * sizeof(BoardRecord));
  out.write(reinterpret_cast<const char *>(transforms.data()), transforms.size() * 4);
  const std::uint32_t na = std::uint32_t(n_all);
  out.write(reinterpret_cast<const char *>(&na), 4);
  for (int f = 0; f < 7; ++f) {
    const std::int32_t code = formats[f];
    out.write(reinterpret_cast<const char *>(&code), 4);
    out.write(reinterpret_cast<const char *>(fm[f].data()), fm[f].size() * 8);
    out.write(reinterpret_cast<const char *>(fv[f].data()), fv[f].size() * 4);
    out.write(reinterpret_cast<const char *>(ft[f].data()), ft[f].size() * 4);
  }
  return out.good() ? 0 : 1;
}

// NN::MoveToNNIndex (src/nn/policy_map.cpp:316-360) for every transform
// (0..7), promotion kind (none, queen, rook, bishop, knight) and (from, to)
// pair: int16 [8][5][64][64], -1 where the reference returns -1.
int DumpMoveIndex(const std::string &out_path) {
  NN::InitPolicyTables();
  const PieceType promo[5] = {NO_PIECE_TYPE, QUEEN, ROOK, BISHOP, KNIGHT};
  std::vector<std::int16_t> table;
  table.reserve(8 * 5 * 4096);
  for (int t = 0; t < 8; ++t)
    for (int k = 0; k < 5; ++k)
      for (int from = 0; from < 64; ++from)
        for (int to = 0; to < 64; ++to) {
          const Move m = k == 0 ? Move(Square(from), Square(to))
                                : Move::make<PROMOTION>(Square(from), Square(to), promo[k]);
          table.push_back(std::int16_t(NN::MoveToNNIndex(m, t)));
        }
  std::ofstream out(out_path, std::ios::binary);
  out.write(reinterpret_cast<const char *>(table.data()), table.size() * 2);
  return out.good() ? 0 : 1;
}

// The reference's FastExp (src/mcts/core.h:38-44) over a raw f32 file.
int FastExpFile(const std::string &in_path, const std::string &out_path) {
  const std::string s = ReadFile(in_path);
  std::vector<float> x(s.size() / 4);
  std::memcpy(x.data(), s.data(), x.size() * 4);
  for (float &v : x) v = MCTS::FastMath::FastExp(v);
  std::ofstream out(out_path, std::ios::binary);
  out.write(reinterpret_cast<const char *>(x.data()), x.size() * 4);
  return out.good() ? 0 : 1;
}

// ------------------------------------------------------------------ network
MetalFishNN::NetworkFormat_ActivationFunction ActivationByName(const std::string &n) {
  using NF = MetalFishNN::NetworkFormat;
  if (n == "mish") return NF::ACTIVATION_MISH;
  if (n == "relu") return NF::ACTIVATION_RELU;
  if (n == "swish") return NF::ACTIVATION_SWISH;
  if (n == "relu_2") return NF::ACTIVATION_RELU_2;
  if (n == "selu") return NF::ACTIVATION_SELU;
  if (n == "tanh") return NF::ACTIVATION_TANH;
  if (n == "sigmoid") return NF::ACTIVATION_SIGMOID;
  if (n == "default" || n.empty()) return NF::ACTIVATION_DEFAULT;
  throw std::runtime_error("unknown activation " + n);
}

using Layer = MetalFishNN::Weights::Layer;

Layer *SmolgenLayer(MetalFishNN::Weights::Smolgen *s, const std::string &f) {
  if (f == "compress") return s->mutable_compress();
  if (f == "dense1_w") return s->mutable_dense1_w();
  if (f == "dense1_b") return s->mutable_dense1_b();
  if (f == "ln1_gammas") return s->mutable_ln1_gammas();
  if (f == "ln1_betas") return s->mutable_ln1_betas();
  if (f == "dense2_w") return s->mutable_dense2_w();
  if (f == "dense2_b") return s->mutable_dense2_b();
  if (f == "ln2_gammas") return s->mutable_ln2_gammas();
  if (f == "ln2_betas") return s->mutable_ln2_betas();
  return nullptr;
}

Layer *FfnLayer(MetalFishNN::Weights::FFN *f, const std::string &n) {
  if (n == "dense1_w") return f->mutable_dense1_w();
  if (n == "dense1_b") return f->mutable_dense1_b();
  if (n == "dense2_w") return f->mutable_dense2_w();
  if (n == "dense2_b") return f->mutable_dense2_b();
  return nullptr;
}

std::vector<std::string> Split(const std::string &s) {
  std::vector<std::string> parts;
  std::stringstream ss(s);
  std::string p;
  while (std::getline(ss, p, '.')) parts.push_back(p);
  return parts;
}

Layer *ResolveLayer(MetalFishNN::Weights *w, const std::string &name) {
  const auto p = Split(name);
  if (p.size() == 1) {
    const std::string &n = p[0];
#define TOP(x) if (n == #x) return w->mutable_##x();
    TOP(ip_emb_preproc_w) TOP(ip_emb_preproc_b) TOP(ip_emb_w) TOP(ip_emb_b)
    TOP(ip_emb_ln_gammas) TOP(ip_emb_ln_betas) TOP(ip_mult_gate) TOP(ip_add_gate)
    TOP(ip_emb_ffn_ln_gammas) TOP(ip_emb_ffn_ln_betas) TOP(smolgen_w)
    TOP(ip_mov_w) TOP(ip_mov_b) TOP(ip1_mov_w) TOP(ip1_mov_b) TOP(ip2_mov_w) TOP(ip2_mov_b)
#undef TOP
    return nullptr;
  }
  if (p[0] == "ip_emb_ffn" && p.size() == 2) return FfnLayer(w->mutable_ip_emb_ffn(), p[1]);
  if (p[0] == "encoder" && p.size() >= 3) {
    const int idx = std::stoi(p[1]);
    while (w->encoder_size() <= idx) w->add_encoder();
    auto *enc = w->mutable_encoder(idx);
    if (p.size() == 3) {
      if (p[2] == "ln1_gammas") return enc->mutable_ln1_gammas();
      if (p[2] == "ln1_betas") return enc->mutable_ln1_betas();
      if (p[2] == "ln2_gammas") return enc->mutable_ln2_gammas();
      if (p[2] == "ln2_betas") return enc->mutable_ln2_betas();
      return nullptr;
    }
    if (p[2] == "ffn" && p.size() == 4) return FfnLayer(enc->mutable_ffn(), p[3]);
    if (p[2] == "mha" && p.size() == 4) {
      auto *m = enc->mutable_mha();
      const std::string &n = p[3];
#define MHA(x) if (n == #x) return m->mutable_##x();
      MHA(q_w) MHA(q_b) MHA(k_w) MHA(k_b) MHA(v_w) MHA(v_b) MHA(dense_w) MHA(dense_b)
#undef MHA
      return nullptr;
    }
    if (p[2] == "mha" && p.size() == 5 && p[3] == "smolgen")
      return SmolgenLayer(enc->mutable_mha()->mutable_smolgen(), p[4]);
    return nullptr;
  }
  if (p[0] == "policy_heads" && p.size() == 3 && p[1] == "vanilla") {
    auto *h = w->mutable_policy_heads()->mutable_vanilla();
    const std::string &n = p[2];
#define POL(x) if (n == #x) return h->mutable_##x();
    POL(ip_pol_w) POL(ip_pol_b) POL(ip2_pol_w) POL(ip2_pol_b) POL(ip3_pol_w) POL(ip3_pol_b)
    POL(ip4_pol_w)
#undef POL
    return nullptr;
  }
  if (p[0] == "value_heads" && p.size() == 3 && p[1] == "winner") {
    auto *h = w->mutable_value_heads()->mutable_winner();
    const std::string &n = p[2];
#define VAL(x) if (n == #x) return h->mutable_##x();
    VAL(ip_val_w) VAL(ip_val_b) VAL(ip1_val_w) VAL(ip1_val_b) VAL(ip2_val_w) VAL(ip2_val_b)
#undef VAL
    return nullptr;
  }
  return nullptr;
}

NN::WeightsFile ReadNet(const std::string &path) {
  const std::string s = ReadFile(path);
  Reader r{s};
  if (r.bytes(4) != "MFNT") throw std::runtime_error("bad net magic");
  (void)r.get<std::uint32_t>();
  const std::uint32_t header_len = r.get<std::uint32_t>();
  std::map<std::string, std::string> header;
  {
    std::stringstream hs(r.bytes(header_len));
    std::string line;
    while (std::getline(hs, line)) {
      const auto eq = line.find('=');
      if (eq != std::string::npos) header[line.substr(0, eq)] = line.substr(eq + 1);
    }
  }
  NN::WeightsFile file;
  file.set_magic(0x1c0);
  using NF = MetalFishNN::NetworkFormat;
  auto *nf = file.mutable_format()->mutable_network_format();
  nf->set_input(NF::INPUT_112_WITH_CANONICALIZATION_V2);
  nf->set_output(NF::OUTPUT_WDL);
  nf->set_network(NF::NETWORK_ATTENTIONBODY_WITH_MULTIHEADFORMAT);
  nf->set_policy(NF::POLICY_ATTENTION);
  nf->set_value(NF::VALUE_WDL);
  nf->set_moves_left(NF::MOVES_LEFT_V1);
  nf->set_input_embedding(NF::INPUT_EMBEDDING_PE_DENSE);
  nf->set_default_activation(header["default_activation"] == "relu"
                                 ? NF::DEFAULT_ACTIVATION_RELU
                                 : NF::DEFAULT_ACTIVATION_MISH);
  nf->set_smolgen_activation(ActivationByName(header["smolgen_activation"]));
  nf->set_ffn_activation(ActivationByName(header["ffn_activation"]));
  auto *w = file.mutable_weights();
  w->set_headcount(std::uint32_t(std::stoul(header.at("heads"))));
  const std::uint32_t count = r.get<std::uint32_t>();
  for (std::uint32_t t = 0; t < count; ++t) {
    const std::string name = r.bytes(r.get<std::uint32_t>());
    const std::uint32_t ndims = r.get<std::uint32_t>();
    std::vector<std::uint32_t> dims(ndims);
    std::size_t elements = 1;
    for (auto &d : dims) { d = r.get<std::uint32_t>(); elements *= d; }
    Layer *layer = ResolveLayer(w, name);
    if (!layer) throw std::runtime_error("unknown tensor name " + name);
    layer->set_encoding(Layer::FLOAT32);
    layer->set_params(r.bytes(elements * 4));
    layer->clear_dims();
    for (auto d : dims) layer->add_dims(d);
  }
  return file;
}

int Eval(const std::string &net_path, const std::string &in_path, const std::string &out_path,
         int threads, int first, int count, const std::string &backend = "cpu") {
  const NN::WeightsFile file = ReadNet(net_path);
  const Inputs in = ReadInputs(in_path);
  if (count < 0) count = in.count - first;
  if (first < 0 || count < 0 || first + count > in.count) throw std::runtime_error("bad range");
  std::unique_ptr<NN::Network> net;
#ifdef MFB_WITH_B200
  if (backend == "b200") {
    // the integration under test: the B200 backend built from the same
    // WeightsFile the CPU backend takes, evaluated through NN::Network
    NN::B200::B200Options opt;
    opt.max_batch = std::max(1, count);
    net = std::make_unique<NN::B200::B200Network>(file, opt);
    threads = 1;  // one handle, batched on the GPU
  }
#endif
  if (!net) net = NN::CreateNetwork(file, backend);
  std::vector<NN::InputPlanes> planes(count);
  for (int b = 0; b < count; ++b) planes[b] = Unpack(in, first + b);
  std::vector<NN::NetworkOutput> outputs(count);
  threads = std::max(1, std::min(threads, std::max(count, 1)));
  const auto t0 = std::chrono::steady_clock::now();
  std::vector<std::thread> pool;
  std::vector<std::string> errors(threads);
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([&, t] {
      const int lo = int(std::int64_t(count) * t / threads);
      const int hi = int(std::int64_t(count) * (t + 1) / threads);
      if (lo >= hi) return;
      try {
        std::vector<NN::InputPlanes> chunk(planes.begin() + lo, planes.begin() + hi);
        auto res = net->EvaluateBatch(chunk);
        for (int i = lo; i < hi; ++i) outputs[i] = res[i - lo];
      } catch (const std::exception &e) {
        errors[t] = e.what();
      }
    });
  }
  for (auto &th : pool) th.join();
  const double secs =
      std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  for (const auto &e : errors)
    if (!e.empty()) throw std::runtime_error(e);
  std::ofstream out(out_path, std::ios::binary);
  out.write("MFOT", 4);
  const std::uint32_t hdr[2] = {1, std::uint32_t(count)};
  out.write(reinterpret_cast<const char *>(hdr), sizeof(hdr));
  for (int b = 0; b < count; ++b)
    out.write(reinterpret_cast<const char *>(outputs[b].policy.data()), NN::kPolicyOutputs * 4);
  for (int b = 0; b < count; ++b)
    out.write(reinterpret_cast<const char *>(outputs[b].wdl), 12);
  for (int b = 0; b < count; ++b)
    out.write(reinterpret_cast<const char *>(&outputs[b].value), 4);
  for (int b = 0; b < count; ++b)
    out.write(reinterpret_cast<const char *>(&outputs[b].moves_left), 4);
  std::printf("{\"positions\": %d, \"threads\": %d, \"seconds\": %.6f, \"pos_per_s\": %.6f, "
              "\"info\": \"%s\"}\n",
              count, threads, secs, secs > 0 ? count / secs : 0.0,
              net->GetBackendCapabilities().Summary().c_str());
  return out.good() ? 0 : 1;
}

int ToPb(const std::string &net_path, const std::string &out_path) {
  const NN::WeightsFile file = ReadNet(net_path);
  std::string bytes;
  file.SerializeToString(&bytes);
  std::ofstream out(out_path, std::ios::binary);
  out.write(bytes.data(), std::streamsize(bytes.size()));
  return out.good() ? 0 : 1;
}

#ifdef MFB_WITH_B200
// The C++ backend's MCTS leaf step: B200Network::EvaluatePriors over the
// fixture positions [0, count) with their legal-move index lists.
int PriorsB200(const std::string &net_path, const std::string &in_path,
               const std::string &moves_path, float temp, const std::string &out_path) {
  const NN::WeightsFile file = ReadNet(net_path);
  const Inputs in = ReadInputs(in_path);
  const std::string s = ReadFile(moves_path);
  Reader r{s};
  if (r.bytes(4) != "MFMV") throw std::runtime_error("bad legal-move magic");
  (void)r.get<std::uint32_t>();
  const int count = int(r.get<std::uint32_t>());
  if (count > in.count) throw std::runtime_error("more move lists than positions");
  std::vector<std::int32_t> off(count + 1);
  for (auto &o : off) o = r.get<std::int32_t>();
  std::vector<std::vector<std::int16_t>> moves(count);
  for (int b = 0; b < count; ++b)
    for (int i = off[b]; i < off[b + 1]; ++i) moves[b].push_back(r.get<std::int16_t>());
  NN::B200::B200Options opt;
  opt.max_batch = std::max(1, count);
  NN::B200::B200Network net(file, opt);
  std::vector<NN::InputPlanes> planes(count);
  for (int b = 0; b < count; ++b) planes[b] = Unpack(in, b);
  const auto res = net.EvaluatePriors(planes, moves, temp);
  std::ofstream out(out_path, std::ios::binary);
  for (const auto &x : res)
    out.write(reinterpret_cast<const char *>(x.priors.data()), x.priors.size() * 4);
  return out.good() ? 0 : 1;
}

// The C++ backend's whole leaf evaluation: B200Network::EvaluateLeaves on
// the fixture games' real Positions and MoveList<LEGAL> moves.
int LeavesB200(const std::string &net_path, std::uint64_t seed, int count, float temp,
               const std::string &out_path) {
  Bitboards::init();
  Position::init();
  const NN::WeightsFile file = ReadNet(net_path);
  std::vector<Game> games(count);
  std::vector<std::vector<const Position *>> hist(count);
  std::vector<std::vector<Move>> moves(count);
  for (int i = 0; i < count; ++i) {
    BuildGame(seed, i, games[i]);
    hist[i] = games[i].ptrs;
    for (Move m : MoveList<LEGAL>(*games[i].ptrs.back())) moves[i].push_back(m);
  }
  NN::B200::B200Options opt;
  opt.max_batch = std::max(1, count);
  NN::B200::B200Network net(file, opt);
  const auto res = net.EvaluateLeaves(
      hist, moves, temp, MetalFishNN::NetworkFormat::INPUT_112_WITH_CANONICALIZATION_V2);
  std::ofstream out(out_path, std::ios::binary);
  for (const auto &x : res)
    out.write(reinterpret_cast<const char *>(x.priors.data()), x.priors.size() * 4);
  return out.good() ? 0 : 1;
}
#endif

} // namespace

int main(int argc, char **argv) {
  try {
    const std::string cmd = argc > 1 ? argv[1] : "";
    if (cmd == "gen-inputs" && argc == 5)
      return GenInputs(std::stoull(argv[2]), std::stoi(argv[3]), argv[4]);
    if (cmd == "eval" && argc >= 5)
      return Eval(argv[2], argv[3], argv[4], argc > 5 ? std::stoi(argv[5]) : 1,
                  argc > 6 ? std::stoi(argv[6]) : 0, argc > 7 ? std::stoi(argv[7]) : -1);
    if (cmd == "to-pb" && argc == 4) return ToPb(argv[2], argv[3]);
    if (cmd == "gen-moves" && argc == 5)
      return GenMoves(std::stoull(argv[2]), std::stoi(argv[3]), argv[4]);
    if (cmd == "fastexp" && argc == 4) return FastExpFile(argv[2], argv[3]);
    if (cmd == "dump-move-index" && argc == 3) return DumpMoveIndex(argv[2]);
    if (cmd == "gen-history" && (argc == 6 || argc == 7))
      return GenHistory(std::stoull(argv[2]), std::stoi(argv[3]), std::stoi(argv[4]), argv[5],
                        argc == 7 ? argv[6] : kStartFen);
#ifdef MFB_WITH_B200
    if (cmd == "priors-b200" && argc == 7)
      return PriorsB200(argv[2], argv[3], argv[4], std::stof(argv[5]), argv[6]);
    if (cmd == "leaves-b200" && argc == 7)
      return LeavesB200(argv[2], std::stoull(argv[3]), std::stoi(argv[4]), std::stof(argv[5]), argv[6]);
#endif
    if (cmd == "eval-backend" && argc >= 6)
      return Eval(argv[3], argv[4], argv[5], argc > 6 ? std::stoi(argv[6]) : 1,
                  argc > 7 ? std::stoi(argv[7]) : 0, argc > 8 ? std::stoi(argv[8]) : -1, argv[2]);
    std::fprintf(stderr,
                 "usage: ref_harness gen-inputs <seed> <count> <out.mfin>\n"
                 "       ref_harness eval <net.mfnt> <in.mfin> <out.mfot> [threads] [first] [count]\n"
                 "       ref_harness to-pb <net.mfnt> <out.pb>\n"
                 "       ref_harness gen-moves <seed> <count> <out.mfmv>\n"
                 "       ref_harness fastexp <in.f32> <out.f32>\n"
                 "       ref_harness dump-move-index <out.i16>\n"
                 "       ref_harness gen-history <seed> <count> <count-all-formats> <out.mfhb> [start-fen]\n"
                 "       ref_harness eval-backend <cpu|b200> <net.mfnt> <in.mfin> <out.mfot> [threads] [first] [count]\n"
                 "       b200_harness priors-b200 <net.mfnt> <in.mfin> <moves.mfmv> <temp> <out.f32>\n"
                 "       b200_harness leaves-b200 <net.mfnt> <seed> <count> <temp> <out.f32>\n");
    return 2;
  } catch (const std::exception &e) {
    std::fprintf(stderr, "ref_harness error: %s\n", e.what());
    return 1;
  }
}
