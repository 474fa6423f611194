// b200_network.h -- MetalFish NN backend over libmfb200 (the B200 BT4 forward).
//
// Drop-in for the engine's backend factory: a Network subclass
// (src/nn/network.h:38-51) that CreateNetwork (src/nn/network.cpp:137-208)
// can return for backend "b200". It takes the same WeightsFile the CPU and
// CUDA backends take, decodes it with the engine's own MultiHeadWeights
// (src/nn/weights.h), and evaluates through the C ABI of include/mfb200.h.
// Errors throw std::runtime_error, as the reference backends do.
#pragma once

#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "core/position.h"
#include "nn/network.h"

struct mfb200_handle;
struct mfb200_board;

namespace MetalFish {
namespace NN {
namespace B200 {

struct B200Options {
  int device = 0;         // first CUDA device
  int num_devices = 1;    // batch sharded over [device, device + num_devices)
  int max_batch = 1024;   // largest EvaluateBatch size
  bool use_graphs = true; // one CUDA graph per batch size
};

class B200Network : public Network {
public:
  B200Network(const WeightsFile &weights, const B200Options &options);
  // BackendConfig mapping: cuda_device -> device, cuda_graph_execution ->
  // use_graphs, cuda_stable_execution_batch_size (if > 0) -> max_batch.
  B200Network(const WeightsFile &weights, const BackendConfig &config);
  ~B200Network() override;

  NetworkOutput Evaluate(const InputPlanes &input) override;
  std::vector<NetworkOutput> EvaluateBatch(const std::vector<InputPlanes> &inputs) override;
  std::string GetNetworkInfo() const override;
  bool HasWDL() const override { return true; }
  bool HasMovesLeft() const override { return true; }
  BackendCapabilities GetBackendCapabilities() const override;

  // The MCTS leaf step on the GPU (mfb200_evaluate_priors): for each input,
  // the normalised priors of its legal moves, given as policy indices (the
  // evaluator's NN::MoveToNNIndex of each move, mirrored for black, with the
  // encoder's transform: src/mcts/evaluator.cpp:195-206), with the softmax of
  // ApplyNNPolicyToNode (src/mcts/search.cpp:127-197) at softmax_temp.
  struct LeafResult {
    std::vector<float> priors;  // one per legal move, in the given order
    float wdl[3];
    float value;                // wdl[0] - wdl[2]
    float moves_left;
  };
  std::vector<LeafResult> EvaluatePriors(const std::vector<InputPlanes> &inputs,
                                         const std::vector<std::vector<std::int16_t>> &move_indices,
                                         float softmax_temp);

  // The whole leaf evaluation on the GPU (mfb200_evaluate_leaves): what
  // NNMCTSEvaluator::EvaluateBatchWithHistoryViews does (encode each history,
  // evaluate, gather the legal moves' logits: src/mcts/evaluator.cpp:140-226)
  // plus ApplyNNPolicyToNode's softmax. histories[i] is the game so far,
  // oldest first, ending with the leaf; legal_moves[i] its moves in edge
  // order; input_format the network's (NetworkFormat::InputFormat).
  std::vector<LeafResult> EvaluateLeaves(const std::vector<std::vector<const Position *>> &histories,
                                         const std::vector<std::vector<Move>> &legal_moves,
                                         float softmax_temp, int input_format);

private:
  mfb200_handle *handle_ = nullptr;
  B200Options options_;
  std::string info_;
  std::vector<std::uint64_t> masks_;  // packing scratch, reused across calls
  std::vector<float> values_;
  std::vector<float> policy_, wdl_, mlh_;
  std::vector<std::int32_t> move_offsets_;  // EvaluatePriors scratch
  std::vector<std::int16_t> move_index_;
  std::vector<float> priors_;
  std::vector<mfb200_board> boards_;        // EvaluateLeaves scratch
  std::vector<std::int32_t> history_offsets_;
  std::vector<std::uint16_t> moves_;
  std::mutex mutex_;
};

}  // namespace B200
}  // namespace NN
}  // namespace MetalFish
