/* mfb200.h -- C ABI of the B200 BT4 forward library (libmfb200.so).
 *
 * This is the boundary a MetalFish NN backend binds: one handle owns a BT4
 * attention-body network resident on one or more B200 GPUs and evaluates
 * batches of packed input planes into raw policy logits, WDL probabilities
 * and moves-left. Plain pointers and sizes only; no C++ or torch types.
 *
 * Reference interfaces replaced (paths in the MetalFish source tree):
 *   mfb200_create       <- NN::CreateNetwork(const WeightsFile&, const BackendConfig&)
 *                          (src/nn/network.h:66-75, src/nn/network.cpp:137-208) together
 *                          with the accelerator constructor Cuda::CudaNetwork
 *                          (src/nn/cuda/cuda_network.h:26-57, cuda_network.cpp:235-343)
 *   mfb200_evaluate     <- NN::Network::EvaluateBatch(const std::vector<InputPlanes>&)
 *                          (src/nn/network.h:44-45); inputs are the packed planes of
 *                          PackInputPlanesRaw (src/nn/input_plane_packing.h:63-83) that
 *                          Cuda::CudaNetwork::RunBatch uploads (cuda_network.cpp:393-417);
 *                          outputs are the fields of NetworkOutput (src/nn/network_output.h:17-24)
 *   mfb200_evaluate_priors <- EvaluateBatch followed by the MCTS leaf step on the
 *                          caller's legal moves: the evaluator's per-move logit gather
 *                          (src/mcts/evaluator.cpp:182-226, NNMCTSEvaluator::Impl::BuildResult)
 *                          and the softmax of ApplyNNPolicyToNode
 *                          (src/mcts/search.cpp:127-197)
 *   mfb200_encode_history / mfb200_evaluate_history
 *                       <- NN::EncodePositionForNN (src/nn/encoder.cpp:249-466) on the
 *                          GPU: position histories in, packed planes (and the forward) out,
 *                          replacing the host encode of NNMCTSEvaluator
 *                          (src/mcts/evaluator.cpp:150-158)
 *   mfb200_evaluate_leaves <- NNMCTSEvaluator::EvaluateBatchWithHistoryViews
 *                          (src/mcts/evaluator.cpp:140-170: encode, EvaluateBatch,
 *                          BuildResult) + ApplyNNPolicyToNode's softmax
 *                          (src/mcts/search.cpp:127-197), all on the GPU
 *   mfb200_submit_leaves / mfb200_wait
 *                       <- the same, asynchronous, for the double-buffered batch
 *                          assembly of src/mcts/search.cpp:1955-2232 (no counterpart API
 *                          in the reference, whose backends evaluate synchronously)
 *   mfb200_capabilities <- NN::Network::GetBackendCapabilities / HasWDL / HasMovesLeft /
 *                          GetNetworkInfo (src/nn/network.h:21-51)
 *   mfb200_last_error   <- the std::runtime_error messages the reference throws
 *                          (src/nn/cuda/cuda_network.cpp:241-320, :457)
 *   mfb200_destroy      <- Network::~Network (src/nn/network.h:40)
 *
 * Status codes: 0 = success, nonzero = error; mfb200_last_error() returns a
 * message for the calling thread's last failure on that handle.
 * Thread safety: calls on one handle are serialised by an internal mutex
 * (as the reference CUDA backend's execution_mutex_, cuda_network.cpp:442).
 */
#ifndef MFB200_H
#define MFB200_H
#include <stddef.h>
#include <stdint.h>
#ifndef MFB200_API
#define MFB200_API __attribute__((visibility("default")))
#endif
#ifdef __cplusplus
extern "C" {
#endif

typedef struct mfb200_handle mfb200_handle;

/* Activation codes (the reference's activation names, network_format.cpp:50-70). */
enum {
  MFB200_ACT_NONE = 0, MFB200_ACT_RELU = 1, MFB200_ACT_RELU2 = 2, MFB200_ACT_TANH = 3,
  MFB200_ACT_SIGMOID = 4, MFB200_ACT_SWISH = 5, MFB200_ACT_MISH = 6, MFB200_ACT_SELU = 7
};
/* BF16: bf16/fp16 tensor-core GEMMs throughout. FP8: the encoder and
 * embedding-FFN GEMMs in e4m3 with per-output-channel weight scales and
 * calibrated per-tensor activation scales. INT8: the same GEMMs at the same
 * 8-bit tensor-core rate with signed 8-bit integer operands: per-output-channel
 * weight scales, per-row (per-square) activation scales computed when the
 * LayerNorm writes the input, calibrated per-tensor scales for the attention
 * context; int32 accumulation. */
enum { MFB200_PRECISION_BF16 = 0, MFB200_PRECISION_FP8 = 1, MFB200_PRECISION_INT8 = 2 };

/* Shape of an attention-body network with PE_DENSE input embedding, smolgen,
 * attention policy, WDL value and moves-left heads (the BT4 family). */
typedef struct {
  int32_t embedding;        /* d (multiple of 64; head depth d/heads must be 32) */
  int32_t layers;           /* encoder layers */
  int32_t heads;
  int32_t dff;              /* encoder FFN hidden */
  int32_t emb_dff;          /* input-embedding FFN hidden */
  int32_t pe;               /* dynamic positional-encoding width per square */
  int32_t smolgen_compress; /* per-token compress width */
  int32_t smolgen_hidden;   /* smolgen dense1 width */
  int32_t smolgen_gen;      /* per-head generator width */
  int32_t policy_d;         /* attention-policy embedding width */
  int32_t value_emb, value_hidden;
  int32_t mlh_emb, mlh_hidden;
  int32_t act_default, act_smolgen, act_ffn; /* MFB200_ACT_* */
} mfb200_net_desc;

typedef struct {
  int32_t device;     /* first CUDA device ordinal */
  int32_t num_devices;/* devices used from `device` on; the batch is sharded, weights replicated */
  int32_t precision;  /* MFB200_PRECISION_* */
  int32_t max_batch;  /* largest batch one evaluate call accepts */
  int32_t use_graphs; /* capture one CUDA graph per batch size (1) or launch eagerly (0) */
  int32_t fp8_gemms;  /* FP8 / INT8 handles: GEMM groups run with 8-bit operands (bit mask:
                         2 QKV, 4 attention output, 8 FFN1, 16 FFN2; 1 the embedding FFN --
                         both of its GEMMs in FP8 handles, its first in INT8 handles, whose
                         bit 16 also covers the embedding FFN2). 0 = the default: every group
                         in FP8 handles; 1|2|4|8 in INT8 handles (the two GEMMs that read the
                         FFN hidden stay bf16) */
} mfb200_config;

typedef struct {
  float h2d_ms, forward_ms, d2h_ms, total_ms; /* device-timed (max over devices) */
} mfb200_timing;

typedef struct {
  int32_t max_batch, precision, num_devices, device;
  int32_t has_wdl, has_moves_left;
  int64_t weight_bytes;      /* device bytes of packed weights (per device) */
  int64_t workspace_bytes;   /* device bytes of activations (per device) */
  char device_name[96];
} mfb200_caps;

/* Number of bytes of the fp32 weight blob mfb200_create expects for `desc`:
 * every tensor of the network in the reference's [out, in] layout,
 * concatenated in the slot order of metalfish_b200/layout.py. */
MFB200_API size_t mfb200_weight_bytes(const mfb200_net_desc *desc);

MFB200_API int mfb200_create(const mfb200_net_desc *desc, const void *weights_f32, size_t bytes,
                  const mfb200_config *cfg, mfb200_handle **out);

/* Host-buffer evaluation (the EvaluateBatch path): masks/values [batch,112]
 * (packed planes), outputs policy [batch,1858] raw logits, wdl [batch,3],
 * moves_left [batch]. Any of the output pointers may be NULL. `timing` may
 * be NULL. Blocks until the results are in host memory. */
MFB200_API int mfb200_evaluate(mfb200_handle *h, const uint64_t *masks, const float *values, int batch,
                    float *policy, float *wdl, float *moves_left, mfb200_timing *timing);

/* Host-buffer evaluation that returns, instead of the 1858 policy logits,
 * the normalised prior of each legal move (what MCTS needs per leaf):
 * move_offsets [batch + 1] is a CSR over move_index (move_offsets[0] is
 * usually 0; the slice [move_offsets[b], move_offsets[b+1]) belongs to
 * position b) and move_index holds the policy index of each legal move as
 * the evaluator computes it (NN::MoveToNNIndex of the move, mirrored for
 * black, with the encoder's transform); an index outside [0, 1858) counts as
 * logit 0. priors [move_offsets[batch] - move_offsets[0]] receives, per
 * position, FastExp((logit - max) / softmax_temp) normalised over its first
 * min(n, 256) moves (uniform if the sum is not positive; moves past the
 * 256th get 0), bit-identical to the reference's float arithmetic. wdl / moves_left as
 * in mfb200_evaluate (either may be NULL). softmax_temp must be > 0; at most
 * 256 moves per position on average. Blocks until the results are in host
 * memory. */
MFB200_API int mfb200_evaluate_priors(mfb200_handle *h, const uint64_t *masks, const float *values,
                                      int batch, const int32_t *move_offsets,
                                      const int16_t *move_index, float softmax_temp,
                                      float *priors, float *wdl, float *moves_left,
                                      mfb200_timing *timing);

/* One position of a game history, as the encoder reads it from a Position
 * (src/core/position.h): bit i of a bitboard is square i (a1 = 0, h8 = 63). */
typedef struct mfb200_board {
  uint64_t pieces[2][6]; /* [white, black][pawn, knight, bishop, rook, queen, king] */
  int32_t rule50;        /* Position::rule50_count() */
  int32_t game_ply;      /* Position::game_ply() */
  int8_t ep_square;      /* Position::ep_square(), -1 for SQ_NONE */
  uint8_t castling;      /* bit 0 white O-O, 1 white O-O-O, 2 black O-O, 3 black O-O-O */
  uint8_t black_to_move; /* Position::side_to_move() == BLACK */
  uint8_t repetition;    /* Position::is_repetition(INT_MAX) */
  uint32_t reserved;     /* 0 */
} mfb200_board;

/* Input formats (MetalFishNN::NetworkFormat::InputFormat, src/nn/proto/net.proto:256-263). */
enum {
  MFB200_INPUT_CLASSICAL_112 = 1,
  MFB200_INPUT_112_WITH_CASTLING_PLANE = 2,
  MFB200_INPUT_112_CANONICAL = 3,
  MFB200_INPUT_112_CANONICAL_HECTOPLIES = 4,
  MFB200_INPUT_112_CANONICAL_V2 = 5,
  MFB200_INPUT_112_CANONICAL_HECTOPLIES_ARMAGEDDON = 132,
  MFB200_INPUT_112_CANONICAL_V2_ARMAGEDDON = 133
};

/* Encode `batch` game histories on the GPU as EncodePositionForNN(format,
 * history, 8 planes, FillEmptyHistory::FEN_ONLY) does, into the packed planes
 * of PackInputPlanesRaw: boards is a CSR over history_offsets [batch + 1],
 * each history oldest first and ending with the position to evaluate (pass at
 * least the plies since the last capture or pawn move; the whole game is
 * fine). Writes masks / values [batch, 112] and the canonicalisation
 * transform of each position (transforms [batch], for NN::MoveToNNIndex),
 * each output optional. Where the reference would extend an empty history
 * forever (a FEN history of one non-start position with a nonzero rule50 in
 * the V2 formats) the GPU stops after 8 synthesised entries. */
MFB200_API int mfb200_encode_history(mfb200_handle *h, const mfb200_board *boards,
                                     const int32_t *history_offsets, int batch, int input_format,
                                     uint64_t *masks, float *values, int32_t *transforms);

/* mfb200_evaluate with the encoding on the GPU: histories in (as in
 * mfb200_encode_history), policy / wdl / moves_left / transforms out. */
MFB200_API int mfb200_evaluate_history(mfb200_handle *h, const mfb200_board *boards,
                                       const int32_t *history_offsets, int batch,
                                       int input_format, float *policy, float *wdl,
                                       float *moves_left, int32_t *transforms,
                                       mfb200_timing *timing);

/* The whole MCTS leaf evaluation on the GPU: game histories in (as in
 * mfb200_encode_history), the legal moves of each position as
 * from | to << 6 | promotion << 12 (squares 0..63 a1..h8; promotion 0 none,
 * 1 queen, 2 rook, 3 bishop, 4 knight; castling as the king's from and the
 * to square Move::to_sq() gives) in a CSR over move_offsets [batch + 1];
 * priors / wdl / moves_left out as in mfb200_evaluate_priors. Each move is
 * mapped to its policy index on the device exactly as the evaluator does
 * (mirror for black, NN::MoveToNNIndex with the encoder's transform). */
MFB200_API int mfb200_evaluate_leaves(mfb200_handle *h, const mfb200_board *boards,
                                      const int32_t *history_offsets, int batch, int input_format,
                                      const uint16_t *moves, const int32_t *move_offsets,
                                      float softmax_temp, float *priors, float *wdl,
                                      float *moves_left, mfb200_timing *timing);

/* Asynchronous mfb200_evaluate_leaves, for MCTS batch assembly that keeps
 * building the next batch while the GPU works: enqueues the whole leaf
 * evaluation and returns at once with a ticket. The caller's input and
 * output buffers must stay valid (and unchanged) until mfb200_wait(ticket)
 * returns; page-locked buffers make the copies asynchronous. At most 4
 * submissions are in flight per handle (a fifth waits for the oldest).
 * Submissions on one handle run in order, pipelined on three streams per GPU:
 * the input copies of submission i+1 and the output copies of submission i-1
 * overlap the GPU work of submission i. */
MFB200_API int mfb200_submit_leaves(mfb200_handle *h, const mfb200_board *boards,
                                    const int32_t *history_offsets, int batch, int input_format,
                                    const uint16_t *moves, const int32_t *move_offsets,
                                    float softmax_temp, float *priors, float *wdl,
                                    float *moves_left, uint64_t *ticket);

/* Blocks until submission `ticket` has completed (its outputs are in the
 * caller's buffers) and reports a device error that submission met (the
 * error stays with its ticket, also when a later submission had to wait for
 * it to free its slot). Returns 0 for a ticket that completed without error. */
MFB200_API int mfb200_wait(mfb200_handle *h, uint64_t ticket);

/* NN::MoveToNNIndex (src/nn/policy_map.cpp:316-360) as this library maps
 * moves: out [8 transforms][5 promotion kinds][64 from][64 to], -1 for no
 * index. Host only (no GPU needed). Returns 0. */
MFB200_API int mfb200_policy_index_table(int16_t *out);

/* Device-buffer evaluation on device `cfg.device`, enqueued on `stream`
 * (a cudaStream_t; NULL = the handle's stream) without synchronising. All
 * pointers are device pointers of that device. */
MFB200_API int mfb200_evaluate_device(mfb200_handle *h, const uint64_t *d_masks, const float *d_values,
                           int batch, float *d_policy, float *d_wdl, float *d_moves_left,
                           void *stream);

/* FP8 / INT8 handles only: set the per-tensor activation scales from the absmax of
 * a bf16 forward over `count` calibration positions (host buffers). Must be
 * called before the first FP8 evaluation. */
MFB200_API int mfb200_calibrate(mfb200_handle *h, const uint64_t *masks, const float *values, int count);

MFB200_API int mfb200_capabilities(mfb200_handle *h, mfb200_caps *caps);

/* Per-stage device time of one eager forward at `batch` (inputs already on
 * the device), for profiling: writes up to `max_stages` entries of ms and
 * algorithmic FLOPs, and stage names separated by '\n' into `names`.
 * Returns the number of stages, or a negative value on error. */
MFB200_API int mfb200_profile(mfb200_handle *h, int batch, int iters, float *stage_ms, double *stage_flops,
                   char *names, size_t names_len, int max_stages);

MFB200_API const char *mfb200_last_error(mfb200_handle *h);

/* For callers that cannot allocate GPU memory -- code running inside another
 * framework's memory pool, or a search thread that must not take the
 * driver's allocation locks or meet an out-of-memory error mid-game. No
 * counterpart in the reference. Computes d_out[M,N] (fp32) = d_A[M,K] .
 * d_W[N,K]^T + d_bias (bf16 operands, bias may be NULL) with the tcgen05 GEMM
 * split into k_splits slices along K, enqueued on `stream` (a cudaStream_t,
 * NULL = legacy default stream). It calls no cudaMalloc/cudaFree: the partial
 * products live in one fixed 8 MiB device array that every GPU loading the
 * library holds until exit, so k_splits*M*N may not exceed 2,097,088 (larger
 * requests return an error). The first call on a device resolves that
 * array's address (cudaGetSymbolAddress); make it before any stream capture.
 * All calls on a device share the array: calls that overlap on the GPU (other
 * streams, other threads) race and must be serialised by the caller. Every
 * partial the reduction reads is written by the same call; the one word that
 * must start at zero (a timeout status flag) is cleared by each call. If a
 * barrier wait inside the GEMM timed out (the kernel gives up after 2 s
 * instead of hanging), every element of d_out is set to NaN, so an
 * incomplete result is never mistaken for a valid one. Requires N % 32 == 0
 * and K % 8 == 0. Returns 0 on success; mfb200_noalloc_last_error() gives the
 * calling thread's last message. */
MFB200_API int mfb200_splitk_gemm_noalloc(const void *d_A, const void *d_W, int M, int N, int K,
                                          int k_splits, const float *d_bias, float *d_out,
                                          void *stream);
MFB200_API const char *mfb200_noalloc_last_error(void);
MFB200_API void mfb200_destroy(mfb200_handle *h);

#ifdef __cplusplus
}
#endif
#endif /* MFB200_H */
