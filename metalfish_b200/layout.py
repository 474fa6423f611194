"""Tensor-slot tables shared by the weight packer and the test oracle.

Each slot names one tensor of the reference weight schema
(``src/nn/proto/net.proto``). The orders below are the C enum orders of the
oracle (``G_*`` / ``L_*``) and of the packed weight directory of the CUDA
library (``metalfish_b200/csrc/mfb200_internal.h``).
"""
GLOBAL_SLOTS = [
    "ip_emb_preproc_w", "ip_emb_preproc_b", "ip_emb_w", "ip_emb_b",
    "ip_emb_ln_gammas", "ip_emb_ln_betas", "ip_mult_gate", "ip_add_gate",
    "ip_emb_ffn.dense1_w", "ip_emb_ffn.dense1_b", "ip_emb_ffn.dense2_w", "ip_emb_ffn.dense2_b",
    "ip_emb_ffn_ln_gammas", "ip_emb_ffn_ln_betas", "smolgen_w",
    "policy_heads.vanilla.ip_pol_w", "policy_heads.vanilla.ip_pol_b",
    "policy_heads.vanilla.ip2_pol_w", "policy_heads.vanilla.ip2_pol_b",
    "policy_heads.vanilla.ip3_pol_w", "policy_heads.vanilla.ip3_pol_b",
    "policy_heads.vanilla.ip4_pol_w",
    "value_heads.winner.ip_val_w", "value_heads.winner.ip_val_b",
    "value_heads.winner.ip1_val_w", "value_heads.winner.ip1_val_b",
    "value_heads.winner.ip2_val_w", "value_heads.winner.ip2_val_b",
    "ip_mov_w", "ip_mov_b", "ip1_mov_w", "ip1_mov_b", "ip2_mov_w", "ip2_mov_b",
]
LAYER_SLOTS = [
    "mha.q_w", "mha.q_b", "mha.k_w", "mha.k_b", "mha.v_w", "mha.v_b", "mha.dense_w", "mha.dense_b",
    "mha.smolgen.compress", "mha.smolgen.dense1_w", "mha.smolgen.dense1_b",
    "mha.smolgen.ln1_gammas", "mha.smolgen.ln1_betas", "mha.smolgen.dense2_w",
    "mha.smolgen.dense2_b", "mha.smolgen.ln2_gammas", "mha.smolgen.ln2_betas",
    "ln1_gammas", "ln1_betas", "ffn.dense1_w", "ffn.dense1_b", "ffn.dense2_w", "ffn.dense2_b",
    "ln2_gammas", "ln2_betas",
]
# activation codes (oracle ACT_* enum and the CUDA epilogue Act enum)
ACTIVATIONS = {"none": 0, "relu": 1, "relu_2": 2, "tanh": 3, "sigmoid": 4, "swish": 5,
               "mish": 6, "selu": 7}


def layer_name(i: int, slot: str) -> str:
    return f"encoder.{i}.{slot}"
