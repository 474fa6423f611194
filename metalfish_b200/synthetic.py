"""Seeded synthetic attention-body networks of the BT4 family.

The real ``BT4-1024x15x32h-swa-6147500.pb`` is not available here, so every
measurement and parity check runs on random-init weights of the same
architecture: weights ~ N(0, 1/fan_in), LayerNorm gamma = 1 and beta = 0.
Biases are small N(0, 0.02^2) so the bias path is exercised, and the input
gates are perturbed around (mult = 1, add = 0) so the channel-major gate
layout (``src/nn/cpu/cpu_network.cpp:1268-1316``) is exercised too.
``perturb_norms=True`` additionally perturbs every LN gamma/beta (used by the
parity tests, so a gamma/beta indexing bug cannot hide behind gamma = 1).

Tensor names/shapes follow the reference schema (``src/nn/proto/net.proto``)
and its ``[out, in]`` dense convention; the step order and the per-stage
semantics they feed are those of ``src/nn/network_execution_plan.cpp:155-223``.
"""
from __future__ import annotations

from dataclasses import dataclass, asdict, replace
from typing import Dict

import numpy as np


@dataclass(frozen=True)
class NetConfig:
    name: str
    embedding: int          # d
    layers: int             # encoder layers
    heads: int              # H (head depth = d / H)
    dff: int                # encoder FFN hidden
    emb_dff: int            # input-embedding FFN hidden
    pe: int = 64            # dynamic PE width per square
    smolgen_compress: int = 32
    smolgen_hidden: int = 256
    smolgen_gen: int = 256  # per-head generator width
    policy_d: int = 0       # attention-policy embedding (0 -> d)
    value_emb: int = 32
    value_hidden: int = 128
    mlh_emb: int = 8
    mlh_hidden: int = 128
    default_activation: str = "mish"
    smolgen_activation: str = "swish"
    ffn_activation: str = "relu_2"

    @property
    def dp(self) -> int:
        return self.policy_d or self.embedding

    @property
    def head_depth(self) -> int:
        return self.embedding // self.heads

    def header(self) -> Dict[str, str]:
        return {"heads": str(self.heads), "default_activation": self.default_activation,
                "smolgen_activation": self.smolgen_activation,
                "ffn_activation": self.ffn_activation, "config": self.name}

    def flops_per_position(self) -> Dict[str, float]:
        """2 x multiply-accumulates per position, from the tensor dims."""
        d, T = self.embedding, 64
        enc_gemm = T * (4 * d * d + 2 * d * self.dff)
        attn = 2 * T * T * d
        smol = (T * d * self.smolgen_compress + T * self.smolgen_compress * self.smolgen_hidden
                + self.smolgen_hidden * self.heads * self.smolgen_gen
                + self.heads * self.smolgen_gen * T * T)
        emb = 768 * T * self.pe + T * (112 + self.pe) * d + 2 * T * d * self.emb_dff
        pol = T * (d * self.dp + 2 * self.dp * self.dp) + T * T * self.dp
        val = (T * d * self.value_emb + T * self.value_emb * self.value_hidden + self.value_hidden * 3
               + T * d * self.mlh_emb + T * self.mlh_emb * self.mlh_hidden + self.mlh_hidden)
        total = self.layers * (enc_gemm + attn + smol) + emb + pol + val
        return {"encoder_gemm_flops": 2.0 * self.layers * enc_gemm, "total_flops": 2.0 * total}


# config 0 of the benchmark plan: small net on the reference CPU backend
SMALL = NetConfig("small-256x6x8h", embedding=256, layers=6, heads=8, dff=256, emb_dff=256)
# configs 1-4: BT4-shaped
BT4 = NetConfig("bt4-1024x15x32h", embedding=1024, layers=15, heads=32, dff=1536, emb_dff=1536)
# a tiny net for fast unit tests (2 layers)
TINY = NetConfig("tiny-128x2x4h", embedding=128, layers=2, heads=4, dff=128, emb_dff=128)

CONFIGS = {c.name: c for c in (SMALL, BT4, TINY)}


def generate(cfg: NetConfig, seed: int = 0, perturb_norms: bool = False) -> Dict[str, np.ndarray]:
    """Generate a seeded synthetic network (fp32 arrays keyed by schema path)."""
    rng = np.random.default_rng(seed)
    t: Dict[str, np.ndarray] = {}
    d, T = cfg.embedding, 64

    def w(name, out_f, in_f):
        t[name] = (rng.standard_normal((out_f, in_f), dtype=np.float32)
                   * np.float32(1.0 / np.sqrt(in_f)))

    def b(name, n):
        t[name] = rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)

    def ln(prefix, n):
        if perturb_norms:
            t[prefix + "_gammas"] = np.float32(1) + np.float32(0.1) * rng.standard_normal(n, dtype=np.float32)
            t[prefix + "_betas"] = np.float32(0.1) * rng.standard_normal(n, dtype=np.float32)
        else:
            t[prefix + "_gammas"] = np.ones(n, np.float32)
            t[prefix + "_betas"] = np.zeros(n, np.float32)

    w("ip_emb_preproc_w", T * cfg.pe, 12 * T)
    b("ip_emb_preproc_b", T * cfg.pe)
    w("ip_emb_w", d, 112 + cfg.pe)
    b("ip_emb_b", d)
    ln("ip_emb_ln", d)
    # gates are channel-major [d][64] (cpu_network.cpp:1290-1296)
    t["ip_mult_gate"] = (np.float32(1) + np.float32(0.1) * rng.standard_normal((d, T), dtype=np.float32))
    t["ip_add_gate"] = np.float32(0.1) * rng.standard_normal((d, T), dtype=np.float32)
    w("ip_emb_ffn.dense1_w", cfg.emb_dff, d)
    b("ip_emb_ffn.dense1_b", cfg.emb_dff)
    w("ip_emb_ffn.dense2_w", d, cfg.emb_dff)
    b("ip_emb_ffn.dense2_b", d)
    ln("ip_emb_ffn_ln", d)
    # shared smolgen generator [64*64, gen]
    w("smolgen_w", T * T, cfg.smolgen_gen)
    for i in range(cfg.layers):
        p = f"encoder.{i}."
        for n in ("q", "k", "v"):
            w(p + f"mha.{n}_w", d, d)
            b(p + f"mha.{n}_b", d)
        w(p + "mha.dense_w", d, d)
        b(p + "mha.dense_b", d)
        s = p + "mha.smolgen."
        w(s + "compress", cfg.smolgen_compress, d)
        w(s + "dense1_w", cfg.smolgen_hidden, T * cfg.smolgen_compress)
        b(s + "dense1_b", cfg.smolgen_hidden)
        ln(s + "ln1", cfg.smolgen_hidden)
        w(s + "dense2_w", cfg.heads * cfg.smolgen_gen, cfg.smolgen_hidden)
        b(s + "dense2_b", cfg.heads * cfg.smolgen_gen)
        ln(s + "ln2", cfg.heads * cfg.smolgen_gen)
        ln(p + "ln1", d)
        w(p + "ffn.dense1_w", cfg.dff, d)
        b(p + "ffn.dense1_b", cfg.dff)
        w(p + "ffn.dense2_w", d, cfg.dff)
        b(p + "ffn.dense2_b", d)
        ln(p + "ln2", d)
    pp = "policy_heads.vanilla."
    w(pp + "ip_pol_w", cfg.dp, d)
    b(pp + "ip_pol_b", cfg.dp)
    w(pp + "ip2_pol_w", cfg.dp, cfg.dp)
    b(pp + "ip2_pol_b", cfg.dp)
    w(pp + "ip3_pol_w", cfg.dp, cfg.dp)
    b(pp + "ip3_pol_b", cfg.dp)
    w(pp + "ip4_pol_w", 4, cfg.dp)
    vp = "value_heads.winner."
    w(vp + "ip_val_w", cfg.value_emb, d)
    b(vp + "ip_val_b", cfg.value_emb)
    w(vp + "ip1_val_w", cfg.value_hidden, T * cfg.value_emb)
    b(vp + "ip1_val_b", cfg.value_hidden)
    w(vp + "ip2_val_w", 3, cfg.value_hidden)
    b(vp + "ip2_val_b", 3)
    w("ip_mov_w", cfg.mlh_emb, d)
    b("ip_mov_b", cfg.mlh_emb)
    w("ip1_mov_w", cfg.mlh_hidden, T * cfg.mlh_emb)
    b("ip1_mov_b", cfg.mlh_hidden)
    w("ip2_mov_w", 1, cfg.mlh_hidden)
    b("ip2_mov_b", 1)
    # smolgen global LN weights and the ip_emb LN are in the plan; nothing else.
    # The layer-norm gammas are stored flat; reshape the 2D gates to flat too
    t["ip_mult_gate"] = t["ip_mult_gate"].reshape(-1)
    t["ip_add_gate"] = t["ip_add_gate"].reshape(-1)
    return t


def config_from_header(header: Dict[str, str]) -> NetConfig:
    return CONFIGS[header["config"]]
