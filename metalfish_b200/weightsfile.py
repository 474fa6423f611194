"""Reader of MetalFish's protobuf weight files (``.pb`` / ``.pb.gz``) for the
Python mirror of the B200 backend.

The engine's C++ side loads weights with the reference's own loader
(``src/nn/loader.cpp:156-175`` ``LoadWeightsFromFile``) and the C++ backend
(``host/b200_network.cpp``) decodes them with ``MultiHeadWeights``. This module
is the same path for Python users: it reads the protobuf wire format of
``src/nn/proto/net.proto`` directly (no protoc-generated code), decodes every
``Weights.Layer`` as ``src/nn/loader.cpp:181-250`` ``DecodeLayer`` does, maps
the legacy single-head fields onto the vanilla policy / winner value heads as
``src/nn/weights.cpp:214-290`` does, infers the network shape from the tensor
sizes and returns ``(NetConfig, tensors)`` ready for ``create_network``.

The field numbers below restate the schema's (they must be equal to read real
files); only the messages the attention-body path reads are listed.
"""
from __future__ import annotations

import gzip
import struct
from typing import Dict, List, Optional, Tuple

import numpy as np

from .synthetic import NetConfig

WEIGHT_MAGIC = 0x1C0  # src/nn/loader.cpp:34

# Weights.Layer.Encoding
UNKNOWN_ENCODING, LINEAR16, FLOAT16, BFLOAT16, FLOAT32 = 0, 1, 2, 3, 4

# schema: message -> {field number: (name, kind)}; kind "layer" (a
# Weights.Layer: min_val 1 float, max_val 2 float, params 3 bytes, encoding 4
# enum), "msg:<Message>", "rmsg:<Message>" (repeated), "u32" (varint), "fx32"
# (fixed32)
_L = "layer"
SCHEMA: Dict[str, Dict[int, Tuple[str, str]]] = {
    "Net": {1: ("magic", "fx32"), 4: ("format", "msg:Format"), 10: ("weights", "msg:Weights")},
    "Format": {2: ("network_format", "msg:NetworkFormat")},
    "NetworkFormat": {1: ("input", "u32"), 2: ("output", "u32"), 3: ("network", "u32"),
                      4: ("policy", "u32"), 5: ("value", "u32"), 6: ("moves_left", "u32"),
                      7: ("default_activation", "u32"), 8: ("smolgen_activation", "u32"),
                      9: ("ffn_activation", "u32"), 10: ("input_embedding", "u32")},
    "Weights": {37: ("ip_emb_preproc_w", _L), 38: ("ip_emb_preproc_b", _L),
                25: ("ip_emb_w", _L), 26: ("ip_emb_b", _L),
                39: ("ip_emb_ln_gammas", _L), 40: ("ip_emb_ln_betas", _L),
                33: ("ip_mult_gate", _L), 34: ("ip_add_gate", _L),
                41: ("ip_emb_ffn", "msg:FFN"), 42: ("ip_emb_ffn_ln_gammas", _L),
                43: ("ip_emb_ffn_ln_betas", _L), 27: ("encoder", "rmsg:EncoderLayer"),
                28: ("headcount", "u32"), 4: ("ip_pol_w", _L), 5: ("ip_pol_b", _L),
                17: ("ip2_pol_w", _L), 18: ("ip2_pol_b", _L), 19: ("ip3_pol_w", _L),
                20: ("ip3_pol_b", _L), 22: ("ip4_pol_w", _L), 29: ("ip_val_w", _L),
                30: ("ip_val_b", _L), 7: ("ip1_val_w", _L), 8: ("ip1_val_b", _L),
                9: ("ip2_val_w", _L), 10: ("ip2_val_b", _L),
                44: ("value_heads", "msg:ValueHeads"), 45: ("policy_heads", "msg:PolicyHeads"),
                31: ("ip_mov_w", _L), 32: ("ip_mov_b", _L), 13: ("ip1_mov_w", _L),
                14: ("ip1_mov_b", _L), 15: ("ip2_mov_w", _L), 16: ("ip2_mov_b", _L),
                35: ("smolgen_w", _L), 36: ("smolgen_b", _L),
                21: ("pol_encoder", "rmsg:EncoderLayer")},
    "EncoderLayer": {1: ("mha", "msg:MHA"), 2: ("ln1_gammas", _L), 3: ("ln1_betas", _L),
                     4: ("ffn", "msg:FFN"), 5: ("ln2_gammas", _L), 6: ("ln2_betas", _L)},
    "MHA": {1: ("q_w", _L), 2: ("q_b", _L), 3: ("k_w", _L), 4: ("k_b", _L), 5: ("v_w", _L),
            6: ("v_b", _L), 7: ("dense_w", _L), 8: ("dense_b", _L),
            9: ("smolgen", "msg:Smolgen"), 10: ("rpe_q", _L), 11: ("rpe_k", _L),
            12: ("rpe_v", _L)},
    "Smolgen": {1: ("compress", _L), 2: ("dense1_w", _L), 3: ("dense1_b", _L),
                4: ("ln1_gammas", _L), 5: ("ln1_betas", _L), 6: ("dense2_w", _L),
                7: ("dense2_b", _L), 8: ("ln2_gammas", _L), 9: ("ln2_betas", _L)},
    "FFN": {1: ("dense1_w", _L), 2: ("dense1_b", _L), 3: ("dense2_w", _L), 4: ("dense2_b", _L)},
    "PolicyHeads": {1: ("ip_pol_w", _L), 2: ("ip_pol_b", _L), 3: ("vanilla", "msg:PolicyHead")},
    "PolicyHead": {1: ("ip_pol_w", _L), 2: ("ip_pol_b", _L), 3: ("ip2_pol_w", _L),
                   4: ("ip2_pol_b", _L), 5: ("ip3_pol_w", _L), 6: ("ip3_pol_b", _L),
                   7: ("ip4_pol_w", _L), 8: ("pol_encoder", "rmsg:EncoderLayer")},
    "ValueHeads": {1: ("winner", "msg:ValueHead")},
    "ValueHead": {1: ("ip_val_w", _L), 2: ("ip_val_b", _L), 3: ("ip1_val_w", _L),
                  4: ("ip1_val_b", _L), 5: ("ip2_val_w", _L), 6: ("ip2_val_b", _L)},
}

# NetworkFormat.ActivationFunction -> name, as ActivationToString
# (src/nn/network_format.cpp:50-70): every other value (NONE, SOFTMAX,
# DEFAULT) reads "relu"
_ACT = {1: "mish", 2: "relu", 4: "tanh", 5: "sigmoid", 6: "selu", 7: "swish", 8: "relu_2"}

# NetworkFormat enum values used below
_NET_CLASSICAL, _NET_SE, _NET_CLASSICAL_HF, _NET_SE_HF = 1, 2, 3, 4
_NET_AB_HF, _NET_AB_MHF, _NET_AB_LEGACY_MHF = 6, 7, 134
_POLICY_ATTENTION, _VALUE_WDL, _MOVES_LEFT_V1 = 3, 2, 1
_EMB_PE_MAP, _EMB_PE_DENSE = 1, 2


def _varint(buf: bytes, pos: int) -> Tuple[int, int]:
    result = shift = 0
    while True:
        if pos >= len(buf):
            raise RuntimeError("Failed to parse protobuf weights file: truncated varint")
        b = buf[pos]
        pos += 1
        result |= (b & 0x7F) << shift
        if not b & 0x80:
            return result, pos
        shift += 7
        if shift > 63:
            raise RuntimeError("Failed to parse protobuf weights file: bad varint")


def _fields(buf: bytes, pos: int, end: int):
    """Yields (field number, wire type, value) of the message in buf[pos:end];
    value is an int (varint, fixed32, fixed64) or, for length-delimited
    fields, the (start, end) offsets of the payload in `buf`."""
    while pos < end:
        key, pos = _varint(buf, pos)
        num, wt = key >> 3, key & 7
        if wt == 0:
            v, pos = _varint(buf, pos)
        elif wt == 1:
            if pos + 8 > end:
                raise RuntimeError("Failed to parse protobuf weights file: truncated fixed64")
            v = struct.unpack_from("<Q", buf, pos)[0]
            pos += 8
        elif wt == 2:
            ln, pos = _varint(buf, pos)
            if pos + ln > end:
                raise RuntimeError("Failed to parse protobuf weights file: truncated field")
            v = (pos, pos + ln)
            pos += ln
        elif wt == 5:
            if pos + 4 > end:
                raise RuntimeError("Failed to parse protobuf weights file: truncated fixed32")
            v = struct.unpack_from("<I", buf, pos)[0]
            pos += 4
        else:
            raise RuntimeError(f"Failed to parse protobuf weights file: wire type {wt}")
        yield num, wt, v


def decode_layer(min_val: float, max_val: float, params: bytes, encoding: int) -> np.ndarray:
    """``DecodeLayer`` (``src/nn/loader.cpp:181-250``): LINEAR16 is
    min + raw/65535 * (max - min) in fp32, FLOAT16 and BFLOAT16 widen exactly,
    FLOAT32 is copied; a missing encoding means LINEAR16."""
    if encoding == UNKNOWN_ENCODING:
        encoding = LINEAR16
    if encoding == FLOAT32:
        return np.frombuffer(params, dtype="<f4", count=len(params) // 4).astype(np.float32)
    if encoding not in (LINEAR16, FLOAT16, BFLOAT16):
        raise RuntimeError("Unsupported weight encoding")
    raw = np.frombuffer(params, dtype="<u2", count=len(params) // 2)
    if encoding == FLOAT16:
        return raw.view(np.float16).astype(np.float32)
    if encoding == BFLOAT16:
        return (raw.astype(np.uint32) << 16).view(np.float32)
    lo, hi = np.float32(min_val), np.float32(max_val)
    return lo + (raw.astype(np.float32) / np.float32(65535.0)) * (hi - lo)


def _parse(buf: bytes, pos: int, end: int, msg: str, prefix: str,
           tensors: Dict[str, np.ndarray], scalars: Dict[str, int]) -> None:
    table = SCHEMA[msg]
    counts: Dict[int, int] = {}
    for num, wt, v in _fields(buf, pos, end):
        if num not in table:
            continue  # fields the attention-body path does not read
        name, kind = table[num]
        path = prefix + name
        if kind in ("u32", "fx32"):
            if wt not in (0, 5):
                raise RuntimeError(f"Failed to parse protobuf weights file: {path}")
            scalars[path] = int(v)
            continue
        if wt != 2:
            raise RuntimeError(f"Failed to parse protobuf weights file: {path} is not a message")
        if kind == _L:
            lo = hi = 0.0
            params = b""
            enc = UNKNOWN_ENCODING
            for lnum, lwt, lv in _fields(buf, v[0], v[1]):
                if lnum == 1 and lwt == 5:
                    lo = struct.unpack("<f", struct.pack("<I", lv))[0]
                elif lnum == 2 and lwt == 5:
                    hi = struct.unpack("<f", struct.pack("<I", lv))[0]
                elif lnum == 3 and lwt == 2:
                    params = buf[lv[0]:lv[1]]
                elif lnum == 4 and lwt == 0:
                    enc = lv
            tensors[path] = decode_layer(lo, hi, params, enc)
        elif kind.startswith("msg:"):
            _parse(buf, v[0], v[1], kind[4:], path + ".", tensors, scalars)
        else:  # rmsg: repeated message, indexed in file order
            i = counts.get(num, 0)
            counts[num] = i + 1
            _parse(buf, v[0], v[1], kind[5:], f"{path}.{i}.", tensors, scalars)


def _read_bytes(path: str) -> bytes:
    # src/nn/loader.cpp:156-175: a ".gz" suffix means gzip
    if path.endswith(".gz"):
        with gzip.open(path, "rb") as f:
            data = f.read()
    else:
        with open(path, "rb") as f:
            data = f.read()
    if len(data) < 2:
        raise RuntimeError("Invalid weight file: too small")
    return data


def parse_weights(data: bytes) -> Tuple[Dict[str, np.ndarray], Dict[str, int]]:
    """All Weights.Layer tensors (keyed by schema path, ``encoder.3.mha.q_w``)
    and the scalar fields (``weights.headcount``, ``format.network_format.*``)
    of one serialised ``Net``."""
    tensors: Dict[str, np.ndarray] = {}
    scalars: Dict[str, int] = {}
    _parse(data, 0, len(data), "Net", "", tensors, scalars)
    if scalars.get("magic") != WEIGHT_MAGIC:
        raise RuntimeError("Invalid weight file: bad magic number")
    return {k[len("weights."):]: v for k, v in tensors.items() if k.startswith("weights.")}, scalars


def _heads(t: Dict[str, np.ndarray]) -> Dict[str, np.ndarray]:
    """The vanilla policy head and winner value head as ``MultiHeadWeights``
    resolves them (``src/nn/weights.cpp:214-290``): the policy embedding comes
    from the head, else ``policy_heads.ip_pol_w``, else the legacy top-level
    ``ip_pol_w``; without ``policy_heads`` / ``value_heads`` the legacy
    top-level fields are the vanilla / winner heads."""
    out = dict(t)
    pv = "policy_heads.vanilla."
    has_policy_heads = any(k.startswith("policy_heads.") for k in t)
    for n in ("w", "b"):
        key = f"ip_pol_{n}"
        if pv + key not in out:
            src = t.get(f"policy_heads.{key}", t.get(key))
            if src is not None:
                out[pv + key] = src
    if not has_policy_heads:
        for key in ("ip2_pol_w", "ip2_pol_b", "ip3_pol_w", "ip3_pol_b", "ip4_pol_w"):
            if key in t:
                out[pv + key] = t[key]
    vw = "value_heads.winner."
    if not any(k.startswith("value_heads.") for k in t):
        for key in ("ip_val_w", "ip_val_b", "ip1_val_w", "ip1_val_b", "ip2_val_w", "ip2_val_b"):
            if key in t:
                out[vw + key] = t[key]
    return out


def _activation(code: int, default: str) -> str:
    # src/nn/network_format.cpp:108-123: ACTIVATION_DEFAULT takes the default
    if code == 0:
        return default
    return _ACT.get(code, "relu")


def fix_older_format(scalars: Dict[str, int], t: Dict[str, np.ndarray]) -> Dict[str, int]:
    """``FixOlderWeightsFile`` (``src/nn/loader.cpp:87-133``) on the
    NetworkFormat fields (``format.network_format.*``; a missing field is
    absent from `scalars`). Returns the fixed fields by bare name."""
    nfp = "format.network_format."
    has_nf = any(k.startswith(nfp) for k in scalars)
    f = {k[len(nfp):]: v for k, v in scalars.items() if k.startswith(nfp)}
    if not has_nf:
        f.update(input=1, output=1, network=_NET_CLASSICAL_HF, value=1, policy=1)
    net = f.get("network", 0)
    has_encoder = any(k.startswith("encoder.") for k in t)
    if net == _NET_CLASSICAL:
        f.update(network=_NET_CLASSICAL_HF, value=1, policy=1)
    elif net == _NET_SE:
        f.update(network=_NET_SE_HF, value=1, policy=1)
    elif net == _NET_SE_HF and has_encoder:
        f["network"] = _NET_AB_HF
        if "smolgen_w" in t:
            f.update(ffn_activation=8, smolgen_activation=7)  # RELU_2, SWISH
    elif net == _NET_AB_LEGACY_MHF:
        f["network"] = _NET_AB_MHF
    if f.get("network") == _NET_AB_HF:
        if (any(k.startswith("policy_heads.") for k in t)
                and any(k.startswith("value_heads.") for k in t)):
            f.update(network=_NET_AB_MHF, input_embedding=_EMB_PE_DENSE)
        if "input_embedding" not in f:
            f["input_embedding"] = _EMB_PE_MAP
    return f


def _require(ok: bool, what: str) -> None:
    if not ok:
        raise RuntimeError("B200 backend does not support this network: " + what)


def config_from_weights(t: Dict[str, np.ndarray], scalars: Dict[str, int],
                        fmt: Dict[str, int], has_policy_heads: bool,
                        name: str = "pb") -> NetConfig:
    """The network shape from the tensor sizes (the C++ backend infers it the
    same way); raises RuntimeError for anything but the attention body with
    PE_DENSE embedding, smolgen, attention policy, WDL and moves-left heads.
    `t` holds the resolved head tensors (``_heads``), `fmt` the fixed-up
    NetworkFormat (``fix_older_format`` of the file as read)."""
    def need(key: str) -> np.ndarray:
        if key not in t:
            raise RuntimeError(f"B200 backend: weight file lacks {key} (attention body with "
                               "PE_DENSE embedding, smolgen, attention policy, WDL and "
                               "moves-left heads required)")
        return t[key]

    # the checks of the C++ backend (host/b200_network.cpp DescribeNet) on
    # DescribeNetworkFormat (src/nn/network_format.cpp:73-125)
    f = fmt
    _require(f.get("network") in (_NET_AB_HF, _NET_AB_MHF), "not an attention-body network")
    _require(f.get("policy") == _POLICY_ATTENTION, "policy head is not attention policy")
    _require(f.get("value") == _VALUE_WDL and f.get("moves_left") == _MOVES_LEFT_V1,
             "needs WDL value and moves-left heads")
    _require(f.get("input_embedding", _EMB_PE_MAP) == _EMB_PE_DENSE,
             "input embedding is not PE_DENSE")
    _require(not any(k.startswith("policy_heads.vanilla.pol_encoder.") for k in t)
             and (has_policy_heads or not any(k.startswith("pol_encoder.") for k in t)),
             "policy-head encoder layers")
    layers = 0
    while f"encoder.{layers}.mha.q_w" in t:
        layers += 1
    _require(layers > 0, "no encoder layers")
    _require("encoder.0.mha.smolgen.compress" in t and t.get("smolgen_w", np.zeros(0)).size > 0,
             "encoder without smolgen")
    heads = int(scalars.get("weights.headcount", 0))
    if heads <= 0:
        raise RuntimeError("B200 backend: weight file has no encoder head count")
    d = need("ip_emb_b").size
    pe = need("ip_emb_preproc_b").size // 64
    sg = "encoder.0.mha.smolgen."
    hidden_x_heads = need(sg + "dense2_b").size
    default = "mish" if f.get("default_activation", 0) == 1 else "relu"
    cfg = NetConfig(
        name=name, embedding=d, layers=layers, heads=heads,
        dff=need("encoder.0.ffn.dense1_b").size, emb_dff=need("ip_emb_ffn.dense1_b").size,
        pe=pe, smolgen_compress=need(sg + "compress").size // d,
        smolgen_hidden=need(sg + "dense1_b").size, smolgen_gen=hidden_x_heads // heads,
        policy_d=need("policy_heads.vanilla.ip_pol_b").size,
        value_emb=need("value_heads.winner.ip_val_b").size,
        value_hidden=need("value_heads.winner.ip1_val_b").size,
        mlh_emb=need("ip_mov_b").size, mlh_hidden=need("ip1_mov_b").size,
        default_activation=default,
        smolgen_activation=_activation(f.get("smolgen_activation", 0), default),
        ffn_activation=_activation(f.get("ffn_activation", 0), default))
    need("smolgen_w")
    need("policy_heads.vanilla.ip4_pol_w")
    need("value_heads.winner.ip2_val_w")
    need("ip2_mov_w")
    if d % heads or hidden_x_heads % heads:
        raise RuntimeError("B200 backend: head count does not divide the embedding")
    return cfg


def expected_sizes(cfg: NetConfig) -> Dict[str, int]:
    """Element count of every tensor the library packs (from the dims the
    synthetic generator uses for the same config)."""
    from .layout import GLOBAL_SLOTS, LAYER_SLOTS, layer_name
    d, T, dp = cfg.embedding, 64, cfg.dp
    g = {"ip_emb_preproc_w": T * cfg.pe * 12 * T, "ip_emb_preproc_b": T * cfg.pe,
         "ip_emb_w": d * (112 + cfg.pe), "ip_emb_b": d, "ip_emb_ln_gammas": d,
         "ip_emb_ln_betas": d, "ip_mult_gate": d * T, "ip_add_gate": d * T,
         "ip_emb_ffn.dense1_w": cfg.emb_dff * d, "ip_emb_ffn.dense1_b": cfg.emb_dff,
         "ip_emb_ffn.dense2_w": d * cfg.emb_dff, "ip_emb_ffn.dense2_b": d,
         "ip_emb_ffn_ln_gammas": d, "ip_emb_ffn_ln_betas": d,
         "smolgen_w": T * T * cfg.smolgen_gen,
         "policy_heads.vanilla.ip_pol_w": dp * d, "policy_heads.vanilla.ip_pol_b": dp,
         "policy_heads.vanilla.ip2_pol_w": dp * dp, "policy_heads.vanilla.ip2_pol_b": dp,
         "policy_heads.vanilla.ip3_pol_w": dp * dp, "policy_heads.vanilla.ip3_pol_b": dp,
         "policy_heads.vanilla.ip4_pol_w": 4 * dp,
         "value_heads.winner.ip_val_w": cfg.value_emb * d,
         "value_heads.winner.ip_val_b": cfg.value_emb,
         "value_heads.winner.ip1_val_w": cfg.value_hidden * T * cfg.value_emb,
         "value_heads.winner.ip1_val_b": cfg.value_hidden,
         "value_heads.winner.ip2_val_w": 3 * cfg.value_hidden, "value_heads.winner.ip2_val_b": 3,
         "ip_mov_w": cfg.mlh_emb * d, "ip_mov_b": cfg.mlh_emb,
         "ip1_mov_w": cfg.mlh_hidden * T * cfg.mlh_emb, "ip1_mov_b": cfg.mlh_hidden,
         "ip2_mov_w": cfg.mlh_hidden, "ip2_mov_b": 1}
    hg = cfg.heads * cfg.smolgen_gen
    per = {"mha.q_w": d * d, "mha.q_b": d, "mha.k_w": d * d, "mha.k_b": d, "mha.v_w": d * d,
           "mha.v_b": d, "mha.dense_w": d * d, "mha.dense_b": d,
           "mha.smolgen.compress": cfg.smolgen_compress * d,
           "mha.smolgen.dense1_w": cfg.smolgen_hidden * T * cfg.smolgen_compress,
           "mha.smolgen.dense1_b": cfg.smolgen_hidden,
           "mha.smolgen.ln1_gammas": cfg.smolgen_hidden, "mha.smolgen.ln1_betas": cfg.smolgen_hidden,
           "mha.smolgen.dense2_w": hg * cfg.smolgen_hidden, "mha.smolgen.dense2_b": hg,
           "mha.smolgen.ln2_gammas": hg, "mha.smolgen.ln2_betas": hg,
           "ln1_gammas": d, "ln1_betas": d, "ffn.dense1_w": cfg.dff * d, "ffn.dense1_b": cfg.dff,
           "ffn.dense2_w": d * cfg.dff, "ffn.dense2_b": d, "ln2_gammas": d, "ln2_betas": d}
    sizes = {n: g[n] for n in GLOBAL_SLOTS}
    for i in range(cfg.layers):
        for n in LAYER_SLOTS:
            sizes[layer_name(i, n)] = per[n]
    return sizes


def load_weights(path: str, name: Optional[str] = None) -> Tuple[NetConfig, Dict[str, np.ndarray]]:
    """``LoadWeightsFromFile`` + the C++ backend's shape inference for a
    ``.pb`` / ``.pb.gz`` file: returns the inferred ``NetConfig`` and the fp32
    tensors keyed by schema path, validated against the packed sizes."""
    tensors, scalars = parse_weights(_read_bytes(path))
    fmt = fix_older_format(scalars, tensors)
    has_policy_heads = any(k.startswith("policy_heads.") for k in tensors)
    t = _heads(tensors)
    cfg = config_from_weights(t, scalars, fmt, has_policy_heads, name or path)
    out: Dict[str, np.ndarray] = {}
    missing: List[str] = []
    for key, n in expected_sizes(cfg).items():
        if key not in t:
            missing.append(key)
            continue
        if t[key].size != n:
            raise RuntimeError(f"B200 backend: {key} has {t[key].size} values, expected {n}")
        out[key] = t[key]
    if missing:
        raise RuntimeError("B200 backend: weight file lacks " + ", ".join(missing[:5]))
    return cfg, out
