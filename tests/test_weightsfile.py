"""The Python reader of MetalFish's protobuf weight files
(``metalfish_b200.weightsfile``) against the reference's own serialiser
(``oracle/_ref/ref_harness to-pb``: ``WeightsFile::SerializeToString`` of the
reference's protobuf classes), the reference's layer decoding
(``src/nn/loader.cpp:181-250``) and legacy head layout
(``src/nn/weights.cpp:214-290``).
"""
import gzip
import os
import struct
import subprocess

import numpy as np
import pytest

from metalfish_b200 import synthetic
from metalfish_b200.netfile import write_net
from metalfish_b200.weightsfile import (BFLOAT16, FLOAT16, FLOAT32, LINEAR16, UNKNOWN_ENCODING,
                                        decode_layer, load_weights)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HARNESS = os.path.join(ROOT, "oracle", "_ref", "ref_harness")


def _u16(*vals):
    return struct.pack(f"<{len(vals)}H", *vals)


def test_decode_float16_known_answers():
    # +0, 1.0, -2.0, smallest subnormal, largest subnormal, -inf, 65504
    raw = _u16(0x0000, 0x3C00, 0xC000, 0x0001, 0x03FF, 0xFC00, 0x7BFF)
    v = decode_layer(0.0, 0.0, raw, FLOAT16)
    np.testing.assert_array_equal(
        v, np.array([0.0, 1.0, -2.0, 2.0 ** -24, 1023 * 2.0 ** -24, -np.inf, 65504.0], np.float32))


def test_decode_bfloat16_and_float32():
    np.testing.assert_array_equal(decode_layer(0, 0, _u16(0x3F80, 0xC040), BFLOAT16),
                                  np.array([1.0, -3.0], np.float32))
    x = np.array([1.5, -7.25e-9, 3e38], np.float32)
    np.testing.assert_array_equal(decode_layer(0, 0, x.tobytes(), FLOAT32), x)


def test_decode_linear16_matches_reference_formula():
    raw = np.array([0, 1, 32768, 65534, 65535], np.uint16)
    lo, hi = np.float32(-0.75), np.float32(1.25)
    # src/nn/loader.cpp:209-210, fp32: min_val + (raw / 65535.0f) * range
    want = lo + (raw.astype(np.float32) / np.float32(65535.0)) * np.float32(hi - lo)
    got = decode_layer(float(lo), float(hi), raw.tobytes(), LINEAR16)
    np.testing.assert_array_equal(got, want)
    # a layer without an encoding is LINEAR16 (loader.cpp:186-190)
    np.testing.assert_array_equal(decode_layer(float(lo), float(hi), raw.tobytes(), UNKNOWN_ENCODING), want)
    assert got[0] == lo and got[-1] == hi


def test_unsupported_encoding_raises():
    with pytest.raises(RuntimeError, match="Unsupported weight encoding"):
        decode_layer(0, 0, b"\0\0\0\0", 9)


needs_harness = pytest.mark.skipif(not os.path.exists(HARNESS),
                                   reason="reference harness not built (make -C oracle ref)")


def _reference_pb(tmp_path, cfg, seed=5, perturb=True):
    t = synthetic.generate(cfg, seed, perturb)
    net = tmp_path / "net.mfnt"
    pb = tmp_path / "net.pb"
    write_net(str(net), cfg.header(), t)
    subprocess.run([HARNESS, "to-pb", str(net), str(pb)], check=True)
    return t, pb


CFG_FIELDS = ("embedding", "layers", "heads", "dff", "emb_dff", "pe", "smolgen_compress",
              "smolgen_hidden", "smolgen_gen", "dp", "value_emb", "value_hidden", "mlh_emb",
              "mlh_hidden", "default_activation", "smolgen_activation", "ffn_activation")


@needs_harness
@pytest.mark.parametrize("name", ["tiny-128x2x4h", "small-256x6x8h"])
def test_reference_serialised_file_round_trips(tmp_path, name):
    cfg = synthetic.CONFIGS[name]
    t, pb = _reference_pb(tmp_path, cfg)
    got_cfg, got = load_weights(str(pb))
    for f in CFG_FIELDS:
        assert getattr(got_cfg, f) == getattr(cfg, f), f
    assert set(got) == set(t)
    for k in t:
        np.testing.assert_array_equal(got[k], t[k].ravel(), err_msg=k)
    # the same file gzip-compressed (".gz" suffix, loader.cpp:159-160)
    gz = tmp_path / "net.pb.gz"
    gz.write_bytes(gzip.compress(pb.read_bytes()))
    _, got_gz = load_weights(str(gz))
    for k in t:
        np.testing.assert_array_equal(got_gz[k], got[k])


# --- a minimal protobuf writer for hand-built files (legacy layouts, errors)
def _varint(v):
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        out.append(b | (0x80 if v else 0))
        if not v:
            return bytes(out)


def _ld(num, payload):
    return _varint(num << 3 | 2) + _varint(len(payload)) + payload


def _vi(num, v):
    return _varint(num << 3) + _varint(v)


def _layer_f16(x):
    # FLOAT16-encoded layer (encoding 2)
    return _ld(3, np.asarray(x, np.float16).tobytes()) + _vi(4, FLOAT16)


# field numbers of src/nn/proto/net.proto (Weights, EncoderLayer, MHA, ...)
W = {"ip_emb_preproc_w": 37, "ip_emb_preproc_b": 38, "ip_emb_w": 25, "ip_emb_b": 26,
     "ip_emb_ln_gammas": 39, "ip_emb_ln_betas": 40, "ip_mult_gate": 33, "ip_add_gate": 34,
     "ip_emb_ffn_ln_gammas": 42, "ip_emb_ffn_ln_betas": 43, "smolgen_w": 35,
     "ip_pol_w": 4, "ip_pol_b": 5, "ip2_pol_w": 17, "ip2_pol_b": 18, "ip3_pol_w": 19,
     "ip3_pol_b": 20, "ip4_pol_w": 22, "ip_val_w": 29, "ip_val_b": 30, "ip1_val_w": 7,
     "ip1_val_b": 8, "ip2_val_w": 9, "ip2_val_b": 10, "ip_mov_w": 31, "ip_mov_b": 32,
     "ip1_mov_w": 13, "ip1_mov_b": 14, "ip2_mov_w": 15, "ip2_mov_b": 16}
FFN = {"dense1_w": 1, "dense1_b": 2, "dense2_w": 3, "dense2_b": 4}
MHA = {"q_w": 1, "q_b": 2, "k_w": 3, "k_b": 4, "v_w": 5, "v_b": 6, "dense_w": 7, "dense_b": 8}
SG = {"compress": 1, "dense1_w": 2, "dense1_b": 3, "ln1_gammas": 4, "ln1_betas": 5,
      "dense2_w": 6, "dense2_b": 7, "ln2_gammas": 8, "ln2_betas": 9}
ENC = {"ln1_gammas": 2, "ln1_betas": 3, "ln2_gammas": 5, "ln2_betas": 6}


def _legacy_file(cfg, t, magic=0x1C0, network=4, input_embedding=2):
    """Single-head legacy layout: policy and value head layers at the top
    level of Weights (no policy_heads / value_heads messages), network
    NETWORK_SE_WITH_HEADFORMAT (FixOlderWeightsFile turns it into an attention
    body and forces RELU_2 / SWISH because smolgen_w is present)."""
    w = b""
    pv, vw = "policy_heads.vanilla.", "value_heads.winner."
    for k, num in W.items():
        src = t.get(k, t.get(pv + k, t.get(vw + k)))
        w += _ld(num, _layer_f16(src))
    w += _ld(41, b"".join(_ld(n, _layer_f16(t["ip_emb_ffn." + k])) for k, n in FFN.items()))
    for i in range(cfg.layers):
        p = f"encoder.{i}."
        sg = b"".join(_ld(n, _layer_f16(t[p + "mha.smolgen." + k])) for k, n in SG.items())
        mha = b"".join(_ld(n, _layer_f16(t[p + "mha." + k])) for k, n in MHA.items()) + _ld(9, sg)
        ffn = b"".join(_ld(n, _layer_f16(t[p + "ffn." + k])) for k, n in FFN.items())
        enc = _ld(1, mha) + _ld(4, ffn) + b"".join(_ld(n, _layer_f16(t[p + k])) for k, n in ENC.items())
        w += _ld(27, enc)
    w += _vi(28, cfg.heads)
    # network, policy ATTENTION, value WDL, moves-left V1, default activation
    # MISH, smolgen / ffn ACTIVATION_DEFAULT (fixed up), input embedding
    nf = _vi(3, network) + _vi(4, 3) + _vi(5, 2) + _vi(6, 1) + _vi(7, 1)
    if input_embedding is not None:
        nf += _vi(10, input_embedding)
    return _varint(1 << 3 | 5) + struct.pack("<I", magic) + _ld(4, _ld(2, nf)) + _ld(10, w)


def test_legacy_single_head_layout(tmp_path):
    cfg = synthetic.TINY
    t = synthetic.generate(cfg, 9, True)
    f = tmp_path / "legacy.pb"
    f.write_bytes(_legacy_file(cfg, t))
    got_cfg, got = load_weights(str(f))
    for fld in CFG_FIELDS:
        assert getattr(got_cfg, fld) == getattr(cfg, fld), fld
    for k in t:
        np.testing.assert_array_equal(got[k], t[k].ravel().astype(np.float16).astype(np.float32),
                                      err_msg=k)


def test_bad_magic_and_truncation_raise(tmp_path):
    cfg = synthetic.TINY
    t = synthetic.generate(cfg, 9)
    f = tmp_path / "bad.pb"
    f.write_bytes(_legacy_file(cfg, t, magic=0x1234))
    with pytest.raises(RuntimeError, match="bad magic"):
        load_weights(str(f))
    good = _legacy_file(cfg, t)
    f.write_bytes(good[: len(good) // 2])
    with pytest.raises(RuntimeError, match="Failed to parse"):
        load_weights(str(f))
    f.write_bytes(b"\0")
    with pytest.raises(RuntimeError, match="too small"):
        load_weights(str(f))


def test_missing_smolgen_is_rejected(tmp_path):
    cfg = synthetic.TINY
    t = synthetic.generate(cfg, 9)
    del t["smolgen_w"]
    t["smolgen_w"] = np.zeros(0, np.float32)  # an empty layer
    f = tmp_path / "nosg.pb"
    f.write_bytes(_legacy_file(cfg, t))
    with pytest.raises(RuntimeError, match="smolgen"):
        load_weights(str(f))


@pytest.mark.gpu
@needs_harness
def test_network_from_weight_file_matches_tensors(tmp_path, positions):
    """A network created from the reference-serialised .pb evaluates bit for
    bit like one created from the same tensors."""
    from metalfish_b200.network import create_network, create_network_from_file
    cfg = synthetic.SMALL
    t, pb = _reference_pb(tmp_path, cfg)
    a = create_network_from_file(str(pb), max_batch=16)
    b = create_network(cfg, t, max_batch=16)
    try:
        oa = a.evaluate_packed(positions.slice(0, 16))
        ob = b.evaluate_packed(positions.slice(0, 16))
    finally:
        a.close()
        b.close()
    np.testing.assert_array_equal(oa.policy, ob.policy)
    np.testing.assert_array_equal(oa.wdl, ob.wdl)
    np.testing.assert_array_equal(oa.moves_left, ob.moves_left)


def test_format_checks_of_the_backend(tmp_path):
    """The C++ backend's format requirements, after the reference's
    FixOlderWeightsFile: a classical network and a file without the PE_DENSE
    input embedding are refused."""
    cfg = synthetic.TINY
    t = synthetic.generate(cfg, 9)
    f = tmp_path / "fmt.pb"
    f.write_bytes(_legacy_file(cfg, t, network=1))
    with pytest.raises(RuntimeError, match="not an attention-body network"):
        load_weights(str(f))
    f.write_bytes(_legacy_file(cfg, t, input_embedding=None))
    with pytest.raises(RuntimeError, match="PE_DENSE"):
        load_weights(str(f))

