"""ctypes binding of the C restatement oracle (oracle/bt4_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker the CUDA path is compared against, and
the "port" CPU baseline. Built by ``make -C oracle port``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

from metalfish_b200 import layout
from metalfish_b200.netfile import Outputs, PackedInputs
from metalfish_b200.synthetic import NetConfig

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libbt4oracle.so")


class _Config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "d", "layers", "heads", "dff", "emb_dff", "pe", "sg_compress", "sg_hidden", "sg_gen",
        "dp", "val_emb", "val_hidden", "mov_emb", "mov_hidden",
        "act_default", "act_smolgen", "act_ffn")]


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)
        _lib = ctypes.CDLL(LIB_PATH)
        _lib.bt4o_forward.restype = ctypes.c_int
        _lib.bt4o_build_policy_map.restype = ctypes.c_int
    return _lib


def _cfg(c: NetConfig) -> _Config:
    a = layout.ACTIVATIONS
    return _Config(c.embedding, c.layers, c.heads, c.dff, c.emb_dff, c.pe, c.smolgen_compress,
                   c.smolgen_hidden, c.smolgen_gen, c.dp, c.value_emb, c.value_hidden,
                   c.mlh_emb, c.mlh_hidden, a[c.default_activation], a[c.smolgen_activation],
                   a[c.ffn_activation])


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def forward(cfg: NetConfig, tensors, inp: PackedInputs, threads: int = 0) -> Outputs:
    """Oracle forward over a batch of packed inputs."""
    L = lib()
    keep = []

    def arr(name):
        a = np.ascontiguousarray(tensors[name], dtype=np.float32)
        keep.append(a)
        return a.ctypes.data

    g = (ctypes.c_void_p * len(layout.GLOBAL_SLOTS))(*[arr(n) for n in layout.GLOBAL_SLOTS])
    ls = (ctypes.c_void_p * (cfg.layers * len(layout.LAYER_SLOTS)))(
        *[arr(layout.layer_name(i, n)) for i in range(cfg.layers) for n in layout.LAYER_SLOTS])
    b = inp.count
    masks = np.ascontiguousarray(inp.masks, np.uint64)
    values = np.ascontiguousarray(inp.values, np.float32)
    pol = np.zeros((b, 1858), np.float32)
    wdl = np.zeros((b, 3), np.float32)
    val = np.zeros(b, np.float32)
    mlh = np.zeros(b, np.float32)
    c = _cfg(cfg)
    if threads <= 0:
        threads = os.cpu_count() or 1
    rc = L.bt4o_forward(ctypes.byref(c), g, ls, _ptr(masks), _ptr(values), b, _ptr(pol),
                        _ptr(wdl), _ptr(val), _ptr(mlh), threads)
    if rc != 0:
        raise RuntimeError(f"oracle forward failed: {rc}")
    return Outputs(pol, wdl, val, mlh)


def policy_map(q: np.ndarray, k: np.ndarray, ppo: np.ndarray) -> np.ndarray:
    """Attention-policy map for one position: q,k [64,dq], ppo [4,dq] -> [1858]."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    ppo = np.ascontiguousarray(ppo, np.float32)
    out = np.zeros(1858, np.float32)
    lib().bt4o_policy_map(_ptr(q), _ptr(k), _ptr(ppo), ctypes.c_int(q.shape[1]), _ptr(out))
    return out


def build_policy_map() -> np.ndarray:
    t = np.zeros(4288, np.int16)
    n = lib().bt4o_build_policy_map(_ptr(t))
    assert n == 1858
    return t


def slot_counts():
    g, l = ctypes.c_int(), ctypes.c_int()
    lib().bt4o_slot_counts(ctypes.byref(g), ctypes.byref(l))
    return g.value, l.value


def fast_exp(x: np.ndarray) -> np.ndarray:
    """The reference FastExp (src/mcts/core.h:38-44), elementwise."""
    L = lib()
    L.bt4o_fast_exp.restype = ctypes.c_float
    L.bt4o_fast_exp.argtypes = [ctypes.c_float]
    return np.array([L.bt4o_fast_exp(float(v)) for v in np.asarray(x, np.float32)], np.float32)


def priors(policy: np.ndarray, offsets: np.ndarray, index: np.ndarray, temp: float) -> np.ndarray:
    """Legal-move priors of the MCTS leaf path (bt4o_priors)."""
    policy = np.ascontiguousarray(policy, np.float32)
    offsets = np.ascontiguousarray(offsets, np.int32)
    index = np.ascontiguousarray(index, np.int16)
    out = np.zeros(int(offsets[-1]), np.float32)
    lib().bt4o_priors(_ptr(policy), ctypes.c_int(policy.shape[0]), _ptr(offsets), _ptr(index),
                      ctypes.c_float(temp), _ptr(out))
    return out


def encode(boards: np.ndarray, offsets: np.ndarray, fmt: int):
    """Reference encoder restatement (bt4o_encode) over board records
    [n, 112] uint8 with CSR offsets: packed masks, values [B, 112], transforms [B]."""
    L = lib()
    assert L.bt4o_board_size() == 112
    b = len(offsets) - 1
    boards = np.ascontiguousarray(boards, np.uint8)
    offsets = np.ascontiguousarray(offsets, np.int32)
    m = np.zeros((b, 112), np.uint64)
    v = np.zeros((b, 112), np.float32)
    t = np.zeros(b, np.int32)
    if L.bt4o_encode(_ptr(boards), _ptr(offsets), ctypes.c_int(b), ctypes.c_int(fmt), _ptr(m), _ptr(v),
                     _ptr(t)) != 0:
        raise RuntimeError("bt4o_encode failed")
    return m, v, t
