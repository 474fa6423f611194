"""Host-side mirror of the reference ``NN::Network`` interface over libmfb200.

``B200Network`` follows ``src/nn/network.h:38-51`` (Evaluate, EvaluateBatch,
GetNetworkInfo, HasWDL, HasMovesLeft, GetBackendCapabilities) and
``create_network`` follows ``CreateNetwork(weights, BackendConfig)``
(``src/nn/network.cpp:137-208``) for the ``"b200"`` backend. Errors raise
``RuntimeError`` carrying the library's message, as the reference throws
``std::runtime_error``. There is no CPU fallback: without a B200 and the built
library every call raises.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import layout
from ._lib import lib
from .netfile import POLICY, Outputs, PackedInputs, pack_planes
from .synthetic import NetConfig


class NetDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "embedding", "layers", "heads", "dff", "emb_dff", "pe", "smolgen_compress",
        "smolgen_hidden", "smolgen_gen", "policy_d", "value_emb", "value_hidden", "mlh_emb",
        "mlh_hidden", "act_default", "act_smolgen", "act_ffn")]


class Config(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("num_devices", ctypes.c_int32),
                ("precision", ctypes.c_int32), ("max_batch", ctypes.c_int32),
                ("use_graphs", ctypes.c_int32), ("fp8_gemms", ctypes.c_int32)]


class Timing(ctypes.Structure):
    _fields_ = [("h2d_ms", ctypes.c_float), ("forward_ms", ctypes.c_float),
                ("d2h_ms", ctypes.c_float), ("total_ms", ctypes.c_float)]


class Caps(ctypes.Structure):
    _fields_ = [("max_batch", ctypes.c_int32), ("precision", ctypes.c_int32),
                ("num_devices", ctypes.c_int32), ("device", ctypes.c_int32),
                ("has_wdl", ctypes.c_int32), ("has_moves_left", ctypes.c_int32),
                ("weight_bytes", ctypes.c_int64), ("workspace_bytes", ctypes.c_int64),
                ("device_name", ctypes.c_char * 96)]


PRECISIONS = {"bf16": 0, "fp8": 1, "int8": 2}


def _declare(L):
    vp, c_int = ctypes.c_void_p, ctypes.c_int
    L.mfb200_weight_bytes.restype = ctypes.c_size_t
    L.mfb200_weight_bytes.argtypes = [ctypes.POINTER(NetDesc)]
    L.mfb200_create.restype = c_int
    L.mfb200_create.argtypes = [ctypes.POINTER(NetDesc), vp, ctypes.c_size_t,
                                ctypes.POINTER(Config), ctypes.POINTER(vp)]
    L.mfb200_evaluate.restype = c_int
    L.mfb200_evaluate.argtypes = [vp, vp, vp, c_int, vp, vp, vp, ctypes.POINTER(Timing)]
    L.mfb200_evaluate_priors.restype = c_int
    L.mfb200_evaluate_priors.argtypes = [vp, vp, vp, c_int, vp, vp, ctypes.c_float, vp, vp, vp,
                                         ctypes.POINTER(Timing)]
    L.mfb200_encode_history.restype = c_int
    L.mfb200_encode_history.argtypes = [vp, vp, vp, c_int, c_int, vp, vp, vp]
    L.mfb200_evaluate_history.restype = c_int
    L.mfb200_evaluate_history.argtypes = [vp, vp, vp, c_int, c_int, vp, vp, vp, vp,
                                          ctypes.POINTER(Timing)]
    L.mfb200_evaluate_leaves.restype = c_int
    L.mfb200_evaluate_leaves.argtypes = [vp, vp, vp, c_int, c_int, vp, vp, ctypes.c_float, vp, vp,
                                         vp, ctypes.POINTER(Timing)]
    L.mfb200_submit_leaves.restype = c_int
    L.mfb200_submit_leaves.argtypes = [vp, vp, vp, c_int, c_int, vp, vp, ctypes.c_float, vp, vp,
                                       vp, ctypes.POINTER(ctypes.c_uint64)]
    L.mfb200_wait.restype = c_int
    L.mfb200_wait.argtypes = [vp, ctypes.c_uint64]
    L.mfb200_policy_index_table.restype = c_int
    L.mfb200_policy_index_table.argtypes = [vp]
    L.mfb200_evaluate_device.restype = c_int
    L.mfb200_evaluate_device.argtypes = [vp, vp, vp, c_int, vp, vp, vp, vp]
    L.mfb200_calibrate.restype = c_int
    L.mfb200_calibrate.argtypes = [vp, vp, vp, c_int]
    L.mfb200_capabilities.restype = c_int
    L.mfb200_capabilities.argtypes = [vp, ctypes.POINTER(Caps)]
    L.mfb200_profile.restype = c_int
    L.mfb200_profile.argtypes = [vp, c_int, c_int, vp, vp, ctypes.c_char_p, ctypes.c_size_t, c_int]
    L.mfb200_last_error.restype = ctypes.c_char_p
    L.mfb200_last_error.argtypes = [vp]
    L.mfb200_destroy.restype = None
    L.mfb200_destroy.argtypes = [vp]


def _lib():
    L = lib()
    if not getattr(L, "_mfb200_declared", False):
        _declare(L)
        L._mfb200_declared = True
    return L


def net_desc(cfg: NetConfig) -> NetDesc:
    a = layout.ACTIVATIONS
    return NetDesc(cfg.embedding, cfg.layers, cfg.heads, cfg.dff, cfg.emb_dff, cfg.pe,
                   cfg.smolgen_compress, cfg.smolgen_hidden, cfg.smolgen_gen, cfg.dp,
                   cfg.value_emb, cfg.value_hidden, cfg.mlh_emb, cfg.mlh_hidden,
                   a[cfg.default_activation], a[cfg.smolgen_activation], a[cfg.ffn_activation])


def weight_blob(cfg: NetConfig, tensors: Dict[str, np.ndarray]) -> np.ndarray:
    """Concatenate the fp32 tensors in the library's slot order."""
    parts = [np.ascontiguousarray(tensors[n], np.float32).ravel() for n in layout.GLOBAL_SLOTS]
    for i in range(cfg.layers):
        parts += [np.ascontiguousarray(tensors[layout.layer_name(i, n)], np.float32).ravel()
                  for n in layout.LAYER_SLOTS]
    return np.concatenate(parts)


@dataclass
class NetworkOutput:
    """``src/nn/network_output.h:17-24``."""
    policy: np.ndarray
    value: float
    wdl: np.ndarray
    has_wdl: bool = True
    moves_left: float = 0.0
    has_moves_left: bool = True


@dataclass
class BackendCapabilities:
    """``src/nn/network.h:21-36`` (the fields this backend fills)."""
    actual_backend: str = "b200"
    has_wdl: bool = True
    has_moves_left: bool = True
    max_batch_size: int = 0
    device_name: str = ""
    precision: str = "bf16"
    num_devices: int = 1
    weight_bytes: int = 0
    workspace_bytes: int = 0

    def summary(self) -> str:
        return (f"actual_backend={self.actual_backend} has_wdl={str(self.has_wdl).lower()} "
                f"has_moves_left={str(self.has_moves_left).lower()} max_batch={self.max_batch_size} "
                f'device="{self.device_name}" precision={self.precision} gpus={self.num_devices}')


class B200Network:
    def __init__(self, cfg: NetConfig, tensors: Dict[str, np.ndarray], *, device: int = 0,
                 num_devices: int = 1, precision: str = "bf16", max_batch: int = 1024,
                 use_graphs: bool = True, fp8_gemms: int = 0):
        L = _lib()
        self.cfg = cfg
        self.precision = precision
        self._desc = net_desc(cfg)
        blob = weight_blob(cfg, tensors)
        expected = L.mfb200_weight_bytes(ctypes.byref(self._desc))
        if blob.nbytes != expected:
            raise RuntimeError(f"weight blob is {blob.nbytes} bytes, library expects {expected}")
        conf = Config(device, num_devices, PRECISIONS[precision], max_batch, int(use_graphs),
                      fp8_gemms)
        h = ctypes.c_void_p()
        rc = L.mfb200_create(ctypes.byref(self._desc), blob.ctypes.data, blob.nbytes,
                             ctypes.byref(conf), ctypes.byref(h))
        if rc != 0:
            raise RuntimeError(L.mfb200_last_error(None).decode())
        self._h = h
        self.max_batch = max_batch

    # -- lifecycle
    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib().mfb200_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _err(self) -> RuntimeError:
        return RuntimeError(_lib().mfb200_last_error(self._h).decode())

    # -- packed-input path (what MCTS batch assembly feeds)
    def evaluate_packed(self, inp: PackedInputs, timing: Optional[Timing] = None) -> Outputs:
        b = inp.count
        masks = np.ascontiguousarray(inp.masks, np.uint64)
        values = np.ascontiguousarray(inp.values, np.float32)
        pol = np.empty((b, POLICY), np.float32)
        wdl = np.empty((b, 3), np.float32)
        mlh = np.empty(b, np.float32)
        rc = _lib().mfb200_evaluate(self._h, masks.ctypes.data, values.ctypes.data, b,
                                    pol.ctypes.data, wdl.ctypes.data, mlh.ctypes.data,
                                    ctypes.byref(timing) if timing is not None else None)
        if rc != 0:
            raise self._err()
        return Outputs(pol, wdl, wdl[:, 0] - wdl[:, 2], mlh)

    def evaluate_priors(self, inp: PackedInputs, move_offsets: np.ndarray, move_index: np.ndarray,
                        softmax_temp: float = 1.0, timing: Optional[Timing] = None):
        """Forward plus the MCTS leaf step on the GPU: the normalised prior of
        each legal move (CSR move_offsets [B+1] over move_index, the policy
        index of each move), instead of the 1858 logits. Returns
        (priors [move_offsets[-1] - move_offsets[0]], wdl [B, 3], moves_left [B])."""
        b = inp.count
        masks = np.ascontiguousarray(inp.masks, np.uint64)
        values = np.ascontiguousarray(inp.values, np.float32)
        off = np.ascontiguousarray(move_offsets, np.int32)
        idx = np.ascontiguousarray(move_index, np.int16)
        if off.shape != (b + 1,):
            raise ValueError("move_offsets must have batch + 1 entries")
        pri = np.empty(int(off[-1] - off[0]), np.float32)
        wdl = np.empty((b, 3), np.float32)
        mlh = np.empty(b, np.float32)
        rc = _lib().mfb200_evaluate_priors(self._h, masks.ctypes.data, values.ctypes.data, b,
                                           off.ctypes.data, idx.ctypes.data if idx.size else None,
                                           ctypes.c_float(softmax_temp), pri.ctypes.data,
                                           wdl.ctypes.data, mlh.ctypes.data,
                                           ctypes.byref(timing) if timing is not None else None)
        if rc != 0:
            raise self._err()
        return pri, wdl, mlh

    # -- position encoding on the GPU (board records: include/mfb200.h mfb200_board,
    #    112 bytes each, as uint8 rows or a structured array)
    def encode_history(self, boards: np.ndarray, history_offsets: np.ndarray,
                       input_format: int = 5):
        """EncodePositionForNN on the GPU: packed masks / values [B, 112] and
        the canonicalisation transforms [B] of B game histories."""
        boards = np.ascontiguousarray(boards).view(np.uint8)
        off = np.ascontiguousarray(history_offsets, np.int32)
        b = len(off) - 1
        m = np.empty((b, 112), np.uint64)
        v = np.empty((b, 112), np.float32)
        t = np.empty(b, np.int32)
        rc = _lib().mfb200_encode_history(self._h, boards.ctypes.data if boards.size else None,
                                          off.ctypes.data, b, input_format, m.ctypes.data,
                                          v.ctypes.data, t.ctypes.data)
        if rc != 0:
            raise self._err()
        return m, v, t

    def evaluate_history(self, boards: np.ndarray, history_offsets: np.ndarray,
                         input_format: int = 5, timing: Optional[Timing] = None):
        """Encode on the GPU and evaluate: (Outputs, transforms [B])."""
        boards = np.ascontiguousarray(boards).view(np.uint8)
        off = np.ascontiguousarray(history_offsets, np.int32)
        b = len(off) - 1
        pol = np.empty((b, POLICY), np.float32)
        wdl = np.empty((b, 3), np.float32)
        mlh = np.empty(b, np.float32)
        t = np.empty(b, np.int32)
        rc = _lib().mfb200_evaluate_history(self._h, boards.ctypes.data if boards.size else None,
                                            off.ctypes.data, b, input_format, pol.ctypes.data,
                                            wdl.ctypes.data, mlh.ctypes.data, t.ctypes.data,
                                            ctypes.byref(timing) if timing is not None else None)
        if rc != 0:
            raise self._err()
        return Outputs(pol, wdl, wdl[:, 0] - wdl[:, 2], mlh), t

    def evaluate_leaves(self, boards: np.ndarray, history_offsets: np.ndarray, moves: np.ndarray,
                        move_offsets: np.ndarray, softmax_temp: float = 1.0, input_format: int = 5,
                        timing: Optional[Timing] = None):
        """The whole MCTS leaf evaluation on the GPU: histories and legal moves
        (uint16 from | to << 6 | promotion << 12) in; (priors, wdl, moves_left) out."""
        boards = np.ascontiguousarray(boards).view(np.uint8)
        hoff = np.ascontiguousarray(history_offsets, np.int32)
        mv = np.ascontiguousarray(moves, np.uint16)
        moff = np.ascontiguousarray(move_offsets, np.int32)
        b = len(hoff) - 1
        if moff.shape != (b + 1,):
            raise ValueError("move_offsets must have batch + 1 entries")
        pri = np.empty(int(moff[-1] - moff[0]), np.float32)
        wdl = np.empty((b, 3), np.float32)
        mlh = np.empty(b, np.float32)
        rc = _lib().mfb200_evaluate_leaves(self._h, boards.ctypes.data if boards.size else None,
                                           hoff.ctypes.data, b, input_format,
                                           mv.ctypes.data if mv.size else None, moff.ctypes.data,
                                           ctypes.c_float(softmax_temp), pri.ctypes.data,
                                           wdl.ctypes.data, mlh.ctypes.data,
                                           ctypes.byref(timing) if timing is not None else None)
        if rc != 0:
            raise self._err()
        return pri, wdl, mlh

    def submit_leaves(self, boards: np.ndarray, history_offsets: np.ndarray, moves: np.ndarray,
                      move_offsets: np.ndarray, softmax_temp: float = 1.0, input_format: int = 5):
        """Asynchronous evaluate_leaves: returns a LeafTicket whose wait()
        gives (priors, wdl, moves_left). The arrays are kept alive by the
        ticket until it is waited for."""
        boards = np.ascontiguousarray(boards).view(np.uint8)
        hoff = np.ascontiguousarray(history_offsets, np.int32)
        mv = np.ascontiguousarray(moves, np.uint16)
        moff = np.ascontiguousarray(move_offsets, np.int32)
        b = len(hoff) - 1
        if moff.shape != (b + 1,):
            raise ValueError("move_offsets must have batch + 1 entries")
        pri = np.empty(int(moff[-1] - moff[0]), np.float32)
        wdl = np.empty((b, 3), np.float32)
        mlh = np.empty(b, np.float32)
        t = ctypes.c_uint64(0)
        rc = _lib().mfb200_submit_leaves(self._h, boards.ctypes.data if boards.size else None,
                                         hoff.ctypes.data, b, input_format,
                                         mv.ctypes.data if mv.size else None, moff.ctypes.data,
                                         ctypes.c_float(softmax_temp), pri.ctypes.data,
                                         wdl.ctypes.data, mlh.ctypes.data, ctypes.byref(t))
        if rc != 0:
            raise self._err()
        return LeafTicket(self, t.value, (boards, hoff, mv, moff), (pri, wdl, mlh))

    def calibrate(self, inp: PackedInputs) -> None:
        """FP8 / INT8 only: absmax calibration of the per-tensor activation scales
        over the given positions (a bf16 forward with probes)."""
        masks = np.ascontiguousarray(inp.masks, np.uint64)
        values = np.ascontiguousarray(inp.values, np.float32)
        if _lib().mfb200_calibrate(self._h, masks.ctypes.data, values.ctypes.data, inp.count) != 0:
            raise self._err()

    def evaluate_device(self, d_masks: int, d_values: int, batch: int, d_policy: int, d_wdl: int,
                        d_mlh: int, stream: int = 0) -> None:
        rc = _lib().mfb200_evaluate_device(self._h, d_masks, d_values, batch, d_policy, d_wdl,
                                           d_mlh, stream or None)
        if rc != 0:
            raise self._err()

    # -- the reference Network interface
    def evaluate_batch(self, inputs: Sequence[np.ndarray]) -> List[NetworkOutput]:
        """EvaluateBatch over InputPlanes ([112, 64] float arrays)."""
        if len(inputs) == 0:
            return []
        planes = np.stack([np.asarray(x, np.float32).reshape(112, 64) for x in inputs])
        out = self.evaluate_packed(pack_planes(planes))
        return [NetworkOutput(out.policy[i], float(out.value[i]), out.wdl[i], True,
                              float(out.moves_left[i]), True) for i in range(len(inputs))]

    def evaluate(self, planes: np.ndarray) -> NetworkOutput:
        return self.evaluate_batch([planes])[0]

    def has_wdl(self) -> bool:
        return True

    def has_moves_left(self) -> bool:
        return True

    def get_backend_capabilities(self) -> BackendCapabilities:
        c = Caps()
        if _lib().mfb200_capabilities(self._h, ctypes.byref(c)) != 0:
            raise self._err()
        return BackendCapabilities("b200", bool(c.has_wdl), bool(c.has_moves_left), c.max_batch,
                                   c.device_name.decode(), self.precision, c.num_devices,
                                   c.weight_bytes, c.workspace_bytes)

    def get_network_info(self) -> str:
        c = self.cfg
        return (f"B200 transformer backend (net={c.name} d={c.embedding} layers={c.layers} "
                f"heads={c.heads} dff={c.dff}, {self.get_backend_capabilities().summary()})")

    def profile(self, batch: int, iters: int = 3):
        n = 512
        ms = (ctypes.c_float * n)()
        fl = (ctypes.c_double * n)()
        names = ctypes.create_string_buffer(1 << 16)
        k = _lib().mfb200_profile(self._h, batch, iters, ms, fl, names, len(names), n)
        if k < 0:
            raise self._err()
        nm = names.value.decode().split("\n")
        return [(nm[i], ms[i], fl[i]) for i in range(k)]


class LeafTicket:
    """An in-flight mfb200_submit_leaves; wait() returns its outputs."""

    def __init__(self, net, ticket: int, inputs, outputs):
        self.net, self.ticket, self._inputs, self._outputs = net, ticket, inputs, outputs

    def wait(self):
        if self._inputs is not None:
            if _lib().mfb200_wait(self.net._h, self.ticket) != 0:
                raise self.net._err()
            self._inputs = None
        return self._outputs


def policy_index_table() -> np.ndarray:
    """The library's NN::MoveToNNIndex table [8 transforms][5 promotions][64][64]."""
    t = np.empty((8, 5, 64, 64), np.int16)
    _lib().mfb200_policy_index_table(t.ctypes.data)
    return t


def create_network(cfg: NetConfig, tensors: Dict[str, np.ndarray], backend: str = "b200",
                   calibration: Optional[PackedInputs] = None, **kwargs) -> B200Network:
    """``CreateNetwork(weights, BackendConfig)`` for the B200 backend. 8-bit
    networks (precision="fp8" or "int8") are calibrated on `calibration` positions."""
    if backend not in ("b200", "auto"):
        raise RuntimeError(f"Unknown NN backend: {backend}")
    net = B200Network(cfg, tensors, **kwargs)
    if net.precision in ("fp8", "int8"):
        if calibration is None:
            raise RuntimeError("an 8-bit (FP8 / INT8) network needs calibration positions")
        net.calibrate(calibration)
    return net


def create_network_from_file(path: str, backend: str = "b200",
                             calibration: Optional[PackedInputs] = None, **kwargs) -> B200Network:
    """``CreateNetwork(LoadWeightsFromFile(path), BackendConfig)``
    (``src/nn/network.cpp:137-208``, ``src/nn/loader.cpp:156-175``) for the
    B200 backend: a ``.pb`` / ``.pb.gz`` weight file, shape inferred from it."""
    from .weightsfile import load_weights
    cfg, tensors = load_weights(path)
    return create_network(cfg, tensors, backend=backend, calibration=calibration, **kwargs)
