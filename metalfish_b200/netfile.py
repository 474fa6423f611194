"""File formats shared by the product, the tests and the oracle harness.

* MFNT -- a named-tensor network file. Tensor names are the field paths of the
  reference weight schema (``src/nn/proto/net.proto``: ``encoder.3.mha.q_w``,
  ``policy_heads.vanilla.ip4_pol_w`` ...), every tensor fp32 with the
  reference's ``[out, in]`` dims convention (``src/nn/network_execution_plan.cpp``
  InferMatrixFromBias). A short ``key=value`` text header carries the head
  count and the activation names.
* MFIN -- packed inputs: per position 112 ``u64`` masks and 112 ``f32`` values,
  the format of ``PackInputPlanesRaw`` (``src/nn/input_plane_packing.h:63-83``).
* MFOT -- outputs: policy ``[B,1858]``, wdl ``[B,3]``, value ``[B]``,
  moves-left ``[B]`` (``src/nn/network_output.h:17-24``).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from typing import Dict, Tuple

import numpy as np

PLANES = 112
SQUARES = 64
POLICY = 1858


def write_net(path: str, header: Dict[str, str], tensors: Dict[str, np.ndarray]) -> None:
    hdr = "".join(f"{k}={v}\n" for k, v in header.items()).encode()
    with open(path, "wb") as f:
        f.write(b"MFNT")
        f.write(struct.pack("<II", 1, len(hdr)))
        f.write(hdr)
        f.write(struct.pack("<I", len(tensors)))
        for name, arr in tensors.items():
            a = np.ascontiguousarray(arr, dtype=np.float32)
            nb = name.encode()
            f.write(struct.pack("<I", len(nb)))
            f.write(nb)
            f.write(struct.pack("<I", a.ndim))
            f.write(struct.pack(f"<{a.ndim}I", *a.shape))
            f.write(a.tobytes())


def read_net(path: str) -> Tuple[Dict[str, str], Dict[str, np.ndarray]]:
    with open(path, "rb") as f:
        data = f.read()
    if data[:4] != b"MFNT":
        raise ValueError("not an MFNT file")
    _, hlen = struct.unpack_from("<II", data, 4)
    off = 12
    header = {}
    for line in data[off:off + hlen].decode().splitlines():
        k, _, v = line.partition("=")
        header[k] = v
    off += hlen
    (count,) = struct.unpack_from("<I", data, off)
    off += 4
    tensors = {}
    for _ in range(count):
        (nl,) = struct.unpack_from("<I", data, off)
        off += 4
        name = data[off:off + nl].decode()
        off += nl
        (nd,) = struct.unpack_from("<I", data, off)
        off += 4
        dims = struct.unpack_from(f"<{nd}I", data, off)
        off += 4 * nd
        n = int(np.prod(dims)) if nd else 1
        tensors[name] = np.frombuffer(data, np.float32, n, off).reshape(dims).copy()
        off += 4 * n
    return header, tensors


@dataclass
class PackedInputs:
    masks: np.ndarray   # [B,112] uint64
    values: np.ndarray  # [B,112] float32

    @property
    def count(self) -> int:
        return int(self.masks.shape[0])

    def slice(self, lo: int, hi: int) -> "PackedInputs":
        return PackedInputs(self.masks[lo:hi].copy(), self.values[lo:hi].copy())


def write_inputs(path: str, inp: PackedInputs) -> None:
    with open(path, "wb") as f:
        f.write(b"MFIN")
        f.write(struct.pack("<III", 1, inp.count, PLANES))
        f.write(np.ascontiguousarray(inp.masks, np.uint64).tobytes())
        f.write(np.ascontiguousarray(inp.values, np.float32).tobytes())


def read_inputs(path: str) -> PackedInputs:
    with open(path, "rb") as f:
        data = f.read()
    if data[:4] != b"MFIN":
        raise ValueError("not an MFIN file")
    _, count, planes = struct.unpack_from("<III", data, 4)
    assert planes == PLANES
    off = 16
    masks = np.frombuffer(data, np.uint64, count * PLANES, off).reshape(count, PLANES).copy()
    off += 8 * count * PLANES
    values = np.frombuffer(data, np.float32, count * PLANES, off).reshape(count, PLANES).copy()
    return PackedInputs(masks, values)


@dataclass
class Outputs:
    policy: np.ndarray      # [B,1858]
    wdl: np.ndarray         # [B,3]
    value: np.ndarray       # [B]
    moves_left: np.ndarray  # [B]


def write_outputs(path: str, out: Outputs) -> None:
    b = out.policy.shape[0]
    with open(path, "wb") as f:
        f.write(b"MFOT")
        f.write(struct.pack("<II", 1, b))
        for a in (out.policy, out.wdl, out.value, out.moves_left):
            f.write(np.ascontiguousarray(a, np.float32).tobytes())


def read_outputs(path: str) -> Outputs:
    with open(path, "rb") as f:
        data = f.read()
    if data[:4] != b"MFOT":
        raise ValueError("not an MFOT file")
    _, b = struct.unpack_from("<II", data, 4)
    a = np.frombuffer(data, np.float32, offset=12)
    pol = a[:b * POLICY].reshape(b, POLICY).copy()
    o = b * POLICY
    wdl = a[o:o + 3 * b].reshape(b, 3).copy()
    o += 3 * b
    val = a[o:o + b].copy()
    o += b
    mlh = a[o:o + b].copy()
    return Outputs(pol, wdl, val, mlh)


def unpack_planes(inp: PackedInputs) -> np.ndarray:
    """[B,112] masks/values -> [B,112,64] float planes (inverse of the packing
    in ``src/nn/input_plane_packing.h:39-61``)."""
    bits = (inp.masks[:, :, None] >> np.arange(SQUARES, dtype=np.uint64)[None, None, :]) & np.uint64(1)
    return np.where(bits.astype(bool), inp.values[:, :, None], np.float32(0)).astype(np.float32)


def _uniform_planes() -> np.ndarray:
    """IsUniformPackedInputPlane (src/nn/input_plane_packing.h:30-37): the
    per-board all-equal plane (index 12 of each 13) and aux planes 2, 3, 5+."""
    p = np.arange(PLANES)
    aux = 13 * 8
    return ((p < aux) & (p % 13 == 12)) | (p == aux + 2) | (p == aux + 3) | (p >= aux + 5)


UNIFORM_PLANES = _uniform_planes()


def pack_planes(planes: np.ndarray) -> PackedInputs:
    """[B,112,64] float planes -> masks/values, as PackInputPlaneRaw
    (src/nn/input_plane_packing.h:39-61): a uniform plane keeps plane[0] and an
    all-ones mask when nonzero; any other plane keeps the FIRST nonzero value and
    the mask of all nonzero squares."""
    planes = np.asarray(planes, np.float32)
    b = planes.shape[0]
    nz = planes != 0
    weights = np.uint64(1) << np.arange(SQUARES, dtype=np.uint64)
    masks = (nz.astype(np.uint64) * weights[None, None, :]).sum(axis=2, dtype=np.uint64)
    first = np.where(nz.any(axis=2), nz.argmax(axis=2), 0)
    values = np.take_along_axis(planes, first[:, :, None], axis=2)[:, :, 0]
    values = np.where(nz.any(axis=2), values, np.float32(0))
    uni = UNIFORM_PLANES[None, :]
    v0 = planes[:, :, 0]
    values = np.where(uni, v0, values).astype(np.float32)
    masks = np.where(uni, np.where(v0 != 0, np.uint64(0xFFFFFFFFFFFFFFFF), np.uint64(0)), masks)
    return PackedInputs(masks.astype(np.uint64), values)
