"""bf16 / e4m3 bit conversions on the host (numpy), round-to-nearest-even."""
import numpy as np


def to_bf16_bits(x) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    rounded = u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    out = (rounded >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(np.asarray(x, np.float32))
    out[nan] = 0x7FC0
    return out


def from_bf16_bits(b) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def round_bf16(x) -> np.ndarray:
    return from_bf16_bits(to_bf16_bits(x))
