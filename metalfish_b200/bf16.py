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


def _e4m3_table() -> np.ndarray:
    """The 128 non-negative e4m3 values (index = bit pattern 0..127; 0x7F is NaN)."""
    vals = np.zeros(128, np.float64)
    for b in range(128):
        e, m = b >> 3, b & 7
        vals[b] = (m / 8.0) * 2.0 ** -6 if e == 0 else (1 + m / 8.0) * 2.0 ** (e - 7)
    vals[0x7F] = np.nan
    return vals


E4M3_VALUES = _e4m3_table()
E4M3_MAX = 448.0


def from_e4m3_bits(b) -> np.ndarray:
    b = np.asarray(b, np.uint8)
    mag = E4M3_VALUES[b & 0x7F]
    return np.where(b & 0x80, -mag, mag).astype(np.float32)


def to_e4m3_bits(x) -> np.ndarray:
    """Round to nearest e4m3 (ties to even), saturating at +-448."""
    x = np.asarray(x, np.float64)
    a = np.minimum(np.abs(x), E4M3_MAX)
    pos = E4M3_VALUES[:0x7F]                       # ascending, 127 finite values
    hi = np.clip(np.searchsorted(pos, a), 1, 126)
    lo = hi - 1
    dlo, dhi = a - pos[lo], pos[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    idx = np.where(pick_hi, hi, lo)
    idx = np.where(a >= pos[126], 126, idx)
    idx = np.where(a <= 0, 0, idx)
    return (idx | np.where(x < 0, 0x80, 0)).astype(np.uint8)
