"""CPU-only checks of the C-ABI library and the host-side logic (no GPU)."""
import ctypes
import os
import re

import numpy as np
import pytest

from metalfish_b200 import layout, synthetic
from metalfish_b200._lib import LIB_PATH, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in ("mfb200.h", "mfb200_testing.h"):
        with open(os.path.join(ROOT, "include", h)) as f:
            names |= set(re.findall(r"MFB200_API\s+[\w\s\*]*?\b(mfb200_\w+)\s*\(", f.read()))
    return names


def test_library_exports_every_declared_symbol():
    assert os.path.exists(LIB_PATH)
    L = lib()
    names = declared_symbols()
    assert len(names) >= 12
    for n in sorted(names):
        assert hasattr(L, n), f"{n} declared in include/ but not exported"


@pytest.mark.parametrize("cfg", [synthetic.TINY, synthetic.SMALL])
def test_weight_blob_size_matches_library(cfg):
    from metalfish_b200.network import _lib as netlib, net_desc, weight_blob
    expected = netlib().mfb200_weight_bytes(ctypes.byref(net_desc(cfg)))
    assert weight_blob(cfg, synthetic.generate(cfg, 0)).nbytes == expected


def test_create_without_gpu_fails_loudly():
    """No CPU fallback: on a machine without a usable B200, creation raises."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from metalfish_b200.network import create_network
    t = synthetic.generate(synthetic.TINY, 0)
    with pytest.raises(RuntimeError):
        create_network(synthetic.TINY, t, max_batch=4)


def test_create_rejects_bad_desc_and_blob():
    from metalfish_b200.network import Config, _lib as netlib, net_desc
    L = netlib()
    d = net_desc(synthetic.TINY)
    d.heads = 3  # head depth must be 32
    h = ctypes.c_void_p()
    conf = Config(0, 1, 0, 4, 1, 0)
    blob = np.zeros(16, np.float32)
    assert L.mfb200_create(ctypes.byref(d), blob.ctypes.data, blob.nbytes, ctypes.byref(conf), ctypes.byref(h)) != 0
    assert b"head depth" in L.mfb200_last_error(None)
    d = net_desc(synthetic.TINY)
    assert L.mfb200_create(ctypes.byref(d), blob.ctypes.data, blob.nbytes, ctypes.byref(conf), ctypes.byref(h)) != 0
    assert b"bytes, expected" in L.mfb200_last_error(None)


def test_slot_tables_cover_generator():
    t = synthetic.generate(synthetic.TINY, 0)
    names = set(layout.GLOBAL_SLOTS) | {layout.layer_name(i, s) for i in range(synthetic.TINY.layers)
                                        for s in layout.LAYER_SLOTS}
    assert names == set(t)


def test_noalloc_rejects_oversize_without_touching_gpu():
    L = lib()
    L.mfb200_splitk_gemm_noalloc.restype = ctypes.c_int
    L.mfb200_noalloc_last_error.restype = ctypes.c_char_p
    rc = L.mfb200_splitk_gemm_noalloc(ctypes.c_void_p(16), ctypes.c_void_p(16), 4096, 1024, 1024, 4,
                                      None, ctypes.c_void_p(16), None)
    assert rc != 0 and b"exceeds" in L.mfb200_noalloc_last_error()


def test_policy_index_table_matches_reference():
    """The move -> policy index mapping the GPU uses (derived from the
    library's own 1858-move list) equals the reference's NN::MoveToNNIndex
    for every transform, promotion kind and square pair (host only)."""
    import os
    from metalfish_b200.network import policy_index_table
    ref = np.load(os.path.join(os.path.dirname(__file__), "golden", "move_index.npz"))["table"]
    np.testing.assert_array_equal(policy_index_table(), ref)
