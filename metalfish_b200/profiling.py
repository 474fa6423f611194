"""Small drivers for profiling the library (e.g. under ncu).

  python -m metalfish_b200.profiling gemm M N K [BN MODE ACT OUT_F32 ITERS DTYPE PAIRS]
      times ITERS back-to-back launches of one tcgen05 GEMM on synthetic
      device data (mfb200_debug_gemm_bench) and prints TFLOP/s. DTYPE: 0
      bf16, 1 e4m3, 2 fp16 operands; PAIRS 0 forbids the CTA-pair kernel.
  python -m metalfish_b200.profiling trace M N K [BN MODE ACT OUT_F32 ITERS DTYPE PAIRS]
      the same, with the kernel's per-role clock-cycle counters
      (mfb200_debug_gemm_trace): how long the epilogue, MMA and producer
      roles spend waiting and working, per CTA and launch.
  python -m metalfish_b200.profiling forward [BATCH] [bf16|fp8|int8|bf16-nofold]
      runs two eager forwards (no CUDA graph, so every kernel is a separate
      launch; the second inside the NVTX range "forward2") of the seeded BT4-shaped network on fixture positions;
      bf16-nofold runs the encoder with separate ln1 / ln2 passes instead of
      the deferred LayerNorm.
  python -m metalfish_b200.profiling leaves [BATCH]
      runs two eager leaf evaluations (mfb200_evaluate_leaves: encoder,
      forward, move mapping + priors) on the fixture game histories.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def gemm(argv) -> None:
    from ._lib import lib
    M, N, K = (int(x) for x in argv[:3])
    bn, mode, act, out_f32, iters, dtype, pairs = (
        int(x) for x in (argv[3:10] + ["256", "0", "0", "0", "10", "0", "1"][len(argv) - 3:]))
    ms = ctypes.c_float()
    lib().mfb200_debug_set_gemm_pairs(pairs)
    rc = lib().mfb200_debug_gemm_bench(M, N, K, bn, mode, act, out_f32, iters, dtype, ctypes.byref(ms))
    if rc:
        raise SystemExit(f"gemm bench failed: rc={rc}")
    print(f"M={M} N={N} K={K} bn={bn} dtype={dtype} pairs={pairs}: {ms.value:.4f} ms  {2.0 * M * N * K / ms.value / 1e9:.1f} TFLOP/s")


def trace(argv) -> None:
    from ._lib import lib
    M, N, K = (int(x) for x in argv[:3])
    bn, mode, act, out_f32, iters, dtype, pairs = (
        int(x) for x in (argv[3:10] + ["256", "0", "0", "0", "10", "0", "1"][len(argv) - 3:]))
    ms = ctypes.c_float()
    tr = (ctypes.c_ulonglong * 8)()
    lib().mfb200_debug_set_gemm_pairs(pairs)
    rc = lib().mfb200_debug_gemm_trace(M, N, K, bn, mode, act, out_f32, iters, dtype,
                                       ctypes.byref(ms), tr)
    if rc:
        raise SystemExit(f"gemm trace failed: rc={rc}")
    ctas = tr[5]
    names = ["epi_wait_acc", "epi_busy", "mma_wait_acc", "mma_wait_operands", "prod_wait_stage",
             "cta_cycles", "epi_tiles", "-"]
    print(f"M={M} N={N} K={K} bn={bn} mode={mode} dtype={dtype} pairs={pairs}: {ms.value:.4f} ms "
          f"{2.0 * M * N * K / ms.value / 1e9:.1f} TFLOP/s; cycles summed over CTAs and launches:")
    print("  " + "  ".join(f"{n}={tr[i]:,}" for i, n in enumerate(names[:7])))
    if ctas:
        print("  fractions of CTA lifetime (epilogue per warp: / epilogue warps): "
              f"mma_wait_acc {tr[2] / ctas:.3f} mma_wait_operands {tr[3] / ctas:.3f} "
              f"prod_wait_stage {tr[4] / ctas:.3f}")


def forward(argv) -> None:
    from .netfile import PackedInputs
    from .network import create_network
    from .synthetic import BT4, generate
    batch = int(argv[0]) if argv else 512
    precision = argv[1] if len(argv) > 1 else "bf16"
    if precision == "bf16-nofold":
        from ._lib import lib
        lib().mfb200_debug_set_fold_ln(0)
        precision = "bf16"
    z = np.load(os.path.join(ROOT, "tests", "golden", "positions.npz"))
    m, v = z["masks"], z["values"]
    reps = (batch + 2048 + len(m) - 1) // len(m)
    m, v = np.tile(m, (reps, 1)), np.tile(v, (reps, 1))
    net = create_network(BT4, generate(BT4, 3), max_batch=batch, use_graphs=False, precision=precision,
                         calibration=(PackedInputs(m[1024:2048], v[1024:2048])
                                      if precision in ("fp8", "int8") else None))
    inp = PackedInputs(m[:batch].copy(), v[:batch].copy())
    import torch
    net.evaluate_packed(inp)
    # the second forward in an NVTX range "forward2", for ncu --nvtx-include "forward2/"
    torch.cuda.nvtx.range_push("forward2")
    net.evaluate_packed(inp)
    torch.cuda.nvtx.range_pop()
    net.close()
    print(f"forward ok: BT4 batch {batch} {precision}")


def leaves(argv) -> None:
    from .network import create_network
    from .synthetic import BT4, generate
    batch = min(int(argv[0]) if argv else 1024, 1024)
    h = np.load(os.path.join(ROOT, "tests", "golden", "history.npz"))
    lm = np.load(os.path.join(ROOT, "tests", "golden", "legal_moves.npz"))
    hoff = h["start/offsets"][:batch + 1]
    moff = lm["offsets"][:batch + 1].astype(np.int32)
    net = create_network(BT4, generate(BT4, 3), max_batch=batch, use_graphs=False)
    for _ in range(2):
        net.evaluate_leaves(h["start/boards"][:hoff[-1]], hoff, lm["raw"][:moff[-1]], moff, 1.0)
    net.close()
    print(f"leaves ok: BT4 batch {batch}")


if __name__ == "__main__":
    cmd, rest = sys.argv[1], sys.argv[2:]
    {"gemm": gemm, "trace": trace, "forward": forward, "leaves": leaves}[cmd](rest)
