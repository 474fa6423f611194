#!/usr/bin/env python3
"""Benchmark of the B200 BT4 forward (positions/s), driver contract.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

One process per GPU (torchrun for N > 1). Each rank holds a replica of a
seeded synthetic BT4-shaped network (1024 x 15 x 32h, dff 1536, smolgen) and
evaluates its own shard of seeded random-playout positions (the committed
fixture tests/golden/positions.npz, produced by the reference's encoder): the
batch is sharded, weights replicated, no collective in the forward
("scaling": "weak", per-GPU batch fixed). A step is one forward of one batch.

* value      -- device-timed (CUDA events on the launching stream, max over
                ranks) positions/s with the inputs resident in HBM.
* e2e        -- the same through the public host API (mfb200_evaluate) from
                pinned host buffers: H2D of the packed planes and D2H of
                policy/WDL/moves-left inside the timed region, wall clock.
* roofline   -- the QKV projection GEMM (the largest stage), algorithmic
                FLOPs / event time of its launches in this run; `gemm_all`
                aggregates all tcgen05 GEMM launches of one forward.
* e2e_priors -- the MCTS leaf path through mfb200_evaluate_priors: the same
                host round trip, returning the softmax priors of each
                position's legal moves (computed on the GPU) instead of the
                1858 logits.
* e2e_leaves -- the whole MCTS leaf evaluation through mfb200_evaluate_leaves:
                game histories (board records) and legal moves in, priors
                out; position encoding, forward, move mapping and softmax on
                the GPU (the host-side encode of the reference evaluator is
                gone).
* int8 / fp8  -- the 8-bit configurations of the same forward at the same
                batch (config 2): device-timed and end-to-end positions/s, and
                the QKV GEMM's roofline against twice the bf16 tensor peak.
                INT8 (signed 8-bit operands, per-row / per-channel scales)
                meets the 8-bit parity bound; FP8-e4m3 in every encoder GEMM
                does not (tests/test_bt4_bench_parity_gpu.py).
* sweep        -- (1 GPU) config 3: ms per batch and positions/s of the bf16
                forward at batch 1, 8, 32, 128, 512, 1024 and 4096.
* config4      -- config 4: a global batch of 8192 split evenly over the N
                GPUs (8192 / N per GPU), inputs from pinned host memory and
                policy / WDL / moves-left gathered back to host memory every
                step through mfb200_evaluate; whole-job positions/s from the
                slowest rank's wall time.
* cpu_baseline -- the reference CPU backend (oracle/_ref, built from the
                reference sources) or, if that binary is absent, the C
                restatement, on a bounded sample on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WEIGHT_SEED = 3
CPU_SAMPLE_TARGET_S = 15.0


def load_positions(n: int):
    from metalfish_b200.netfile import PackedInputs
    z = np.load(os.path.join(ROOT, "tests", "golden", "positions.npz"))
    m, v = z["masks"], z["values"]
    reps = (n + len(m) - 1) // len(m)
    return PackedInputs(np.tile(m, (reps, 1))[:n].copy(), np.tile(v, (reps, 1))[:n].copy())


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return j.get("bf16_tflops", 1590.0), j.get("bf16_tflops_sustained", 1400.0), "measured"
    return 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.out = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.out, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.out.flush()
        self.out.seek(0)
        rows = [r.split(",") for r in self.out.read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.out.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def cpu_baseline(cfg, tensors, sample_positions: int | None = None):
    """Time the reference CPU backend (or the oracle port) on a bounded sample."""
    from metalfish_b200 import netfile
    threads = os.cpu_count() or 1
    harness = os.path.join(ROOT, "oracle", "_ref", "ref_harness")
    # ~0.12 positions/s per core for BT4 shapes on the naive fp32 loops
    n = sample_positions or max(threads, int(0.12 * threads * CPU_SAMPLE_TARGET_S))
    inp = load_positions(n)
    if os.path.exists(harness):
        with tempfile.TemporaryDirectory() as tmp:
            net = os.path.join(tmp, "net.mfnt")
            netfile.write_net(net, cfg.header(), tensors)
            pos = os.path.join(tmp, "pos.mfin")
            netfile.write_inputs(pos, inp)
            r = subprocess.run([harness, "eval", net, pos, os.path.join(tmp, "o.mfot"),
                                str(threads)], check=True, capture_output=True, text=True)
            j = json.loads(r.stdout.strip().splitlines()[-1])
        return {"value": j["pos_per_s"], "unit": "positions/s", "cores": threads,
                "kind": "reference",
                "sample": f"{n} positions, reference Cpu::CpuNetwork (fp32), {threads} threads, "
                          f"{j['seconds']:.1f} s"}
    from oracle import port
    t0 = time.perf_counter()
    port.forward(cfg, tensors, inp, threads)
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "positions/s", "cores": threads, "kind": "port",
            "sample": f"{n} positions, C restatement oracle (fp32), {threads} threads, {dt:.1f} s"}


# DRAM bytes (read + write) of one QKV GEMM launch at batch 1024: an ncu
# capture of the same kernel at M=16384 (batch 256; dram__bytes_read.sum +
# dram__bytes_write.sum = 40.2 + 54.0 MB) scaled by 4 to M=65536, since the
# operand and output bytes grow with M. Part of the output is still in L2
# when a launch ends, so the write half is an upper estimate.
QKV_TRAFFIC = {
    "bf16": (4 * (40.235e6 + 53.987e6), "ncu capture at M=16384, scaled x4 to M=65536"),
    # ncu launch lists of the 8-bit forwards at batch 256 (M=16384): DRAM read + write
    # bytes of the 15 QKV launches / 15, scaled x4 to M=65536
    "int8": (4 * (308.8e6 + 1443.5e6) / 15, "ncu launch list at M=16384 (15 launches), scaled x4 to M=65536"),
    "fp8": (4 * (308.9e6 + 1418.2e6) / 15, "ncu launch list at M=16384 (15 launches), scaled x4 to M=65536"),
}


def stage_summary(stages):
    """Per stage name (summed over layers): ms and achieved TFLOP/s."""
    agg = {}
    for n, m, f in stages:
        a = agg.setdefault(n, [0.0, 0.0])
        a[0] += m
        a[1] += f
    return {n: {"ms": round(m, 4), "tflops": round(f / (m / 1e3) / 1e12, 1) if m > 0 and f else None}
            for n, (m, f) in sorted(agg.items(), key=lambda kv: -kv[1][0])}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        # keep stdout to the one JSON line (NCCL otherwise announces its version there)
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        import torch.distributed as dist
        import torch
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        if backend == "nccl":
            dist.init_process_group(backend, device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend)
    return rank, local, world


def barrier(world):
    if world > 1:
        # keep stdout to the one JSON line (NCCL otherwise announces its version there)
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        import torch.distributed as dist
        dist.barrier()


def all_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64,
                     device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_reference(args, rank, world):
    """--impl reference: the reference CPU implementation on the host cores."""
    from metalfish_b200 import synthetic
    if rank != 0:
        return
    cfg = synthetic.BT4
    tensors = synthetic.generate(cfg, WEIGHT_SEED)
    threads = os.cpu_count() or 1
    per_step = max(threads, 8)
    vals = []
    kind = sample = None
    for i in range(args.warmup + args.steps):
        cb = cpu_baseline(cfg, tensors, per_step)
        if i >= args.warmup:
            vals.append(cb["value"])
        kind, sample = cb["kind"], cb["sample"]
    v = float(np.mean(vals))
    line = {"metric": "BT4-shape positions/sec", "value": v, "unit": "positions/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": per_step / v * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded random-playout positions, random-init BT4-shaped weights)",
            "config": {"workload": f"{cfg.name} forward, {per_step} positions per step on the host cores",
                       "batch": per_step},
            "impl": "reference",
            "cpu_baseline": {"value": v, "unit": "positions/s", "cores": threads, "kind": kind,
                             "sample": sample},
            "e2e": {"value": v, "unit": "positions/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1024, help="positions per GPU per step")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default="bf16", choices=["bf16", "fp8", "int8"])
    ap.add_argument("--fp8-gemms", type=int, default=0, help="FP8 GEMM-group mask (0 = all)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--headline-only", action="store_true",
                    help="skip the 8-bit, sweep and config-4 measurements")
    ap.add_argument("--sweep", default="",
                    help="comma-separated batch sizes: print one latency/throughput JSON line per "
                         "batch on 1 GPU instead of the contract line")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, local, world = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    from metalfish_b200 import synthetic
    from metalfish_b200.network import Timing, create_network

    if args.sweep:
        run_sweep(args, [int(x) for x in args.sweep.split(",")])
        return
    cfg = synthetic.BT4
    B = args.batch
    tensors = synthetic.generate(cfg, WEIGHT_SEED)
    # FP8: per-tensor activation scales from absmax over 1024 seeded positions
    # (positions 1024..2047 of the fixture, disjoint from the first shard)
    net = create_network(cfg, tensors, device=local, max_batch=B, precision=args.precision,
                         fp8_gemms=args.fp8_gemms,
                         calibration=load_positions(2048).slice(1024, 2048) if args.precision in ("fp8", "int8") else None)
    inp = load_positions(B * world)
    shard = inp.slice(rank * B, (rank + 1) * B)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    d_masks = torch.from_numpy(shard.masks.view(np.int64)).to(dev)
    d_values = torch.from_numpy(shard.values).to(dev)
    d_pol = torch.empty((B, 1858), dtype=torch.float32, device=dev)
    d_wdl = torch.empty((B, 3), dtype=torch.float32, device=dev)
    d_mlh = torch.empty((B,), dtype=torch.float32, device=dev)
    # a dedicated (non-default) stream: the library enqueues on it and the
    # CUDA events below are recorded on the same stream
    stream = torch.cuda.Stream(dev)

    def step():
        net.evaluate_device(d_masks.data_ptr(), d_values.data_ptr(), B, d_pol.data_ptr(),
                            d_wdl.data_ptr(), d_mlh.data_ptr(), stream.cuda_stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    stages = net.profile(B, iters=3)
    launches_per_step = len(stages)

    # ---- device-resident timed region
    barrier(world)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    assert stream.cuda_stream != 0
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    ms = e0.elapsed_time(e1)
    ms_max = all_max(ms, world)
    clocks = clk.summary()
    value = B * world * args.steps / (ms_max / 1e3)

    # ---- end to end through the host API, pinned buffers
    pin_m = torch.from_numpy(shard.masks.view(np.int64)).pin_memory()
    pin_v = torch.from_numpy(shard.values).pin_memory()
    h_pol = torch.empty((B, 1858), dtype=torch.float32).pin_memory()
    h_wdl = torch.empty((B, 3), dtype=torch.float32).pin_memory()
    h_mlh = torch.empty((B,), dtype=torch.float32).pin_memory()
    from metalfish_b200.network import _lib
    import ctypes
    L = _lib()

    def e2e_step():
        rc = L.mfb200_evaluate(net._h, pin_m.data_ptr(), pin_v.data_ptr(), B, h_pol.data_ptr(),
                               h_wdl.data_ptr(), h_mlh.data_ptr(), None)
        if rc:
            raise RuntimeError(L.mfb200_last_error(net._h).decode())

    for _ in range(args.warmup):
        e2e_step()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_s = all_max(time.perf_counter() - t0, world)
    barrier(world)
    e2e_value = B * world * args.steps / e2e_s

    # ---- the MCTS leaf path through mfb200_evaluate_priors: the same forward,
    # then the priors of each position's legal moves computed on the GPU and
    # copied back instead of the 1858 logits (fixture legal-move lists)
    mv = np.load(os.path.join(ROOT, "tests", "golden", "legal_moves.npz"))
    ids = np.arange(rank * B, (rank + 1) * B) % len(mv["offsets"][:-1])
    counts = mv["offsets"][ids + 1] - mv["offsets"][ids]
    m_off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    m_idx = np.concatenate([mv["index"][mv["offsets"][i]:mv["offsets"][i + 1]] for i in ids]).astype(np.int16)
    h_pri = torch.empty(int(m_off[-1]), dtype=torch.float32).pin_memory()
    pin_off = torch.from_numpy(m_off).pin_memory()
    pin_idx = torch.from_numpy(m_idx).pin_memory()

    def priors_step():
        rc = L.mfb200_evaluate_priors(net._h, pin_m.data_ptr(), pin_v.data_ptr(), B, pin_off.data_ptr(),
                                      pin_idx.data_ptr(), ctypes.c_float(1.0), h_pri.data_ptr(),
                                      h_wdl.data_ptr(), h_mlh.data_ptr(), None)
        if rc:
            raise RuntimeError(L.mfb200_last_error(net._h).decode())

    for _ in range(args.warmup):
        priors_step()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        priors_step()
    pr_s = all_max(time.perf_counter() - t0, world)
    barrier(world)
    e2e_priors = {"value": B * world * args.steps / pr_s, "unit": "positions/s",
                  "h2d_bytes_per_step": int(B * 112 * 12 + (B + 1) * 4 + len(m_idx) * 2),
                  "d2h_bytes_per_step": int(len(m_idx) * 4 + B * 16),
                  "legal_moves_per_step": int(len(m_idx))}

    # ---- the whole MCTS leaf path through mfb200_evaluate_leaves: game
    # histories (board records of the fixture games) and their legal moves
    # in, priors out -- encoding, forward, move mapping and softmax on the GPU
    hz = np.load(os.path.join(ROOT, "tests", "golden", "history.npz"))
    h_off_all, h_boards_all = hz["start/offsets"], hz["start/boards"]
    gid = np.arange(rank * B, (rank + 1) * B) % (len(h_off_all) - 1)
    h_counts = h_off_all[gid + 1] - h_off_all[gid]
    h_off = np.concatenate([[0], np.cumsum(h_counts)]).astype(np.int32)
    h_boards = np.concatenate([h_boards_all[h_off_all[i]:h_off_all[i + 1]] for i in gid])
    l_counts = mv["offsets"][gid + 1] - mv["offsets"][gid]
    l_off = np.concatenate([[0], np.cumsum(l_counts)]).astype(np.int32)
    l_raw = np.concatenate([mv["raw"][mv["offsets"][i]:mv["offsets"][i + 1]] for i in gid]).astype(np.uint16)
    pin_hb = torch.from_numpy(h_boards).pin_memory()
    pin_ho = torch.from_numpy(h_off).pin_memory()
    pin_lr = torch.from_numpy(l_raw.view(np.int16)).pin_memory()
    pin_lo = torch.from_numpy(l_off).pin_memory()
    h_lpri = torch.empty(int(l_off[-1]), dtype=torch.float32).pin_memory()

    def leaves_step():
        rc = L.mfb200_evaluate_leaves(net._h, pin_hb.data_ptr(), pin_ho.data_ptr(), B, 5,
                                      pin_lr.data_ptr(), pin_lo.data_ptr(), ctypes.c_float(1.0),
                                      h_lpri.data_ptr(), h_wdl.data_ptr(), h_mlh.data_ptr(), None)
        if rc:
            raise RuntimeError(L.mfb200_last_error(net._h).decode())

    for _ in range(args.warmup):
        leaves_step()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        leaves_step()
    lv_s = all_max(time.perf_counter() - t0, world)
    barrier(world)
    # the same, double-buffered: batch i+1 is submitted before batch i is
    # waited for (mfb200_submit_leaves / mfb200_wait), so the host's
    # submission work overlaps the GPU's
    tickets = [ctypes.c_uint64(0), ctypes.c_uint64(0)]

    def submit(k):
        rc = L.mfb200_submit_leaves(net._h, pin_hb.data_ptr(), pin_ho.data_ptr(), B, 5,
                                    pin_lr.data_ptr(), pin_lo.data_ptr(), ctypes.c_float(1.0),
                                    h_lpri.data_ptr(), h_wdl.data_ptr(), h_mlh.data_ptr(),
                                    ctypes.byref(tickets[k & 1]))
        if rc:
            raise RuntimeError(L.mfb200_last_error(net._h).decode())

    def wait(k):
        if L.mfb200_wait(net._h, tickets[k & 1].value):
            raise RuntimeError(L.mfb200_last_error(net._h).decode())

    barrier(world)
    t0 = time.perf_counter()
    submit(0)
    for k in range(1, args.steps):
        submit(k)
        wait(k - 1)
    wait(args.steps - 1)
    la_s = all_max(time.perf_counter() - t0, world)
    barrier(world)
    e2e_leaves = {"value": B * world * args.steps / lv_s, "unit": "positions/s",
                  "pipelined_value": B * world * args.steps / la_s,
                  "h2d_bytes_per_step": int(h_boards.nbytes + h_off.nbytes + l_raw.nbytes + l_off.nbytes),
                  "d2h_bytes_per_step": int(len(l_raw) * 4 + B * 16),
                  "history_boards_per_step": int(len(h_boards))}

    # ---- batch-1 latency (the per-leaf MCTS case): device time of one
    # graph-launched forward, and the host round trip through mfb200_evaluate
    lat = batch1_latency(net, dev, stream, shard, L) if rank == 0 else None
    e2e_leaves["small_batches"] = leaves_small_batches(net, L) if rank == 0 else None
    net.close()
    extra = {}
    if args.precision == "bf16" and not args.headline_only:
        for prec in ("int8", "fp8"):
            extra[prec] = eight_bit_line(cfg, tensors, prec, B, local, dev, stream, shard, L, args, world)
        if world == 1:
            extra["sweep"] = run_sweep_rows(cfg, tensors, local, dev, stream, args)
        extra["config4"] = run_config4(cfg, tensors, rank, local, world, args, L)

    # ---- roofline. Dominant kernel: the QKV(+smolgen compress) projection
    # GEMM, the largest single stage (15 launches per forward; the CTA-pair
    # tcgen05 kernel in bf16, the single-CTA one in e4m3), achieved = its
    # algorithmic FLOPs / its CUDA-event time measured in this run. `gemm_all`
    # aggregates every GEMM launch of the forward the same way.
    gemm = [(n, m, f) for (n, m, f) in stages if f > 0 and n not in ("attention", "policy_map")]
    g_ms = sum(m for _, m, _ in gemm)
    g_fl = sum(f for _, _, f in gemm)
    qkv = [(m, f) for (n, m, f) in stages if n == "qkv"]
    q_ms = sum(m for m, _ in qkv)
    q_fl = sum(f for _, f in qkv)
    burst, sustained, src = measured_peaks()
    peak_note = f"{src} bf16_tflops_sustained (kernel timed inside a long step)"
    if args.precision != "bf16":
        # no 8-bit peak was measured on this pool; the e4m3 / int8 dense rate is twice bf16
        sustained *= 2.0
        peak_note = f"2 x {src} bf16_tflops_sustained (8-bit dense = 2x bf16)"
    achieved = q_fl / (q_ms / 1e3) / 1e12 if q_ms > 0 else 0.0
    g_achieved = g_fl / (g_ms / 1e3) / 1e12 if g_ms > 0 else 0.0
    traffic, traffic_src = QKV_TRAFFIC.get(args.precision, (None, None)) if B == 1024 else (None, None)
    total_stage_ms = sum(m for _, m, _ in stages)
    enc = cfg.flops_per_position()

    if rank == 0:
        line = {
            "metric": "BT4-shape positions/sec", "value": value, "unit": "positions/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": {"bf16": "bf16", "fp8": "e4m3", "int8": "s8"}[args.precision],
            "data": "synthetic (seeded random-playout positions from the reference encoder, "
                    "random-init BT4-shaped weights)",
            "config": {"workload": f"{cfg.name} forward, {args.precision}, batch {B} per GPU",
                       "batch_per_gpu": B, "global_batch": B * world,
                       "parallelism": f"batch-sharded x{world}, replicated weights, no collective",
                       "l2": "per-step working set ~3 GB (activations) > 126 MB L2",
                       "graphs": True},
            "e2e": {"value": e2e_value, "unit": "positions/s",
                    "h2d_bytes_per_step": int(B * 112 * 12),
                    "d2h_bytes_per_step": int(B * (1858 + 3 + 1) * 4)},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": sustained,
                         "unit": "TFLOP/s", "frac": achieved / sustained, "traffic": traffic,
                         "kernel": ("gemm_pair_kernel<bf16/fp16>" if args.precision == "bf16"
                                    else "gemm_pair_kernel<8-bit> (e4m3 or s8)")
                                   + f": QKV+compress projection, M={B * 64} N=3104 K=1024, "
                                     f"{len(qkv)} launches per forward",
                         "traffic_source": traffic_src,
                         "peak_source": peak_note,
                         "gemm_all": {"achieved": g_achieved, "frac": g_achieved / sustained,
                                      "launches": len(gemm)}},
            "flops_per_position": {"encoder_gemm": enc["encoder_gemm_flops"], "all_matmul": enc["total_flops"]},
            "model_tflops": value * enc["total_flops"] / 1e12 / world,
            "tensor_roofline": {
                "per_gpu_encoder_tflops": value * enc["encoder_gemm_flops"] / 1e12 / world,
                "frac_of_measured_burst": value * enc["encoder_gemm_flops"] / 1e12 / world
                / (burst * (2.0 if args.precision != "bf16" else 1.0)),
                "frac_of_nominal_dense": value * enc["encoder_gemm_flops"] / 1e12 / world
                / (4500.0 if args.precision != "bf16" else 2250.0),
                "note": "encoder QKV/O/FFN FLOPs (14.09 GFLOP per position) per GPU against the "
                        "measured cuBLAS bf16 burst peak (x2 for e4m3) and the nominal dense peak"},
            "latency_batch1_ms": lat,
            "e2e_priors": e2e_priors,
            "e2e_leaves": e2e_leaves,
            "stage_ms": stage_summary(stages),
            "stage_ms_total": total_stage_ms,
            "clocks": clocks,
        }
        line.update(extra)
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(cfg, tensors)
        print(json.dumps(line), flush=True)


def leaves_small_batches(net, L, batches=(16, 32), steps=200):
    """The MCTS leaf path at the batch sizes the reference search uses
    (minibatch 32, 16 on CUDA): synchronous mfb200_evaluate_leaves round trips
    against double-buffered mfb200_submit_leaves / mfb200_wait, positions/s
    from wall time."""
    import ctypes
    import torch
    mv = np.load(os.path.join(ROOT, "tests", "golden", "legal_moves.npz"))
    hz = np.load(os.path.join(ROOT, "tests", "golden", "history.npz"))
    h_off_all, h_boards_all = hz["start/offsets"], hz["start/boards"]
    out = {}
    for B in batches:
        bufs = []
        for k in range(2):  # two input / output sets, alternated by the pipelined loop
            gid = (np.arange(B) + k * B) % (len(h_off_all) - 1)
            hc = h_off_all[gid + 1] - h_off_all[gid]
            h_off = np.concatenate([[0], np.cumsum(hc)]).astype(np.int32)
            hb = np.concatenate([h_boards_all[h_off_all[i]:h_off_all[i + 1]] for i in gid])
            lc = mv["offsets"][gid + 1] - mv["offsets"][gid]
            l_off = np.concatenate([[0], np.cumsum(lc)]).astype(np.int32)
            lr = np.concatenate([mv["raw"][mv["offsets"][i]:mv["offsets"][i + 1]] for i in gid]).astype(np.uint16)
            bufs.append([torch.from_numpy(hb).pin_memory(), torch.from_numpy(h_off).pin_memory(),
                         torch.from_numpy(lr.view(np.int16)).pin_memory(),
                         torch.from_numpy(l_off).pin_memory(),
                         torch.empty(int(l_off[-1]), dtype=torch.float32).pin_memory(),
                         torch.empty((B, 3), dtype=torch.float32).pin_memory(),
                         torch.empty((B,), dtype=torch.float32).pin_memory()])

        def args(k):
            b = bufs[k & 1]
            return (net._h, b[0].data_ptr(), b[1].data_ptr(), B, 5, b[2].data_ptr(), b[3].data_ptr(),
                    ctypes.c_float(1.0), b[4].data_ptr(), b[5].data_ptr(), b[6].data_ptr())

        def sync_step(k):
            if L.mfb200_evaluate_leaves(*args(k), None):
                raise RuntimeError(L.mfb200_last_error(net._h).decode())

        for k in range(10):
            sync_step(k)
        t0 = time.perf_counter()
        for k in range(steps):
            sync_step(k)
        sync_s = time.perf_counter() - t0
        tickets = [ctypes.c_uint64(0), ctypes.c_uint64(0)]

        def submit(k):
            if L.mfb200_submit_leaves(*args(k), ctypes.byref(tickets[k & 1])):
                raise RuntimeError(L.mfb200_last_error(net._h).decode())

        def wait(k):
            if L.mfb200_wait(net._h, tickets[k & 1].value):
                raise RuntimeError(L.mfb200_last_error(net._h).decode())

        t0 = time.perf_counter()
        submit(0)
        for k in range(1, steps):
            submit(k)
            wait(k - 1)
        wait(steps - 1)
        pipe_s = time.perf_counter() - t0
        out[str(B)] = {"sync_value": B * steps / sync_s, "pipelined_value": B * steps / pipe_s,
                       "sync_ms_per_batch": sync_s / steps * 1e3,
                       "pipelined_ms_per_batch": pipe_s / steps * 1e3, "unit": "positions/s"}
    return out


def device_ms(net, dev, stream, shard, B, steps, warmup, world):
    """Device time (CUDA events on the launching stream, max over ranks) of
    `steps` forwards at batch B with the inputs resident in HBM."""
    import torch
    d_m = torch.from_numpy(shard.masks[:B].view(np.int64)).to(dev)
    d_v = torch.from_numpy(shard.values[:B]).to(dev)
    d_p = torch.empty((B, 1858), dtype=torch.float32, device=dev)
    d_w = torch.empty((B, 3), dtype=torch.float32, device=dev)
    d_l = torch.empty((B,), dtype=torch.float32, device=dev)

    def step():
        net.evaluate_device(d_m.data_ptr(), d_v.data_ptr(), B, d_p.data_ptr(), d_w.data_ptr(),
                            d_l.data_ptr(), stream.cuda_stream)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    return all_max(e0.elapsed_time(e1), world)


def host_s(net, L, shard, B, steps, warmup, world):
    """Wall time (max over ranks) of `steps` host round trips through
    mfb200_evaluate: pinned inputs copied in, all outputs copied back."""
    import torch
    pin_m = torch.from_numpy(shard.masks[:B].view(np.int64)).pin_memory()
    pin_v = torch.from_numpy(shard.values[:B]).pin_memory()
    h_pol = torch.empty((B, 1858), dtype=torch.float32).pin_memory()
    h_wdl = torch.empty((B, 3), dtype=torch.float32).pin_memory()
    h_mlh = torch.empty((B,), dtype=torch.float32).pin_memory()

    def step():
        rc = L.mfb200_evaluate(net._h, pin_m.data_ptr(), pin_v.data_ptr(), B, h_pol.data_ptr(),
                               h_wdl.data_ptr(), h_mlh.data_ptr(), None)
        if rc:
            raise RuntimeError(L.mfb200_last_error(net._h).decode())

    for _ in range(warmup):
        step()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = all_max(time.perf_counter() - t0, world)
    barrier(world)
    return dt


def eight_bit_line(cfg, tensors, precision, B, local, dev, stream, shard, L, args, world):
    """Config 2: the 8-bit forward at the headline batch."""
    from metalfish_b200.network import create_network
    net = create_network(cfg, tensors, device=local, max_batch=B, precision=precision,
                         calibration=load_positions(2048).slice(1024, 2048))
    ms = device_ms(net, dev, stream, shard, B, args.steps, args.warmup, world)
    e2e = host_s(net, L, shard, B, args.steps, args.warmup, world)
    stages = net.profile(B, iters=3)
    net.close()
    burst, sustained, src = measured_peaks()
    qkv = [(m, f) for (n, m, f) in stages if n == "qkv"]
    q_ms, q_fl = sum(m for m, _ in qkv), sum(f for _, f in qkv)
    achieved = q_fl / (q_ms / 1e3) / 1e12 if q_ms > 0 else 0.0
    enc = cfg.flops_per_position()["encoder_gemm_flops"]
    value = B * world * args.steps / (ms / 1e3)
    return {"value": value, "unit": "positions/s", "ms_per_step": ms / args.steps,
            "dtype": "s8 operands, s32 accumulate" if precision == "int8" else "e4m3 operands, f32 accumulate",
            "e2e": {"value": B * world * args.steps / e2e, "unit": "positions/s"},
            "parity": ("meets the 8-bit bound (top-1 >= 99%, |dWDL| <= 2e-2)" if precision == "int8"
                       else "misses the 8-bit |dWDL| bound (e4m3 mantissa noise, ~0.05)"),
            "roofline": {"bound": "tensor", "kernel": "QKV+compress GEMM", "achieved": achieved,
                         "peak": 2.0 * sustained, "unit": "TFLOP/s",
                         "frac": achieved / (2.0 * sustained),
                         "traffic": QKV_TRAFFIC[precision][0] if B == 1024 else None,
                         "traffic_source": QKV_TRAFFIC[precision][1],
                         "peak_source": f"2 x {src} bf16_tflops_sustained (8-bit dense = 2x bf16)"},
            "encoder_tflops_per_gpu": value * enc / 1e12 / world,
            "frac_of_bf16_burst": value * enc / 1e12 / world / burst,
            "stage_ms": stage_summary(stages)}


def run_sweep_rows(cfg, tensors, local, dev, stream, args, batches=(1, 8, 32, 128, 512, 1024, 4096)):
    """Config 3 on one GPU: device ms per batch and positions/s (bf16)."""
    from metalfish_b200.network import create_network
    net = create_network(cfg, tensors, device=local, max_batch=max(batches))
    inp = load_positions(max(batches))
    rows = {}
    for B in batches:
        steps = max(5, min(args.steps, 20))
        ms = device_ms(net, dev, stream, inp, B, steps, args.warmup, 1) / steps
        rows[str(B)] = {"ms": ms, "positions_per_s": B / (ms / 1e3)}
    net.close()
    return rows


def run_config4(cfg, tensors, rank, local, world, args, L, global_batch=8192):
    """Config 4: global batch split evenly over the ranks, host round trips."""
    from metalfish_b200.network import create_network
    per = global_batch // world
    net = create_network(cfg, tensors, device=local, max_batch=per)
    inp = load_positions(global_batch).slice(rank * per, (rank + 1) * per)
    steps = max(3, min(args.steps, 10))
    dt = host_s(net, L, inp, per, steps, args.warmup, world)
    net.close()
    return {"global_batch": global_batch, "per_gpu": per, "n_gpus": world, "steps": steps,
            "value": global_batch * steps / dt, "unit": "positions/s",
            "ms_per_step": dt / steps * 1e3,
            "timing": "wall time of mfb200_evaluate round trips (pinned H2D of the packed planes, "
                      "forward, D2H of policy / WDL / moves-left), max over ranks"}


def batch1_latency(net, dev, stream, shard, L, iters: int = 200):
    """p50/p99 of the batch-1 forward: device time (CUDA events around one
    graph launch) and the host round trip through mfb200_evaluate."""
    import torch
    d_m = torch.from_numpy(shard.masks[:1].view(np.int64)).to(dev)
    d_v = torch.from_numpy(shard.values[:1]).to(dev)
    d_p = torch.empty((1, 1858), dtype=torch.float32, device=dev)
    d_w = torch.empty((1, 3), dtype=torch.float32, device=dev)
    d_l = torch.empty((1,), dtype=torch.float32, device=dev)
    h_m = torch.from_numpy(shard.masks[:1].view(np.int64)).pin_memory()
    h_v = torch.from_numpy(shard.values[:1]).pin_memory()
    h_p = torch.empty((1, 1858), dtype=torch.float32).pin_memory()
    h_w = torch.empty((1, 3), dtype=torch.float32).pin_memory()
    h_l = torch.empty((1,), dtype=torch.float32).pin_memory()

    def dev_step():
        net.evaluate_device(d_m.data_ptr(), d_v.data_ptr(), 1, d_p.data_ptr(), d_w.data_ptr(),
                            d_l.data_ptr(), stream.cuda_stream)

    for _ in range(5):
        dev_step()
    torch.cuda.synchronize(dev)
    dev_ms = []
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dev_step()
        e1.record(stream)
        e1.synchronize()
        dev_ms.append(e0.elapsed_time(e1))
    host_ms = []
    for i in range(iters + 5):
        t0 = time.perf_counter()
        rc = L.mfb200_evaluate(net._h, h_m.data_ptr(), h_v.data_ptr(), 1, h_p.data_ptr(),
                               h_w.data_ptr(), h_l.data_ptr(), None)
        if rc:
            raise RuntimeError(L.mfb200_last_error(net._h).decode())
        if i >= 5:
            host_ms.append((time.perf_counter() - t0) * 1e3)
    q = lambda xs, f: float(np.percentile(np.asarray(xs), f))
    return {"device_p50": q(dev_ms, 50), "device_p99": q(dev_ms, 99),
            "e2e_p50": q(host_ms, 50), "e2e_p99": q(host_ms, 99), "iters": iters}


def run_sweep(args, batches):
    """Config 3 of the baseline: latency and positions/s per batch size on
    one GPU (device time of graph-launched forwards, inputs resident)."""
    import torch
    from metalfish_b200 import synthetic
    from metalfish_b200.network import create_network
    cfg = synthetic.BT4
    tensors = synthetic.generate(cfg, WEIGHT_SEED)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    net = create_network(cfg, tensors, device=0, max_batch=max(batches), precision=args.precision,
                         fp8_gemms=args.fp8_gemms,
                         calibration=load_positions(2048).slice(1024, 2048) if args.precision in ("fp8", "int8") else None)
    stream = torch.cuda.Stream(dev)
    inp = load_positions(max(batches))
    d_m = torch.from_numpy(inp.masks.view(np.int64)).to(dev)
    d_v = torch.from_numpy(inp.values).to(dev)
    nb = max(batches)
    d_p = torch.empty((nb, 1858), dtype=torch.float32, device=dev)
    d_w = torch.empty((nb, 3), dtype=torch.float32, device=dev)
    d_l = torch.empty((nb,), dtype=torch.float32, device=dev)
    for B in batches:
        def step():
            net.evaluate_device(d_m.data_ptr(), d_v.data_ptr(), B, d_p.data_ptr(), d_w.data_ptr(),
                                d_l.data_ptr(), stream.cuda_stream)
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / args.steps
        print(json.dumps({"batch": B, "ms_per_batch": ms, "positions_per_s": B / (ms / 1e3),
                          "precision": args.precision, "steps": args.steps}), flush=True)
    net.close()


def dist_teardown():
    try:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()
    except Exception:  # noqa: BLE001 -- best effort at exit
        pass


if __name__ == "__main__":
    try:
        main()
    finally:
        dist_teardown()
