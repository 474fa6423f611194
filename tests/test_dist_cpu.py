"""Two gloo ranks on CPU exercise the bench's multi-rank plumbing: rendezvous,
barrier, max-over-ranks timing and the contiguous batch shard."""
import os
import subprocess
import sys
import textwrap

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = textwrap.dedent("""
    import os, sys
    sys.path.insert(0, %r)
    import bench
    rank, local, world = bench.dist_setup(2)
    assert world == 2
    bench.barrier(world)
    m = bench.all_max(float(rank + 1) * 1.5, world)
    inp = bench.load_positions(8 * world)
    shard = inp.slice(rank * 8, (rank + 1) * 8)
    print(f"rank={rank} max={m} first_mask={int(shard.masks[0, 0])}", flush=True)
""") % ROOT


def test_two_rank_gloo_plumbing(tmp_path):
    script = tmp_path / "ranks.py"
    script.write_text(SCRIPT)
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr", "127.0.0.1", "--master-port", "29517", str(script)],
                       capture_output=True, text=True, env=env, timeout=240)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = sorted(l for l in r.stdout.splitlines() if l.startswith("rank="))
    assert len(lines) == 2
    assert all("max=3.0" in l for l in lines)
    assert lines[0].split("first_mask=")[1] != lines[1].split("first_mask=")[1]
