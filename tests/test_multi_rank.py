"""The N > 1 path on CPU: two gloo ranks launched by torch.distributed.run (as
the driver launches bench.py) give every rank its own frames (weak scaling) and take the max
time over ranks; plus the frame-assignment rule for every world size the scaling run uses."""
import hashlib
import json
import os
import socket
import subprocess
import sys

import pytest

from conftest import ROOT

pytest.importorskip("torch")


def _bench():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_for_tests", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("per_gpu", [64, 16, 3])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_rank_frames_weak_scaling(per_gpu, world):
    """Every rank encodes per_gpu frames of its own: the ranks' blocks tile [0, per_gpu * world)."""
    bench = _bench()
    seen = []
    for r in range(world):
        first, n = bench.rank_frames(per_gpu, r)
        assert n == per_gpu
        seen.extend(range(first, first + n))
    assert seen == list(range(per_gpu * world))


@pytest.mark.parametrize("total", [64, 16, 10, 3])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_frames_partition(total, world):
    bench = _bench()
    seen = []
    sizes = []
    for r in range(world):
        first, n = bench.shard_frames(total, r, world)
        seen.extend(range(first, first + n))
        sizes.append(n)
    assert seen == list(range(total))
    assert max(sizes) - min(sizes) <= 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_two_gloo_ranks(tmp_path):
    per_gpu = 3
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "multirank_worker.py"), str(tmp_path), str(per_gpu)]
    env = dict(os.environ, OMP_NUM_THREADS="1", MASTER_ADDR="127.0.0.1")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    ranks = [json.load(open(tmp_path / f"rank{i}.json")) for i in range(2)]
    # disjoint, complete, and each frame generated from its own seed (same bytes as a 1-rank run)
    bench = _bench()
    bench.load_pkg()
    from sam3_b200 import synth
    ref = [hashlib.sha256(f.tobytes()).hexdigest() for f in synth.frames_u8(2 * per_gpu, 8, base_seed=1000)]
    got = []
    for d in sorted(ranks, key=lambda d: d["rank"]):
        assert d["world"] == 2
        got.extend(d["digests"])
    assert got == ref
    # every rank reports the job time = max over ranks
    tmax = max(d["t_local"] for d in ranks)
    assert all(d["t_job"] == tmax for d in ranks)
