"""One rank of the CPU multi-rank test (launched by torch.distributed.run with
the gloo backend): runs the benchmark's frame sharding and max-over-ranks
timing exactly as bench.py does on GPUs, with the per-rank frames generated
from their seeds, and writes what it saw to <outdir>/rank<r>.json."""
import datetime
import hashlib
import importlib.util
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    outdir, per_gpu = sys.argv[1], int(sys.argv[2])
    import torch.distributed as dist
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    bench = load("bench_under_test", os.path.join(ROOT, "bench.py"))
    bench.load_pkg()
    from sam3_b200 import synth
    first, n = bench.rank_frames(per_gpu, rank)
    frames = synth.frames_u8(n, 8, base_seed=1000 + first)
    digests = [hashlib.sha256(f.tobytes()).hexdigest() for f in frames]
    # each rank reports a different "time"; every rank must see the max
    t_local = 10.0 + 7.5 * rank
    t_job = bench.max_over_ranks(t_local, world, "cpu")
    dist.barrier()
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump({"rank": rank, "world": world, "first": first, "n": n, "digests": digests, "t_local": t_local,
                   "t_job": t_job}, f)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
