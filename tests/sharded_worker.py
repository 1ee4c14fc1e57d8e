"""One rank of the multi-GPU sharded test (launched by tests/test_sharded_multi_gpu.py under
torchrun, one process per GPU, NCCL). Rank 0 compares the ids with the CPU oracle and writes
the verdict to the file named by ``--out``."""

from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from tests.helpers import compare, to_device  # noqa: E402
from vinfer_b200 import SAMPLER, BackendContext  # noqa: E402
from vinfer_b200.sharded import B200ShardKernels, ShardedSampler, shard_range  # noqa: E402
from vinfer_b200.workloads import make  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--config", type=int, default=4)
    ap.add_argument("--batch", type=int, default=64)
    args = ap.parse_args()
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    try:
        w = make(args.config, batch=args.batch)
        lg, params, u, hist = to_device(w, dev)
        lo, hi = shard_range(w.vocab, world, rank)
        shard = lg[:, lo:hi].contiguous()
        backend = SAMPLER.resolve("b200", BackendContext(dev, torch.bfloat16))
        sampler = ShardedSampler(B200ShardKernels(backend))
        probs = torch.empty(w.batch, hi - lo, dtype=torch.float32, device=dev)
        ids = sampler.sample_batch(shard, params, u, hist, w.vocab, probs_out=probs)
        widths = [b - a for a, b in (shard_range(w.vocab, world, r) for r in range(world))]
        parts = [torch.empty(w.batch, n, dtype=torch.float32, device=dev) for n in widths]
        dist.all_gather(parts, probs)
        all_ids = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(all_ids, ids)
        torch.cuda.synchronize()
        backend.check()
        if rank == 0:
            same = all(torch.equal(all_ids[0], t) for t in all_ids)
            full = torch.cat(parts, dim=1).cpu().numpy()
            rep = compare(w, ids.cpu().numpy(), full)
            Path(args.out).write_text(json.dumps({
                "same_on_all_ranks": same, "failures": [list(map(str, f)) for f in rep.failures],
                "report": str(rep), "unresolved": sampler.last_unresolved, "world": world}))
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
